"""Expert parallelism across two GPUs with the in-kernel NVLink peer exchange: one process per GPU,
each owning half of the experts (popularity stripe) or half of every expert's units, both mapping
each other's exchange buffers.
Every rank must return the same full layer output, bit for bit, and it must match the oracle; the
same for the whole MoE block (moe_block_forward: router GEMV, routed experts, shared expert at its
full width on every rank, residual combine).
Needs two GPUs (skipped otherwise): kernels that wait on each other must never share one GPU."""
import os
import socket

import numpy as np
import pytest
import torch

from tests.parity import assert_close
from tests.test_gpu_block import _ulp_bf16, assert_bf16_close

pytestmark = pytest.mark.gpu

H, F, E, K, L = 2048, 256, 16, 4, 1
TS = (1, 5, 16, 40)  # fused decode path for T <= 16, multi-kernel path (+ exchange kernel) for 40


def _weights(seed):
    from npu_offload_b200.synth import f2bf
    rng = np.random.default_rng(seed)
    return [(f2bf(rng.standard_normal((F, H), np.float32) * 0.05), f2bf(rng.standard_normal((F, H), np.float32) * 0.05),
             f2bf(rng.standard_normal((H, F), np.float32) * 0.05)) for _ in range(E)]


def _inputs(T, seed):
    from npu_offload_b200.synth import f2bf
    rng = np.random.default_rng(seed)
    return f2bf(rng.standard_normal((T, H), np.float32)), rng.standard_normal((T, E)).astype(np.float32)


BLOCK_TS = (1, 5, 40)  # fused block path for T <= 16, composed calls for 40


def _shared(seed):
    """The shared expert (gate, up [F,H], down [H,F]) at the full width F and the router [E,H]."""
    from npu_offload_b200.synth import f2bf
    rng = np.random.default_rng(seed)
    return (f2bf(rng.standard_normal((F, H), np.float32) * 0.05), f2bf(rng.standard_normal((F, H), np.float32) * 0.05),
            f2bf(rng.standard_normal((H, F), np.float32) * 0.05), f2bf(rng.standard_normal((E, H), np.float32) * 0.05))


def _rank(rank, world, port, q, mode):
    try:
        import datetime
        import torch.distributed as dist
        from npu_offload_b200.moe import MoEDataPlane
        from npu_offload_b200.parallel import attach_peers, shard_map, unit_ranges, unit_slice
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        torch.cuda.set_device(rank)
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
        if mode == "units":  # this rank: its slice of the units of every expert
            f0, f1 = unit_ranges(F, world)[rank]
            smap = np.full((L, E), rank, np.int32)
        else:
            f0, f1 = 0, F
            smap = shard_map(np.arange(E)[None, :][::-1].copy(), world)
        p = MoEDataPlane(H, f1 - f0, E, K, n_layers=L, max_tokens=64, device=rank, ep_rank=rank, ep_world=world,
                         shard_map=smap)
        for e, (g, u, d) in enumerate(_weights(5)):
            if smap[0, e] == rank:
                g, u, d = unit_slice(g, u, d, f0, f1)
                p.load_expert(0, e, torch.from_numpy(np.ascontiguousarray(g).view(np.int16)).view(torch.bfloat16).cuda(),
                              torch.from_numpy(np.ascontiguousarray(u).view(np.int16)).view(torch.bfloat16).cuda(),
                              torch.from_numpy(np.ascontiguousarray(d).view(np.int16)).view(torch.bfloat16).cuda())
        attach_peers(p)
        res = {}
        for T in TS:
            x, lg = _inputs(T, 100 + T)
            xd = torch.from_numpy(x.view(np.int16)).view(torch.bfloat16).cuda()
            out = p.forward(0, xd, torch.from_numpy(lg).cuda(), sync=True)
            res[T] = out.cpu().numpy()
        # the whole MoE block (router GEMV, routed experts with the peer exchange, the shared expert
        # replicated on every rank at its full width, residual combine) on both splits
        sg, su, sd, wr = _shared(6)
        p.load_shared(0, *(torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).view(torch.bfloat16).cuda()
                           for a in (sg, su, sd, wr)))
        for T in BLOCK_TS:
            h2, x2 = _inputs(T, 200 + T)[0], _inputs(T, 300 + T)[0]
            xn = p.block_forward(0, *(torch.from_numpy(a.view(np.int16)).view(torch.bfloat16).cuda() for a in (h2, x2)),
                                 sync=True)
            res[("block", T)] = xn.view(torch.int16).cpu().numpy().view(np.uint16)
        x, lg = _inputs(3, 103)  # host buffers (pinned, in place) on the fused path
        px = torch.from_numpy(x.view(np.int16)).view(torch.bfloat16).pin_memory()
        pl = torch.from_numpy(lg).pin_memory()
        po = torch.full((3, H), 0.5, dtype=torch.float32).pin_memory()
        p.forward_host(0, px, pl, out=po, accumulate=True)
        res["host_acc"] = po.numpy().copy()
        dist.barrier()  # no rank frees its exchange buffer while a peer may still use it
        p.close()
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, res))
    except Exception as e:
        import traceback
        q.put((rank, traceback.format_exc()[-3000:]))


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


@pytest.mark.parametrize("mode", ["experts", "units"])
def test_peer_exchange_two_gpus_matches_single_rank(mode):
    """experts: each rank owns half of the experts (popularity stripe); units: each rank owns half of
    the intermediate units of every expert."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import multiprocessing as mp
    from oracle.oracle import Port
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    ps = [ctx.Process(target=_rank, args=(r, 2, port, q, mode)) for r in range(2)]
    for p in ps:
        p.start()
    got = dict(q.get(timeout=300) for _ in ps)
    for p in ps:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    for r in range(2):
        assert not isinstance(got[r], str), got[r]
    W = _weights(5)
    ex = {e: ("bf16", np.concatenate([g, u], 0), d) for e, (g, u, d) in enumerate(W)}
    for T in TS:
        np.testing.assert_array_equal(got[0][T], got[1][T])  # the same bits on every rank
        x, lg = _inputs(T, 100 + T)
        ref, _, _, st = Port.moe_layer(x, lg, ex, K)
        assert st == 0
        assert_close(got[0][T], ref, what=f"ep2 {mode} peer exchange T={T}")
    sg, su, sd, wr = _shared(6)
    from oracle.oracle import bf2f
    for T in BLOCK_TS:
        np.testing.assert_array_equal(got[0][("block", T)], got[1][("block", T)])
        h2, x2 = _inputs(T, 200 + T)[0], _inputs(T, 300 + T)[0]
        logits = Port.router_logits(h2, wr)
        moe, _, _, st = Port.moe_layer(h2, logits, ex, K)
        assert st == 0
        y, _ = Port.shared_expert(h2, x2, sg, su, sd)
        ref = Port.combine_residual(y, None, moe)
        # x_next = bf16(y + moe): one rounding step of x_next and of y apart at most, plus the
        # north-star bar of the routed output moe (max-abs 2e-2; with these weights, scale 0.05, one
        # SwiGLU activation of ~50 rounding the other way moves it by ~0.01)
        assert_bf16_close(got[0][("block", T)], ref, f"ep2 {mode} moe_block_forward T={T}", slack=_ulp_bf16(bf2f(y)),
                          atol=2e-2)
    np.testing.assert_array_equal(got[0]["host_acc"], got[1]["host_acc"])
    x, lg = _inputs(3, 103)
    ref, _, _, _ = Port.moe_layer(x, lg, ex, K)
    assert_close(got[0]["host_acc"], ref + 0.5, what="ep2 host accumulate")
