"""Expert-parallel host logic on CPU: the shard map (placement plan -> owner rank) and the partial-sum
combine over a world-size-2 gloo process group.  Each rank computes, with the CPU oracle, the cold-
expert path (solar_hybrid/cpu_moe.cpp:38-96) over only the experts it owns; the all-reduce of the
partials must reproduce the single-rank layer."""
import os
import socket

import numpy as np
import pytest

from npu_offload_b200.parallel import local_experts, ranks_by_count, shard_map
from oracle.oracle import Port
from tests.parity import assert_close

H, F, E, K, T = 256, 128, 8, 2, 3


def _weights(seed):
    rng = np.random.default_rng(seed)
    from npu_offload_b200.synth import f2bf
    ex = {}
    for e in range(E):
        gu = f2bf(rng.standard_normal((2 * F, H), np.float32) * 0.05)
        d = f2bf(rng.standard_normal((H, F), np.float32) * 0.05)
        ex[e] = ("bf16", gu, d)
    x = f2bf(rng.standard_normal((T, H), np.float32))
    lg = rng.standard_normal((T, E)).astype(np.float32)
    return ex, x, lg


def _partial(ex, x, lg, owned):
    """Oracle layer restricted to the experts in `owned`: route, group, run local jobs in job order."""
    idx, w, st = Port.route_softmax(lg, K)
    assert st == 0
    pm = Port.permute(idx, E)
    jobs, toks, ws = [], [], []
    for e in pm["job_order"]:
        e = int(e)
        if e not in owned:
            continue
        ps = pm["perm"][pm["offsets"][e]:pm["offsets"][e + 1]]
        jobs.append(ex[e])
        toks.append((ps // K).astype(np.int64))
        ws.append(w.reshape(-1)[ps].astype(np.float32))
    return Port.cpu_moe(x, jobs, toks, ws)


def test_shard_map_stripe_balances_hot_and_cold():
    counts = np.array([[50, 10, 40, 0, 5, 30, 20, 1]])
    order = ranks_by_count(counts[0])
    assert order == [0, 2, 5, 6, 1, 4, 7, 3]
    smap = shard_map(counts, 2)
    # popularity rank r -> rank r % 2: each rank gets every other expert of the hotness order
    assert [int(smap[0, e]) for e in order] == [0, 1, 0, 1, 0, 1, 0, 1]
    assert sorted(local_experts(smap, 0, 0) + local_experts(smap, 0, 1)) == list(range(E))
    top = shard_map(counts, 2, policy="top")
    assert [int(top[0, e]) for e in order] == [0, 0, 0, 0, 1, 1, 1, 1]


def test_shard_map_uneven_world():
    counts = np.arange(10)[None, :]
    smap = shard_map(counts, 4)
    sizes = [len(local_experts(smap, 0, r)) for r in range(4)]
    assert sorted(sizes) == [2, 2, 3, 3] and sum(sizes) == 10


def _worker(rank, world, port, q):
    import torch
    import torch.distributed as dist
    from npu_offload_b200.parallel import allreduce_partial
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    try:
        import datetime
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
        ex, x, lg = _weights(7)
        idx, _, _ = Port.route_softmax(lg, K)
        counts = np.bincount(idx.ravel(), minlength=E)[None, :]
        smap = shard_map(counts, world)
        part = _partial(ex, x, lg, set(local_experts(smap, 0, rank)))
        t = torch.from_numpy(part.copy())
        allreduce_partial(t)
        q.put((rank, t.numpy()))
        dist.barrier()
        dist.destroy_process_group()
    except Exception as e:  # reported to the parent, which fails the test
        q.put((rank, repr(e)))


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def test_expert_parallel_partials_allreduce_to_the_full_layer_gloo():
    import multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = dict(q.get(timeout=120) for _ in ps)
    for p in ps:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    for r in range(2):
        assert not isinstance(res[r], str), res[r]
    ex, x, lg = _weights(7)
    full, _, _, st = Port.moe_layer(x, lg, ex, K)
    assert st == 0
    np.testing.assert_array_equal(res[0], res[1])  # every rank holds the same combined output
    assert_close(res[0], full, max_abs=1e-5, min_cos=0.9999999, what="ep2 gloo vs single rank")


def test_unit_ranges_partition_every_expert():
    from npu_offload_b200.parallel import unit_ranges
    for F, world in ((1280, 8), (1280, 2), (1280, 4), (256, 2), (640, 3)):
        r = unit_ranges(F, world)
        assert r[0][0] == 0 and r[-1][1] == F and len(r) == world
        assert all(a[1] == b[0] for a, b in zip(r, r[1:]))
        sizes = [b - a for a, b in r]
        assert all(s % 64 == 0 and s > 0 for s in sizes) and max(sizes) - min(sizes) <= 64
    with pytest.raises(ValueError):
        unit_ranges(1280, 32)  # 20 chunks of 64 units cannot feed 32 ranks


def test_unit_sharding_partials_sum_to_the_expert():
    """The ranks' partial outputs over their unit slices add up to the whole expert (restated cpu_moe)."""
    from npu_offload_b200 import synth
    from npu_offload_b200.parallel import unit_ranges, unit_slice
    H, F, T = 256, 256, 3
    g, u, d = synth.expert_weights(9, 0, 0, H, F)
    x = synth.hidden(19, T, H)
    w = np.array([0.7, 0.2, 1.0], np.float32)
    full = Port.cpu_moe(x, [("bf16", np.concatenate([g, u], 0), d)], [np.arange(T)], [w])
    parts = []
    for f0, f1 in unit_ranges(F, 4):
        gs, us, ds = unit_slice(g, u, d, f0, f1)
        parts.append(Port.cpu_moe(x, [("bf16", np.concatenate([gs, us], 0), np.ascontiguousarray(ds))],
                                  [np.arange(T)], [w]))
    assert_close(np.sum(parts, axis=0), full, max_abs=1e-5, min_cos=0.9999999, what="unit shards")
