"""The fused decode kernel (routing + expert GEMV + combine in one persistent launch) against the
multi-kernel path and the oracle, its bounded-wait error path, and expert-parallel partial sums."""
import numpy as np
import pytest
import torch

from npu_offload_b200 import synth
from tests.gpu_util import bf16_np, gpu_experts, oracle_layer
from tests.parity import assert_close

pytestmark = pytest.mark.gpu

H, F, E, K = 4096, 1280, 128, 8


@pytest.fixture(scope="module")
def layer():
    from npu_offload_b200.moe import MoEDataPlane
    W = gpu_experts(33, E, H, F)
    from npu_offload_b200._lib import MOE_OPT_PREFILL_MIN_T
    p = MoEDataPlane(H, F, E, K, n_layers=1, max_tokens=32)
    for e, (g, u, d) in enumerate(W):
        p.load_expert(0, e, g, u, d)
    p.set_option(MOE_OPT_PREFILL_MIN_T, 0)  # every batch up to 16 tokens on the fused kernel
    yield p, W
    p.close()


def _inputs(seed, T):
    x = synth.hidden(seed, T, H)
    lg = synth.logits(seed, T, E)
    return x, lg, torch.from_numpy(x.view(np.int16)).view(torch.bfloat16).cuda(), torch.from_numpy(lg).cuda()


@pytest.mark.parametrize("T", [1, 3, 8, 12, 16])
def test_fused_matches_multikernel_path_and_oracle(layer, T):
    from npu_offload_b200._lib import MOE_OPT_FUSED_DECODE
    p, W = layer
    x, lg, xd, lgd = _inputs(900 + T, T)
    fused, fi, fw = p.forward(0, xd, lgd, return_topk=True, sync=True)
    p.set_option(MOE_OPT_FUSED_DECODE, 0)
    try:
        multi, mi, mw = p.forward(0, xd, lgd, return_topk=True, sync=True)
    finally:
        p.set_option(MOE_OPT_FUSED_DECODE, 1)
    np.testing.assert_array_equal(fi.cpu().numpy(), mi.cpu().numpy())
    np.testing.assert_array_equal(fw.cpu().numpy(), mw.cpu().numpy())
    assert_close(fused.cpu().numpy(), multi.cpu().numpy(), max_abs=1e-4, min_cos=0.9999999, what="fused vs multi")
    ids = sorted(set(fi.cpu().numpy().ravel().tolist()))
    ex = {e: ("bf16", np.concatenate([bf16_np(W[e][0]), bf16_np(W[e][1])], 0), bf16_np(W[e][2])) for e in ids}
    ref, idx, _, _, kind = oracle_layer(x, lg, ex, K)
    np.testing.assert_array_equal(fi.cpu().numpy(), idx)
    assert_close(fused.cpu().numpy(), ref, what=f"fused T={T} vs {kind}")


def test_fused_back_to_back_layers_are_independent(layer):
    """Consecutive launches overlap (programmatic dependent launch, fewer reducers, smaller shares for
    the CTAs that start late); results must not mix.  A call planned while the previous one still runs
    cuts its shares differently from a call made alone, so the summation order (not the arithmetic)
    differs: equal within fp32 rounding.  With MOE_OPT_REDUCERS = 0 every call uses the even cut and
    the bits are identical."""
    from npu_offload_b200._lib import MOE_OPT_REDUCERS
    p, _ = layer
    ins = [_inputs(1000 + i, 1 + (i % 4)) for i in range(12)]

    def run():
        outs, refs = [], []
        for _, _, xd, lgd in ins:
            outs.append(p.forward(0, xd, lgd))
        torch.cuda.synchronize()
        for _, _, xd, lgd in ins:
            refs.append(p.forward(0, xd, lgd, sync=True))
        return [(a.cpu().numpy(), b.cpu().numpy()) for a, b in zip(outs, refs)]

    for a, b in run():
        np.testing.assert_allclose(a, b, rtol=1e-5, atol=1e-6)
    p.set_option(MOE_OPT_REDUCERS, 0)
    try:
        for a, b in run():
            np.testing.assert_array_equal(a, b)
    finally:
        p.set_option(MOE_OPT_REDUCERS, 48)


def test_bounded_wait_reports_timeout_and_context_recovers(layer):
    """A readiness count that is never published: the kernel gives up after the bound, reports
    MOE_ETIMEOUT, and the next call on the same context is correct."""
    from npu_offload_b200._lib import (MOE_ETIMEOUT, MOE_OPT_INJECT_WAIT_TIMEOUT, MOE_OPT_WAIT_TIMEOUT_US, MoEError)
    p, _ = layer
    x, lg, xd, lgd = _inputs(77, 2)
    good = p.forward(0, xd, lgd, sync=True).cpu().numpy()
    p.set_option(MOE_OPT_WAIT_TIMEOUT_US, 20000)
    p.set_option(MOE_OPT_INJECT_WAIT_TIMEOUT, 1)
    try:
        with pytest.raises(MoEError) as ei:
            p.forward(0, xd, lgd, sync=True)
        assert ei.value.status == MOE_ETIMEOUT
    finally:
        p.set_option(MOE_OPT_INJECT_WAIT_TIMEOUT, 0)
        p.set_option(MOE_OPT_WAIT_TIMEOUT_US, 1000000)
    again = p.forward(0, xd, lgd, sync=True).cpu().numpy()
    np.testing.assert_array_equal(again, good)


def test_host_buffers_errors_timeout_and_accumulate(layer):
    """Host-buffer calls on the fused path: the kernels read the pinned logits and write the pinned
    output in place and leave their error bits in a pinned word.  A NaN logit is reported and does not
    leak into the next call; an injected timeout is reported and the context recovers; accumulate adds
    to the caller's output."""
    from npu_offload_b200._lib import (MOE_ENONFINITE, MOE_ETIMEOUT, MOE_OPT_INJECT_WAIT_TIMEOUT,
                                       MOE_OPT_WAIT_TIMEOUT_US, MoEError)
    p, _ = layer
    T = 3
    x, lg, xd, lgd = _inputs(55, T)
    ref = p.forward(0, xd, lgd, sync=True).cpu().numpy()
    px = torch.from_numpy(x.view(np.int16)).view(torch.bfloat16).pin_memory()
    pl = torch.from_numpy(lg).pin_memory()
    po = torch.empty(T, H, dtype=torch.float32).pin_memory()
    p.forward_host(0, px, pl, out=po)
    np.testing.assert_array_equal(po.numpy(), ref)
    bad = pl.clone().pin_memory()
    bad[1, 5] = float("nan")
    with pytest.raises(MoEError) as ei:
        p.forward_host(0, px, bad, out=po)
    assert ei.value.status == MOE_ENONFINITE
    p.forward_host(0, px, pl, out=po)  # no error carried over
    np.testing.assert_array_equal(po.numpy(), ref)
    p.set_option(MOE_OPT_WAIT_TIMEOUT_US, 20000)
    p.set_option(MOE_OPT_INJECT_WAIT_TIMEOUT, 1)
    try:
        with pytest.raises(MoEError) as ei:
            p.forward_host(0, px, pl, out=po)
        assert ei.value.status == MOE_ETIMEOUT
    finally:
        p.set_option(MOE_OPT_INJECT_WAIT_TIMEOUT, 0)
        p.set_option(MOE_OPT_WAIT_TIMEOUT_US, 1000000)
    p.forward_host(0, px, pl, out=po)
    np.testing.assert_array_equal(po.numpy(), ref)
    base = torch.full((T, H), 0.5, dtype=torch.float32).pin_memory()
    p.forward_host(0, px, pl, out=base, accumulate=True)
    np.testing.assert_allclose(base.numpy(), ref + 0.5, atol=1e-6)


def test_forward_layers_matches_single_calls(layer):
    """moe_forward_layers enqueues the calls moe_forward would make, in order: the same outputs (a
    streamed call may cut its shares differently, so within fp32 summation order), and an error of a
    later call (a NaN logit) is reported."""
    from npu_offload_b200._lib import MOE_ENONFINITE, MoEError
    p, _ = layer
    ins = [_inputs(700 + i, 1 + i % 3) for i in range(6)]
    for T in (1, 2, 3):
        sel = [c for c in ins if c[2].shape[0] == T]
        outs = [torch.empty(T, H, dtype=torch.float32, device="cuda") for _ in sel]
        p.forward_layers([0] * len(sel), [c[2] for c in sel], [c[3] for c in sel], outs, sync=True)
        for c, o in zip(sel, outs):
            ref = p.forward(0, c[2], c[3], sync=True)
            np.testing.assert_allclose(o.cpu().numpy(), ref.cpu().numpy(), rtol=1e-5, atol=1e-6)
    bad = ins[1][3].clone()
    bad[0, 3] = float("nan")
    outs = [torch.empty(2, H, dtype=torch.float32, device="cuda") for _ in range(2)]
    with pytest.raises(MoEError) as ei:
        p.forward_layers([0, 0], [ins[4][2], ins[1][2]], [ins[4][3], bad], outs, sync=True)
    assert ei.value.status == MOE_ENONFINITE
    p.forward(0, ins[1][2], ins[1][3], sync=True)  # the error does not stick


def test_host_calls_interleaved_with_device_calls(layer):
    """Host-buffer calls alternating with device-buffer calls on one context, each host call made
    right after a device call: every host call must wait for all of its own input copies (a host call
    must never see the copy count of an earlier one) and match the device call on the same inputs."""
    p, _ = layer
    T = 2
    cases = []
    for i in range(6):
        x, lg, xd, lgd = _inputs(300 + i, T)
        cases.append((torch.from_numpy(x.view(np.int16)).view(torch.bfloat16).pin_memory(),
                      torch.from_numpy(lg).pin_memory(), xd, lgd))
    refs = [p.forward(0, xd, lgd, sync=True).cpu().numpy() for _, _, xd, lgd in cases]
    po = torch.empty(T, H, dtype=torch.float32).pin_memory()
    for rep in range(3):
        for i, (px, pl, xd, lgd) in enumerate(cases):
            p.forward(0, cases[(i + 1) % len(cases)][2], cases[(i + 1) % len(cases)][3])  # device call in flight
            p.forward_host(0, px, pl, out=po)
            np.testing.assert_array_equal(po.numpy(), refs[i])


def test_expert_parallel_partials_sum_to_the_full_layer(layer):
    """Two expert-parallel rank contexts on one GPU: each computes its local experts only; the sum of
    the partials equals the unsharded layer."""
    from npu_offload_b200.moe import MoEDataPlane
    from npu_offload_b200.parallel import shard_map
    p, W = layer
    smap = shard_map(np.exp(synth.zipf_bias(5, E))[None, :], 2)
    ranks = [MoEDataPlane(H, F, E, K, n_layers=1, max_tokens=32, ep_rank=r, ep_world=2, shard_map=smap)
             for r in range(2)]
    try:
        from npu_offload_b200._lib import MOE_OPT_PREFILL_MIN_T
        for e in range(E):
            ranks[int(smap[0, e])].load_expert(0, e, *W[e])
        for r in ranks:
            r.set_option(MOE_OPT_PREFILL_MIN_T, 0)  # the same paths as the unsharded layer's
        for T in (1, 4, 16, 24):
            x, lg, xd, lgd = _inputs(1200 + T, T)
            full = p.forward(0, xd, lgd, sync=True).cpu().numpy()
            parts = [r.forward(0, xd, lgd, sync=True).cpu().numpy() for r in ranks]
            assert_close(parts[0] + parts[1], full, max_abs=1e-4, min_cos=0.9999999, what=f"ep2 T={T}")
    finally:
        for r in ranks:
            r.close()


@pytest.mark.parametrize("T", [8, 16])
def test_batches_from_8_tokens_take_the_tensor_core_path(layer, T):
    """With the threshold at 8 tokens (MOE_OPT_PREFILL_MIN_T; the default is 10) a bf16 layer's batch
    of 8 or more tokens runs as grouped tensor-core GEMMs (each routed expert read once): the same
    top-k, the output within the parity bar of the fused kernel's and of the oracle, and more than one
    launch."""
    from npu_offload_b200._lib import MOE_OPT_PREFILL_MIN_T
    p, W = layer
    x, lg, xd, lgd = _inputs(1400 + T, T)
    fused, fi, _ = p.forward(0, xd, lgd, return_topk=True, sync=True)
    p.set_option(MOE_OPT_PREFILL_MIN_T, 8)
    try:
        n0 = p.launch_count
        tc, ti, _ = p.forward(0, xd, lgd, return_topk=True, sync=True)
        assert p.launch_count - n0 > 1
    finally:
        p.set_option(MOE_OPT_PREFILL_MIN_T, 0)
    np.testing.assert_array_equal(ti.cpu().numpy(), fi.cpu().numpy())
    assert_close(tc.cpu().numpy(), fused.cpu().numpy(), what=f"tensor cores vs fused T={T}")
    ids = sorted(set(fi.cpu().numpy().ravel().tolist()))
    ex = {e: ("bf16", np.concatenate([bf16_np(W[e][0]), bf16_np(W[e][1])], 0), bf16_np(W[e][2])) for e in ids}
    ref, idx, _, _, kind = oracle_layer(x, lg, ex, K)
    np.testing.assert_array_equal(ti.cpu().numpy(), idx)
    assert_close(tc.cpu().numpy(), ref, what=f"tensor cores T={T} vs {kind}")
