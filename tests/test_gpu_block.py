"""The steps either side of the routed experts in one Solar MoE block (solar_engine/src/layer.rs:1-6):
router-logit producer + shared expert (dense/shared.rs:1-3) and the residual combine into the next
layer's input (dense/combine.rs:1), alone and fused around the routed experts (moe_block_forward),
against the oracle restatements."""
import numpy as np
import pytest
import torch

from npu_offload_b200 import synth
from oracle.oracle import Port, bf2f
from tests.gpu_util import bf16_np, gpu_experts
from tests.parity import assert_close, cosine

pytestmark = pytest.mark.gpu


def _ulp_bf16(v):
    """Spacing of bf16 values at |v| (the smallest normal spacing for tiny |v|)."""
    a = np.maximum(np.abs(np.asarray(v, np.float32)), np.float32(2.0 ** -126))
    return np.exp2(np.floor(np.log2(a)) - 7).astype(np.float32)


def assert_bf16_close(got_bits, ref_bits, what, slack=0.0, atol=1e-3):
    """bf16 outputs of fp32 sums whose summation order differs from the oracle's.  Every element is
    within one bf16 spacing of the oracle's (one rounding step), plus `slack` (the spacing of an input
    that was itself rounded once, e.g. y inside x_next), plus `atol` for the fp32 sum's own difference
    (a SwiGLU activation that rounds the other way moves an expert output by ~1e-4; it shows where
    x2 + shared cancels to a tiny |y|).  Nearly all elements are identical, and the north-star
    cosine holds."""
    g, r = bf2f(got_bits), bf2f(ref_bits)
    assert np.all(np.isfinite(g)), what
    d = np.abs(g - r)
    tol = _ulp_bf16(r) + slack + atol
    assert np.all(d <= tol), f"{what}: {int(np.sum(d > tol))} elements beyond the rounding steps"
    same = float(np.mean(got_bits == ref_bits))
    assert same >= 0.95, f"{what}: only {same:.3f} of the elements bit-identical"
    assert cosine(g, r) >= 0.9999, what


def _plane(H, F, E, K, seed, max_tokens=512):
    from npu_offload_b200.moe import MoEDataPlane
    W = gpu_experts(seed, E, H, F)
    p = MoEDataPlane(H, F, E, K, n_layers=2, max_tokens=max_tokens)
    for layer in range(2):
        for e, (g, u, d) in enumerate(W):
            p.load_expert(layer, e, g, u, d)
    gen = torch.Generator(device="cuda")
    shared = []
    for layer in range(2):
        gen.manual_seed(seed * 7 + layer)
        sg = (torch.randn(F, H, generator=gen, device="cuda") * 0.02).bfloat16()
        su = (torch.randn(F, H, generator=gen, device="cuda") * 0.02).bfloat16()
        sd = (torch.randn(H, F, generator=gen, device="cuda") * 0.02).bfloat16()
        wr = (torch.randn(E, H, generator=gen, device="cuda") * 0.02).bfloat16()
        p.load_shared(layer, sg, su, sd, wr)
        shared.append(tuple(bf16_np(t) for t in (sg, su, sd, wr)))
    ex = {e: ("bf16", np.concatenate([bf16_np(g), bf16_np(u)], 0), bf16_np(d)) for e, (g, u, d) in enumerate(W)}
    return p, ex, shared


def _inputs(T, H, seed):
    h2 = synth.hidden(seed, T, H)
    x2 = synth.hidden(seed + 1, T, H)
    return h2, x2


def _dev(bits):
    return torch.from_numpy(bits.view(np.int16)).view(torch.bfloat16).cuda()


@pytest.mark.parametrize("T", [1, 5, 16, 40, 300])
def test_shared_router_and_block_small(T):
    H, F, E, K = 1024, 256, 16, 4
    p, ex, shared = _plane(H, F, E, K, 3)
    try:
        layer = 1
        sg, su, sd, wr = shared[layer]
        h2, x2 = _inputs(T, H, 50 + T)
        extra = np.random.default_rng(T).standard_normal((T, H)).astype(np.float32) * 0.1
        # router-logit producer + shared expert
        y, lg = p.shared_router(layer, _dev(h2), _dev(x2), sync=True)
        lg = lg.cpu().numpy()
        lg_ref = Port.router_logits(h2, wr)
        np.testing.assert_allclose(lg, lg_ref, rtol=1e-5, atol=1e-5)
        y_ref, s_ref = Port.shared_expert(h2, x2, sg, su, sd)
        assert_bf16_close(bf16_np(y), y_ref, f"y T={T}")
        # the reference's own device-rounding checker (host_util.rs:35-57: 2 % + 1e-3, < 1 % outliers)
        y_dev, _ = Port.shared_expert(h2, x2, sg, su, sd, device_rounding=True)
        d = np.abs(bf2f(bf16_np(y)) - bf2f(y_dev))
        assert np.mean(d > 0.02 * np.abs(bf2f(y_dev)) + 0.01 + 1e-3) < 0.01
        # routed experts on the produced logits, then the residual combine
        moe = p.forward(layer, _dev(h2), torch.from_numpy(lg).cuda(), sync=True)
        xn = p.combine_residual(y, moe, extra=torch.from_numpy(extra).cuda(), sync=True)
        xb, yb, lb = p.block_forward(layer, _dev(h2), _dev(x2), extra=torch.from_numpy(extra).cuda(),
                                     return_parts=True, sync=True)
        np.testing.assert_array_equal(lb.cpu().numpy(), lg)
        if T < 8:  # from 8 tokens on the tensor-core path composes the separate calls
            # one fused decode grid streams the shared expert with the routed ones: its share
            # boundaries, hence the partial-sum order, differ from the separate calls'
            assert_bf16_close(bf16_np(yb), bf16_np(y), f"fused y T={T}")
            assert_bf16_close(bf16_np(xb), bf16_np(xn), f"fused x_next T={T}", slack=_ulp_bf16(bf2f(bf16_np(y))))
        else:  # the composition of the separate calls, bit for bit
            np.testing.assert_array_equal(bf16_np(yb), bf16_np(y))
            np.testing.assert_array_equal(bf16_np(xb), bf16_np(xn))
        # against the oracle: routed layer on the same logits, residual combine restated
        moe_ref, idx, _, st = Port.moe_layer(h2, lg, ex, K)
        assert st == 0
        assert_close(moe.cpu().numpy(), moe_ref, what=f"routed T={T}")
        # the combine itself is element-wise fp32: bit-exact on identical inputs
        np.testing.assert_array_equal(bf16_np(xn), Port.combine_residual(bf16_np(y), extra, moe.cpu().numpy()))
        assert_bf16_close(bf16_np(xb), Port.combine_residual(y_ref, extra, moe_ref), f"x_next T={T}",
                          slack=_ulp_bf16(bf2f(y_ref)))
        # host buffers give the same bits
        xh = p.block_forward_host(layer, torch.from_numpy(h2.view(np.int16)).view(torch.bfloat16),
                                  torch.from_numpy(x2.view(np.int16)).view(torch.bfloat16), extra=torch.from_numpy(extra))
        np.testing.assert_array_equal(bf16_np(xh), bf16_np(xb))
        # no extra: x_next = bf16(y + moe); repeated calls give the same bits
        xb0 = p.block_forward(layer, _dev(h2), _dev(x2), sync=True)
        np.testing.assert_array_equal(bf16_np(p.block_forward(layer, _dev(h2), _dev(x2), sync=True)), bf16_np(xb0))
        ref0 = Port.combine_residual(bf16_np(y), None, moe.cpu().numpy())
        if T < 8:
            assert_bf16_close(bf16_np(xb0), ref0, f"fused x_next, no extra, T={T}", slack=_ulp_bf16(bf2f(bf16_np(y))))
        else:
            np.testing.assert_array_equal(bf16_np(xb0), ref0)
    finally:
        p.close()


def test_block_solar_shape_decode():
    H, F, E, K, T = 4096, 1280, 128, 8, 1
    p, ex, shared = _plane(H, F, E, K, 4, max_tokens=16)
    try:
        sg, su, sd, wr = shared[0]
        h2, x2 = _inputs(T, H, 77)
        xb, yb, lb = p.block_forward(0, _dev(h2), _dev(x2), return_parts=True, sync=True)
        lg = lb.cpu().numpy()
        np.testing.assert_allclose(lg, Port.router_logits(h2, wr), rtol=1e-5, atol=1e-5)
        y_ref, _ = Port.shared_expert(h2, x2, sg, su, sd)
        assert_bf16_close(bf16_np(yb), y_ref, "y Solar")
        moe_ref, _, _, st = Port.moe_layer(h2, lg, ex, K)
        assert st == 0
        assert_bf16_close(bf16_np(xb), Port.combine_residual(y_ref, None, moe_ref), "x_next Solar",
                          slack=_ulp_bf16(bf2f(y_ref)))
    finally:
        p.close()


def test_block_needs_shared_weights():
    from npu_offload_b200._lib import MoEError
    from npu_offload_b200.moe import MoEDataPlane
    p = MoEDataPlane(256, 64, 8, 2, n_layers=2, max_tokens=8)
    try:
        h = torch.zeros(1, 256, dtype=torch.bfloat16, device="cuda")
        with pytest.raises(MoEError):
            p.block_forward(0, h, h, sync=True)
        with pytest.raises(MoEError):
            p.shared_router(0, h, h, sync=True)
    finally:
        p.close()
