"""Prefill batches (many tokens per expert): the expert FFN as grouped tensor-core GEMMs over the unit
tables, against the CUDA-core multi-kernel path and the oracle (solar_hybrid/cpu_moe.cpp:38-96)."""
import numpy as np
import pytest
import torch

from npu_offload_b200 import synth
from tests.gpu_util import bf16_np, gpu_experts
from tests.parity import assert_close

pytestmark = pytest.mark.gpu


def _plane(H, F, E, K, seed, q8=()):
    from npu_offload_b200.moe import MoEDataPlane
    W = gpu_experts(seed, E, H, F)
    p = MoEDataPlane(H, F, E, K, n_layers=1, max_tokens=512)
    for e, (g, u, d) in enumerate(W):
        p.load_expert(0, e, g, u, d)
    for e in q8:
        p.quantize_expert_q8(0, e)
    return p, W


def _run(p, x, lg, prefill, tc=True):
    from npu_offload_b200._lib import MOE_OPT_PREFILL_MIN_T, MOE_OPT_PREFILL_TC
    p.set_option(MOE_OPT_PREFILL_MIN_T, 64 if prefill else 0)
    p.set_option(MOE_OPT_PREFILL_TC, 1 if tc else 0)
    xd = torch.from_numpy(x.view(np.int16)).view(torch.bfloat16).cuda()
    out, idx, w = p.forward(0, xd, torch.from_numpy(lg).cuda(), return_topk=True, sync=True)
    return out.cpu().numpy(), idx.cpu().numpy()


# T=512 with skewed routing gives jobs of 26..440 pairs: one- and two-tile jobs, half-full tiles
@pytest.mark.parametrize("T,zipf", [(64, False), (300, False), (512, True)])
def test_prefill_matches_cuda_core_path_and_oracle_small(T, zipf):
    from oracle.oracle import Port
    H, F, E, K = 1024, 256, 16, 4
    p, W = _plane(H, F, E, K, 41)
    try:
        x = synth.hidden(T, T, H)
        lg = synth.logits(T, T, E, zipf=zipf)
        pre, pi = _run(p, x, lg, True)
        core, ci = _run(p, x, lg, False)
        np.testing.assert_array_equal(pi, ci)
        assert_close(pre, core, what=f"prefill vs cuda cores T={T}")
        ex = {e: ("bf16", np.concatenate([bf16_np(g), bf16_np(u)], 0), bf16_np(d)) for e, (g, u, d) in enumerate(W)}
        ref, idx, _, st = Port.moe_layer(x, lg, ex, K)
        assert st == 0
        np.testing.assert_array_equal(pi, idx)
        assert_close(pre, ref, what=f"prefill vs oracle T={T}")
    finally:
        p.close()


def test_prefill_solar_shape_and_int8_fallback():
    H, F, E, K, T = 4096, 1280, 128, 8, 256
    p, _ = _plane(H, F, E, K, 42)
    try:
        x = synth.hidden(7, T, H)
        lg = synth.logits(7, T, E, zipf=False)
        pre, _ = _run(p, x, lg, True)
        core, _ = _run(p, x, lg, False)
        lib_gemm, _ = _run(p, x, lg, True, tc=False)
        # the tcgen05 kernels keep g, u and y in fp32 like the CUDA-core path (only the summation
        # order differs); the library GEMMs round g, u and y to bf16
        d_tc, _ = assert_close(pre, core, what="tcgen05 prefill vs cuda cores, Solar shape")
        d_lib, _ = assert_close(lib_gemm, core, what="library-GEMM prefill vs cuda cores, Solar shape")
        assert d_tc < d_lib, (d_tc, d_lib)
        # a routed int8 expert keeps the batch on the CUDA-core path (same bits as forcing it)
        p.quantize_expert_q8(0, 3)
        pre8, _ = _run(p, x, lg, True)
        core8, _ = _run(p, x, lg, False)
        np.testing.assert_array_equal(pre8, core8)
    finally:
        p.close()
