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


def _library_gemm_layer(x, lg, W, K):
    """The same layer with library GEMMs (torch.matmul on bf16 operands, which returns bf16): g, u
    and y are rounded to bf16 at the GEMM outputs; act = bf16(SwiGLU) as cpu_moe rounds it."""
    from oracle.oracle import Port
    idx, w, _ = Port.route_softmax(lg, K)
    xd = torch.from_numpy(x.view(np.int16)).view(torch.bfloat16).cuda()
    out = torch.zeros(x.shape[0], x.shape[1], dtype=torch.float32, device="cuda")
    for e in sorted(set(idx.ravel().tolist())):
        rows, ks = np.nonzero(idx == e)
        r = torch.from_numpy(rows).cuda()
        xs = xd[r]
        g = (xs @ W[e][0].T).float()
        u = (xs @ W[e][1].T).float()
        act = (g / (1 + torch.exp(-g)) * u).to(torch.bfloat16)
        y = (act @ W[e][2].T).float()
        out.index_add_(0, r, y * torch.from_numpy(w[rows, ks]).cuda()[:, None])
    return out.cpu().numpy()


def test_prefill_solar_shape_and_int8_fallback():
    H, F, E, K, T = 4096, 1280, 128, 8, 256
    p, W = _plane(H, F, E, K, 42)
    try:
        x = synth.hidden(7, T, H)
        lg = synth.logits(7, T, E, zipf=False)
        pre, _ = _run(p, x, lg, True)
        core, _ = _run(p, x, lg, False)
        lib_gemm = _library_gemm_layer(x, lg, W, K)
        # the tcgen05 kernels keep g, u and y in fp32 like the CUDA-core path (only the summation
        # order differs); library GEMMs with bf16 outputs round g, u and y to bf16
        d_tc, _ = assert_close(pre, core, what="tcgen05 prefill vs cuda cores, Solar shape")
        d_lib, _ = assert_close(lib_gemm, core, what="library-GEMM layer vs cuda cores, Solar shape")
        assert d_tc < d_lib, (d_tc, d_lib)
        # a routed int8 expert keeps the batch on the CUDA-core path (same bits as forcing it)
        p.quantize_expert_q8(0, 3)
        pre8, _ = _run(p, x, lg, True)
        core8, _ = _run(p, x, lg, False)
        np.testing.assert_array_equal(pre8, core8)
    finally:
        p.close()


def test_prefill_configs3_matches_reference_cpu_moe():
    """configs[3] exactly: one Solar-shaped layer (H 4096, 128 experts, F 1280, top-8) at 2048 prefill
    tokens with uniform routing (about 128 tokens per expert: 16,384 pairs, jobs of one and two
    256-pair tiles), on the default path (the tcgen05 grouped GEMMs), against the reference's own
    compiled cpu_moe (solar_hybrid/cpu_moe.cpp:38-96; the C restatement where this host cannot run it).
    The CUDA-core path on the same batch must agree too, and differ from it in the last bits (it is a
    different summation order, so the default run did take the tensor-core kernels)."""
    from npu_offload_b200.moe import MoEDataPlane
    from tests.gpu_util import oracle_layer
    H, F, E, K, T = 4096, 1280, 128, 8, 2048
    W = gpu_experts(43, E, H, F)
    p = MoEDataPlane(H, F, E, K, n_layers=1, max_tokens=T)
    try:
        for e, (g, u, d) in enumerate(W):
            p.load_expert(0, e, g, u, d)
        x = synth.hidden(2048, T, H)
        lg = synth.logits(2048, T, E, zipf=False)
        xd = torch.from_numpy(x.view(np.int16)).view(torch.bfloat16).cuda()
        out, gi, _ = p.forward(0, xd, torch.from_numpy(lg).cuda(), return_topk=True, sync=True)
        out = out.cpu().numpy()
        core, ci = _run(p, x, lg, False)
        np.testing.assert_array_equal(gi.cpu().numpy(), ci)
        assert not np.array_equal(out, core)
        ex = {e: ("bf16", np.concatenate([bf16_np(W[e][0]), bf16_np(W[e][1])], 0), bf16_np(W[e][2])) for e in range(E)}
        ref, idx, _, pm, kind = oracle_layer(x, lg, ex, K)
        np.testing.assert_array_equal(gi.cpu().numpy(), idx)
        assert pm["counts"].min() > 64 and len(pm["job_order"]) == E
        d, c = assert_close(out, ref, what=f"configs[3] tcgen05 prefill vs {kind}")
        d2, c2 = assert_close(core, ref, what=f"configs[3] CUDA-core path vs {kind}")
        print(f"configs[3] T={T}: tcgen05 vs {kind}: max-abs {d:.3g}, cosine {c:.8f}; "
              f"CUDA cores: max-abs {d2:.3g}, cosine {c2:.8f}")
    finally:
        p.close()
