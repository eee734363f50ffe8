"""moe_ck_moe3_noalloc: the ck_moe3 surface for callers that may not allocate device memory.

Some callers cannot call cudaMalloc at all -- a serving process whose own allocator already owns
all of HBM (expert tables plus KV cache), or a framework that forbids allocations outside its
pool -- so they cannot create a moe_ctx, whose creation allocates.  This entry point needs no
context: the caller passes inputs and outputs, and the working memory is a 1 MiB file-scope device
array inside libmoe_dp.so.  These tests call it through the C ABI and compare it with the existing
context-based moe_ck_moe3 and with the reference's own ck_moe3 (track2_opt/solar_engine/csrc/
cpu_kern.c:141-172, compiled from the reference sources; the C restatement where this host cannot
run it) on two calls in a row (different experts, tokens and weights, so stale scratch from the
first call cannot leak into the second), within the parity tolerance used everywhere else (max-abs
2e-2, cosine 0.9999).  The file name makes pytest collect it last.
"""
import ctypes

import numpy as np
import pytest
import torch

from tests.parity import assert_close

pytestmark = pytest.mark.gpu

H, F = 4096, 1280


def _bases(n, seed):
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    return [(torch.randn(3 * F * H, generator=g, device="cuda") * 0.02).to(torch.bfloat16) for _ in range(n)]


def _noalloc(bases, w, x, out):
    from npu_offload_b200._lib import lib
    arr = (ctypes.c_void_p * len(bases))(*[b.data_ptr() for b in bases])
    return lib().moe_ck_moe3_noalloc(len(bases), arr, ctypes.c_void_p(w.data_ptr()), ctypes.c_void_p(x.data_ptr()),
                                     ctypes.c_void_p(out.data_ptr()), H, F,
                                     ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))


def _reference_ck_moe3(bases, w, x, init):
    """out = init + sum_e w[e] * expert_e(x) on the CPU: the reference's ck_moe3 when it runs here."""
    from oracle.oracle import Port, Reference
    from tests.gpu_util import bf16_np
    b = [bf16_np(t) for t in bases]
    wn, xn, out = w.cpu().numpy().astype(np.float32), bf16_np(x), init.cpu().numpy().astype(np.float32).copy()
    if Reference.available():
        return Reference.ck_moe3(b, wn, xn, out), "reference ck_moe3"
    jobs = [("bf16", a[:2 * F * H].reshape(2 * F, H), a[2 * F * H:].reshape(H, F)) for a in b]
    acc = out[None].copy()
    Port.cpu_moe(xn[None], jobs, [[0]] * len(b), [[v] for v in wn], out=acc, accumulate=True)
    return acc[0], "oracle ck_moe3 restatement"


def test_noalloc_matches_ck_moe3_on_two_calls():
    from npu_offload_b200._lib import MOE_OK
    from npu_offload_b200.moe import MoEDataPlane
    cases = []
    for n, seed in ((8, 101), (5, 202)):
        bases = _bases(n, seed)
        gen = torch.Generator(device="cuda")
        gen.manual_seed(seed + 1)
        x = torch.randn(H, generator=gen, device="cuda").to(torch.bfloat16)
        w = torch.rand(n, generator=gen, device="cuda") * 0.3 + 0.05
        init = torch.randn(H, generator=gen, device="cuda") * 0.1
        cases.append((bases, w, x, init))
    with MoEDataPlane(H, F, 16, 16, max_tokens=4) as plane:
        refs = []
        for bases, w, x, init in cases:
            acc = init.clone()
            plane.ck_moe3(bases, w, x, acc)
            refs.append(acc)
        torch.cuda.synchronize()
    outs = [init.clone() for _, _, _, init in cases]
    torch.cuda.synchronize()
    for i, (bases, w, x, _) in enumerate(cases):
        free_before = torch.cuda.mem_get_info()[0]
        assert _noalloc(bases, w, x, outs[i]) == MOE_OK
        torch.cuda.synchronize()
        if i == 1:  # the first call may trigger the lazy module load; later calls must not allocate
            assert torch.cuda.mem_get_info()[0] == free_before
        got = outs[i].cpu().numpy()
        assert_close(got, refs[i].cpu().numpy(), what=f"noalloc call {i + 1} vs moe_ck_moe3")
        ref, kind = _reference_ck_moe3(bases, w, x, cases[i][3])
        d, c = assert_close(got, ref, what=f"noalloc call {i + 1} vs {kind}")
        print(f"noalloc call {i + 1} vs {kind}: max-abs {d:.3g}, cosine {c:.7f}")


def test_noalloc_rejects_sizes_beyond_its_scratch():
    from npu_offload_b200._lib import MOE_EINVAL, MOE_OK, last_error, lib
    x = torch.zeros(H, dtype=torch.bfloat16, device="cuda")
    out = torch.zeros(H, device="cuda")
    w = torch.ones(17, device="cuda")
    one = _bases(1, 7)[0]
    arr = (ctypes.c_void_p * 17)(*([one.data_ptr()] * 17))
    st = lib().moe_ck_moe3_noalloc(17, arr, ctypes.c_void_p(w.data_ptr()), ctypes.c_void_p(x.data_ptr()),
                                   ctypes.c_void_p(out.data_ptr()), H, F, None)
    assert st == MOE_EINVAL and "16-expert limit" in last_error()
    # 16 experts at H = 16384, F = 2048 need more than the 1 MiB array
    st = lib().moe_ck_moe3_noalloc(16, arr, ctypes.c_void_p(w.data_ptr()), ctypes.c_void_p(x.data_ptr()),
                                   ctypes.c_void_p(out.data_ptr()), 16384, 2048, None)
    assert st == MOE_EINVAL and "1 MiB" in last_error()
    assert lib().moe_ck_moe3_noalloc(0, None, None, None, None, H, F, None) == MOE_OK
    assert float(out.abs().sum()) == 0.0
