"""Router + permutation on the GPU, through the C ABI, against the oracle: bit-exact indices,
permutation and job order (the north-star parity bar), weights within 1e-6 relative; the routers'
exp bit-exact against the oracle's over every float of its domain."""
import json
import os

import numpy as np
import pytest

from oracle.oracle import Port
from tests.conftest import GOLDEN

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def planes():
    from npu_offload_b200.moe import MoEDataPlane
    cache = {}

    def get(E, K, scoring="softmax"):
        key = (E, K, scoring)
        if key not in cache:
            cache[key] = MoEDataPlane(256, 64, E, K, n_layers=1, max_tokens=4096, scoring=scoring)
        return cache[key]
    yield get
    for p in cache.values():
        p.close()


def _kat():
    with open(os.path.join(GOLDEN, "route_softmax_kat.json")) as f:
        return json.load(f)["cases"]


@pytest.mark.parametrize("case", _kat(), ids=lambda c: c["name"])
def test_softmax_known_answers(planes, case):
    from npu_offload_b200._lib import MOE_ENONFINITE, MOE_OK
    p = planes(case["E"], case["K"])
    lg = np.array([[float(v) for v in case["logits"]]], np.float32)
    r = p.route(lg)
    if case["error"]:
        assert r["status"] == MOE_ENONFINITE
        assert p.route(np.zeros((1, case["E"]), np.float32))["status"] == MOE_OK  # status was cleared
        return
    assert r["status"] == MOE_OK
    assert r["idx"][0].tolist() == case["idx"]
    if case["w_exact"]:
        assert r["w"][0].tolist() == case["w"]
    else:
        np.testing.assert_allclose(r["w"][0], case["w"], rtol=2e-6)


def _check_route(r, lg, K, E, scoring=0, bias=None):
    if scoring == 0:
        idx, w, st = Port.route_softmax(lg, K)
    else:
        idx, w, st = Port.route_sigmoid(lg, bias, K)
    np.testing.assert_array_equal(r["idx"], idx)
    np.testing.assert_allclose(r["w"], w, rtol=1e-6, atol=1e-12)
    pm = Port.permute(idx, E)
    for k in ("counts", "offsets", "perm", "job_order"):
        np.testing.assert_array_equal(r[k], pm[k], err_msg=k)
    assert int(r["n_jobs"][0]) == len(pm["job_order"])
    return float(np.mean(r["w"] == w))


@pytest.mark.parametrize("T", [1, 3, 4, 16, 64, 65, 257, 2048, 4096])
def test_route_matches_oracle_zipf(planes, T):
    from npu_offload_b200 import synth
    E, K = 128, 8
    lg = synth.logits(1000 + T, T, E, zipf=True)
    p = planes(E, K)
    _check_route(p.route(lg), lg, K, E)


def test_route_topk_bitexact_100k_tokens(planes):
    """100k Zipf-biased tokens: no top-k index may differ from the oracle's."""
    from npu_offload_b200 import synth
    E, K, T = 128, 8, 4096
    p = planes(E, K)
    exact_w = []
    for b in range(25):
        lg = synth.logits(50000 + b, T, E, zipf=True)
        exact_w.append(_check_route(p.route(lg), lg, K, E))
    print("fraction of bit-identical weights:", float(np.mean(exact_w)))


def test_route_ties_break_to_lower_index(planes):
    rng = np.random.default_rng(5)
    E, K, T = 128, 8, 512
    lg = np.round(rng.standard_normal((T, E)) * 2.0) / 2.0  # many exact ties
    lg = lg.astype(np.float32)
    p = planes(E, K)
    _check_route(p.route(lg), lg, K, E)


@pytest.mark.parametrize("E,K", [(16, 4), (32, 1), (64, 16), (256, 8), (200, 7)])
def test_route_other_shapes(planes, E, K):
    from npu_offload_b200 import synth
    T = 97
    lg = synth.logits(7 + E + K, T, E, zipf=True)
    _check_route(planes(E, K).route(lg), lg, K, E)


@pytest.mark.parametrize("E,K,T", [(256, 16, 4096), (200, 7, 1000), (16, 4, 33)])
def test_permutation_large_and_ragged(planes, E, K, T):
    """Largest shared-memory footprint (4096 tokens x top-16 over 256 experts) and ragged token tiles."""
    from npu_offload_b200 import synth
    lg = synth.logits(11 + T, T, E, zipf=True)
    _check_route(planes(E, K).route(lg), lg, K, E)


def test_route_sigmoid_reference_golden(planes, golden):
    g = golden("route_sigmoid.npz")
    E, K = g["logits"].shape[1], int(g["K"])
    p = planes(E, K, "sigmoid")
    r = p.route(g["logits"], bias=g["bias"])
    _check_route(r, g["logits"], K, E, scoring=1, bias=g["bias"])
    for t in range(g["logits"].shape[0]):
        assert sorted(r["idx"][t].tolist()) == sorted(g["idx"][t].tolist())


def test_route_empty_batch(planes):
    p = planes(128, 8)
    r = p.route(np.zeros((0, 128), np.float32))
    assert r["status"] == 0 and int(r["n_jobs"][0]) == 0 and r["counts"].sum() == 0


def test_router_exp_matches_oracle_over_the_whole_domain():
    """Every float x in [-104, 0] (the softmax's exp(v - max)) and in [0, 88.72] (the sigmoid's
    exp(-v)): the GPU routers' exp (moe_router_exp, the device function every router kernel calls)
    gives the same fp32 bits as the oracle's.  Outside that range both give 0 / +inf."""
    import ctypes
    import torch
    from npu_offload_b200._lib import MOE_OK, lib
    neg0, neg104 = 0x80000000, int(np.float32(-104.0).view(np.uint32))
    pos8872 = int(np.float32(88.72).view(np.uint32))
    chunk = 1 << 26
    x = torch.empty(chunk, dtype=torch.int64, device="cuda")
    y = torch.empty(chunk, dtype=torch.float32, device="cuda")
    yh = torch.empty(chunk, dtype=torch.float32).pin_memory()
    total = bad = 0
    for lo, hi in ((neg0, neg104), (0, pos8872)):
        for b0 in range(lo, hi + 1, chunk):
            n = min(chunk, hi + 1 - b0)
            torch.arange(b0, b0 + n, dtype=torch.int64, device="cuda", out=x[:n])
            xb = torch.where(x[:n] >= 2 ** 31, x[:n] - 2 ** 32, x[:n]).to(torch.int32).view(torch.float32)
            st = lib().moe_router_exp(ctypes.c_void_p(xb.data_ptr()), ctypes.c_void_p(y.data_ptr()), n,
                                      ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
            assert st == MOE_OK
            yh[:n].copy_(y[:n])
            ref = Port.router_exp_range(b0, n)
            got = yh[:n].numpy()
            bad += int(np.count_nonzero(got.view(np.uint32) != ref.view(np.uint32)))
            total += n
    print(f"router exp: {bad} mismatches over {total} floats")
    assert total == (neg104 - neg0 + 1) + (pos8872 + 1)
    assert bad == 0
