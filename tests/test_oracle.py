"""Pin the CPU oracle (oracle/moe_oracle.c) against the reference's own outputs (CPU only).

Golden fixtures come from the reference itself (tests/golden/make_golden.py): its compiled
cpu_moe.cpp / cpu_kern.c and its Python router.  When the compiled reference can run on this host,
the oracle is also compared with it live on fresh seeded inputs.
"""
import json
import os

import numpy as np
import pytest

from npu_offload_b200 import synth
from oracle.oracle import OR_ENONFINITE, OR_OK, Port, Reference
from tests.conftest import GOLDEN
from tests.parity import assert_close, sha


def _kat_cases():
    with open(os.path.join(GOLDEN, "route_softmax_kat.json")) as f:
        return json.load(f)["cases"]


@pytest.mark.parametrize("case", _kat_cases(), ids=lambda c: c["name"])
def test_softmax_router_known_answers(case):
    lg = np.array([[float(v) for v in case["logits"]]], np.float32)
    idx, w, st = Port.route_softmax(lg, case["K"])
    if case["error"]:
        assert st == OR_ENONFINITE
        return
    assert st == OR_OK
    assert idx[0].tolist() == case["idx"]
    if case["w_exact"]:
        assert w[0].tolist() == case["w"]
    else:
        np.testing.assert_allclose(w[0], case["w"], rtol=2e-6)


# The routers' exp domain: the softmax evaluates exp(v - max) <= 0 (below -104 it is 0 in fp32);
# the sigmoid evaluates exp(-v) for any v (above 88.72 it is +inf).
NEG_ZERO, NEG_104, POS_8872 = 0x80000000, int(np.float32(-104.0).view(np.uint32)), int(np.float32(88.72).view(np.uint32))
N_SOFTMAX = NEG_104 - NEG_ZERO + 1


def test_router_exp_is_correctly_rounded():
    """The routers' exp (double exp rounded once) equals the long-double exp rounded to fp32 on every
    61st float of [-104, 0] and every 61st float of [0, 88.72]."""
    assert Port.router_exp_vs_long_double(NEG_ZERO, N_SOFTMAX // 61, 61) == 0
    assert Port.router_exp_vs_long_double(0, (POS_8872 + 1) // 61, 61) == 0


def test_libm_expf_differs_from_router_exp_by_at_most_one_ulp():
    """The reference evaluates f32::exp through the platform libm (host.rs.tpl:249).  On this host's
    libm some of the 1.12e9 softmax-domain results are one ulp away from the correctly rounded value
    the routers use; none is further off."""
    bad, worst = Port.libm_expf_mismatches(NEG_ZERO, N_SOFTMAX)
    print(f"host libm expf differs from the correctly rounded exp on {bad} of {N_SOFTMAX} floats in [-104, 0]")
    assert worst <= 1, worst


def test_sigmoid_router_matches_reference_python(golden):
    g = golden("route_sigmoid.npz")
    idx, w, st = Port.route_sigmoid(g["logits"], g["bias"], int(g["K"]))
    assert st == OR_OK
    # the reference uses torch.topk(sorted=False): compare as sets, weights matched per expert
    for t in range(idx.shape[0]):
        assert sorted(idx[t].tolist()) == sorted(g["idx"][t].tolist()), t
        ref = dict(zip(g["idx"][t].tolist(), g["w"][t].tolist()))
        for e, v in zip(idx[t].tolist(), w[t].tolist()):
            assert abs(v - ref[e]) <= 1e-6 * max(1.0, abs(ref[e])), (t, e)


def _jobs(idx, w, E):
    pm = Port.permute(idx, E)
    K = idx.shape[1]
    toks, ws = [], []
    for e in pm["job_order"]:
        ps = pm["perm"][pm["offsets"][e]:pm["offsets"][e + 1]]
        toks.append((ps // K).astype(np.int64))
        ws.append(w.reshape(-1)[ps])
    return pm, toks, ws


def test_permutation_semantics():
    rng = np.random.default_rng(0)
    T, E, K = 37, 16, 4
    idx = np.stack([rng.choice(E, K, replace=False) for _ in range(T)]).astype(np.int32)
    pm = Port.permute(idx, E)
    assert pm["status"] == OR_OK
    # first-appearance job order of the t-major, k-minor scan (runtime.py:343-347)
    seen = []
    for t in range(T):
        for k in range(K):
            if idx[t, k] not in seen:
                seen.append(int(idx[t, k]))
    assert pm["job_order"].tolist() == seen
    assert pm["counts"].tolist() == np.bincount(idx.ravel(), minlength=E).tolist()
    assert pm["offsets"][-1] == T * K
    for e in range(E):
        ps = pm["perm"][pm["offsets"][e]:pm["offsets"][e + 1]]
        assert np.all(idx.reshape(-1)[ps] == e)
        assert np.all(np.diff(ps // K) > 0)  # tokens strictly ascending within an expert


def test_permutation_rejects_bad_indices():
    assert Port.permute(np.array([[0, 0]], np.int32), 4)["status"] != OR_OK  # repeated within a token
    assert Port.permute(np.array([[0, 9]], np.int32), 4)["status"] != OR_OK  # out of range


def test_ffn_small_golden(golden):
    g = golden("ffn_small.npz")
    seed, H, F, E, K = (int(g[k]) for k in ("seed", "H", "F", "E", "K"))
    experts = [synth.expert_weights(seed, 0, e, H, F) for e in range(E)]
    assert sha(*[a for trip in experts for a in trip]) == str(g["wsha"]), "seeded weights changed"
    idx, w, st = Port.route_softmax(g["logits"], K)
    assert st == OR_OK
    np.testing.assert_array_equal(idx, g["idx"])
    np.testing.assert_array_equal(w, g["w"])
    pm, toks, ws = _jobs(idx, w, E)
    np.testing.assert_array_equal(pm["job_order"], g["job_order"])
    jobs = [("bf16", np.concatenate(experts[e][:2], 0), experts[e][2]) for e in pm["job_order"]]
    out = Port.cpu_moe(g["x"], jobs, toks, ws)
    assert_close(out, g["out"], max_abs=1e-5, min_cos=0.9999999, what="port cpu_moe vs reference")
    full, idx2, _, st = Port.moe_layer(g["x"], g["logits"], {e: ("bf16", np.concatenate(experts[e][:2], 0),
                                                                 experts[e][2]) for e in range(E)}, K)
    assert st == OR_OK
    np.testing.assert_array_equal(idx2, g["idx"])
    np.testing.assert_array_equal(full, out)


def test_ffn_solar_golden(golden):
    g = golden("ffn_solar.npz")
    seed, H, F = int(g["seed"]), 4096, 1280
    for T in (1, 4):
        ex = g[f"T{T}_experts"].tolist()
        W = [synth.expert_weights(seed, 0, e, H, F) for e in ex]
        assert sha(*[a for trip in W for a in trip]) == str(g[f"T{T}_wsha"]), "seeded weights changed"
        off = g[f"T{T}_tok_off"]
        toks = [g[f"T{T}_toks"][off[j]:off[j + 1]] for j in range(len(ex))]
        ws = [g[f"T{T}_ws"][off[j]:off[j + 1]] for j in range(len(ex))]
        jobs = [("bf16", np.concatenate(W[j][:2], 0), W[j][2]) for j in range(len(ex))]
        out = Port.cpu_moe(g[f"T{T}_x"], jobs, toks, ws)
        assert_close(out, g[f"T{T}_out"], max_abs=2e-4, min_cos=0.999999, what=f"port cpu_moe T={T}")
        if T == 1:
            acc = np.full((1, H), 0.5, np.float32)
            Port.cpu_moe(g["T1_x"], jobs, toks, ws, out=acc, accumulate=True)
            assert_close(acc[0], g["ck_moe3_out"], max_abs=2e-4, min_cos=0.999999, what="port vs ck_moe3")


def test_q8_small_golden(golden):
    g = golden("q8.npz")
    for i in range(g["small_gate"].shape[0]):
        q, sc, rs = Port.place_expert_q8(g["small_gate"][i], g["small_up"][i], g["small_down"][i])
        np.testing.assert_array_equal(q, g["small_q"][i])
        np.testing.assert_array_equal(sc, g["small_sc"][i])
        np.testing.assert_array_equal(rs, g["small_rs"][i])
    jobs = [("q8", g["small_q"][i], g["small_sc"][i]) for i in range(3)]
    out = Port.cpu_moe(g["small_x"][None], jobs, [[0]] * 3, [[v] for v in g["small_w"]])
    assert_close(out[0], g["small_out"], max_abs=1e-5, min_cos=0.9999999, what="port q8w vs ck_moe_q8w")


def test_q8_solar_golden(golden):
    g = golden("q8.npz")
    seed, H, F = int(g["solar_seed"]), 4096, 1280
    jobs = []
    for e in range(2):
        q, sc, _ = Port.place_expert_q8(*synth.expert_weights(seed, 0, e, H, F))
        assert sha(q) == str(g["solar_qsha"][e]) and sha(sc) == str(g["solar_scsha"][e])
        jobs.append(("q8", q, sc))
    out = Port.cpu_moe(g["solar_x"][None], jobs, [[0], [0]], [[v] for v in g["solar_w"]])
    assert_close(out[0], g["solar_out"], max_abs=2e-4, min_cos=0.999999, what="port q8w solar")


@pytest.mark.skipif(not Reference.available(), reason="compiled reference unavailable: " + Reference.why_unavailable())
def test_oracle_matches_compiled_reference_live():
    rng = np.random.default_rng(1234)
    H, F, E, K, T = 512, 256, 12, 3, 9
    experts = {e: synth.expert_weights(99, 0, e, H, F) for e in range(E)}
    x = synth.hidden(99, T, H)
    lg = synth.logits(99, T, E)
    idx, w, st = Port.route_softmax(lg, K)
    pm, toks, ws = _jobs(idx, w, E)
    gus = [np.concatenate(experts[e][:2], 0) for e in pm["job_order"]]
    ds = [experts[e][2] for e in pm["job_order"]]
    ref = Reference.cpu_moe(x, gus, ds, toks, ws)
    port = Port.cpu_moe(x, [("bf16", a, b) for a, b in zip(gus, ds)], toks, ws)
    assert_close(port, ref, max_abs=1e-5, min_cos=0.9999999, what="live")
    # int8 tables are bit-identical to ck_place_expert_q8
    g0, u0, d0 = experts[0]
    for a, b in zip(Port.place_expert_q8(g0, u0, d0), Reference.place_expert_q8(g0, u0, d0)):
        np.testing.assert_array_equal(a, b)
    _ = rng


# ---- the steps either side of the path: router-logit producer, shared expert, residual combine ----

def _bf(a):
    from oracle.oracle import f2bf
    return f2bf(np.asarray(a, np.float32))


def test_router_logits_restatement():
    """logits = h2 . Wr^T in fp32 (solar_engine/src/dense/shared.rs:3) against a float64 product."""
    from oracle.oracle import bf2f
    rng = np.random.default_rng(7)
    h2, wr = _bf(rng.standard_normal((5, 512))), _bf(rng.standard_normal((24, 512)) * 0.02)
    got = Port.router_logits(h2, wr)
    ref = bf2f(h2).astype(np.float64) @ bf2f(wr).astype(np.float64).T
    np.testing.assert_allclose(got, ref, rtol=1e-5, atol=1e-6)


def test_shared_expert_restatement_rounding_points():
    """y = bf16(x2 + shared) with the shared expert in cpu_moe's rounding points: its fp32 output is
    exactly the restated cpu_moe with weight 1 for every token; device_rounding (the reference's
    expert_ref, host_util.rs:35-46) differs only by the bf16 rounding of g and u."""
    from oracle.oracle import bf2f
    H, F, T = 256, 128, 3
    g, u, d = synth.expert_weights(5, 0, 0, H, F)
    h2, x2 = synth.hidden(11, T, H), synth.hidden(12, T, H)
    y, s = Port.shared_expert(h2, x2, g, u, d)
    ref = Port.cpu_moe(h2, [("bf16", np.concatenate([g, u], 0), d)], [np.arange(T)], [np.ones(T, np.float32)])
    np.testing.assert_array_equal(s, ref)
    np.testing.assert_array_equal(y, _bf(bf2f(x2) + s))
    y2, s2 = Port.shared_expert(h2, x2, g, u, d, device_rounding=True)
    assert_close(s2, s, max_abs=2e-3, min_cos=0.9999, what="device rounding")


def test_combine_residual_restatement():
    """x_next = bf16((y + extra) + moe) (combine.rs:1): one rounding of the fp32 sum, exactly."""
    from oracle.oracle import bf2f
    rng = np.random.default_rng(3)
    y = _bf(rng.standard_normal(1000))
    ex = rng.standard_normal(1000).astype(np.float32)
    moe = rng.standard_normal(1000).astype(np.float32)
    np.testing.assert_array_equal(Port.combine_residual(y, ex, moe), _bf((bf2f(y) + ex) + moe))
    np.testing.assert_array_equal(Port.combine_residual(y, None, moe), _bf(bf2f(y) + moe))


@pytest.mark.skipif(not Reference.available(), reason="compiled reference unavailable: " + Reference.why_unavailable())
def test_shared_expert_matches_compiled_reference():
    """The shared expert in cpu_moe semantics against the compiled reference cpu_moe (weight 1)."""
    H, F, T = 512, 256, 4
    g, u, d = synth.expert_weights(21, 0, 0, H, F)
    h2, x2 = synth.hidden(31, T, H), synth.hidden(32, T, H)
    _, s = Port.shared_expert(h2, x2, g, u, d)
    ref = Reference.cpu_moe(h2, [np.concatenate([g, u], 0)], [d], [np.arange(T)], [np.ones(T, np.float32)])
    assert_close(s, ref, max_abs=1e-5, min_cos=0.9999999, what="shared vs cpu_moe")
