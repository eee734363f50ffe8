"""Expert FFN on the GPU through the C ABI against the reference (compiled cpu_moe when the host can
run it, else the C restatement).  Parity bar: max-abs <= 2e-2 and cosine >= 0.9999 (bf16 weights,
fp32 accumulation); top-k indices bit-exact."""
import numpy as np
import pytest
import torch

from npu_offload_b200 import synth
from oracle.oracle import Port, Reference
from tests.gpu_util import bf16_np, gpu_experts, oracle_layer
from tests.parity import assert_close, sha

pytestmark = pytest.mark.gpu

H, F, E, K = 4096, 1280, 128, 8


@pytest.fixture(scope="module")
def solar():
    """One Solar-shaped layer (128 experts, 4 GB) resident on the GPU."""
    from npu_offload_b200.moe import MoEDataPlane
    p = MoEDataPlane(H, F, E, K, n_layers=1, max_tokens=64)
    W = gpu_experts(21, E, H, F)
    for e, (g, u, d) in enumerate(W):
        p.load_expert(0, e, g, u, d)
    yield p, W
    p.close()


def _experts_np(W, ids):
    return {e: ("bf16", np.concatenate([bf16_np(W[e][0]), bf16_np(W[e][1])], 0), bf16_np(W[e][2])) for e in ids}


@pytest.mark.parametrize("T", [1, 2, 4, 8, 16])
def test_forward_matches_reference(solar, T):
    p, W = solar
    x = synth.hidden(300 + T, T, H)
    lg = synth.logits(300 + T, T, E)
    idx0, _, _ = Port.route_softmax(lg, K)
    ex = _experts_np(W, sorted(set(idx0.ravel().tolist())))
    ref, idx, w, pm, kind = oracle_layer(x, lg, ex, K)
    xd = torch.from_numpy(x.view(np.int16)).view(torch.bfloat16).cuda()
    out, gi, gw = p.forward(0, xd, torch.from_numpy(lg).cuda(), return_topk=True, sync=True)
    np.testing.assert_array_equal(gi.cpu().numpy(), idx)
    d, c = assert_close(out.cpu().numpy(), ref, what=f"forward T={T} vs {kind}")
    print(f"T={T} vs {kind}: max-abs {d:.3g} cosine {c:.8f}")


def test_forward_deterministic_and_host_mode(solar):
    p, _ = solar
    T = 5
    x = synth.hidden(77, T, H)
    lg = synth.logits(77, T, E)
    xd = torch.from_numpy(x.view(np.int16)).view(torch.bfloat16).cuda()
    a = p.forward(0, xd, torch.from_numpy(lg).cuda(), sync=True).cpu().numpy()
    b = p.forward(0, xd, torch.from_numpy(lg).cuda(), sync=True).cpu().numpy()
    np.testing.assert_array_equal(a, b)
    h = p.forward_host(0, x, lg).numpy()
    np.testing.assert_array_equal(a, h)
    pinned_x = torch.from_numpy(x.view(np.int16)).view(torch.bfloat16).pin_memory()
    pinned_l = torch.from_numpy(lg).pin_memory()
    pinned_o = torch.empty(T, H, dtype=torch.float32).pin_memory()
    p.forward_host(0, pinned_x, pinned_l, out=pinned_o)
    np.testing.assert_array_equal(a, pinned_o.numpy())


def test_forward_accumulate(solar):
    p, _ = solar
    T = 3
    x = synth.hidden(88, T, H)
    lg = synth.logits(88, T, E)
    xd = torch.from_numpy(x.view(np.int16)).view(torch.bfloat16).cuda()
    base = torch.full((T, H), 0.25, device="cuda")
    plain = p.forward(0, xd, torch.from_numpy(lg).cuda(), sync=True)
    acc = p.forward(0, xd, torch.from_numpy(lg).cuda(), out=base.clone(), accumulate=True, sync=True)
    np.testing.assert_allclose(acc.cpu().numpy(), plain.cpu().numpy() + 0.25, atol=1e-6)


def test_forward_empty_and_errors(solar):
    from npu_offload_b200._lib import MOE_ENONFINITE, MOE_OK, MoEError
    p, _ = solar
    x = torch.zeros(0, H, dtype=torch.bfloat16, device="cuda")
    out = p.forward(0, x, torch.zeros(0, E, device="cuda"), sync=True)
    assert out.shape == (0, H)
    lg = torch.zeros(2, E, device="cuda")
    lg[1, 3] = float("nan")
    with pytest.raises(MoEError) as ei:
        p.forward(0, torch.zeros(2, H, dtype=torch.bfloat16, device="cuda"), lg, sync=True)
    assert ei.value.status == MOE_ENONFINITE
    assert p.status() == MOE_OK
    with pytest.raises(MoEError):
        p.forward(1, torch.zeros(1, H, dtype=torch.bfloat16, device="cuda"), torch.zeros(1, E, device="cuda"))
    with pytest.raises(MoEError):
        p.forward(0, torch.zeros(65, H, dtype=torch.bfloat16, device="cuda"), torch.zeros(65, E, device="cuda"))


def test_unloaded_expert_is_a_state_error():
    from npu_offload_b200._lib import MOE_ESTATE, MoEError
    from npu_offload_b200.moe import MoEDataPlane
    with MoEDataPlane(256, 64, 16, 4, max_tokens=8) as p:
        for e in range(8):
            g, u, d = synth.expert_weights(3, 0, e, 256, 64)
            p.load_expert(0, e, g, u, d)
        lg = np.full((1, 16), -10.0, np.float32)
        lg[0, 12] = 5.0  # routes to experts 12 and 0..2; 12 was never loaded
        x = torch.zeros(1, 256, dtype=torch.bfloat16, device="cuda")
        with pytest.raises(MoEError) as ei:
            p.forward(0, x, torch.from_numpy(lg).cuda(), sync=True)
        assert ei.value.status == MOE_ESTATE


def test_small_shape_golden(golden):
    """The ffn_small fixture (compiled-reference output) through the full moe_forward path."""
    from npu_offload_b200.moe import MoEDataPlane
    g = golden("ffn_small.npz")
    seed, h, f, e_, k = (int(g[n]) for n in ("seed", "H", "F", "E", "K"))
    ex = [synth.expert_weights(seed, 0, e, h, f) for e in range(e_)]
    assert sha(*[a for trip in ex for a in trip]) == str(g["wsha"])
    with MoEDataPlane(h, f, e_, k, max_tokens=16) as p:
        for e in range(e_):
            p.load_expert(0, e, *ex[e])
        out, gi, gw = p.forward(0, torch.from_numpy(g["x"].view(np.int16)).view(torch.bfloat16).cuda(),
                                torch.from_numpy(g["logits"]).cuda(), return_topk=True, sync=True)
        np.testing.assert_array_equal(gi.cpu().numpy(), g["idx"])
        assert_close(out.cpu().numpy(), g["out"], what="ffn_small golden")


def test_solar_golden_cpu_moe_surface(golden):
    """ffn_solar fixture: the cpu_moe surface (moe_experts) and the ck_moe3 surface."""
    from npu_offload_b200.moe import MoEDataPlane
    g = golden("ffn_solar.npz")
    seed = int(g["seed"])
    with MoEDataPlane(H, F, 16, 16, max_tokens=16) as p:
        for T in (1, 4):
            ex = g[f"T{T}_experts"].tolist()
            Wn = [synth.expert_weights(seed, 0, e, H, F) for e in ex]
            assert sha(*[a for trip in Wn for a in trip]) == str(g[f"T{T}_wsha"])
            off = g[f"T{T}_tok_off"]
            toks = [g[f"T{T}_toks"][off[j]:off[j + 1]] for j in range(len(ex))]
            ws = [g[f"T{T}_ws"][off[j]:off[j + 1]] for j in range(len(ex))]
            gus = [np.concatenate(w[:2], 0) for w in Wn]
            ds = [w[2] for w in Wn]
            out = p.experts(g[f"T{T}_x"], gus, ds, toks, ws)
            assert_close(out.cpu().numpy(), g[f"T{T}_out"], what=f"cpu_moe surface T={T}")
            if T == 1:
                bases = [torch.from_numpy(np.concatenate([a.ravel(), b.ravel(), c.ravel()]).view(np.int16)).cuda()
                         for a, b, c in Wn]
                acc = torch.full((H,), 0.5, device="cuda")
                p.ck_moe3(bases, g["ck_moe3_w"], g["T1_x"][0], acc)
                torch.cuda.synchronize()
                assert_close(acc.cpu().numpy(), g["ck_moe3_out"], what="ck_moe3 surface")


def test_gpu_moe_dropin_matches_reference_signature():
    from npu_offload_b200.moe import gpu_moe
    T, h, f = 6, 512, 256
    Wn = [synth.expert_weights(17, 0, e, h, f) for e in range(5)]
    x = synth.hidden(17, T, h)
    rng = np.random.default_rng(17)
    toks = [np.sort(rng.choice(T, size=int(rng.integers(1, T + 1)), replace=False)) for _ in Wn]
    ws = [rng.uniform(0.05, 0.5, size=len(t)).astype(np.float32) for t in toks]
    tt = lambda a: torch.from_numpy(a.view(np.int16)).view(torch.bfloat16)
    gus = [tt(np.concatenate(w[:2], 0)) for w in Wn]
    ds = [tt(w[2]) for w in Wn]
    out = gpu_moe(tt(x), gus, ds, [torch.from_numpy(t.astype(np.int64)) for t in toks],
                  [torch.from_numpy(w) for w in ws])
    assert out.device.type == "cpu" and out.dtype == torch.float32 and out.shape == (T, h)
    if Reference.available():
        ref = Reference.cpu_moe(x, [g.view(torch.int16).numpy().view(np.uint16) for g in gus],
                                [d.view(torch.int16).numpy().view(np.uint16) for d in ds], toks, ws)
    else:
        ref = Port.cpu_moe(x, [("bf16", g.view(torch.int16).numpy().view(np.uint16),
                                d.view(torch.int16).numpy().view(np.uint16)) for g, d in zip(gus, ds)], toks, ws)
    assert_close(out.numpy(), ref, what="gpu_moe drop-in")
    outd = gpu_moe(tt(x).cuda(), [g.cuda() for g in gus], [d.cuda() for d in ds], toks, ws)
    assert outd.is_cuda
    np.testing.assert_array_equal(outd.cpu().numpy(), out.numpy())


def test_int8_quantiser_bitexact_and_q8_layer(golden):
    """Device quant_row == reference tables; a mixed bf16/int8 layer matches ck_moe_q8w semantics."""
    from npu_offload_b200.moe import MoEDataPlane
    g = golden("q8.npz")
    with MoEDataPlane(128, 64, 4, 2, max_tokens=8) as p:
        for i in range(g["small_gate"].shape[0]):
            q, sc, rs = p.place_expert_q8(g["small_gate"][i], g["small_up"][i], g["small_down"][i])
            np.testing.assert_array_equal(q.cpu().numpy(), g["small_q"][i])
            np.testing.assert_array_equal(sc.cpu().numpy(), g["small_sc"][i])
            np.testing.assert_array_equal(rs.cpu().numpy(), g["small_rs"][i])
        qs = [torch.from_numpy(g["small_q"][i]).cuda() for i in range(3)]
        scs = [torch.from_numpy(g["small_sc"][i]).cuda() for i in range(3)]
        acc = torch.zeros(128, device="cuda")
        p.ck_moe_q8w(qs, scs, g["small_w"], g["small_x"], acc)
        torch.cuda.synchronize()
        assert_close(acc.cpu().numpy(), g["small_out"], what="ck_moe_q8w surface (small)")
    # Solar-size: quantise on the GPU, check against the reference tables' sha256 and outputs
    seed = int(g["solar_seed"])
    with MoEDataPlane(H, F, 2, 2, max_tokens=4) as p:
        Wn = [synth.expert_weights(seed, 0, e, H, F) for e in range(2)]
        for e in range(2):
            p.load_expert(0, e, *Wn[e])
            p.quantize_expert_q8(0, e)
            assert p.expert_kind(0, e) == 2
            q, sc, _ = p.place_expert_q8(*Wn[e])
            assert sha(q.cpu().numpy()) == str(g["solar_qsha"][e]) and sha(sc.cpu().numpy()) == str(g["solar_scsha"][e])
        lg = np.array([[1.0, 0.5]], np.float32)
        out, gi, gw = p.forward(0, torch.from_numpy(g["solar_x"][None].view(np.int16)).view(torch.bfloat16).cuda(),
                                torch.from_numpy(lg).cuda(), return_topk=True, sync=True)
        jobs = [("q8",) + tuple(a for a in Port.place_expert_q8(*Wn[e])[:2]) for e in gi.cpu().numpy()[0]]
        ref = Port.cpu_moe(g["solar_x"][None], jobs, [[0], [0]], [[v] for v in gw.cpu().numpy()[0]])
        assert_close(out.cpu().numpy(), ref, what="int8 forward vs ck_moe_q8w semantics")


def test_mixed_bf16_int8_layer(solar):
    """C5-style layer: least popular experts int8, the rest bf16 (on a separate context)."""
    from npu_offload_b200.moe import MoEDataPlane
    _, W = solar
    order = synth.popularity_order(5, E)
    cold = set(order[32:].tolist())
    with MoEDataPlane(H, F, E, K, max_tokens=8) as p:
        for e in range(E):
            p.load_expert(0, e, *W[e])
            if e in cold:
                p.quantize_expert_q8(0, e)
        T = 4
        x = synth.hidden(5, T, H)
        lg = synth.logits(5, T, E)
        idx0, _, _ = Port.route_softmax(lg, K)
        ex = {}
        for e in sorted(set(idx0.ravel().tolist())):
            gate, up, down = bf16_np(W[e][0]), bf16_np(W[e][1]), bf16_np(W[e][2])
            if e in cold:
                q, sc, _ = Port.place_expert_q8(gate, up, down)
                ex[e] = ("q8", q, sc)
            else:
                ex[e] = ("bf16", np.concatenate([gate, up], 0), down)
        ref, idx, _, _, kind = oracle_layer(x, lg, ex, K)
        out, gi, _ = p.forward(0, torch.from_numpy(x.view(np.int16)).view(torch.bfloat16).cuda(),
                               torch.from_numpy(lg).cuda(), return_topk=True, sync=True)
        np.testing.assert_array_equal(gi.cpu().numpy(), idx)
        assert any(e in cold for e in idx.ravel()), "case must route to an int8 expert"
        assert_close(out.cpu().numpy(), ref, what=f"mixed layer vs {kind}")


@pytest.mark.parametrize("seed", [2, 5])
def test_configs4_int8_cold_experts_t1_matches_reference(solar, seed):
    """configs[4] exactly: a Solar-shaped layer whose 96 least popular experts (by the Zipf rank of the
    routing bias) are stored int8 weight-only, quantised on the GPU with the reference's quant_row
    rule, and the top 32 stay bf16; decode batch 1, top-8 Zipf routing.  The routed int8 experts'
    tables must equal the reference's ck_place_expert_q8 tables (cpu_kern.c:227-241) bit for bit;
    the layer output is checked against the reference itself: ck_moe_q8w (cpu_kern.c:306-333) for
    the int8 jobs plus cpu_moe (cpu_moe.cpp:38-96) for the bf16 jobs (the C restatement where this
    host cannot run the reference).  The seeds route at least one token pair to an int8 expert."""
    from npu_offload_b200.moe import MoEDataPlane
    _, W = solar
    order = synth.popularity_order(seed, E)
    cold = set(order[32:].tolist())
    x = synth.hidden(seed, 1, H)
    lg = synth.logits(seed, 1, E)
    with MoEDataPlane(H, F, E, K, max_tokens=1) as p:
        for e in range(E):
            p.load_expert(0, e, *W[e])
            if e in cold:
                p.quantize_expert_q8(0, e)
        assert sum(p.expert_kind(0, e) == 2 for e in range(E)) == 96
        out, gi, gw = p.forward(0, torch.from_numpy(x.view(np.int16)).view(torch.bfloat16).cuda(),
                                torch.from_numpy(lg).cuda(), return_topk=True, sync=True)
        idx, w, st = Port.route_softmax(lg, K)
        assert st == 0
        np.testing.assert_array_equal(gi.cpu().numpy(), idx)
        ids, ws = idx[0].tolist(), w[0].tolist()
        assert any(e in cold for e in ids) and any(e not in cold for e in ids)
        use_ref = Reference.available()
        hot_gu, hot_d, hot_w, qs, scs, q_w = [], [], [], [], [], []
        for e, we in zip(ids, ws):
            gate, up, down = bf16_np(W[e][0]), bf16_np(W[e][1]), bf16_np(W[e][2])
            if e in cold:
                q, sc, _ = (Reference if use_ref else Port).place_expert_q8(gate, up, down)
                gq, gsc, _ = p.place_expert_q8(W[e][0], W[e][1], W[e][2])
                np.testing.assert_array_equal(gq.cpu().numpy(), q)
                np.testing.assert_array_equal(gsc.cpu().numpy(), sc)
                qs.append(q)
                scs.append(sc)
                q_w.append(we)
            else:
                hot_gu.append(np.concatenate([gate, up], 0))
                hot_d.append(down)
                hot_w.append(we)
        if use_ref:
            ref = Reference.cpu_moe(x, hot_gu, hot_d, [np.zeros(1, np.int64)] * len(hot_gu),
                                    [np.array([v], np.float32) for v in hot_w]).copy()
            Reference.ck_moe_q8w(qs, scs, np.array(q_w, np.float32), x[0], ref[0])
            kind = "reference cpu_moe + ck_moe_q8w"
        else:
            jobs = [("bf16", a, b) for a, b in zip(hot_gu, hot_d)] + [("q8", a, b) for a, b in zip(qs, scs)]
            ref = Port.cpu_moe(x, jobs, [[0]] * len(jobs), [[v] for v in hot_w + q_w])
            kind = "oracle restatement"
        d, c = assert_close(out.cpu().numpy(), ref, what=f"configs[4] seed {seed} vs {kind}")
        print(f"configs[4] seed {seed}: {len(qs)} int8 + {len(hot_w)} bf16 experts vs {kind}: "
              f"max-abs {d:.3g}, cosine {c:.8f}")
