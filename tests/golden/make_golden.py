"""Regenerate the golden fixtures in tests/golden/ from the reference itself.

Run in a container that holds the reference tree (read-only) and a CPU with AVX-512 BF16:

    python oracle/build.py && python tests/golden/make_golden.py

Sources of truth (paths relative to the ai-computing/npu-offload project root):

* ``cpu_moe`` outputs: the reference's ``solar_hybrid/cpu_moe.cpp`` compiled by ``oracle/build.py``.
* ``ck_moe3`` / ``ck_place_expert_q8`` / ``ck_moe_q8w`` outputs: the reference's
  ``track2_opt/solar_engine/csrc/cpu_kern.c`` compiled by ``oracle/build.py``.
* sigmoid-router outputs: the reference's Python ``solar_hybrid/model.py:77-93`` (``route``),
  imported from the reference tree (n_group = 1, norm_topk = True, scale = 1).
* softmax-router known answers: ``route_softmax_kat.json``, written by hand from the rules of
  ``npu-kernels/npu_kernels/rngd/layer_template/src/host.rs.tpl:247-268`` (the Rust template
  cannot be compiled here); each case states the rule it exercises.

Large weights are not stored: they are regenerated from their seeds with npu_offload_b200.synth and
checked against the stored sha256.
"""
import hashlib
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

from npu_offload_b200 import synth  # noqa: E402
from oracle.oracle import Port, Reference  # noqa: E402

OUT = os.path.dirname(os.path.abspath(__file__))
# The reference tree: $NPU_OFFLOAD_REF, else a directory named "reference" beside this repository.
REF_ROOT = os.environ.get("NPU_OFFLOAD_REF") or os.path.join(os.path.dirname(ROOT), "reference")


def sha(*arrs):
    h = hashlib.sha256()
    for a in arrs:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


def jobs_from_route(idx, w, E):
    pm = Port.permute(idx, E)
    K = idx.shape[1]
    toks, ws = [], []
    for e in pm["job_order"]:
        ps = pm["perm"][pm["offsets"][e]:pm["offsets"][e + 1]]
        toks.append((ps // K).astype(np.int64))
        ws.append(w.reshape(-1)[ps].astype(np.float32))
    return pm["job_order"], toks, ws


def ffn_small():
    """Small shapes (weights regenerated from the seed and checked by sha256): cpu_moe over a routed batch, softmax router."""
    seed, T, H, F, E, K = 7, 6, 256, 128, 16, 4
    experts = [synth.expert_weights(seed, 0, e, H, F) for e in range(E)]
    x = synth.hidden(seed, T, H)
    lg = synth.logits(seed, T, E)
    idx, w, st = Port.route_softmax(lg, K)
    assert st == 0
    order, toks, ws = jobs_from_route(idx, w, E)
    gus = [np.concatenate([experts[e][0], experts[e][1]], 0) for e in order]
    ds = [experts[e][2] for e in order]
    out = Reference.cpu_moe(x, gus, ds, toks, ws)
    np.savez_compressed(os.path.join(OUT, "ffn_small.npz"), seed=seed, H=H, F=F, E=E, K=K, x=x, logits=lg,
                        wsha=np.array(sha(*[a for trip in experts for a in trip])), idx=idx, w=w,
                        job_order=order, out=out)


def ffn_solar():
    """Solar shapes (H=4096, F=1280): cpu_moe for T=1 and T=4 over 8/11 experts; weights regenerated."""
    seed, H, F = 11, 4096, 1280
    rec = {}
    for T, experts_used in ((1, list(range(8))), (4, list(range(11)))):
        x = synth.hidden(seed + T, T, H)
        rng = np.random.default_rng(seed + 100 + T)
        toks, ws = [], []
        for j, e in enumerate(experts_used):
            n = 1 if T == 1 else int(rng.integers(1, T + 1))
            t = np.sort(rng.choice(T, size=n, replace=False)).astype(np.int64)
            toks.append(t)
            ws.append(rng.uniform(0.05, 0.3, size=n).astype(np.float32))
        W = [synth.expert_weights(seed, 0, e, H, F) for e in experts_used]
        gus = [np.concatenate([g, u], 0) for g, u, _ in W]
        ds = [d for _, _, d in W]
        out = Reference.cpu_moe(x, gus, ds, toks, ws)
        rec[f"T{T}_x"] = x
        rec[f"T{T}_experts"] = np.array(experts_used, np.int32)
        rec[f"T{T}_tok_off"] = np.cumsum([0] + [len(t) for t in toks]).astype(np.int64)
        rec[f"T{T}_toks"] = np.concatenate(toks)
        rec[f"T{T}_ws"] = np.concatenate(ws)
        rec[f"T{T}_out"] = out
        rec[f"T{T}_wsha"] = np.array(sha(*[a for trip in W for a in trip]))
        if T == 1:
            # ck_moe3 on the same single token (NUMA-placed layout [g][u][d]), accumulating into out0
            bases = [Reference.place_expert(g, u, d) for g, u, d in W]
            acc = np.full(H, 0.5, np.float32)
            Reference.ck_moe3(bases, ws_flat := np.concatenate(ws), x[0], acc)
            rec["ck_moe3_w"] = ws_flat
            rec["ck_moe3_out"] = acc
    rec["seed"] = seed
    np.savez_compressed(os.path.join(OUT, "ffn_solar.npz"), **rec)


def q8():
    """int8 weight-only: ck_place_expert_q8 tables (small: stored; Solar: sha256) + ck_moe_q8w outputs."""
    rec = {}
    seed, H, F = 5, 128, 64
    W = [synth.expert_weights(seed, 0, e, H, F) for e in range(3)]
    # plant exact ties and a zero row so the rounding / zero-scale rules are exercised
    g0 = W[0][0].copy()
    g0[0, :] = 0
    g0[1, :8] = synth.f2bf(np.array([0.5, -0.5, 1.0, -1.0, 0.25, 127.0, -127.0, 63.5], np.float32))
    g0[1, 8:] = 0
    W[0] = (g0, W[0][1], W[0][2])
    qs, scs, rss = zip(*[Reference.place_expert_q8(*w) for w in W])
    x = synth.hidden(seed, 1, H)[0]
    wts = np.array([0.5, 0.3, 0.2], np.float32)
    out = np.zeros(H, np.float32)
    Reference.ck_moe_q8w(list(qs), list(scs), wts, x, out)
    rec.update(small_gate=np.stack([w[0] for w in W]), small_up=np.stack([w[1] for w in W]),
               small_down=np.stack([w[2] for w in W]), small_q=np.stack(qs), small_sc=np.stack(scs),
               small_rs=np.stack(rss), small_x=x, small_w=wts, small_out=out)
    seed, H, F = 13, 4096, 1280
    W = [synth.expert_weights(seed, 0, e, H, F) for e in range(2)]
    qs, scs, rss = zip(*[Reference.place_expert_q8(*w) for w in W])
    x = synth.hidden(seed, 1, H)[0]
    wts = np.array([0.6, 0.4], np.float32)
    out = np.zeros(H, np.float32)
    Reference.ck_moe_q8w(list(qs), list(scs), wts, x, out)
    rec.update(solar_seed=seed, solar_qsha=np.array([sha(q) for q in qs]), solar_scsha=np.array([sha(s) for s in scs]),
               solar_x=x, solar_w=wts, solar_out=out)
    np.savez_compressed(os.path.join(OUT, "q8.npz"), **rec)


def route_sigmoid():
    """The reference's own torch router (sigmoid + correction bias, n_group = 1)."""
    import torch
    sys.path.insert(0, os.path.join(REF_ROOT, "solar_hybrid"))
    import model as ref_model  # the reference's solar_hybrid/model.py

    class Cfg:
        n_group, topk_group, topk, E, norm_topk, scale = 1, 1, 8, 128, True, 1.0

    seed, T, E, H = 3, 64, 128, 64
    rng = np.random.default_rng(seed)
    h = synth.hidden(seed, T, H)
    router_w = (rng.standard_normal((E, H)) * 0.2).astype(np.float32)
    bias = (rng.standard_normal(E) * 0.05).astype(np.float32)
    ht = torch.from_numpy(h.view(np.int16)).view(torch.bfloat16)
    idx, w = ref_model.route(Cfg, ht, torch.from_numpy(router_w), torch.from_numpy(bias))
    logits = torch.nn.functional.linear(ht.float(), torch.from_numpy(router_w)).numpy()
    np.savez_compressed(os.path.join(OUT, "route_sigmoid.npz"), logits=logits, bias=bias, idx=idx.numpy().astype(np.int32),
                        w=w.numpy().astype(np.float32), K=8)


def main():
    if not Reference.available():
        raise SystemExit("compiled reference unavailable: " + Reference.why_unavailable())
    ffn_small()
    ffn_solar()
    q8()
    route_sigmoid()
    print("fixtures written to", OUT)


if __name__ == "__main__":
    main()
