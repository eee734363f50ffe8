"""Helpers for the GPU parity tests (inputs, weight generation, oracle selection)."""
import numpy as np
import torch

from npu_offload_b200 import synth
from oracle.oracle import Port, Reference


def bf16_np(t):
    """torch bf16 tensor (any device) -> numpy uint16 bits."""
    return t.detach().contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


def gpu_experts(seed, E, H, F, device="cuda:0", layer=0, scale=0.02):
    """Seeded N(0, scale) bf16 experts generated on the GPU: list of (gate, up, down) device tensors."""
    g = torch.Generator(device=device)
    out = []
    for e in range(E):
        g.manual_seed(seed * 100003 + layer * 1009 + e)
        gu = (torch.randn(2 * F, H, generator=g, device=device) * scale).to(torch.bfloat16)
        d = (torch.randn(H, F, generator=g, device=device) * scale).to(torch.bfloat16)
        out.append((gu[:F].contiguous(), gu[F:].contiguous(), d))
    return out


def oracle_layer(x, logits, experts_np, K, scoring=0, bias=None, prefer_reference=True):
    """Reference result for one layer.  experts_np[e] = ("bf16", gu, d) | ("q8", q, sc) for routed e.

    Routing and grouping always come from the restated router (the reference's router is Rust);
    the expert math comes from the compiled reference cpu_moe when this host can run it and every
    routed expert is bf16, else from the C restatement."""
    if scoring == 0:
        idx, w, st = Port.route_softmax(logits, K)
    else:
        idx, w, st = Port.route_sigmoid(logits, bias, K)
    E = logits.shape[1]
    pm = Port.permute(idx, E)
    toks, ws, jobs = [], [], []
    for e in pm["job_order"]:
        ps = pm["perm"][pm["offsets"][e]:pm["offsets"][e + 1]]
        toks.append((ps // K).astype(np.int64))
        ws.append(w.reshape(-1)[ps].astype(np.float32))
        jobs.append(experts_np[int(e)])
    if prefer_reference and Reference.available() and all(j[0] == "bf16" for j in jobs) and jobs:
        out = Reference.cpu_moe(x, [j[1] for j in jobs], [j[2] for j in jobs], toks, ws)
        kind = "reference"
    else:
        out = Port.cpu_moe(x, jobs, toks, ws)
        kind = "port"
    return out, idx, w, pm, kind


def routed_experts(logits, K):
    idx, _, _ = Port.route_softmax(logits, K)
    return sorted(set(idx.ravel().tolist()))


def zipf_logits(seed, T, E):
    return synth.logits(seed, T, E, zipf=True)
