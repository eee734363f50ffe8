"""Seeded synthetic inputs for the routed-expert MoE layer (no checkpoint or routing profile exists here).

The shapes and distributions are the benchmark's: bf16 expert weights N(0, 0.02), bf16 hidden
states N(0, 1), fp32 router logits N(0, 1) plus a log-Zipf(s=1) expert-popularity bias
b_e = -s * ln(rank(e)), where rank is a seeded permutation of the experts.  Host generation uses
numpy's PCG64 (deterministic for a given seed), so the same bytes can be regenerated on any machine.

Per-expert seed: ``seed + 1000 * layer + expert``; hidden states ``seed + 1``; logits ``seed + 2``;
popularity permutation ``seed + 3``.
"""
import numpy as np


def f2bf(a):
    """fp32 -> bf16 bits (uint16), round to nearest even."""
    u = np.ascontiguousarray(a, dtype=np.float32).view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFFFFFF
    return (u >> 16).astype(np.uint16)


def bf2f(b):
    return (np.ascontiguousarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def _rng(seed):
    return np.random.Generator(np.random.PCG64(int(seed)))


def expert_weights(seed, layer, expert, H, F, scale=0.02):
    """(gate [F,H], up [F,H], down [H,F]) bf16 bits for one expert."""
    r = _rng(seed + 1000 * layer + expert)
    s = np.float32(scale)
    gu = f2bf(r.standard_normal((2 * F, H), dtype=np.float32) * s)
    d = f2bf(r.standard_normal((H, F), dtype=np.float32) * s)
    return gu[:F], gu[F:], d


def hidden(seed, T, H):
    return f2bf(_rng(seed + 1).standard_normal((T, H), dtype=np.float32))


def zipf_bias(seed, E, s=1.0):
    rank = _rng(seed + 3).permutation(E).astype(np.float64) + 1.0
    return (-s * np.log(rank)).astype(np.float32)


def popularity_order(seed, E):
    """Experts from most to least popular under zipf_bias (rank 1 first)."""
    return np.argsort(_rng(seed + 3).permutation(E), kind="stable")


def logits(seed, T, E, zipf=True):
    lg = _rng(seed + 2).standard_normal((T, E), dtype=np.float32)
    if zipf:
        lg = lg + zipf_bias(seed, E)[None, :]
    return np.ascontiguousarray(lg, dtype=np.float32)
