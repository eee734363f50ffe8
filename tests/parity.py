"""Parity criteria shared by the tests (bf16 outputs within max-abs 2e-2 and
cosine >= 0.9999 of the reference with fp32 accumulation; indices and permutations bit-exact)."""
import hashlib

import numpy as np

MAX_ABS = 2e-2
MIN_COS = 0.9999


def cosine(a, b):
    a = np.asarray(a, np.float64).ravel()
    b = np.asarray(b, np.float64).ravel()
    na, nb = np.linalg.norm(a), np.linalg.norm(b)
    if na == 0 and nb == 0:
        return 1.0
    return float(a @ b / (na * nb))


def assert_close(got, ref, max_abs=MAX_ABS, min_cos=MIN_COS, what=""):
    got = np.asarray(got, np.float32)
    ref = np.asarray(ref, np.float32)
    assert got.shape == ref.shape, (what, got.shape, ref.shape)
    assert np.all(np.isfinite(got)), f"{what}: non-finite output"
    d = float(np.max(np.abs(got - ref))) if got.size else 0.0
    c = cosine(got, ref)
    assert d <= max_abs, f"{what}: max-abs {d:.3g} > {max_abs}"
    assert c >= min_cos, f"{what}: cosine {c:.7f} < {min_cos}"
    return d, c


def sha(*arrs):
    h = hashlib.sha256()
    for a in arrs:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()
