"""ctypes/numpy bindings of the CPU checkers.

TEST INFRASTRUCTURE ONLY: tests/, ``__graft_entry__.smoke()`` and bench.py's CPU-baseline and
reference legs use this module as the checker; the product path never imports it.

Two checkers live here:

* ``Port`` -- the plain-C restatement ``oracle/moe_oracle.c`` (always available; built by
  ``oracle/build.py``).
* ``Reference`` -- the reference's own CPU kernels compiled from the reference tree into
  ``oracle/_ref``: ``cpu_moe`` (``solar_hybrid/cpu_moe.cpp:38-96``) and the ``ck_*`` C ABI of
  ``track2_opt/solar_engine/csrc/cpu_kern.c``.  They need AVX-512 BF16/VNNI on the host CPU;
  ``Reference.available()`` says whether they can run here.

bf16 tensors are carried as ``numpy.uint16`` arrays of raw bits.
"""
import ctypes
import importlib.machinery
import importlib.util
import os

import numpy as np

from . import build as _build

_c_i32p = ctypes.POINTER(ctypes.c_int32)
_c_i64p = ctypes.POINTER(ctypes.c_int64)
_c_f32p = ctypes.POINTER(ctypes.c_float)
_c_u16p = ctypes.POINTER(ctypes.c_uint16)
_c_i8p = ctypes.POINTER(ctypes.c_int8)

OR_OK, OR_EINVAL, OR_ENONFINITE = 0, 1, 2


def _p(a, t):
    return a.ctypes.data_as(t)


def _ptr_array(arrs):
    return (ctypes.c_void_p * max(1, len(arrs)))(*[a.ctypes.data if a is not None else None for a in arrs])


def f2bf(a):
    """fp32 -> bf16 bits, round-to-nearest-even without NaN special-casing (cpu_moe.cpp:30-34)."""
    u = np.ascontiguousarray(a, dtype=np.float32).view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFFFFFF
    return (u >> 16).astype(np.uint16)


def bf2f(b):
    return (np.ascontiguousarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


class Port:
    """The C restatement (oracle/moe_oracle.c)."""

    _lib = None

    @classmethod
    def lib(cls):
        if cls._lib is None:
            so = _build.ORACLE_SO
            if not os.path.exists(so):
                _build.build_oracle()
            lib = ctypes.CDLL(so)
            lib.or_route_softmax.argtypes = [ctypes.c_int] * 3 + [_c_f32p, _c_i32p, _c_f32p]
            lib.or_route_sigmoid.argtypes = [ctypes.c_int] * 3 + [_c_f32p, _c_f32p, _c_i32p, _c_f32p]
            lib.or_permute.argtypes = [ctypes.c_int] * 3 + [_c_i32p] * 6
            lib.or_cpu_moe.argtypes = [ctypes.c_int] * 4 + [_c_u16p, ctypes.c_void_p, ctypes.c_void_p,
                                                             ctypes.c_void_p, ctypes.c_void_p, _c_i64p, _c_i64p,
                                                             _c_f32p, _c_f32p, ctypes.c_int]
            lib.or_place_expert_q8.argtypes = [_c_u16p] * 3 + [_c_i8p, _c_f32p, _c_i32p, ctypes.c_int, ctypes.c_int]
            lib.or_place_expert_q8.restype = None
            lib.or_moe_layer.argtypes = [ctypes.c_int] * 6 + [_c_u16p, _c_f32p, _c_f32p] + [ctypes.c_void_p] * 4 + \
                [_c_f32p, _c_i32p, _c_f32p]
            lib.or_router_logits.argtypes = [ctypes.c_int] * 3 + [_c_u16p, _c_u16p, _c_f32p]
            lib.or_router_logits.restype = None
            lib.or_shared_expert.argtypes = [ctypes.c_int] * 3 + [_c_u16p] * 4 + [ctypes.c_int, ctypes.c_void_p,
                                                                                  ctypes.c_void_p]
            lib.or_shared_expert.restype = None
            lib.or_combine_residual.argtypes = [ctypes.c_long, _c_u16p, ctypes.c_void_p, _c_f32p, _c_u16p]
            lib.or_combine_residual.restype = None
            lib.or_router_exp_range.argtypes = [ctypes.c_uint32, ctypes.c_int64, _c_f32p]
            lib.or_router_exp_range.restype = None
            lib.or_router_exp_vs_long_double.argtypes = [ctypes.c_uint32, ctypes.c_int64, ctypes.c_int32]
            lib.or_router_exp_vs_long_double.restype = ctypes.c_int64
            lib.or_libm_expf_mismatches.argtypes = [ctypes.c_uint32, ctypes.c_int64, _c_i32p]
            lib.or_libm_expf_mismatches.restype = ctypes.c_int64
            lib.or_set_threads.argtypes = [ctypes.c_int]
            lib.or_set_threads.restype = None
            lib.or_max_threads.restype = ctypes.c_int
            cls._lib = lib
        return cls._lib

    @classmethod
    def set_threads(cls, n):
        cls.lib().or_set_threads(int(n))

    @classmethod
    def router_exp_range(cls, first_bits, n):
        """The routers' exp (double exp rounded once) of the n floats whose bit patterns follow first_bits."""
        out = np.empty(int(n), np.float32)
        cls.lib().or_router_exp_range(int(first_bits), int(n), _p(out, _c_f32p))
        return out

    @classmethod
    def router_exp_vs_long_double(cls, first_bits, n, stride):
        return int(cls.lib().or_router_exp_vs_long_double(int(first_bits), int(n), int(stride)))

    @classmethod
    def libm_expf_mismatches(cls, first_bits, n):
        """(count, max ulp) of floats in the range where the host libm's expf differs from the routers' exp."""
        worst = np.zeros(1, np.int32)
        bad = cls.lib().or_libm_expf_mismatches(int(first_bits), int(n), _p(worst, _c_i32p))
        return int(bad), int(worst[0])

    @classmethod
    def route_softmax(cls, logits, K):
        logits = np.ascontiguousarray(logits, dtype=np.float32)
        T, E = logits.shape
        idx = np.zeros((T, K), np.int32)
        w = np.zeros((T, K), np.float32)
        st = cls.lib().or_route_softmax(T, E, K, _p(logits, _c_f32p), _p(idx, _c_i32p), _p(w, _c_f32p))
        return idx, w, st

    @classmethod
    def route_sigmoid(cls, logits, bias, K):
        logits = np.ascontiguousarray(logits, dtype=np.float32)
        T, E = logits.shape
        idx = np.zeros((T, K), np.int32)
        w = np.zeros((T, K), np.float32)
        b = None if bias is None else np.ascontiguousarray(bias, dtype=np.float32)
        st = cls.lib().or_route_sigmoid(T, E, K, _p(logits, _c_f32p), None if b is None else _p(b, _c_f32p),
                                        _p(idx, _c_i32p), _p(w, _c_f32p))
        return idx, w, st

    @classmethod
    def permute(cls, idx, E):
        idx = np.ascontiguousarray(idx, dtype=np.int32)
        T, K = idx.shape
        counts = np.zeros(E, np.int32)
        offsets = np.zeros(E + 1, np.int32)
        perm = np.zeros(max(1, T * K), np.int32)
        job_order = np.zeros(E, np.int32)
        nj = np.zeros(1, np.int32)
        st = cls.lib().or_permute(T, K, E, _p(idx, _c_i32p), _p(counts, _c_i32p), _p(offsets, _c_i32p),
                                  _p(perm, _c_i32p), _p(job_order, _c_i32p), _p(nj, _c_i32p))
        return dict(counts=counts, offsets=offsets, perm=perm[:T * K], job_order=job_order[:nj[0]], status=st)

    @classmethod
    def cpu_moe(cls, x, jobs, toks, ws, out=None, accumulate=False):
        """cpu_moe surface.  jobs[j] = ("bf16", gu[2F,H], d[H,F]) or ("q8", q, sc)."""
        x = np.ascontiguousarray(x, dtype=np.uint16)
        T, H = x.shape
        F = None
        gus, ds, qs, scs = [], [], [], []
        for j in jobs:
            if j[0] == "bf16":
                gu, d = np.ascontiguousarray(j[1], np.uint16), np.ascontiguousarray(j[2], np.uint16)
                F = d.shape[1]
                gus.append(gu); ds.append(d); qs.append(None); scs.append(None)
            else:
                q, sc = np.ascontiguousarray(j[1], np.int8), np.ascontiguousarray(j[2], np.float32)
                F = (sc.shape[0] - H) // 2
                gus.append(None); ds.append(None); qs.append(q); scs.append(sc)
        if out is None:
            out = np.zeros((T, H), np.float32)
        if F is None:
            F = 1
        off = np.zeros(len(jobs) + 1, np.int64)
        for j, t in enumerate(toks):
            off[j + 1] = off[j] + len(t)
        tk = np.ascontiguousarray(np.concatenate([np.asarray(t, np.int64) for t in toks]) if toks else np.zeros(1, np.int64))
        w = np.ascontiguousarray(np.concatenate([np.asarray(v, np.float32) for v in ws]) if ws else np.zeros(1, np.float32))
        has_q = any(q is not None for q in qs)
        st = cls.lib().or_cpu_moe(T, H, F, len(jobs), _p(x, _c_u16p), _ptr_array(gus), _ptr_array(ds),
                                  _ptr_array(qs) if has_q else None, _ptr_array(scs), _p(off, _c_i64p),
                                  _p(tk, _c_i64p), _p(w, _c_f32p), _p(out, _c_f32p), int(accumulate))
        if st != OR_OK:
            raise ValueError(f"or_cpu_moe status {st}")
        return out

    @classmethod
    def place_expert_q8(cls, g, u, d):
        g, u, d = (np.ascontiguousarray(a, np.uint16) for a in (g, u, d))
        F, H = g.shape
        q = np.zeros(2 * F * H + H * F, np.int8)
        sc = np.zeros(2 * F + H, np.float32)
        rs = np.zeros(2 * F + H, np.int32)
        cls.lib().or_place_expert_q8(_p(g, _c_u16p), _p(u, _c_u16p), _p(d, _c_u16p), _p(q, _c_i8p),
                                     _p(sc, _c_f32p), _p(rs, _c_i32p), H, F)
        return q, sc, rs

    @classmethod
    def moe_layer(cls, x, logits, experts, K, scoring=0, bias=None):
        """Full layer: route -> group -> experts.  experts[e] = ("bf16", gu, d) | ("q8", q, sc)."""
        x = np.ascontiguousarray(x, np.uint16)
        logits = np.ascontiguousarray(logits, np.float32)
        T, H = x.shape
        E = logits.shape[1]
        gus = [None] * E; ds = [None] * E; qs = [None] * E; scs = [None] * E
        F = 1
        for e, ex in experts.items():
            if ex[0] == "bf16":
                gus[e] = np.ascontiguousarray(ex[1], np.uint16); ds[e] = np.ascontiguousarray(ex[2], np.uint16)
                F = ds[e].shape[1]
            else:
                qs[e] = np.ascontiguousarray(ex[1], np.int8); scs[e] = np.ascontiguousarray(ex[2], np.float32)
                F = (scs[e].shape[0] - H) // 2
        out = np.zeros((T, H), np.float32)
        idx = np.zeros((max(T, 1), K), np.int32)
        w = np.zeros((max(T, 1), K), np.float32)
        b = None if bias is None else np.ascontiguousarray(bias, np.float32)
        st = cls.lib().or_moe_layer(T, H, F, E, K, scoring, _p(x, _c_u16p), _p(logits, _c_f32p),
                                    None if b is None else _p(b, _c_f32p), _ptr_array(gus), _ptr_array(ds),
                                    _ptr_array(qs) if any(q is not None for q in qs) else None, _ptr_array(scs),
                                    _p(out, _c_f32p), _p(idx, _c_i32p), _p(w, _c_f32p))
        return out, idx[:T], w[:T], st


    @classmethod
    def router_logits(cls, h2, wr):
        """logits [T, E] = h2 . wr^T in fp32 (solar_engine/src/dense/shared.rs:3)."""
        h2, wr = np.ascontiguousarray(h2, np.uint16), np.ascontiguousarray(wr, np.uint16)
        T, H = h2.shape
        E = wr.shape[0]
        out = np.zeros((T, E), np.float32)
        cls.lib().or_router_logits(T, E, H, _p(h2, _c_u16p), _p(wr, _c_u16p), _p(out, _c_f32p))
        return out

    @classmethod
    def shared_expert(cls, h2, x2, g, u, d, device_rounding=False):
        """(y bf16 [T,H], shared fp32 [T,H]): y = bf16(x2 + down . SwiGLU(gate . h2, up . h2)) (shared.rs:1-3).
        device_rounding follows the reference's host checker expert_ref (host_util.rs:35-46)."""
        h2, x2 = np.ascontiguousarray(h2, np.uint16), np.ascontiguousarray(x2, np.uint16)
        gu = np.ascontiguousarray(np.concatenate([g, u], 0), np.uint16)
        d = np.ascontiguousarray(d, np.uint16)
        T, H = h2.shape
        F = d.shape[1]
        y = np.zeros((T, H), np.uint16)
        s = np.zeros((T, H), np.float32)
        cls.lib().or_shared_expert(T, H, F, _p(h2, _c_u16p), _p(x2, _c_u16p), _p(gu, _c_u16p), _p(d, _c_u16p),
                                   int(bool(device_rounding)), s.ctypes.data, y.ctypes.data)
        return y, s

    @classmethod
    def combine_residual(cls, y, extra, moe):
        """x_next = bf16((y + extra) + moe) (combine.rs:1, layer.rs:4); extra may be None."""
        y = np.ascontiguousarray(y, np.uint16)
        moe = np.ascontiguousarray(moe, np.float32)
        ex = None if extra is None else np.ascontiguousarray(extra, np.float32)
        out = np.zeros(y.shape, np.uint16)
        cls.lib().or_combine_residual(y.size, _p(y, _c_u16p), None if ex is None else ex.ctypes.data,
                                      _p(moe, _c_f32p), _p(out, _c_u16p))
        return out


def cpu_flags():
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("flags"):
                    return set(line.split(":", 1)[1].split())
    except OSError:
        pass
    return set()


def cpu_model():
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


class Reference:
    """The reference's compiled CPU kernels (oracle/_ref)."""

    _kern = None
    _moe = None
    NEEDED = {"avx512f", "avx512bw", "avx512vl", "avx512_bf16", "avx512_vnni"}

    @classmethod
    def available(cls):
        return (os.path.exists(_build.CPU_KERN_SO) and os.path.exists(_build.CPU_MOE_SO)
                and cls.NEEDED <= cpu_flags())

    @classmethod
    def why_unavailable(cls):
        if not os.path.exists(_build.CPU_KERN_SO) or not os.path.exists(_build.CPU_MOE_SO):
            return "oracle/_ref not built"
        missing = cls.NEEDED - cpu_flags()
        return f"host CPU lacks {sorted(missing)}" if missing else ""

    @classmethod
    def kern(cls):
        if cls._kern is None:
            lib = ctypes.CDLL(_build.CPU_KERN_SO)
            lib.ck_set_threads.argtypes = [ctypes.c_int]
            lib.ck_set_threads.restype = None
            lib.ck_moe3.argtypes = [ctypes.c_int, ctypes.c_void_p, _c_f32p, _c_u16p, _c_f32p, ctypes.c_int, ctypes.c_int]
            lib.ck_moe3.restype = None
            lib.ck_place_expert.argtypes = [_c_u16p] * 4 + [ctypes.c_int, ctypes.c_int]
            lib.ck_place_expert.restype = None
            lib.ck_place_expert_q8.argtypes = [_c_u16p] * 3 + [_c_i8p, _c_f32p, _c_i32p, ctypes.c_int, ctypes.c_int]
            lib.ck_place_expert_q8.restype = None
            lib.ck_moe_q8w.argtypes = [ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p, _c_f32p, _c_u16p, _c_f32p,
                                       ctypes.c_int, ctypes.c_int]
            lib.ck_moe_q8w.restype = None
            cls._kern = lib
        return cls._kern

    @classmethod
    def moe_ext(cls):
        """The cpu_moe torch extension (pybind module built from solar_hybrid/cpu_moe.cpp)."""
        if cls._moe is None:
            import torch  # noqa: F401  (the extension links against libtorch)
            loader = importlib.machinery.ExtensionFileLoader("cpu_moe_ext", _build.CPU_MOE_SO)
            spec = importlib.util.spec_from_file_location("cpu_moe_ext", _build.CPU_MOE_SO, loader=loader)
            mod = importlib.util.module_from_spec(spec)
            loader.exec_module(mod)
            cls._moe = mod
        return cls._moe

    @classmethod
    def set_threads(cls, n):
        cls.kern().ck_set_threads(int(n))
        cls.moe_ext().set_threads(int(n))

    @classmethod
    def cpu_moe(cls, x, gus, ds, toks, ws):
        """ext.cpu_moe(x [T,H] bf16, gus [[2F,H]], ds [[H,F]], toks [int64], ws [f32]) -> [T,H] f32 (numpy)."""
        import torch
        bf = lambda a: torch.from_numpy(np.ascontiguousarray(a, np.uint16).view(np.int16)).view(torch.bfloat16)
        out = cls.moe_ext().cpu_moe(bf(x), [bf(g) for g in gus], [bf(d) for d in ds],
                                    [torch.as_tensor(np.asarray(t, np.int64)) for t in toks],
                                    [torch.as_tensor(np.asarray(w, np.float32)) for w in ws])
        return out.numpy()

    @classmethod
    def place_expert(cls, g, u, d):
        g, u, d = (np.ascontiguousarray(a, np.uint16) for a in (g, u, d))
        F, H = g.shape
        dst = np.zeros(3 * F * H, np.uint16)
        cls.kern().ck_place_expert(_p(g, _c_u16p), _p(u, _c_u16p), _p(d, _c_u16p), _p(dst, _c_u16p), H, F)
        return dst

    @classmethod
    def ck_moe3(cls, bases, w, x, out):
        """out[H] += sum_e w[e] * expert_e(x) for ck_place_expert layouts (cpu_kern.c:141-172)."""
        x = np.ascontiguousarray(x, np.uint16)
        w = np.ascontiguousarray(w, np.float32)
        H = x.shape[0]
        F = bases[0].shape[0] // (3 * H)
        cls.kern().ck_moe3(len(bases), _ptr_array(bases), _p(w, _c_f32p), _p(x, _c_u16p), _p(out, _c_f32p), H, F)
        return out

    @classmethod
    def place_expert_q8(cls, g, u, d):
        g, u, d = (np.ascontiguousarray(a, np.uint16) for a in (g, u, d))
        F, H = g.shape
        q = np.zeros(2 * F * H + H * F, np.int8)
        sc = np.zeros(2 * F + H, np.float32)
        rs = np.zeros(2 * F + H, np.int32)
        cls.kern().ck_place_expert_q8(_p(g, _c_u16p), _p(u, _c_u16p), _p(d, _c_u16p), _p(q, _c_i8p),
                                      _p(sc, _c_f32p), _p(rs, _c_i32p), H, F)
        return q, sc, rs

    @classmethod
    def ck_moe_q8w(cls, qs, scs, w, x, out):
        x = np.ascontiguousarray(x, np.uint16)
        w = np.ascontiguousarray(w, np.float32)
        H = x.shape[0]
        F = (scs[0].shape[0] - H) // 2
        cls.kern().ck_moe_q8w(len(qs), _ptr_array(qs), _ptr_array(scs), _p(w, _c_f32p), _p(x, _c_u16p),
                              _p(out, _c_f32p), H, F)
        return out
