"""Host-side API of the B200 routed-expert MoE data plane (a thin layer over the C ABI).

* ``MoEDataPlane`` -- one context per GPU: expert tables resident in HBM, and the per-layer hot path
  ``forward(layer, hidden, logits) -> out`` (the surface of the reference engine's
  ``Model::moe_phase``, track2_opt/solar_engine/src/main.rs:149-209, and of ``Runtime._moe``,
  solar_hybrid/runtime.py:338-423).
* ``gpu_moe`` / ``set_threads`` -- drop-in replacements for ``cpu_moe_ext.cpu_moe`` /
  ``cpu_moe_ext.set_threads`` (solar_hybrid/cpu_moe.cpp:38-105): same arguments, same result
  layout, same error on H or F not a multiple of 32.

PyTorch only provides device memory and streams here; every computation runs in libmoe_dp.so.
"""
import ctypes

import numpy as np
import torch

from . import _lib
from ._lib import (MOE_F_ACCUMULATE, MOE_F_HOST, MOE_F_SYNC, MOE_SCORING_SIGMOID, MOE_SCORING_SOFTMAX, MoeConfig,
                   check, lib)

__all__ = ["MoEDataPlane", "gpu_moe", "set_threads", "as_bf16"]


def _vp(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def as_bf16(a, device=None):
    """numpy uint16 (bf16 bits) or torch bf16 -> contiguous torch bf16 tensor (optionally moved)."""
    if isinstance(a, np.ndarray):
        assert a.dtype == np.uint16, a.dtype
        t = torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).view(torch.bfloat16)
    else:
        t = a
        if t.dtype == torch.int16 or t.dtype == torch.uint16:
            t = t.view(torch.bfloat16)
        assert t.dtype == torch.bfloat16, t.dtype
    if device is not None:
        t = t.to(device, non_blocking=False)
    return t.contiguous()


def _as(a, dtype, device=None):
    t = torch.as_tensor(a) if not isinstance(a, torch.Tensor) else a
    t = t.to(dtype)
    if device is not None:
        t = t.to(device)
    return t.contiguous()


def _stream_ptr(stream, device):
    if stream is None:
        stream = torch.cuda.current_stream(device)
    return ctypes.c_void_p(stream.cuda_stream)


class MoEDataPlane:
    """Expert tables + routed-expert forward for ``n_layers`` MoE layers on one GPU.

    Expert-parallel use: pass ``ep_rank`` / ``ep_world`` (and optionally a ``shard_map`` of shape
    [n_layers, n_experts] giving each expert's owner rank); ``forward`` then returns this rank's
    partial sum over its local experts, which npu_offload_b200.parallel combines across ranks.
    """

    def __init__(self, hidden, inter, n_experts, top_k=8, n_layers=1, max_tokens=64, scoring="softmax", device=0,
                 ep_rank=0, ep_world=1, shard_map=None):
        self.H, self.F, self.E, self.K, self.L = int(hidden), int(inter), int(n_experts), int(top_k), int(n_layers)
        self.max_tokens = int(max_tokens)
        self.device = torch.device("cuda", device) if isinstance(device, int) else torch.device(device)
        self.scoring = scoring
        sc = {"softmax": MOE_SCORING_SOFTMAX, "sigmoid": MOE_SCORING_SIGMOID}[scoring]
        self._shard = None
        if shard_map is not None:
            self._shard = np.ascontiguousarray(np.asarray(shard_map, dtype=np.int32).reshape(-1))
        cfg = MoeConfig(self.H, self.F, self.E, self.K, self.L, self.max_tokens, sc, self.device.index or 0,
                        int(ep_rank), int(ep_world),
                        None if self._shard is None else self._shard.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)))
        self.ep_rank, self.ep_world = int(ep_rank), int(ep_world)
        self.ep_attached = False
        h = ctypes.c_void_p()
        check(lib().moe_create(ctypes.byref(cfg), ctypes.byref(h)))
        self._h = h

    # ---- lifetime ----
    # ---- expert-parallel peer exchange (collective set-up; see parallel.attach_peers) ----
    def ep_export(self):
        """This rank's exchange-buffer handle record (bytes)."""
        from ._lib import MOE_EP_RECORD_BYTES
        buf = ctypes.create_string_buffer(MOE_EP_RECORD_BYTES)
        check(lib().moe_ep_export(self._h, buf, MOE_EP_RECORD_BYTES))
        return buf.raw

    def ep_import(self, records):
        """Map every rank's exchange buffer (records of all ranks, rank order, concatenated); from
        then on forward() returns the full combined output on every rank."""
        check(lib().moe_ep_import(self._h, records, self.ep_world))
        self.ep_attached = True

    def close(self):
        if getattr(self, "_h", None):
            lib().moe_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()

    @property
    def handle(self):
        return self._h

    def owner(self, layer, expert):
        if self._shard is not None:
            return int(self._shard[layer * self.E + expert])
        return 0 if self.ep_world == 1 else expert % self.ep_world

    # ---- expert tables ----
    def load_expert(self, layer, expert, gate, up, down):
        """gate/up [F,H], down [H,F] bf16 (torch, host or device, or numpy uint16 bits)."""
        g, u, d = (as_bf16(a) for a in (gate, up, down))
        assert g.shape == (self.F, self.H) and u.shape == (self.F, self.H) and d.shape == (self.H, self.F)
        flags = 0 if g.is_cuda else MOE_F_HOST
        if not g.is_cuda:
            u, d = u.cpu(), d.cpu()
        else:
            u, d = u.to(g.device), d.to(g.device)
        check(lib().moe_load_expert_bf16(self._h, layer, expert, _vp(g), _vp(u), _vp(d), flags))

    def load_expert_q8(self, layer, expert, q, scales):
        """q int8 [3*F*H] in the ck_place_expert_q8 layout, scales fp32 [2F+H]."""
        qt = _as(q, torch.int8)
        st = _as(scales, torch.float32, qt.device)
        flags = 0 if qt.is_cuda else MOE_F_HOST
        check(lib().moe_load_expert_q8(self._h, layer, expert, _vp(qt), _vp(st), flags))

    def quantize_expert_q8(self, layer, expert):
        check(lib().moe_quantize_expert_q8(self._h, layer, expert))

    def evict_expert(self, layer, expert):
        """Frees the expert's HBM slot (MOE_OPT_LAYER_SLOTS tables); it reads as not loaded afterwards."""
        check(lib().moe_evict_expert(self._h, layer, expert))

    def expert_kind(self, layer, expert):
        return lib().moe_expert_kind(self._h, layer, expert)

    def set_bias(self, layer, bias):
        if bias is None:
            check(lib().moe_set_bias(self._h, layer, None, 0))
            return
        b = _as(bias, torch.float32)
        check(lib().moe_set_bias(self._h, layer, _vp(b), 0 if b.is_cuda else MOE_F_HOST))

    # ---- hot path ----
    def forward(self, layer, hidden, logits, out=None, return_topk=False, accumulate=False, stream=None, sync=False):
        """hidden [T,H] bf16, logits [T,E] fp32 (device tensors) -> out [T,H] fp32 on the device.

        Asynchronous on ``stream`` (default: torch's current stream) unless ``sync``."""
        x = as_bf16(hidden)
        lg = _as(logits, torch.float32)
        T = x.shape[0]
        assert x.is_cuda and lg.is_cuda and x.shape[1] == self.H and lg.shape == (T, self.E)
        if out is None:
            out = torch.empty(T, self.H, dtype=torch.float32, device=x.device)
        idx = w = None
        if return_topk:
            idx = torch.empty(T, self.K, dtype=torch.int32, device=x.device)
            w = torch.empty(T, self.K, dtype=torch.float32, device=x.device)
        flags = (MOE_F_ACCUMULATE if accumulate else 0) | (MOE_F_SYNC if sync else 0)
        check(lib().moe_forward(self._h, layer, T, _vp(x), _vp(lg), _vp(out), _vp(idx), _vp(w), flags,
                                _stream_ptr(stream, x.device)))
        return (out, idx, w) if return_topk else out

    def forward_layers(self, layers, hiddens, logits, outs, accumulate=False, stream=None, sync=False):
        """Several layer calls enqueued by one C call (moe_forward_layers): layer layers[i] on
        hiddens[i] [T,H] bf16 and logits[i] [T,E] fp32 into outs[i] [T,H] fp32, device tensors, in
        order."""
        n = len(layers)
        assert len(hiddens) == len(logits) == len(outs) == n
        T = hiddens[0].shape[0] if n else 0
        for x, lg, o in zip(hiddens, logits, outs):
            assert x.is_cuda and x.dtype == torch.bfloat16 and x.shape == (T, self.H)
            assert lg.is_cuda and lg.dtype == torch.float32 and lg.shape == (T, self.E)
            assert o.is_cuda and o.dtype == torch.float32 and o.shape == (T, self.H)
        la = (ctypes.c_int32 * max(n, 1))(*layers)
        xa = (ctypes.c_void_p * max(n, 1))(*[t.data_ptr() for t in hiddens])
        ga = (ctypes.c_void_p * max(n, 1))(*[t.data_ptr() for t in logits])
        oa = (ctypes.c_void_p * max(n, 1))(*[t.data_ptr() for t in outs])
        flags = (MOE_F_ACCUMULATE if accumulate else 0) | (MOE_F_SYNC if sync else 0)
        dev = hiddens[0].device if n else self.device
        check(lib().moe_forward_layers(self._h, n, la, T, xa, ga, oa, flags, _stream_ptr(stream, dev)))
        return outs

    # ---- the steps either side of the routed experts (one Solar MoE block, solar_engine/src/layer.rs:1-6) ----
    def load_shared(self, layer, gate=None, up=None, down=None, router=None):
        """Shared expert gate/up [Fs,H], down [H,Fs] and router weights [E,H] (bf16) of one layer.
        Fs may differ from the routed F (a context holding a slice of every routed expert's units
        still holds the whole shared expert); it is fixed by the first load."""
        from ._lib import MOE_OPT_SHARED_INTER
        ws = [None if a is None else as_bf16(a) for a in (gate, up, down, router)]
        on_dev = [w.is_cuda for w in ws if w is not None]
        dev = bool(on_dev) and on_dev[0]
        ws = [None if w is None else (w.to(self.device) if dev else w.cpu()) for w in ws]
        if ws[0] is not None:
            fs = ws[0].shape[0]
            assert ws[0].shape == (fs, self.H) and ws[1].shape == (fs, self.H) and ws[2].shape == (self.H, fs)
            if getattr(self, "_shared_inter", None) != fs:
                self.set_option(MOE_OPT_SHARED_INTER, fs)
                self._shared_inter = fs
        if ws[3] is not None:
            assert ws[3].shape == (self.E, self.H)
        check(lib().moe_load_shared(self._h, layer, *[_vp(w) for w in ws], 0 if dev else MOE_F_HOST))

    def shared_router(self, layer, h2, x2, y=True, logits=True, stream=None, sync=False):
        """(y bf16 [T,H] = bf16(x2 + shared(h2)), logits f32 [T,E] = h2 . Wr^T) on the device
        (dense/shared.rs:1-3); either may be skipped."""
        h = as_bf16(h2)
        T = h.shape[0]
        x = as_bf16(x2) if y else None
        yo = torch.empty(T, self.H, dtype=torch.bfloat16, device=h.device) if y else None
        lo = torch.empty(T, self.E, dtype=torch.float32, device=h.device) if logits else None
        check(lib().moe_shared_router(self._h, layer, T, _vp(h), _vp(x), _vp(yo), _vp(lo), MOE_F_SYNC if sync else 0,
                                      _stream_ptr(stream, h.device)))
        return yo, lo

    def combine_residual(self, y, moe_out, extra=None, stream=None, sync=False):
        """x_next bf16 [T,H] = bf16((y + extra) + moe_out) (dense/combine.rs:1)."""
        yy = as_bf16(y)
        m = _as(moe_out, torch.float32)
        e = None if extra is None else _as(extra, torch.float32)
        T = yy.shape[0]
        xn = torch.empty(T, self.H, dtype=torch.bfloat16, device=yy.device)
        check(lib().moe_combine_residual(self._h, T, _vp(yy), _vp(e), _vp(m), _vp(xn), MOE_F_SYNC if sync else 0,
                                         _stream_ptr(stream, yy.device)))
        return xn

    def block_forward(self, layer, h2, x2, extra=None, return_parts=False, stream=None, sync=False):
        """One MoE block: x_next = bf16((bf16(x2 + shared(h2)) + extra) + routed(h2, h2 . Wr^T)).
        Device tensors in, device x_next out (with y and the logits when return_parts)."""
        h = as_bf16(h2)
        x = as_bf16(x2)
        e = None if extra is None else _as(extra, torch.float32)
        T = h.shape[0]
        xn = torch.empty(T, self.H, dtype=torch.bfloat16, device=h.device)
        yo = torch.empty(T, self.H, dtype=torch.bfloat16, device=h.device) if return_parts else None
        lo = torch.empty(T, self.E, dtype=torch.float32, device=h.device) if return_parts else None
        check(lib().moe_block_forward(self._h, layer, T, _vp(h), _vp(x), _vp(e), _vp(xn), _vp(yo), _vp(lo),
                                      MOE_F_SYNC if sync else 0, _stream_ptr(stream, h.device)))
        return (xn, yo, lo) if return_parts else xn

    def block_forward_host(self, layer, h2, x2, extra=None):
        """block_forward with host buffers (synchronous): returns x_next as a CPU bf16 tensor."""
        h = as_bf16(h2).cpu()
        x = as_bf16(x2).cpu()
        e = None if extra is None else _as(extra, torch.float32).cpu()
        xn = torch.empty(h.shape[0], self.H, dtype=torch.bfloat16)
        check(lib().moe_block_forward(self._h, layer, h.shape[0], _vp(h), _vp(x), _vp(e), _vp(xn), None, None,
                                      MOE_F_HOST, _stream_ptr(None, self.device)))
        return xn

    def forward_host(self, layer, hidden, logits, out=None, return_topk=False, accumulate=False):
        """Host buffers in and out (numpy or CPU tensors).  On the fused path pinned logits and
        16-byte-aligned pinned outputs are used in place by the kernels; others are staged."""
        x = as_bf16(hidden)
        lg = _as(logits, torch.float32)
        T = x.shape[0]
        if out is None:
            out = torch.empty(T, self.H, dtype=torch.float32)
        idx = w = None
        if return_topk:
            idx = torch.empty(T, self.K, dtype=torch.int32)
            w = torch.empty(T, self.K, dtype=torch.float32)
        flags = MOE_F_HOST | (MOE_F_ACCUMULATE if accumulate else 0)
        check(lib().moe_forward(self._h, layer, T, _vp(x), _vp(lg), _vp(out), _vp(idx), _vp(w), flags,
                                _stream_ptr(None, self.device)))
        return (out, idx, w) if return_topk else out

    def route(self, logits, bias=None, stream=None):
        """Router + permutation on the GPU; returns a dict of host numpy arrays (synchronous)."""
        lg = _as(logits, torch.float32, self.device)
        T = lg.shape[0]
        b = None if bias is None else _as(bias, torch.float32, self.device)
        dev = self.device
        r = dict(idx=torch.empty(T, self.K, dtype=torch.int32, device=dev),
                 w=torch.empty(T, self.K, dtype=torch.float32, device=dev),
                 counts=torch.empty(self.E, dtype=torch.int32, device=dev),
                 offsets=torch.empty(self.E + 1, dtype=torch.int32, device=dev),
                 perm=torch.empty(max(1, T * self.K), dtype=torch.int32, device=dev),
                 job_order=torch.empty(self.E, dtype=torch.int32, device=dev),
                 n_jobs=torch.empty(1, dtype=torch.int32, device=dev))
        status = lib().moe_route(self._h, T, _vp(lg), _vp(b), _vp(r["idx"]), _vp(r["w"]), _vp(r["counts"]),
                                 _vp(r["offsets"]), _vp(r["perm"]), _vp(r["job_order"]), _vp(r["n_jobs"]), MOE_F_SYNC,
                                 _stream_ptr(stream, dev))
        res = {k: v.cpu().numpy() for k, v in r.items()}
        res["perm"] = res["perm"][:T * self.K]
        res["job_order"] = res["job_order"][:int(res["n_jobs"][0])]
        res["status"] = status
        return res

    # ---- reference CPU-kernel surfaces ----
    def experts(self, x, gus, ds, toks, ws, out=None, accumulate=False, stream=None):
        """cpu_moe surface with device-resident weights: out[T,H] fp32 (device)."""
        xd = as_bf16(x, self.device)
        T = xd.shape[0]
        gus = [as_bf16(g, self.device) for g in gus]
        ds = [as_bf16(d, self.device) for d in ds]
        n = len(gus)
        off = np.zeros(n + 1, np.int64)
        for j, t in enumerate(toks):
            off[j + 1] = off[j] + len(t)
        tk = np.ascontiguousarray(np.concatenate([np.asarray(_cpu(t), np.int64) for t in toks]) if n else np.zeros(1, np.int64))
        wv = np.ascontiguousarray(np.concatenate([np.asarray(_cpu(w), np.float32) for w in ws]) if n else np.zeros(1, np.float32))
        gp = (ctypes.c_void_p * max(1, n))(*[g.data_ptr() for g in gus])
        dp = (ctypes.c_void_p * max(1, n))(*[d.data_ptr() for d in ds])
        if out is None:
            out = torch.empty(T, self.H, dtype=torch.float32, device=self.device)
        flags = MOE_F_ACCUMULATE if accumulate else 0
        check(lib().moe_experts(self._h, T, _vp(xd), n, gp, dp, off.ctypes.data_as(ctypes.c_void_p),
                                tk.ctypes.data_as(ctypes.c_void_p), wv.ctypes.data_as(ctypes.c_void_p), _vp(out),
                                flags, _stream_ptr(stream, self.device)))
        self._keep = (gus, ds)
        return out

    def ck_moe3(self, bases, w, x, out, stream=None):
        """ck_moe3: out[H] += sum_e w[e] * expert_e(x); bases = device bf16 tensors [3*F*H]."""
        n = len(bases)
        bp = (ctypes.c_void_p * max(1, n))(*[b.data_ptr() for b in bases])
        wd = _as(w, torch.float32, self.device)
        xd = as_bf16(x, self.device)
        check(lib().moe_ck_moe3(self._h, n, bp, _vp(wd), _vp(xd), _vp(out), 0, _stream_ptr(stream, self.device)))
        return out

    def ck_moe_q8w(self, qs, scs, w, x, out, stream=None):
        n = len(qs)
        qp = (ctypes.c_void_p * max(1, n))(*[q.data_ptr() for q in qs])
        sp = (ctypes.c_void_p * max(1, n))(*[s.data_ptr() for s in scs])
        wd = _as(w, torch.float32, self.device)
        xd = as_bf16(x, self.device)
        check(lib().moe_ck_moe_q8w(self._h, n, qp, sp, _vp(wd), _vp(xd), _vp(out), 0, _stream_ptr(stream, self.device)))
        return out

    def place_expert_q8(self, g, u, d, stream=None):
        """ck_place_expert_q8 on the GPU -> (q int8 [3FH], sc fp32 [2F+H], rs int32 [2F+H]) device tensors."""
        g, u, d = (as_bf16(a, self.device) for a in (g, u, d))
        q = torch.empty(3 * self.F * self.H, dtype=torch.int8, device=self.device)
        sc = torch.empty(2 * self.F + self.H, dtype=torch.float32, device=self.device)
        rs = torch.empty(2 * self.F + self.H, dtype=torch.int32, device=self.device)
        check(lib().moe_place_expert_q8(self._h, _vp(g), _vp(u), _vp(d), _vp(q), _vp(sc), _vp(rs), MOE_F_SYNC,
                                        _stream_ptr(stream, self.device)))
        return q, sc, rs

    def status(self, stream=None):
        return lib().moe_status(self._h, _stream_ptr(stream, self.device))

    @property
    def launch_count(self):
        return int(lib().moe_launch_count(self._h))

    def set_option(self, option, value):
        check(lib().moe_set_option(self._h, int(option), int(value)))

    def timeline(self):
        """Per-CTA phase stamps of the latest fused launch (MOE_OPT_TIMELINE on): [SMs, 24] ns."""
        sms = torch.cuda.get_device_properties(self.device).multi_processor_count
        n = sms * 24 + 3 * 1024
        buf = np.zeros(n, np.uint64)
        check(lib().moe_timeline_read(self._h, buf.ctypes.data_as(ctypes.c_void_p), n))
        self.stage_log = buf[sms * 24:].reshape(3, 1024)
        return buf[:sms * 24].reshape(-1, 24)

    def profile(self, enable=True):
        check(lib().moe_profile(self._h, int(bool(enable))))

    def profile_read(self, n_stages=4):
        """Summed ms per stage (route, gate/up, down, combine) of the profiled forwards, and their count."""
        ms = (ctypes.c_double * n_stages)()
        n = ctypes.c_int64()
        check(lib().moe_profile_read(self._h, ms, n_stages, ctypes.byref(n)))
        return list(ms), int(n.value)


def _cpu(t):
    return t.cpu() if isinstance(t, torch.Tensor) else t


# ---------------- cpu_moe_ext drop-in ----------------
_planes = {}


class _WeightCache:
    """Device copies of CPU weight tensors for gpu_moe, keyed on the tensor object itself.

    An entry holds a weak reference to the host tensor and the tensor's version counter
    (``Tensor._version``, bumped by every in-place write), so a tensor that is freed (its storage
    possibly reused at the same address) or overwritten in place (the reference's expert swap,
    runtime.py:287-311) is copied again instead of returning stale weights.  Entries die with their
    host tensor, and the cache keeps at most ``limit_bytes`` of device copies, evicting the least
    recently used first.
    """

    def __init__(self, limit_bytes):
        import collections
        self.limit = int(limit_bytes)
        self.bytes = 0
        self.entries = collections.OrderedDict()  # id(t) -> (weakref, version, device, copy)

    def _drop(self, key):
        e = self.entries.pop(key, None)
        if e is not None:
            self.bytes -= e[3].numel() * e[3].element_size()

    def get(self, t, device):
        import weakref
        key = id(t)
        e = self.entries.get(key)
        if e is not None and e[0]() is t and e[1] == t._version and e[2] == device:
            self.entries.move_to_end(key)
            return e[3]
        self._drop(key)
        d = as_bf16(t, device)
        nb = d.numel() * d.element_size()
        while self.entries and self.bytes + nb > self.limit:
            self._drop(next(iter(self.entries)))
        if nb <= self.limit:
            ref = weakref.ref(t, lambda _r, k=key, c=self: c._drop(k) if k in c.entries and c.entries[k][0] is _r else None)
            self.entries[key] = (ref, t._version, device, d)
            self.bytes += nb
        return d

    def clear(self):
        self.entries.clear()
        self.bytes = 0


# device copies of CPU weights: 8 GiB by default (NPU_OFFLOAD_GPU_MOE_CACHE_GB overrides)
_wcache = _WeightCache(float(__import__("os").environ.get("NPU_OFFLOAD_GPU_MOE_CACHE_GB", "8")) * (1 << 30))


def _plane_for(device, H, F, pairs, T, n_jobs):
    key = (device.index, H, F)
    p = _planes.get(key)
    if p is None or p.max_tokens * p.K < pairs or p.max_tokens < T or p.E < n_jobs:
        if p is not None:
            p.close()
        mt = 64
        while mt * 16 < pairs or mt < T:
            mt *= 2
        # scratch capacity is max_tokens * top_k pairs (top_k=16 needs n_experts >= 16)
        ne = 16
        while ne < n_jobs:
            ne *= 2
        if ne > 256:
            raise RuntimeError("gpu_moe supports at most 256 experts per call")
        p = MoEDataPlane(H, F, n_experts=ne, top_k=16, n_layers=1, max_tokens=min(mt, 4096), device=device)
        _planes[key] = p
    return p


def _device_weight(t, device):
    if t.is_cuda:
        return as_bf16(t)
    return _wcache.get(t, device)


def gpu_moe(x, gus, ds, toks, ws):
    """Drop-in for ``cpu_moe_ext.ext.cpu_moe`` (solar_hybrid/cpu_moe.cpp:38-96).

    x [T,H] bf16; gus[e] [2F,H] bf16 (gate rows then up rows); ds[e] [H,F] bf16; toks[e] int64 token
    rows; ws[e] fp32 routing weights.  Returns out [T,H] fp32 = sum_e ws[e] * expert_e(x[toks[e]]),
    on x's device (a CPU x gives a CPU result, as the reference does).  CPU weight tensors are copied
    to the GPU and cached per tensor object and version (a bounded cache: see _WeightCache); pass
    CUDA tensors to avoid the cache.
    """
    T, H = x.shape
    E = len(gus)
    if E == 0:
        return torch.zeros(T, H, dtype=torch.float32, device=x.device)
    F = ds[0].shape[1]
    if H % 32 != 0 or F % 32 != 0:
        raise RuntimeError("H,F must be multiples of 32")
    if H % 256 != 0 or F % 64 != 0:
        raise RuntimeError("gpu_moe needs H % 256 == 0 and F % 64 == 0")
    device = x.device if x.is_cuda else torch.device("cuda", torch.cuda.current_device())
    pairs = sum(len(t) for t in toks)
    plane = _plane_for(device, H, F, pairs, T, E)
    g = [_device_weight(a, device) for a in gus]
    d = [_device_weight(a, device) for a in ds]
    out = plane.experts(x, g, d, toks, ws)
    return out if x.is_cuda else out.cpu()


def set_threads(n):
    """Accepted for compatibility with cpu_moe_ext.set_threads; the GPU path has no host thread pool."""
    return None
