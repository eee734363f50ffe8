"""B200 expert server speaking the stdin/stdout protocol of the reference's generated expert server
(npu-kernels/npu_kernels/rngd/template/src/bin/server.rs.tpl:1-8, 63-97), for one shape (H, F, E, K):

    python -m npu_offload_b200.expert_server --hidden H --inter F --experts E --top-k K [--layers L] [--device D]

On start the server writes b"RDY1".  Requests are little endian, every field a u32 unless noted:

    op 1 LOAD      layer, path_len, path[u8]            -> u32 status
                   the layer's E slots from <path>.g, <path>.u, <path>.d (raw bf16)
    op 2 RUN       layer, n (<= K), slots[n], x[H] bf16 -> rows [n][H] bf16 (slot k's expert applied to x)
    op 3 UPDATE    layer, slot, path_len, path[u8]      -> u32 status
                   one slot from <path>.g, <path>.u, <path>.d (one expert each)
    op 4 RUN_WSUM  layer, n (<= K), slots[n], weights[n] f32, x[H] bf16 -> [H] f32 = sum_k w_k * row_k
    op 0 EXIT
    any other op                                        -> u32 1

File layout: the reference writes its chip's permuted device layouts; here every file is row-major
bf16 per slot -- .g [F][H] gate rows, .u [F][H] up rows, .d [H][F] down -- with LOAD files holding the
E slots back to back.  Status codes: 0 ok, 1 unknown op, 2 bad layer or slot, 3 bad file, 4 device
error.  RUN and RUN_WSUM reply data only (the reference has no status there and panics on a layer it
never loaded); on such a request the server reports the error on stderr and exits with status 2.

Compute: each RUN / RUN_WSUM is one call of the fused decode path (moe_forward): the n copies of x
are n tokens, and token k's router logits select only slot k with top-1 routing, whose renormalised
weight is exactly 1, so row k is slot k's fp32 output with cpu_moe's rounding points
(solar_hybrid/cpu_moe.cpp:63-93).  RUN rounds the rows to bf16 once; RUN_WSUM adds the fp32 rows,
weighted, in k order on the host -- where and how the reference server adds its rows
(server.rs.tpl:84-90).
"""
import argparse
import os
import struct
import sys

import numpy as np

OP_EXIT, OP_LOAD, OP_RUN, OP_UPDATE, OP_RUN_WSUM = 0, 1, 2, 3, 4
ST_OK, ST_UNKNOWN, ST_BAD_INDEX, ST_BAD_FILE, ST_DEVICE = 0, 1, 2, 3, 4


class ProtocolError(Exception):
    """A RUN / RUN_WSUM request the server cannot answer (the reference panics there)."""


def _read_exact(r, n):
    b = r.read(n)
    if b is None or len(b) != n:
        raise EOFError
    return b


def _u32(r):
    return struct.unpack("<I", _read_exact(r, 4))[0]


def _path(r):
    return _read_exact(r, _u32(r)).decode("utf-8", errors="replace")


def read_bf16(path, count):
    """count bf16 values (uint16 bits) from a raw file; ValueError when the size differs."""
    a = np.fromfile(path, dtype=np.uint16)
    if a.size != count:
        raise ValueError(f"{path}: {a.size} bf16 values, expected {count}")
    return a


def serve_stream(inp, out, backend):
    """Serves requests from the binary stream inp until EXIT or end of input; replies go to out.
    backend: load(layer, g [E,F,H], u [E,F,H], d [E,H,F]), update(layer, slot, g, u, d),
    rows(layer, slots, x) -> [n, H] float32 rows; H, F, E, K, L attributes."""
    H, F, E, K, L = backend.H, backend.F, backend.E, backend.K, backend.L
    out.write(b"RDY1")
    out.flush()
    while True:
        try:
            op = _u32(inp)
        except EOFError:
            return 0
        if op == OP_EXIT:
            return 0
        if op in (OP_LOAD, OP_UPDATE):
            layer = _u32(inp)
            slot = _u32(inp) if op == OP_UPDATE else None
            path = _path(inp)
            st = ST_OK
            if layer >= L or (slot is not None and slot >= E):
                st = ST_BAD_INDEX
            else:
                n = 1 if op == OP_UPDATE else E
                try:
                    g = read_bf16(path + ".g", n * F * H).reshape(n, F, H)
                    u = read_bf16(path + ".u", n * F * H).reshape(n, F, H)
                    d = read_bf16(path + ".d", n * H * F).reshape(n, H, F)
                except (OSError, ValueError) as ex:
                    print(f"[expert_server] {ex}", file=sys.stderr, flush=True)
                    st = ST_BAD_FILE
                if st == ST_OK:
                    try:
                        if op == OP_LOAD:
                            backend.load(layer, g, u, d)
                        else:
                            backend.update(layer, slot, g[0], u[0], d[0])
                    except Exception as ex:
                        print(f"[expert_server] device error: {ex}", file=sys.stderr, flush=True)
                        st = ST_DEVICE
            out.write(struct.pack("<I", st))
            out.flush()
        elif op in (OP_RUN, OP_RUN_WSUM):
            layer, n = _u32(inp), _u32(inp)
            if n > K:  # the request's length is unknown past this point: the stream cannot resync
                raise ProtocolError(f"n = {n} slots exceeds K = {K}")
            slots = list(struct.unpack(f"<{n}I", _read_exact(inp, 4 * n)))
            wts = np.frombuffer(_read_exact(inp, 4 * n), dtype="<f4") if op == OP_RUN_WSUM else None
            x = np.frombuffer(_read_exact(inp, 2 * H), dtype="<u2").copy()
            if layer >= L or any(s >= E for s in slots) or not backend.loaded(layer):
                raise ProtocolError(f"layer {layer} / slots {slots} not loaded")
            rows = backend.rows(layer, slots, x)  # [n, H] float32
            if op == OP_RUN:
                out.write(np.ascontiguousarray(f2bf(rows)).astype("<u2").tobytes())
            else:
                acc = np.zeros(H, np.float32)
                for k in range(n):  # sum_k w_k * row_k in k order, fp32 (server.rs.tpl:84-90)
                    acc += np.float32(wts[k]) * rows[k]
                out.write(acc.astype("<f4").tobytes())
            out.flush()
        else:
            out.write(struct.pack("<I", ST_UNKNOWN))
            out.flush()


def f2bf(a):
    """fp32 -> bf16 bits, round to nearest even."""
    u = np.ascontiguousarray(a, dtype=np.float32).view(np.uint32).astype(np.uint64)
    return (((u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFFFFFF) >> 16).astype(np.uint16)


class GpuBackend:
    """E expert slots per layer in HBM; every request is one fused decode call (top-1 per row token)."""

    def __init__(self, H, F, E, K, L, device=0):
        import torch
        from .moe import MoEDataPlane
        self.torch = torch
        self.H, self.F, self.E, self.K, self.L = H, F, E, K, L
        self.dev = torch.device("cuda", device)
        torch.cuda.set_device(self.dev)
        self.plane = MoEDataPlane(H, F, E, 1, n_layers=L, max_tokens=K, device=device)
        self._loaded = set()
        self.x = torch.empty(K, H, dtype=torch.bfloat16, device=self.dev)
        self.lg = torch.zeros(K, E, dtype=torch.float32, device=self.dev)
        self.out = torch.empty(K, H, dtype=torch.float32, device=self.dev)
        self.x_host = torch.empty(H, dtype=torch.bfloat16).pin_memory()
        self.lg_host = torch.zeros(K, E, dtype=torch.float32).pin_memory()
        self.out_host = torch.empty(K, H, dtype=torch.float32).pin_memory()

    def loaded(self, layer):
        return layer in self._loaded

    def load(self, layer, g, u, d):
        for e in range(self.E):
            self.plane.load_expert(layer, e, g[e], u[e], d[e])
        self._loaded.add(layer)

    def update(self, layer, slot, g, u, d):
        if layer not in self._loaded:
            raise RuntimeError(f"layer {layer} is not loaded")
        self.plane.load_expert(layer, slot, g, u, d)  # the slot's unit table is rewritten in place

    def rows(self, layer, slots, x_bits):
        torch = self.torch
        n = len(slots)
        self.x_host.view(torch.int16).numpy()[:] = x_bits.view(np.int16)
        self.x[:n].copy_(self.x_host.to(self.dev, non_blocking=True).expand(n, self.H))
        lg = self.lg_host.numpy()
        lg[:] = 0.0
        lg[np.arange(n), slots] = 1.0  # top-1 = slot k; the renormalised weight is exactly 1
        self.lg[:n].copy_(self.lg_host[:n], non_blocking=True)
        self.plane.forward(layer, self.x[:n], self.lg[:n], out=self.out[:n])
        self.out_host[:n].copy_(self.out[:n])
        return self.out_host[:n].numpy().copy()

    def close(self):
        self.plane.close()


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--hidden", type=int, required=True)
    ap.add_argument("--inter", type=int, required=True)
    ap.add_argument("--experts", type=int, required=True, help="expert slots per layer (E)")
    ap.add_argument("--top-k", type=int, required=True, help="largest n of a RUN request (K)")
    ap.add_argument("--layers", type=int, default=64)
    ap.add_argument("--device", type=int, default=int(os.environ.get("EXPERT_SERVER_DEVICE", "0")))
    a = ap.parse_args(argv)
    be = GpuBackend(a.hidden, a.inter, a.experts, a.top_k, a.layers, a.device)
    inp = sys.stdin.buffer
    out = sys.stdout.buffer
    try:
        return serve_stream(inp, out, be)
    except ProtocolError as ex:
        print(f"[expert_server] {ex}", file=sys.stderr, flush=True)
        return 2
    finally:
        be.close()


if __name__ == "__main__":
    sys.exit(main())
