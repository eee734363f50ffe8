"""B200 hot-expert server speaking track2_opt/expert_srv's shared-memory mailbox protocol.

Drop-in for ``expert_srv <shm_path> <weights_dir> <n_layers>`` (track2_opt/expert_srv/src/main.rs:1-20),
the server that solar_hybrid/opt_client.py (``OptExpertServer``) starts and drives:

    python -m npu_offload_b200.expert_srv <shm_path> <weights_dir> <n_layers> [--hidden H --inter F --device D]

weights_dir/layer_<l>.bin holds E = 32 experts of raw row-major bf16, per slot [Wg F*H][Wu F*H][Wd H*F]
(opt_client.export_tables).  Mailbox layout (little endian), as main.rs:10-20:

    0  u64 req_seq    client increments after writing a request
    8  u64 resp_seq   server sets = req_seq when done
    16 u32 op         1 = expert rows (ffn_k8u), 3 = quit
    20 u32 layer
    24 u64 packed ids count << 56 | slot_k << 6k
    32 u32 status     0 ok, nonzero error (1 unknown op, 2 bad layer, 3 bad slot, 4 device error)
    36 u32 ready      server sets 1 once the tables are resident
    40 f64 last_us    server-side latency of the last request
    64      x   : H bf16
    16384   out : K*H bf16, row k = expert slot_k's output (unweighted; the client combines)

Each request runs on the fused decode path: the K copies of x are K tokens, and token k's logits
select only slot_k with top-1 routing, so its weight renormalises to exactly 1.  Expert k's fp32
output (cpu_moe rounding points, solar_hybrid/cpu_moe.cpp:63-93) lands in row k and is rounded to
bf16 once for the mailbox.
"""
import argparse
import mmap
import os
import struct
import sys
import time

import numpy as np

E_SRV, K_MAX = 32, 8
OFF_X, OFF_OUT = 64, 16384


def shm_bytes(H, K=K_MAX):
    return OFF_OUT + K * H * 2 + 4096


def unpack_ids(packed):
    """(count, [slot_k]) of a packed id word: count << 56 | slot_k << 6k (opt_client.ffn)."""
    n = (packed >> 56) & 0xFF
    return n, [(packed >> (6 * k)) & 0x3F for k in range(min(n, K_MAX))]


def load_layer_file(path, H, F, E=E_SRV):
    """[E] (gate [F,H], up [F,H], down [H,F]) uint16 views of one layer_<l>.bin."""
    a = np.fromfile(path, dtype=np.uint16)
    per = 3 * F * H
    if a.size != E * per:
        raise ValueError(f"{path}: {a.size * 2} bytes, expected {E * per * 2}")
    out = []
    for e in range(E):
        s = a[e * per:(e + 1) * per]
        out.append((s[:F * H].reshape(F, H), s[F * H:2 * F * H].reshape(F, H), s[2 * F * H:].reshape(H, F)))
    return out


class ExpertServer:
    """The data plane behind the mailbox: E_SRV slots per layer, top-1 routing per row token."""

    def __init__(self, weights_dir, n_layers, H=4096, F=1280, device=0):
        import torch
        from .moe import MoEDataPlane
        self.torch = torch
        self.H, self.F, self.L = H, F, n_layers
        self.dev = torch.device("cuda", device)
        torch.cuda.set_device(self.dev)
        self.plane = MoEDataPlane(H, F, E_SRV, 1, n_layers=n_layers, max_tokens=K_MAX, device=device)
        for l in range(n_layers):
            for e, (g, u, d) in enumerate(load_layer_file(os.path.join(weights_dir, f"layer_{l}.bin"), H, F)):
                self.plane.load_expert(l, e, g, u, d)
        self.x = torch.empty(K_MAX, H, dtype=torch.bfloat16, device=self.dev)
        self.lg = torch.zeros(K_MAX, E_SRV, dtype=torch.float32, device=self.dev)
        self.out = torch.empty(K_MAX, H, dtype=torch.float32, device=self.dev)
        self.lg_host = torch.zeros(K_MAX, E_SRV, dtype=torch.float32).pin_memory()
        self.rows_host = torch.empty(K_MAX, H, dtype=torch.bfloat16).pin_memory()
        self.x_host = torch.empty(H, dtype=torch.bfloat16).pin_memory()

    def rows(self, layer, slots, x_bits):
        """[len(slots), H] bf16 bits: expert slot_k applied to x (uint16 bits [H])."""
        torch = self.torch
        n = len(slots)
        self.x_host.view(torch.int16).numpy()[:] = x_bits.view(np.int16)
        self.x[:n].copy_(self.x_host.to(self.dev, non_blocking=True).expand(n, self.H))
        lg = self.lg_host.numpy()
        lg[:] = 0.0
        lg[np.arange(n), slots] = 1.0  # top-1 = slot_k; the renormalised weight is exactly 1
        self.lg[:n].copy_(self.lg_host[:n].to(self.dev, non_blocking=True))
        self.plane.forward(layer, self.x[:n], self.lg[:n], out=self.out[:n])
        self.rows_host[:n].copy_(self.out[:n].to(torch.bfloat16))  # one RNE rounding per element
        return self.rows_host[:n].view(torch.int16).numpy().view(np.uint16)

    def close(self):
        self.plane.close()


def serve(shm_path, weights_dir, n_layers, H=4096, F=1280, device=0, idle_sleep=True):
    nbytes = shm_bytes(H)
    f = open(shm_path, "r+b")
    mm = mmap.mmap(f.fileno(), nbytes)
    x_view = np.frombuffer(mm, dtype=np.uint16, count=H, offset=OFF_X)
    out_view = np.frombuffer(mm, dtype=np.uint16, count=K_MAX * H, offset=OFF_OUT)
    srv = ExpertServer(weights_dir, n_layers, H, F, device)
    # warm the path once, then signal ready (main.rs:88-92)
    srv.rows(0, [0], np.zeros(H, np.uint16))
    struct.pack_into("<Q", mm, 8, struct.unpack_from("<Q", mm, 0)[0])
    struct.pack_into("<I", mm, 36, 1)
    print(f"[expert_srv] ready: {n_layers} layers x {E_SRV} experts", file=sys.stderr, flush=True)
    last = struct.unpack_from("<Q", mm, 0)[0]
    try:
        while True:
            cur = struct.unpack_from("<Q", mm, 0)[0]
            spins = 0
            while cur == last:
                spins += 1
                if idle_sleep and spins > 4096:
                    time.sleep(0)
                cur = struct.unpack_from("<Q", mm, 0)[0]
            last = cur
            t0 = time.perf_counter()
            op, layer, packed = struct.unpack_from("<IIQ", mm, 16)
            if op == 3:
                struct.pack_into("<I", mm, 32, 0)
                struct.pack_into("<Q", mm, 8, cur)
                break
            st = 0
            if op != 1:
                st = 1
            elif layer >= n_layers:
                st = 2
            else:
                n, slots = unpack_ids(packed)
                if n < 1 or n > K_MAX or any(s >= E_SRV for s in slots):
                    st = 3
                else:
                    try:
                        out_view[:n * H] = srv.rows(layer, slots, x_view.copy()).ravel()
                    except Exception as ex:  # device-side status (e.g. MOE_ETIMEOUT) -> mailbox status
                        print(f"[expert_srv] request failed: {ex}", file=sys.stderr, flush=True)
                        st = 4
            struct.pack_into("<d", mm, 40, (time.perf_counter() - t0) * 1e6)
            struct.pack_into("<I", mm, 32, st)
            struct.pack_into("<Q", mm, 8, cur)  # publish last (x86 TSO keeps the order)
    finally:
        srv.close()
        del x_view, out_view  # release the buffer exports before unmapping
        mm.close()
        f.close()
        print("[expert_srv] quit", file=sys.stderr, flush=True)


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("shm_path")
    ap.add_argument("weights_dir")
    ap.add_argument("n_layers", type=int)
    ap.add_argument("--hidden", type=int, default=4096)
    ap.add_argument("--inter", type=int, default=1280)
    ap.add_argument("--device", type=int, default=int(os.environ.get("EXPERT_SRV_DEVICE", "0")))
    a = ap.parse_args(argv)
    serve(a.shm_path, a.weights_dir, a.n_layers, a.hidden, a.inter, a.device)
    return 0


if __name__ == "__main__":
    sys.exit(main())
