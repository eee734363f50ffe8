#!/usr/bin/env python
"""Benchmark: routed-expert MoE layer decode on B200 (BASELINE metric "MoE-layer decode tokens/s and
achieved HBM GB/s vs peak at 1/2/4/8 B200").

A step is one decode pass of the expert stack over one batch: for each MoE layer, router +
permutation + expert FFN (GEMV path) + combine, through the library's hot path (moe_forward).

  N = 1: configs[1] -- 8 Solar-shaped MoE layers (H 4096, 128 experts, F 1280, top-8), 32.2 GB of
         bf16 expert weights resident, decode batch --batch (default 1; --sweep adds 4 and 16).
  N > 1: configs[2] pro-rated -- 6*N layers (48 at N = 8), expert-parallel with every GPU holding the
         same slice of the intermediate units of every expert (--ep-shard units, the default;
         --ep-shard experts deals whole experts by popularity stripe instead), combined per layer
         inside the decode kernel over NVLink peer memory (--ep nccl: one NCCL all-reduce).  Weak
         scaling: per-GPU expert bytes stay fixed.

value = MoE-layer tokens/s = batch * layers / step time (max over ranks, CUDA events).
Synthetic seeded inputs (no checkpoint exists here): weights N(0, 0.02) bf16, hidden N(0,1) bf16,
logits N(0,1) + log-Zipf(1.0) popularity bias.  Per step every layer streams its routed experts
(about 2 GB at N = 1, batch 1), far above the 126 MB L2, so no flush is needed between steps.

`--impl reference` times the reference's own CPU implementation (cpu_moe compiled from the
reference sources into oracle/_ref when that runs on this host, else the C restatement) on the
host cores, on a bounded sample of the same workload.
"""
import argparse
import ctypes
import json
import os
import statistics
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

H, F, E, K = 4096, 1280, 128, 8
EXPERT_BYTES = 3 * H * F * 2          # 31,457,280 B per bf16 expert
DOWN_BYTES = H * F * 2
METRIC = "MoE-layer decode tokens/s and achieved HBM GB/s vs peak"
UNIT = "MoE-layer tokens/s"
# DRAM bytes (read + write) per algorithmic byte of decode_kernel, from the committed ncu capture of
# one T=1 layer (profiles/decode_kernel_T1.md); None until a capture exists.
TRAFFIC_RATIO = 255.503 / 251.658
TRAFFIC_SOURCE = "profiles/decode_kernel_T1.md"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=400)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--batch", type=int, default=1, help="decode tokens per step")
    ap.add_argument("--layers", type=int, default=0, help="0: 8 at N=1, 6*N at N>1")
    ap.add_argument("--sweep", default="4,16", help="extra decode batches reported in 'sweep' ('' to skip)")
    ap.add_argument("--rotate", type=int, default=4, help="distinct input sets cycled across steps")
    ap.add_argument("--seed", type=int, default=1234)
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-seconds", type=float, default=10.0, help="CPU-baseline sample budget")
    ap.add_argument("--prefill-tokens", type=int, default=2048,
                    help="configs[3] prefill measurement at N=1 (0 to skip)")
    ap.add_argument("--no-block", action="store_true", help="skip the moe_block_forward measurement")
    ap.add_argument("--no-int8", action="store_true", help="skip the configs[4] int8 measurement")
    ap.add_argument("--int8-experts", type=int, default=96,
                    help="int8 measurement: the N least popular experts of every layer stored int8 (configs[4]: 96)")
    ap.add_argument("--cold-slots", type=int, default=0,
                    help="HBM slots per layer for the host-cold tier measurement (0: skip)")
    ap.add_argument("--no-alt-split", action="store_true",
                    help="N > 1 with --ep-shard units: skip the expert-sharded split's batch-1 measurement")
    ap.add_argument("--ep-shard", choices=["units", "experts"], default="units",
                    help="N>1 split: every rank a slice of every expert's units, or whole experts per rank")
    ap.add_argument("--ep", choices=["p2p", "nccl"], default="p2p",
                    help="N>1 combine: in-kernel NVLink peer exchange (p2p) or an NCCL all-reduce per layer")
    return ap.parse_args()


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


# ---------------------------------------------------------------- clocks during the timed region
class ClockSampler:
    """Samples SM clock / throttle reasons with NVML every ~2 ms on a thread."""

    REASONS = {"hw_slowdown": 0x8, "hw_thermal_slowdown": 0x40, "sw_thermal_slowdown": 0x20,
               "sw_power_cap": 0x4, "hw_power_brake_slowdown": 0x80}

    def __init__(self, dev_index):
        self.samples, self.reasons = [], set()
        self.max_mhz = None
        self._stop = threading.Event()
        self._t = None
        try:
            import pynvml
            import torch
            pynvml.nvmlInit()
            self.nv = pynvml
            try:
                p = torch.cuda.get_device_properties(dev_index)
                bus = "%08x:%02x:%02x.0" % (p.pci_domain_id, p.pci_bus_id, p.pci_device_id)
                self.h = pynvml.nvmlDeviceGetHandleByPciBusId(bus)
            except Exception:
                self.h = pynvml.nvmlDeviceGetHandleByIndex(dev_index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
            self._reasons_fn = getattr(pynvml, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
                getattr(pynvml, "nvmlDeviceGetCurrentClocksThrottleReasons")
        except Exception:
            self.nv = None

    def _run(self):
        nv = self.nv
        while not self._stop.is_set():
            try:
                self.samples.append(nv.nvmlDeviceGetClockInfo(self.h, nv.NVML_CLOCK_SM))
                r = self._reasons_fn(self.h)
                for name, bit in self.REASONS.items():
                    if r & bit:
                        self.reasons.add(name)
            except Exception:
                pass
            time.sleep(0.002)

    def __enter__(self):
        if self.nv:
            self._t = threading.Thread(target=self._run, daemon=True)
            self._t.start()
        return self

    def __exit__(self, *a):
        self._stop.set()
        if self._t:
            self._t.join()

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": sorted(self.reasons), "samples": 0}
        return {"sm_mhz": float(statistics.median(self.samples)), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons), "samples": len(self.samples)}


# ---------------------------------------------------------------- workload
def dist_env():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return ws, rank, local


def make_inputs(seed, R, L, T):
    from npu_offload_b200 import synth
    xs = np.stack([np.stack([synth.hidden(seed + 7919 * r + 31 * l, T, H) for l in range(L)]) for r in range(R)])
    # noise varies per input set; the popularity bias is a property of the layer (fixed across steps)
    lgs = np.stack([np.stack([synth.logits(seed + 7919 * r + 31 * l, T, E, zipf=False) + synth.zipf_bias(seed + 31 * l, E)
                              for l in range(L)]) for r in range(R)]).astype(np.float32)
    return xs, lgs  # [R, L, T, H] uint16, [R, L, T, E] f32


def popularity_counts(seed, L):
    """Per-layer popularity used for the shard map: the Zipf prior of the synthetic logits."""
    from npu_offload_b200 import synth
    out = np.zeros((L, E))
    for l in range(L):
        b = synth.zipf_bias(seed + 31 * l, E)  # the popularity bias make_inputs adds to layer l
        out[l] = np.exp(b)
    return out


def load_weights(plane, layers, owner, rank, seed, device, units=None):
    """This rank's experts (owner[l, e] == rank); with units = (f0, f1) only those units of each."""
    import torch
    from npu_offload_b200.parallel import unit_slice
    gen = torch.Generator(device=device)
    FH = F * H
    for l in range(layers):
        for e in range(E):
            if owner[l, e] != rank:
                continue
            gen.manual_seed(seed * 1_000_003 + 1009 * l + e)
            buf = (torch.randn(3 * FH, generator=gen, device=device) * 0.02).to(torch.bfloat16)
            g, u, d = buf[:FH].view(F, H), buf[FH:2 * FH].view(F, H), buf[2 * FH:].view(H, F)
            if units is not None:
                g, u, d = unit_slice(g, u, d, *units)
            plane.load_expert(l, e, g, u, d)
    torch.cuda.synchronize(device)


class Stack:
    """The measured workload on one rank."""

    def __init__(self, args, ws, rank, device, T, L):
        import torch
        from npu_offload_b200.moe import MoEDataPlane
        from npu_offload_b200.parallel import shard_map
        from npu_offload_b200.parallel import unit_ranges
        self.T, self.L, self.ws, self.rank, self.device = T, L, ws, rank, device
        self.units = None
        self.shard = getattr(args, "ep_shard", "units") if ws > 1 else None
        if ws > 1 and self.shard == "units":  # every rank owns its slice of the units of every expert
            self.units = unit_ranges(F, ws)[rank]
            self.owner = np.full((L, E), rank, np.int32)
        else:
            self.owner = shard_map(popularity_counts(args.seed, L), ws) if ws > 1 else np.zeros((L, E), np.int32)
        F_local = F if self.units is None else self.units[1] - self.units[0]
        self.ebytes = 3 * H * F_local * 2  # streamed bytes of one routed expert on this rank
        self.plane = MoEDataPlane(H, F_local, E, K, n_layers=L,
                                  max_tokens=max(T, 16, getattr(args, "prefill_tokens", 0)), device=device.index,
                                  ep_rank=rank, ep_world=ws, shard_map=self.owner if ws > 1 else None)
        load_weights(self.plane, L, self.owner, rank, args.seed, device, self.units)
        if ws > 1 and getattr(args, "ep", "p2p") == "p2p":
            from npu_offload_b200.parallel import attach_peers
            attach_peers(self.plane)  # the decode kernel combines over NVLink peer memory
        self.R = args.rotate
        self.set_batch(T, args.seed)

    def set_batch(self, T, seed):
        import torch
        self.T = T
        xs, lgs = make_inputs(seed, self.R, self.L, T)
        self.xs_np, self.lgs_np = xs, lgs
        self.x = torch.from_numpy(xs.view(np.int16)).view(torch.bfloat16).to(self.device)
        self.lg = torch.from_numpy(lgs).to(self.device)
        self.out = torch.empty(self.L, T, H, dtype=torch.float32, device=self.device)
        # per (rotation, layer) ctypes arguments of moe_forward, and per rotation the argument arrays of
        # moe_forward_layers, so the timed loop is one C call per step
        vp = ctypes.c_void_p
        self.args = [[(l, T, vp(self.x[r, l].data_ptr()), vp(self.lg[r, l].data_ptr()), vp(self.out[l].data_ptr()))
                      for l in range(self.L)] for r in range(self.R)]
        L = self.L
        self.step_args = [((ctypes.c_int32 * L)(*range(L)),
                           (vp * L)(*[self.x[r, l].data_ptr() for l in range(L)]),
                           (vp * L)(*[self.lg[r, l].data_ptr() for l in range(L)]),
                           (vp * L)(*[self.out[l].data_ptr() for l in range(L)])) for r in range(self.R)]
        self.sp = vp(torch.cuda.current_stream(self.device).cuda_stream)
        # algorithmic bytes per (rotation, layer): this rank's distinct routed experts
        self.ubytes = np.zeros((self.R, self.L))
        self.ucount = np.zeros((self.R, self.L))
        for r in range(self.R):
            for l in range(self.L):
                _, idx, _ = self.plane.forward(l, self.x[r, l], self.lg[r, l], out=self.out[l], return_topk=True)
                ids = set(idx.cpu().numpy().ravel().tolist())
                loc = [e for e in ids if self.owner[l, e] == self.rank]
                self.ucount[r, l] = len(loc)
                self.ubytes[r, l] = len(loc) * self.ebytes
        torch.cuda.synchronize(self.device)

    def step(self, s):
        from npu_offload_b200._lib import check, lib
        h, sp = self.plane.handle, self.sp
        if self.ws == 1 or self.plane.ep_attached:  # every layer of the step in one C call
            la, xa, ga, oa = self.step_args[s % self.R]
            check(lib().moe_forward_layers(h, self.L, la, self.T, xa, ga, oa, 0, sp))
            return
        fn = lib().moe_forward
        for l, T, x, lg, out in self.args[s % self.R]:
            check(fn(h, l, T, x, lg, out, None, None, 0, sp))
            from npu_offload_b200.parallel import allreduce_partial
            allreduce_partial(self.out[l])


def barrier(ws):
    if ws > 1:
        import torch.distributed as dist
        dist.barrier()


def max_over_ranks(v, ws):
    if ws == 1:
        return v
    import torch
    import torch.distributed as dist
    t = torch.tensor([v], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def sum_over_ranks(v, ws):
    if ws == 1:
        return v
    import torch
    import torch.distributed as dist
    t = torch.tensor([v], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return float(t.item())


def timed(stack, steps, warmup, ws, profile=False):
    import torch
    for s in range(warmup):
        stack.step(s)
    torch.cuda.synchronize(stack.device)
    barrier(ws)
    torch.cuda.synchronize(stack.device)
    if profile:
        stack.plane.profile(True)
    l0 = stack.plane.launch_count
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record()
    for s in range(steps):
        stack.step(warmup + s)
    ev1.record()
    torch.cuda.synchronize(stack.device)
    launches = stack.plane.launch_count - l0
    stage = None
    if profile:
        stage, ncalls = stack.plane.profile_read()
        stack.plane.profile(False)
    barrier(ws)
    ms = ev0.elapsed_time(ev1)
    return ms, launches, stage


def e2e_run(stack, steps, warmup, ws):
    """Same metric through the C ABI with host buffers: per layer pinned H2D of hidden+logits, the
    kernels, and a D2H of the output, all inside the timed region (MOE_F_HOST calls)."""
    import torch
    from npu_offload_b200._lib import MOE_F_HOST, check, lib
    L, T, R = stack.L, stack.T, stack.R
    xh = torch.from_numpy(stack.xs_np.view(np.int16)).pin_memory()
    lh = torch.from_numpy(stack.lgs_np).pin_memory()
    oh = torch.empty(L, T, H, dtype=torch.float32).pin_memory()
    fn = lib().moe_forward
    h = stack.plane.handle
    sp = ctypes.c_void_p(torch.cuda.current_stream(stack.device).cuda_stream)
    ptrs = [[(ctypes.c_void_p(xh[r, l].data_ptr()), ctypes.c_void_p(lh[r, l].data_ptr())) for l in range(L)]
            for r in range(R)]
    optr = [ctypes.c_void_p(oh[l].data_ptr()) for l in range(L)]

    def one(s):
        r = s % R
        for l in range(L):
            if ws == 1:
                check(fn(h, l, T, ptrs[r][l][0], ptrs[r][l][1], optr[l], None, None, MOE_F_HOST, sp))
            else:
                # expert parallel: host inputs -> device, partial, NCCL all-reduce, result -> host
                stack.x[r, l].copy_(xh[r, l], non_blocking=True)
                stack.lg[r, l].copy_(lh[r, l], non_blocking=True)
                stack.plane.forward(l, stack.x[r, l], stack.lg[r, l], out=stack.out[l])
                if not stack.plane.ep_attached:
                    from npu_offload_b200.parallel import allreduce_partial
                    allreduce_partial(stack.out[l])
                oh[l].copy_(stack.out[l], non_blocking=True)
        if ws > 1:
            torch.cuda.current_stream(stack.device).synchronize()

    for s in range(warmup):
        one(s)
    torch.cuda.synchronize(stack.device)
    barrier(ws)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record()
    for s in range(steps):
        one(warmup + s)
    ev1.record()
    torch.cuda.synchronize(stack.device)
    barrier(ws)
    ms = max_over_ranks(ev0.elapsed_time(ev1), ws)
    h2d = L * (T * H * 2 + T * E * 4) * ws
    d2h = L * T * H * 4 * (ws if ws > 1 else 1)
    return T * L * steps / (ms / 1e3), h2d, d2h


def prefill_run(stack, T, reps=5, warmup=2, ws=1):
    """one MoE layer (layer 0 of the stack) at T prefill tokens with uniform routing
    (logits N(0,1), no popularity bias; ~T*K/E tokens per expert).  Device-resident inputs, CUDA
    events around `reps` back-to-back layer calls; with ws > 1 every rank runs its share of the
    experts (its slice of every expert's units under unit sharding) and the partial outputs are
    combined across ranks, timed as the max over ranks."""
    import torch
    from npu_offload_b200 import synth
    x = torch.from_numpy(synth.hidden(99, T, H).view(np.int16)).view(torch.bfloat16).to(stack.device)
    lg = torch.from_numpy(synth.logits(99, T, E, zipf=False)).to(stack.device)
    out = torch.empty(T, H, dtype=torch.float32, device=stack.device)
    _, idx, _ = stack.plane.forward(0, x, lg, out=out, return_topk=True, sync=True)
    experts = len(set(idx.cpu().numpy().ravel().tolist()))
    for _ in range(warmup):
        stack.plane.forward(0, x, lg, out=out)
    torch.cuda.synchronize(stack.device)
    barrier(ws)
    l0 = stack.plane.launch_count
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record()
    for _ in range(reps):
        stack.plane.forward(0, x, lg, out=out)
    ev1.record()
    torch.cuda.synchronize(stack.device)
    barrier(ws)
    ms = max_over_ranks(ev0.elapsed_time(ev1), ws) / reps
    flops = 2.0 * T * K * 3 * H * F
    wbytes = experts * EXPERT_BYTES / ws  # each rank's streamed weight bytes (an even split)
    return {"workload": f"configs[3]: 1 layer, {T} prefill tokens, uniform routing ({T * K / E:.0f} tokens/expert)",
            "tokens_per_s": T / (ms / 1e3), "ms_per_layer": ms, "tflops": flops / (ms / 1e3) / 1e12,
            "weights_gbs": wbytes / (ms / 1e3) / 1e9, "experts": experts, "n_gpus": ws,
            "path": "tcgen05 kernels: gate/up with fused SwiGLU, down with fp32 output; gather + combine kernels",
            "gpu_launches_per_layer": (stack.plane.launch_count - l0) / reps}


def block_run(stack, steps, warmup, T=1):
    """The whole MoE block around the path (the steps either side of the routed experts, layer.rs:1-6):
    router GEMV producing the logits,
    routed experts, the shared expert and the residual combine into the next layer's input
    (moe_block_forward), per layer of the stack, device-resident inputs, CUDA events."""
    import torch
    from npu_offload_b200 import synth
    L, R, dev = stack.L, stack.R, stack.device
    gen = torch.Generator(device=dev)
    for l in range(L):
        gen.manual_seed(7919 + l)
        w = [(torch.randn(*shape, generator=gen, device=dev) * 0.02).to(torch.bfloat16)
             for shape in ((F, H), (F, H), (H, F), (E, H))]
        stack.plane.load_shared(l, *w)
    h2 = torch.from_numpy(np.stack([np.stack([synth.hidden(500 + 31 * r + l, T, H) for l in range(L)])
                                    for r in range(R)]).view(np.int16)).view(torch.bfloat16).to(dev)
    x2 = torch.from_numpy(np.stack([np.stack([synth.hidden(900 + 31 * r + l, T, H) for l in range(L)])
                                    for r in range(R)]).view(np.int16)).view(torch.bfloat16).to(dev)
    routed = np.zeros((R, L))
    for r in range(R):
        for l in range(L):
            _, _, lg = stack.plane.block_forward(l, h2[r, l], x2[r, l], return_parts=True)
            top = np.argsort(-lg.cpu().numpy(), axis=1, kind="stable")[:, :K]
            routed[r, l] = len(set(top.ravel().tolist()))
    xn = torch.empty(L, T, H, dtype=torch.bfloat16, device=dev)
    from npu_offload_b200._lib import check, lib
    fn, h = lib().moe_block_forward, stack.plane.handle
    sp = ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)

    vp = ctypes.c_void_p
    ind = [[(l, vp(h2[r, l].data_ptr()), vp(x2[r, l].data_ptr()), vp(xn[l].data_ptr())) for l in range(L)]
           for r in range(R)]

    def one(s):
        for l, a, b, o in ind[s % R]:
            check(fn(h, l, T, a, b, None, o, None, None, 0, sp))

    # dependent chain: block l's x_next is block l+1's h2 and x2, as in the engine's layer loop
    # (main.rs:267-289, with attention left out), so the router logits of a layer exist only once
    # the previous layer is done
    xc = torch.empty(L + 1, T, H, dtype=torch.bfloat16, device=dev)
    chain = [(l, vp(xc[l].data_ptr()), vp(xc[l + 1].data_ptr())) for l in range(L)]

    def one_chain(s):
        xc[0].copy_(h2[s % R, 0])
        for l, a, o in chain:
            check(fn(h, l, T, a, a, None, o, None, None, 0, sp))

    def run(f):
        for s in range(warmup):
            f(s)
        torch.cuda.synchronize(dev)
        l0 = stack.plane.launch_count
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ev0.record()
        for s in range(steps):
            f(warmup + s)
        ev1.record()
        torch.cuda.synchronize(dev)
        return ev0.elapsed_time(ev1), stack.plane.launch_count - l0

    ms, nl = run(one)
    reps = [(warmup + s) % R for s in range(steps)]
    nbytes = sum(routed[r].sum() for r in reps) * EXPERT_BYTES + steps * L * (EXPERT_BYTES + E * H * 2)
    us_layer = ms * 1e3 / (steps * L)
    # the chain's routed experts are only known on the device: count them from one untimed pass
    routed_chain = []
    one_chain(0)
    torch.cuda.synchronize(dev)
    for l in range(L):
        lg = torch.empty(T, E, dtype=torch.float32, device=dev)
        check(lib().moe_shared_router(h, l, T, vp(xc[l].data_ptr()), None, None, vp(lg.data_ptr()), 0, sp))
        torch.cuda.synchronize(dev)
        top = np.argsort(-lg.cpu().numpy(), axis=1, kind="stable")[:, :K]
        routed_chain.append(len(set(top.ravel().tolist())))
    cms, cnl = run(one_chain)
    cbytes = steps * (sum(routed_chain) * EXPERT_BYTES + L * (EXPERT_BYTES + E * H * 2))
    return {"workload": f"moe_block_forward: router GEMV + routed experts + shared expert + residual combine, "
                        f"batch {T}, {L} layers",
            "us_per_layer": us_layer, "tokens_per_s": T * L * steps / (ms / 1e3),
            "bytes_per_layer": nbytes / (steps * L), "gbs": nbytes / (ms / 1e3) / 1e9,
            "gpu_launches_per_layer": nl / (steps * L),
            "chain": {"workload": "dependent chain: each block's x_next is the next block's h2 and x2 (its "
                                  "router logits exist only after the previous block)",
                      "us_per_layer": cms * 1e3 / (steps * L), "tokens_per_s": T * L * steps / (cms / 1e3),
                      "bytes_per_layer": cbytes / (steps * L), "gbs": cbytes / (cms / 1e3) / 1e9,
                      "frac": cbytes / (cms / 1e3) / 1e9 / peaks()[0],
                      "gpu_launches_per_layer": cnl / (steps * L)}}


Q8_BYTES = 3 * H * F + (2 * F + H) * 4  # one int8 weight-only expert: q tables + fp32 scales


def int8_run(stack, args, steps, warmup):
    """the stack's --int8-experts (96) least popular experts of every layer (by the Zipf rank of the layer's
    routing bias) re-stored int8 weight-only (quantised on the GPU with the reference's quant_row
    rule), the top 32 kept bf16; decode batch 1, the same Zipf-routed inputs.  Roofline bytes: the
    routed experts' stored bytes (bf16 31,457,280 B; int8 15,728,640 B of tables + 26,624 B of scales)."""
    import torch
    from npu_offload_b200 import synth
    L = stack.L
    cold = []
    for l in range(L):
        order = np.argsort(-synth.zipf_bias(args.seed + 31 * l, E), kind="stable")  # most popular first
        c = set(order[E - args.int8_experts:].tolist()) if args.int8_experts > 0 else set()
        for e in sorted(c):
            stack.plane.quantize_expert_q8(l, e)
        cold.append(c)
    stack.set_batch(1, args.seed)
    R = stack.R
    nbytes = np.zeros((R, L))
    n8 = np.zeros((R, L))
    for r in range(R):
        for l in range(L):
            _, idx, _ = stack.plane.forward(l, stack.x[r, l], stack.lg[r, l], out=stack.out[l], return_topk=True)
            ids = set(idx.cpu().numpy().ravel().tolist())
            n8[r, l] = sum(e in cold[l] for e in ids)
            nbytes[r, l] = n8[r, l] * Q8_BYTES + (len(ids) - n8[r, l]) * EXPERT_BYTES
    torch.cuda.synchronize(stack.device)
    ms, launches, _ = timed(stack, steps, warmup, 1)
    reps = [(warmup + s) % R for s in range(steps)]
    tot = sum(nbytes[r].sum() for r in reps)
    gbs = tot / (ms / 1e3) / 1e9
    peak = peaks()[0]
    return {"workload": f"configs[4]: {L}-layer stack, {args.int8_experts} least popular experts per layer int8 "
                        f"weight-only, top {E - args.int8_experts} bf16; decode batch 1, Zipf routing",
            "tokens_per_s": L * steps / (ms / 1e3), "us_per_layer": ms * 1e3 / (steps * L),
            "int8_experts_per_layer": float(n8.mean()), "bytes_per_layer": tot / (steps * L),
            "roofline": {"bound": "hbm", "kernel": "decode_kernel", "achieved": gbs, "peak": peak, "unit": "GB/s",
                         "frac": gbs / peak},
            "gpu_launches": launches}


def cold_run(args, device, L=2, steps=256, warmup=32):
    """HBM-hot / host-cold tier (solar_hybrid/runtime.py:287-311): `--cold-slots` HBM slots per layer, the other
    experts in pinned host memory, batch-1 decode with Zipf routing through ExpertCache (swap on miss
    plus the LFU-decay follow rule).  MoE-layer tokens/s over `steps` layer calls, wall clock (misses
    synchronise), with the hit rate and the swaps."""
    import torch
    from npu_offload_b200 import synth
    from npu_offload_b200.cache import ExpertCache
    from npu_offload_b200.moe import MoEDataPlane
    S = args.cold_slots
    gen = torch.Generator(device=device)
    host = []
    for l in range(L):
        row = []
        for e in range(E):
            gen.manual_seed(args.seed * 1_000_003 + 1009 * l + e)
            buf = (torch.randn(3 * F * H, generator=gen, device=device) * 0.02).to(torch.bfloat16).cpu().pin_memory()
            row.append((buf[:F * H].view(F, H), buf[F * H:2 * F * H].view(F, H), buf[2 * F * H:].view(H, F)))
        host.append(row)
    plane = MoEDataPlane(H, F, E, K, n_layers=L, max_tokens=16, device=device.index)
    prior = popularity_counts(args.seed, L)
    cache = ExpertCache(plane, host, S, prior=prior, swap_per_tok=1)
    x = torch.from_numpy(np.stack([synth.hidden(700 + i, 1, H) for i in range(64)]).view(np.int16)).view(
        torch.bfloat16).to(device)
    lg = torch.from_numpy(np.stack([synth.logits(700 + i, 1, E, zipf=False) + synth.zipf_bias(args.seed + 31 * (i % L), E)
                                    for i in range(64)]).astype(np.float32)).to(device)
    out = torch.empty(1, H, dtype=torch.float32, device=device)
    for i in range(warmup):
        cache.forward(i % L, x[i % 64], lg[i % 64], out=out)
    torch.cuda.synchronize(device)
    st0 = dict(cache.stats)
    t0 = time.perf_counter()
    for i in range(steps):
        cache.forward(i % L, x[i % 64], lg[i % 64], out=out)
    torch.cuda.synchronize(device)
    dt = time.perf_counter() - t0
    d = {k: cache.stats[k] - st0[k] for k in st0}
    n = d["hits"] + d["misses"]
    plane.close()
    return {"workload": f"{L} layers x {E} experts, {S} HBM slots per layer, the rest in pinned host memory; "
                        "batch 1, Zipf routing", "tokens_per_s": steps / dt, "us_per_layer": dt / steps * 1e6,
            "hit_rate": d["hits"] / n if n else None, "swaps_per_layer": (d["swaps"] + d["follow_swaps"]) / steps}


# ---------------------------------------------------------------- CPU baseline (reference / port)
def cpu_threads():
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count() or 1


def cpu_sample(stack_np, T, L, seed, budget_s, pool_src=None, steps=None):
    """Run the reference's CPU path (route on the host, then cpu_moe over the job list) for a bounded
    sample of the workload; expert weights come from a pool of 64 experts (2 GB, larger than any
    host LLC) as the reference's p0/cpu_microbench.py does.  Returns (tokens/s, info)."""
    from oracle.oracle import Port, Reference, cpu_model
    n = cpu_threads()
    use_ref = Reference.available()
    if use_ref:
        Reference.set_threads(n)
    else:
        Port.set_threads(n)
    P = 64
    pool = pool_src(P)
    xs, lgs = stack_np
    R = xs.shape[0]

    def layer(r, l):
        idx, w, _ = Port.route_softmax(lgs[r, l], K)
        pm = Port.permute(idx, E)
        toks, ws_, gus, ds, jobs = [], [], [], [], []
        for j, e in enumerate(pm["job_order"]):
            ps = pm["perm"][pm["offsets"][e]:pm["offsets"][e + 1]]
            toks.append((ps // K).astype(np.int64))
            ws_.append(w.reshape(-1)[ps].astype(np.float32))
            gu, d = pool[(int(e) + 17 * l) % P]
            gus.append(gu)
            ds.append(d)
            jobs.append(("bf16", gu, d))
        if use_ref:
            Reference.cpu_moe(xs[r, l], gus, ds, toks, ws_)
        else:
            Port.cpu_moe(xs[r, l], jobs, toks, ws_)

    layer(0, 0)  # warm-up
    t0 = time.perf_counter()
    done = 0
    s = 0
    while True:
        layer(s % R, s % L)
        done += 1
        s += 1
        el = time.perf_counter() - t0
        if (steps is None and el >= budget_s) or (steps is not None and done >= steps):
            break
    el = time.perf_counter() - t0
    info = {"kind": "reference" if use_ref else "port", "cores": n, "cpu": cpu_model(),
            "sample": f"{done} MoE-layer forwards at batch {T} (router + cpu_moe over the routed experts), "
                      f"experts drawn from a 64-expert / 2.0 GB pool, {el:.1f} s"}
    return T * done / el, info


def reference_arm(args):
    """The reference's CPU path on the host cores: one step = one MoE-layer forward at the same
    batch (cycling the stack's layers and input sets), K timed steps after W warm-up steps."""
    ws, rank, local = dist_env()
    if rank != 0:
        return 0
    L = args.layers or (8 if ws == 1 else 6 * ws)
    T = args.batch
    xs, lgs = make_inputs(args.seed, args.rotate, L, T)

    def pool(P):
        from npu_offload_b200 import synth
        out = []
        for e in range(P):
            g, u, d = synth.expert_weights(args.seed, 0, e, H, F)
            out.append((np.concatenate([g, u], 0), d))
        return out

    P = pool(64)
    cpu_sample((xs, lgs), T, L, args.seed, 0.0, pool_src=lambda n: P, steps=max(1, args.warmup))
    v, info = cpu_sample((xs, lgs), T, L, args.seed, 0.0, pool_src=lambda n: P, steps=max(1, args.steps))
    line = {"impl": "reference", "metric": METRIC, "value": v, "unit": UNIT, "n_gpus": ws, "steps": args.steps,
            "warmup": args.warmup, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "bf16", "data": "synthetic",
            "config": {"workload": (f"configs[1]: {L}-layer Solar-shaped MoE stack" if ws == 1 else
                                    f"configs[2] pro-rated: {L}-layer stack") + f", decode batch {T}, host CPU",
                       "layers": L, "batch": T, "hidden": H, "experts": E, "inter": F, "top_k": K,
                       "step": "one MoE-layer forward (router + cpu_moe) per step"},
            "cpu_baseline": dict(info, value=v, unit=UNIT),
            "e2e": {"value": v, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


# ---------------------------------------------------------------- our arm
def our_arm(args):
    import torch
    ws, rank, local = dist_env()
    if ws > 1:
        import datetime
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120))
    device = torch.device("cuda", local if ws > 1 else 0)
    torch.cuda.set_device(device)
    L = args.layers or (8 if ws == 1 else 6 * ws)
    T = args.batch
    stack = Stack(args, ws, rank, device, T, L)
    peak, peak_kind = peaks()

    with ClockSampler(device.index) as clk:
        ms, launches, _ = timed(stack, args.steps, args.warmup, ws, profile=False)
    ms_max = max_over_ranks(ms, ws)
    step_ms = ms_max / args.steps
    value = T * L * args.steps / (ms_max / 1e3)

    # Roofline of the dominant kernel (decode_kernel, one launch per layer): algorithmic bytes per
    # launch = this rank's distinct routed experts x their gate/up/down bytes; launch duration = the
    # timed region / decode launches (back-to-back launches overlap their start-up with the previous
    # grid's tail through programmatic dependent launch; events between launches would break that).
    R = stack.R
    reps = [(args.warmup + s) % R for s in range(args.steps)]
    n_dec = args.steps * L
    all_bytes = sum(stack.ucount[r].sum() for r in reps) * stack.ebytes
    bpl = all_bytes / n_dec
    dur_s = ms / 1e3 / n_dec
    achieved = bpl / dur_s / 1e9
    roof = {"bound": "hbm", "kernel": "decode_kernel", "achieved": achieved, "peak": peak, "unit": "GB/s",
            "frac": achieved / peak, "peak_source": f"{peak_kind} hbm_gbs",
            "traffic": TRAFFIC_RATIO * bpl if TRAFFIC_RATIO else None,
            "traffic_source": TRAFFIC_SOURCE if TRAFFIC_RATIO else None,
            "algorithmic_bytes_per_launch": bpl, "launch_us": dur_s * 1e6,
            "timed_region": "the K timed steps; per-launch duration = timed region / decode launches"}

    e2e = None
    if not args.no_e2e:
        ev, h2d, d2h = e2e_run(stack, max(1, args.steps // 4), min(args.warmup, 3), ws)
        e2e = {"value": ev, "unit": UNIT, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h}

    ucount_main, ubytes_main = stack.ucount.copy(), stack.ubytes.copy()
    sweep = []
    for tb in [int(v) for v in args.sweep.split(",") if v.strip()]:
        if tb == T:
            continue
        stack.set_batch(tb, args.seed)
        ks = max(1, args.steps // 4)
        sms, _, _ = timed(stack, ks, min(args.warmup, 3), ws, profile=False)
        sms = max_over_ranks(sms, ws)
        reps = [(min(args.warmup, 3) + s) % R for s in range(ks)]
        ub = sum(stack.ucount[r].sum() for r in reps) * stack.ebytes
        sweep.append({"batch": tb, "value": tb * L * ks / (sms / 1e3), "layer_gbs": ub / (sms / 1e3) / 1e9,
                      "experts_per_layer": float(np.mean([stack.ucount[r].mean() for r in reps]))})
    launches_all = int(sum_over_ranks(launches, ws))
    prefill = None
    if args.prefill_tokens > 0:
        prefill = prefill_run(stack, args.prefill_tokens, ws=ws)
    block = None
    if ws == 1 and not args.no_block:
        block = block_run(stack, max(1, args.steps // 4), min(args.warmup, 3))
    cold = None
    if ws == 1 and args.cold_slots > 0:
        cold = cold_run(args, device)
    int8 = None
    if ws == 1 and not args.no_int8:  # last: it re-stores most of the stack's experts as int8
        int8 = int8_run(stack, args, max(1, args.steps // 4), min(args.warmup, 3))

    alt = None
    if ws > 1 and stack.shard == "units" and not args.no_alt_split:
        # configs[2]'s own split beside the default one, same build and run: each rank owns 16 experts
        # per layer (at N = 8) by the popularity stripe of the placement plan.  The unit-sharded stack
        # is released first (after every rank is done with its peers' buffers).
        barrier(ws)
        stack.plane.close()
        alt_args = argparse.Namespace(**vars(args))
        alt_args.ep_shard = "experts"
        astack = Stack(alt_args, ws, rank, device, 1, L)
        ks = max(1, args.steps // 4)
        ams, _, _ = timed(astack, ks, min(args.warmup, 3), ws, profile=False)
        ams = max_over_ranks(ams, ws)
        busiest = max_over_ranks(float(np.max(astack.ucount)), ws)
        alt = {"ep_shard": "experts: popularity stripe (configs[2]: 16 experts per GPU per layer at N = 8)",
               "batch": 1, "value": L * ks / (ams / 1e3), "us_per_layer": ams * 1e3 / (ks * L),
               "routed_experts_busiest_rank_max": busiest}
        barrier(ws)
        stack = astack  # closed below like the main stack

    cpu = None
    if rank == 0 and ws == 1 and not args.no_cpu_baseline:
        def pool(P):
            W = []
            gen = torch.Generator(device=device)
            for e in range(P):
                gen.manual_seed(args.seed * 7 + e)
                buf = (torch.randn(3 * F * H, generator=gen, device=device) * 0.02).to(torch.bfloat16)
                a = buf.view(torch.int16).cpu().numpy().view(np.uint16)
                W.append((a[:2 * F * H].reshape(2 * F, H), a[2 * F * H:].reshape(H, F)))
            return W
        try:
            xs, lgs = make_inputs(args.seed, stack.R, L, T)
            v, info = cpu_sample((xs, lgs), T, L, args.seed, args.cpu_seconds, pool_src=pool)
            cpu = dict(info, value=v, unit=UNIT)
        except Exception as ex:  # the baseline is reported, never required
            cpu = {"value": None, "unit": UNIT, "error": str(ex)[:200]}

    if rank == 0:
        line = {"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": ws, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": step_ms, "higher_is_better": True, "scaling": "weak",
                "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
                "config": {"workload": (f"configs[1]: {L}-layer Solar-shaped MoE stack on 1 GPU" if ws == 1 else
                                        f"configs[2] pro-rated: {L}-layer stack, expert-parallel over {ws} GPUs"),
                           "layers": L, "batch": T, "hidden": H, "experts": E, "inter": F, "top_k": K,
                           "weights_gb": round(L * E * EXPERT_BYTES / 1e9, 1),
                           "parallelism": f"ep{ws}" if ws > 1 else "single",
                           "combine": ("in-kernel NVLink peer exchange" if args.ep == "p2p" else "NCCL all-reduce")
                                      if ws > 1 else None,
                           "ep_shard": (f"units: each GPU {stack.units[1] - stack.units[0]} of {F} units of every "
                                        "expert" if stack.shard == "units" else "experts: popularity stripe")
                                       if ws > 1 else None,
                           "l2": "no flush: each step streams its routed experts (~%.1f GB/step/GPU) >> 126 MB L2"
                                 % (ubytes_main.mean() * L / 1e9),
                           "experts_per_layer": float(ucount_main.mean())},
                "roofline": roof, "e2e": e2e, "gpu_launches": launches_all,
                "clocks": clk.summary(), "cpu_baseline": cpu, "sweep": sweep, "prefill": prefill,
                "block": block, "cold": cold, "int8": int8, "alt_split": alt}
        print(json.dumps(line), flush=True)
    if ws > 1:
        barrier(ws)  # no rank frees its exchange buffer while a peer may still use it
    stack.plane.close()
    if ws > 1:
        import torch.distributed as dist
        dist.barrier()
        dist.destroy_process_group()
    return 0


def main():
    args = parse()
    if args.impl == "reference":
        return reference_arm(args)
    return our_arm(args)


if __name__ == "__main__":
    sys.exit(main())
