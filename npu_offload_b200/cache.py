"""HBM-hot / host-cold expert tier for models whose experts do not all fit in HBM.

The reference keeps a fixed number of expert slots per layer on the accelerator and the rest in host
DRAM (moe_offload/budget.py:32-52 sizes the slots), and moves experts between them with an LFU-decay
policy (`Runtime.follow`, solar_hybrid/runtime.py:287-311: recent-use counts halved every 128 decode
tokens; swap the hottest non-resident expert in for the coldest resident one when it is used at least
twice as often plus 2) by overwriting a device table slot in place (experts_b.rs:162-186
`swap_slot`).  There, a token routed to a non-resident expert runs on the CPU.

On B200 every routed expert runs on the GPU: a call that routes to a non-resident expert first
brings it into a slot (host -> HBM copy of its 3.F.H bf16, then the unit-table layout), evicting the
resident expert with the lowest decayed count that the call does not need.  `follow` additionally
swaps ahead of need, with the reference's rule, so that a hot expert is resident before it is routed.
"""
import ctypes

import numpy as np

SWAP_HALF = 128  # halve the recent-use counts every this many decode tokens (runtime.py:278)
SWAP_MIN = 2     # follow(): swap when in.recent >= 2 * out.recent + SWAP_MIN (runtime.py:279)


def choose_victim(recent, resident, need):
    """The resident expert to evict: lowest decayed count among those this call does not need
    (ties to the lower id); None if every resident expert is needed."""
    cands = [e for e in resident if e not in need]
    if not cands:
        return None
    return min(cands, key=lambda e: (float(recent[e]), e))


def follow_candidate(recent, resident, E):
    """(e_in, e_out) the follow rule swaps, or None: the hottest non-resident expert among the 8
    hottest, against the coldest resident one (runtime.py:297-306); ties to the lower id."""
    recent = np.asarray(recent, np.float64)
    if not resident:
        return None
    res = np.zeros(E, bool)
    res[list(resident)] = True
    order = np.argsort(-recent, kind="stable")[:8]
    nonres = [int(e) for e in order if not res[e] and recent[e] > 0]
    if not nonres:
        return None
    e_in = nonres[0]
    ridx = np.flatnonzero(res)
    e_out = int(ridx[np.argmin(recent[ridx])])
    if recent[e_in] >= 2 * recent[e_out] + SWAP_MIN:
        return e_in, e_out
    return None


class ExpertCache:
    """Routed-expert forward over `slots` HBM expert slots per layer, the other experts in host memory.

    plane: a MoEDataPlane with no expert loaded yet (the cache sets MOE_OPT_LAYER_SLOTS).
    host_weights[l][e] = (gate [F,H], up [F,H], down [H,F]) bf16 CPU tensors (pinned for fast swaps).
    prior[l] (optional): expert popularity, the `slots` most popular are loaded first.
    bias[l] (optional): sigmoid-scoring bias of layer l (the same as the plane's)."""

    def __init__(self, plane, host_weights, slots, prior=None, bias=None, swap_per_tok=0):
        import torch
        from ._lib import MOE_OPT_LAYER_SLOTS
        self.torch = torch
        self.plane = plane
        self.L, self.E, self.K = plane.L, plane.E, plane.K
        if not 0 < slots <= self.E:
            raise ValueError(f"slots {slots} not in [1, {self.E}]")
        self.slots = slots
        self.host = [[tuple(t if t.is_pinned() else t.pin_memory() for t in host_weights[l][e])
                      for e in range(self.E)] for l in range(self.L)]
        self.bias = bias
        self.swap_per_tok = swap_per_tok
        plane.set_option(MOE_OPT_LAYER_SLOTS, slots)
        self.recent = np.zeros((self.L, self.E), np.float64)
        self.resident = [set() for _ in range(self.L)]
        for l in range(self.L):
            first = (sorted(range(self.E), key=lambda e: (-float(prior[l][e]), e)) if prior is not None
                     else list(range(self.E)))[:slots]
            for e in first:
                self._load(l, e)
        self.tokens = 0
        self.stats = dict(hits=0, misses=0, swaps=0, follow_swaps=0)
        n = plane.max_tokens * self.K
        self._idx_dev = torch.empty(n, dtype=torch.int32, device=plane.device)
        self._idx_host = torch.empty(n, dtype=torch.int32).pin_memory()

    def _route(self, logits, bias):
        """Top-k expert ids of the call (the library's router on the GPU, one synchronisation)."""
        from ._lib import check, lib
        torch = self.torch
        lg = logits.to(torch.float32).contiguous()
        T = lg.shape[0]
        n = T * self.K
        b = None if bias is None else torch.as_tensor(bias, dtype=torch.float32, device=lg.device).contiguous()
        stream = torch.cuda.current_stream(self.plane.device)
        vp = lambda t: None if t is None else ctypes.c_void_p(t.data_ptr())
        check(lib().moe_route(self.plane.handle, T, vp(lg), vp(b), vp(self._idx_dev), None, None, None, None, None,
                              None, 0, ctypes.c_void_p(stream.cuda_stream)))
        self._idx_host[:n].copy_(self._idx_dev[:n], non_blocking=True)
        stream.synchronize()
        return self._idx_host[:n].numpy().reshape(T, self.K)

    def _load(self, l, e):
        self.plane.load_expert(l, e, *self.host[l][e])
        self.resident[l].add(e)

    def _swap(self, l, e_in, e_out):
        self.plane.evict_expert(l, e_out)
        self.resident[l].discard(e_out)
        self._load(l, e_in)

    def forward(self, layer, hidden, logits, out=None):
        """moe_forward of one layer (device tensors), after making every routed expert resident."""
        torch = self.torch
        b = None if self.bias is None else self.bias[layer]
        idx = self._route(logits, b)
        need = set(int(e) for e in np.unique(idx))
        if len(need) > self.slots:
            raise ValueError(f"layer {layer}: {len(need)} distinct experts routed, only {self.slots} slots")
        np.add.at(self.recent[layer], idx.ravel(), 1.0)
        miss = sorted(need - self.resident[layer])
        self.stats["hits"] += len(need) - len(miss)
        self.stats["misses"] += len(miss)
        if miss:
            torch.cuda.synchronize(self.plane.device)  # no earlier call of this layer still reads a slot
            for e in miss:
                if len(self.resident[layer]) < self.slots:
                    self._load(layer, e)
                    continue
                self._swap(layer, e, choose_victim(self.recent[layer], self.resident[layer], need))
                self.stats["swaps"] += 1
        out = self.plane.forward(layer, hidden, logits, out=out)
        T = int(idx.shape[0])
        for _ in range(T):
            self.tokens += 1
            if self.tokens % SWAP_HALF == 0:
                self.recent *= 0.5
        if self.swap_per_tok:
            self.follow(self.swap_per_tok)
        return out

    def follow(self, max_swaps=1):
        """The reference's follow rule across layers: at most max_swaps swaps, largest gain first."""
        cands = []
        for l in range(self.L):
            c = follow_candidate(self.recent[l], self.resident[l], self.E)
            if c is not None:
                cands.append((float(self.recent[l][c[0]] - self.recent[l][c[1]]), l, c[0], c[1]))
        cands.sort(reverse=True)
        if cands[:max_swaps]:
            self.torch.cuda.synchronize(self.plane.device)
        for _, l, e_in, e_out in cands[:max_swaps]:
            self._swap(l, e_in, e_out)
            self.stats["follow_swaps"] += 1

    def hit_rate(self):
        n = self.stats["hits"] + self.stats["misses"]
        return self.stats["hits"] / n if n else 0.0
