"""Expert parallelism across the GPUs of one box (one process per GPU, torch.distributed).

Two ways to split the experts: by expert (``shard_map``: each rank owns whole experts) or by unit
(``unit_ranges``: each rank owns the same slice of the intermediate units of every expert; the
context of rank r is then created with ``inter = f1 - f0`` and owns all experts).

The shard map is npu-offload's placement plan turned into ownership: experts are ranked by
popularity (profile counts, moe_offload/placement.py:15-16 ``ranks``) and dealt round-robin to the
ranks (the alternating assignment of solar_hybrid/runtime.py:522-533), so every rank gets a
balanced mix of hot and cold experts.  ``top`` (contiguous rank blocks, placement.py:22-24) is
available for comparison.

Per layer every rank routes the same tokens (identical inputs give bit-identical top-k on every
rank), runs its local experts and produces a partial [T,H] fp32 sum; one exchange completes the
combine.  With ``attach_peers`` the exchange happens inside the decode kernel over NVLink peer
memory (every rank ends with the full output); otherwise ``allreduce_partial`` (NCCL) sums the
partials.
"""
import numpy as np


def ranks_by_count(counts):
    """Experts ordered hottest first; ties to the lower id (moe_offload/placement.py:15-16)."""
    counts = np.asarray(counts)
    return sorted(range(len(counts)), key=lambda e: (-counts[e], e))


def shard_map(counts_per_layer, world, policy="stripe"):
    """[layers][E] owner rank for each expert.

    stripe: popularity rank r goes to rank r % world (balanced hot/cold mix per rank).
    top:    ranks take contiguous popularity blocks of E/world experts (placement.py "top")."""
    counts_per_layer = np.asarray(counts_per_layer)
    L, E = counts_per_layer.shape
    out = np.zeros((L, E), np.int32)
    per = -(-E // world)
    for l in range(L):
        order = ranks_by_count(counts_per_layer[l])
        for r, e in enumerate(order):
            out[l, e] = r % world if policy == "stripe" else min(r // per, world - 1)
    return out


def unit_ranges(F, world, align=64):
    """Unit sharding: rank r owns units [f0, f1) of EVERY expert (gate rows, up rows and down columns
    f0..f1), contiguous multiples of `align`, as even as possible.  A unit's activation needs only
    its own gate and up rows, and its down column adds into all H outputs, so the per-rank partial
    sums add up to the full expert output.  Every rank then streams the same share of each routed
    expert, however the router skews the expert choice."""
    chunks = F // align
    if F % align or chunks < world:
        raise ValueError(f"F={F} does not split into {world} shares of {align}-unit multiples")
    base, extra = divmod(chunks, world)
    out, f = [], 0
    for r in range(world):
        n = (base + (1 if r < extra else 0)) * align
        out.append((f, f + n))
        f += n
    return out


def unit_slice(gate, up, down, f0, f1):
    """This rank's part of one expert under unit sharding: gate/up rows and down columns f0..f1."""
    return gate[f0:f1], up[f0:f1], down[:, f0:f1]


def local_experts(smap, layer, rank):
    return [int(e) for e in np.nonzero(np.asarray(smap)[layer] == rank)[0]]


def attach_peers(plane, group=None):
    """Collective: map every rank's exchange buffer into this rank's context (CUDA IPC handles
    all-gathered over the process group).  Afterwards plane.forward returns the full output."""
    import torch.distributed as dist
    mine = plane.ep_export()
    recs = [None] * dist.get_world_size(group)
    dist.all_gather_object(recs, mine, group=group)
    plane.ep_import(b"".join(recs))
    dist.barrier(group)


def allreduce_partial(out, group=None):
    """Sum the per-rank partial outputs in place (NCCL over NVLink when the group is NCCL)."""
    import torch.distributed as dist
    dist.all_reduce(out, op=dist.ReduceOp.SUM, group=group)
    return out
