// Tensor-core (tcgen05) prefill kernels: launch interface.
#pragma once
#include <cstddef>
#include <cstdint>
#include <cuda_runtime.h>

#include "common.cuh"

namespace moe {

// One output tile: gathered rows [row0, row0 + rows) (<= 256) of one job, whose expert sits in arena
// slot `slot`; f0 = the first of 128 intermediate indices (gate/up) or of 256 outputs h (down).
struct TcItem {
    int32_t row0, rows, slot, f0;
};

bool tc_available();  // the driver's tensor-map encoder is reachable
cudaError_t tc_set_smem_limit();

// act[p, f] for every item (fused SwiGLU, bf16).  xg: gathered token rows [xrows][H] bf16; arena: the
// layer's unit tables (n_slots slots of slot_bytes).  H % 64 == 0, F % 128 == 0.
// Both kernels are persistent: min(n_items, grid_max) CTAs (one per SM) take items from the
// schedule counter pair `sched` (2 device words, zero before the first launch; every launch leaves
// them zero).  Launches sharing a counter pair must be stream-ordered.
// n_items_dev (nullable): the item count in device memory (a tile list built on the device); the
// grid is then grid_max CTAs and n_items is ignored.
// mt_done (nullable): per-m-tile counters (zeroed by launch_tc_items); with them the gate/up grid
// counts each m-tile's stored activation rows and lets the down grid launched right after it start
// early (launch_down_tc with the same counters), so the down GEMM fills the gate/up tail.
cudaError_t launch_gateup_tc(const uint16_t* xg, int xrows, const void* arena, int n_slots, size_t slot_bytes,
                             const TcItem* items, int n_items, const int* n_items_dev, int H, int F, uint16_t* act,
                             uint32_t* sched, uint32_t* err, uint64_t timeout_ns, int grid_max, uint32_t* mt_done,
                             cudaStream_t st);

// y[p, h] (fp32) for every item (TcItem.f0 = first output h, 256 per tile).  act: [arows][F] bf16
// activation rows; arena as above.  H % 256 == 0, F % 64 == 0.
cudaError_t launch_down_tc(const uint16_t* act, int arows, const void* arena, int n_slots, size_t slot_bytes,
                           const TcItem* items, int n_items, const int* n_items_dev, int H, int F, float* y,
                           uint32_t* sched, uint32_t* err, uint64_t timeout_ns, int grid_max, uint32_t* mt_done,
                           cudaStream_t st);

// Both tile lists from the permutation's local job list (jobs[0 .. *n_jobs)), heaviest job first:
// gate/up items into gu[cap_gu], down items into dn[cap_dn]; cnt[0], cnt[1] = their counts,
// cnt[2] = local pairs.  One CTA; E <= 256.
cudaError_t launch_tc_items(const Job* jobs, const int* n_jobs, int E, const void* arena, size_t stride, int F, int H,
                            TcItem* gu, int cap_gu, TcItem* dn, int cap_dn, int* cnt, uint32_t* err, uint32_t* mt_done,
                            cudaStream_t st);

}  // namespace moe
