// Tensor-core (tcgen05) prefill kernels: launch interface.
#pragma once
#include <cstddef>
#include <cstdint>
#include <cuda_runtime.h>

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
cudaError_t launch_gateup_tc(const uint16_t* xg, int xrows, const void* arena, int n_slots, size_t slot_bytes,
                             const TcItem* items, int n_items, int H, int F, uint16_t* act, uint32_t* sched,
                             uint32_t* err, uint64_t timeout_ns, int grid_max, cudaStream_t st);

// y[p, h] (fp32) for every item (TcItem.f0 = first output h, 256 per tile).  act: [arows][F] bf16
// activation rows; arena as above.  H % 256 == 0, F % 64 == 0.
cudaError_t launch_down_tc(const uint16_t* act, int arows, const void* arena, int n_slots, size_t slot_bytes,
                           const TcItem* items, int n_items, int H, int F, float* y, uint32_t* sched, uint32_t* err,
                           uint64_t timeout_ns, int grid_max, cudaStream_t st);

}  // namespace moe
