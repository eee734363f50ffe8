// Launch interface of the block-level kernels (block.cu): router GEMV and the residual steps.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

namespace moe {

// logits [T, E] fp32 = x [T, H] bf16 . wr [E, H]^T.  H % 8 == 0, 16-byte aligned operands.
cudaError_t launch_router_gemv(const uint16_t* wr, const uint16_t* x, int T, int E, int H, float* logits,
                               cudaStream_t st);

// Over n elements (n % 8 == 0, 16-byte aligned): y = y_in, or bf16(x2 + shared) when y_in is null
// (stored to y_out when set); x_next = bf16((y + extra) + moe) when x_next is set (extra nullable).
cudaError_t launch_residual(const uint16_t* y_in, const uint16_t* x2, const float* shared, const float* extra,
                            const float* moe, long n, uint16_t* y_out, uint16_t* x_next, int sm_count, cudaStream_t st);

}  // namespace moe
