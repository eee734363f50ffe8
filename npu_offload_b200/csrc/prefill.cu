// Prefill (many tokens per expert) for the B200 MoE data plane: the expert FFN as grouped dense GEMMs.
//
// Semantics as the decode path (solar_hybrid/cpu_moe.cpp:38-96): g, u = gate/up rows . x_t,
// act = bf16_rne(g / (1 + exp(-g)) * u), y = down . act, out[t] = sum of w * y over the token's
// experts in job order.  The two contractions run on the tcgen05 tensor cores (prefill_tc.cu: bf16
// operands, fp32 accumulation, g, u and y kept in fp32, SwiGLU fused), reading the context's unit
// tables in place.  The kernels here supply the token gather and the weighted combine (fp32).
#include <algorithm>

#include "common.cuh"
#include "experts.h"

namespace moe {

// xg[p, :] = x[ptok[p], :] for the n pairs of the local jobs (job-major): 16-byte vectors.  n_dev
// (nullable) holds n in device memory (job list built on the device).
__global__ void __launch_bounds__(256) gather_rows_kernel(const uint16_t* x, const int32_t* ptok, int n,
                                                          const int* n_dev, int H, uint16_t* xg) {
    if (n_dev) n = min(n, *n_dev);
    const int per = H / 8;
    const long total = (long)n * per;
    for (long i = blockIdx.x * 256L + threadIdx.x; i < total; i += (long)gridDim.x * 256) {
        const int p = (int)(i / per), c = (int)(i % per);
        reinterpret_cast<uint4*>(xg + (size_t)p * H)[c] = __ldg(reinterpret_cast<const uint4*>(x + (size_t)ptok[p] * H) + c);
    }
}

// out[t, h] = (accumulate ? out : 0) + sum over the token's pairs (comb lists, job order) of
// w[p] * y[p, h]; y is the down GEMM's fp32 output.
__device__ __forceinline__ void load8(const float* y, float v[8]) {
    const float4 a = reinterpret_cast<const float4*>(y)[0], b = reinterpret_cast<const float4*>(y)[1];
    v[0] = a.x, v[1] = a.y, v[2] = a.z, v[3] = a.w, v[4] = b.x, v[5] = b.y, v[6] = b.z, v[7] = b.w;
}

__global__ void __launch_bounds__(256) combine_rows_kernel(const float* y, const float* w, const int32_t* comb_off,
                                                           const int32_t* comb_p, int H, int accumulate, float* out) {
    const int t = blockIdx.y;
    const int h = (blockIdx.x * 256 + threadIdx.x) * 8;
    if (h >= H) return;
    float acc[8];
    float* o = out + (size_t)t * H + h;
#pragma unroll
    for (int k = 0; k < 8; k++) acc[k] = accumulate ? o[k] : 0.f;
    for (int i = comb_off[t]; i < comb_off[t + 1]; i++) {
        const int p = comb_p[i];
        if (p < 0) continue;
        const float wp = w[p];
        float v[8];
        load8(y + (size_t)p * H + h, v);
#pragma unroll
        for (int k = 0; k < 8; k++) acc[k] = fmaf(wp, v[k], acc[k]);
    }
    reinterpret_cast<float4*>(o)[0] = make_float4(acc[0], acc[1], acc[2], acc[3]);
    reinterpret_cast<float4*>(o)[1] = make_float4(acc[4], acc[5], acc[6], acc[7]);
}

cudaError_t launch_combine_rows(const float* y, const float* w, const int32_t* comb_off, const int32_t* comb_p, int T,
                                int H, int accumulate, float* out, cudaStream_t st) {
    if (T <= 0) return cudaSuccess;
    dim3 g((H / 8 + 255) / 256, T);
    combine_rows_kernel<<<g, 256, 0, st>>>(y, w, comb_off, comb_p, H, accumulate, out);
    return cudaGetLastError();
}

cudaError_t launch_gather_rows(const uint16_t* x, const int32_t* ptok, int n, int H, uint16_t* xg, int sm_count,
                               cudaStream_t st, const int* n_dev) {
    if (n <= 0) return cudaSuccess;
    const long total = (long)n * (H / 8);
    const int grid = (int)std::min<long>((total + 255) / 256, (long)sm_count * 16);
    gather_rows_kernel<<<grid, 256, 0, st>>>(x, ptok, n, n_dev, H, xg);
    return cudaGetLastError();
}

}  // namespace moe
