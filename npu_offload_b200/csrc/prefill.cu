// Prefill (many tokens per expert) for the B200 MoE data plane: the expert FFN as grouped dense GEMMs.
//
// Semantics as the decode path (solar_hybrid/cpu_moe.cpp:38-96): g, u = gate/up rows . x_t,
// act = bf16_rne(g / (1 + exp(-g)) * u), y = down . act, out[t] = sum of w * y over the token's
// experts in job order.  The two contractions run on the tensor cores (bf16 operands, fp32
// accumulation), reading the context's unit tables in place: either the tcgen05 kernels of
// prefill_tc.cu (g, u and y stay fp32, SwiGLU fused) or the library grouped GEMM, whose interface
// returns bf16, so there g, u and y are rounded to bf16 once at the GEMM outputs.  The kernels here
// supply the token gather, the library path's SwiGLU and the weighted combine (fp32).
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

// act[i] = bf16_rne(g[i] / (1 + exp(-g[i])) * u[i]) over n * F values (cpu_moe.cpp:70-77); g and u
// arrive as bf16 GEMM outputs (fp32 accumulation, one rounding).
__global__ void __launch_bounds__(256) swiglu_rows_kernel(const uint16_t* g, const uint16_t* u, long count,
                                                          uint16_t* act) {
    for (long i = (blockIdx.x * 256L + threadIdx.x) * 8; i < count; i += (long)gridDim.x * 256 * 8) {
        const uint4 gv = *reinterpret_cast<const uint4*>(g + i);
        const uint4 uv = *reinterpret_cast<const uint4*>(u + i);
        const uint32_t gw[4] = {gv.x, gv.y, gv.z, gv.w}, uw[4] = {uv.x, uv.y, uv.z, uv.w};
        uint32_t o[4];
#pragma unroll
        for (int k = 0; k < 4; k++)
            o[k] = (uint32_t)swiglu_bf16(bf_lo(gw[k]), bf_lo(uw[k])) |
                   ((uint32_t)swiglu_bf16(bf_hi(gw[k]), bf_hi(uw[k])) << 16);
        *reinterpret_cast<uint4*>(act + i) = make_uint4(o[0], o[1], o[2], o[3]);
    }
}

// out[t, h] = (accumulate ? out : 0) + sum over the token's pairs (comb lists, job order) of
// w[p] * y[p, h]; y is the down GEMM's output, fp32 (tensor-core kernels) or bf16 (library GEMM).
__device__ __forceinline__ void load8(const float* y, float v[8]) {
    const float4 a = reinterpret_cast<const float4*>(y)[0], b = reinterpret_cast<const float4*>(y)[1];
    v[0] = a.x, v[1] = a.y, v[2] = a.z, v[3] = a.w, v[4] = b.x, v[5] = b.y, v[6] = b.z, v[7] = b.w;
}
__device__ __forceinline__ void load8(const uint16_t* y, float v[8]) {
    const uint4 q = *reinterpret_cast<const uint4*>(y);
    const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
    for (int k = 0; k < 4; k++) v[2 * k] = bf_lo(w[k]), v[2 * k + 1] = bf_hi(w[k]);
}

template <typename Y>
__global__ void __launch_bounds__(256) combine_rows_kernel(const Y* y, const float* w, const int32_t* comb_off,
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

template <typename Y>
static cudaError_t launch_combine_y(const Y* y, const float* w, const int32_t* comb_off, const int32_t* comb_p, int T,
                                   int H, int accumulate, float* out, cudaStream_t st) {
    if (T <= 0) return cudaSuccess;
    dim3 g((H / 8 + 255) / 256, T);
    combine_rows_kernel<Y><<<g, 256, 0, st>>>(y, w, comb_off, comb_p, H, accumulate, out);
    return cudaGetLastError();
}

cudaError_t launch_combine_bf16(const uint16_t* y, const float* w, const int32_t* comb_off, const int32_t* comb_p,
                                int T, int H, int accumulate, float* out, cudaStream_t st) {
    return launch_combine_y(y, w, comb_off, comb_p, T, H, accumulate, out, st);
}

cudaError_t launch_combine_rows(const float* y, const float* w, const int32_t* comb_off, const int32_t* comb_p, int T,
                                int H, int accumulate, float* out, cudaStream_t st) {
    return launch_combine_y(y, w, comb_off, comb_p, T, H, accumulate, out, st);
}

cudaError_t launch_gather_rows(const uint16_t* x, const int32_t* ptok, int n, int H, uint16_t* xg, int sm_count,
                               cudaStream_t st, const int* n_dev) {
    if (n <= 0) return cudaSuccess;
    const long total = (long)n * (H / 8);
    const int grid = (int)std::min<long>((total + 255) / 256, (long)sm_count * 16);
    gather_rows_kernel<<<grid, 256, 0, st>>>(x, ptok, n, n_dev, H, xg);
    return cudaGetLastError();
}

cudaError_t launch_swiglu_rows(const uint16_t* g, const uint16_t* u, long count, uint16_t* act, int sm_count,
                               cudaStream_t st) {
    if (count <= 0) return cudaSuccess;
    const int grid = (int)std::min<long>((count / 8 + 255) / 256, (long)sm_count * 16);
    swiglu_rows_kernel<<<grid, 256, 0, st>>>(g, u, count, act);
    return cudaGetLastError();
}

}  // namespace moe
