// The calls on either side of the routed-expert path, for one MoE block of the Solar engine
// (track2_opt/solar_engine/src/layer.rs:1-6):
//   router-logit producer   logits[t, e] = h2_t . Wr[e]  (fp32 accumulate; dense/shared.rs:1-3)
//   shared-expert residual  y = bf16(x2 + shared(h2))    (fp32 add, one rounding; shared.rs:2)
//   residual combine        x_next = bf16((y + extra) + moe_out)  (fp32, one rounding; combine.rs:1)
// The shared expert itself runs through the routed-expert machinery (a one-expert context whose
// router always gives weight 1), so only the GEMV and the element-wise steps live here.
#include <algorithm>

#include "block.h"
#include "common.cuh"
#include "ptx.cuh"

namespace moe {

constexpr int kRtThreads = 256;  // one CTA per (expert, tile of kRtTok tokens)
constexpr int kRtTok = 16;

// logits[t, e] = x[t] . wr[e] in fp32.  Latency-bound (1 MB of router weights for the Solar shape),
// so every thread issues all its loads at once: thread i covers 16-byte chunks i, i + 256, ... of
// the row, then the CTA sums the per-thread dot products (warp shuffles, then the 8 warps in order).
// Launched with programmatic dependent launch: the CTAs take SMs as the previous grid frees them and
// wait for its completion (x may be its output) before reading; they never trigger their dependents
// early, so a dependent kernel starts only once the logits are written.
__global__ void __launch_bounds__(kRtThreads) router_gemv_kernel(const uint16_t* __restrict__ wr,
                                                               const uint16_t* __restrict__ x, int T, int E, int H,
                                                               float* __restrict__ logits) {
    __shared__ float part[kRtThreads / 32][kRtTok];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int e = blockIdx.x, t0 = blockIdx.y * kRtTok, nt = min(kRtTok, T - t0);
    griddep_wait();
    float acc[kRtTok];
#pragma unroll
    for (int t = 0; t < kRtTok; t++) acc[t] = 0.f;
    const uint4* w4 = reinterpret_cast<const uint4*>(wr + (size_t)e * H);
    const uint4* x4 = reinterpret_cast<const uint4*>(x + (size_t)t0 * H);
    const int n8 = H / 8;
#pragma unroll 2
    for (int c = tid; c < n8; c += kRtThreads) {
        const uint4 wv = __ldg(w4 + c);
        uint4 xv[kRtTok];
#pragma unroll
        for (int t = 0; t < kRtTok; t++)
            if (t < nt) xv[t] = __ldg(x4 + (size_t)t * n8 + c);
        const uint32_t ww[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
        for (int t = 0; t < kRtTok; t++)
            if (t < nt) {
                const uint32_t xw[4] = {xv[t].x, xv[t].y, xv[t].z, xv[t].w};
#pragma unroll
                for (int k = 0; k < 4; k++) {
                    acc[t] = fmaf(bf_lo(ww[k]), bf_lo(xw[k]), acc[t]);
                    acc[t] = fmaf(bf_hi(ww[k]), bf_hi(xw[k]), acc[t]);
                }
            }
    }
#pragma unroll
    for (int t = 0; t < kRtTok; t++) {
        if (t < nt) {
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) acc[t] += __shfl_xor_sync(0xffffffffu, acc[t], o);
            if (lane == 0) part[warp][t] = acc[t];
        }
    }
    __syncthreads();
    if (tid < nt) {
        float v = 0.f;
#pragma unroll
        for (int w = 0; w < kRtThreads / 32; w++) v += part[w][tid];
        logits[(size_t)(t0 + tid) * E + e] = v;
    }
}

cudaError_t launch_router_gemv(const uint16_t* wr, const uint16_t* x, int T, int E, int H, float* logits,
                               cudaStream_t st) {
    if (T <= 0) return cudaSuccess;
    if (H % 8 || ((uintptr_t)wr | (uintptr_t)x) & 15) return cudaErrorInvalidValue;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(E, (T + kRtTok - 1) / kRtTok);
    cfg.blockDim = dim3(kRtThreads);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, router_gemv_kernel, wr, x, T, E, H, logits);
}

__global__ void __launch_bounds__(256) residual_kernel(const uint16_t* __restrict__ y_in, const uint16_t* __restrict__ x2,
                                                       const float* __restrict__ shared, const float* __restrict__ extra,
                                                       const float* __restrict__ moe, long n, uint16_t* __restrict__ y_out,
                                                       uint16_t* __restrict__ x_next) {
    for (long i = (blockIdx.x * 256L + threadIdx.x) * 8; i < n; i += (long)gridDim.x * 256 * 8) {
        float y[8];
        if (y_in) {
            const uint4 v = *reinterpret_cast<const uint4*>(y_in + i);
            const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
            for (int k = 0; k < 4; k++) y[2 * k] = bf_lo(w[k]), y[2 * k + 1] = bf_hi(w[k]);
        } else {
            const uint4 v = *reinterpret_cast<const uint4*>(x2 + i);
            const uint32_t w[4] = {v.x, v.y, v.z, v.w};
            const float4 s0 = reinterpret_cast<const float4*>(shared + i)[0], s1 = reinterpret_cast<const float4*>(shared + i)[1];
            const float s[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
            uint32_t o[4];
#pragma unroll
            for (int k = 0; k < 4; k++) {
                const uint16_t lo = f2bf(bf_lo(w[k]) + s[2 * k]), hi = f2bf(bf_hi(w[k]) + s[2 * k + 1]);
                y[2 * k] = bf_lo(lo);
                y[2 * k + 1] = bf_lo(hi);
                o[k] = (uint32_t)lo | ((uint32_t)hi << 16);
            }
            if (y_out) *reinterpret_cast<uint4*>(y_out + i) = make_uint4(o[0], o[1], o[2], o[3]);
        }
        if (x_next) {
            const float4 m0 = reinterpret_cast<const float4*>(moe + i)[0], m1 = reinterpret_cast<const float4*>(moe + i)[1];
            const float m[8] = {m0.x, m0.y, m0.z, m0.w, m1.x, m1.y, m1.z, m1.w};
            float ex[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
            if (extra) {
                const float4 e0 = reinterpret_cast<const float4*>(extra + i)[0], e1 = reinterpret_cast<const float4*>(extra + i)[1];
                ex[0] = e0.x, ex[1] = e0.y, ex[2] = e0.z, ex[3] = e0.w, ex[4] = e1.x, ex[5] = e1.y, ex[6] = e1.z, ex[7] = e1.w;
            }
            uint32_t o[4];
#pragma unroll
            for (int k = 0; k < 4; k++) {
                const float s0 = extra ? y[2 * k] + ex[2 * k] : y[2 * k];
                const float s1 = extra ? y[2 * k + 1] + ex[2 * k + 1] : y[2 * k + 1];
                o[k] = (uint32_t)f2bf(s0 + m[2 * k]) | ((uint32_t)f2bf(s1 + m[2 * k + 1]) << 16);
            }
            *reinterpret_cast<uint4*>(x_next + i) = make_uint4(o[0], o[1], o[2], o[3]);
        }
    }
}

cudaError_t launch_residual(const uint16_t* y_in, const uint16_t* x2, const float* shared, const float* extra,
                            const float* moe, long n, uint16_t* y_out, uint16_t* x_next, int sm_count, cudaStream_t st) {
    if (n <= 0) return cudaSuccess;
    if (n % 8) return cudaErrorInvalidValue;
    const int grid = (int)std::min<long>((n / 8 + 255) / 256, (long)sm_count * 8);
    residual_kernel<<<grid, 256, 0, st>>>(y_in, x2, shared, extra, moe, n, y_out, x_next);
    return cudaGetLastError();
}

}  // namespace moe
