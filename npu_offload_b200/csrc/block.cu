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

namespace moe {

constexpr int kRtWarps = 8;   // experts per CTA (a warp per expert)
constexpr int kRtTok = 16;    // tokens per CTA row of the grid

// Warp per expert row of Wr (H bf16, read once per token block with 16-byte loads); lane-strided
// 8-element chunks accumulated in fp32 in element order, then a fixed butterfly: the same bits on
// every run.
__global__ void __launch_bounds__(kRtWarps * 32) router_gemv_kernel(const uint16_t* __restrict__ wr,
                                                                  const uint16_t* __restrict__ x, int T, int E, int H,
                                                                  float* __restrict__ logits) {
    const int lane = threadIdx.x & 31;
    const int e = blockIdx.x * kRtWarps + (threadIdx.x >> 5);
    const int t0 = blockIdx.y * kRtTok, nt = min(kRtTok, T - t0);
    if (e >= E || nt <= 0) return;
    float acc[kRtTok];
#pragma unroll
    for (int t = 0; t < kRtTok; t++) acc[t] = 0.f;
    const uint4* w4 = reinterpret_cast<const uint4*>(wr + (size_t)e * H);
    const uint4* x4 = reinterpret_cast<const uint4*>(x + (size_t)t0 * H);
    const int n8 = H / 8;
    for (int c = lane; c < n8; c += 32) {
        const uint4 wv = __ldg(w4 + c);
        const uint32_t ww[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
        for (int t = 0; t < kRtTok; t++)
            if (t < nt) {
                const uint4 xv = __ldg(x4 + (size_t)t * n8 + c);
                const uint32_t xw[4] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
                for (int k = 0; k < 4; k++) {
                    acc[t] = fmaf(bf_lo(ww[k]), bf_lo(xw[k]), acc[t]);
                    acc[t] = fmaf(bf_hi(ww[k]), bf_hi(xw[k]), acc[t]);
                }
            }
    }
#pragma unroll
    for (int t = 0; t < kRtTok; t++)
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) acc[t] += __shfl_xor_sync(0xffffffffu, acc[t], o);
    if (lane == 0) {
#pragma unroll
        for (int t = 0; t < kRtTok; t++)
            if (t < nt) logits[(size_t)(t0 + t) * E + e] = acc[t];
    }
}

cudaError_t launch_router_gemv(const uint16_t* wr, const uint16_t* x, int T, int E, int H, float* logits,
                               cudaStream_t st) {
    if (T <= 0) return cudaSuccess;
    if (H % 8 || ((uintptr_t)wr | (uintptr_t)x) & 15) return cudaErrorInvalidValue;
    dim3 g((E + kRtWarps - 1) / kRtWarps, (T + kRtTok - 1) / kRtTok);
    router_gemv_kernel<<<g, kRtWarps * 32, 0, st>>>(wr, x, T, E, H, logits);
    return cudaGetLastError();
}

// 8 elements per thread.  y = y_in, or bf16(x2 + shared) when y_in is null (stored to y_out when
// set); x_next = bf16((y + extra) + moe) when x_next is set (extra may be null).
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
