// Decode expert FFN for the B200 MoE data plane: memory-bound grouped SwiGLU GEMV.
//
// Semantics follow the reference's cold-expert kernel solar_hybrid/cpu_moe.cpp:38-96:
//   g, u   = gate/up rows . x_t, fp32, not rounded                      (:63-66)
//   act    = bf16_rne(g / (1 + exp(-g)) * u)                           (:70-77)
//   out[t] = sum over jobs (job order) of w * (down rows . act)         (:81-93)
// and, for int8 weight-only experts, ck_moe_q8w (track2_opt/solar_engine/csrc/cpu_kern.c:306-333):
//   g = (x . q_row) * sc_row, act as above, y = (w * (act . qd_row)) * sc_d.
//
// Pipeline (three launches):
//   gateup_kernel   one warp per (job, f): streams gate row f and up row f once (128-bit no-allocate
//                   loads), dots them with the job's tokens, writes act[pair, f] in bf16.
//   down_kernel     one warp per (job, h): streams down row h once, dots with the job's activations,
//                   writes y[pair, h] = w_pair * dot (fp32).
//   combine_kernel  out[t, h] = sum of y over the token's pairs in job order.
#include <algorithm>

#include "common.cuh"
#include "experts.h"

namespace moe {

constexpr int kWarps = 8;  // warps per CTA in the GEMV kernels
constexpr int kTB = 4;     // tokens per register block

__device__ __forceinline__ int njobs_of(const ExpertArgs& a) { return a.n_jobs_host >= 0 ? a.n_jobs_host : *a.n_jobs; }

__global__ void __launch_bounds__(kWarps * 32) gateup_kernel(ExpertArgs a) {
    const int nj = njobs_of(a);
    const int upj = a.F / kWarps;
    const long total = (long)nj * upj;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int H = a.H, F = a.F;
    for (long u = blockIdx.x; u < total; u += gridDim.x) {
        const int j = (int)(u / upj);
        const int f = (int)(u % upj) * kWarps + warp;
        const Job jb = a.jobs[j];
        for (int t0 = 0; t0 < jb.n; t0 += kTB) {
            const int nt = min(kTB, jb.n - t0);
            const uint16_t* xs[kTB];
#pragma unroll
            for (int i = 0; i < kTB; i++) xs[i] = a.x + (size_t)a.ptok[jb.p0 + t0 + min(i, nt - 1)] * H;
            float ag[kTB], au[kTB];
#pragma unroll
            for (int i = 0; i < kTB; i++) ag[i] = au[i] = 0.f;
            if (jb.ex.kind == kKindBF16) {
                const uint16_t* rg = (const uint16_t*)jb.ex.w1 + gate_row(jb.ex, f, H, F);
                const uint16_t* ru = (const uint16_t*)jb.ex.w1 + up_row(jb.ex, f, H, F);
                for (int c = lane * 8; c < H; c += 1024) {
                    uint4 wg[4], wu[4];
#pragma unroll
                    for (int s = 0; s < 4; s++) {
                        const int cc = c + s * 256;
                        wg[s] = cc < H ? ldg_stream(rg + cc) : make_uint4(0, 0, 0, 0);
                        wu[s] = cc < H ? ldg_stream(ru + cc) : make_uint4(0, 0, 0, 0);
                    }
#pragma unroll
                    for (int s = 0; s < 4; s++) {
                        const int cc = c + s * 256;
                        if (cc < H) {
#pragma unroll
                            for (int i = 0; i < kTB; i++) {
                                const uint4 xv = __ldg(reinterpret_cast<const uint4*>(xs[i] + cc));
                                ag[i] = dot8_bf16(wg[s], xv, ag[i]);
                                au[i] = dot8_bf16(wu[s], xv, au[i]);
                            }
                        }
                    }
                }
            } else {
                const int8_t* qg = (const int8_t*)jb.ex.w1 + gate_row(jb.ex, f, H, F);
                const int8_t* qu = (const int8_t*)jb.ex.w1 + up_row(jb.ex, f, H, F);
                for (int c = lane * 16; c < H; c += 1024) {
                    uint4 wg[2], wu[2];
#pragma unroll
                    for (int s = 0; s < 2; s++) {
                        const int cc = c + s * 512;
                        wg[s] = cc < H ? ldg_stream(qg + cc) : make_uint4(0, 0, 0, 0);
                        wu[s] = cc < H ? ldg_stream(qu + cc) : make_uint4(0, 0, 0, 0);
                    }
#pragma unroll
                    for (int s = 0; s < 2; s++) {
                        const int cc = c + s * 512;
                        if (cc < H) {
#pragma unroll
                            for (int i = 0; i < kTB; i++) {
                                const uint4 x0 = __ldg(reinterpret_cast<const uint4*>(xs[i] + cc));
                                const uint4 x1 = __ldg(reinterpret_cast<const uint4*>(xs[i] + cc + 8));
                                float g = ag[i], v = au[i];
                                g = dot4_i8(wg[s].x, x0.x, x0.y, g);
                                g = dot4_i8(wg[s].y, x0.z, x0.w, g);
                                g = dot4_i8(wg[s].z, x1.x, x1.y, g);
                                g = dot4_i8(wg[s].w, x1.z, x1.w, g);
                                v = dot4_i8(wu[s].x, x0.x, x0.y, v);
                                v = dot4_i8(wu[s].y, x0.z, x0.w, v);
                                v = dot4_i8(wu[s].z, x1.x, x1.y, v);
                                v = dot4_i8(wu[s].w, x1.z, x1.w, v);
                                ag[i] = g;
                                au[i] = v;
                            }
                        }
                    }
                }
            }
            float mg = 0.f, mu = 0.f;
#pragma unroll
            for (int i = 0; i < kTB; i++) {
                const float sg = warp_sum(ag[i]), su = warp_sum(au[i]);
                if (lane == i) {
                    mg = sg;
                    mu = su;
                }
            }
            if (lane < nt) {
                if (jb.ex.kind == kKindQ8) {
                    mg *= jb.ex.sc[f];
                    mu *= jb.ex.sc[F + f];
                }
                a.act[(size_t)(jb.p0 + t0 + lane) * F + f] = swiglu_bf16(mg, mu);
            }
        }
    }
}

__global__ void __launch_bounds__(kWarps * 32) down_kernel(ExpertArgs a) {
    const int nj = njobs_of(a);
    const int uph = a.H / kWarps;
    const long total = (long)nj * uph;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int H = a.H, F = a.F;
    for (long u = blockIdx.x; u < total; u += gridDim.x) {
        const int j = (int)(u / uph);
        const int h = (int)(u % uph) * kWarps + warp;
        const Job jb = a.jobs[j];
        const bool q8 = jb.ex.kind == kKindQ8;
        for (int t0 = 0; t0 < jb.n; t0 += kTB) {
            const int nt = min(kTB, jb.n - t0);
            const uint16_t* as[kTB];
#pragma unroll
            for (int i = 0; i < kTB; i++) as[i] = a.act + (size_t)(jb.p0 + t0 + min(i, nt - 1)) * F;
            float acc[kTB];
#pragma unroll
            for (int i = 0; i < kTB; i++) acc[i] = 0.f;
            if (!q8) {
                const uint16_t* row = (const uint16_t*)jb.ex.w2 + (size_t)h * F;
                uint4 wv[8];
#pragma unroll
                for (int s = 0; s < 8; s++) {
                    const int c = lane * 8 + s * 256;
                    wv[s] = c < F ? ldg_stream(row + c) : make_uint4(0, 0, 0, 0);
                }
#pragma unroll
                for (int s = 0; s < 8; s++) {
                    const int c = lane * 8 + s * 256;
                    if (c < F) {
#pragma unroll
                        for (int i = 0; i < kTB; i++)
                            acc[i] = dot8_bf16(wv[s], __ldg(reinterpret_cast<const uint4*>(as[i] + c)), acc[i]);
                    }
                }
            } else {
                const int8_t* row = (const int8_t*)jb.ex.w2 + (size_t)h * F;
                uint4 wv[4];
#pragma unroll
                for (int s = 0; s < 4; s++) {
                    const int c = lane * 16 + s * 512;
                    wv[s] = c < F ? ldg_stream(row + c) : make_uint4(0, 0, 0, 0);
                }
#pragma unroll
                for (int s = 0; s < 4; s++) {
                    const int c = lane * 16 + s * 512;
                    if (c < F) {
#pragma unroll
                        for (int i = 0; i < kTB; i++) {
                            const uint4 x0 = __ldg(reinterpret_cast<const uint4*>(as[i] + c));
                            const uint4 x1 = __ldg(reinterpret_cast<const uint4*>(as[i] + c + 8));
                            float v = acc[i];
                            v = dot4_i8(wv[s].x, x0.x, x0.y, v);
                            v = dot4_i8(wv[s].y, x0.z, x0.w, v);
                            v = dot4_i8(wv[s].z, x1.x, x1.y, v);
                            v = dot4_i8(wv[s].w, x1.z, x1.w, v);
                            acc[i] = v;
                        }
                    }
                }
            }
            float mine = 0.f;
#pragma unroll
            for (int i = 0; i < kTB; i++) {
                const float s = warp_sum(acc[i]);
                if (lane == i) mine = s;
            }
            if (lane < nt) {
                const int p = jb.p0 + t0 + lane;
                float yv = a.pw[p] * mine;
                if (q8) yv *= jb.ex.sc[2 * F + h];
                a.y[(size_t)p * H + h] = yv;
            }
        }
    }
}

__global__ void __launch_bounds__(256) combine_kernel(ExpertArgs a) {
    const int t = blockIdx.y;
    const int h = (blockIdx.x * 256 + threadIdx.x) * 4;
    if (h >= a.H) return;
    float4* o = reinterpret_cast<float4*>(a.out + (size_t)t * a.H + h);
    float4 acc = a.accumulate ? *o : make_float4(0.f, 0.f, 0.f, 0.f);
    for (int i = a.comb_off[t]; i < a.comb_off[t + 1]; i++) {
        const int p = a.comb_p[i];
        if (p < 0) continue;
        const float4 v = *reinterpret_cast<const float4*>(a.y + (size_t)p * a.H + h);
        acc.x += v.x;
        acc.y += v.y;
        acc.z += v.z;
        acc.w += v.w;
    }
    *o = acc;
}

cudaError_t launch_experts(const ExpertArgs& a, int sm_count, cudaStream_t st, int* launches, cudaEvent_t* marks) {
    if (a.T <= 0) return cudaSuccess;
    const int nj = a.n_jobs_host >= 0 ? a.n_jobs_host : a.n_jobs_max;
    const int cap = sm_count * 8;
    if (nj > 0) {
        const long gu_units = (long)nj * (a.F / kWarps);
        gateup_kernel<<<(int)std::min<long>(gu_units, cap), kWarps * 32, 0, st>>>(a);
        *launches += 1;
    }
    if (marks) cudaEventRecord(marks[0], st);
    if (nj > 0) {
        const long dn_units = (long)nj * (a.H / kWarps);
        down_kernel<<<(int)std::min<long>(dn_units, cap), kWarps * 32, 0, st>>>(a);
        *launches += 1;
    }
    if (marks) cudaEventRecord(marks[1], st);
    dim3 g((a.H / 4 + 255) / 256, a.T);
    combine_kernel<<<g, 256, 0, st>>>(a);
    *launches += 1;
    if (marks) cudaEventRecord(marks[2], st);
    return cudaGetLastError();
}

// quant_row (cpu_kern.c:218-224) per row: one warp per row.  Input gate row f at g + f*gu_pitch,
// up row f at u + f*gu_pitch, down row h at d + h*F; output gate row f at q + f*q_pitch, up row f at
// q + f*q_pitch + q_up_off, down row h at q + q_down_off + h*F; scales / row sums in the reference's
// row order (gate rows, up rows, down rows).
__global__ void __launch_bounds__(256) quantize_q8_kernel(const uint16_t* g, const uint16_t* u, size_t gu_pitch,
                                                          const uint16_t* d, int H, int F, int8_t* q, size_t q_pitch,
                                                          size_t q_up_off, size_t q_down_off, float* sc, int32_t* rs) {
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    const int rows = 2 * F + H;
    if (warp >= rows) return;
    const uint16_t* src;
    int8_t* dst;
    int n;
    if (warp < F) {
        src = g + (size_t)warp * gu_pitch; dst = q + (size_t)warp * q_pitch; n = H;
    } else if (warp < 2 * F) {
        src = u + (size_t)(warp - F) * gu_pitch; dst = q + (size_t)(warp - F) * q_pitch + q_up_off; n = H;
    } else {
        const int h = warp - 2 * F;
        src = d + (size_t)h * F; dst = q + q_down_off + (size_t)h * F; n = F;
    }
    float m = 0.f;
    for (int i = lane; i < n; i += 32) m = fmaxf(m, fabsf(bf2f(src[i])));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    const float s = m > 0.f ? __fdiv_rn(m, 127.f) : 1.f;
    const float inv = __fdiv_rn(1.f, s);
    int sum = 0;
    for (int i = lane; i < n; i += 32) {
        int v = __float2int_rn(__fmul_rn(bf2f(src[i]), inv));
        v = v > 127 ? 127 : (v < -127 ? -127 : v);
        dst[i] = (int8_t)v;
        sum += v;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    if (lane == 0) {
        sc[warp] = s;
        if (rs) rs[warp] = sum;
    }
}

cudaError_t launch_quantize_q8(const uint16_t* g, const uint16_t* u, const uint16_t* d, int H, int F, int8_t* q,
                               float* sc, int32_t* rs, cudaStream_t st, int* launches, int interleaved) {
    const int rows = 2 * F + H;
    const size_t FH = (size_t)F * H;
    if (interleaved)
        quantize_q8_kernel<<<(rows * 32 + 255) / 256, 256, 0, st>>>(g, u, 2 * (size_t)H, d, H, F, q, 2 * (size_t)H,
                                                                    (size_t)H, 2 * FH, sc, rs);
    else
        quantize_q8_kernel<<<(rows * 32 + 255) / 256, 256, 0, st>>>(g, u, (size_t)H, d, H, F, q, (size_t)H, FH, 2 * FH,
                                                                    sc, rs);
    *launches += 1;
    return cudaGetLastError();
}

}  // namespace moe
