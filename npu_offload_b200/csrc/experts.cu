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
//                   writes y[pair, h] = w_pair * dot (fp32).  For unit-layout tables (down columns
//                   stored per f) down_unit_kernel computes the same y as a sum of columns scaled
//                   by the activations, with each warp owning 256 consecutive h.
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

// y[p, h] = w_p * sum_f act[p, f] * down[h, f] for unit-layout tables: CTA = (job, block of 4
// tokens, 2048 h); warp w owns h0 + 256w + 8*lane .. +8 and walks f in order, so every y is a
// sequential fp32 sum over f.  The block's activation rows are staged in shared memory.
constexpr int kDUTok = 4;
constexpr int kDUH = kWarps * 256;
__global__ void __launch_bounds__(kWarps * 32) down_unit_kernel(ExpertArgs a) {
    extern __shared__ __align__(16) unsigned char dsm[];
    uint16_t* sact = reinterpret_cast<uint16_t*>(dsm);  // [kDUTok][F]
    const int nj = njobs_of(a);
    const int H = a.H, F = a.F;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int ntb = (a.max_pairs + kDUTok - 1) / kDUTok, nhb = (H + kDUH - 1) / kDUH;
    const long total = (long)nj * ntb * nhb;
    for (long it = blockIdx.x; it < total; it += gridDim.x) {
        const int j = (int)(it / ((long)ntb * nhb));
        const int tb = (int)(it / nhb % ntb), hb = (int)(it % nhb);
        const Job jb = a.jobs[j];
        const int t0 = tb * kDUTok;
        if (t0 >= jb.n) continue;  // uniform across the CTA
        const int nt = min(kDUTok, jb.n - t0);
        __syncthreads();  // previous item's readers are done with sact
        for (int q = threadIdx.x; q < nt * F / 8; q += kWarps * 32) {
            const int i = q / (F / 8), c = q % (F / 8);
            reinterpret_cast<uint4*>(sact + (size_t)i * F)[c] =
                __ldg(reinterpret_cast<const uint4*>(a.act + (size_t)(jb.p0 + t0 + i) * F) + c);
        }
        __syncthreads();
        const int h = hb * kDUH + warp * 256 + lane * 8;
        if (h >= H) continue;
        const bool q8 = jb.ex.kind == kKindQ8;
        const size_t pitch = unit_pitch(jb.ex.kind, H);
        float acc[kDUTok][8];
#pragma unroll
        for (int i = 0; i < kDUTok; i++)
#pragma unroll
            for (int e = 0; e < 8; e++) acc[i][e] = 0.f;
        if (!q8) {
            const uint16_t* col = (const uint16_t*)jb.ex.w2 + h;
#pragma unroll 4
            for (int f = 0; f < F; f++) {
                const uint4 d = ldg_stream(col + (size_t)f * pitch);
                const float dv[8] = {bf_lo(d.x), bf_hi(d.x), bf_lo(d.y), bf_hi(d.y),
                                     bf_lo(d.z), bf_hi(d.z), bf_lo(d.w), bf_hi(d.w)};
#pragma unroll
                for (int i = 0; i < kDUTok; i++) {
                    const float av = bf2f(sact[(size_t)min(i, nt - 1) * F + f]);
#pragma unroll
                    for (int e = 0; e < 8; e++) acc[i][e] = fmaf(av, dv[e], acc[i][e]);
                }
            }
        } else {
            const int8_t* col = (const int8_t*)jb.ex.w2 + h;
#pragma unroll 4
            for (int f = 0; f < F; f++) {
                const uint2 d = __ldg(reinterpret_cast<const uint2*>(col + (size_t)f * pitch));
                const float dv[8] = {i8f(d.x, 0), i8f(d.x, 1), i8f(d.x, 2), i8f(d.x, 3),
                                     i8f(d.y, 0), i8f(d.y, 1), i8f(d.y, 2), i8f(d.y, 3)};
#pragma unroll
                for (int i = 0; i < kDUTok; i++) {
                    const float av = bf2f(sact[(size_t)min(i, nt - 1) * F + f]);
#pragma unroll
                    for (int e = 0; e < 8; e++) acc[i][e] = fmaf(av, dv[e], acc[i][e]);
                }
            }
        }
#pragma unroll
        for (int i = 0; i < kDUTok; i++) {
            if (i < nt) {
                const int p = jb.p0 + t0 + i;
                float o[8];
#pragma unroll
                for (int e = 0; e < 8; e++) o[e] = q8 ? (a.pw[p] * acc[i][e]) * jb.ex.sc[2 * F + h + e] : a.pw[p] * acc[i][e];
                float4* dst = reinterpret_cast<float4*>(a.y + (size_t)p * H + h);
                dst[0] = make_float4(o[0], o[1], o[2], o[3]);
                dst[1] = make_float4(o[4], o[5], o[6], o[7]);
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
        float4 v = *reinterpret_cast<const float4*>(a.y + (size_t)p * a.H + h);
        if (a.comb_w) {
            const float w = a.comb_w[p];
            v.x *= w;
            v.y *= w;
            v.z *= w;
            v.w *= w;
        }
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
    if (nj > 0 && a.unit_layout) {
        const long items = (long)nj * ((a.max_pairs + kDUTok - 1) / kDUTok) * ((a.H + kDUH - 1) / kDUH);
        down_unit_kernel<<<(int)std::min<long>(items, cap), kWarps * 32, (size_t)kDUTok * a.F * 2, st>>>(a);
        *launches += 1;
    } else if (nj > 0) {
        const long dn_units = (long)nj * (a.H / kWarps);
        down_kernel<<<(int)std::min<long>(dn_units, cap), kWarps * 32, 0, st>>>(a);
        *launches += 1;
    }
    if (marks) cudaEventRecord(marks[1], st);
    cudaError_t e = launch_combine(a, st, launches);
    if (marks) cudaEventRecord(marks[2], st);
    return e;
}

cudaError_t launch_combine(const ExpertArgs& a, cudaStream_t st, int* launches) {
    dim3 g((a.H / 4 + 255) / 256, a.T);
    combine_kernel<<<g, 256, 0, st>>>(a);
    *launches += 1;
    return cudaGetLastError();
}

// quant_row (cpu_kern.c:218-224) per row, one warp per row, in the reference's row order (F gate
// rows, F up rows, H down rows).  Element i of row r is read at src(r) + i * in_step and written at
// dst(r) + i * out_step, with the per-row bases and steps given by QuantGeom; scales / row sums go
// to sc[r] / rs[r], and (unit layout) the gate/up scales of unit f also to the unit's trailer.
__global__ void __launch_bounds__(256) quantize_q8_kernel(QuantGeom q, int H, int F, float* sc, int32_t* rs) {
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    const int rows = 2 * F + H;
    if (warp >= rows) return;
    const uint16_t* src;
    int8_t* dst;
    size_t si, di;
    int n;
    if (warp < 2 * F) {
        const int f = warp < F ? warp : warp - F;
        src = (warp < F ? q.g : q.u) + (size_t)f * q.gu_pitch;
        dst = q.q + (size_t)f * q.q_pitch + (warp < F ? 0 : q.q_up_off);
        si = di = 1;
        n = H;
    } else {
        const int h = warp - 2 * F;
        src = q.d + (size_t)h * q.d_row_step;
        dst = q.q + q.q_down_off + (size_t)h * q.q_down_row_step;
        si = q.d_elem_step;
        di = q.q_down_elem_step;
        n = F;
    }
    float m = 0.f;
    for (int i = lane; i < n; i += 32) m = fmaxf(m, fabsf(bf2f(src[(size_t)i * si])));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    const float s = m > 0.f ? __fdiv_rn(m, 127.f) : 1.f;
    const float inv = __fdiv_rn(1.f, s);
    int sum = 0;
    for (int i = lane; i < n; i += 32) {
        int v = __float2int_rn(__fmul_rn(bf2f(src[(size_t)i * si]), inv));
        v = v > 127 ? 127 : (v < -127 ? -127 : v);
        dst[(size_t)i * di] = (int8_t)v;
        sum += v;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    if (lane == 0) {
        sc[warp] = s;
        if (rs) rs[warp] = sum;
        if (q.trailer && warp < 2 * F) {  // unit trailer: sc_gate f, sc_up f, 0, 0
            const int f = warp < F ? warp : warp - F;
            float* t = reinterpret_cast<float*>(q.q + (size_t)f * q.q_pitch + 3 * (size_t)H);
            t[warp < F ? 0 : 1] = s;
            t[warp < F ? 2 : 3] = 0.f;
        }
    }
}

cudaError_t launch_quantize_q8(const QuantGeom& q, int H, int F, float* sc, int32_t* rs, cudaStream_t st,
                               int* launches) {
    const int rows = 2 * F + H;
    quantize_q8_kernel<<<(rows * 32 + 255) / 256, 256, 0, st>>>(q, H, F, sc, rs);
    *launches += 1;
    return cudaGetLastError();
}

QuantGeom quant_geom_split(const uint16_t* g, const uint16_t* u, const uint16_t* d, int H, int F, int8_t* q) {
    const size_t FH = (size_t)F * H;
    QuantGeom r{};
    r.g = g;
    r.u = u;
    r.d = d;
    r.gu_pitch = H;
    r.d_row_step = F;
    r.d_elem_step = 1;
    r.q = q;
    r.q_pitch = H;
    r.q_up_off = FH;
    r.q_down_off = 2 * FH;
    r.q_down_row_step = F;
    r.q_down_elem_step = 1;
    r.trailer = 0;
    return r;
}

QuantGeom quant_geom_unit(const uint16_t* unit_bf16, int H, int F, int8_t* q_unit) {
    const size_t pb = unit_pitch(kKindBF16, H), pq = unit_pitch(kKindQ8, H);
    QuantGeom r{};
    r.g = unit_bf16;
    r.u = unit_bf16 + H;
    r.d = unit_bf16 + 2 * (size_t)H;  // down row h = column h of the stored down columns
    r.gu_pitch = pb;
    r.d_row_step = 1;
    r.d_elem_step = pb;
    r.q = q_unit;
    r.q_pitch = pq;
    r.q_up_off = H;
    r.q_down_off = 2 * (size_t)H;
    r.q_down_row_step = 1;
    r.q_down_elem_step = pq;
    r.trailer = 1;
    return r;
}

// dst[f * pitch + h] = src[h * F + f]: an [H, F] row-major down matrix into the down columns of a
// unit table (32 x 32 tiles through shared memory, coalesced on both sides).
template <class T>
__global__ void __launch_bounds__(256) scatter_down_kernel(const T* src, T* dst, size_t pitch, int H, int F) {
    __shared__ T tile[32][33];
    const int f0 = blockIdx.x * 32, h0 = blockIdx.y * 32;
    const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
    for (int r = ty; r < 32; r += 8)
        if (h0 + r < H && f0 + tx < F) tile[r][tx] = src[(size_t)(h0 + r) * F + f0 + tx];
    __syncthreads();
    for (int r = ty; r < 32; r += 8)
        if (f0 + r < F && h0 + tx < H) dst[(size_t)(f0 + r) * pitch + h0 + tx] = tile[tx][r];
}

cudaError_t launch_scatter_down(const void* src, void* dst, size_t pitch, int H, int F, int esize, cudaStream_t st,
                                int* launches) {
    const dim3 grid((F + 31) / 32, (H + 31) / 32);
    if (esize == 2)
        scatter_down_kernel<uint16_t><<<grid, 256, 0, st>>>((const uint16_t*)src, (uint16_t*)dst, pitch, H, F);
    else
        scatter_down_kernel<int8_t><<<grid, 256, 0, st>>>((const int8_t*)src, (int8_t*)dst, pitch, H, F);
    *launches += 1;
    return cudaGetLastError();
}

}  // namespace moe
