// Fused persistent decode kernel for the B200 MoE data plane: one launch per layer performs
// routing, the grouped SwiGLU expert GEMV (gate/up + down) and the weighted combine.
//
// Semantics are the reference's cold-expert path (solar_hybrid/cpu_moe.cpp:38-96, int8 weight-only
// form cpu_kern.c:306-333) behind the layer surface of track2_opt/solar_engine/src/main.rs:149-209:
//   g, u = gate/up rows . x_t (fp32)      act = bf16_rne(g / (1 + exp(-g)) * u)
//   out[t, h] = sum over the token's experts in job order of w * (down row h . act)
//
// Structure (one CTA per SM, grid = SM count, every CTA resident):
//   prologue      every CTA routes the T <= 16 tokens itself (route_core.cuh; bit-identical in all
//                 CTAs) and builds the local job list in first-appearance order (runtime.py:343-354).
//   partition     a static, byte-balanced share per CTA: output rows [h0, h1) of every job's down
//                 matrix (phase 2) plus a contiguous range of gate/up units (phase 1) sized so that
//                 every CTA streams the same number of bytes.
//   producer      one thread streams the CTA's weights with 1-D bulk async copies (TMA engine) into
//                 an NS-deep shared-memory ring guarded by mbarriers (L2 evict-first: read once).
//   consumers     8 warps take ring stages round-robin.  Phase-1 stage = gate row f + up row f of one
//                 job: 128-bit shared loads, fp32 FMAs, warp-shuffle reductions, SwiGLU -> act[pair, f]
//                 (global, bf16).  A warp publishes finished units per job with a release-ordered
//                 counter.  Phase-2 stage = up to rs down rows of one job, dotted with that job's
//                 activations (staged in shared memory) -> per-pair partial outputs in shared memory.
//   act loader    one warp waits (bounded) until every CTA has published all F units of job j, then
//                 stages act rows of job j into a double-buffered shared slot.
//   combine       after its phase-2 stages each CTA sums, per token and in job order, the partial
//                 outputs of its own rows and writes out[t, h0:h1) -- deterministic, no atomics.
// Every wait is bounded (globaltimer); a timeout raises kErrTimeout, stops all roles, drains the
// bulk copies in flight and returns.  Programmatic dependent launch lets the next layer's prologue
// and weight streaming start while this grid drains; everything that touches state written by the
// previous grid (act, counters, outputs) runs after griddepcontrol.wait.
#include <climits>
#include <cstddef>

#include "common.cuh"
#include "decode.h"
#include "ptx.cuh"

namespace moe {

constexpr int kNWC = 8;                // consumer warps
constexpr int kProdWarp = kNWC;        // bulk-copy producer
constexpr int kActWarp = kNWC + 1;     // activation loader
constexpr int kDecThreads = (kNWC + 2) * 32;
constexpr int kMaxNS = 16;
constexpr int kRSMaxBF = 8;
constexpr int kRSMaxQ8 = 8;
constexpr size_t kSmemCap = 227 * 1024;
constexpr int kMaxSeg = 128;

struct __align__(16) Ctrl {
    uint64_t full[kMaxNS];
    uint64_t empty[kMaxNS];
    uint64_t x_full, p1_done;
    int abort_flag;
    int act_job[2];        // job whose activations occupy act slot b (-1: none)
    int act_done[2];       // phase-2 stages finished on act slot b
    int fill_seq[kMaxNS];  // fill number last issued into each ring slot (-1: none)
    int ticket;            // next ring stage for a consumer warp
    PlanCta me;            // this CTA's share (copied from the plan; 16-byte aligned member)
    PlanShared sh;         // routing result and job list (copied from the plan; 16-byte aligned member)
};
static_assert(offsetof(Ctrl, me) % 16 == 0 && offsetof(Ctrl, sh) % 16 == 0, "int4 copies into Ctrl");

__device__ __forceinline__ bool timed_out(Ctrl& c, uint32_t* err, uint64_t deadline) {
    if (*(volatile int*)&c.abort_flag) return true;
    if (globaltimer_ns() > deadline) {
        *(volatile int*)&c.abort_flag = 1;
        atomicOr(err, kErrTimeout);
        return true;
    }
    return false;
}

// Bounded mbarrier wait; false when the kernel is aborting.
__device__ __forceinline__ bool wait_bar(uint64_t* bar, uint32_t parity, Ctrl& c, uint32_t* err, uint64_t deadline) {
    while (!mbar_try_wait(bar, parity))
        if (timed_out(c, err, deadline)) return false;
    return true;
}

// Bounded wait used while draining copies: ignores the abort flag, only the deadline.
__device__ __forceinline__ void drain_bar(uint64_t* bar, uint32_t parity, uint64_t deadline) {
    while (!mbar_try_wait(bar, parity))
        if (globaltimer_ns() > deadline) return;
}

__device__ __forceinline__ int esize(int kind) { return kind == kKindBF16 ? 2 : 1; }

// ---- phase 1: gate row + up row of one job, NTB tokens -> per-lane-replicated sums ----
template <int NTB>
__device__ __forceinline__ void p1_bf16(const uint16_t* gr, const uint16_t* ur, const uint16_t* const* xr, int H,
                                        float* g, float* u) {
    const int lane = threadIdx.x & 31;
    f32x2 ag[NTB][2], au[NTB][2];
#pragma unroll
    for (int i = 0; i < NTB; i++) ag[i][0] = ag[i][1] = au[i][0] = au[i][1] = 0ull;
#pragma unroll 4
    for (int c = lane * 8; c < H; c += 256) {
        const uint4 wg = *reinterpret_cast<const uint4*>(gr + c);
        const uint4 wu = *reinterpret_cast<const uint4*>(ur + c);
        const f32x2 g0 = bf16x2_to_f32x2(wg.x), g1 = bf16x2_to_f32x2(wg.y), g2 = bf16x2_to_f32x2(wg.z),
                    g3 = bf16x2_to_f32x2(wg.w);
        const f32x2 u0 = bf16x2_to_f32x2(wu.x), u1 = bf16x2_to_f32x2(wu.y), u2 = bf16x2_to_f32x2(wu.z),
                    u3 = bf16x2_to_f32x2(wu.w);
#pragma unroll
        for (int i = 0; i < NTB; i++) {
            const uint4 xv = *reinterpret_cast<const uint4*>(xr[i] + c);
            const f32x2 x0 = bf16x2_to_f32x2(xv.x), x1 = bf16x2_to_f32x2(xv.y), x2 = bf16x2_to_f32x2(xv.z),
                        x3 = bf16x2_to_f32x2(xv.w);
            ag[i][0] = ffma2(g0, x0, ag[i][0]);
            ag[i][1] = ffma2(g1, x1, ag[i][1]);
            ag[i][0] = ffma2(g2, x2, ag[i][0]);
            ag[i][1] = ffma2(g3, x3, ag[i][1]);
            au[i][0] = ffma2(u0, x0, au[i][0]);
            au[i][1] = ffma2(u1, x1, au[i][1]);
            au[i][0] = ffma2(u2, x2, au[i][0]);
            au[i][1] = ffma2(u3, x3, au[i][1]);
        }
    }
#pragma unroll
    for (int i = 0; i < NTB; i++) {
        g[i] = warp_sum(sum_f32x2(ag[i][0]) + sum_f32x2(ag[i][1]));
        u[i] = warp_sum(sum_f32x2(au[i][0]) + sum_f32x2(au[i][1]));
    }
}

// Same with x already widened to fp32 in shared memory (small batches): no x conversion per use.
template <int NTB>
__device__ __forceinline__ void p1_bf16_xf(const uint16_t* gr, const uint16_t* ur, const float* const* xr, int H,
                                           float* g, float* u) {
    const int lane = threadIdx.x & 31;
    f32x2 ag[NTB][2], au[NTB][2];
#pragma unroll
    for (int i = 0; i < NTB; i++) ag[i][0] = ag[i][1] = au[i][0] = au[i][1] = 0ull;
#pragma unroll 4
    for (int c = lane * 8; c < H; c += 256) {
        const uint4 wg = *reinterpret_cast<const uint4*>(gr + c);
        const uint4 wu = *reinterpret_cast<const uint4*>(ur + c);
        const f32x2 g0 = bf16x2_to_f32x2(wg.x), g1 = bf16x2_to_f32x2(wg.y), g2 = bf16x2_to_f32x2(wg.z),
                    g3 = bf16x2_to_f32x2(wg.w);
        const f32x2 u0 = bf16x2_to_f32x2(wu.x), u1 = bf16x2_to_f32x2(wu.y), u2 = bf16x2_to_f32x2(wu.z),
                    u3 = bf16x2_to_f32x2(wu.w);
#pragma unroll
        for (int i = 0; i < NTB; i++) {
            const ulonglong2 xa = *reinterpret_cast<const ulonglong2*>(xr[i] + c);
            const ulonglong2 xb = *reinterpret_cast<const ulonglong2*>(xr[i] + c + 4);
            ag[i][0] = ffma2(g0, xa.x, ag[i][0]);
            ag[i][1] = ffma2(g1, xa.y, ag[i][1]);
            ag[i][0] = ffma2(g2, xb.x, ag[i][0]);
            ag[i][1] = ffma2(g3, xb.y, ag[i][1]);
            au[i][0] = ffma2(u0, xa.x, au[i][0]);
            au[i][1] = ffma2(u1, xa.y, au[i][1]);
            au[i][0] = ffma2(u2, xb.x, au[i][0]);
            au[i][1] = ffma2(u3, xb.y, au[i][1]);
        }
    }
#pragma unroll
    for (int i = 0; i < NTB; i++) {
        g[i] = warp_sum(sum_f32x2(ag[i][0]) + sum_f32x2(ag[i][1]));
        u[i] = warp_sum(sum_f32x2(au[i][0]) + sum_f32x2(au[i][1]));
    }
}

template <int NTB>
__device__ __forceinline__ void p1_q8(const int8_t* gr, const int8_t* ur, const uint16_t* const* xr, int H, float* g,
                                      float* u) {
    const int lane = threadIdx.x & 31;
    float ag[NTB], au[NTB];
#pragma unroll
    for (int i = 0; i < NTB; i++) ag[i] = au[i] = 0.f;
#pragma unroll 2
    for (int c = lane * 16; c < H; c += 512) {
        const uint4 wg = *reinterpret_cast<const uint4*>(gr + c);
        const uint4 wu = *reinterpret_cast<const uint4*>(ur + c);
#pragma unroll
        for (int i = 0; i < NTB; i++) {
            const uint4 x0 = *reinterpret_cast<const uint4*>(xr[i] + c);
            const uint4 x1 = *reinterpret_cast<const uint4*>(xr[i] + c + 8);
            float a = ag[i], b = au[i];
            a = dot4_i8(wg.x, x0.x, x0.y, a);
            a = dot4_i8(wg.y, x0.z, x0.w, a);
            a = dot4_i8(wg.z, x1.x, x1.y, a);
            a = dot4_i8(wg.w, x1.z, x1.w, a);
            b = dot4_i8(wu.x, x0.x, x0.y, b);
            b = dot4_i8(wu.y, x0.z, x0.w, b);
            b = dot4_i8(wu.z, x1.x, x1.y, b);
            b = dot4_i8(wu.w, x1.z, x1.w, b);
            ag[i] = a;
            au[i] = b;
        }
    }
#pragma unroll
    for (int i = 0; i < NTB; i++) {
        g[i] = warp_sum(ag[i]);
        u[i] = warp_sum(au[i]);
    }
}

template <int NTB>
__device__ __forceinline__ void p1_q8_xf(const int8_t* gr, const int8_t* ur, const float* const* xr, int H, float* g,
                                         float* u) {
    const int lane = threadIdx.x & 31;
    float ag[NTB], au[NTB];
#pragma unroll
    for (int i = 0; i < NTB; i++) ag[i] = au[i] = 0.f;
#pragma unroll 2
    for (int c = lane * 16; c < H; c += 512) {
        const uint4 wg = *reinterpret_cast<const uint4*>(gr + c);
        const uint4 wu = *reinterpret_cast<const uint4*>(ur + c);
        const uint32_t gw[4] = {wg.x, wg.y, wg.z, wg.w}, uw[4] = {wu.x, wu.y, wu.z, wu.w};
#pragma unroll
        for (int i = 0; i < NTB; i++) {
#pragma unroll
            for (int q = 0; q < 4; q++) {
                const float4 xv = *reinterpret_cast<const float4*>(xr[i] + c + 4 * q);
                float a = ag[i], b = au[i];
                a = fmaf(i8f(gw[q], 0), xv.x, a);
                a = fmaf(i8f(gw[q], 1), xv.y, a);
                a = fmaf(i8f(gw[q], 2), xv.z, a);
                a = fmaf(i8f(gw[q], 3), xv.w, a);
                b = fmaf(i8f(uw[q], 0), xv.x, b);
                b = fmaf(i8f(uw[q], 1), xv.y, b);
                b = fmaf(i8f(uw[q], 2), xv.z, b);
                b = fmaf(i8f(uw[q], 3), xv.w, b);
                ag[i] = a;
                au[i] = b;
            }
        }
    }
#pragma unroll
    for (int i = 0; i < NTB; i++) {
        g[i] = warp_sum(ag[i]);
        u[i] = warp_sum(au[i]);
    }
}

// ---- phase 2: nr down rows of one job, NTB tokens; results go straight to the ybuf rows ----
// yb[i] = ybuf row of token slot i (nullptr for padded slots), wp[i] = routing weight,
// sc = per-row int8 scales (nullptr for bf16).
template <int NTB, int RSM>
__device__ __forceinline__ void p2_store(float (&acc)[RSM][NTB], int nr, float* const* yb, const float* wp,
                                         const float* sc) {
    static_assert(RSM == 8, "butterfly reduction of 8 rows");
    const int lane = threadIdx.x & 31;
    const int r = lane >> 2;  // the row whose total this lane receives
    const float s = (sc && r < nr) ? __ldg(sc + r) : 1.f;
#pragma unroll
    for (int i = 0; i < NTB; i++) {
        float v[8];
#pragma unroll
        for (int k = 0; k < 8; k++) v[k] = acc[k][i];
        const float tot = warp_sum8(v);
        if ((lane & 3) == 0 && r < nr && yb[i]) yb[i][r] = sc ? (wp[i] * tot) * s : wp[i] * tot;
    }
}

template <int NTB, int RSM>
__device__ __forceinline__ void p2_bf16(const uint16_t* S, int nr, const uint16_t* const* ar, int F, float* const* yb,
                                        const float* wp) {
    const int lane = threadIdx.x & 31;
    f32x2 acc2[RSM][NTB];
#pragma unroll
    for (int r = 0; r < RSM; r++)
#pragma unroll
        for (int i = 0; i < NTB; i++) acc2[r][i] = 0ull;
    for (int c = lane * 8; c < F; c += 256) {
        f32x2 av[NTB][4];
#pragma unroll
        for (int i = 0; i < NTB; i++) {
            const uint4 a4 = *reinterpret_cast<const uint4*>(ar[i] + c);
            av[i][0] = bf16x2_to_f32x2(a4.x);
            av[i][1] = bf16x2_to_f32x2(a4.y);
            av[i][2] = bf16x2_to_f32x2(a4.z);
            av[i][3] = bf16x2_to_f32x2(a4.w);
        }
#pragma unroll
        for (int r = 0; r < RSM; r++) {
            if (r < nr) {
                const uint4 wv = *reinterpret_cast<const uint4*>(S + (size_t)r * F + c);
                const f32x2 w0 = bf16x2_to_f32x2(wv.x), w1 = bf16x2_to_f32x2(wv.y), w2 = bf16x2_to_f32x2(wv.z),
                            w3 = bf16x2_to_f32x2(wv.w);
#pragma unroll
                for (int i = 0; i < NTB; i++) {
                    f32x2 t = ffma2(w0, av[i][0], acc2[r][i]);
                    t = ffma2(w1, av[i][1], t);
                    t = ffma2(w2, av[i][2], t);
                    acc2[r][i] = ffma2(w3, av[i][3], t);
                }
            }
        }
    }
    float acc[RSM][NTB];
#pragma unroll
    for (int r = 0; r < RSM; r++)
#pragma unroll
        for (int i = 0; i < NTB; i++) acc[r][i] = r < nr ? sum_f32x2(acc2[r][i]) : 0.f;
    p2_store<NTB, RSM>(acc, nr, yb, wp, nullptr);
}

template <int NTB, int RSM>
__device__ __forceinline__ void p2_q8(const int8_t* S, int nr, const uint16_t* const* ar, int F, float* const* yb,
                                      const float* wp, const float* sc) {
    const int lane = threadIdx.x & 31;
    float acc[RSM][NTB];
#pragma unroll
    for (int r = 0; r < RSM; r++)
#pragma unroll
        for (int i = 0; i < NTB; i++) acc[r][i] = 0.f;
    for (int c = lane * 16; c < F; c += 512) {
        uint4 a0[NTB], a1[NTB];
#pragma unroll
        for (int i = 0; i < NTB; i++) {
            a0[i] = *reinterpret_cast<const uint4*>(ar[i] + c);
            a1[i] = *reinterpret_cast<const uint4*>(ar[i] + c + 8);
        }
#pragma unroll
        for (int r = 0; r < RSM; r++) {
            if (r < nr) {
                const uint4 wv = *reinterpret_cast<const uint4*>(S + (size_t)r * F + c);
#pragma unroll
                for (int i = 0; i < NTB; i++) {
                    float v = acc[r][i];
                    v = dot4_i8(wv.x, a0[i].x, a0[i].y, v);
                    v = dot4_i8(wv.y, a0[i].z, a0[i].w, v);
                    v = dot4_i8(wv.z, a1[i].x, a1[i].y, v);
                    v = dot4_i8(wv.w, a1[i].z, a1[i].w, v);
                    acc[r][i] = v;
                }
            }
        }
    }
    p2_store<NTB, RSM>(acc, nr, yb, wp, sc);
}

// One phase-1 stage: unit (job j, f) for all of the job's tokens.
__device__ void stage_p1(const DecodeArgs& a, Ctrl& c, const unsigned char* S, const unsigned char* xreg, int j, int f) {
    const int lane = threadIdx.x & 31;
    const int H = a.H, F = a.F;
    const int kind = c.sh.jkind[j];
    const int p0 = c.sh.jp0[j], n = c.sh.jp0[j + 1] - p0;
    const size_t rb = (size_t)H * esize(kind);
    for (int t0 = 0; t0 < n; t0 += 4) {
        const int nt = min(4, n - t0);
        float g[4] = {0.f, 0.f, 0.f, 0.f}, u[4] = {0.f, 0.f, 0.f, 0.f};
        if (a.x_f32) {
            const float* xr[4];
#pragma unroll
            for (int i = 0; i < 4; i++)
                xr[i] = reinterpret_cast<const float*>(xreg) + (size_t)c.sh.ptok[p0 + t0 + min(i, nt - 1)] * H;
            if (kind == kKindBF16) {
                const uint16_t* gr = reinterpret_cast<const uint16_t*>(S);
                const uint16_t* ur = reinterpret_cast<const uint16_t*>(S + rb);
                if (nt == 1) p1_bf16_xf<1>(gr, ur, xr, H, g, u);
                else if (nt == 2) p1_bf16_xf<2>(gr, ur, xr, H, g, u);
                else p1_bf16_xf<4>(gr, ur, xr, H, g, u);
            } else {
                const int8_t* gr = reinterpret_cast<const int8_t*>(S);
                const int8_t* ur = reinterpret_cast<const int8_t*>(S + rb);
                if (nt == 1) p1_q8_xf<1>(gr, ur, xr, H, g, u);
                else p1_q8_xf<4>(gr, ur, xr, H, g, u);
            }
        } else {
            const uint16_t* xr[4];
#pragma unroll
            for (int i = 0; i < 4; i++)
                xr[i] = reinterpret_cast<const uint16_t*>(xreg) + (size_t)c.sh.ptok[p0 + t0 + min(i, nt - 1)] * H;
            if (kind == kKindBF16) {
                const uint16_t* gr = reinterpret_cast<const uint16_t*>(S);
                const uint16_t* ur = reinterpret_cast<const uint16_t*>(S + rb);
                if (nt == 1) p1_bf16<1>(gr, ur, xr, H, g, u);
                else if (nt == 2) p1_bf16<2>(gr, ur, xr, H, g, u);
                else p1_bf16<4>(gr, ur, xr, H, g, u);
            } else {
                const int8_t* gr = reinterpret_cast<const int8_t*>(S);
                const int8_t* ur = reinterpret_cast<const int8_t*>(S + rb);
                if (nt == 1) p1_q8<1>(gr, ur, xr, H, g, u);
                else if (nt == 2) p1_q8<2>(gr, ur, xr, H, g, u);
                else p1_q8<4>(gr, ur, xr, H, g, u);
            }
        }
        float mg = 0.f, mu = 0.f;
#pragma unroll
        for (int i = 0; i < 4; i++)
            if (lane == i) {
                mg = g[i];
                mu = u[i];
            }
        if (lane < nt) {
            if (kind == kKindQ8) {
                const float* sc = c.sh.jsc[j];
                mg *= __ldg(sc + f);
                mu *= __ldg(sc + F + f);
            }
            a.act[(size_t)(p0 + t0 + lane) * F + f] = swiglu_bf16(mg, mu);
        }
    }
}

// One phase-2 stage: rows [row0, row0 + nr) (relative to h0) of job j's down matrix.
__device__ void stage_p2(const DecodeArgs& a, Ctrl& c, float* ybuf, const unsigned char* S, const uint16_t* A, int j,
                         int row0, int nr) {
    const int F = a.F;
    const int kind = c.sh.jkind[j];
    const int p0 = c.sh.jp0[j], n = c.sh.jp0[j + 1] - p0;
    const float* sc = kind == kKindQ8 ? c.sh.jsc[j] + 2 * F + c.me.h0 + row0 : nullptr;
    for (int t0 = 0; t0 < n; t0 += 4) {
        const int nt = min(4, n - t0);
        const uint16_t* ar[4];
        float* yb[4];
        float wp[4];
#pragma unroll
        for (int i = 0; i < 4; i++) {
            ar[i] = A + (size_t)(t0 + min(i, nt - 1)) * F;
            const int p = p0 + t0 + min(i, nt - 1);
            yb[i] = i < nt ? ybuf + (size_t)p * a.hr_max + row0 : nullptr;
            wp[i] = c.sh.pw[p];
        }
        if (kind == kKindBF16) {
            const uint16_t* W = reinterpret_cast<const uint16_t*>(S);
            if (nt == 1) p2_bf16<1, kRSMaxBF>(W, nr, ar, F, yb, wp);
            else if (nt == 2) p2_bf16<2, kRSMaxBF>(W, nr, ar, F, yb, wp);
            else p2_bf16<4, kRSMaxBF>(W, nr, ar, F, yb, wp);
        } else {
            const int8_t* W = reinterpret_cast<const int8_t*>(S);
            if (nt == 1) p2_q8<1, kRSMaxQ8>(W, nr, ar, F, yb, wp, sc);
            else p2_q8<4, kRSMaxQ8>(W, nr, ar, F, yb, wp, sc);
        }
    }
}

// Warp-wide copy of activation rows written by other SMs during this kernel (L2-coherent loads,
// eight 16-byte loads in flight per lane).  bytes is a multiple of 16.
__device__ __forceinline__ void copy_act_l2(unsigned char* dst, const unsigned char* src, uint32_t bytes) {
    const int lane = threadIdx.x & 31;
    uint32_t o = lane * 16;
    for (; o + 7 * 512 < bytes; o += 8 * 512) {
        uint4 v[8];
#pragma unroll
        for (int k = 0; k < 8; k++) v[k] = __ldcg(reinterpret_cast<const uint4*>(src + o + k * 512));
#pragma unroll
        for (int k = 0; k < 8; k++) *reinterpret_cast<uint4*>(dst + o + k * 512) = v[k];
    }
    for (; o < bytes; o += 512) *reinterpret_cast<uint4*>(dst + o) = __ldcg(reinterpret_cast<const uint4*>(src + o));
}

// Phase-2 stage cursor: stage k (0-based within phase 2) -> job j and first row.
struct P2Cursor {
    int j = 0, start = 0;
    __device__ __forceinline__ int stages_of(const Ctrl& c, const DecodeArgs& a, int jj) const {
        const int rs = c.sh.jkind[jj] == kKindBF16 ? a.rs_bf16 : a.rs_q8;
        const int hr = c.me.h1 - c.me.h0;
        return (hr + rs - 1) / rs;
    }
    __device__ __forceinline__ void seek(const Ctrl& c, const DecodeArgs& a, int k) {
        while (k >= start + stages_of(c, a, j)) {
            start += stages_of(c, a, j);
            j++;
        }
    }
};

// Phase-1 stage cursor: stage i -> (job, first unit f, units nu) through the segment table; callers
// visit stages in increasing order, so the segment index only moves forward.
struct SegCursor {
    int g = 0;
    __device__ __forceinline__ void at(const Ctrl& c, int i, int& j, int& f, int& nu) {
        while (i >= c.me.seg_stage[g + 1]) g++;
        j = c.me.seg_j[g];
        const int ups = c.me.seg_ups[g];
        f = c.me.seg_f0[g] + (i - c.me.seg_stage[g]) * ups;
        nu = min(ups, c.me.seg_fend[g] - f);
    }
};

__global__ void __launch_bounds__(kDecThreads, 1) decode_kernel(const DecodeArgs a) {
    extern __shared__ __align__(128) unsigned char smem[];
    Ctrl& c = *reinterpret_cast<Ctrl*>(smem);
    float* ybuf = reinterpret_cast<float*>(smem + a.off_ybuf);
    unsigned char* xreg = smem + a.off_x;
    unsigned char* ring = smem + a.off_ring;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int T = a.T, H = a.H, F = a.F, NS = a.NS;
    const int s = blockIdx.x;
    const int par = a.epoch & 1;
    uint32_t* ctr = a.ctr + par * kDecodeMaxPairs;

    uint64_t* tl = a.timeline ? a.timeline + (size_t)s * kTimelineSlots : nullptr;  // optional phase stamps
    if (tl && tid == 0) tl[0] = globaltimer_ns();

    // ---------------- prologue: barriers, then this call's plan (written by plan_kernel) ----------------
    if (tid == 0) {
        for (int i = 0; i < NS; i++) {
            mbar_init(&c.full[i], 1);
            mbar_init(&c.empty[i], 1);
            c.fill_seq[i] = -1;
        }
        mbar_init(&c.x_full, 1);
        mbar_init(&c.p1_done, kNWC);
        for (int b = 0; b < 2; b++) {
            c.act_job[b] = -1;
            c.act_done[b] = 0;
        }
        c.abort_flag = 0;
        c.ticket = 0;
        fence_mbar_init();
        // The plan kernel published the plan before launching this grid; the acquire makes it visible
        // (bounded in case the launch order was violated).
        const uint64_t dl = globaltimer_ns() + a.timeout_ns;
        while (ld_acquire_gpu(a.flag) != a.stamp)
            if (globaltimer_ns() > dl) {
                c.abort_flag = 1;
                atomicOr(a.err, kErrTimeout);
                break;
            }
    }
    __syncthreads();
    if (c.abort_flag) {  // no plan: write nothing, the call reports MOE_ETIMEOUT
        return;
    }
    {
        const int4* src = reinterpret_cast<const int4*>(&a.plan->sh);
        int4* dst = reinterpret_cast<int4*>(&c.sh);
        for (int q = tid; q < (int)(sizeof(PlanShared) / 16); q += kDecThreads) dst[q] = __ldcg(src + q);
        const int4* srcm = reinterpret_cast<const int4*>(&a.plan->cta[s]);
        int4* dstm = reinterpret_cast<int4*>(&c.me);
        for (int q = tid; q < (int)(sizeof(PlanCta) / 16); q += kDecThreads) dstm[q] = __ldcg(srcm + q);
    }
    __syncthreads();
    if (tid == 0) griddep_launch_dependents();
    if (tl && tid == 0) tl[1] = globaltimer_ns();

    const int n1 = c.me.n1, n2 = c.me.n2, ntot = n1 + n2;
    const uint32_t SB = a.slot_bytes;

    // ---------------- producer: bulk copies of this CTA's weights ----------------
    if (warp == kProdWarp) {
        if (lane == 0) {
            const uint64_t deadline = globaltimer_ns() + 4 * a.timeout_ns;
            const uint64_t pol = l2_evict_first();
            if (!a.x_f32) {  // bf16 x via one bulk copy (read by every CTA: default L2 policy)
                const uint32_t xb = (uint32_t)T * H * 2;
                mbar_arrive_expect_tx(&c.x_full, xb);
                bulk_g2s(xreg, a.x, xb, &c.x_full);
            }
            P2Cursor cur;
            SegCursor seg;
            int i = 0;
            for (; i < ntot; i++) {
                const int slot = i % NS;
                unsigned char* dst = ring + (size_t)slot * SB;
                if (tl && i == n1) tl[2] = globaltimer_ns();
                if (i >= NS && !wait_bar(&c.empty[slot], ((i / NS) & 1) ^ 1, c, a.err, deadline)) break;
                if (i < n1) {
                    int j, f, nu;
                    seg.at(c, i, j, f, nu);
                    const uint32_t rb = (uint32_t)H * esize(c.sh.jkind[j]);
                    const unsigned char* w1 = c.sh.jw1[j];
                    if (c.sh.jlayout[j] == kLayoutInterleaved) {  // nu units [gate|up] contiguous
                        mbar_arrive_expect_tx(&c.full[slot], 2 * rb * nu);
                        bulk_g2s(dst, w1 + (size_t)f * 2 * rb, 2 * rb * nu, &c.full[slot], pol);
                    } else {
                        mbar_arrive_expect_tx(&c.full[slot], 2 * rb);
                        bulk_g2s(dst, w1 + (size_t)f * rb, rb, &c.full[slot], pol);
                        bulk_g2s(dst + rb, w1 + (size_t)(F + f) * rb, rb, &c.full[slot], pol);
                    }
                } else {
                    const int k = i - n1;
                    cur.seek(c, a, k);
                    const int j = cur.j;
                    const int rs = c.sh.jkind[j] == kKindBF16 ? a.rs_bf16 : a.rs_q8;
                    const int row0 = (k - cur.start) * rs;
                    const int nr = min(rs, c.me.h1 - c.me.h0 - row0);
                    const uint32_t rowb = (uint32_t)F * esize(c.sh.jkind[j]);
                    mbar_arrive_expect_tx(&c.full[slot], nr * rowb);
                    bulk_g2s(dst, c.sh.jw2[j] + (size_t)(c.me.h0 + row0) * rowb, nr * rowb, &c.full[slot], pol);
                }
                *(volatile int*)&c.fill_seq[slot] = i / NS;  // consumers may now wait on this fill's phase
                if (a.stage_log && s == 0 && i < kStageLogMax) a.stage_log[i] = globaltimer_ns();
            }
            if (tl) tl[3] = globaltimer_ns();
            // every issued copy lands before this CTA may exit
            const uint64_t dd = globaltimer_ns() + a.timeout_ns;
            if (!a.x_f32) drain_bar(&c.x_full, 0, dd);
            for (int k = i > NS ? i - NS : 0; k < i; k++) drain_bar(&c.full[k % NS], (k / NS) & 1, dd);
        }
        return;
    }

    griddep_wait();  // the previous grid's act / counter / output writes are complete beyond this point
    const uint64_t deadline = globaltimer_ns() + a.timeout_ns;
    const uint32_t act_pitch = ((uint32_t)T * F * 2 + 127u) & ~127u;

    // ---------------- activation loader ----------------
    if (warp == kActWarp) {
        if (s == 0)  // housekeeping of CTA 0: clear the other parity's counters for the next call
            for (int q = lane; q < kDecodeMaxPairs; q += 32) a.ctr[(par ^ 1) * kDecodeMaxPairs + q] = 0;
        if (!wait_bar(&c.p1_done, 0, c, a.err, deadline)) return;
        if (tl && lane == 0) tl[13] = globaltimer_ns();
        if (c.me.h1 <= c.me.h0) return;
        const uint32_t target = (uint32_t)F + (a.inject_timeout ? 1u : 0u);
        if (a.act_resident) {
            // All jobs' activations fit in shared memory: poll every job's counter in parallel
            // (lane l owns jobs l, l + 32, ...), then stage all rows with one pass of 16-byte loads.
            int ok = 1;
            for (int j = lane; ok && j < c.sh.nj; j += 32)
                while (ld_acquire_gpu(&ctr[j]) < target) {
                    if (timed_out(c, a.err, deadline)) {
                        ok = 0;
                        break;
                    }
                    __nanosleep(64);
                }
            if (!__all_sync(0xffffffffu, ok)) return;
            if (tl && lane == 0) tl[12] = globaltimer_ns();
            for (int j = 0; j < c.sh.nj; j++) (void)ld_acquire_gpu(&ctr[j]);  // every lane acquires every job
            copy_act_l2(xreg, reinterpret_cast<const unsigned char*>(a.act), (uint32_t)c.sh.jp0[c.sh.nj] * F * 2);
            __threadfence_block();
            __syncwarp();
            if (lane == 0) *(volatile int*)&c.act_job[0] = INT_MAX;
            if (tl && lane == 0) tl[4] = globaltimer_ns();
            return;
        }
        // Rolling mode: job j's activations go to slot j & 1 once job j-2 is done with that slot.
        P2Cursor cur;
        for (int j = 0; j < c.sh.nj; j++) {
            const int b = j & 1;
            int ok = 1;
            if (lane == 0) {
                if (j >= 2) {
                    const int need = cur.stages_of(c, a, j - 2);
                    while (*(volatile int*)&c.act_done[b] < need)
                        if (timed_out(c, a.err, deadline)) {
                            ok = 0;
                            break;
                        }
                    c.act_done[b] = 0;
                }
                while (ok && ld_acquire_gpu(&ctr[j]) < target) {  // all F units of job j published grid-wide
                    if (timed_out(c, a.err, deadline)) {
                        ok = 0;
                        break;
                    }
                    __nanosleep(64);
                }
            }
            ok = __shfl_sync(0xffffffffu, ok, 0);
            if (!ok) return;
            (void)ld_acquire_gpu(&ctr[j]);
            const int p0 = c.sh.jp0[j], n = c.sh.jp0[j + 1] - p0;
            copy_act_l2(xreg + (size_t)b * act_pitch, reinterpret_cast<const unsigned char*>(a.act + (size_t)p0 * F),
                        (uint32_t)n * F * 2);
            __threadfence_block();
            __syncwarp();
            if (lane == 0) *(volatile int*)&c.act_job[b] = j;
        }
        return;
    }

    // ---------------- consumers ----------------
    int curj = -1, cnt = 0;
    bool p1_signalled = false;
    auto flush = [&]() {
        if (curj >= 0 && cnt > 0) {
            __threadfence();
            __syncwarp();
            if (lane == 0) atomicAdd(&ctr[curj], (uint32_t)cnt);
        }
        curj = -1;
        cnt = 0;
    };
    auto signal_p1 = [&]() {
        flush();
        __syncwarp();
        if (lane == 0) mbar_arrive(&c.p1_done);
        if (tl && warp == 0 && lane == 0) tl[5] = globaltimer_ns();
        p1_signalled = true;
    };
    P2Cursor cur;
    SegCursor seg;
    const int nwc = a.nwc;  // consumer warps taking ring stages
    bool ok = true;
    if (a.x_f32) {  // widen x to fp32 in shared memory once (all consumer warps), then meet
        const uint4* xs = reinterpret_cast<const uint4*>(a.x);
        float4* xd = reinterpret_cast<float4*>(xreg);
        for (int q = tid; q < T * H / 8; q += kNWC * 32) {
            const uint4 v = __ldg(xs + q);
            xd[2 * q] = make_float4(bf_lo(v.x), bf_hi(v.x), bf_lo(v.y), bf_hi(v.y));
            xd[2 * q + 1] = make_float4(bf_lo(v.z), bf_hi(v.z), bf_lo(v.w), bf_hi(v.w));
        }
        named_bar_sync(2, kNWC * 32);
    } else {
        ok = wait_bar(&c.x_full, 0, c, a.err, deadline);
    }
    long long cyc_wait[2] = {0, 0}, cyc_work[2] = {0, 0};  // timeline instrumentation (warp 0)
    // Stages are taken in ticket order (a stage that has landed goes to the next free warp).
    while (ok && warp < nwc) {
        int i = 0;
        if (lane == 0) i = atomicAdd(&c.ticket, 1);
        i = __shfl_sync(0xffffffffu, i, 0);
        if (i >= ntot) break;
        const int slot = i % NS, fill = i / NS;
        // publish finished gate/up units before anything that may wait on other CTAs' publications
        if (i >= n1 && !p1_signalled) signal_p1();
        const long long tw0 = tl ? clock64() : 0;
        // the slot's parity is only meaningful once this fill has been issued (fill_seq), so a warp
        // running ahead of the others never reads a phase from an older round of the ring
        int issued = 1;
        while (*(volatile int*)&c.fill_seq[slot] != fill)
            if (timed_out(c, a.err, deadline)) {
                issued = 0;
                break;
            }
        if (!__all_sync(0xffffffffu, issued)) break;
        if (!wait_bar(&c.full[slot], fill & 1, c, a.err, deadline)) break;
        const unsigned char* S = ring + (size_t)slot * SB;
        const long long tw1 = tl ? clock64() : 0;
        if (a.stage_log && s == 0 && lane == 0 && i < kStageLogMax) a.stage_log[kStageLogMax + i] = globaltimer_ns();
        if (i < n1) {
            int j, f, nu;
            seg.at(c, i, j, f, nu);
            if (j != curj) {
                flush();
                curj = j;
            }
            const size_t ub = (size_t)2 * H * esize(c.sh.jkind[j]);  // one unit = [gate row | up row] in the slot
            for (int k = 0; k < nu; k++) stage_p1(a, c, S + k * ub, xreg, j, f + k);
            cnt += nu;
        } else {
            const int k = i - n1;
            cur.seek(c, a, k);
            const int j = cur.j;
            const int rs = c.sh.jkind[j] == kKindBF16 ? a.rs_bf16 : a.rs_q8;
            const int row0 = (k - cur.start) * rs;
            const int nr = min(rs, c.me.h1 - c.me.h0 - row0);
            const int b = a.act_resident ? 0 : (j & 1);
            const int want = a.act_resident ? INT_MAX : j;
            int ready = 1;
            while (*(volatile int*)&c.act_job[b] != want)  // every lane observes the hand-off itself
                if (timed_out(c, a.err, deadline)) {
                    ready = 0;
                    break;
                }
            if (!__all_sync(0xffffffffu, ready)) break;
            __threadfence_block();
            if (tl) cyc_wait[1] += clock64() - tw1;  // act hand-off wait counts as waiting
            const unsigned char* A = a.act_resident ? xreg + (size_t)c.sh.jp0[j] * F * 2 : xreg + (size_t)b * act_pitch;
            stage_p2(a, c, ybuf, S, reinterpret_cast<const uint16_t*>(A), j, row0, nr);
            __syncwarp();
            if (lane == 0 && !a.act_resident) atomicAdd(&c.act_done[b], 1);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&c.empty[slot]);
        if (a.stage_log && s == 0 && lane == 0 && i < kStageLogMax) a.stage_log[2 * kStageLogMax + i] = globaltimer_ns();
        if (tl) {
            const int ph = i >= n1;
            cyc_wait[ph] += tw1 - tw0;
            cyc_work[ph] += clock64() - tw1;
        }
    }
    if (!p1_signalled) signal_p1();
    if (tl && warp == 0 && lane == 0) {
        tl[8] = (uint64_t)cyc_wait[0];
        tl[9] = (uint64_t)cyc_work[0];
        tl[10] = (uint64_t)cyc_wait[1];
        tl[11] = (uint64_t)(cyc_work[1] - cyc_wait[1]);
    }
    named_bar_sync(1, kNWC * 32);
    if (tl && tid == 0) tl[6] = globaltimer_ns();

    // ---------------- combine: out[t, h0:h1) in job order ----------------
    const int h0 = c.me.h0, hr = c.me.h1 - c.me.h0;
    for (int q = tid; q < T * hr; q += kNWC * 32) {
        const int t = q / hr, r = q % hr;
        float* o = a.out + (size_t)t * H + h0 + r;
        float acc = a.accumulate ? *o : 0.f;
        for (int m = 0; m < c.sh.tpn[t]; m++) acc += ybuf[(size_t)c.sh.tpair[t][m] * a.hr_max + r];
        *o = acc;
    }
    if (tl && tid == 0) tl[7] = globaltimer_ns();
}

static size_t up128(size_t v) { return (v + 127) / 128 * 128; }

bool plan_decode(DecodeArgs& a, int grid, size_t* smem_bytes) {
    if (a.T < 1 || a.T > kDecodeMaxT || a.H > 8192 || a.H % 64 || a.F % 64 || a.E > kMaxExperts || a.K > kMaxTopK)
        return false;
    if (std::min(a.E, a.T * a.K) > kDecodePlanJobs || grid < 1 || grid > kPlanMaxGrid) return false;
    const size_t slot = (size_t)4 * a.H;  // one bf16 gate/up unit
    a.slot_bytes = (uint32_t)slot;
    a.rs_bf16 = (int)std::min<size_t>(kRSMaxBF, slot / ((size_t)a.F * 2));
    a.rs_q8 = (int)std::min<size_t>(kRSMaxQ8, slot / (size_t)a.F);
    if (a.rs_bf16 < 1) return false;
    a.hr_max = (a.H + grid - 1) / grid;
    const size_t ctrl = up128(sizeof(Ctrl));
    const size_t ybuf = up128((size_t)a.T * a.K * a.hr_max * 4);
    const size_t act_pitch = up128((size_t)a.T * a.F * 2);
    a.x_f32 = a.T <= 4 ? 1 : 0;  // small batches keep x widened to fp32 in shared memory
    const size_t xrows = (size_t)a.T * a.H * (a.x_f32 ? 4 : 2);
    // Resident mode keeps every pair's activations in shared memory (no slot reuse) when that still
    // leaves room for an 8-deep ring; otherwise two rolling per-job slots.
    const size_t act_all = up128((size_t)a.T * a.K * a.F * 2);
    size_t xb = up128(std::max(xrows, act_all));
    a.act_resident = ctrl + ybuf + xb + 10 * slot <= kSmemCap ? 1 : 0;
    if (!a.act_resident) xb = up128(std::max(xrows, 2 * act_pitch));
    a.off_ybuf = (uint32_t)ctrl;
    a.off_x = (uint32_t)(ctrl + ybuf);
    a.off_ring = (uint32_t)(ctrl + ybuf + xb);
    const size_t fixed = ctrl + ybuf + xb;
    if (fixed + 2 * slot > kSmemCap) return false;
    // A warp takes stages i, i + nwc, ...; with NS a multiple of nwc the previous user of its ring
    // slot is the same warp, so no mbarrier is ever waited on more than one phase ahead.
    int ns = (int)std::min<size_t>(kMaxNS, (kSmemCap - fixed) / slot);
    if (a.ns_cap > 0) ns = std::min(ns, a.ns_cap);
    if (ns < 2) return false;
    a.nwc = a.nwc >= 1 && a.nwc <= kNWC ? a.nwc : kNWC;  // requested consumer warps (tuning), else all
    a.NS = ns;
    *smem_bytes = fixed + (size_t)a.NS * slot;
    return true;
}

cudaError_t decode_set_smem_limit() {
    return cudaFuncSetAttribute(decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemCap);
}

cudaError_t launch_decode(const DecodeArgs& a, int grid, size_t smem, cudaStream_t st) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kDecThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, decode_kernel, a);
}

}  // namespace moe
