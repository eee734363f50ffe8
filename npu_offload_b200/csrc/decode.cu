// Fused persistent decode kernel for the B200 MoE data plane: one launch per layer routes the call
// (plan.cuh: in every CTA, or published by a one-CTA planner kernel while the previous call streams)
// and performs the grouped SwiGLU expert GEMV (gate/up + down) and the weighted combine.
//
// Semantics are the reference's cold-expert path (solar_hybrid/cpu_moe.cpp:38-96, int8 weight-only
// form cpu_kern.c:306-333) behind the layer surface of track2_opt/solar_engine/src/main.rs:149-209:
//   g, u = gate/up rows . x_t (fp32)      act = bf16_rne(g / (1 + exp(-g)) * u)
//   out[t, h] = sum over the token's experts in job order of w * sum_f down[h, f] * act[f]
//
// Work split.  Expert tables hold one unit per intermediate index f: [gate row f | up row f | down
// column f].  A unit is self-contained -- act[f] needs only gate/up row f, and its contribution to
// the output is act[f] * down column f -- so the plan cuts the stream of all units of the call into
// one contiguous, cost-balanced share per CTA with no dependency between CTAs until the very end.
//   producer   one thread of its own warpgroup streams the CTA's units with 1-D bulk async copies
//              (TMA engine) into an NS-deep shared-memory ring guarded by mbarriers (L2 evict-first:
//              read once).  Issuing a copy can stall the issuing thread for a large part of a
//              microsecond, so no consumer ever issues one.
//   consumers  8 warps; warp w owns the hidden slice [w*H/8, (w+1)*H/8) of every row, a lane 8
//              consecutive elements per 256-element chunk.  Per batch of up to 2 units: partial
//              gate/up dots over the slice (packed f32x2 FMAs on 128-bit shared loads), a
//              multi-value butterfly inside the warp, an exchange of the 8 slice sums through shared
//              memory (one mbarrier phase), the sums added in slice order by every warp (identical
//              bits everywhere), SwiGLU + bf16 rounding, then y[t, slice] += act * down column.
//              x and y of the segment's token group (<= 4 tokens) stay in registers.
//   partials   at the end of a segment every warp stores its y slice as that segment's fp32 partial
//              sums (int8 experts: times the down-row scales).
//   reduction  after a grid-wide arrival counter, the last nred CTAs to arrive each own a slice of
//              output quads: per pair they add its group's segment partials in segment order, then
//              per token the pairs in job order, weighted -- a fixed order, so results are
//              deterministic for a given partition.  The other CTAs leave at once.
// Every wait is bounded (globaltimer); a timeout raises kErrTimeout, stops the CTA, drains the bulk
// copies in flight and returns.  Programmatic dependent launch lets the next call's CTAs take the SMs
// this grid frees and start streaming while its reducers finish; the call counters (DecodeArgs::cnt)
// order what one call writes and the next reads (partial sums, outputs, exchange buffers).
#include <climits>
#include <cstddef>

#include "common.cuh"
#include "decode.h"
#include "plan.cuh"
#include "ptx.cuh"

namespace moe {

// Warp roles: warpgroups 0-1 (warps 0-7) consume, one warp per hidden slice; warpgroup 2 (warps
// 8-11) produces -- lane 0 of warp 8 issues the bulk copies, warps 9-11 leave after the register
// hand-over.  Registers: launched at 168 per thread (384 * 168 = 64512), the producer warpgroup
// drops to 40 and the consumer warpgroups rise to 232: 128 * 40 + 256 * 232 = 64512.
constexpr int kCW = 8;
constexpr int kDecThreads = 12 * 32;
constexpr int kCThreads = kCW * 32;
constexpr int kProdRegs = 40, kConsRegs = 232;
static_assert(4 * 32 * kProdRegs + 8 * 32 * kConsRegs <= kDecThreads * 168, "register split exceeds the launch pool");
constexpr int kMaxNS = 16;
constexpr size_t kSmemCap = 227 * 1024;
constexpr uint32_t kStageTarget = 49152;  // default bytes per ring stage
// Default planning cost of an int8 unit, per mille of its bytes: the consumers spend about as long on
// an int8 unit's dequantising dots as on streaming a bf16 unit (measured on B200 at the Solar shape,
// batch 1, a layer of 96 int8 and 32 bf16 experts: 66.1 us per layer with shares cut by bytes, 49.6 us
// at 2500).
constexpr int kQ8CostDefault = 2500;
constexpr int kBatch = 4;  // units per exchange (a batch may span ring stages)
// Exchange buffers.  A warp writes buffer k % kXB for batch k + kXB after its exchange wait for batch
// k + kXB - 1, i.e. after every warp arrived for that batch; each warp arrives for batch k + 1 only
// after it has read the buffer of batch k.  Any kXB >= 2 is safe; 4 costs 4 KB of shared memory.
constexpr int kXB = 4;

struct __align__(16) Ctrl {
    uint64_t full[kMaxNS];
    uint64_t empty[kMaxNS];
    uint64_t xbar[kXB];     // slice-sum exchange of a batch (8 warp arrivals), batch % kXB
    int abort_flag;
    int ticket;             // this CTA's arrival order (-1: it gave up)
    int use_pub;            // the CTA took the published plan
    int pad;
    float red[kXB][kCW][32];  // slice sums of one batch, by batch % kXB
    PlanCta me;             // this CTA's share
    PlanShared sh;          // reduction tables
    CallPlan P;             // the call's routing and job structure (plan.cuh)
};
static_assert(offsetof(Ctrl, me) % 16 == 0 && offsetof(Ctrl, sh) % 16 == 0 && offsetof(Ctrl, P) % 16 == 0,
              "16-byte aligned plan structs");
static_assert(kDecThreads == kPlanThr, "the planning steps use every thread of the CTA");

__device__ __forceinline__ bool timed_out(Ctrl& c, uint32_t* err, uint64_t deadline) {
    if (*(volatile int*)&c.abort_flag) return true;
    if (globaltimer_ns() > deadline) {
        *(volatile int*)&c.abort_flag = 1;
        atomicOr(err, kErrTimeout);
        return true;
    }
    return false;
}

// Bounded mbarrier wait; false when the kernel is aborting.  Waiting threads sleep inside try_wait
// (100 us per attempt at most) rather than spin, so they do not take issue slots from working warps.
__device__ __forceinline__ bool wait_bar(uint64_t* bar, uint32_t parity, Ctrl& c, uint32_t* err, uint64_t deadline) {
    while (!mbar_try_wait_sleep(bar, parity, 100000u))
        if (timed_out(c, err, deadline)) return false;
    return true;
}

// Bounded wait used while draining copies: ignores the abort flag, only the deadline.
__device__ __forceinline__ void drain_bar(uint64_t* bar, uint32_t parity, uint64_t deadline) {
    while (!mbar_try_wait(bar, parity))
        if (globaltimer_ns() > deadline) return;
}

template <int N>
struct Pow2Up {
    static constexpr int v = N <= 1 ? 1 : N <= 2 ? 2 : N <= 4 ? 4 : N <= 8 ? 8 : N <= 16 ? 16 : 32;
};

struct LoopStat {
    long long wait = 0, work = 0, bar = 0, dots = 0, bfly = 0, act = 0, axpy = 0;
};

// 8 int8 weights (8 bytes of shared memory) as fp32 (exact).
__device__ __forceinline__ void load_q8_f32(uint32_t p, float (&w)[8]) {
    const uint2 v = lds64(p);
#pragma unroll
    for (int k = 0; k < 4; k++) {
        w[k] = i8f(v.x, k);
        w[4 + k] = i8f(v.y, k);
    }
}

// One segment: NT tokens, CH chunks of 8 elements per lane and row (FULL: every lane has all CH
// chunks, H == 2048 * CH).  stage = the CTA's ring stage counter, batch = its exchange counter (both
// advance across segments).  Returns false on abort.
//
// bf16 experts use the mixed-precision FMA on packed bf16 operands (x, weights and the bf16 SwiGLU
// output are never widened); int8 experts widen weights and x to fp32.  Either way every product
// and sum is the fp32 arithmetic of the widened values.
//
// Units are processed in batches of KB (one exchange per batch); a batch may span ring stages and a
// stage may hold several batches: a stage is waited for when the first of its units is needed and
// released once all of its units have been applied.  A full batch runs as one straight-line block
// so the units' independent FMA chains interleave.  (Overlapping a batch's exchange with the next
// batch's dot products measured slower than batches of 4 units: it holds more ring stages and adds
// bookkeeping.)
template <int CH, bool Q8, int NT, bool FULL>
__device__ bool run_segment(const DecodeArgs& a, Ctrl& c, const unsigned char* ring, const Seg& sg, int& stage,
                            int& batch, uint64_t deadline, LoopStat* ls) {
    constexpr int KB = CH <= 2 ? kBatch : 2;  // units per exchange (H > 4096: 2, for registers)
    constexpr int VP = Pow2Up<2 * KB * NT>::v;              // values exchanged per batch (padded)
    static_assert(2 * KB * NT <= 32, "one value per lane at most");
    constexpr int NA = NT == 1 ? 4 : 2;                     // accumulators per row and token
    constexpr int ES = Q8 ? 1 : 2;                          // bytes per weight element
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int H = a.H, NS = a.NS;
    const int slice = H / kCW;
    const int ub = (int)unit_bytes(Q8 ? kKindQ8 : kKindBF16, H);
    const int ups = Q8 ? a.ups_q8 : a.ups_bf16;
    const int nu = sg.nu;
    bool valid[CH];
    int eoff[CH];
#pragma unroll
    for (int cc = 0; cc < CH; cc++) {
        valid[cc] = FULL || cc * 256 + lane * 8 < slice;
        eoff[cc] = warp * slice + cc * 256 + lane * 8;
    }
    // x of the group's tokens as packed bf16 pairs; y accumulators in fp32
    uint32_t xw[NT][CH][4];
    float y[NT][CH][8];
#pragma unroll
    for (int t = 0; t < NT; t++)
#pragma unroll
        for (int cc = 0; cc < CH; cc++) {
            const uint4 xv = valid[cc] ? ld_cg_u4(a.x + (size_t)sg.tok[t] * H + eoff[cc])
                                       : make_uint4(0, 0, 0, 0);
            xw[t][cc][0] = xv.x;
            xw[t][cc][1] = xv.y;
            xw[t][cc][2] = xv.z;
            xw[t][cc][3] = xv.w;
#pragma unroll
            for (int e = 0; e < 8; e++) y[t][cc][e] = 0.f;
        }

    // Ring cursor over the segment's units: stage cst (absolute), its slot cslot, unit coff inside it.
    // Advanced with compare-and-wrap only (no division in the loop).
    const int stage0 = stage;
    const uint32_t ring_s = smem_u32(ring);
    int cst = stage0, cslot = stage0 % NS, coff = 0;
    int waited = stage0 - 1, released = stage0 - 1;
    auto wait_through = [&](int st) -> bool {  // stages <= st have landed
        while (waited < st) {
            ++waited;
            const long long t0 = ls ? clock64() : 0;
            int ws = waited - (waited / NS) * NS;
            if (!wait_bar(&c.full[ws], (waited / NS) & 1, c, a.err, deadline)) return false;
            if (ls) ls->wait += clock64() - t0;
            if (a.stage_log && blockIdx.x == 0 && warp == 0 && lane == 0 && waited < kStageLogMax)
                a.stage_log[kStageLogMax + waited] = globaltimer_ns();
        }
        return true;
    };
    auto release_below = [&](int st) {  // release stages < st
        if (released >= st - 1) return;
        __syncwarp();
        while (released < st - 1) {
            ++released;
            if (lane == 0) mbar_arrive(&c.empty[released % NS]);
            if (a.stage_log && blockIdx.x == 0 && warp == 0 && lane == 0 && released < kStageLogMax)
                a.stage_log[2 * kStageLogMax + released] = globaltimer_ns();
        }
    };

    // slice dot products of one unit: v[base + 2t] = gate . x_t, v[base + 2t + 1] = up . x_t
    auto unit_dots = [&](uint32_t U, float (&v)[VP], const int base) {
        float ag[NT][NA], au[NT][NA];
#pragma unroll
        for (int t = 0; t < NT; t++)
#pragma unroll
            for (int k = 0; k < NA; k++) ag[t][k] = au[t][k] = 0.f;
#pragma unroll
        for (int cc = 0; cc < CH; cc++) {
            if (!valid[cc]) continue;
            if (!Q8) {
                const uint4 g4 = lds128(U + (uint32_t)eoff[cc] * 2);
                const uint4 u4 = lds128(U + (uint32_t)(H + eoff[cc]) * 2);
                const uint32_t wg[4] = {g4.x, g4.y, g4.z, g4.w}, wu[4] = {u4.x, u4.y, u4.z, u4.w};
#pragma unroll
                for (int q = 0; q < 4; q++)
#pragma unroll
                    for (int t = 0; t < NT; t++) {
                        const int k0 = NA == 4 ? (q & 1) * 2 : 0;
                        fma_bf16x2(wg[q], xw[t][cc][q], ag[t][k0], ag[t][k0 + 1]);
                        fma_bf16x2(wu[q], xw[t][cc][q], au[t][k0], au[t][k0 + 1]);
                    }
            } else {
                // packed f32x2 FMAs: (even, odd) element pairs, the same bits as two fmaf
                float wg[8], wu[8];
                load_q8_f32(U + eoff[cc], wg);
                load_q8_f32(U + H + eoff[cc], wu);
#pragma unroll
                for (int q = 0; q < 4; q++) {
                    const f32x2 g2 = pack_f32x2(wg[2 * q], wg[2 * q + 1]), u2 = pack_f32x2(wu[2 * q], wu[2 * q + 1]);
#pragma unroll
                    for (int t = 0; t < NT; t++) {
                        const f32x2 x2 = bf16x2_to_f32x2(xw[t][cc][q]);
                        const int k0 = NA == 4 ? (q & 1) * 2 : 0;
                        f32x2 a2 = pack_f32x2(ag[t][k0], ag[t][k0 + 1]), b2 = pack_f32x2(au[t][k0], au[t][k0 + 1]);
                        a2 = ffma2(g2, x2, a2);
                        b2 = ffma2(u2, x2, b2);
                        unpack_f32x2(a2, ag[t][k0], ag[t][k0 + 1]);
                        unpack_f32x2(b2, au[t][k0], au[t][k0 + 1]);
                    }
                }
            }
        }
#pragma unroll
        for (int t = 0; t < NT; t++) {
            float gs = ag[t][0] + ag[t][1], us = au[t][0] + au[t][1];
            if (NA == 4) {
                gs += ag[t][2] + ag[t][3];
                us += au[t][2] + au[t][3];
            }
            v[base + 2 * t] = gs;
            v[base + 2 * t + 1] = us;
        }
    };
    // y[t, slice] += act[t] * down column of one unit (ab[t]: bf16 bits of act in the low half)
    auto unit_axpy = [&](uint32_t U, const uint32_t (&ab)[NT]) {
        const uint32_t D = U + 2u * H * ES;
#pragma unroll
        for (int cc = 0; cc < CH; cc++) {
            if (!valid[cc]) continue;
            if (!Q8) {
                const uint4 wd = lds128(D + (uint32_t)eoff[cc] * 2);
#pragma unroll
                for (int t = 0; t < NT; t++) {
                    fma_bf16x2_s(wd.x, ab[t], y[t][cc][0], y[t][cc][1]);
                    fma_bf16x2_s(wd.y, ab[t], y[t][cc][2], y[t][cc][3]);
                    fma_bf16x2_s(wd.z, ab[t], y[t][cc][4], y[t][cc][5]);
                    fma_bf16x2_s(wd.w, ab[t], y[t][cc][6], y[t][cc][7]);
                }
            } else {
                float wd[8];
                load_q8_f32(D + eoff[cc], wd);
#pragma unroll
                for (int t = 0; t < NT; t++) {
                    const float at = bf_lo(ab[t]);
                    const f32x2 a2 = pack_f32x2(at, at);
#pragma unroll
                    for (int e = 0; e < 8; e += 2) {
                        const f32x2 r = ffma2(pack_f32x2(wd[e], wd[e + 1]), a2, pack_f32x2(y[t][cc][e], y[t][cc][e + 1]));
                        unpack_f32x2(r, y[t][cc][e], y[t][cc][e + 1]);
                    }
                }
            }
        }
    };

    // pending batch: exchanged but not yet applied
    bool pend = false;
    int pnb = 0, pbatch = 0, pnext = 0;  // units, exchange number, stage of the unit after the batch
    uint32_t pptr[KB];
    // exchange wait + SwiGLU + down-column update of the pending batch, then stage releases
    auto finish = [&]() -> bool {
        const long long t2 = ls ? clock64() : 0;
        const int buf = pbatch % kXB;
        if (!wait_bar(&c.xbar[buf], (pbatch / kXB) & 1, c, a.err, deadline)) return false;
        const long long t3 = ls ? clock64() : 0;
        // every warp adds the 8 slice sums in slice order: identical bits in all warps
        float sum = 0.f;
        if (lane < VP) {
#pragma unroll
            for (int w = 0; w < kCW; w++) sum += c.red[buf][w][lane];
        }
        const float upv = __shfl_down_sync(0xffffffffu, sum, 1);
        uint32_t actb = 0;  // bf16 bits of act in the low half
        {
            const int item = lane >> 1, uu = item / NT;
            if (!(lane & 1) && lane < 2 * KB * NT && uu < pnb) {
                float g = sum, u = upv;
                if (Q8) {  // per-unit scales ride in the unit's trailer
                    uint32_t U = pptr[0];
#pragma unroll
                    for (int k = 1; k < KB; k++)
                        if (uu == k) U = pptr[k];
                    g *= lds_f32(U + 3u * H);
                    u *= lds_f32(U + 3u * H + 4u);
                }
                actb = swiglu_bf16(g, u);
            }
        }
        const long long t4 = ls ? clock64() : 0;
        uint32_t ab[KB][NT];
#pragma unroll
        for (int uu = 0; uu < KB; uu++)
#pragma unroll
            for (int t = 0; t < NT; t++) ab[uu][t] = __shfl_sync(0xffffffffu, actb, 2 * (uu * NT + t));
        if (pnb == KB) {
#pragma unroll
            for (int uu = 0; uu < KB; uu++) unit_axpy(pptr[uu], ab[uu]);
        } else {
#pragma unroll
            for (int uu = 0; uu < KB; uu++)
                if (uu < pnb) unit_axpy(pptr[uu], ab[uu]);
        }
        release_below(pnext);
        if (ls) {
            const long long t5 = clock64();
            ls->bar += t3 - t2;
            ls->act += t4 - t3;
            ls->axpy += t5 - t4;
        }
        pend = false;
        return true;
    };

    for (int i0 = 0; i0 < nu; i0 += KB, batch++) {
        const int nb = min(KB, nu - i0);
        uint32_t uptr[KB];
        int last_st = cst;
#pragma unroll
        for (int uu = 0; uu < KB; uu++) {
            uptr[uu] = ring_s + (uint32_t)cslot * a.slot_bytes + (uint32_t)coff * ub;
            if (uu < nb) {
                last_st = cst;
                if (++coff == ups) {
                    coff = 0;
                    ++cst;
                    if (++cslot == NS) cslot = 0;
                }
            }
        }
        if (!wait_through(last_st)) return false;
        const long long tbs = ls ? clock64() : 0;
        float v[VP];
#pragma unroll
        for (int k = 0; k < VP; k++) v[k] = 0.f;
        if (nb == KB) {
#pragma unroll
            for (int uu = 0; uu < KB; uu++) unit_dots(uptr[uu], v, 2 * NT * uu);
        } else {
#pragma unroll
            for (int uu = 0; uu < KB; uu++)
                if (uu < nb) unit_dots(uptr[uu], v, 2 * NT * uu);
        }
        const long long tb0 = ls ? clock64() : 0;
        // slice sums: value i ends in the lanes of group i (32 / VP lanes each)
        const float tot = warp_sum_multi<VP>(v);
        const int buf = batch % kXB;
        if ((lane & (32 / VP - 1)) == 0) c.red[buf][warp][lane / (32 / VP)] = tot;
        __syncwarp();
        if (lane == 0) mbar_arrive(&c.xbar[buf]);
        if (ls) {
            const long long tb1 = clock64();
            ls->dots += tb0 - tbs;
            ls->bfly += tb1 - tb0;
        }
        pend = true;
        pnb = nb;
        pbatch = batch;
        pnext = cst;  // stages < cst hold only units of this batch or earlier
#pragma unroll
        for (int uu = 0; uu < KB; uu++) pptr[uu] = uptr[uu];
        if (!finish()) return false;
    }
    release_below(waited + 1);
    stage = waited + 1;
    // the segment's partial sums: part[gidx][t][h] (int8: times the down-row scales)
    float* P = a.part + (size_t)sg.gidx * kGroupMax * H;
#pragma unroll
    for (int t = 0; t < NT; t++)
#pragma unroll
        for (int cc = 0; cc < CH; cc++) {
            if (!valid[cc]) continue;
            float o[8];
#pragma unroll
            for (int e = 0; e < 8; e++) o[e] = y[t][cc][e];
            if (Q8) {
                const float4 s0 = __ldg(reinterpret_cast<const float4*>(sg.sc + 2 * a.F + eoff[cc]));
                const float4 s1 = __ldg(reinterpret_cast<const float4*>(sg.sc + 2 * a.F + eoff[cc] + 4));
                o[0] *= s0.x, o[1] *= s0.y, o[2] *= s0.z, o[3] *= s0.w;
                o[4] *= s1.x, o[5] *= s1.y, o[6] *= s1.z, o[7] *= s1.w;
            }
            float4* d = reinterpret_cast<float4*>(P + (size_t)t * H + eoff[cc]);
            d[0] = make_float4(o[0], o[1], o[2], o[3]);
            d[1] = make_float4(o[4], o[5], o[6], o[7]);
        }
    return true;
}

template <int CH, bool FULL>
__device__ bool run_segment_nt(const DecodeArgs& a, Ctrl& c, const unsigned char* ring, const Seg& sg, int& stage,
                               int& batch, uint64_t deadline, LoopStat* ls) {
    const bool q8 = sg.kind == kKindQ8;
#define MOE_SEG(NT_) (q8 ? run_segment<CH, true, NT_, FULL>(a, c, ring, sg, stage, batch, deadline, ls) \
                         : run_segment<CH, false, NT_, FULL>(a, c, ring, sg, stage, batch, deadline, ls))
    if (CH == 4) return sg.nt == 1 ? MOE_SEG(1) : MOE_SEG(2);  // H > 4096: groups of at most 2 tokens
    switch (sg.nt) {
        case 1: return MOE_SEG(1);
        case 2: return MOE_SEG(2);
        case 3: return MOE_SEG(3);
        default: return MOE_SEG(4);
    }
#undef MOE_SEG
}

template <int CH>
__device__ bool run_segment_any(const DecodeArgs& a, Ctrl& c, const unsigned char* ring, const Seg& sg, int& stage,
                                int& batch, uint64_t deadline, LoopStat* ls) {
    if (a.H == 2048 * CH) return run_segment_nt<CH, true>(a, c, ring, sg, stage, batch, deadline, ls);
    return run_segment_nt<CH, false>(a, c, ring, sg, stage, batch, deadline, ls);
}

// Cross-rank combine of output quads [q0, q0 + nq) of tokens [0, T) (see EpExchange): mine[t * nq + q]
// holds this rank's sums in shared memory; out receives (accumulate ? out : 0) + the partials of ranks
// 0..world-1 added in that order.  The nthr threads of named barrier 1 take part.  Returns false when
// a rank's values did not arrive in time (kErrTimeout raised, *abort set).
__device__ bool ep_combine(const EpExchange& ep, const float4* mine, float* out, int T, int H, int q0, int nq,
                           int accumulate, uint32_t* err, uint64_t deadline, int nthr, int* abort) {
    const int tid = threadIdx.x, W = ep.world, par = ep.epoch & 1;
    const int nv = nq * 4, ne = T * nv;  // values of the slice per token, of the slice
    const uint64_t tag = (uint64_t)ep.epoch << 32;
    const float* mv = reinterpret_cast<const float*>(mine);
    for (int f = tid; f < W * ne; f += nthr) {  // this rank's values into every rank's buffer
        const int r = f / ne, i = f - r * ne, t = i / nv, j = i - t * nv;
        uint64_t* dst = ep.peer_x[r] + ((size_t)(par * W + ep.rank) * ep.tstride + t) * H + 4 * q0 + j;
        st_relaxed_sys_u64(dst, tag | __float_as_uint(mv[i]));
    }
    bool ok = true;
    for (int i = tid; i < ne; i += nthr) {  // every rank adds the same values in rank order
        const int t = i / nv, j = i - t * nv;
        float* o = out + (size_t)t * H + 4 * q0 + j;
        float acc = accumulate ? *o : 0.f;
        for (int r = 0; r < W && ok; r++) {
            const uint64_t* src = ep.x_local + ((size_t)(par * W + r) * ep.tstride + t) * H + 4 * q0 + j;
            uint64_t w = ld_relaxed_sys_u64(src);
            for (int spin = 0; (uint32_t)(w >> 32) != ep.epoch; spin++) {
                if ((spin & 31) == 31 && (*(volatile int*)abort || globaltimer_ns() > deadline)) {
                    atomicOr(err, kErrTimeout);
                    *(volatile int*)abort = 1;
                    ok = false;
                    break;
                }
                __nanosleep(32);
                w = ld_relaxed_sys_u64(src);
            }
            acc += __uint_as_float((uint32_t)w);
        }
        if (ok) *o = acc;
    }
    named_bar_sync(1, nthr);
    return !*(volatile int*)abort;
}

template <int CH>
__global__ void __launch_bounds__(kDecThreads, 1) decode_kernel(const DecodeArgs a) {
    extern __shared__ __align__(128) unsigned char smem[];
    Ctrl& c = *reinterpret_cast<Ctrl*>(smem);
    unsigned char* ring = smem + a.off_ring;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int NS = a.NS, G = gridDim.x;
    const int s = blockIdx.x;

    uint64_t* tl = a.timeline ? a.timeline + (size_t)s * kTimelineSlots : nullptr;  // optional phase stamps
    if (tl && tid == 0) tl[0] = globaltimer_ns();
    // CTA 0 leaves the call's error bits in host memory when asked to (host callers read it after
    // their stream synchronisation instead of copying the device word back)
    auto snapshot_err = [&]() {
        if (a.err_host && s == 0 && tid == 0) *(volatile uint32_t*)a.err_host = atomicOr(a.err, 0u);
    };

    // ---------------- prologue: barriers, inputs, the call's plan ----------------
    if (tid == 0) {
        for (int i = 0; i < NS; i++) {
            mbar_init(&c.full[i], 1);
            mbar_init(&c.empty[i], kCW);
        }
        for (int b = 0; b < kXB; b++) mbar_init(&c.xbar[b], kCW);
        c.abort_flag = 0;
        fence_mbar_init();
        // the next call's CTAs may take the SMs this grid frees; they wait below for its completion
        griddep_launch_dependents();
    }
    // Routing reads only the router logits, the bias and the expert table, which no decode grid
    // writes, so the plan is made while the previous grid of the stream still finishes.  Everything
    // that grid may touch (hidden states, partial sums, counters, outputs) waits for its completion
    // (griddepcontrol.wait) first: host calls here, the consumers before their first segment.
    if (a.x_src) {  // host call: the pinned inputs move to the device
        griddep_wait();
        // the logits, which every CTA's plan needs: CTA 0 copies them (16-byte reads) and publishes
        // the call's number; every CTA copies a slice of the hidden states, which only the consumers
        // read, after planning (waited for there).  (Each CTA reading the pinned logits itself queued
        // 147 CTAs' small reads on the host link: plan ready at 22 us, measured.)
        if (s == 0) {  // both buffers 16-byte aligned (the host stages unaligned pinned logits)
            const int nl = a.T * a.E, nl4 = nl / 4;
            float4* ld = reinterpret_cast<float4*>(const_cast<float*>(a.logits));
            const float4* ls = reinterpret_cast<const float4*>(a.lg_src);
            for (int i = tid; i < nl4; i += kDecThreads) ld[i] = ls[i];
            for (int i = 4 * nl4 + tid; i < nl; i += kDecThreads) const_cast<float*>(a.logits)[i] = a.lg_src[i];
            __threadfence();
            __syncthreads();
            if (tid == 0) asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(a.hctr + 1), "r"(a.hidx + 1u) : "memory");
        }
        const int nx = a.T * a.H / 8;
        const int x0 = (int)((long long)s * nx / G), x1 = (int)((long long)(s + 1) * nx / G);
        uint4* xd = reinterpret_cast<uint4*>(const_cast<uint16_t*>(a.x));
        const uint4* xs = reinterpret_cast<const uint4*>(a.x_src);
        for (int i = x0 + tid; i < x1; i += kDecThreads) xd[i] = xs[i];
        __threadfence();
        __syncthreads();
        if (tid == 0) {
            atomicAdd(a.hctr, 1u);  // this CTA's slice of the hidden states is in place
            const uint64_t dl = globaltimer_ns() + a.timeout_ns;
            while ((int)(ld_acquire_gpu(a.hctr + 1) - (a.hidx + 1u)) < 0) {  // the logits are in place
                if (globaltimer_ns() > dl) {
                    c.abort_flag = 1;
                    atomicOr(a.err, kErrTimeout);
                    break;
                }
                __nanosleep(32);
            }
        }
    }
    // A call with a planner always takes the published plan (only the planner may cut late shares,
    // so every CTA of the call must see its cut); a call without one plans in every CTA.
    if (tid == 0) {
        c.use_pub = 0;
        if (a.pub) {
            const uint64_t dl = globaltimer_ns() + a.timeout_ns;
            while (ld_acquire_gpu(a.pub_flag) != a.stamp) {
                if (globaltimer_ns() > dl) {
                    c.abort_flag = 1;
                    atomicOr(a.err, kErrTimeout);
                    break;
                }
                __nanosleep(64);
            }
            c.use_pub = 1;
        }
    }
    __syncthreads();  // also makes the barrier initialisation visible
    if (c.abort_flag) {  // the inputs never arrived: write nothing, the call reports MOE_ETIMEOUT
        snapshot_err();
        return;
    }
    if (c.use_pub) {  // the planner got ahead: this CTA's share, as published
        if (tl && tid == 0) tl[6] = 1;  // (timeline: marks a published plan; plan_call stamps slot 6 otherwise)
        const int4* src = reinterpret_cast<const int4*>(&a.pub->cta[s]);
        int4* dst = reinterpret_cast<int4*>(&c.me);
        for (int q = tid; q < (int)(sizeof(PlanCta) / 16); q += kDecThreads) dst[q] = __ldcg(src + q);
    } else {
        PlanIn pin;
        pin.logits = a.logits;
        pin.bias = a.bias;
        pin.desc = a.desc;
        pin.shared = a.shared;
        pin.idx_out = a.idx_out;
        pin.w_out = a.w_out;
        pin.err = a.err;
        pin.T = a.T;
        pin.E = a.E;
        pin.K = a.K;
        pin.H = a.H;
        pin.F = a.F;
        pin.scoring = a.scoring;
        pin.G = G;
        pin.gmax = a.gmax;
        pin.ups_bf16 = a.ups_bf16;
        pin.ups_q8 = a.ups_q8;
        pin.q8_cost = a.q8_cost;
        pin.nlate = a.nlate;  // applied when the call is streamed (the previous call's reducers hold SMs)
        pin.late_cost = a.late_cost;
        pin.nred = a.nred;
        pin.decide = a.decide;
        pin.cnt1 = &a.cnt[1];
        pin.epoch = a.epoch;
        // the planning scratch aliases the ring: no copy is issued before plan_call returns
        plan_call(pin, c.P, *reinterpret_cast<PlanScratch*>(ring), c.sh, c.me, tl);
    }
    fence_proxy_async_smem();  // generic accesses of the ring before the bulk copies overwrite it
    __syncthreads();
    if (tl && tid == 0) tl[1] = globaltimer_ns();
    const int nseg = c.me.nseg;
    // ---------------- producer warpgroup: bulk copies of this CTA's units ----------------
    if (warp >= kCW) {
        setmaxnreg_dec<kProdRegs>();
        if (warp == kCW && lane == 0) {
            const uint64_t deadline = globaltimer_ns() + 4 * a.timeout_ns;
            const uint64_t pol = l2_evict_first();
            int stage = 0;
            bool ok = true;
            for (int k = 0; ok && k < nseg; k++) {
                const Seg& sg = c.me.seg[k];
                const uint32_t ub = (uint32_t)unit_bytes(sg.kind, a.H);
                const int ups = sg.kind == kKindQ8 ? a.ups_q8 : a.ups_bf16;
                for (int u = 0; u < sg.nu; u += ups, stage++) {
                    const int slot = stage % NS;
                    if (stage >= NS && !wait_bar(&c.empty[slot], ((stage / NS) & 1) ^ 1, c, a.err, deadline)) {
                        ok = false;
                        break;
                    }
                    const uint32_t bytes = (uint32_t)min(ups, sg.nu - u) * ub;
                    mbar_arrive_expect_tx(&c.full[slot], bytes);
                    bulk_g2s(ring + (size_t)slot * a.slot_bytes, sg.src + (size_t)u * ub, bytes, &c.full[slot], pol);
                    if (a.stage_log && s == 0 && stage < kStageLogMax) a.stage_log[stage] = globaltimer_ns();
                }
            }
            if (tl) tl[2] = globaltimer_ns();
            // every issued copy lands before this CTA may exit
            const uint64_t dd = globaltimer_ns() + a.timeout_ns;
            for (int k = stage > NS ? stage - NS : 0; k < stage; k++) drain_bar(&c.full[k % NS], (k / NS) & 1, dd);
        }
        return;
    }

    // ---------------- consumer warpgroups ----------------
    setmaxnreg_inc<kConsRegs>();
    const uint64_t deadline = globaltimer_ns() + a.timeout_ns;
    const unsigned long long cbase = (unsigned long long)a.epoch * (unsigned long long)G;
    // Partial sums alternate between two buffers by call parity (the host passes call e's buffer).
    // Call e - 2, the last user of this call's buffer, has staged its partial sums
    // (cnt[2] >= (e - 1) * G): the buffer is free.  The previous call may still be arriving and
    // reducing (this call's reducers wait for it below).
    float* const part = a.part;
    if (tid == 0) {
        const unsigned long long free_at = cbase >= (unsigned long long)G ? cbase - (unsigned long long)G : 0ull;
        while (ld_acquire_gpu_u64(&a.cnt[2]) < free_at) {
            if (timed_out(c, a.err, deadline)) break;
            __nanosleep(32);
        }
        // host calls: every CTA's slice of the hidden states is on the device
        while (a.x_src && (int)(ld_acquire_gpu(a.hctr) - (a.hbase + (uint32_t)G)) < 0) {
            if (timed_out(c, a.err, deadline)) break;
            __nanosleep(32);
        }
    }
    named_bar_sync(1, kCThreads);
    LoopStat st, *ls = (tl && warp == 0) ? &st : nullptr;
    int stage = 0, batch = 0;
    bool ok = true;
    for (int k = 0; ok && k < nseg; k++) {
        const Seg& sg = c.me.seg[k];
        ok = run_segment_any<CH>(a, c, ring, sg, stage, batch, deadline, ls);
    }
    if (tl && warp == 0 && lane == 0) {
        tl[3] = globaltimer_ns();
        tl[8] = (uint64_t)st.wait;
        tl[9] = (uint64_t)st.work;
        tl[10] = (uint64_t)st.bar;
        tl[11] = (uint64_t)st.dots;
        tl[12] = (uint64_t)st.bfly;
        tl[13] = (uint64_t)st.act;
        tl[14] = (uint64_t)st.axpy;
    }
    // ---------------- arrival: a ticket per CTA; the last nred CTAs to arrive reduce ----------------
    // A CTA whose partial sums are written takes a ticket and, unless it is among the last nred to
    // arrive, exits at once: its SM is free for the next call (whose CTAs plan and start their weight
    // stream while this call's reduction finishes).  Reducer r owns output quads [r*H/4/nred, ...).
    // Arrival counts alternate by call parity (cnt[0] even calls, cnt[3] odd calls): a CTA of the next
    // call can finish its share before a straggler of this call arrives.  Call e owns the counts
    // [(e / 2) * G, (e / 2 + 1) * G) of its counter.
    unsigned long long* const arr = &a.cnt[(a.epoch & 1) ? 3 : 0];
    const unsigned long long abase = (unsigned long long)(a.epoch >> 1) * (unsigned long long)G;
    __threadfence();
    named_bar_sync(1, kCThreads);
    if (tid == 0) c.ticket = ok && !*(volatile int*)&c.abort_flag ? (int)(atomicAdd(arr, 1ull) - abase) : -1;
    named_bar_sync(1, kCThreads);
    const int NR = min(max(c.me.nred, 1), G), tk = c.ticket;
    if (tk < 0) {  // gave up (its error is raised): leave the error bits for host callers
        if (tid == 0) griddep_wait();
        if (a.err_host && tid == 0) *(volatile uint32_t*)a.err_host = atomicOr(a.err, 0u);
        return;
    }
    // Every CTA of a call adds one to cnt[2] (partial sums read, or none to read) and one to cnt[1]
    // (outputs written, or none to write); the CTA that completes cnt[1] leaves the call's error bits
    // for host callers.
    auto count_finished = [&]() {
        if (atomicAdd(&a.cnt[1], 1ull) == cbase + (unsigned long long)(G - 1) && a.err_host) {
            // host callers: the error bits, then the call's completion tag (every CTA's outputs were
            // made visible system-wide before its count)
            *(volatile uint32_t*)a.err_host = atomicOr(a.err, 0u);
            __threadfence_system();
            asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(a.err_host + 1), "r"(a.epoch + 1u) : "memory");
        }
    };
    if (tk < G - NR) {  // not a reducer: its SM is free for the next call
        if (tid == 0) {
            atomicAdd(&a.cnt[2], 1ull);
            griddep_wait();  // this grid completes after its predecessor (the call's planner)
            count_finished();
        }
        if (tl && tid == 0) tl[4] = tl[5] = globaltimer_ns();
        return;
    }
    const int rr = tk - (G - NR);
    auto reducer_done = [&]() {
        // this reducer's outputs before its count (the next call waits for the count; for host
        // callers the CTA that counts last fences at system scope before the completion tag, which
        // covers every output ordered before its count)
        __threadfence();
        named_bar_sync(1, kCThreads);
        if (tid == 0) {
            griddep_wait();  // this grid completes after its predecessor (the call's planner)
            count_finished();
        }
    };
    // the reduction's segment tables (the same in every CTA) while the last CTAs arrive: published
    // with the plan, or built here
    if (c.use_pub) {
        const int4* s1 = reinterpret_cast<const int4*>(&a.pub->sh);
        int4* d1 = reinterpret_cast<int4*>(&c.sh);
        for (int q = tid; q < (int)(sizeof(PlanShared) / 16); q += kCThreads) d1[q] = __ldcg(s1 + q);
        const int4* s2 = reinterpret_cast<const int4*>(&a.pub->P);
        int4* d2 = reinterpret_cast<int4*>(&c.P);
        for (int q = tid; q < (int)(sizeof(CallPlan) / 16); q += kCThreads) d2[q] = __ldcg(s2 + q);
    } else {
        plan_tables(c.P, c.sh, G, a.F, a.H, a.gmax, tid, kCThreads, 1);
    }
    named_bar_sync(1, kCThreads);

    if (tid == 0) {
        const unsigned long long target = abase + (unsigned long long)G + (a.inject_timeout ? 1ull : 0ull);
        while (!*(volatile int*)&c.abort_flag && ld_acquire_gpu_u64(arr) < target) {
            if (timed_out(c, a.err, deadline)) break;
            __nanosleep(32);
        }
    } else if (tid == 32) {
        // meanwhile: the previous calls' reducers are done with the outputs and the exchange buffer
        // (this call writes them only after staging, below)
        while (!*(volatile int*)&c.abort_flag && ld_acquire_gpu_u64(&a.cnt[1]) < cbase) {
            if (globaltimer_ns() > deadline) {
                *(volatile int*)&c.abort_flag = 1;
                atomicOr(a.err, kErrTimeout);
                break;
            }
            __nanosleep(32);
        }
    }
    named_bar_sync(1, kCThreads);
    if (*(volatile int*)&c.abort_flag) {
        if (tid == 0) atomicAdd(&a.cnt[2], 1ull);
        reducer_done();
        return;
    }
    if (tl && tid == 0) tl[4] = globaltimer_ns();

    // ---------------- reduction of output quads [q0, q0 + nq) ----------------
    const int H = a.H, H4 = H / 4;
    const int q0 = (int)((long long)rr * H4 / NR), nq = (int)((long long)(rr + 1) * H4 / NR) - q0;
    const int nsegtot = min(c.sh.nsegtot, kMaxSegTotal), np = min(c.sh.np, kDecodeMaxPairs);
    const int nrows = c.sh.srow0[nsegtot];
    float4* Q = reinterpret_cast<float4*>(ring);       // [nrows][nq] staged partial sums of the quads
    float4* R = Q + (size_t)nrows * nq;                // [np][nq] per-pair sums
    {   // every segment row's quads into shared memory: eight tasks of up to kGroupMax loads per thread in flight
        constexpr int U = 8;
        const int ntask = nsegtot * nq;
        for (int f0 = tid; f0 < ntask; f0 += U * kCThreads) {
            float4 v[U][kGroupMax];
#pragma unroll
            for (int u = 0; u < U; u++) {
                const int f = f0 + u * kCThreads;
                if (f < ntask) {
                    const int k = f / nq, q = f % nq, rows = c.sh.segrows[k];
                    const float4* src =
                        reinterpret_cast<const float4*>(part + (size_t)c.P.segslot[k] * kGroupMax * H) + q0 + q;
#pragma unroll
                    for (int i = 0; i < kGroupMax; i++)
                        if (i < rows) v[u][i] = __ldcg(src + (size_t)i * H4);
                }
            }
#pragma unroll
            for (int u = 0; u < U; u++) {
                const int f = f0 + u * kCThreads;
                if (f < ntask) {
                    const int k = f / nq, q = f % nq, rows = c.sh.segrows[k], r0 = c.sh.srow0[k];
#pragma unroll
                    for (int i = 0; i < kGroupMax; i++)
                        if (i < rows) Q[(size_t)(r0 + i) * nq + q] = v[u][i];
                }
            }
        }
    }
    named_bar_sync(1, kCThreads);
    if (tl && tid == 0) tl[19] = globaltimer_ns();
    if (tid == 0) atomicAdd(&a.cnt[2], 1ull);  // this reducer's partial sums are read: the next call may overwrite them
    for (int f = tid; f < np * nq; f += kCThreads) {
        const int p = f / nq, q = f % nq, g = min(max(c.sh.pgrp[p], 0), kMaxGroups - 1);
        const int row = min(max(c.sh.prow[p], 0), kGroupMax - 1);
        const int k0 = max(c.sh.gvs0[g], 0), k1 = min(c.sh.gvs1[g], nsegtot);
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int k = k0; k < k1; k++) {
            const float4 v = Q[(size_t)(c.sh.srow0[k] + row) * nq + q];
            acc.x += v.x;
            acc.y += v.y;
            acc.z += v.z;
            acc.w += v.w;
        }
        R[(size_t)p * nq + q] = acc;
    }
    named_bar_sync(1, kCThreads);
    if (a.ep.world > 1) {  // expert parallel: this rank's slice sums, then the cross-rank combine
        float4* mine = R + (size_t)np * nq;  // [T][nq]
        for (int f = tid; f < a.T * nq; f += kCThreads) {
            const int t = f / nq, q = f % nq;
            float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
            const int npt = min(c.sh.tpn[t], kMaxTopK);
            for (int m = 0; m < npt; m++) {
                const int p = min(max(c.sh.tpair[t][m], 0), np - 1);
                const float w = c.sh.pw[p];
                const float4 v = R[(size_t)p * nq + q];
                acc.x = fmaf(w, v.x, acc.x);
                acc.y = fmaf(w, v.y, acc.y);
                acc.z = fmaf(w, v.z, acc.z);
                acc.w = fmaf(w, v.w, acc.w);
            }
            mine[f] = acc;
        }
        named_bar_sync(1, kCThreads);
        if (tl && tid == 0) tl[20] = globaltimer_ns();
        ep_combine(a.ep, mine, a.out, a.T, H, q0, nq, a.accumulate, a.err, deadline, kCThreads, &c.abort_flag);
        if (tl && tid == 0) tl[5] = globaltimer_ns();
        reducer_done();
        return;
    }
    if (a.block) {  // MoE block: residual and combine into the next layer's input (combine.rs:1)
        const int sp0 = min(max(c.sh.sp0, 0), np - a.T);
        for (int f = tid; f < a.T * nq; f += kCThreads) {
            const int t = f / nq, q = f % nq;
            const size_t e0 = (size_t)t * H + 4 * (size_t)(q0 + q);  // first of the quad's 4 elements
            float r[4] = {0.f, 0.f, 0.f, 0.f};
            const int npt = min(c.sh.tpn[t], kMaxTopK);
            for (int m = 0; m < npt; m++) {
                const int p = min(max(c.sh.tpair[t][m], 0), np - 1);
                const float w = c.sh.pw[p];
                const float4 v = R[(size_t)p * nq + q];
                r[0] = fmaf(w, v.x, r[0]);
                r[1] = fmaf(w, v.y, r[1]);
                r[2] = fmaf(w, v.z, r[2]);
                r[3] = fmaf(w, v.w, r[3]);
            }
            const float4 sv = R[(size_t)(sp0 + t) * nq + q];
            const float sh[4] = {sv.x, sv.y, sv.z, sv.w};
            const uint2 xv = *reinterpret_cast<const uint2*>(a.x2 + e0);
            const float x2v[4] = {bf_lo(xv.x), bf_hi(xv.x), bf_lo(xv.y), bf_hi(xv.y)};
            float ex[4] = {0.f, 0.f, 0.f, 0.f};
            if (a.extra) {
                const float4 ev = *reinterpret_cast<const float4*>(a.extra + e0);
                ex[0] = ev.x, ex[1] = ev.y, ex[2] = ev.z, ex[3] = ev.w;
            }
            uint16_t yb[4], xb[4];
#pragma unroll
            for (int k = 0; k < 4; k++) {
                yb[k] = f2bf(x2v[k] + sh[k]);  // y = bf16(x2 + shared): shared.rs:2
                const float y = bf_lo(yb[k]);
                xb[k] = f2bf((a.extra ? y + ex[k] : y) + r[k]);
            }
            *reinterpret_cast<uint2*>(a.x_next + e0) =
                make_uint2((uint32_t)xb[0] | ((uint32_t)xb[1] << 16), (uint32_t)xb[2] | ((uint32_t)xb[3] << 16));
            if (a.y_out)
                *reinterpret_cast<uint2*>(a.y_out + e0) =
                    make_uint2((uint32_t)yb[0] | ((uint32_t)yb[1] << 16), (uint32_t)yb[2] | ((uint32_t)yb[3] << 16));
        }
        if (tl && tid == 0) tl[5] = globaltimer_ns();
        reducer_done();
        return;
    }
    for (int f = tid; f < a.T * nq; f += kCThreads) {
        const int t = f / nq, q = f % nq;
        float4* o = reinterpret_cast<float4*>(a.out + (size_t)t * H) + q0 + q;
        float4 acc = a.accumulate ? *o : make_float4(0.f, 0.f, 0.f, 0.f);
        const int npt = min(c.sh.tpn[t], kMaxTopK);
        for (int m = 0; m < npt; m++) {
            const int p = min(max(c.sh.tpair[t][m], 0), np - 1);
            const float w = c.sh.pw[p];
            const float4 v = R[(size_t)p * nq + q];
            acc.x = fmaf(w, v.x, acc.x);
            acc.y = fmaf(w, v.y, acc.y);
            acc.z = fmaf(w, v.z, acc.z);
            acc.w = fmaf(w, v.w, acc.w);
        }
        *o = acc;
    }
    if (tl && tid == 0) tl[5] = globaltimer_ns();
    reducer_done();
}

static size_t up128(size_t v) { return (v + 127) / 128 * 128; }

bool plan_decode(DecodeArgs& a, int grid, size_t* smem_bytes) {
    if (a.T < 1 || a.T > kDecodeMaxT || a.H % 64 || a.H > 8192 || a.F % 64 || a.E > kMaxExperts || a.K > kMaxTopK)
        return false;
    if (grid < 1 || grid > kPlanMaxGrid) return false;
    a.ch = a.H <= 2048 ? 1 : (a.H <= 4096 ? 2 : 4);
    a.gmax = a.ch == 4 ? 2 : 4;
    const int np = a.T * a.K;
    if (grid + np > kMaxSegTotal) return false;  // segments <= grid + groups <= grid + pairs
    const size_t target = a.stage_target ? a.stage_target : kStageTarget;
    const size_t ubf = unit_bytes(kKindBF16, a.H), uq = unit_bytes(kKindQ8, a.H);
    a.ups_bf16 = (int)std::max<size_t>(1, target / ubf);
    a.ups_q8 = (int)std::max<size_t>(1, target / uq);
    if (a.q8_cost <= 0) a.q8_cost = (int)(uq * kQ8CostDefault / 1000);
    const size_t slot = up128(std::max(a.ups_bf16 * ubf, a.ups_q8 * uq));
    a.slot_bytes = (uint32_t)slot;
    const size_t ctrl = up128(sizeof(Ctrl));
    a.off_ring = (uint32_t)ctrl;
    int ns = (int)std::min<size_t>(kMaxNS, (kSmemCap - ctrl) / slot);
    if (a.ns_cap > 0) ns = std::min(ns, a.ns_cap);
    if (ns < 2) return false;
    // A batch of kb units starting at a multiple of kb spans at most span(kb, ups) stages; consumers
    // hold the stages of the batch they are waiting for, so the ring must have room for all of them
    // or the producer could never issue the last one.
    auto gcd = [](int x, int y) {
        while (y) {
            const int t = x % y;
            x = y;
            y = t;
        }
        return x;
    };
    auto span = [&](int kb, int ups) { return (ups - gcd(kb, ups) + kb - 1) / ups + 1; };
    for (int kb : {kBatch, 2})
        for (int ups : {a.ups_bf16, a.ups_q8})
            if (span(kb, ups) > ns) return false;
    // The ring doubles as reduction scratch once every stage is consumed: each CTA stages one output
    // slice of every segment's partial-sum rows.  Rows <= pairs (a shared expert's included) + one
    // extra segment per share boundary.  (Letting only the last CTAs to arrive reduce, so that the
    // others free their SMs early, measured slower: the next call's CTAs that land on the reducers'
    // SMs start late with full-size shares and become its stragglers.)
    // Reducers: the requested count (a.nred on entry; 0 = every CTA) raised until a reducer's slice
    // of the partial sums fits the ring.  With fewer reducers than CTAs the last nred CTAs by index
    // get shares smaller by a.late_cost (requested on entry): in a stream of calls they take the SMs
    // of the previous call's reducers and start that much later.
    const size_t npt = (size_t)np + a.T;
    const size_t rows = npt + (size_t)(grid - 1) * std::min(a.gmax, a.T);
    auto fits = [&](int nr) {
        const size_t nqr = (size_t)(a.H / 4 + nr - 1) / nr;
        return (rows * nqr + npt * nqr + (size_t)a.T * nqr) * 16 <= (size_t)ns * slot;
    };
    int nr = a.nred > 0 ? std::min(a.nred, grid) : grid;
    while (nr < grid && !fits(nr)) nr++;
    if (!fits(nr) || sizeof(PlanScratch) > (size_t)ns * slot) return false;
    a.nred = nr;
    a.nlate = nr < grid ? nr : 0;
    if (a.nlate == 0 || a.late_cost < 0) a.late_cost = 0;
    a.NS = ns;
    *smem_bytes = ctrl + (size_t)ns * slot;
    return true;
}

bool decode_register_split_fits() {
    // setmaxnreg.inc waits until the pool has the registers: the launch must provide all of them
    const void* fns[3] = {(const void*)decode_kernel<1>, (const void*)decode_kernel<2>, (const void*)decode_kernel<4>};
    for (const void* f : fns) {
        cudaFuncAttributes at;
        if (cudaFuncGetAttributes(&at, f) != cudaSuccess) {
            cudaGetLastError();
            return false;
        }
        if ((long)at.numRegs * kDecThreads < 4L * 32 * kProdRegs + 8L * 32 * kConsRegs) return false;
    }
    return true;
}

// Cross-rank combine for the multi-kernel path: CTA s owns the same output slice as decode CTA s.
__global__ void __launch_bounds__(512) ep_exchange_kernel(const EpExchange ep, const float* part, float* out, int T,
                                                          int H, int accumulate, uint32_t* err, uint64_t timeout_ns) {
    __shared__ int abort_flag;
    const int s = blockIdx.x, G = gridDim.x, H4 = H / 4, W = ep.world, par = ep.epoch & 1;
    const int q0 = (int)((long long)s * H4 / G), nq = (int)((long long)(s + 1) * H4 / G) - q0;
    const int nv = nq * 4, ne = T * nv, nthr = blockDim.x, tid = threadIdx.x;
    const uint64_t tag = (uint64_t)ep.epoch << 32;
    const uint64_t deadline = globaltimer_ns() + timeout_ns;
    if (tid == 0) abort_flag = 0;
    // every value of this rank's partial slice, straight from global memory, into every rank's buffer
    // (all tokens of the call first, then the collection: one round of exchange latency)
    for (int i = tid; i < ne; i += nthr) {
        const int t = i / nv, j = i - t * nv;
        const uint64_t w = tag | __float_as_uint(__ldcg(part + (size_t)t * H + 4 * q0 + j));
        for (int r = 0; r < W; r++)
            st_relaxed_sys_u64(ep.peer_x[r] + ((size_t)(par * W + ep.rank) * ep.tstride + t) * H + 4 * q0 + j, w);
    }
    named_bar_sync(1, nthr);
    for (int i = tid; i < ne; i += nthr) {  // every rank adds the same values in rank order
        const int t = i / nv, j = i - t * nv;
        float* o = out + (size_t)t * H + 4 * q0 + j;
        float acc = accumulate ? *o : 0.f;
        bool ok = true;
        for (int r = 0; r < W && ok; r++) {
            const uint64_t* src = ep.x_local + ((size_t)(par * W + r) * ep.tstride + t) * H + 4 * q0 + j;
            uint64_t w = ld_relaxed_sys_u64(src);
            for (int spin = 0; (uint32_t)(w >> 32) != ep.epoch; spin++) {
                if ((spin & 31) == 31 && (*(volatile int*)&abort_flag || globaltimer_ns() > deadline)) {
                    atomicOr(err, kErrTimeout);
                    *(volatile int*)&abort_flag = 1;
                    ok = false;
                    break;
                }
                __nanosleep(32);
                w = ld_relaxed_sys_u64(src);
            }
            acc += __uint_as_float((uint32_t)w);
        }
        if (!ok) break;
        *o = acc;
    }
}

cudaError_t launch_ep_exchange(const EpExchange& ep, const float* part, float* out, int T, int H, int accumulate,
                               uint32_t* err, uint64_t timeout_ns, int grid, cudaStream_t st) {
    if (T > ep.tstride) return cudaErrorInvalidValue;
    ep_exchange_kernel<<<grid, 512, 0, st>>>(ep, part, out, T, H, accumulate, err, timeout_ns);
    return cudaGetLastError();
}

// The planner: one CTA computes the whole plan of a call with the decode CTAs' own code and
// publishes it (st.release of the stamp); it lets its decode grid launch at once and runs on the SM
// that grid leaves free, while the previous call still streams.  Before exiting it waits for its
// predecessor grid: that keeps the spare SM from the decode CTAs (measured: a planner that leaves at
// once hands its SM to a decode CTA, and the next planner starts late), and the completion of a
// decode grid implies that of every grid before it in the stream.  Plans rotate over four buffers:
// the planner of call e + 4 starts only once every CTA of call e + 3 started, i.e. once the CTAs of
// call e + 2 left their SMs, each after waiting for call e to finish staging its partial sums; plan e
// is read before that.
struct __align__(16) PlannerSmem {
    CallPlan P;
    PlanShared sh;
    PlanCta me;
    PlanScratch R;
};

__global__ void __launch_bounds__(kDecThreads, 1) planner_kernel(const DecodeArgs a, int G, PubPlan* out, uint32_t* flag,
                                                                 uint32_t stamp) {
    extern __shared__ __align__(16) unsigned char psm[];
    PlannerSmem& m = *reinterpret_cast<PlannerSmem*>(psm);
    const int tid = threadIdx.x;
    if (tid == 0) griddep_launch_dependents();
    // optional stamps in the timeline row after the decode grid's: 0 start, 1 planned, 2 published,
    // 3 predecessor complete
    uint64_t* ptl = a.timeline ? a.timeline + (size_t)G * kTimelineSlots : nullptr;
    if (ptl && tid == 0) ptl[0] = globaltimer_ns();
    PlanIn pin;
    pin.logits = a.logits;
    pin.bias = a.bias;
    pin.desc = a.desc;
    pin.shared = a.shared;
    pin.idx_out = a.idx_out;
    pin.w_out = a.w_out;
    pin.err = a.err;
    pin.T = a.T;
    pin.E = a.E;
    pin.K = a.K;
    pin.H = a.H;
    pin.F = a.F;
    pin.scoring = a.scoring;
    pin.G = G;
    pin.gmax = a.gmax;
    pin.ups_bf16 = a.ups_bf16;
    pin.ups_q8 = a.ups_q8;
    pin.q8_cost = a.q8_cost;
    // Late shares only when the previous call is still running: then the last CTAs of this call start
    // when its reducers leave their SMs.  (A call whose inputs come from the previous call's outputs
    // is planned after that call finished: every CTA starts at once and shares stay even.)
    const bool prev_running = a.epoch > 0 && ld_acquire_gpu_u64(&a.cnt[1]) < (unsigned long long)a.epoch * (unsigned long long)G;
    pin.nlate = prev_running ? a.nlate : 0;
    pin.late_cost = prev_running ? a.late_cost : 0;
    pin.nred = prev_running ? a.nred : G;  // fewer reducers free SMs for the next call; alone, all reduce
    pin.decide = nullptr;                  // decided here
    pin.cnt1 = nullptr;
    pin.epoch = a.epoch;
    plan_call(pin, m.P, m.R, m.sh, m.me);
    if (ptl && tid == 0) ptl[1] = globaltimer_ns();
    plan_tables(m.P, m.sh, G, a.F, a.H, a.gmax, tid, kDecThreads, 1);
    named_bar_sync(1, kDecThreads);
    for (int ss = tid >> 5; ss < G; ss += kDecThreads / 32)  // every share, a warp each, straight to the plan
        plan_share_warp(pin, m.P, ss, &out->cta[ss]);
    {
        const int4* s1 = reinterpret_cast<const int4*>(&m.P);
        int4* d1 = reinterpret_cast<int4*>(&out->P);
        for (int q = tid; q < (int)(sizeof(CallPlan) / 16); q += kDecThreads) d1[q] = s1[q];
        const int4* s2 = reinterpret_cast<const int4*>(&m.sh);
        int4* d2 = reinterpret_cast<int4*>(&out->sh);
        for (int q = tid; q < (int)(sizeof(PlanShared) / 16); q += kDecThreads) d2[q] = s2[q];
    }
    __threadfence();
    __syncthreads();
    if (tid == 0) {
        asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(flag), "r"(stamp) : "memory");
        if (ptl) ptl[2] = globaltimer_ns();
        griddep_wait();  // hold this SM until the preceding grid completes (see above)
        if (ptl) ptl[3] = globaltimer_ns();
    }
}

size_t pub_plan_bytes() { return sizeof(PubPlan); }

cudaError_t launch_planner(const DecodeArgs& a, int grid, PubPlan* out, uint32_t* flag, uint32_t stamp, cudaStream_t st) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(1);
    cfg.blockDim = dim3(kDecThreads);
    cfg.dynamicSmemBytes = sizeof(PlannerSmem);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, planner_kernel, a, grid, out, flag, stamp);
}

cudaError_t decode_set_smem_limit() {
    cudaError_t e = cudaFuncSetAttribute(planner_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sizeof(PlannerSmem));
    if (e == cudaSuccess) e = cudaFuncSetAttribute(decode_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemCap);
    if (e == cudaSuccess) e = cudaFuncSetAttribute(decode_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemCap);
    if (e == cudaSuccess) e = cudaFuncSetAttribute(decode_kernel<4>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemCap);
    return e;
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
    if (a.ch == 1) return cudaLaunchKernelEx(&cfg, decode_kernel<1>, a);
    if (a.ch == 2) return cudaLaunchKernelEx(&cfg, decode_kernel<2>, a);
    return cudaLaunchKernelEx(&cfg, decode_kernel<4>, a);
}

}  // namespace moe
