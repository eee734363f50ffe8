// Plan kernel of the fused decode path: one CTA computes everything the decode grid needs before it
// can stream weights, and publishes it with a release flag:
//   routing      route_core.cuh, one warp per token
//   grouping     local expert jobs in first-appearance order of the flattened top-k list
//                (solar_hybrid/runtime.py:343-354), each job's pairs in token order
//   token groups each job's pairs split into groups of at most gmax tokens; a group is one pass
//                over the job's unit table (F units: gate row f, up row f, down column f)
//   partition    the unit stream (all groups' units, in group order) cut into G byte-balanced
//                contiguous shares at unit boundaries; a share is a list of segments (runs of one
//                group's units), numbered call-wide in stream order -- the numbering fixes where
//                each segment's partial sums go and the order in which they are added up
//   reduction    per pair: its group and row; per group: its segment range; per token: its pairs
//                in job order
//
// It is launched with programmatic dependent launch right after the previous decode grid triggers
// and runs on the one SM that grid leaves free, so for back-to-back layers the plan of layer l+1
// is ready while layer l still streams.  It lets its own decode grid launch at once (the decode
// CTAs set up and wait on the plan flag), and before exiting it waits for its predecessor grid,
// which makes "plan(l) complete" imply "decode(l-1) complete" for the decode grid that depends on it.
#include <algorithm>
#include <climits>
#include <cstddef>

#include "common.cuh"
#include "decode.h"
#include "ptx.cuh"
#include "route_core.cuh"

namespace moe {

constexpr int kPlanThreads = kDecodeMaxT * 32;  // one warp per token
constexpr int kPlanJobs = kDecodeMaxPairs;      // local jobs <= pairs

struct PlanSmem {
    int idx[kDecodeMaxT][kMaxTopK];
    float w[kDecodeMaxT][kMaxTopK];
    int counts[kMaxExperts];
    int firstpos[kMaxExperts];
    uint32_t tokmask[kMaxExperts];
    int jmap[kMaxExperts];
    int pos2e[kDecodeMaxPairs];
    int ptok[kDecodeMaxPairs];            // token of pair p (job-major)
    int jkind[kPlanJobs];
    int jp0[kPlanJobs + 1];               // pair offsets
    int jg0[kPlanJobs + 1];               // group offsets
    const unsigned char* jw1[kPlanJobs];  // unit 0 of the job's table
    const float* jsc[kPlanJobs];
    int gjob[kMaxGroups];
    long long gcum[kMaxGroups + 1];       // unit-stream bytes of groups < g
    int cta_nseg[kPlanMaxGrid];
    int cta_seg0[kPlanMaxGrid + 1];
    int cta_uf[kPlanMaxGrid + 1];         // first unit of each CTA's share (cta_uf[G] = all units)
    int nj, np, ngrp, pad;
    alignas(16) float rscr[kDecodeMaxT][kMaxExperts];              // routing: exp values (read as float4)
    alignas(16) unsigned long long rck[kDecodeMaxT][kMaxExperts];  // routing: composite keys of each token
    alignas(16) int rrank[kDecodeMaxT][kMaxExperts];               // routing: ranks (partial counts summed)
    PlanShared sh;
};
static_assert(offsetof(PlanSmem, sh) % 16 == 0, "int4 copies from PlanSmem::sh");
static_assert(offsetof(PlanSmem, rscr) % 16 == 0 && (kMaxExperts * sizeof(float)) % 16 == 0,
              "route_keys_s reads its scratch as float4");
static_assert(offsetof(PlanCta, seg) == 64, "PlanCta header is 64 bytes");
static_assert(sizeof(Seg) % 16 == 0, "segments are copied as int4");

// Routing of T <= 16 tokens with all 16 warps: the first warp of each token's group computes its
// scores and keys (route_core.cuh), the group's warps count the keys ordered before each key over a
// slice of the experts each (shared-memory atomics sum the partial counts), and the first warp
// selects the top-k.  Same bits as route_token (the rank is an exact count).
__device__ __forceinline__ int plan_wpt(int T) { return T == 1 ? 16 : T == 2 ? 8 : T <= 4 ? 4 : T <= 8 ? 2 : 1; }

template <int S>
__device__ void plan_route(const PlanArgs& a, PlanSmem& m) {
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int T = a.T, E = a.E, K = a.K;
    const int wpt = plan_wpt(T);  // warps per token
    const int t = warp / wpt, g = warp % wpt;
    unsigned long long mine[S];
    float val[S];
    bool bad = false;
    if (t < T && g == 0)
        bad = route_keys_s<S>(a.logits + (size_t)t * E, a.bias, E, a.scoring, m.rscr[t], m.rck[t], mine, val);
    for (int q = tid; q < T * kMaxExperts; q += kPlanThreads) m.rrank[q / kMaxExperts][q % kMaxExperts] = 0;
    __syncthreads();
    if (t < T) {
        unsigned long long km[S];
#pragma unroll
        for (int s = 0; s < S; s++) {
            const int i = lane + 32 * s;
            km[s] = i < E ? m.rck[t][i] : 0ull;
        }
        const int per = (E + wpt - 1) / wpt, j0 = g * per, j1 = min(E, j0 + per);
        int r[S];
        route_rank_s<S>(m.rck[t], j0, j1, km, r);
#pragma unroll
        for (int s = 0; s < S; s++) {
            const int i = lane + 32 * s;
            if (i < E && r[s]) atomicAdd(&m.rrank[t][i], r[s]);
        }
    }
    __syncthreads();
    if (t < T && g == 0) {
        int r[S];
#pragma unroll
        for (int s = 0; s < S; s++) {
            const int i = lane + 32 * s;
            r[s] = i < E ? m.rrank[t][i] : INT_MAX;
        }
        route_select_s<S>(E, K, a.scoring, r, val, m.idx[t], m.w[t], m.rscr[t]);
        if (bad && lane == 0) atomicOr(a.err, kErrNonFinite);
    }
}

__global__ void __launch_bounds__(kPlanThreads, 1) plan_kernel(const PlanArgs a) {
    extern __shared__ __align__(16) unsigned char dyn[];
    PlanSmem& m = *reinterpret_cast<PlanSmem*>(dyn);
    PlanCta* cs = reinterpret_cast<PlanCta*>(dyn + ((sizeof(PlanSmem) + 15) / 16) * 16);  // [G] staged shares
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int T = a.T, E = a.E, K = a.K, H = a.H, F = a.F, G = a.G, GM = a.gmax;
    const int NP = T * K;
    uint64_t* tl = a.timeline;
    auto stamp = [&](int i) {
        if (tl && tid == 0) tl[i] = globaltimer_ns();
    };
    stamp(0);
    // The decode grid may be scheduled at once: it acquires this call's flag (bounded) before it
    // reads the plan, and its griddepcontrol.wait still waits for this grid to complete.
    if (tid == 0) griddep_launch_dependents();
    // host-buffer calls: the hidden states come straight from pinned host memory and the release of
    // the plan flag publishes them with the plan.  The warps that do not score a token copy them
    // while the scoring warps route (T <= 8); otherwise every thread copies after routing.
    const int wpt = plan_wpt(T);
    const uint4* xsrc = reinterpret_cast<const uint4*>(a.x_src);
    uint4* xdst = reinterpret_cast<uint4*>(a.x_dst);
    const int n16 = T * H / 8;
    if (a.x_src && wpt > 1 && !(warp % wpt == 0 && warp / wpt < T)) {
        const int below = min(T, (warp + wpt - 1) / wpt);  // scoring warps below this one
        for (int i = tid - 32 * below; i < n16; i += kPlanThreads - 32 * T) xdst[i] = xsrc[i];
    }

    // ---- routing ----
    if (E <= 32) plan_route<1>(a, m);
    else if (E <= 64) plan_route<2>(a, m);
    else if (E <= 128) plan_route<4>(a, m);
    else plan_route<8>(a, m);
    if (a.x_src && wpt == 1)
        for (int i = tid; i < n16; i += kPlanThreads) xdst[i] = xsrc[i];
    for (int e = tid; e < E; e += kPlanThreads) {
        m.counts[e] = 0;
        m.firstpos[e] = INT_MAX;
        m.tokmask[e] = 0;
        m.jmap[e] = -1;
    }
    for (int q = tid; q < NP; q += kPlanThreads) m.pos2e[q] = -1;
    for (int g = tid; g < kMaxGroups; g += kPlanThreads) m.sh.gvs0[g] = m.sh.gvs1[g] = 0;
    for (int k = tid; k < kMaxSegTotal; k += kPlanThreads) m.sh.segrows[k] = 0;
    __syncthreads();
    for (int q = tid; q < NP; q += kPlanThreads) {
        const int t = q / K, k = q % K, e = m.idx[t][k];
        atomicAdd(&m.counts[e], 1);
        atomicMin(&m.firstpos[e], q);
        atomicOr(&m.tokmask[e], 1u << t);
        if (a.idx_out) a.idx_out[q] = e;
        if (a.w_out) a.w_out[q] = m.w[t][k];
    }
    __syncthreads();
    for (int e = tid; e < E; e += kPlanThreads)
        if (m.counts[e] > 0) m.pos2e[m.firstpos[e]] = e;
    __syncthreads();
    stamp(1);

    // ---- local jobs in first-appearance order: pair and group offsets ----
    if (warp == 0) {
        int nj = 0, np = 0, ng = 0;
        for (int q0 = 0; q0 < NP; q0 += 32) {
            const int q = q0 + lane;
            const int e = q < NP ? m.pos2e[q] : -1;
            const int kind = e >= 0 ? __ldg(&a.desc[e].kind) : kKindRemote;
            const bool local = kind == kKindBF16 || kind == kKindQ8;
            if (e >= 0 && kind == kKindNone) atomicOr(a.err, kErrBadExpert);
            const unsigned msk = __ballot_sync(0xffffffffu, local);
            const int n = local ? m.counts[e] : 0;
            const int ngj = (n + GM - 1) / GM;
            int incl = n, gincl = ngj;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int y = __shfl_up_sync(0xffffffffu, incl, o);
                const int gy = __shfl_up_sync(0xffffffffu, gincl, o);
                if (lane >= o) {
                    incl += y;
                    gincl += gy;
                }
            }
            if (local) {
                const int j = nj + __popc(msk & ((1u << lane) - 1u));
                const ExpDesc d = a.desc[e];
                m.jkind[j] = kind;
                m.jw1[j] = static_cast<const unsigned char*>(d.w1);
                m.jsc[j] = d.sc;
                m.jp0[j] = np + incl - n;
                m.jg0[j] = ng + gincl - ngj;
                m.jmap[e] = j;
            }
            nj += __popc(msk);
            np += __shfl_sync(0xffffffffu, incl, 31);
            ng += __shfl_sync(0xffffffffu, gincl, 31);
        }
        if (lane == 0) {
            m.sh.sp0 = -1;
            if (a.shared) {  // block call: the shared expert is one more job, every token at weight 1
                const ExpDesc d = *a.shared;
                m.jkind[nj] = d.kind;
                m.jw1[nj] = static_cast<const unsigned char*>(d.w1);
                m.jsc[nj] = d.sc;
                m.jp0[nj] = np;
                m.jg0[nj] = ng;
                m.sh.sp0 = np;
                if (d.kind != kKindBF16 && d.kind != kKindQ8) atomicOr(a.err, kErrBadExpert);
                nj++;
                np += T;
                ng += (T + GM - 1) / GM;
            }
            m.nj = nj;
            m.np = np;
            m.ngrp = ng;
            m.jp0[nj] = np;
            m.jg0[nj] = ng;
        }
    }
    __syncthreads();
    stamp(2);
    const int nj = m.nj, np = m.np, ngrp = m.ngrp;

    // ---- pairs (job-major, tokens in order inside a job), token -> pairs, group -> job ----
    for (int q = tid; q < NP; q += kPlanThreads) {
        const int t = q / K, k = q % K, e = m.idx[t][k], j = m.jmap[e];
        if (j >= 0) {
            const int r = __popc(m.tokmask[e] & ((1u << t) - 1u));  // rank of t among the job's tokens
            const int p = m.jp0[j] + r;
            m.ptok[p] = t;
            m.sh.pgrp[p] = m.jg0[j] + r / GM;
            m.sh.prow[p] = r % GM;
            m.sh.pw[p] = m.w[t][k];
            int slot = 0;
            for (int k2 = 0; k2 < K; k2++) {
                const int j2 = m.jmap[m.idx[t][k2]];
                if (j2 >= 0 && j2 < j) slot++;
            }
            m.sh.tpair[t][slot] = p;
        }
    }
    for (int t = tid; t < T; t += kPlanThreads) {
        int n = 0;
        for (int k = 0; k < K; k++) n += m.jmap[m.idx[t][k]] >= 0;
        m.sh.tpn[t] = n;  // routed pairs only: the shared expert's pair is added apart
        const int sp0 = m.sh.sp0;
        if (sp0 >= 0) {
            const int p = sp0 + t, j = nj - 1;
            m.ptok[p] = t;
            m.sh.pgrp[p] = m.jg0[j] + t / GM;
            m.sh.prow[p] = t % GM;
            m.sh.pw[p] = 1.f;
        }
    }
    for (int j = tid; j < nj; j += kPlanThreads)
        for (int g = m.jg0[j]; g < m.jg0[j + 1]; g++) m.gjob[g] = j;
    __syncthreads();

    // ---- unit-stream byte prefix over groups (warp 0) ----
    if (warp == 0) {
        long long run = 0;
        for (int g0 = 0; g0 < ngrp; g0 += 32) {
            const int g = g0 + lane;
            const long long b = g < ngrp ? (long long)F * (long long)unit_bytes(m.jkind[m.gjob[g]], H) : 0;
            long long incl = b;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const long long y = __shfl_up_sync(0xffffffffu, incl, o);
                if (lane >= o) incl += y;
            }
            if (g < ngrp) m.gcum[g] = run + incl - b;
            run += __shfl_sync(0xffffffffu, incl, 31);
        }
        if (lane == 0) m.gcum[ngrp] = run;
    }
    __syncthreads();

    stamp(3);
    // ---- partition: CTA ss owns units [U(ss), U(ss+1)) of the stream ----
    const long long total = m.gcum[ngrp];
    const double per = (double)total / G;
    auto unit_at = [&](int ss) -> int {  // first unit starting at or after byte ss * total / G
        if (ss >= G) return ngrp * F;
        const long long B = (long long)(ss * per);
        if (B >= total) return ngrp * F;
        int lo = 0, hi = ngrp - 1;  // group g with gcum[g] <= B < gcum[g+1]
        while (lo < hi) {
            const int mid = (lo + hi + 1) >> 1;
            if (m.gcum[mid] <= B) lo = mid;
            else hi = mid - 1;
        }
        const uint32_t ub = (uint32_t)((m.gcum[lo + 1] - m.gcum[lo]) / F);
        const uint32_t off = (uint32_t)(B - m.gcum[lo]);  // < F * ub < 2^31
        return lo * F + (int)((off + ub - 1) / ub);
    };
    for (int ss = tid; ss <= G; ss += kPlanThreads) m.cta_uf[ss] = unit_at(ss);
    __syncthreads();
    for (int ss = tid; ss < G; ss += kPlanThreads) {
        const int uf = m.cta_uf[ss], ue = m.cta_uf[ss + 1];
        m.cta_nseg[ss] = ue > uf ? (ue - 1) / F - uf / F + 1 : 0;
    }
    __syncthreads();
    if (warp == 0) {  // exclusive scan of segment counts -> call-wide segment numbers
        int run = 0;
        for (int s0 = 0; s0 < G; s0 += 32) {
            const int ss = s0 + lane;
            const int v = ss < G ? m.cta_nseg[ss] : 0;
            int incl = v;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int y = __shfl_up_sync(0xffffffffu, incl, o);
                if (lane >= o) incl += y;
            }
            if (ss < G) m.cta_seg0[ss] = run + incl - v;
            run += __shfl_sync(0xffffffffu, incl, 31);
        }
        if (lane == 0) m.cta_seg0[G] = run;
    }
    __syncthreads();
    const int H4 = H / 4;
    for (int ss = tid; ss < G; ss += kPlanThreads) {  // shares staged in shared memory
        PlanCta* pc = &cs[ss];
        const int uf = m.cta_uf[ss], ue = m.cta_uf[ss + 1];
        int nseg = m.cta_nseg[ss];
        if (nseg > kSegPerCta) {  // never expected: a share spans at most groups/G + 2 groups
            atomicOr(a.err, kErrBadIndex);
            nseg = kSegPerCta;
        }
        int stage = 0;
        for (int k = 0; k < nseg; k++) {
            const int g = uf / F + k, j = m.gjob[g], kind = m.jkind[j];
            const int f0 = k == 0 ? uf % F : 0;
            const int fend = g == (ue - 1) / F ? (ue - 1) % F + 1 : F;
            const int r0 = (g - m.jg0[j]) * GM;  // first pair rank of the group
            const int nt = min(GM, m.jp0[j + 1] - m.jp0[j] - r0);
            const int gidx = m.cta_seg0[ss] + k;
            Seg& sg = pc->seg[k];
            sg.src = m.jw1[j] + (size_t)f0 * unit_bytes(kind, H);
            sg.sc = kind == kKindQ8 ? m.jsc[j] : nullptr;
            sg.kind = kind;
            sg.f0 = f0;
            sg.nu = fend - f0;
            sg.nt = nt;
            sg.gidx = gidx;
            sg.grp = g;
            sg.pad0 = sg.pad1 = 0;
#pragma unroll
            for (int i = 0; i < kGroupMax; i++) sg.tok[i] = m.ptok[m.jp0[j] + r0 + min(i, nt - 1)];
            pc->seg_stage[k] = stage;
            const int ups = kind == kKindQ8 ? a.ups_q8 : a.ups_bf16;
            stage += (sg.nu + ups - 1) / ups;
            if (gidx < kMaxSegTotal) m.sh.segrows[gidx] = nt;
            if (f0 == 0) m.sh.gvs0[g] = gidx;
            if (fend == F) m.sh.gvs1[g] = gidx + 1;
        }
        pc->seg_stage[nseg] = stage;
        pc->nseg = nseg;
        pc->nstage = stage;
        pc->q0 = (int)((long long)ss * H4 / G);
        pc->q1 = (int)((long long)(ss + 1) * H4 / G);
    }
    stamp(4);
    if (tid == 0) {
        m.sh.T = T;
        m.sh.np = np;
        m.sh.ngrp = ngrp;
        m.sh.nsegtot = m.cta_seg0[G];
        if (m.cta_seg0[G] > kMaxSegTotal) atomicOr(a.err, kErrBadIndex);  // the host bounds it; never expected
    }
    __syncthreads();
    // publish: each share's header and used segments, a warp per share (coalesced 16-byte stores)
    for (int ss = warp; ss < G; ss += kPlanThreads / 32) {
        const int4* src = reinterpret_cast<const int4*>(&cs[ss]);
        int4* dst = reinterpret_cast<int4*>(&a.plan->cta[ss]);
        const int n16 = (int)((offsetof(PlanCta, seg) + (size_t)cs[ss].nseg * sizeof(Seg)) / 16);
        for (int q = lane; q < n16; q += 32) dst[q] = src[q];
    }
    {
        const int4* src = reinterpret_cast<const int4*>(&m.sh);
        int4* dst = reinterpret_cast<int4*>(&a.plan->sh);
        for (int q = tid; q < (int)(sizeof(PlanShared) / 16); q += kPlanThreads) dst[q] = src[q];
    }
    __syncthreads();
    stamp(5);
    if (tid == 0) {
        __threadfence();
        asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(a.flag), "r"(a.stamp) : "memory");
        stamp(6);
        griddep_wait();  // complete only after the preceding grid: orders this call after the previous one
        stamp(7);
    }
}

constexpr size_t kPlanSmemCap = 227 * 1024;

static size_t plan_smem_bytes(int G) { return ((sizeof(PlanSmem) + 15) / 16) * 16 + (size_t)G * sizeof(PlanCta); }

int plan_max_grid() {
    const size_t fixed = ((sizeof(PlanSmem) + 15) / 16) * 16;
    return (int)std::min<size_t>(kPlanMaxGrid, (kPlanSmemCap - fixed) / sizeof(PlanCta));
}

cudaError_t plan_set_smem_limit() {
    return cudaFuncSetAttribute(plan_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kPlanSmemCap);
}

cudaError_t launch_plan(const PlanArgs& p, cudaStream_t st) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(1);
    cfg.blockDim = dim3(kPlanThreads);
    cfg.dynamicSmemBytes = plan_smem_bytes(p.G);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, plan_kernel, p);
}

}  // namespace moe
