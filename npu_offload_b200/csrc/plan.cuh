// In-kernel planning of the fused decode path.  Every decode CTA computes the call's routing and job
// structure itself, from the same inputs with the same code, so all CTAs agree bit for bit and no
// separate plan launch or global publication sits between the router logits and the weight stream:
//   routing      route_core.cuh semantics: max, exp, sequential softmax sum, probabilities and keys,
//                exact ranks, top-k and renormalised weights, with the work of every phase spread
//                over all 12 warps (only the per-token sum is sequential, as the reference's is)
//   grouping     local expert jobs in first-appearance order of the flattened top-k list
//                (solar_hybrid/runtime.py:343-354), each job's pairs in token order; a block call
//                appends the shared expert as one more job (every token, weight 1)
//   token groups each job's pairs split into groups of at most gmax tokens; a group is one pass
//                over the job's unit table (F units: gate row f, up row f, down column f)
//   own share    the unit stream (all groups' units, in group order) cut into G cost-balanced
//                contiguous shares at unit boundaries; CTA s computes only share s (two binary
//                searches over the jobs), its segments (runs of one group's units) and their stages
//   reduction    per pair: its group and row; per token: its pairs in job order; per group: its
//                segments across the shares (plan_tables, once the CTA's own segments are done)
// The planning is latency-bound (one CTA, a few microseconds), so it is organised as few barrier
// phases with one global-memory round trip: the logits and the layer's whole expert table are loaded
// into shared memory first.  A segment's partial sums go to part[(s * kSegPerCta + k) * kGroupMax + row]
// (share s, k-th segment of that share), so writing them needs nothing but the CTA's own share.
#pragma once
#include <climits>

#include "common.cuh"
#include "decode.h"
#include "ptx.cuh"
#include "route_core.cuh"

namespace moe {

constexpr int kPlanJobs = kDecodeMaxPairs;  // jobs (routed local + shared) <= pairs
constexpr int kNW = 12;                     // warps of a decode CTA
constexpr int kPlanThr = kNW * 32;

// The call's routing and job structure: identical in every CTA, alive for the whole kernel.
struct __align__(16) CallPlan {
    int idx[kDecodeMaxT][kMaxTopK];
    float w[kDecodeMaxT][kMaxTopK];
    int ptok[kDecodeMaxPairs];              // token of pair p (pairs job-major)
    int jkind[kPlanJobs];
    int jp0[kPlanJobs + 1];                 // pair offsets of the jobs
    int jg0[kPlanJobs + 1];                 // group offsets of the jobs
    const unsigned char* jw1[kPlanJobs];    // unit 0 of the job's table
    const float* jsc[kPlanJobs];            // int8 scales (null for bf16)
    long long jb0[kPlanJobs + 1];           // unit-stream cost (unit_cost) of the jobs before job j
    int gjob[kMaxGroups];                   // job of group g
    int uf[kPlanMaxGrid + 1];               // first unit of every share (uf[G] = all units)
    int nseg[kPlanMaxGrid];                 // segments of every share
    int seg0[kPlanMaxGrid + 1];             // call-wide index of every share's first segment
    int segslot[kMaxSegTotal];              // partial-sum slot (s * kSegPerCta + k) of call-wide segment i
    int nj, np, ngrp, q8c;                  // q8c: planning cost of an int8 unit (unit_cost)
    long long late_cost;                    // the last nlate shares are smaller by this cost
    int nlate, pad2;
};

// Scratch of the planning steps; aliases the ring (no weight copy is issued before the plan exists).
struct __align__(16) PlanScratch {
    float lg[kDecodeMaxT][kMaxExperts];                // the call's router logits
    float mx[kDecodeMaxT];                             // softmax: each token's largest logit
    float ev[kDecodeMaxT][kMaxExperts];                // softmax numerators
    float pv[kDecodeMaxT][kMaxExperts];                // probabilities (softmax) / sigmoid values
    unsigned long long ck[kDecodeMaxT][kMaxExperts];   // composite keys: ordered value bits, complemented index
    float selv[kDecodeMaxT][kMaxTopK];                 // top-k values by rank
    int seli[kDecodeMaxT][kMaxTopK];                   // top-k experts by rank
    const void* dw1[kMaxExperts];                      // the layer's expert table
    const float* dsc[kMaxExperts];
    int dkind[kMaxExperts];
    int counts[kMaxExperts];
    int firstpos[kMaxExperts];
    uint32_t tokmask[kMaxExperts];
    int jmap[kMaxExperts];
    int bad;
    int streamed;                                      // the call's share-cut decision (PlanIn::decide)
};

struct PlanIn {
    const float* logits;   // [T, E] device memory
    const float* bias;     // [E] or null
    const ExpDesc* desc;   // [E] expert table of the layer
    const ExpDesc* shared; // block calls: the layer's shared expert, else null
    int32_t* idx_out;      // [T, K] router indices (written by CTA 0), or null
    float* w_out;          // [T, K] router weights, or null
    uint32_t* err;
    int T, E, K, H, F, scoring, G, gmax, ups_bf16, ups_q8;
    int q8_cost;           // planning cost of an int8 unit in bf16-stream bytes (unit_cost)
    int nlate;             // the last nlate CTAs' shares are smaller by late_cost (they start late)
    long long late_cost;
    int nred;              // the call's reducing CTAs (PlanCta::nred)
    // Calls planned in every CTA: decide (non-null) holds one word per call (call mod 4),
    // (epoch << 8) | streamed, set by compare-and-swap by the first CTA to decide from whether call
    // epoch - 1 still runs (cnt1 < epoch * G).  Streamed calls use nlate / late_cost / nred, the
    // others even shares on every reducing CTA.  With decide null the values apply as given.
    unsigned long long* decide;
    const unsigned long long* cnt1;
    unsigned long long epoch;
};

// The call's share-cut decision (PlanIn::decide): two global round trips, made by one thread while
// the other warps route.
__device__ __forceinline__ int plan_decide(unsigned long long* dw, const unsigned long long* cnt1,
                                          unsigned long long epoch, int G) {
    const unsigned long long tagged = epoch << 8;
    unsigned long long v = atomicAdd(dw, 0ull);
    const bool pr = epoch > 0 && ld_acquire_gpu_u64(cnt1) < epoch * (unsigned long long)G;
    const unsigned long long mine = tagged | (pr ? 1ull : 0ull);
    for (int tries = 0; (v & ~0xffull) != tagged && tries < 64; tries++) {
        const unsigned long long old = atomicCAS(dw, v, mine);
        v = old == v ? mine : old;
    }
    return (v & ~0xffull) == tagged ? (int)(v & 1ull) : 0;
}

// Cost at which share ss starts.  Shares 0 .. G - nlate - 1 get cost S each, the last nlate shares
// max(0, S - late) each, with S chosen so that the shares add up to the total (costs: unit_cost, i.e.
// bytes for bf16 units).  With nlate == 0 this is ss * total / G.
__device__ __forceinline__ long long plan_share_start(long long total, int ss, int G, int nlate, long long late) {
    if (nlate <= 0 || late <= 0) return (long long)ss * total / G;
    const int ne = G - nlate;  // early shares
    // S >= late: G*S - nlate*late = total; else the late shares are empty and ne*S = total
    if (total + (long long)nlate * late >= (long long)G * late) {
        const long long num = total + (long long)nlate * late;  // G * S
        const long long lo = (long long)min(ss, ne) * num / G;
        if (ss <= ne) return lo;
        return (long long)ss * num / G - (long long)(ss - ne) * late;
    }
    return ss >= ne ? total : (long long)ss * total / ne;
}

// First unit of share ss: the first unit starting at or after the share's starting cost.
__device__ __forceinline__ int plan_unit_at(const CallPlan& P, int ss, int G, int F, int H) {
    const int nj = P.nj;
    const long long total = P.jb0[nj];
    if (ss >= G || total <= 0) return P.jg0[nj] * F;
    const long long B = plan_share_start(total, ss, G, P.nlate, P.late_cost);
    int lo = 0, hi = nj - 1;  // job j with jb0[j] <= B < jb0[j+1]
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (P.jb0[mid] <= B) lo = mid;
        else hi = mid - 1;
    }
    const long long ub = unit_cost(P.jkind[lo], H, P.q8c);
    const long long off = B - P.jb0[lo];  // < the job's cost
    return P.jg0[lo] * F + (int)((off + ub - 1) / ub);
}

// Routing, jobs, groups, the pair tables of the reduction and this CTA's share (me).  All kPlanThr
// threads take part; ends with __syncthreads.  tl (optional): phase stamps 6 (routed), 7 (jobs),
// 15 (pairs and share bounds).
__device__ void plan_call(const PlanIn& a, CallPlan& P, PlanScratch& R, PlanShared& sh, PlanCta& me,
                          uint64_t* tl = nullptr) {
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int T = a.T, E = a.E, K = a.K, H = a.H, F = a.F, G = a.G, GM = a.gmax;
    const int NP = T * K, S32 = (E + 31) / 32, NIT = T * S32;
    static_assert(kMaxExperts % 32 == 0, "expert slices of 32");
    const int s = blockIdx.x;
    const bool softmax = a.scoring == 0;
    auto stamp = [&](int i) {
        if (tl && tid == 0) tl[i] = globaltimer_ns();
    };

    // The routing steps P0-P2 run on warps 0 .. kNW - 2 (named barrier 2); the last warp makes the
    // call's share-cut decision meanwhile.
    constexpr int NWP = kNW - 1, TPP = NWP * 32;
    if (warp == NWP) {
        if (lane == 0) R.streamed = a.decide ? plan_decide(a.decide + (a.epoch & 3), a.cnt1, a.epoch, G) : 1;
        if (tl && lane == 0) tl[16] = globaltimer_ns();
    } else {
    // ---- P0: one global round trip: logits (a warp per token, which also takes the max) and the
    // layer's expert table into shared memory ----
    for (int t = warp; t < T; t += NWP) {
        float m = -INFINITY;  // f32::max fold: NaN never replaces the running max
        for (int i = lane; i < E; i += 32) {
            const float v = a.logits[(size_t)t * E + i];
            R.lg[t][i] = v;
            m = v > m ? v : m;
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float y = __shfl_xor_sync(0xffffffffu, m, o);
            m = y > m ? y : m;
        }
        if (lane == 0) R.mx[t] = m;
    }
    for (int e = tid; e < E; e += TPP) {
        const ExpDesc d = a.desc[e];
        R.dw1[e] = d.w1;
        R.dsc[e] = d.sc;
        R.dkind[e] = d.kind;
        R.counts[e] = 0;
        R.firstpos[e] = INT_MAX;
        R.tokmask[e] = 0;
        R.jmap[e] = -1;
    }
    if (tid == 0) R.bad = 0;
    named_bar_sync(2, TPP);
    stamp(17);

    // ---- P1: per (token, 32-expert slice): softmax numerators, or sigmoid values and keys ----
    for (int it = warp; it < NIT; it += NWP) {
        const int t = it / S32, i = (it % S32) * 32 + lane;
        if (i >= E) continue;
        if (softmax) {
            R.ev[t][i] = router_exp(R.lg[t][i] - R.mx[t]);
        } else {
            const float sg = __fdiv_rn(1.0f, 1.0f + router_exp(-R.lg[t][i]));
            const float k = sg + (a.bias ? a.bias[i] : 0.f);
            R.pv[t][i] = sg;
            if (k != k) R.bad = 1;
            R.ck[t][i] = ((unsigned long long)ordered_bits(k != k ? -INFINITY : k) << 32) | (uint32_t)(0xFFFFFFFFu - (uint32_t)i);
        }
    }
    named_bar_sync(2, TPP);

    // ---- P2: a warp per token: (softmax) the sequential sum in index order, probabilities and keys;
    // then the top K by key ("larger value first, ties to the lower index") ----
    for (int t = warp; t < T; t += NWP) {
        constexpr int SM = kMaxExperts / 32;
        unsigned long long key[SM];
        if (softmax) {
            float z = 0.f;  // every lane runs the same chain of additions: all lanes agree
            const float4* e4 = reinterpret_cast<const float4*>(R.ev[t]);
            const int nq = E >> 2;
#pragma unroll 8
            for (int q = 0; q < nq; q++) {
                const float4 v = e4[q];
                z += v.x;
                z += v.y;
                z += v.z;
                z += v.w;
            }
            for (int j = nq * 4; j < E; j++) z += R.ev[t][j];
#pragma unroll
            for (int sl = 0; sl < SM; sl++) {
                const int i = lane + 32 * sl;
                key[sl] = 0ull;
                if (sl < S32 && i < E) {
                    const float p = __fdiv_rn(R.ev[t][i], z);
                    R.pv[t][i] = p;
                    if (p != p) R.bad = 1;
                    key[sl] = ((unsigned long long)ordered_bits(p != p ? -INFINITY : p) << 32) | (uint32_t)(0xFFFFFFFFu - (uint32_t)i);
                }
            }
        } else {
#pragma unroll
            for (int sl = 0; sl < SM; sl++) {
                const int i = lane + 32 * sl;
                key[sl] = (sl < S32 && i < E) ? R.ck[t][i] : 0ull;
            }
        }
        // Every real key is above 0.  tau = the K-th largest of the 32 lane maxima: at least K keys are
        // >= tau, and every key that outranks one of them is >= tau too, so ranking the keys >= tau among
        // themselves gives the exact top K.
        unsigned long long km = 0ull;
#pragma unroll
        for (int sl = 0; sl < SM; sl++) km = key[sl] > km ? key[sl] : km;
        int r = 0;
#pragma unroll 8
        for (int l = 0; l < 32; l++) r += __shfl_sync(0xffffffffu, km, l) > km ? 1 : 0;
        const unsigned hit = __ballot_sync(0xffffffffu, r == K - 1 && km != 0ull);
        const unsigned long long tau = __shfl_sync(0xffffffffu, km, hit ? __ffs(hit) - 1 : 0);
        unsigned long long* cand = R.ck[t];  // the candidates, compacted (the keys are in registers)
        __syncwarp();
        int C = 0;
#pragma unroll
        for (int sl = 0; sl < SM; sl++) {
            const bool c = key[sl] != 0ull && key[sl] >= tau;
            const unsigned m = __ballot_sync(0xffffffffu, c);
            if (c) cand[C + __popc(m & ((1u << lane) - 1u))] = key[sl];
            C += __popc(m);
        }
        __syncwarp();
        for (int p = lane; p < C; p += 32) {
            const unsigned long long mine = cand[p];
            int rk = 0;
            for (int q = 0; q < C; q++) rk += cand[q] > mine ? 1 : 0;
            if (rk < K) {
                const int i = (int)(0xFFFFFFFFu - (uint32_t)mine);
                R.seli[t][rk] = i;
                R.selv[t][rk] = R.pv[t][i];
            }
        }
    }
    }  // routing warps
    __syncthreads();
    stamp(18);
    const bool streamed = R.streamed != 0;
    const int nlate = streamed ? a.nlate : 0, nred = streamed ? a.nred : G;
    const long long late_cost = streamed ? a.late_cost : 0;

    // ---- P4: per pair (t, k): renormalised weight (sum in k order), grouping counts ----
    for (int q = tid; q < NP; q += kPlanThr) {
        const int t = q / K, k = q % K;
        float tot = 0.f;
        for (int k2 = 0; k2 < K; k2++) tot += R.selv[t][k2];
        if (!softmax) tot += 1e-20f;
        const int e = R.seli[t][k];
        const float w = __fdiv_rn(R.selv[t][k], tot);
        P.idx[t][k] = e;
        P.w[t][k] = w;
        atomicAdd(&R.counts[e], 1);
        atomicMin(&R.firstpos[e], q);
        atomicOr(&R.tokmask[e], 1u << t);
        if (s == 0) {
            if (a.idx_out) a.idx_out[q] = e;
            if (a.w_out) a.w_out[q] = w;
        }
    }
    __syncthreads();
    if (R.bad && s == 0 && tid == 0) atomicOr(a.err, kErrNonFinite);
    stamp(6);

    // ---- P5: local jobs in first-appearance order: pair, group and byte offsets (warp 0) ----
    if (warp == 0) {
        int nj = 0, np = 0, ng = 0;
        long long nb = 0;
        for (int q0 = 0; q0 < NP; q0 += 32) {
            const int q = q0 + lane;
            const int e = q < NP ? P.idx[q / K][q % K] : 0;
            const bool first = q < NP && R.firstpos[e] == q;
            const int kind = first ? R.dkind[e] : kKindRemote;
            const bool local = kind == kKindBF16 || kind == kKindQ8;
            if (first && kind == kKindNone && s == 0) atomicOr(a.err, kErrBadExpert);
            const unsigned msk = __ballot_sync(0xffffffffu, local);
            const int n = local ? R.counts[e] : 0;
            const int ngj = (n + GM - 1) / GM;
            const long long bj = local ? (long long)ngj * F * unit_cost(kind, H, a.q8_cost) : 0;
            int incl = n, gincl = ngj;
            long long bincl = bj;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int y = __shfl_up_sync(0xffffffffu, incl, o);
                const int gy = __shfl_up_sync(0xffffffffu, gincl, o);
                const long long by = __shfl_up_sync(0xffffffffu, bincl, o);
                if (lane >= o) {
                    incl += y;
                    gincl += gy;
                    bincl += by;
                }
            }
            if (local) {
                const int j = nj + __popc(msk & ((1u << lane) - 1u));
                P.jkind[j] = kind;
                P.jw1[j] = static_cast<const unsigned char*>(R.dw1[e]);
                P.jsc[j] = R.dsc[e];
                P.jp0[j] = np + incl - n;
                P.jg0[j] = ng + gincl - ngj;
                P.jb0[j] = nb + bincl - bj;
                R.jmap[e] = j;
            }
            nj += __popc(msk);
            np += __shfl_sync(0xffffffffu, incl, 31);
            ng += __shfl_sync(0xffffffffu, gincl, 31);
            nb += __shfl_sync(0xffffffffu, bincl, 31);
        }
        if (lane == 0) {
            sh.sp0 = -1;
            if (a.shared) {  // block call: the shared expert is one more job, every token at weight 1
                const ExpDesc d = *a.shared;
                P.jkind[nj] = d.kind;
                P.jw1[nj] = static_cast<const unsigned char*>(d.w1);
                P.jsc[nj] = d.sc;
                P.jp0[nj] = np;
                P.jg0[nj] = ng;
                P.jb0[nj] = nb;
                sh.sp0 = np;
                if (d.kind != kKindBF16 && d.kind != kKindQ8 && s == 0) atomicOr(a.err, kErrBadExpert);
                nb += (long long)((T + GM - 1) / GM) * F * unit_cost(d.kind, H, a.q8_cost);
                nj++;
                np += T;
                ng += (T + GM - 1) / GM;
            }
            P.nj = nj;
            P.np = np;
            P.ngrp = ng;
            P.q8c = a.q8_cost;
            P.nlate = nlate;
            P.late_cost = late_cost;
            P.jp0[nj] = np;
            P.jg0[nj] = ng;
            P.jb0[nj] = nb;
        }
    }
    __syncthreads();
    stamp(7);
    const int nj = P.nj, np = P.np;

    // ---- P6: pairs (job-major, tokens in order inside a job), token -> pairs, group -> job, and the
    // bounds of this CTA's share ----
    for (int q = tid; q < NP; q += kPlanThr) {
        const int t = q / K, k = q % K, e = P.idx[t][k], j = R.jmap[e];
        if (j >= 0) {
            const int r = __popc(R.tokmask[e] & ((1u << t) - 1u));  // rank of t among the job's tokens
            const int p = P.jp0[j] + r;
            P.ptok[p] = t;
            sh.pgrp[p] = P.jg0[j] + r / GM;
            sh.prow[p] = r % GM;
            sh.pw[p] = P.w[t][k];
            int slot = 0;
            for (int k2 = 0; k2 < K; k2++) {
                const int j2 = R.jmap[P.idx[t][k2]];
                if (j2 >= 0 && j2 < j) slot++;
            }
            sh.tpair[t][slot] = p;
        }
    }
    for (int t = tid; t < T; t += kPlanThr) {
        int n = 0;
        for (int k = 0; k < K; k++) n += R.jmap[P.idx[t][k]] >= 0;
        sh.tpn[t] = n;  // routed pairs only: the shared expert's pair is added apart
        const int sp0 = sh.sp0;
        if (sp0 >= 0) {
            const int p = sp0 + t, j = nj - 1;
            P.ptok[p] = t;
            sh.pgrp[p] = P.jg0[j] + t / GM;
            sh.prow[p] = t % GM;
            sh.pw[p] = 1.f;
        }
    }
    for (int j = tid; j < nj; j += kPlanThr)
        for (int g = P.jg0[j]; g < P.jg0[j + 1]; g++) P.gjob[g] = j;
    if (tid >= kPlanThr - 2) P.uf[s + tid - (kPlanThr - 2)] = plan_unit_at(P, s + tid - (kPlanThr - 2), G, F, H);
    __syncthreads();
    stamp(15);

    // ---- P7: this CTA's segments: units [uf(s), uf(s + 1)) of the stream, a thread per segment ----
    {
        const int uf = P.uf[s], ue = P.uf[s + 1];
        const int nseg = min(kSegPerCta, ue > uf ? (ue - 1) / F - uf / F + 1 : 0);
        auto seg_units = [&](int k, int& g, int& f0, int& fend) {
            g = uf / F + k;
            f0 = k == 0 ? uf % F : 0;
            fend = g == (ue - 1) / F ? (ue - 1) % F + 1 : F;
        };
        if (tid < nseg) {
            const int k = tid;
            int g, f0, fend, stage = 0;
            for (int k2 = 0; k2 < k; k2++) {  // ring stages of the segments before this one
                int g2, a0, a1;
                seg_units(k2, g2, a0, a1);
                const int ups = P.jkind[P.gjob[g2]] == kKindQ8 ? a.ups_q8 : a.ups_bf16;
                stage += (a1 - a0 + ups - 1) / ups;
            }
            seg_units(k, g, f0, fend);
            const int j = P.gjob[g], kind = P.jkind[j];
            const int r0 = (g - P.jg0[j]) * GM;  // first pair rank of the group
            const int nt = min(GM, P.jp0[j + 1] - P.jp0[j] - r0);
            Seg& sg = me.seg[k];
            sg.src = P.jw1[j] + (size_t)f0 * unit_bytes(kind, H);
            sg.sc = kind == kKindQ8 ? P.jsc[j] : nullptr;
            sg.kind = kind;
            sg.f0 = f0;
            sg.nu = fend - f0;
            sg.nt = nt;
            sg.gidx = s * kSegPerCta + k;
            sg.grp = g;
            sg.pad0 = sg.pad1 = 0;
#pragma unroll
            for (int i = 0; i < kGroupMax; i++) sg.tok[i] = P.ptok[P.jp0[j] + r0 + min(i, nt - 1)];
            me.seg_stage[k] = stage;
            if (k == nseg - 1) {
                const int ups = kind == kKindQ8 ? a.ups_q8 : a.ups_bf16;
                me.seg_stage[nseg] = me.nstage = stage + (fend - f0 + ups - 1) / ups;
            }
        }
        if (tid == kPlanThr - 1) {
            if (ue > uf && (ue - 1) / F - uf / F + 1 > kSegPerCta) atomicOr(a.err, kErrBadIndex);  // never expected
            if (nseg == 0) me.seg_stage[0] = me.nstage = 0;
            me.nseg = nseg;
            me.nred = nred;
            const int H4 = H / 4;
            me.q0 = (int)((long long)s * H4 / G);
            me.q1 = (int)((long long)(s + 1) * H4 / G);
            sh.T = T;
            sh.np = np;
            sh.ngrp = P.ngrp;
        }
    }
    __syncthreads();
}

// A call's plan as a planner CTA publishes it for the decode grid: the structures every decode CTA
// would otherwise compute itself (routing and jobs, the reduction tables, every CTA's share).
struct __align__(16) PubPlan {
    CallPlan P;
    PlanShared sh;
    PlanCta cta[kPlanMaxGrid];
};

// Share s's segments written straight to `out` by one warp (the planner's: a warp per share), lane k
// building segment k, after plan_tables filled P.uf.  The same segments as plan_call's P7 builds
// for its own share.
__device__ void plan_share_warp(const PlanIn& a, const CallPlan& P, int s, PlanCta* out) {
    const int lane = threadIdx.x & 31;
    const int H = a.H, F = a.F, G = a.G, GM = a.gmax;
    const int uf = P.uf[s], ue = P.uf[s + 1];
    const int nseg = min(kSegPerCta, ue > uf ? (ue - 1) / F - uf / F + 1 : 0);
    int nst = 0;  // ring stages of this lane's segment
    if (lane < nseg) {
        const int k = lane, g = uf / F + k, j = P.gjob[g], kind = P.jkind[j];
        const int f0 = k == 0 ? uf % F : 0;
        const int fend = g == (ue - 1) / F ? (ue - 1) % F + 1 : F;
        const int r0 = (g - P.jg0[j]) * GM;
        const int nt = min(GM, P.jp0[j + 1] - P.jp0[j] - r0);
        Seg sg;
        sg.src = P.jw1[j] + (size_t)f0 * unit_bytes(kind, H);
        sg.sc = kind == kKindQ8 ? P.jsc[j] : nullptr;
        sg.kind = kind;
        sg.f0 = f0;
        sg.nu = fend - f0;
        sg.nt = nt;
        sg.gidx = s * kSegPerCta + k;
        sg.grp = g;
        sg.pad0 = sg.pad1 = 0;
#pragma unroll
        for (int i = 0; i < kGroupMax; i++) sg.tok[i] = P.ptok[P.jp0[j] + r0 + min(i, nt - 1)];
        out->seg[k] = sg;
        const int ups = kind == kKindQ8 ? a.ups_q8 : a.ups_bf16;
        nst = (sg.nu + ups - 1) / ups;
    }
    int incl = nst;  // stage prefix over the segments
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += y;
    }
    if (lane <= nseg) out->seg_stage[lane] = incl - nst;  // lane nseg: the total
    const int total = __shfl_sync(0xffffffffu, incl, 31);
    if (lane == 0) {
        out->nseg = nseg;
        out->nstage = total;
        out->nred = a.nred;
        const int H4 = H / 4;
        out->q0 = (int)((long long)s * H4 / G);
        out->q1 = (int)((long long)(s + 1) * H4 / G);
    }
}

// The reduction's segment tables: every share's boundaries, segment counts and call-wide numbering,
// then per call-wide segment its slot and rows and per group its segment range.  The nthr threads
// with ids tid in [0, nthr) of named barrier `bar` take part; G <= kPlanMaxGrid.
__device__ void plan_tables(CallPlan& P, PlanShared& sh, int G, int F, int H, int GM, int tid, int nthr, int bar) {
    const int ngrp = P.ngrp;
    for (int ss = tid; ss <= G; ss += nthr) P.uf[ss] = plan_unit_at(P, ss, G, F, H);
    for (int g = tid; g < kMaxGroups; g += nthr) sh.gvs0[g] = sh.gvs1[g] = 0;
    named_bar_sync(bar, nthr);
    for (int ss = tid; ss < G; ss += nthr) {
        const int uf = P.uf[ss], ue = P.uf[ss + 1];
        P.nseg[ss] = ue > uf ? min(kSegPerCta, (ue - 1) / F - uf / F + 1) : 0;
    }
    named_bar_sync(bar, nthr);
    if (tid < 32) {  // exclusive scan of segment counts -> call-wide segment numbers
        int run = 0;
        for (int s0 = 0; s0 < G; s0 += 32) {
            const int ss = s0 + tid;
            const int v = ss < G ? P.nseg[ss] : 0;
            int incl = v;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int y = __shfl_up_sync(0xffffffffu, incl, o);
                if (tid >= o) incl += y;
            }
            if (ss < G) P.seg0[ss] = run + incl - v;
            run += __shfl_sync(0xffffffffu, incl, 31);
        }
        if (tid == 0) {
            P.seg0[G] = run;
            sh.nsegtot = min(run, kMaxSegTotal);
        }
    }
    named_bar_sync(bar, nthr);
    for (int ss = tid; ss < G; ss += nthr) {
        const int uf = P.uf[ss], ue = P.uf[ss + 1];
        for (int k = 0; k < P.nseg[ss]; k++) {
            const int g = uf / F + k, gidx = P.seg0[ss] + k;
            if (gidx >= kMaxSegTotal || g >= ngrp) break;
            const int j = P.gjob[g];
            const int r0 = (g - P.jg0[j]) * GM;
            P.segslot[gidx] = ss * kSegPerCta + k;
            sh.segrows[gidx] = min(GM, P.jp0[j + 1] - P.jp0[j] - r0);
            const int f0 = k == 0 ? uf % F : 0;
            const int fend = g == (ue - 1) / F ? (ue - 1) % F + 1 : F;
            if (f0 == 0) sh.gvs0[g] = gidx;
            if (fend == F) sh.gvs1[g] = gidx + 1;
        }
    }
    named_bar_sync(bar, nthr);
    if (tid < 32) {  // staged-row prefix of the segments
        const int n = sh.nsegtot;
        int run = 0;
        for (int k0 = 0; k0 < n; k0 += 32) {
            const int k = k0 + tid;
            const int v = k < n ? sh.segrows[k] : 0;
            int incl = v;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int y = __shfl_up_sync(0xffffffffu, incl, o);
                if (tid >= o) incl += y;
            }
            if (k < n) sh.srow0[k] = run + incl - v;
            run += __shfl_sync(0xffffffffu, incl, 31);
        }
        if (tid == 0) sh.srow0[n] = run;
    }
}

}  // namespace moe
