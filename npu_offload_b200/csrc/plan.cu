// Plan kernel of the fused decode path: one CTA computes everything the decode grid needs before it
// can stream weights -- routing (route_core.cuh), the token->expert grouping in first-appearance
// order (solar_hybrid/runtime.py:343-354), the local job list, and every decode CTA's byte-balanced
// share -- into a global plan, then publishes it with a release flag.
//
// It is launched with programmatic dependent launch right after the previous decode grid triggers,
// and runs on the one SM that decode grid leaves free, so for back-to-back layers the plan of layer
// l+1 is ready while layer l still streams.  Before exiting it waits for its predecessor grid, which
// makes "plan(l) complete" imply "decode(l-1) complete" for the decode grid that depends on it.
#include <climits>
#include <cstddef>

#include "common.cuh"
#include "decode.h"
#include "ptx.cuh"
#include "route_core.cuh"

namespace moe {

constexpr int kPlanThreads = kDecodeMaxT * 32;  // one warp per token

struct PlanSmem {
    int idx[kDecodeMaxT][kMaxTopK];
    float w[kDecodeMaxT][kMaxTopK];
    int counts[kMaxExperts];
    int firstpos[kMaxExperts];
    uint32_t tokmask[kMaxExperts];
    int jmap[kMaxExperts];
    int pos2e[kDecodeMaxPairs];
    long long cum1[kDecodePlanJobs + 1];  // gate/up bytes of jobs < j
    long long P1, R;
    int nbf, nq8;
    PlanShared sh;
};
static_assert(offsetof(PlanSmem, sh) % 16 == 0, "int4 copies from PlanSmem::sh");

__global__ void __launch_bounds__(kPlanThreads, 1) plan_kernel(const PlanArgs a) {
    extern __shared__ __align__(16) unsigned char dyn[];
    PlanSmem& m = *reinterpret_cast<PlanSmem*>(dyn);
    float* scr = reinterpret_cast<float*>(dyn + ((sizeof(PlanSmem) + 15) / 16) * 16);  // [warps][2*kMaxExperts]
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int T = a.T, E = a.E, K = a.K, H = a.H, F = a.F, G = a.G;
    const int NP = T * K;

    // routing: one warp per token
    if (warp < T) {
        const bool bad = route_token(a.logits + (size_t)warp * E, a.bias, E, K, a.scoring, m.idx[warp], m.w[warp],
                                     scr + warp * 2 * kMaxExperts);
        if (bad && lane == 0) atomicOr(a.err, kErrNonFinite);
    }
    for (int e = tid; e < E; e += kPlanThreads) {
        m.counts[e] = 0;
        m.firstpos[e] = INT_MAX;
        m.tokmask[e] = 0;
        m.jmap[e] = -1;
    }
    for (int q = tid; q < NP; q += kPlanThreads) m.pos2e[q] = -1;
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
    if (warp == 0) {  // local jobs in first-appearance order, pair offsets, gate/up byte prefix
        int nj = 0, np = 0, nbf = 0, nq8 = 0;
        long long cum = 0, R = 0;
        for (int q0 = 0; q0 < NP; q0 += 32) {
            const int q = q0 + lane;
            const int e = q < NP ? m.pos2e[q] : -1;
            const int kind = e >= 0 ? __ldg(&a.desc[e].kind) : kKindRemote;
            const bool local = kind == kKindBF16 || kind == kKindQ8;
            if (e >= 0 && kind == kKindNone) atomicOr(a.err, kErrBadExpert);
            const unsigned msk = __ballot_sync(0xffffffffu, local);
            const int n = local ? m.counts[e] : 0;
            const long long ub = local ? 2LL * H * (kind == kKindBF16 ? 2 : 1) * F : 0;
            int incl = n;
            long long cincl = ub;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int y = __shfl_up_sync(0xffffffffu, incl, o);
                const long long cy = __shfl_up_sync(0xffffffffu, cincl, o);
                if (lane >= o) {
                    incl += y;
                    cincl += cy;
                }
            }
            if (local) {
                const int j = nj + __popc(msk & ((1u << lane) - 1u));
                if (j < kDecodePlanJobs) {
                    const ExpDesc d = a.desc[e];
                    m.sh.jexp[j] = e;
                    m.sh.jkind[j] = kind;
                    m.sh.jlayout[j] = d.layout;
                    m.sh.jw1[j] = static_cast<const unsigned char*>(d.w1);
                    m.sh.jw2[j] = static_cast<const unsigned char*>(d.w2);
                    m.sh.jsc[j] = d.sc;
                    m.sh.jp0[j] = np + incl - n;
                    m.cum1[j] = cum + cincl - ub;
                    m.jmap[e] = j;
                }
            }
            nbf += __popc(__ballot_sync(0xffffffffu, local && kind == kKindBF16));
            nq8 += __popc(__ballot_sync(0xffffffffu, local && kind == kKindQ8));
            R += __shfl_sync(0xffffffffu, cincl, 31) / (2LL * H);
            nj += __popc(msk);
            np += __shfl_sync(0xffffffffu, incl, 31);
            cum += __shfl_sync(0xffffffffu, cincl, 31);
        }
        if (lane == 0) {
            if (nj > kDecodePlanJobs) {  // the host checks min(E, T*K) <= kDecodePlanJobs; never expected
                atomicOr(a.err, kErrBadIndex);
                nj = kDecodePlanJobs;
            }
            m.sh.nj = nj;
            m.sh.np = np;
            m.sh.T = T;
            m.sh.jp0[nj] = np;
            m.cum1[nj] = cum;
            m.P1 = cum;
            m.R = R;
            m.nbf = nbf;
            m.nq8 = nq8;
        }
    }
    __syncthreads();
    for (int q = tid; q < NP; q += kPlanThreads) {
        const int t = q / K, k = q % K, e = m.idx[t][k], j = m.jmap[e];
        if (j >= 0) {
            const int p = m.sh.jp0[j] + __popc(m.tokmask[e] & ((1u << t) - 1u));
            m.sh.ptok[p] = t;
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
        m.sh.tpn[t] = n;
    }
    __syncthreads();
    // publish the shared part
    {
        const int4* src = reinterpret_cast<const int4*>(&m.sh);
        int4* dst = reinterpret_cast<int4*>(&a.plan->sh);
        for (int q = tid; q < (int)(sizeof(PlanShared) / 16); q += kPlanThreads) dst[q] = src[q];
    }
    // every decode CTA's share: CTA ss starts at byte ss*total/G of the weight stream minus the down
    // rows of CTAs < ss (down rows split evenly by h); one thread per CTA, all evaluating the same
    // expressions, so neighbouring CTAs agree on their shared boundary
    const int nj = m.sh.nj;
    const long long P1 = m.P1, R = m.R, total = P1 + (long long)H * R;
    const double per = (double)total / G;
    auto bound = [&](int ss) -> long long {
        if (ss >= G) return P1;
        const long long hh = (long long)ss * H / G;
        const long long b = (long long)(ss * per) - hh * R;
        return b < 0 ? 0 : (b > P1 ? P1 : b);
    };
    auto unit_at = [&](long long B) -> int {  // first unit starting at or after byte B of the gate/up stream
        if (B >= P1) return nj * F;
        int lo = 0, hi = nj - 1;  // job j with cum1[j] <= B < cum1[j+1]
        while (lo < hi) {
            const int mid = (lo + hi + 1) >> 1;
            if (m.cum1[mid] <= B) lo = mid;
            else hi = mid - 1;
        }
        const long long ub = 2LL * H * (m.sh.jkind[lo] == kKindBF16 ? 2 : 1);
        return lo * F + (int)((double)(B - m.cum1[lo] + ub - 1) / (double)ub);
    };
    for (int ss = tid; ss < G; ss += kPlanThreads) {
        PlanCta pc;
        const int uf = unit_at(bound(ss)), ue0 = unit_at(bound(ss + 1));
        const int ue = ue0 > uf ? ue0 : uf;
        pc.u_first = uf;
        pc.u_end = ue;
        int n1 = 0, ns = 0;
        for (int u = uf; u < ue;) {
            const int j = u / F, seg_end = min(ue, (j + 1) * F);
            int ups = 1;
            if (m.sh.jlayout[j] == kLayoutInterleaved)
                ups = max(1, (int)(a.slot_bytes / (2u * H * (m.sh.jkind[j] == kKindBF16 ? 2u : 1u))));
            if (ns == kSegPerCta) {  // never expected: nj / G + 2 segments per CTA at most
                atomicOr(a.err, kErrBadIndex);
                break;
            }
            pc.seg_j[ns] = j;
            pc.seg_f0[ns] = u - j * F;
            pc.seg_fend[ns] = seg_end - j * F;
            pc.seg_ups[ns] = ups;
            pc.seg_stage[ns] = n1;
            n1 += (seg_end - u + ups - 1) / ups;
            ns++;
            u = seg_end;
        }
        pc.seg_stage[ns] = n1;
        pc.nseg = ns;
        pc.n1 = n1;
        pc.h0 = (int)((long long)ss * H / G);
        pc.h1 = (int)((long long)(ss + 1) * H / G);
        const int hr = pc.h1 - pc.h0;
        pc.n2 = hr > 0 ? m.nbf * ((hr + a.rs_bf16 - 1) / a.rs_bf16) + m.nq8 * ((hr + a.rs_q8 - 1) / a.rs_q8) : 0;
        pc.pad = 0;
        a.plan->cta[ss] = pc;
    }
    __syncthreads();
    if (tid == 0) {
        __threadfence();
        asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(a.flag), "r"(a.stamp) : "memory");
        griddep_launch_dependents();
        griddep_wait();  // complete only after the preceding grid: orders this call after the previous one
    }
}

static size_t plan_smem_bytes() {
    return ((sizeof(PlanSmem) + 15) / 16) * 16 + (size_t)kDecodeMaxT * 2 * kMaxExperts * sizeof(float);
}

cudaError_t plan_set_smem_limit() {
    return cudaFuncSetAttribute(plan_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)plan_smem_bytes());
}

cudaError_t launch_plan(const PlanArgs& p, cudaStream_t st) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(1);
    cfg.blockDim = dim3(kPlanThreads);
    cfg.dynamicSmemBytes = plan_smem_bytes();
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, plan_kernel, p);
}

}  // namespace moe
