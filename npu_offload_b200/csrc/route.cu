// Router kernels (fused softmax or sigmoid+bias / top-k / renormalise; per-token math in
// route_core.cuh) and the deterministic token->expert permutation for the B200 MoE data plane.
//
// Permutation semantics: solar_hybrid/runtime.py:343-354 -- pairs (t, k) grouped per expert with
// tokens ascending; experts listed in first-appearance order of the t-major, k-minor scan.
#include <algorithm>

#include "common.cuh"
#include "route.h"
#include "route_core.cuh"

namespace moe {

// One warp routes one token t into the global idx/w arrays (scr: the warp's shared scratch).
__device__ __forceinline__ void route_token_warp(const RouteArgs& a, int t, float* scr) {
    const bool bad = route_token(a.logits + (size_t)t * a.E, a.bias, a.E, a.K, a.scoring, a.idx + (size_t)t * a.K,
                                 a.w + (size_t)t * a.K, scr);
    if (bad && (threadIdx.x & 31) == 0) atomicOr(a.err, kErrNonFinite);
}

__global__ void __launch_bounds__(256) route_topk_kernel(RouteArgs a) {
    __shared__ __align__(16) float scr[8][2 * kMaxExperts];
    const int warp = threadIdx.x >> 5;
    const int t = blockIdx.x * 8 + warp;
    if (t < a.T) route_token_warp(a, t, scr[warp]);
}

// Counting-sort permutation of the routed pairs; one 1024-thread block.  Tokens are taken in tiles
// of 32 (one token per lane, one warp per tile): a tile's pairs of expert e are the lanes set in a
// per-warp 32-bit mask, so a pair's rank inside its tile is a popcount and the tile's count of e
// one more; an exclusive scan over the tiles per expert turns the counts into tile bases.  Every
// result is a pure function of idx (masks are ORed, first positions taken by min), so the
// permutation is deterministic.  Dynamic shared layout (permute_smem_bytes): per-warp masks
// [32][E] u32, tile counts / bases [ceil(T/32)][E] u16 (a per-expert count is at most T), then
// 8-bit copies of idx [T*K].
__host__ __device__ constexpr size_t permute_smem_bytes(int T, int K, int E) {
    return (size_t)32 * E * 4 + (((size_t)(T + 31) / 32 * E * 2 + 15) & ~(size_t)15) + (size_t)T * K;
}

struct PermShared {
    int firstpos[kMaxExperts];  // first pair index q = t*K + k of each expert (INT_MAX: absent)
    int counts[kMaxExperts];
    int offs[kMaxExperts + 1];  // expert-major grouped offsets (expert id order)
    int jrank[kMaxExperts];     // first-appearance rank among active experts (-1: absent)
    int lrank[kMaxExperts];     // the same among active local experts
    unsigned char remote[kMaxExperts];
};

// Count pass over one tile: idx -> idx8 (validated), tile counts, first appearances.
template <int KM>
__device__ __forceinline__ void permute_count_tile(const RouteArgs& a, PermShared& ps, uint32_t* wmask, uint16_t* tcnt,
                                                   unsigned char* idx8, int tile) {
    const int lane = threadIdx.x & 31, K = a.K, E = a.E;
    const int t = tile * 32 + lane;
    const bool on = t < a.T;
    const uint32_t lt = (1u << lane) - 1u;
    int ek[KM];
#pragma unroll
    for (int k = 0; k < KM; k++) ek[k] = (on && k < K) ? a.idx[(size_t)t * K + k] : 0;
#pragma unroll
    for (int k = 0; k < KM; k++)
        if (on && k < K) {
            if (ek[k] < 0 || ek[k] >= E) {  // only reachable through a corrupted idx buffer
                atomicOr(a.err, kErrBadIndex);
                ek[k] = 0;
            }
            idx8[t * K + k] = (unsigned char)ek[k];
            atomicOr(&wmask[ek[k]], 1u << lane);
        }
    __syncwarp();
#pragma unroll
    for (int k = 0; k < KM; k++)
        if (on && k < K) {
            const uint32_t m = wmask[ek[k]];
            if (!(m & lt)) {  // the tile's first pair of this expert
                tcnt[tile * E + ek[k]] = (uint16_t)__popc(m);
                atomicMin(&ps.firstpos[ek[k]], t * K + k);
            }
        }
    __syncwarp();
#pragma unroll
    for (int k = 0; k < KM; k++)
        if (on && k < K) wmask[ek[k]] = 0;
    __syncwarp();
}

// Placement pass over one tile: grouped position = expert offset + tile base + rank in the tile
// (tokens ascending, cpu_moe's per-expert token lists); the token's combine list is its positions
// ordered by job rank (the order the reference accumulates, cpu_moe.cpp:81-93), pairs owned by
// another rank marked -1.  idx: the 8-bit copy (shared) or the router's int32 output (global, an
// out-of-range id read as 0 as in the count pass); tb: the tile's bases [E].
__device__ __forceinline__ int perm_id(const unsigned char* idx, size_t q, int) { return idx[q]; }
__device__ __forceinline__ int perm_id(const int32_t* idx, size_t q, int E) {
    const int e = idx[q];
    return e < 0 || e >= E ? 0 : e;
}

template <int KM, typename IX, typename TB>
__device__ __forceinline__ void permute_place_tile(const RouteArgs& a, const int* offs, const int* jrank,
                                                   const unsigned char* remote, uint32_t* wmask, const TB* tb,
                                                   const IX* idx, int tile) {
    const int lane = threadIdx.x & 31, K = a.K, E = a.E;
    const int t = tile * 32 + lane;
    const bool on = t < a.T;
    const uint32_t lt = (1u << lane) - 1u;
    int ek[KM];
    float wk[KM];
#pragma unroll
    for (int k = 0; k < KM; k++) {
        ek[k] = (on && k < K) ? perm_id(idx, (size_t)t * K + k, E) : 0;
        wk[k] = (on && k < K && a.pw) ? a.w[(size_t)t * K + k] : 0.f;
    }
#pragma unroll
    for (int k = 0; k < KM; k++)
        if (on && k < K) atomicOr(&wmask[ek[k]], 1u << lane);
    __syncwarp();
    int rk[KM], pp[KM];
#pragma unroll
    for (int k = 0; k < KM; k++) {
        rk[k] = 0x7fffffff;
        pp[k] = -1;
        if (on && k < K) {
            const int e = ek[k];
            const int pos = offs[e] + (int)tb[e] + __popc(wmask[e] & lt);
            const int q = t * K + k;
            if (a.perm) a.perm[pos] = q;
            if (a.ptok) a.ptok[pos] = t;
            if (a.pw) a.pw[pos] = wk[k];
            if (a.pairpos) a.pairpos[q] = pos;
            rk[k] = jrank[e];
            pp[k] = remote[e] ? -1 : pos;
        }
    }
    __syncwarp();
#pragma unroll
    for (int k = 0; k < KM; k++)
        if (on && k < K) wmask[ek[k]] = 0;
    __syncwarp();
    if (a.comb_p && on) {
        // odd-even transposition sort by job rank (distinct for a token's distinct experts)
#pragma unroll
        for (int r = 0; r < KM; r++)
#pragma unroll
            for (int i = r & 1; i + 1 < KM; i += 2)
                if (rk[i] > rk[i + 1]) {
                    const int tr = rk[i], tp = pp[i];
                    rk[i] = rk[i + 1], pp[i] = pp[i + 1];
                    rk[i + 1] = tr, pp[i + 1] = tp;
                }
#pragma unroll
        for (int k = 0; k < KM; k++)
            if (k < K) a.comb_p[t * K + k] = pp[k];
        a.comb_off[t] = t * K;
    }
}

// Permutation scratch in global memory (RouteArgs::scratch, route_scratch_ints) between the counting
// block and the many-CTA placement: tile bases [ceil(T/32)][E], then offsets [E], job ranks [E],
// remote flags [E].

// place = false: the placement is left to permute_place_kernel (many CTAs: a single SM's scattered
// stores of every pair were the bottleneck); the block publishes what it needs in a.scratch.
__device__ void permute_block(const RouteArgs& a, unsigned char* dyn, bool place) {
    __shared__ PermShared ps;
    const int E = a.E, K = a.K, T = a.T;
    const int tid = threadIdx.x, nth = blockDim.x;
    const int lane = tid & 31, warp = tid >> 5, nwarps = nth >> 5;
    const int ntiles = (T + 31) / 32;
    uint32_t* wmask = reinterpret_cast<uint32_t*>(dyn) + warp * E;  // this warp's masks
    uint16_t* tcnt = reinterpret_cast<uint16_t*>(dyn + (size_t)32 * E * 4);
    unsigned char* idx8 = dyn + permute_smem_bytes(T, K, E) - (size_t)T * K;
    for (int e = tid; e < E; e += nth) {
        ps.firstpos[e] = 0x7fffffff;
        ps.remote[e] = a.desc != nullptr && a.desc[e].kind == kKindRemote;
    }
    for (int i = tid; i < 32 * E; i += nth) reinterpret_cast<uint32_t*>(dyn)[i] = 0;
    for (int i = tid; i < ntiles * E; i += nth) tcnt[i] = 0;
    __syncthreads();
    for (int tile = warp; tile < ntiles; tile += nwarps) {
        if (K <= 8)
            permute_count_tile<8>(a, ps, wmask, tcnt, idx8, tile);
        else
            permute_count_tile<kMaxTopK>(a, ps, wmask, tcnt, idx8, tile);
    }
    __syncthreads();
    for (int e = tid; e < E; e += nth) {  // exclusive scan over tiles: counts -> tile bases
        int acc = 0;
        for (int tile = 0; tile < ntiles; tile++) {
            const int c = tcnt[tile * E + e];
            tcnt[tile * E + e] = (uint16_t)acc;
            acc += c;
        }
        ps.counts[e] = acc;
    }
    __syncthreads();
    if (warp == 0) {  // expert offsets (ascending id), job counts: one warp, E/32 experts per lane
        const int per = (E + 31) / 32, e0 = lane * per;
        int sum = 0, nj = 0, nl = 0;
        for (int e = e0; e < e0 + per && e < E; e++) {
            sum += ps.counts[e];
            nj += ps.counts[e] > 0;
            nl += ps.counts[e] > 0 && !ps.remote[e];
        }
        int inc = sum;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, inc, o);
            if (lane >= o) inc += y;
        }
        int acc = inc - sum;
        for (int e = e0; e < e0 + per && e < E; e++) {
            ps.offs[e] = acc;
            acc += ps.counts[e];
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            nj += __shfl_xor_sync(0xffffffffu, nj, o);
            nl += __shfl_xor_sync(0xffffffffu, nl, o);
        }
        if (lane == 31) ps.offs[E] = inc;
        if (lane == 0) {
            if (a.n_jobs) *a.n_jobs = nj;
            if (a.n_ljobs) *a.n_ljobs = nl;
        }
    }
    // job rank = rank of the first appearance among active experts (runtime.py:343-354): a warp per
    // expert, the lanes splitting the comparison set
    for (int e = warp; e < E; e += nwarps) {
        const int fp = ps.firstpos[e];
        int r = 0, lr = 0;
        for (int e2 = lane; e2 < E; e2 += 32)
            if (ps.firstpos[e2] < fp) {
                r++;
                lr += !ps.remote[e2];
            }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            r += __shfl_xor_sync(0xffffffffu, r, o);
            lr += __shfl_xor_sync(0xffffffffu, lr, o);
        }
        if (lane == 0) {
            ps.jrank[e] = fp == 0x7fffffff ? -1 : r;
            ps.lrank[e] = fp == 0x7fffffff || ps.remote[e] ? -1 : lr;
        }
    }
    __syncthreads();
    for (int e = tid; e < E; e += nth) {
        const int cnt = ps.counts[e];
        if (a.counts) a.counts[e] = cnt;
        if (a.offsets) a.offsets[e] = ps.offs[e];
        if (cnt > 0) {
            if (a.job_order) a.job_order[ps.jrank[e]] = e;
            if (a.jobs && ps.lrank[e] >= 0) {
                Job jb;
                if (a.desc) {
                    jb.ex = a.desc[e];
                    if (jb.ex.kind != kKindBF16 && jb.ex.kind != kKindQ8) atomicOr(a.err, kErrBadExpert);
                } else {
                    jb.ex = ExpDesc{nullptr, nullptr, nullptr, 0, 0};
                }
                jb.p0 = ps.offs[e];
                jb.n = jb.ex.kind == kKindBF16 || jb.ex.kind == kKindQ8 ? cnt : 0;
                a.jobs[ps.lrank[e]] = jb;
            }
        }
    }
    if (tid == 0 && a.offsets) a.offsets[E] = ps.offs[E];
    if (!place) {
        int32_t* tb = a.scratch;
        int32_t* meta = a.scratch + (size_t)ntiles * E;
        for (int i = tid; i < ntiles * E; i += nth) tb[i] = tcnt[i];
        for (int e = tid; e < E; e += nth) {
            meta[e] = ps.offs[e];
            meta[E + e] = ps.jrank[e];
            meta[2 * E + e] = ps.remote[e];
        }
        return;
    }
    for (int tile = warp; tile < ntiles; tile += nwarps) {
        if (K <= 8)
            permute_place_tile<8>(a, ps.offs, ps.jrank, ps.remote, wmask, tcnt + (size_t)tile * E, idx8, tile);
        else
            permute_place_tile<kMaxTopK>(a, ps.offs, ps.jrank, ps.remote, wmask, tcnt + (size_t)tile * E, idx8, tile);
    }
    if (a.comb_p && tid == 0) a.comb_off[T] = T * K;
}

// Placement over many CTAs (a warp per 32-token tile) from the counting block's scratch.
constexpr int kPlaceWarps = 8;
__global__ void __launch_bounds__(kPlaceWarps * 32) permute_place_kernel(RouteArgs a) {
    __shared__ uint32_t wm[kPlaceWarps][kMaxExperts];
    __shared__ int offs[kMaxExperts], jrank[kMaxExperts];
    __shared__ unsigned char remote[kMaxExperts];
    const int E = a.E, K = a.K, T = a.T, ntiles = (T + 31) / 32;
    const int warp = threadIdx.x >> 5;
    const int32_t* meta = a.scratch + (size_t)ntiles * E;
    for (int e = threadIdx.x; e < E; e += blockDim.x) {
        offs[e] = meta[e];
        jrank[e] = meta[E + e];
        remote[e] = (unsigned char)meta[2 * E + e];
    }
    for (int i = threadIdx.x; i < kPlaceWarps * kMaxExperts; i += blockDim.x) (&wm[0][0])[i] = 0;
    __syncthreads();
    const int tile = blockIdx.x * kPlaceWarps + warp;
    if (tile < ntiles) {
        const int32_t* tb = a.scratch + (size_t)tile * E;
        if (K <= 8)
            permute_place_tile<8>(a, offs, jrank, remote, wm[warp], tb, a.idx, tile);
        else
            permute_place_tile<kMaxTopK>(a, offs, jrank, remote, wm[warp], tb, a.idx, tile);
    }
    if (a.comb_p && blockIdx.x == 0 && threadIdx.x == 0) a.comb_off[T] = T * K;
}

__global__ void __launch_bounds__(1024) permute_kernel(RouteArgs a) {
    extern __shared__ __align__(16) unsigned char pdyn[];
    permute_block(a, pdyn, a.scratch == nullptr);
}

// Small batches: routing and permutation in one launch.
__global__ void __launch_bounds__(1024) route_fused_kernel(RouteArgs a) {
    extern __shared__ __align__(16) unsigned char dyn[];
    float* scr = reinterpret_cast<float*>(dyn);  // [32][2 * kMaxExperts]
    const int warp = threadIdx.x >> 5;
    for (int t = warp; t < a.T; t += 32) route_token_warp(a, t, scr + warp * 2 * kMaxExperts);
    __syncthreads();
    permute_block(a, dyn + 32 * 2 * kMaxExperts * sizeof(float), true);
}

cudaError_t launch_route(const RouteArgs& a, cudaStream_t st, int* launches) {
    if (a.T <= 64) {
        size_t sm = 32 * 2 * kMaxExperts * sizeof(float) + permute_smem_bytes(a.T, a.K, a.E);
        route_fused_kernel<<<1, 1024, sm, st>>>(a);
        if (launches) *launches += 1;
        return cudaGetLastError();
    }
    if (a.T > 0) route_topk_kernel<<<(a.T + 7) / 8, 256, 0, st>>>(a);
    size_t sm = permute_smem_bytes(a.T, a.K, a.E);
    permute_kernel<<<1, 1024, sm, st>>>(a);
    if (launches) *launches += a.T > 0 ? 2 : 1;
    if (a.scratch && a.T > 0) {
        permute_place_kernel<<<((a.T + 31) / 32 + kPlaceWarps - 1) / kPlaceWarps, kPlaceWarps * 32, 0, st>>>(a);
        if (launches) *launches += 1;
    }
    return cudaGetLastError();
}

// The router's exponential over an array (tests compare it with the CPU oracle over every float of
// the domain the softmax sees).
__global__ void __launch_bounds__(256) router_exp_kernel(const float* x, float* y, long long n) {
    for (long long i = blockIdx.x * 256ll + threadIdx.x; i < n; i += (long long)gridDim.x * 256) y[i] = router_exp(x[i]);
}

cudaError_t launch_router_exp(const float* x, float* y, long long n, int sms, cudaStream_t st) {
    if (n <= 0) return cudaSuccess;
    const long long blocks = std::min<long long>((n + 255) / 256, (long long)sms * 8);
    router_exp_kernel<<<(unsigned)blocks, 256, 0, st>>>(x, y, n);
    return cudaGetLastError();
}

cudaError_t route_set_smem_limits() {
    cudaError_t e = cudaFuncSetAttribute(permute_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)permute_smem_bytes(kMaxTokens, kMaxTopK, kMaxExperts));
    if (e != cudaSuccess) return e;
    return cudaFuncSetAttribute(route_fused_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                (int)(32 * 2 * kMaxExperts * sizeof(float) + permute_smem_bytes(64, kMaxTopK, kMaxExperts)));
}

}  // namespace moe
