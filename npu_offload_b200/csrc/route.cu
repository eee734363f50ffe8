// Router kernels (fused softmax or sigmoid+bias / top-k / renormalise; per-token math in
// route_core.cuh) and the deterministic token->expert permutation for the B200 MoE data plane.
//
// Permutation semantics: solar_hybrid/runtime.py:343-354 -- pairs (t, k) grouped per expert with
// tokens ascending; experts listed in first-appearance order of the t-major, k-minor scan.
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

__device__ void permute_block(const RouteArgs& a, unsigned char* dyn) {
    __shared__ int counts[kMaxExperts];
    __shared__ int firstpos[kMaxExperts];
    __shared__ int offs[kMaxExperts + 1];
    __shared__ int jrank[kMaxExperts];
    __shared__ int lrank[kMaxExperts];
    const int E = a.E, K = a.K, T = a.T, NP = T * K;
    const int tid = threadIdx.x, nth = blockDim.x;
    const int lane = tid & 31, warp = tid >> 5, nwarps = nth >> 5;
    const int ntiles = (T + 31) / 32;
    uint32_t* wmask = reinterpret_cast<uint32_t*>(dyn) + warp * E;  // this warp's masks
    uint16_t* tcnt = reinterpret_cast<uint16_t*>(dyn + (size_t)32 * E * 4);
    unsigned char* idx8 = dyn + permute_smem_bytes(T, K, E) - (size_t)NP;
    const uint32_t lt = (1u << lane) - 1u;
    for (int e = tid; e < E; e += nth) firstpos[e] = 0x7fffffff;
    for (int i = tid; i < 32 * E; i += nth) reinterpret_cast<uint32_t*>(dyn)[i] = 0;
    for (int i = tid; i < ntiles * E; i += nth) tcnt[i] = 0;
    for (int q = tid; q < NP; q += nth) {
        int e = a.idx[q];
        if (e < 0 || e >= E) {  // only reachable through a corrupted idx buffer
            atomicOr(a.err, kErrBadIndex);
            e = 0;
        }
        idx8[q] = (unsigned char)e;
    }
    __syncthreads();
    // per-tile counts and first appearances (the lowest lane of a mask holds the tile's first pair)
    for (int tile = warp; tile < ntiles; tile += nwarps) {
        const int t = tile * 32 + lane;
        const bool on = t < T;
        for (int k = 0; k < K; k++)
            if (on) atomicOr(&wmask[idx8[t * K + k]], 1u << lane);
        __syncwarp();
        for (int k = 0; k < K; k++)
            if (on) {
                const int e = idx8[t * K + k];
                const uint32_t m = wmask[e];
                if (!(m & lt)) {
                    tcnt[tile * E + e] = (uint16_t)__popc(m);
                    atomicMin(&firstpos[e], t * K + k);
                }
            }
        __syncwarp();
        for (int k = 0; k < K; k++)
            if (on) wmask[idx8[t * K + k]] = 0;
        __syncwarp();
    }
    __syncthreads();
    for (int e = tid; e < E; e += nth) {  // exclusive scan over tiles: counts -> tile bases
        int acc = 0;
        for (int tile = 0; tile < ntiles; tile++) {
            const int c = tcnt[tile * E + e];
            tcnt[tile * E + e] = (uint16_t)acc;
            acc += c;
        }
        counts[e] = acc;
    }
    __syncthreads();
    if (tid == 0) {
        int acc = 0;
        for (int e = 0; e < E; e++) {
            offs[e] = acc;
            acc += counts[e];
        }
        offs[E] = acc;
    }
    // job rank = rank of the first appearance among active experts (runtime.py:343-354)
    for (int e = tid; e < E; e += nth) {
        int r = -1, lr = -1;
        if (counts[e] > 0) {
            r = 0;
            lr = 0;
            for (int e2 = 0; e2 < E; e2++)
                if (counts[e2] > 0 && firstpos[e2] < firstpos[e]) {
                    r++;
                    if (a.desc == nullptr || a.desc[e2].kind != kKindRemote) lr++;
                }
        }
        jrank[e] = r;
        lrank[e] = lr;
    }
    __syncthreads();
    if (tid == 0) {
        int nj = 0, nl = 0;
        for (int e = 0; e < E; e++)
            if (counts[e] > 0) {
                nj++;
                if (a.desc == nullptr || a.desc[e].kind != kKindRemote) nl++;
            }
        if (a.n_jobs) *a.n_jobs = nj;
        if (a.n_ljobs) *a.n_ljobs = nl;
    }
    for (int e = tid; e < E; e += nth) {
        if (a.counts) a.counts[e] = counts[e];
        if (a.offsets) a.offsets[e] = offs[e];
        if (counts[e] > 0) {
            if (a.job_order) a.job_order[jrank[e]] = e;
            if (a.jobs && lrank[e] >= 0 && (a.desc == nullptr || a.desc[e].kind != kKindRemote)) {
                Job jb;
                if (a.desc) {
                    jb.ex = a.desc[e];
                    if (jb.ex.kind != kKindBF16 && jb.ex.kind != kKindQ8) atomicOr(a.err, kErrBadExpert);
                } else {
                    jb.ex = ExpDesc{nullptr, nullptr, nullptr, 0, 0};
                }
                jb.p0 = offs[e];
                jb.n = jb.ex.kind == kKindBF16 || jb.ex.kind == kKindQ8 ? counts[e] : 0;
                a.jobs[lrank[e]] = jb;
            }
        }
    }
    if (tid == 0 && a.offsets) a.offsets[E] = offs[E];
    __syncthreads();
    // stable placement: position = expert offset + tile base + rank inside the tile (tokens ascending)
    for (int tile = warp; tile < ntiles; tile += nwarps) {
        const int t = tile * 32 + lane;
        const bool on = t < T;
        for (int k = 0; k < K; k++)
            if (on) atomicOr(&wmask[idx8[t * K + k]], 1u << lane);
        __syncwarp();
        for (int k = 0; k < K; k++)
            if (on) {
                const int e = idx8[t * K + k];
                const int pos = offs[e] + tcnt[tile * E + e] + __popc(wmask[e] & lt);
                const int q = t * K + k;
                if (a.perm) a.perm[pos] = q;
                if (a.ptok) a.ptok[pos] = t;
                if (a.pw) a.pw[pos] = a.w[q];
                if (a.pairpos) a.pairpos[q] = pos;
            }
        __syncwarp();
        for (int k = 0; k < K; k++)
            if (on) wmask[idx8[t * K + k]] = 0;
        __syncwarp();
    }
    __syncthreads();
    // per-token pair list in job order (the order the reference accumulates, cpu_moe.cpp:81-93);
    // pairs of experts owned by another rank are marked -1
    if (a.comb_p) {
        for (int t = tid; t < T; t += nth) {
            int rk[kMaxTopK], pp[kMaxTopK];
            for (int k = 0; k < K; k++) {
                int e = idx8[t * K + k];
                rk[k] = jrank[e];
                bool remote = a.desc != nullptr && a.desc[e].kind == kKindRemote;
                pp[k] = remote ? -1 : a.pairpos[t * K + k];
            }
            for (int i = 1; i < K; i++) {  // insertion sort by job rank
                int r = rk[i], p = pp[i], j = i - 1;
                while (j >= 0 && rk[j] > r) {
                    rk[j + 1] = rk[j];
                    pp[j + 1] = pp[j];
                    j--;
                }
                rk[j + 1] = r;
                pp[j + 1] = p;
            }
            for (int k = 0; k < K; k++) a.comb_p[t * K + k] = pp[k];
            a.comb_off[t] = t * K;
            if (t == T - 1) a.comb_off[T] = T * K;
        }
        if (T == 0 && tid == 0) a.comb_off[0] = 0;
    }
}

__global__ void __launch_bounds__(1024) permute_kernel(RouteArgs a) {
    extern __shared__ __align__(16) unsigned char pdyn[];
    permute_block(a, pdyn);
}

// Small batches: routing and permutation in one launch.
__global__ void __launch_bounds__(1024) route_fused_kernel(RouteArgs a) {
    extern __shared__ __align__(16) unsigned char dyn[];
    float* scr = reinterpret_cast<float*>(dyn);  // [32][2 * kMaxExperts]
    const int warp = threadIdx.x >> 5;
    for (int t = warp; t < a.T; t += 32) route_token_warp(a, t, scr + warp * 2 * kMaxExperts);
    __syncthreads();
    permute_block(a, dyn + 32 * 2 * kMaxExperts * sizeof(float));
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
