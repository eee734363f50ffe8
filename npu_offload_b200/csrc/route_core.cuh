// Per-token router shared by the standalone router kernels and the fused decode kernel, so both
// produce the same bits.
//
// Semantics: npu-kernels/npu_kernels/rngd/layer_template/src/host.rs.tpl:247-268 (softmax) and
// track2_opt/solar_engine/src/host.rs:119-128 (sigmoid + correction bias):
//   softmax: m = max v; e_i = exp(v_i - m); z = sum_i e_i in index order; p_i = e_i / z;
//            top-k by p, ties -> lower index; w_k = p_k / sum_k p_k in k order (no epsilon)
//   sigmoid: s_i = 1 / (1 + exp(-v_i)); key_i = s_i + bias_i; top-k by key; w_k = s_k / (sum s + 1e-20)
// exp is evaluated in double and rounded once (router_exp: a correctly rounded expf), so the fp32
// probabilities -- and the top-k order including rounding ties -- are those of a correctly rounded
// expf.  The reference's f32::exp goes to the platform libm, which need not be correctly rounded
// (glibc 2.39's expf differs from it by one ulp on 97,052 of the 1,120,927,745 floats in [-104, 0]);
// the CPU oracle uses the same correctly rounded evaluation, and a test compares the two over every
// float of that domain.
// Both sums run sequentially in the reference's order: every lane performs the same chain of fp32
// additions on values read back (broadcast) from the warp's shared scratch, so all lanes agree.
// Top-k is a rank count over 64-bit composite keys (ordered fp32 bits, then the complemented index),
// which is exactly "larger value first, ties to the lower index".
#pragma once
#include "common.cuh"

namespace moe {

// The router's exponential: exp in double, rounded once to fp32 (host.rs.tpl:249 softmax numerator,
// host.rs:121 sigmoid denominator).
__device__ __forceinline__ float router_exp(float x) { return (float)exp((double)x); }

// Order-preserving map of a float to uint32 (NaN excluded by the caller).
__device__ __forceinline__ uint32_t ordered_bits(float f) {
    const uint32_t u = __float_as_uint(f);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// Scores of one token, one warp; S = number of 32-expert slices (E <= 32 * S).  scr: this warp's
// shared scratch of at least kMaxExperts floats (16-byte aligned); ck: shared [E] composite keys
// (written; may alias scr).  Lane l keeps element i = l + 32 s in key[s] / val[s] (its composite key and its
// probability or sigmoid value).  Returns true on every lane when some probability/key was NaN (an
// error the caller reports); NaN keys then order as -inf so the selected indices stay distinct.
template <int S>
__device__ __forceinline__ bool route_keys_s(const float* v, const float* bias, int E, int scoring, float* scr,
                                             unsigned long long* ck, unsigned long long (&mine)[S], float (&val)[S]) {
    const int lane = threadIdx.x & 31;
    float key[S];
    bool bad = false;
    const int nq = E >> 2;  // whole float4 groups of the scratch
    if (scoring == 0) {
        float m = -INFINITY;
#pragma unroll
        for (int s = 0; s < S; s++) {
            const int i = lane + 32 * s;
            key[s] = i < E ? v[i] : -INFINITY;
            m = key[s] > m ? key[s] : m;  // f32::max fold: NaN never replaces the running max
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float y = __shfl_xor_sync(0xffffffffu, m, o);
            m = y > m ? y : m;
        }
#pragma unroll
        for (int s = 0; s < S; s++) {
            const int i = lane + 32 * s;
            val[s] = i < E ? router_exp(key[s] - m) : 0.f;
            if (i < E) scr[i] = val[s];
        }
        __syncwarp();
        float z = 0.f;
        const float4* s4 = reinterpret_cast<const float4*>(scr);
#pragma unroll 8
        for (int q = 0; q < nq; q++) {
            const float4 e4 = s4[q];
            z += e4.x;
            z += e4.y;
            z += e4.z;
            z += e4.w;
        }
        for (int i = nq * 4; i < E; i++) z += scr[i];
#pragma unroll
        for (int s = 0; s < S; s++) {
            const int i = lane + 32 * s;
            const float p = __fdiv_rn(val[s], z);
            key[s] = i < E ? p : -INFINITY;
            val[s] = p;
            bad |= (i < E) && (p != p);
        }
    } else {
#pragma unroll
        for (int s = 0; s < S; s++) {
            const int i = lane + 32 * s;
            key[s] = -INFINITY;
            val[s] = 0.f;
            if (i < E) {
                const float sg = __fdiv_rn(1.0f, 1.0f + router_exp(-v[i]));
                const float k = sg + (bias ? bias[i] : 0.f);
                key[s] = k;
                val[s] = sg;
                bad |= (k != k);
            }
        }
    }
    bad = __any_sync(0xffffffffu, bad);
    __syncwarp();  // every lane's z-sum reads of scr precede key writes (ck may alias scr)
    // composite keys: ordered key bits, then the complemented index -> strictly ordered, larger first
#pragma unroll
    for (int s = 0; s < S; s++) {
        const int i = lane + 32 * s;
        const float k = key[s] != key[s] ? -INFINITY : key[s];
        mine[s] = ((unsigned long long)ordered_bits(k) << 32) | (uint32_t)(0xFFFFFFFFu - (uint32_t)i);
        if (i < E) ck[i] = mine[s];
    }
    return bad;
}

// Number of keys ck[j], j in [j0, j1), ordered before each of this lane's keys.
template <int S>
__device__ __forceinline__ void route_rank_s(const unsigned long long* ck, int j0, int j1,
                                             const unsigned long long (&mine)[S], int (&rank)[S]) {
#pragma unroll
    for (int s = 0; s < S; s++) rank[s] = 0;
#pragma unroll 4
    for (int jj = j0; jj < j1; jj++) {
        const unsigned long long kj = ck[jj];
#pragma unroll
        for (int s = 0; s < S; s++) rank[s] += kj > mine[s] ? 1 : 0;
    }
}

// The K elements of rank < K are the top-k; weights renormalised in k order (softmax: no epsilon;
// sigmoid: + 1e-20).  scr: the warp's scratch (>= 2 * kMaxTopK floats).  Lanes 0..K-1 write idx/w.
template <int S>
__device__ __forceinline__ void route_select_s(int E, int K, int scoring, const int (&rank)[S], const float (&val)[S],
                                               int* idx, float* w, float* scr) {
    const int lane = threadIdx.x & 31;
    int* sel_i = reinterpret_cast<int*>(scr);
    float* sel_v = scr + kMaxTopK;
    __syncwarp();
#pragma unroll
    for (int s = 0; s < S; s++) {
        const int i = lane + 32 * s;
        if (i < E && rank[s] < K) {
            sel_i[rank[s]] = i;
            sel_v[rank[s]] = val[s];
        }
    }
    __syncwarp();
    float tot = 0.f;
    for (int k = 0; k < K; k++) tot += sel_v[k];
    if (scoring != 0) tot += 1e-20f;
    if (lane < K) {
        idx[lane] = sel_i[lane];
        w[lane] = __fdiv_rn(sel_v[lane], tot);
    }
    __syncwarp();
}

// One warp routes one token.  scr: this warp's shared scratch of at least 2 * kMaxExperts floats
// (16-byte aligned).  Lanes 0..K-1 write idx[0..K) and w[0..K) (generic pointers: global or shared).
// Returns true on every lane when some probability/key was NaN.
template <int S>
__device__ __forceinline__ bool route_token_s(const float* v, const float* bias, int E, int K, int scoring, int* idx,
                                              float* w, float* scr) {
    unsigned long long mine[S];
    float val[S];
    // exp values, then (aliasing them) the composite keys: E <= 256 keys fill the 2 KB scratch
    unsigned long long* ck = reinterpret_cast<unsigned long long*>(scr);
    const bool bad = route_keys_s<S>(v, bias, E, scoring, scr, ck, mine, val);
    __syncwarp();
    int rank[S];
    route_rank_s<S>(ck, 0, E, mine, rank);
    route_select_s<S>(E, K, scoring, rank, val, idx, w, scr);
    return bad;
}

__device__ __forceinline__ bool route_token(const float* v, const float* bias, int E, int K, int scoring, int* idx,
                                            float* w, float* scr) {
    if (E <= 32) return route_token_s<1>(v, bias, E, K, scoring, idx, w, scr);
    if (E <= 64) return route_token_s<2>(v, bias, E, K, scoring, idx, w, scr);
    if (E <= 128) return route_token_s<4>(v, bias, E, K, scoring, idx, w, scr);
    return route_token_s<8>(v, bias, E, K, scoring, idx, w, scr);
}

}  // namespace moe
