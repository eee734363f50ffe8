// Shared device helpers for the B200 MoE data plane (sm_100a).
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

namespace moe {

constexpr int kMaxExperts = 256;
constexpr int kMaxTopK = 16;
constexpr int kMaxTokens = 4096;

// Latched device-side error bits (ctx->dev_err); host maps them to MOE_E* codes.
constexpr uint32_t kErrNonFinite = 1u;
constexpr uint32_t kErrTimeout = 2u;
constexpr uint32_t kErrBadExpert = 4u;
constexpr uint32_t kErrBadIndex = 8u;

// ExpDesc::kind values (kKindRemote: owned by another expert-parallel rank, skipped here).
constexpr int kKindNone = 0;
constexpr int kKindBF16 = 1;
constexpr int kKindQ8 = 2;
constexpr int kKindRemote = 3;

// Weight layouts of ExpDesc.
//   kLayoutSplit: w1 = [F gate rows][F up rows] of H (the reference's [Wg; Wu], cpu_moe.cpp:4),
//                 w2 = [H, F] down rows; int8 scales sc = [2F + H] (gate f, up F+f, down 2F+h).
//   kLayoutUnit:  expert tables held by a context.  One unit per intermediate index f, stored
//                 contiguously so that a CTA owning units [f0, f1) streams them as one run:
//                   bf16: [gate row f | up row f | down column f] = 3H elements
//                   int8: [gate row f | up row f | down column f | sc_gate f, sc_up f, 0, 0 (fp32)]
//                         = 3H + 16 bytes
//                 (down column f = W2[:, f]).  w1 = unit 0, w2 = w1 + 2H elements (down column 0),
//                 sc = the separate [2F + H] scale array (also used for the down scales).
constexpr int kLayoutSplit = 0;
constexpr int kLayoutUnit = 2;

// Per (layer, expert) storage descriptor, resident in HBM.
struct ExpDesc {
    const void* w1;
    const void* w2;
    const float* sc;
    int32_t kind;
    int32_t layout;
};

// Elements (bf16) or bytes (int8) between consecutive units of a kLayoutUnit table.
__host__ __device__ __forceinline__ size_t unit_pitch(int kind, int H) {
    return kind == kKindQ8 ? (size_t)3 * H + 16 : (size_t)3 * H;
}
// Bytes of one unit.
__host__ __device__ __forceinline__ size_t unit_bytes(int kind, int H) {
    return kind == kKindQ8 ? (size_t)3 * H + 16 : (size_t)6 * H;
}
// Planning cost of one unit, in bytes of the bf16 stream: a bf16 unit costs its bytes; an int8 unit
// costs q8_cost (its bytes are half, but its dequantising dots take longer per byte, so a byte
// balance would leave the CTAs holding int8 units last to finish).
__host__ __device__ __forceinline__ long long unit_cost(int kind, int H, int q8_cost) {
    return kind == kKindQ8 ? (long long)q8_cost : (long long)6 * H;
}

// Element offsets of gate row f and up row f inside w1.
__host__ __device__ __forceinline__ size_t gate_row(const ExpDesc& d, int f, int H, int F) {
    return d.layout == kLayoutUnit ? (size_t)f * unit_pitch(d.kind, H) : (size_t)f * H;
}
__host__ __device__ __forceinline__ size_t up_row(const ExpDesc& d, int f, int H, int F) {
    return d.layout == kLayoutUnit ? (size_t)f * unit_pitch(d.kind, H) + H : (size_t)(F + f) * H;
}

// One expert job of a forward call: which weights, which pairs.
//   pairs [p0, p0+n) of the expert-major pair list; pair p -> token tok[p], weight wt[p]
struct Job {
    ExpDesc ex;
    int32_t p0;
    int32_t n;
};

__device__ __forceinline__ float bf_lo(uint32_t v) { return __uint_as_float(v << 16); }
__device__ __forceinline__ float bf_hi(uint32_t v) { return __uint_as_float(v & 0xFFFF0000u); }
__device__ __forceinline__ float bf2f(uint16_t b) { return __uint_as_float(((uint32_t)b) << 16); }

// fp32 -> bf16 bits, round to nearest even with no NaN special case (same bits as the
// reference's f2bf, solar_hybrid/cpu_moe.cpp:30-34, for every input).
__device__ __forceinline__ uint16_t f2bf(float f) {
    uint32_t u = __float_as_uint(f);
    u += 0x7FFFu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}

// SwiGLU activation rounded to bf16, the reference's expression order: g / (1 + exp(-g)) * u
// (cpu_moe.cpp:75).  expf/IEEE division (no fast-math) keep it within an ulp of the host value.
__device__ __forceinline__ uint16_t swiglu_bf16(float g, float u) { return f2bf(g / (1.f + expf(-g)) * u); }

// Streaming 128-bit load: read-only, no L1 allocation (weights are read exactly once per call).
__device__ __forceinline__ uint4 ldg_stream(const void* p) {
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
    return r;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// 8 bf16 (one uint4) dot 8 bf16, fp32 FMA into acc.
__device__ __forceinline__ float dot8_bf16(uint4 w, uint4 x, float acc) {
    acc = fmaf(bf_lo(w.x), bf_lo(x.x), acc);
    acc = fmaf(bf_hi(w.x), bf_hi(x.x), acc);
    acc = fmaf(bf_lo(w.y), bf_lo(x.y), acc);
    acc = fmaf(bf_hi(w.y), bf_hi(x.y), acc);
    acc = fmaf(bf_lo(w.z), bf_lo(x.z), acc);
    acc = fmaf(bf_hi(w.z), bf_hi(x.z), acc);
    acc = fmaf(bf_lo(w.w), bf_lo(x.w), acc);
    acc = fmaf(bf_hi(w.w), bf_hi(x.w), acc);
    return acc;
}

// Packed fp32 pairs (sm_100 f32x2 arithmetic): low word = lower address element.
typedef unsigned long long f32x2;
__device__ __forceinline__ f32x2 pack_f32x2(float lo, float hi) {
    f32x2 r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
    return r;
}
__device__ __forceinline__ float sum_f32x2(f32x2 v) {
    float lo, hi;
    asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
    return lo + hi;
}
__device__ __forceinline__ void unpack_f32x2(f32x2 v, float& lo, float& hi) {
    asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
// two bf16 (one 32-bit word) widened to an fp32 pair
__device__ __forceinline__ f32x2 bf16x2_to_f32x2(uint32_t w) { return pack_f32x2(bf_lo(w), bf_hi(w)); }
// d = a * b + c per element, round to nearest (two fmaf in one instruction)
__device__ __forceinline__ f32x2 ffma2(f32x2 a, f32x2 b, f32x2 c) {
    f32x2 d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
    return d;
}

// Mixed-precision FMA (sm_100): bf16 x bf16 products accumulated in fp32 with one rounding -- the
// same bits as fmaf on the widened operands (a bf16 product is exact in fp32), without widening.
// lo += w.lo * x.lo, hi += w.hi * x.hi for two packed bf16 pairs.
__device__ __forceinline__ void fma_bf16x2(uint32_t w, uint32_t x, float& lo, float& hi) {
    asm("{\n\t.reg .b16 wl, wh, xl, xh;\n\t"
        "mov.b32 {wl, wh}, %2;\n\t"
        "mov.b32 {xl, xh}, %3;\n\t"
        "fma.rn.f32.bf16 %0, wl, xl, %0;\n\t"
        "fma.rn.f32.bf16 %1, wh, xh, %1;\n\t}"
        : "+f"(lo), "+f"(hi)
        : "r"(w), "r"(x));
}
// lo += w.lo * s, hi += w.hi * s with s the bf16 in the low half of a (a scalar times a pair).
__device__ __forceinline__ void fma_bf16x2_s(uint32_t w, uint32_t a, float& lo, float& hi) {
    asm("{\n\t.reg .b16 wl, wh, al, ah;\n\t"
        "mov.b32 {wl, wh}, %2;\n\t"
        "mov.b32 {al, ah}, %3;\n\t"
        "fma.rn.f32.bf16 %0, wl, al, %0;\n\t"
        "fma.rn.f32.bf16 %1, wh, al, %1;\n\t}"
        : "+f"(lo), "+f"(hi)
        : "r"(w), "r"(a));
}

// Sums 8 per-lane values across the warp with 9 shuffles: afterwards lane l holds the total of
// value (l >> 2).
__device__ __forceinline__ float warp_sum8(const float (&v)[8]) {
    const int lane = threadIdx.x & 31;
    float a[4], b[2];
    const bool h16 = (lane >> 4) & 1, h8 = (lane >> 3) & 1, h4 = (lane >> 2) & 1;
#pragma unroll
    for (int k = 0; k < 4; k++)
        a[k] = (h16 ? v[k + 4] : v[k]) + __shfl_xor_sync(0xffffffffu, h16 ? v[k] : v[k + 4], 16);
#pragma unroll
    for (int k = 0; k < 2; k++)
        b[k] = (h8 ? a[k + 2] : a[k]) + __shfl_xor_sync(0xffffffffu, h8 ? a[k] : a[k + 2], 8);
    float c = (h4 ? b[1] : b[0]) + __shfl_xor_sync(0xffffffffu, h4 ? b[0] : b[1], 4);
    c += __shfl_xor_sync(0xffffffffu, c, 2);
    c += __shfl_xor_sync(0xffffffffu, c, 1);
    return c;
}

// Sums V per-lane values (V a power of two, <= 32) across the warp with V - 1 + 5 - log2(V)
// shuffles (recursive halving).  Afterwards every lane of the group of 32/V consecutive lanes
// l with l / (32 / V) == i holds the total of value i; the additions follow a fixed tree, so
// every warp computing the same inputs gets the same bits.
template <int V>
__device__ __forceinline__ float warp_sum_multi(float (&v)[V]) {
    static_assert(V >= 1 && V <= 32 && (V & (V - 1)) == 0, "V must be a power of two <= 32");
    const int lane = threadIdx.x & 31;
    int n = V;
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) {
        if (n > 1) {
            const bool up = (lane & o) != 0;
#pragma unroll
            for (int k = 0; k < V / 2; k++) {
                if (k < n / 2) {
                    const float keep = up ? v[k + n / 2] : v[k];
                    const float give = up ? v[k] : v[k + n / 2];
                    v[k] = keep + __shfl_xor_sync(0xffffffffu, give, o);
                }
            }
            n >>= 1;
        } else {
            v[0] += __shfl_xor_sync(0xffffffffu, v[0], o);
        }
    }
    return v[0];
}

// int8 value k (0..3) of a 32-bit word, exactly as float.  The byte plus 128 (the sign bit flipped)
// is moved into the low mantissa bits of 2^23 by one byte permute, and 2^23 + 128 is subtracted:
// exact for every int8, and it keeps the conversion off the slower integer-to-float pipe.
__device__ __forceinline__ float i8f(uint32_t v, int k) {
    return __uint_as_float(__byte_perm(v ^ 0x80808080u, 0x4B000000u, 0x7540 | k)) - 8388736.f;
}

// 4 int8 weights (one u32) dot 4 bf16 activations (two u32), fp32.
__device__ __forceinline__ float dot4_i8(uint32_t w, uint32_t x01, uint32_t x23, float acc) {
    acc = fmaf(i8f(w, 0), bf_lo(x01), acc);
    acc = fmaf(i8f(w, 1), bf_hi(x01), acc);
    acc = fmaf(i8f(w, 2), bf_lo(x23), acc);
    acc = fmaf(i8f(w, 3), bf_hi(x23), acc);
    return acc;
}

}  // namespace moe
