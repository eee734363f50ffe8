// Prefill expert GEMMs on the 5th-generation tensor cores (tcgen05, sm_100a), for the pairs p of
// every local bf16 expert job (solar_hybrid/cpu_moe.cpp:63-93):
//   gate/up  act[p, f] = bf16_rne(g / (1 + exp(-g)) * u), g / u = gate / up row f . x_p in fp32
//            (SwiGLU fused into the epilogue)
//   down     y[p, h] = down row h . act_p in fp32 (MN-major weight operand: the stored down columns)
//
// One CTA = one tile: 256 pairs (two 128-row halves) x 128 intermediate indices of one job.
//   producer warp   TMA (cp.async.bulk.tensor, 128-byte swizzle) of the gathered token rows
//                   [256 x 64] and the job's gate and up rows [128 x 64] per K step into a 3-stage
//                   shared-memory ring (mbarrier complete_tx)
//   MMA warp        allocates 512 TMEM columns; one thread issues tcgen05.mma kind::f16 (bf16 x bf16
//                   -> fp32, M 128, N 128, K 16) into four accumulators (gate / up x two halves) and
//                   commits each stage back to the producer; the second half is skipped when the job
//                   has <= 128 pairs in the tile
//   8 epilogue warps  tcgen05.ld the fp32 accumulators (warp w: TMEM lanes 32 (w % 4) .., half w / 4),
//                   apply SwiGLU, round to bf16, store the pair's 128 activations
// Weights are read in place from the unit tables through a 3-D tensor map (unit element, f, expert
// slot); the gathered rows through a 2-D map.  Every wait is bounded; a CTA that gives up raises
// kErrTimeout, lets its in-flight MMAs finish and frees its TMEM before returning.
#include <cuda.h>

#include <cute/arch/mma_sm100_desc.hpp>

#include "common.cuh"
#include "prefill_tc.h"
#include "ptx.cuh"

namespace moe {

constexpr int kTcBM = 256, kTcBN = 128, kTcBK = 64, kTcStages = 3;
constexpr int kTcEpiWarps = 8, kTcProdWarp = kTcEpiWarps, kTcMmaWarp = kTcEpiWarps + 1, kTcThreads = 10 * 32;
constexpr uint32_t kTcABytes = kTcBM * kTcBK * 2, kTcBBytes = kTcBN * kTcBK * 2;
constexpr uint32_t kTcStageBytes = kTcABytes + 2 * kTcBBytes;  // A, gate, up
constexpr size_t kTcSmem = (size_t)kTcStages * kTcStageBytes + 1024 + 256;

struct TcCtrl {
    uint64_t full[kTcStages], empty[kTcStages], accum, done;
    uint32_t tmem;
    int abort;
};

__device__ __forceinline__ bool tc_wait(uint64_t* bar, uint32_t parity, int* abort, uint32_t* err, uint64_t deadline) {
    while (!mbar_try_wait_sleep(bar, parity, 20000u)) {
        if (*(volatile int*)abort) return false;
        if (globaltimer_ns() > deadline) {
            *(volatile int*)abort = 1;
            atomicOr(err, kErrTimeout);
            return false;
        }
    }
    return true;
}

// K-major operand in the 128-byte swizzle layout TMA writes for a 64-element (128-byte) inner box:
// rows 128 bytes apart, 8-row (1 KB) swizzle atoms stacked at 1 KB (SBO); the K-slice of a K=16 MMA
// starts 32 bytes further per step inside the atom.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
    cute::UMMA::SmemDescriptor d;
    d.desc_ = 0;
    d.start_address_ = (uint16_t)(saddr >> 4);
    d.leading_byte_offset_ = 1;
    d.stride_byte_offset_ = 1024 >> 4;
    d.version_ = 1;
    d.base_offset_ = 0;
    d.lbo_mode_ = 0;
    d.layout_type_ = (uint8_t)cute::UMMA::LayoutType::SWIZZLE_128B;
    return d.desc_;
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
            smem_u32(dst)),
        "l"(map), "r"(smem_u32(bar)), "r"(x), "r"(y)
        : "memory");
}

__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, int x, int y, int z, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(
            smem_u32(dst)),
        "l"(map), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z)
        : "memory");
}

__device__ __forceinline__ void umma_bf16(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(da), "l"(db), "r"(idesc), "r"(acc));
}

__device__ __forceinline__ void umma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&v)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
          "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]),
          "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]),
          "=r"(v[24]), "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
        : "r"(taddr));
}

__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__global__ void __launch_bounds__(kTcThreads, 1)
    gateup_tc_kernel(const __grid_constant__ CUtensorMap map_x, const __grid_constant__ CUtensorMap map_w,
                     const TcItem* __restrict__ items, int H, int F, uint16_t* __restrict__ act, uint32_t* err,
                     uint64_t timeout_ns) {
    extern __shared__ __align__(1024) unsigned char tsm[];
    unsigned char* ring = reinterpret_cast<unsigned char*>(((uintptr_t)tsm + 1023) & ~(uintptr_t)1023);
    TcCtrl& c = *reinterpret_cast<TcCtrl*>(ring + (size_t)kTcStages * kTcStageBytes);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const TcItem it = items[blockIdx.x];
    const int nk = H / kTcBK;
    const bool two = it.rows > 128;  // the second 128-row half has pairs of this job
    if (threadIdx.x == 0) {
        for (int s = 0; s < kTcStages; s++) {
            mbar_init(&c.full[s], 1);
            mbar_init(&c.empty[s], 1);
        }
        mbar_init(&c.accum, 1);
        mbar_init(&c.done, 1);
        c.abort = 0;
        fence_mbar_init();
    }
    if (warp == kTcMmaWarp) {  // whole warp: allocate the four 128-column accumulators
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&c.tmem)),
                     "r"(512));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::);
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = c.tmem;
    const uint64_t deadline = globaltimer_ns() + timeout_ns;

    if (warp == kTcProdWarp) {
        if (lane == 0) {
            int k = 0;
            for (; k < nk; k++) {
                const int s = k % kTcStages;
                if (k >= kTcStages && !tc_wait(&c.empty[s], ((k / kTcStages) & 1) ^ 1, &c.abort, err, deadline)) break;
                unsigned char* st = ring + (size_t)s * kTcStageBytes;
                mbar_arrive_expect_tx(&c.full[s], kTcStageBytes);
                tma_load_2d(st, &map_x, k * kTcBK, it.row0, &c.full[s]);
                tma_load_3d(st + kTcABytes, &map_w, k * kTcBK, it.f0, it.slot, &c.full[s]);
                tma_load_3d(st + kTcABytes + kTcBBytes, &map_w, H + k * kTcBK, it.f0, it.slot, &c.full[s]);
            }
            // every issued copy lands before the CTA may exit
            const uint64_t dd = globaltimer_ns() + timeout_ns;
            for (int q = k > kTcStages ? k - kTcStages : 0; q < k; q++)
                while (!mbar_try_wait(&c.full[q % kTcStages], (q / kTcStages) & 1))
                    if (globaltimer_ns() > dd) break;
        }
    } else if (warp == kTcMmaWarp) {
        if (lane == 0) {
            const uint32_t idesc = (uint32_t)cute::UMMA::make_instr_desc<cute::bfloat16_t, cute::bfloat16_t, float, 128, 128,
                                                                          cute::UMMA::Major::K, cute::UMMA::Major::K>();
            for (int k = 0; k < nk; k++) {
                const int s = k % kTcStages;
                if (!tc_wait(&c.full[s], (k / kTcStages) & 1, &c.abort, err, deadline)) break;
                tc_fence_after();
                const uint32_t sa = smem_u32(ring + (size_t)s * kTcStageBytes);
                const uint32_t sg = sa + kTcABytes, su = sg + kTcBBytes;
#pragma unroll
                for (int kk = 0; kk < kTcBK / 16; kk++) {
                    const uint32_t acc = (k | kk) != 0;
                    const uint64_t dg = sw128_desc(sg + kk * 32), du = sw128_desc(su + kk * 32);
                    const uint64_t da0 = sw128_desc(sa + kk * 32);
                    umma_bf16(tmem + 0, da0, dg, idesc, acc);    // gate, rows 0..127
                    umma_bf16(tmem + 128, da0, du, idesc, acc);  // up,   rows 0..127
                    if (two) {
                        const uint64_t da1 = sw128_desc(sa + 128 * 128 + kk * 32);
                        umma_bf16(tmem + 256, da1, dg, idesc, acc);  // gate, rows 128..255
                        umma_bf16(tmem + 384, da1, du, idesc, acc);  // up,   rows 128..255
                    }
                }
                umma_commit(&c.empty[s]);  // the stage is free once these MMAs have read it
            }
            umma_commit(&c.accum);  // accumulators complete (also the final fence for every MMA issued)
        }
    } else {
        // epilogue: warp w -> TMEM lanes [32 (w % 4), +32), half w / 4
        const int h = warp / 4, q = warp % 4;
        const int r = h * 128 + q * 32 + lane;  // row of the tile this thread writes
        if (tc_wait(&c.accum, 0, &c.abort, err, deadline) && (h == 0 || two)) {
            tc_fence_after();
            const uint32_t lane_addr = (uint32_t)(q * 32) << 16;
            for (int c0 = 0; c0 < kTcBN; c0 += 32) {
                uint32_t g[32], u[32];
                tmem_ld32(tmem + lane_addr + h * 256 + c0, g);
                tmem_ld32(tmem + lane_addr + h * 256 + 128 + c0, u);
                tmem_wait_ld();
                if (r < it.rows) {
                    uint32_t o[16];
#pragma unroll
                    for (int e = 0; e < 16; e++)
                        o[e] = (uint32_t)swiglu_bf16(__uint_as_float(g[2 * e]), __uint_as_float(u[2 * e])) |
                               ((uint32_t)swiglu_bf16(__uint_as_float(g[2 * e + 1]), __uint_as_float(u[2 * e + 1])) << 16);
                    uint4* dst = reinterpret_cast<uint4*>(act + (size_t)(it.row0 + r) * F + it.f0 + c0);
                    dst[0] = make_uint4(o[0], o[1], o[2], o[3]);
                    dst[1] = make_uint4(o[4], o[5], o[6], o[7]);
                    dst[2] = make_uint4(o[8], o[9], o[10], o[11]);
                    dst[3] = make_uint4(o[12], o[13], o[14], o[15]);
                }
            }
        }
    }
    // all MMAs are complete before TMEM is released: the accum commit covers them; after an abort the
    // MMA thread commits once more and waits (bounded) for it
    if (warp == kTcMmaWarp && lane == 0 && *(volatile int*)&c.abort) {
        umma_commit(&c.done);
        const uint64_t dd = globaltimer_ns() + timeout_ns;
        while (!mbar_try_wait(&c.done, 0))
            if (globaltimer_ns() > dd) break;
    }
    tc_fence_before();
    __syncthreads();
    if (warp == kTcMmaWarp) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512));
    }
}

// ---- down projection: y[p, h] = sum_f act[p, f] * W2[h, f] (fp32) ----
// One CTA = 256 pairs (two halves) x 256 outputs of one job.  A = activation rows (K-major, as above);
// B = the job's down columns for f in the K step: a [64 f x 64 h] box per 64 outputs, i.e. MN-major
// with 128-byte swizzle -- 64 h (128 bytes) contiguous per f row, 8-row swizzle atoms 1 KB apart
// (SBO), the four 64-output chunks 8 KB apart (LBO); a K=16 step advances two whole atoms (2 KB).
constexpr int kDnBN = 256;
constexpr uint32_t kDnBBytes = kTcBK * kDnBN * 2;
constexpr uint32_t kDnStageBytes = kTcABytes + kDnBBytes;
constexpr size_t kDnSmem = (size_t)kTcStages * kDnStageBytes + 1024 + 256;

__device__ __forceinline__ uint64_t sw128_mn_desc(uint32_t saddr) {
    cute::UMMA::SmemDescriptor d;
    d.desc_ = 0;
    d.start_address_ = (uint16_t)(saddr >> 4);
    d.leading_byte_offset_ = (kTcBK * 128) >> 4;  // next 64-output chunk
    d.stride_byte_offset_ = 1024 >> 4;            // next 8 K rows
    d.version_ = 1;
    d.base_offset_ = 0;
    d.lbo_mode_ = 0;
    d.layout_type_ = (uint8_t)cute::UMMA::LayoutType::SWIZZLE_128B;
    return d.desc_;
}

__global__ void __launch_bounds__(kTcThreads, 1)
    down_tc_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_d,
                   const TcItem* __restrict__ items, int H, int F, float* __restrict__ y, uint32_t* err,
                   uint64_t timeout_ns) {
    extern __shared__ __align__(1024) unsigned char tsm[];
    unsigned char* ring = reinterpret_cast<unsigned char*>(((uintptr_t)tsm + 1023) & ~(uintptr_t)1023);
    TcCtrl& c = *reinterpret_cast<TcCtrl*>(ring + (size_t)kTcStages * kDnStageBytes);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const TcItem it = items[blockIdx.x];  // f0 holds the first output h of the tile
    const int nk = F / kTcBK;
    const bool two = it.rows > 128;
    if (threadIdx.x == 0) {
        for (int s = 0; s < kTcStages; s++) {
            mbar_init(&c.full[s], 1);
            mbar_init(&c.empty[s], 1);
        }
        mbar_init(&c.accum, 1);
        mbar_init(&c.done, 1);
        c.abort = 0;
        fence_mbar_init();
    }
    if (warp == kTcMmaWarp) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&c.tmem)),
                     "r"(512));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::);
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = c.tmem;
    const uint64_t deadline = globaltimer_ns() + timeout_ns;

    if (warp == kTcProdWarp) {
        if (lane == 0) {
            int k = 0;
            for (; k < nk; k++) {
                const int s = k % kTcStages;
                if (k >= kTcStages && !tc_wait(&c.empty[s], ((k / kTcStages) & 1) ^ 1, &c.abort, err, deadline)) break;
                unsigned char* st = ring + (size_t)s * kDnStageBytes;
                mbar_arrive_expect_tx(&c.full[s], kDnStageBytes);
                tma_load_2d(st, &map_a, k * kTcBK, it.row0, &c.full[s]);
#pragma unroll
                for (int j = 0; j < kDnBN / 64; j++)
                    tma_load_3d(st + kTcABytes + j * (kTcBK * 128), &map_d, 2 * H + it.f0 + j * 64, k * kTcBK, it.slot,
                                &c.full[s]);
            }
            const uint64_t dd = globaltimer_ns() + timeout_ns;
            for (int q = k > kTcStages ? k - kTcStages : 0; q < k; q++)
                while (!mbar_try_wait(&c.full[q % kTcStages], (q / kTcStages) & 1))
                    if (globaltimer_ns() > dd) break;
        }
    } else if (warp == kTcMmaWarp) {
        if (lane == 0) {
            const uint32_t idesc = (uint32_t)cute::UMMA::make_instr_desc<cute::bfloat16_t, cute::bfloat16_t, float, 128, kDnBN,
                                                                          cute::UMMA::Major::K, cute::UMMA::Major::MN>();
            for (int k = 0; k < nk; k++) {
                const int s = k % kTcStages;
                if (!tc_wait(&c.full[s], (k / kTcStages) & 1, &c.abort, err, deadline)) break;
                tc_fence_after();
                const uint32_t sa = smem_u32(ring + (size_t)s * kDnStageBytes), sb = sa + kTcABytes;
#pragma unroll
                for (int kk = 0; kk < kTcBK / 16; kk++) {
                    const uint32_t acc = (k | kk) != 0;
                    const uint64_t db = sw128_mn_desc(sb + kk * 2048);
                    umma_bf16(tmem + 0, sw128_desc(sa + kk * 32), db, idesc, acc);
                    if (two) umma_bf16(tmem + 256, sw128_desc(sa + 128 * 128 + kk * 32), db, idesc, acc);
                }
                umma_commit(&c.empty[s]);
            }
            umma_commit(&c.accum);
        }
    } else {
        const int h = warp / 4, q = warp % 4;
        const int r = h * 128 + q * 32 + lane;
        if (tc_wait(&c.accum, 0, &c.abort, err, deadline) && (h == 0 || two)) {
            tc_fence_after();
            const uint32_t lane_addr = (uint32_t)(q * 32) << 16;
            for (int c0 = 0; c0 < kDnBN; c0 += 32) {
                uint32_t v[32];
                tmem_ld32(tmem + lane_addr + h * 256 + c0, v);
                tmem_wait_ld();
                if (r < it.rows) {
                    float4* dst = reinterpret_cast<float4*>(y + (size_t)(it.row0 + r) * H + it.f0 + c0);
#pragma unroll
                    for (int e = 0; e < 8; e++)
                        dst[e] = make_float4(__uint_as_float(v[4 * e]), __uint_as_float(v[4 * e + 1]),
                                             __uint_as_float(v[4 * e + 2]), __uint_as_float(v[4 * e + 3]));
                }
            }
        }
    }
    if (warp == kTcMmaWarp && lane == 0 && *(volatile int*)&c.abort) {
        umma_commit(&c.done);
        const uint64_t dd = globaltimer_ns() + timeout_ns;
        while (!mbar_try_wait(&c.done, 0))
            if (globaltimer_ns() > dd) break;
    }
    tc_fence_before();
    __syncthreads();
    if (warp == kTcMmaWarp) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512));
    }
}

// ---- host side ----

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    static bool tried = false;
    if (!tried) {
        tried = true;
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
        else
            cudaGetLastError();
    }
    return fn;
}

bool tc_available() { return encode_fn() != nullptr; }

cudaError_t tc_set_smem_limit() {
    cudaError_t e = cudaFuncSetAttribute(gateup_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kTcSmem);
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(down_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kDnSmem);
    return e;
}

cudaError_t launch_down_tc(const uint16_t* act, int arows, const void* arena, int n_slots, size_t slot_bytes,
                           const TcItem* items, int n_items, int H, int F, float* y, uint32_t* err, uint64_t timeout_ns,
                           cudaStream_t st) {
    EncodeTiledFn enc = encode_fn();
    if (!enc) return cudaErrorNotSupported;
    if (H % kDnBN || F % kTcBK || slot_bytes % 16 || ((uintptr_t)act | (uintptr_t)arena) & 15) return cudaErrorInvalidValue;
    CUtensorMap ma, md;
    {  // activation rows: [arows][F] bf16
        const cuuint64_t dims[2] = {(cuuint64_t)F, (cuuint64_t)arows};
        const cuuint64_t strides[1] = {(cuuint64_t)F * 2};
        const cuuint32_t box[2] = {kTcBK, kTcBM}, es[2] = {1, 1};
        if (enc(&ma, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, (void*)act, dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return cudaErrorInvalidValue;
    }
    {  // unit tables, down columns at element 2H of each unit: boxes of 64 outputs x 64 f
        const cuuint64_t dims[3] = {(cuuint64_t)3 * H, (cuuint64_t)F, (cuuint64_t)n_slots};
        const cuuint64_t strides[2] = {(cuuint64_t)6 * H, (cuuint64_t)slot_bytes};
        const cuuint32_t box[3] = {64, kTcBK, 1}, es[3] = {1, 1, 1};
        if (enc(&md, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, (void*)arena, dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return cudaErrorInvalidValue;
    }
    if (n_items <= 0) return cudaSuccess;
    down_tc_kernel<<<n_items, kTcThreads, kDnSmem, st>>>(ma, md, items, H, F, y, err, timeout_ns);
    return cudaGetLastError();
}

cudaError_t launch_gateup_tc(const uint16_t* xg, int xrows, const void* arena, int n_slots, size_t slot_bytes,
                             const TcItem* items, int n_items, int H, int F, uint16_t* act, uint32_t* err,
                             uint64_t timeout_ns, cudaStream_t st) {
    EncodeTiledFn enc = encode_fn();
    if (!enc) return cudaErrorNotSupported;
    if (H % kTcBK || F % kTcBN || slot_bytes % 16 || ((uintptr_t)xg | (uintptr_t)arena) & 15) return cudaErrorInvalidValue;
    CUtensorMap mx, mw;
    {  // gathered token rows: [xrows][H] bf16
        const cuuint64_t dims[2] = {(cuuint64_t)H, (cuuint64_t)xrows};
        const cuuint64_t strides[1] = {(cuuint64_t)H * 2};
        const cuuint32_t box[2] = {kTcBK, kTcBM}, es[2] = {1, 1};
        if (enc(&mx, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, (void*)xg, dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return cudaErrorInvalidValue;
    }
    {  // unit tables: [slot][f][3H] bf16 (gate row f at element 0 of unit f, up row at element H)
        const cuuint64_t dims[3] = {(cuuint64_t)3 * H, (cuuint64_t)F, (cuuint64_t)n_slots};
        const cuuint64_t strides[2] = {(cuuint64_t)6 * H, (cuuint64_t)slot_bytes};
        const cuuint32_t box[3] = {kTcBK, kTcBN, 1}, es[3] = {1, 1, 1};
        if (enc(&mw, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, (void*)arena, dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return cudaErrorInvalidValue;
    }
    if (n_items <= 0) return cudaSuccess;
    gateup_tc_kernel<<<n_items, kTcThreads, kTcSmem, st>>>(mx, mw, items, H, F, act, err, timeout_ns);
    return cudaGetLastError();
}

}  // namespace moe
