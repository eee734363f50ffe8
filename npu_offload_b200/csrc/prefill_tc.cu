// Prefill expert GEMMs on the 5th-generation tensor cores (tcgen05, sm_100a), for the pairs p of
// every local bf16 expert job (solar_hybrid/cpu_moe.cpp:63-93):
//   gate/up  act[p, f] = bf16_rne(g / (1 + exp(-g)) * u), g / u = gate / up row f . x_p in fp32
//            (SwiGLU fused into the epilogue)
//   down     y[p, h] = down row h . act_p in fp32 (MN-major weight operand: the stored down columns)
//
// Persistent kernel, one CTA per SM, taking tiles from a global counter (dynamic schedule; the last
// CTA to exit re-arms it).  A tile is 256 pairs (two 128-row halves) of one job x 128 intermediate
// indices (gate/up) or 256 outputs (down).
//   producer warp   TMA (cp.async.bulk.tensor, 128-byte swizzle) per K step of 64: the A rows (one
//                   [128 x 64] box per populated half) and the job's weights (gate/up: gate and up
//                   rows [128 x 64] K-major; down: four [64 f x 64 h] boxes MN-major) into a 3-stage
//                   shared-memory ring (mbarrier complete_tx) that runs on across tiles
//   MMA warp        allocates 512 TMEM columns; one thread issues tcgen05.mma kind::f16 (bf16 x bf16
//                   -> fp32, M 128, N 256, K 16; gate/up: the gate and up rows form one 256-row
//                   operand) for each populated half, commits each stage back to the producer and the
//                   finished accumulators to the epilogue
//   8 epilogue warps  tcgen05.ld the fp32 accumulators (warp w: TMEM lanes 32 (w % 4) .., half w / 4),
//                   gate/up: SwiGLU -> bf16 act rows; down: fp32 y rows; then hand the TMEM back
//                   (the producer keeps prefetching the next tile meanwhile)
// Weights are read in place from the unit tables through a 3-D tensor map (unit element, f, expert
// slot); the A rows through a 2-D map.  Every wait is bounded; a CTA that gives up raises kErrTimeout,
// lets its in-flight copies and MMAs finish and frees its TMEM before returning.
#include <cuda.h>

#include <algorithm>

#include <cute/arch/mma_sm100_desc.hpp>

#include "common.cuh"
#include "prefill_tc.h"
#include "ptx.cuh"

namespace moe {

constexpr int kTcBK = 64, kTcStages = 3;
constexpr int kTcEpiWarps = 8, kTcProdWarp = kTcEpiWarps, kTcMmaWarp = kTcEpiWarps + 1, kTcThreads = 10 * 32;
constexpr uint32_t kTcHalfA = 128 * kTcBK * 2;                 // one 128-row half of A per K step
constexpr uint32_t kTcBBytes = 32768;                          // gate + up [2 x 128 x 64] or down [64 x 256]
constexpr uint32_t kTcStage = 2 * kTcHalfA + kTcBBytes;        // 64 KB
constexpr size_t kTcSmem = (size_t)kTcStages * kTcStage + 1024 + 256;

struct TcCtrl {
    uint64_t full[kTcStages], empty[kTcStages], accum, tfree, done;
    uint64_t tq_full[2], tq_empty[2];  // tile-index hand-off: producer -> MMA thread + epilogue warps
    int tq[2];
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

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar,
                                            uint64_t policy) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1, {%3, %4}], "
        "[%2], %5;" ::"r"(smem_u32(dst)),
        "l"(map), "r"(smem_u32(bar)), "r"(x), "r"(y), "l"(policy)
        : "memory");
}

__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, int x, int y, int z, uint64_t* bar,
                                            uint64_t policy) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1, {%3, %4, "
        "%5}], [%2], %6;" ::"r"(smem_u32(dst)),
        "l"(map), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z), "l"(policy)
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


// MN-major operand (down columns): 64 outputs (128 bytes) contiguous per f row as TMA writes a
// [64 f x 64 h] box with 128-byte swizzle; 8-row swizzle atoms 1 KB apart along K (SBO), the
// 64-output chunks 8 KB apart along N (LBO); a K=16 step advances two whole atoms (2 KB).
__device__ __forceinline__ uint64_t sw128_mn_desc(uint32_t saddr) {
    cute::UMMA::SmemDescriptor d;
    d.desc_ = 0;
    d.start_address_ = (uint16_t)(saddr >> 4);
    d.leading_byte_offset_ = (kTcBK * 128) >> 4;
    d.stride_byte_offset_ = 1024 >> 4;
    d.version_ = 1;
    d.base_offset_ = 0;
    d.lbo_mode_ = 0;
    d.layout_type_ = (uint8_t)cute::UMMA::LayoutType::SWIZZLE_128B;
    return d.desc_;
}

template <bool DOWN>
__global__ void __launch_bounds__(kTcThreads, 1)
    tc_gemm_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_w,
                   const TcItem* __restrict__ items, int n_items, const int* __restrict__ n_items_dev, int H, int F,
                   void* __restrict__ out, uint32_t* sched, uint32_t* err, uint64_t timeout_ns, uint32_t* mt_done) {
    // mt_done (nullable): per m-tile count of gate/up epilogue warps whose activation rows are stored.
    // The gate/up grid lets the down grid launch at its start; a down CTA (on an SM a finished gate/up
    // CTA left) loads an m-tile's activation rows once all of its gate/up tiles are stored, so the
    // down GEMM fills the gate/up grid's last, partly empty wave.
    if (!DOWN && mt_done && threadIdx.x == 0) griddep_launch_dependents();
    if (n_items_dev) n_items = *n_items_dev;  // tile list built on the device (every CTA reads it)
    const uint32_t mt_full = (uint32_t)(F / 128) * kTcEpiWarps;  // counts of a finished m-tile
    extern __shared__ __align__(1024) unsigned char tsm[];
    unsigned char* ring = reinterpret_cast<unsigned char*>(((uintptr_t)tsm + 1023) & ~(uintptr_t)1023);
    TcCtrl& c = *reinterpret_cast<TcCtrl*>(ring + (size_t)kTcStages * kTcStage);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nk = (DOWN ? F : H) / kTcBK;
    if (threadIdx.x == 0) {
        for (int s = 0; s < kTcStages; s++) {
            mbar_init(&c.full[s], 1);
            mbar_init(&c.empty[s], 1);
        }
        mbar_init(&c.accum, 1);
        mbar_init(&c.tfree, kTcEpiWarps);
        mbar_init(&c.done, 1);
        for (int q = 0; q < 2; q++) {
            mbar_init(&c.tq_full[q], 1);
            mbar_init(&c.tq_empty[q], 1 + kTcEpiWarps);
        }
        c.abort = 0;
        fence_mbar_init();
    }
    if (warp == kTcMmaWarp) {  // whole warp: 512 columns = the accumulators of both halves
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&c.tmem)),
                     "r"(512));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::);
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = c.tmem;

    if (warp == kTcProdWarp) {
        if (lane == 0) {
            uint32_t g = 0;  // stages issued over all tiles
            bool ok = true;
            const uint64_t pol_w = l2_evict_first(), pol_a = l2_evict_last();  // weights read once; rows reused
            for (int n = 0; ok; n++) {
                const uint64_t deadline = globaltimer_ns() + timeout_ns;
                const int slot = n & 1;
                if (n >= 2 && !tc_wait(&c.tq_empty[slot], ((n >> 1) & 1) ^ 1, &c.abort, err, deadline)) break;
                const int i = (int)atomicAdd(&sched[0], 1u);  // dynamic tile schedule
                c.tq[slot] = i;
                mbar_arrive(&c.tq_full[slot]);  // release: the index is visible to the waiters
                if (i >= n_items) break;
                const TcItem it = items[i];
                const bool two = it.rows > 128;
                if (DOWN && mt_done) {  // the m-tile's activation rows are all stored (bounded wait)
                    const uint32_t* done = mt_done + i / (H / 256);
                    while (ld_acquire_gpu(done) < mt_full) {
                        if (*(volatile int*)&c.abort || globaltimer_ns() > deadline) {
                            if (!*(volatile int*)&c.abort) atomicOr(err, kErrTimeout);
                            *(volatile int*)&c.abort = 1;
                            ok = false;
                            break;
                        }
                        __nanosleep(64);
                    }
                    if (!ok) break;
                    fence_proxy_async_global();  // generic-proxy stores of other CTAs, before these TMA reads
                }
                for (int k = 0; k < nk; k++, g++) {
                    const int s = g % kTcStages;
                    if (g >= kTcStages &&
                        !tc_wait(&c.empty[s], ((g / kTcStages) & 1) ^ 1, &c.abort, err, deadline)) {
                        ok = false;
                        break;
                    }
                    unsigned char* st = ring + (size_t)s * kTcStage;
                    unsigned char* sb = st + 2 * kTcHalfA;
                    mbar_arrive_expect_tx(&c.full[s], (two ? 2 : 1) * kTcHalfA + kTcBBytes);
                    tma_load_2d(st, &map_a, k * kTcBK, it.row0, &c.full[s], pol_a);
                    if (two) tma_load_2d(st + kTcHalfA, &map_a, k * kTcBK, it.row0 + 128, &c.full[s], pol_a);
                    if (DOWN) {
#pragma unroll
                        for (int j = 0; j < 4; j++)
                            tma_load_3d(sb + j * (kTcBK * 128), &map_w, 2 * H + it.f0 + j * 64, k * kTcBK, it.slot,
                                        &c.full[s], pol_w);
                    } else {  // gate rows then up rows: one 256-row K-major operand
                        tma_load_3d(sb, &map_w, k * kTcBK, it.f0, it.slot, &c.full[s], pol_w);
                        tma_load_3d(sb + kTcBBytes / 2, &map_w, H + k * kTcBK, it.f0, it.slot, &c.full[s], pol_w);
                    }
                }
            }
            // every issued copy lands before the CTA may exit
            const uint64_t dd = globaltimer_ns() + timeout_ns;
            for (uint32_t q = g > (uint32_t)kTcStages ? g - kTcStages : 0; q < g; q++)
                while (!mbar_try_wait(&c.full[q % kTcStages], (q / kTcStages) & 1))
                    if (globaltimer_ns() > dd) break;
        }
    } else if (warp == kTcMmaWarp) {
        if (lane == 0) {
            const uint32_t idesc =
                DOWN ? (uint32_t)cute::UMMA::make_instr_desc<cute::bfloat16_t, cute::bfloat16_t, float, 128, 256,
                                                             cute::UMMA::Major::K, cute::UMMA::Major::MN>()
                     : (uint32_t)cute::UMMA::make_instr_desc<cute::bfloat16_t, cute::bfloat16_t, float, 128, 256,
                                                             cute::UMMA::Major::K, cute::UMMA::Major::K>();
            uint32_t g = 0;
            bool ok = true;
            for (int n = 0; ok; n++) {
                const uint64_t deadline = globaltimer_ns() + timeout_ns;
                const int slot = n & 1;
                if (!tc_wait(&c.tq_full[slot], (n >> 1) & 1, &c.abort, err, deadline)) break;
                const int i = *(volatile int*)&c.tq[slot];
                mbar_arrive(&c.tq_empty[slot]);
                if (i >= n_items) break;
                const bool two = items[i].rows > 128;
                if (n > 0 && !tc_wait(&c.tfree, (n - 1) & 1, &c.abort, err, deadline)) break;  // TMEM drained
                tc_fence_after();
                for (int k = 0; k < nk; k++, g++) {
                    const int s = g % kTcStages;
                    if (!tc_wait(&c.full[s], (g / kTcStages) & 1, &c.abort, err, deadline)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t sa = smem_u32(ring + (size_t)s * kTcStage), sb = sa + 2 * kTcHalfA;
#pragma unroll
                    for (int kk = 0; kk < kTcBK / 16; kk++) {
                        const uint32_t acc = (k | kk) != 0;
                        const uint64_t da0 = sw128_desc(sa + kk * 32), da1 = sw128_desc(sa + kTcHalfA + kk * 32);
                        // gate/up: columns [0, 128) gate, [128, 256) up of each half's accumulator
                        const uint64_t db = DOWN ? sw128_mn_desc(sb + kk * 2048) : sw128_desc(sb + kk * 32);
                        umma_bf16(tmem + 0, da0, db, idesc, acc);
                        if (two) umma_bf16(tmem + 256, da1, db, idesc, acc);
                    }
                    umma_commit(&c.empty[s]);  // the stage is free once these MMAs have read it
                }
                if (ok) umma_commit(&c.accum);  // this tile's accumulators are complete
            }
        }
    } else {
        // epilogue: warp w -> TMEM lanes [32 (w % 4), +32), half w / 4
        const int h = warp / 4, q = warp % 4;
        const int r = h * 128 + q * 32 + lane;  // row of the tile this thread writes
        const uint32_t taddr = tmem + ((uint32_t)(q * 32) << 16) + h * 256;
        for (int n = 0;; n++) {
            const uint64_t deadline = globaltimer_ns() + timeout_ns;
            const int slot = n & 1;
            if (!tc_wait(&c.tq_full[slot], (n >> 1) & 1, &c.abort, err, deadline)) break;
            const int i = *(volatile int*)&c.tq[slot];
            __syncwarp();
            if (lane == 0) mbar_arrive(&c.tq_empty[slot]);
            if (i >= n_items) break;
            const TcItem it = items[i];
            if (!tc_wait(&c.accum, n & 1, &c.abort, err, deadline)) break;
            tc_fence_after();
            if (h == 0 || it.rows > 128) {
                if (DOWN) {
                    float* y = static_cast<float*>(out);
                    for (int c0 = 0; c0 < 256; c0 += 32) {
                        uint32_t v[32];
                        tmem_ld32(taddr + c0, v);
                        tmem_wait_ld();
                        if (r < it.rows) {
                            float4* dst = reinterpret_cast<float4*>(y + (size_t)(it.row0 + r) * H + it.f0 + c0);
#pragma unroll
                            for (int e = 0; e < 8; e++)
                                dst[e] = make_float4(__uint_as_float(v[4 * e]), __uint_as_float(v[4 * e + 1]),
                                                     __uint_as_float(v[4 * e + 2]), __uint_as_float(v[4 * e + 3]));
                        }
                    }
                } else {
                    uint16_t* act = static_cast<uint16_t*>(out);
                    for (int c0 = 0; c0 < 128; c0 += 32) {
                        uint32_t g[32], u[32];
                        tmem_ld32(taddr + c0, g);
                        tmem_ld32(taddr + 128 + c0, u);
                        tmem_wait_ld();
                        if (r < it.rows) {
                            uint32_t o[16];
#pragma unroll
                            for (int e = 0; e < 16; e++)
                                o[e] = (uint32_t)swiglu_bf16(__uint_as_float(g[2 * e]), __uint_as_float(u[2 * e])) |
                                       ((uint32_t)swiglu_bf16(__uint_as_float(g[2 * e + 1]), __uint_as_float(u[2 * e + 1]))
                                        << 16);
                            uint4* dst = reinterpret_cast<uint4*>(act + (size_t)(it.row0 + r) * F + it.f0 + c0);
                            dst[0] = make_uint4(o[0], o[1], o[2], o[3]);
                            dst[1] = make_uint4(o[4], o[5], o[6], o[7]);
                            dst[2] = make_uint4(o[8], o[9], o[10], o[11]);
                            dst[3] = make_uint4(o[12], o[13], o[14], o[15]);
                        }
                    }
                }
            }
            tc_fence_before();
            if (!DOWN && mt_done) {  // this warp's activation rows of the tile are stored
                __threadfence();
                __syncwarp();
                if (lane == 0) atomicAdd(mt_done + i / (F / 128), 1u);
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&c.tfree);  // this warp's TMEM reads are complete
        }
    }
    // all MMAs are complete before TMEM is released: the last accum commit covers them; after an abort
    // the MMA thread commits once more and waits (bounded) for it
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
    // the last CTA out re-arms the schedule for the next launch (every tile index has been taken)
    if (threadIdx.x == 0 && atomicAdd(&sched[1], 1u) == gridDim.x - 1) {
        atomicExch(&sched[0], 0u);
        atomicExch(&sched[1], 0u);
    }
}

// ---- tile lists from the permutation's job list, on the device (no host round trip) ----
// Jobs heaviest first (stable), each job's 256-pair m-tiles in order, then the tile's n-blocks:
// gate/up items (f0 = first of 128 f) into gu, down items (f0 = first of 256 h) into dn.
// cnt[0] = gate/up items, cnt[1] = down items, cnt[2] = local pairs (rows of the gathered x).
__global__ void __launch_bounds__(256) tc_items_kernel(const Job* __restrict__ jobs, const int* __restrict__ n_jobs, int E,
                                                       const char* arena, size_t stride, int F, int H, TcItem* gu,
                                                       int cap_gu, TcItem* dn, int cap_dn, int* cnt, uint32_t* err,
                                                       uint32_t* mt_done) {
    __shared__ int n_s[kMaxExperts], order_s[kMaxExperts], off_s[kMaxExperts + 1];
    __shared__ int np_s;
    const int tid = threadIdx.x;
    const int nj = min(max(*n_jobs, 0), E);
    if (tid == 0) np_s = 0;
    for (int j = tid; j < nj; j += blockDim.x) n_s[j] = jobs[j].n;
    __syncthreads();
    for (int j = tid; j < nj; j += blockDim.x) {
        int r = 0;
        for (int i = 0; i < nj; i++) r += n_s[i] > n_s[j] || (n_s[i] == n_s[j] && i < j);
        order_s[r] = j;
        atomicMax(&np_s, jobs[j].p0 + n_s[j]);
    }
    __syncthreads();
    if (tid < 32) {  // exclusive scan of the m-tile counts in job order: one warp, 8 jobs per lane
        const int per = (nj + 31) / 32, r0 = tid * per;
        int sum = 0;
        for (int r = r0; r < r0 + per && r < nj; r++) sum += (n_s[order_s[r]] + 255) / 256;
        int inc = sum;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, inc, o);
            if (tid >= o) inc += y;
        }
        int acc = inc - sum;
        for (int r = r0; r < r0 + per && r < nj; r++) {
            off_s[r] = acc;
            acc += (n_s[order_s[r]] + 255) / 256;
        }
        if (tid == 31) off_s[nj] = inc;
    }
    __syncthreads();
    const int nf = F / 128, nh = H / 256, mt = off_s[nj];
    const bool fits = mt * nf <= cap_gu && mt * nh <= cap_dn;
    if (mt_done)
        for (int m = tid; m < mt; m += blockDim.x) mt_done[m] = 0;
    if (fits)
        for (int r = tid; r < nj; r += blockDim.x) {
            const Job jb = jobs[order_s[r]];
            const int slot = (int)(((const char*)jb.ex.w1 - arena) / (long)stride);
            for (int t = 0; t * 256 < jb.n; t++) {
                const int row0 = jb.p0 + t * 256, rows = min(256, jb.n - t * 256), m = off_s[r] + t;
                for (int f = 0; f < nf; f++) gu[(size_t)m * nf + f] = TcItem{row0, rows, slot, f * 128};
                for (int h = 0; h < nh; h++) dn[(size_t)m * nh + h] = TcItem{row0, rows, slot, h * 256};
            }
        }
    if (tid == 0) {
        if (!fits) atomicOr(err, kErrBadIndex);  // sized by the host for max_tokens: never expected
        cnt[0] = fits ? mt * nf : 0;
        cnt[1] = fits ? mt * nh : 0;
        cnt[2] = np_s;
    }
}

cudaError_t launch_tc_items(const Job* jobs, const int* n_jobs, int E, const void* arena, size_t stride, int F, int H,
                            TcItem* gu, int cap_gu, TcItem* dn, int cap_dn, int* cnt, uint32_t* err, uint32_t* mt_done,
                            cudaStream_t st) {
    if (E > kMaxExperts) return cudaErrorInvalidValue;
    tc_items_kernel<<<1, 256, 0, st>>>(jobs, n_jobs, E, static_cast<const char*>(arena), stride, F, H, gu, cap_gu, dn,
                                       cap_dn, cnt, err, mt_done);
    return cudaGetLastError();
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
    cudaError_t e = cudaFuncSetAttribute(tc_gemm_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kTcSmem);
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(tc_gemm_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kTcSmem);
    return e;
}

// [rows][cols] bf16, 128-row x 64-column boxes, 128-byte swizzle
static bool encode_rows(EncodeTiledFn enc, CUtensorMap* m, const void* base, int cols, int rows) {
    const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)cols * 2};
    const cuuint32_t box[2] = {kTcBK, 128}, es[2] = {1, 1};
    return enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, es,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// the layer's unit tables as [slot][f][3H] bf16 with the given box (inner, f)
static bool encode_units(EncodeTiledFn enc, CUtensorMap* m, const void* arena, int H, int F, int n_slots,
                         size_t slot_bytes, cuuint32_t box_x, cuuint32_t box_f) {
    const cuuint64_t dims[3] = {(cuuint64_t)3 * H, (cuuint64_t)F, (cuuint64_t)n_slots};
    const cuuint64_t strides[2] = {(cuuint64_t)6 * H, (cuuint64_t)slot_bytes};
    const cuuint32_t box[3] = {box_x, box_f, 1}, es[3] = {1, 1, 1};
    return enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(arena), dims, strides, box, es,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

cudaError_t launch_down_tc(const uint16_t* act, int arows, const void* arena, int n_slots, size_t slot_bytes,
                           const TcItem* items, int n_items, const int* n_items_dev, int H, int F, float* y,
                           uint32_t* sched, uint32_t* err, uint64_t timeout_ns, int grid_max, uint32_t* mt_done,
                           cudaStream_t st) {
    EncodeTiledFn enc = encode_fn();
    if (!enc) return cudaErrorNotSupported;
    if (H % 256 || F % kTcBK || slot_bytes % 16 || ((uintptr_t)act | (uintptr_t)arena) & 15) return cudaErrorInvalidValue;
    CUtensorMap ma, md;
    // activation rows [arows][F]; down columns at element 2H of each unit, boxes of 64 outputs x 64 f
    if (!encode_rows(enc, &ma, act, F, arows) || !encode_units(enc, &md, arena, H, F, n_slots, slot_bytes, 64, kTcBK))
        return cudaErrorInvalidValue;
    if (!n_items_dev && n_items <= 0) return cudaSuccess;
    const int grid = n_items_dev ? grid_max : std::min(n_items, grid_max);
    if (!mt_done) {
        tc_gemm_kernel<true><<<grid, kTcThreads, kTcSmem, st>>>(ma, md, items, n_items, n_items_dev, H, F, y, sched,
                                                               err, timeout_ns, nullptr);
        return cudaGetLastError();
    }
    // programmatic dependent launch behind the gate/up grid (which triggers at its start): the CTAs
    // take the SMs its finished CTAs leave and wait per m-tile for its activation rows
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kTcThreads);
    cfg.dynamicSmemBytes = kTcSmem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, tc_gemm_kernel<true>, ma, md, items, n_items, n_items_dev, H, F, (void*)y, sched,
                              err, timeout_ns, mt_done);
}

cudaError_t launch_gateup_tc(const uint16_t* xg, int xrows, const void* arena, int n_slots, size_t slot_bytes,
                             const TcItem* items, int n_items, const int* n_items_dev, int H, int F, uint16_t* act,
                             uint32_t* sched, uint32_t* err, uint64_t timeout_ns, int grid_max, uint32_t* mt_done,
                             cudaStream_t st) {
    EncodeTiledFn enc = encode_fn();
    if (!enc) return cudaErrorNotSupported;
    if (H % kTcBK || F % 128 || slot_bytes % 16 || ((uintptr_t)xg | (uintptr_t)arena) & 15) return cudaErrorInvalidValue;
    CUtensorMap mx, mw;
    // gathered token rows [xrows][H]; gate row f at element 0 of unit f, up row at element H
    if (!encode_rows(enc, &mx, xg, H, xrows) || !encode_units(enc, &mw, arena, H, F, n_slots, slot_bytes, kTcBK, 128))
        return cudaErrorInvalidValue;
    if (!n_items_dev && n_items <= 0) return cudaSuccess;
    const int grid = n_items_dev ? grid_max : std::min(n_items, grid_max);
    tc_gemm_kernel<false><<<grid, kTcThreads, kTcSmem, st>>>(mx, mw, items, n_items, n_items_dev, H, F, act, sched, err,
                                                            timeout_ns, mt_done);
    return cudaGetLastError();
}

}  // namespace moe
