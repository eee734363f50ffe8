// moe_ck_moe3_noalloc: the ck_moe3 surface with no allocation at all.
//
// Who needs it: callers that own every byte of device memory themselves and may not call
// cudaMalloc -- an inference server whose allocator has already carved HBM into expert tables and
// KV cache, a framework that forbids side allocations outside its pool, or code that runs where an
// allocation would block or fail.  Such a caller cannot create a moe_ctx (creation allocates the
// context's tables and scratch), so this entry point takes only its inputs and outputs and keeps
// its working memory in the library's own file-scope device array below.
//
// Limits and sharing rules (also stated at the declaration in include/moe_dp.h):
//   * the array is kNoAllocScratchBytes (1 MiB) per GPU and lives until the process exits;
//   * at most kNoAllocMaxExperts (16) experts per call, and E * (2F + 4H) + 4 KiB bytes of scratch;
//   * every call on a device uses the same array, so calls that overlap on the GPU race: order them
//     on one stream (or synchronise between them);
//   * the first call on a device looks up the array's device address (cudaGetSymbolAddress) and
//     should therefore come before any stream capture.
#include <cuda_runtime.h>

#include <cstring>
#include <mutex>

#include "../../include/moe_dp.h"
#include "common.cuh"
#include "experts.h"

namespace moe {
int internal_fail(int code, const char* msg);
}

using namespace moe;

namespace {

constexpr size_t kNoAllocScratchBytes = 1u << 20;
constexpr int kNoAllocMaxExperts = 16;
constexpr int kMaxDevices = 64;

// The call's working memory: job table, pair lists, SwiGLU activations and per-expert outputs.
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

// Per device: the array's device address and the SM count (looked up once, with that device current).
void* g_scratch_addr[kMaxDevices] = {};
int g_sm_count[kMaxDevices] = {};
std::mutex g_scratch_mu;

// Scratch layout inside g_noalloc_scratch (offsets in bytes, each 256-aligned).
struct Layout {
    size_t jobs, ptok, pw, comb_off, comb_p, act, y, end;
};

size_t up256(size_t v) { return (v + 255) / 256 * 256; }

Layout layout(int E, int H, int F) {
    Layout L{};
    size_t o = 0;
    L.jobs = o; o = up256(o + sizeof(Job) * E);
    L.ptok = o; o = up256(o + 4 * E);
    L.pw = o; o = up256(o + 4 * E);
    L.comb_off = o; o = up256(o + 8);
    L.comb_p = o; o = up256(o + 4 * E);
    L.act = o; o = up256(o + (size_t)E * F * 2);
    L.y = o; o = up256(o + (size_t)E * H * 4);
    L.end = o;
    return L;
}

// The expert list travels by value in the launch parameters (no host->device copy needed).
struct NoAllocTable {
    const uint16_t* base[kNoAllocMaxExperts];
    int E;
    int H;
    int F;
};

// Writes the job table, the single-token pair lists and the routing weights into the scratch.
__global__ void noalloc_setup_kernel(NoAllocTable t, const float* w, unsigned char* scratch, Layout L) {
    const int e = threadIdx.x;
    const size_t FH = (size_t)t.F * t.H;
    Job* jobs = reinterpret_cast<Job*>(scratch + L.jobs);
    int32_t* ptok = reinterpret_cast<int32_t*>(scratch + L.ptok);
    float* pw = reinterpret_cast<float*>(scratch + L.pw);
    int32_t* comb_off = reinterpret_cast<int32_t*>(scratch + L.comb_off);
    int32_t* comb_p = reinterpret_cast<int32_t*>(scratch + L.comb_p);
    if (e < t.E) {
        jobs[e] = Job{ExpDesc{t.base[e], t.base[e] + 2 * FH, nullptr, kKindBF16, 0}, e, 1};
        ptok[e] = 0;
        pw[e] = w[e];
        comb_p[e] = e;
    }
    if (e == 0) {
        comb_off[0] = 0;
        comb_off[1] = t.E;
    }
}

// The calling thread's current device, the scratch array's address on it and its SM count.
int scratch_address(void** out, int* sms) {
    int dev = -1;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
        cudaGetLastError();
        return internal_fail(MOE_ECUDA, "moe_ck_moe3_noalloc: no usable current CUDA device");
    }
    std::lock_guard<std::mutex> lk(g_scratch_mu);
    if (!g_scratch_addr[dev]) {
        void* p = nullptr;
        int n = 0;
        e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess || !p) {
            cudaGetLastError();
            return internal_fail(MOE_ECUDA, "moe_ck_moe3_noalloc: cudaGetSymbolAddress of the scratch array failed");
        }
        e = cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        if (e != cudaSuccess || n <= 0) {
            cudaGetLastError();
            return internal_fail(MOE_ECUDA, "moe_ck_moe3_noalloc: SM count query failed");
        }
        g_sm_count[dev] = n;
        g_scratch_addr[dev] = p;
    }
    *out = g_scratch_addr[dev];
    *sms = g_sm_count[dev];
    return MOE_OK;
}

}  // namespace

extern "C" int moe_ck_moe3_noalloc(int E, const uint16_t* const* base, const float* w, const uint16_t* x, float* out,
                                   int H, int F, void* stream) {
    if (E <= 0) return MOE_OK;  // like ck_moe3 (cpu_kern.c:142): no experts, nothing to add
    if (E > kNoAllocMaxExperts)
        return internal_fail(MOE_EINVAL, "moe_ck_moe3_noalloc: E exceeds the 16-expert limit of the static scratch");
    if (!base || !w || !x || !out) return internal_fail(MOE_EINVAL, "moe_ck_moe3_noalloc: null argument");
    if (H <= 0 || H % 64 != 0 || H > 16384 || F <= 0 || F % 64 != 0 || F > 2048)
        return internal_fail(MOE_EINVAL, "moe_ck_moe3_noalloc: H must be a multiple of 64 <= 16384 and F a multiple "
                                         "of 64 <= 2048");
    const Layout L = layout(E, H, F);
    if (L.end > kNoAllocScratchBytes)
        return internal_fail(MOE_EINVAL, "moe_ck_moe3_noalloc: E * (2F + 4H) bytes exceed the 1 MiB static scratch");
    if (((uintptr_t)x | (uintptr_t)out) & 15u)
        return internal_fail(MOE_EINVAL, "moe_ck_moe3_noalloc: x/out must be 16-byte aligned");
    NoAllocTable t{};
    t.E = E;
    t.H = H;
    t.F = F;
    for (int e = 0; e < E; e++) {
        if (!base[e] || ((uintptr_t)base[e] & 15u))
            return internal_fail(MOE_EINVAL, "moe_ck_moe3_noalloc: base pointers must be non-null and 16-byte aligned");
        t.base[e] = base[e];
    }
    void* sp = nullptr;
    int sms = 0;
    int st = scratch_address(&sp, &sms);
    if (st != MOE_OK) return st;
    unsigned char* s = static_cast<unsigned char*>(sp);
    cudaStream_t cs = static_cast<cudaStream_t>(stream);
    noalloc_setup_kernel<<<1, 32, 0, cs>>>(t, w, s, L);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return internal_fail(MOE_ECUDA, cudaGetErrorString(e));
    ExpertArgs a{};
    a.x = x;
    a.T = 1;
    a.H = H;
    a.F = F;
    a.jobs = reinterpret_cast<const Job*>(s + L.jobs);
    a.n_jobs = nullptr;
    a.n_jobs_host = E;
    a.n_jobs_max = E;
    a.max_pairs = 1;
    a.ptok = reinterpret_cast<const int32_t*>(s + L.ptok);
    a.pw = reinterpret_cast<const float*>(s + L.pw);
    a.act = reinterpret_cast<uint16_t*>(s + L.act);
    a.y = reinterpret_cast<float*>(s + L.y);
    a.comb_off = reinterpret_cast<const int32_t*>(s + L.comb_off);
    a.comb_p = reinterpret_cast<const int32_t*>(s + L.comb_p);
    a.out = out;
    a.accumulate = 1;
    a.err = nullptr;
    int launches = 0;
    e = launch_experts(a, sms, cs, &launches, nullptr);
    if (e != cudaSuccess) return internal_fail(MOE_ECUDA, cudaGetErrorString(e));
    return MOE_OK;
}
