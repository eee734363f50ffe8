// libmoe_dp: context, expert tables and the C ABI declared in include/moe_dp.h.
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <string>
#include <vector>

#include "../../include/moe_dp.h"
#include "common.cuh"
#include "decode.h"
#include "prefill_tc.h"
#include "block.h"
#include "experts.h"
#include "route.h"

using namespace moe;

static constexpr int kProfMarks = 5;  // before route, after route, after each of the 3 expert kernels

namespace {

thread_local std::string g_err;

int fail(int code, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    g_err = buf;
    return code;
}

#define CUDA_TRY(expr)                                                                              \
    do {                                                                                            \
        cudaError_t e_ = (expr);                                                                    \
        if (e_ != cudaSuccess) return fail(MOE_ECUDA, "%s: %s", #expr, cudaGetErrorString(e_));     \
    } while (0)

size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

// Restores the caller's current device on scope exit.
struct DeviceGuard {
    int prev = -1;
    explicit DeviceGuard(int dev) {
        cudaGetDevice(&prev);
        if (prev != dev) cudaSetDevice(dev);
    }
    ~DeviceGuard() {
        int cur;
        cudaGetDevice(&cur);
        if (prev >= 0 && cur != prev) cudaSetDevice(prev);
    }
};

// Pinned host staging buffer guarded by an event (reuse waits for the previous copy).
struct Staging {
    void* host = nullptr;
    size_t cap = 0;
    cudaEvent_t ev = nullptr;
    bool pending = false;
    int reserve(size_t bytes) {
        if (pending) {
            cudaEventSynchronize(ev);
            pending = false;
        }
        if (bytes <= cap) return MOE_OK;
        if (host) cudaFreeHost(host);
        host = nullptr;
        cap = 0;
        size_t n = align_up(std::max<size_t>(bytes, 1 << 16), 1 << 16);
        if (cudaMallocHost(&host, n) != cudaSuccess) return fail(MOE_ENOMEM, "pinned staging of %zu bytes", n);
        cap = n;
        return MOE_OK;
    }
    void mark(cudaStream_t st) {
        cudaEventRecord(ev, st);
        pending = true;
    }
};

}  // namespace

namespace moe {
// Error reporting for entry points defined in other translation units of the library.
int internal_fail(int code, const char* msg) { return fail(code, "%s", msg); }
}  // namespace moe

struct moe_ctx {
    moe_config cfg{};
    int dev = 0;
    int sm_count = 148;
    std::vector<int32_t> owner;           // [L*E] owning rank
    std::vector<int32_t> slot;            // [L*E] local slot, -1 if remote
    std::vector<int32_t> n_local;         // [L]
    std::vector<int32_t> res;             // [L*E] arena slot of a resident local expert, -1 if not resident
    std::vector<int32_t> arena_slots;     // [L] slots of each layer's arena
    int slot_budget = 0;                  // MOE_OPT_LAYER_SLOTS: slots per layer (0: every local expert)
    void* d_down_stage = nullptr;         // [F*H] bf16: host down matrices on their way to the unit tables
    std::vector<void*> arena;             // [L] lazily allocated expert storage
    size_t stride = 0;                    // bytes per expert slot
    std::vector<ExpDesc> h_desc;          // [L*E]
    ExpDesc* d_desc = nullptr;            // [L*E]
    float* d_bias = nullptr;              // [L*E]
    std::vector<char> has_bias;           // [L]
    // routing / pipeline scratch, sized by max_tokens
    int32_t *d_idx = nullptr, *d_counts = nullptr, *d_offsets = nullptr, *d_perm = nullptr, *d_jobord = nullptr;
    int32_t *d_nj = nullptr, *d_nlj = nullptr, *d_ptok = nullptr, *d_pairpos = nullptr, *d_comb_off = nullptr;
    int32_t* d_comb_p = nullptr;
    int32_t* d_route_scratch = nullptr;  // permutation scratch (route_scratch_ints(max_tokens, E))
    float *d_w = nullptr, *d_pw = nullptr;
    Job* d_jobs = nullptr;
    uint16_t* d_act = nullptr;
    float* d_y = nullptr;
    uint32_t* d_err = nullptr;
    uint32_t* h_err = nullptr;  // pinned
    uint32_t* h_errsnap = nullptr;  // pinned, written by the decode kernel on host-buffer calls
    // MOE_F_HOST staging
    uint16_t* d_hidden = nullptr;
    float* d_logits = nullptr;
    float* d_out = nullptr;
    Staging in_stage, out_stage, job_stage;
    int64_t launches = 0;
    uint32_t latched = 0;
    // fused decode kernel state
    unsigned long long* d_decide = nullptr;  // [4] fused decode: per-call share-cut decisions (call mod 4)
    unsigned long long* d_cnt = nullptr;  // [4] fused decode calls: arrived (even calls), finished, past their
                                          //   partial-sum reads, arrived (odd calls)
    float* d_part = nullptr;    // fused decode partial sums: two buffers, used by alternate calls
    // expert-parallel exchange over NVLink peer memory (moe_ep_export / moe_ep_import)
    uint64_t* d_xbuf = nullptr;         // [2][world][ep_tcap][H] words {epoch, fp32}: this rank's receive buffer
    int ep_tcap = kEpMaxT;              // tokens per (parity, rank) slot of the exchange buffers
    uint64_t** d_peer_x = nullptr;      // [kEpMaxWorld] device copy of every rank's buffer pointer
    float* d_xpart = nullptr;           // multi-kernel path: this rank's partial before the exchange
    std::vector<void*> ipc_opened;      // peer mappings to close
    bool ep_attached = false;
    uint32_t xepoch = 0;
    // prefill: grouped GEMMs on the tcgen05 tensor cores between the gather and the combine
    bool prefill = true;
    int prefill_min_t = 10;             // smallest batch that takes the tensor-core path (measured crossover)
    uint16_t* d_pf_x = nullptr;         // [NP, H] gathered token rows (job-major pairs)
    float* d_pf_yf = nullptr;           // [NP, H] down . act (fp32)
    bool prefill_tc = true;             // prefill batches on the tcgen05 kernels; else the CUDA-core path
    TcItem* d_tc_items = nullptr;       // tile lists of the tcgen05 kernels (gate/up, then down)
    int* d_tc_cnt = nullptr;            // [4] device-built counts: gate/up items, down items, local pairs
    uint32_t* d_tc_mtdone = nullptr;    // per m-tile: gate/up epilogue warps done (the down GEMM starts early)
    uint32_t* d_tc_sched = nullptr;     // [4] tile-schedule counters (gate/up, down), left zero by each launch
    // MoE-block calls (moe_load_shared, moe_shared_router, moe_block_forward)
    moe_ctx* shared = nullptr;          // one-expert context holding each layer's shared expert
    int shared_inter = 0;               // its intermediate size (MOE_OPT_SHARED_INTER; 0 = cfg.inter)
    std::vector<uint16_t*> d_router;    // [L] router weights [E, H] bf16 (null until loaded)
    float* d_blk_zero = nullptr;        // [max_tokens] zero logits: the shared context routes with weight 1
    float* d_blk_logits = nullptr;      // [max_tokens, E]
    float* d_blk_shared = nullptr;      // [max_tokens, H] shared-expert output
    float* d_blk_moe = nullptr;         // [max_tokens, H] routed-expert output
    uint16_t* d_blk_y = nullptr;        // [max_tokens, H] y = bf16(x2 + shared)
    uint16_t* d_blk_io = nullptr;       // [3][max_tokens, H] host-buffer calls: h2, x2, x_next
    float* d_blk_extra = nullptr;       // [max_tokens, H] host-buffer calls: extra
    uint32_t* d_hctr = nullptr;     // [2] host calls: [0] CTAs whose slice of the inputs is on the device,
                                    //   counted over the context's host calls
    uint32_t hcalls = 0;            // host fused calls launched since the count was last cleared
    PubPlan* d_pub = nullptr;       // [4] plans published by the planner kernel (call number mod 4)
    uint32_t* d_pub_flag = nullptr; // [4] their stamps
    uint32_t epoch = 0;
    bool fused = true;
    uint64_t timeout_ns = 1000000000ull;
    int inject_timeout = 0;
    uint64_t* d_timeline = nullptr;  // [sm_count][kTimelineSlots] when MOE_OPT_TIMELINE is on
    int ns_cap = 0;
    uint32_t stage_target = 0;  // fused kernel bytes per ring stage (0: default)
    int q8_cost_pm = 0;         // planning cost of an int8 unit, per mille of its bytes (0: default)
    int reducers = kReducersDefault;     // fused decode: CTAs that reduce (0: all)
    bool use_planner = kPlannerDefault;  // fused decode: a planner kernel per device-buffer call
    long long late_bytes = kLateBytesDefault;  // fused decode: share reduction of the late CTAs
    // per-stage event timing of moe_forward (moe_profile / moe_profile_read)
    bool prof_on = false;
    std::vector<cudaEvent_t> prof_ev;  // kProfMarks events per profiled call
    cudaEvent_t dec_ev = nullptr;      // recorded after every fused decode launch (is the last call still running?)
    bool dec_ev_used = false;
    size_t prof_calls = 0;
};

namespace {

bool is_pinned_host(const void* p) {
    cudaPointerAttributes at;
    if (cudaPointerGetAttributes(&at, p) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    return at.type == cudaMemoryTypeHost;
}

// True when p is page-locked host memory that device code can address through p itself (unified
// addressing maps cudaMallocHost / cudaHostAlloc memory at the same address).
bool device_mapped(const void* p) {
    cudaPointerAttributes at;
    if (cudaPointerGetAttributes(&at, p) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    return at.type == cudaMemoryTypeHost && at.devicePointer == p;
}

int map_err(uint32_t bits) {
    if (bits & kErrTimeout) return fail(MOE_ETIMEOUT, "device-side bounded wait gave up");
    if (bits & kErrNonFinite) return fail(MOE_ENONFINITE, "router logits produced a NaN probability (NaN/+inf logit or all -inf)");
    if (bits & kErrBadExpert) return fail(MOE_ESTATE, "a routed expert is not loaded on this context");
    if (bits & kErrBadIndex) return fail(MOE_EINVAL, "corrupted expert index");
    return MOE_OK;
}

// Reads and clears the device error word (the stream must be synchronised by the caller after).
void queue_err_readback(moe_ctx* c, cudaStream_t st) {
    cudaMemcpyAsync(c->h_err, c->d_err, sizeof(uint32_t), cudaMemcpyDeviceToHost, st);
    cudaMemsetAsync(c->d_err, 0, sizeof(uint32_t), st);
}

// After a fused call gave up, its counts fall short: every call so far counts as finished.
int reset_counters(moe_ctx* c) {
    const unsigned long long G = (unsigned long long)(c->sm_count - 1), e = c->epoch;
    const unsigned long long v = e * G;
    const unsigned long long h[4] = {(e + 1) / 2 * G, v, v, e / 2 * G};  // even calls so far, all, all, odd calls
    CUDA_TRY(cudaMemcpy(c->d_cnt, h, sizeof(h), cudaMemcpyHostToDevice));
    CUDA_TRY(cudaMemset(c->d_hctr, 0, 2 * sizeof(uint32_t)));
    c->hcalls = 0;
    return MOE_OK;
}

int finish_sync(moe_ctx* c, cudaStream_t st) {
    queue_err_readback(c, st);
    CUDA_TRY(cudaStreamSynchronize(st));
    uint32_t bits = *c->h_err | c->latched;
    c->latched = 0;
    // a fused call that gave up may leave its grid-arrival counter short of the grid: clear both
    if ((bits & kErrTimeout) && c->d_cnt) {
        int r = reset_counters(c);
        if (r) return r;
    }
    return map_err(bits);
}

template <class T>
int dalloc(T** p, size_t n) {
    if (cudaMalloc((void**)p, std::max<size_t>(n, 1) * sizeof(T)) != cudaSuccess) {
        cudaGetLastError();
        return fail(MOE_ENOMEM, "cudaMalloc of %zu bytes", n * sizeof(T));
    }
    return MOE_OK;
}

int check_layer_expert(moe_ctx* c, int layer, int expert) {
    if (!c) return fail(MOE_EINVAL, "null context");
    if (layer < 0 || layer >= c->cfg.n_layers) return fail(MOE_EINVAL, "layer %d out of range [0,%d)", layer, c->cfg.n_layers);
    if (expert < 0 || expert >= c->cfg.n_experts)
        return fail(MOE_EINVAL, "expert %d out of range [0,%d)", expert, c->cfg.n_experts);
    if (c->slot[(size_t)layer * c->cfg.n_experts + expert] < 0)
        return fail(MOE_ESTATE, "expert (%d,%d) is owned by rank %d, not this rank %d", layer, expert,
                    c->owner[(size_t)layer * c->cfg.n_experts + expert], c->cfg.ep_rank);
    return MOE_OK;
}

int ensure_arena(moe_ctx* c, int layer) {
    if (c->arena[layer]) return MOE_OK;
    int n = std::max(1, c->n_local[layer]);
    if (c->slot_budget > 0 && c->slot_budget < n) {  // fewer slots than experts: residency set at load
        n = c->slot_budget;
        const int E = c->cfg.n_experts;
        for (int e = 0; e < E; e++) c->res[(size_t)layer * E + e] = -1;
    }
    c->arena_slots[layer] = n;
    size_t bytes = c->stride * (size_t)n;
    if (cudaMalloc(&c->arena[layer], bytes) != cudaSuccess) {
        cudaGetLastError();
        return fail(MOE_ENOMEM, "expert table of layer %d (%zu bytes)", layer, bytes);
    }
    return MOE_OK;
}

char* slot_ptr(moe_ctx* c, int layer, int expert) {
    return (char*)c->arena[layer] + c->stride * (size_t)c->res[(size_t)layer * c->cfg.n_experts + expert];
}

// Gives a local expert an arena slot for loading: its own if resident, else a free one.
int acquire_slot(moe_ctx* c, int layer, int expert) {
    const int E = c->cfg.n_experts;
    int32_t* r = &c->res[(size_t)layer * E];
    if (r[expert] >= 0) return MOE_OK;
    std::vector<char> used(c->arena_slots[layer], 0);
    for (int e = 0; e < E; e++)
        if (r[e] >= 0) used[r[e]] = 1;
    for (int s = 0; s < c->arena_slots[layer]; s++)
        if (!used[s]) {
            r[expert] = s;
            return MOE_OK;
        }
    return fail(MOE_ESTATE, "layer %d: all %d expert slots are in use; evict an expert first", layer,
                c->arena_slots[layer]);
}

int upload_desc(moe_ctx* c, int layer, int expert, const ExpDesc& d) {
    size_t i = (size_t)layer * c->cfg.n_experts + expert;
    c->h_desc[i] = d;
    CUDA_TRY(cudaMemcpy(c->d_desc + i, &d, sizeof(ExpDesc), cudaMemcpyHostToDevice));
    return MOE_OK;
}

// int8 unit tables: F units of 3H + 16 bytes, then the [2F + H] fp32 scales.
size_t q8_scale_off(const moe_ctx* c) {
    return align_up((size_t)c->cfg.inter * unit_pitch(kKindQ8, c->cfg.hidden), 256);
}

// Scatters a row-major [H, F] down matrix (device or host memory) into the down columns of the
// unit table at dst (pitch in elements of esize bytes).  Host sources go through a temporary
// device buffer.
int load_down_columns(moe_ctx* c, void* dst, const void* src, size_t pitch, int esize, bool host) {
    const size_t H = c->cfg.hidden, F = c->cfg.inter, bytes = F * H * esize;
    if (host) {  // staged in a context buffer kept for later loads (expert swaps reload often)
        if (!c->d_down_stage) {
            if (cudaMalloc(&c->d_down_stage, F * H * 2) != cudaSuccess) {
                cudaGetLastError();
                c->d_down_stage = nullptr;
                return fail(MOE_ENOMEM, "down-matrix staging (%zu bytes)", F * H * 2);
            }
        }
        cudaError_t e = cudaMemcpyAsync(c->d_down_stage, src, bytes, cudaMemcpyHostToDevice, 0);
        if (e != cudaSuccess) return fail(MOE_ECUDA, "down-matrix copy: %s", cudaGetErrorString(e));
        src = c->d_down_stage;
    }
    int n = 0;
    cudaError_t e = launch_scatter_down(src, dst, pitch, (int)H, (int)F, esize, 0, &n);
    c->launches += n;
    if (e == cudaSuccess) e = cudaStreamSynchronize(0);
    if (e != cudaSuccess) return fail(MOE_ECUDA, "down-matrix scatter: %s", cudaGetErrorString(e));
    return MOE_OK;
}

// Copies n bytes into device memory dst from src (host when host != 0).
int copy_in(void* dst, const void* src, size_t n, bool host, cudaStream_t st) {
    CUDA_TRY(cudaMemcpyAsync(dst, src, n, host ? cudaMemcpyHostToDevice : cudaMemcpyDeviceToDevice, st));
    return MOE_OK;
}

// The exchange arguments of one call (next epoch); world = 0 when no peers are attached.
EpExchange next_ep(moe_ctx* c) {
    EpExchange ep{};
    if (!c->ep_attached) return ep;
    ep.peer_x = c->d_peer_x;
    ep.x_local = c->d_xbuf;
    ep.rank = c->cfg.ep_rank;
    ep.world = c->cfg.ep_world;
    ep.epoch = ++c->xepoch;
    ep.tstride = c->ep_tcap;
    return ep;
}

// Fills the fused-path arguments that do not depend on the call's buffers; false when the call does
// not fit the fused path (then the multi-kernel path runs).
bool prepare_fused(moe_ctx* c, int T, int flags, DecodeArgs& da, size_t* dsmem) {
    const int dgrid = c->sm_count - 1;  // one persistent CTA per SM; one SM for the next call's planner
    if (T <= 0 || !c->fused || dgrid < 1) return false;
    da = DecodeArgs{};
    da.part = c->d_part;
    da.cnt = c->d_cnt;
    da.decide = c->d_decide;
    da.err = c->d_err;
    da.T = T;
    da.E = c->cfg.n_experts;
    da.K = c->cfg.top_k;
    da.H = c->cfg.hidden;
    da.F = c->cfg.inter;
    da.scoring = c->cfg.scoring;
    da.accumulate = (flags & MOE_F_ACCUMULATE) ? 1 : 0;
    da.timeout_ns = c->timeout_ns;
    da.inject_timeout = c->inject_timeout;
    da.timeline = c->d_timeline;
    da.stage_log = c->d_timeline ? reinterpret_cast<uint64_t*>(c->d_timeline + (size_t)c->sm_count * kTimelineSlots) : nullptr;
    da.ns_cap = c->ns_cap;
    da.stage_target = c->stage_target;
    da.q8_cost = c->q8_cost_pm ? (int)(unit_bytes(kKindQ8, da.H) * (size_t)c->q8_cost_pm / 1000) : 0;
    da.nred = c->reducers;
    da.late_cost = c->late_bytes;
    return plan_decode(da, dgrid, dsmem);
}

// Launches the fused decode kernel for one layer (da prepared by prepare_fused, x / out set).  Host
// calls pass the pinned sources: the kernel copies them to da.x and the context's logits buffer.
int launch_fused(moe_ctx* c, int layer, const float* lg, DecodeArgs& da, size_t dsmem, cudaStream_t st,
                 cudaEvent_t* marks, const uint16_t* x_host = nullptr, const ExpDesc* shared = nullptr,
                 bool planner = true) {
    const int E = c->cfg.n_experts, dgrid = c->sm_count - 1;
    da.ep = next_ep(c);
    da.epoch = c->epoch++;
    da.part = c->d_part + (size_t)(da.epoch & 1) * decode_part_floats(c->cfg.hidden, c->sm_count);
    da.bias = c->has_bias[layer] ? c->d_bias + (size_t)layer * E : nullptr;
    da.desc = c->d_desc + (size_t)layer * E;
    da.shared = shared;
    da.idx_out = c->d_idx;
    da.w_out = c->d_w;
    da.hctr = c->d_hctr;
    if (x_host) {
        da.hidx = c->hcalls;
        da.hbase = c->hcalls++ * (uint32_t)dgrid;
        da.x_src = x_host;
        da.lg_src = lg;
        da.logits = c->d_logits;
    } else {
        da.x_src = nullptr;
        da.lg_src = nullptr;
        da.logits = lg;
    }
    da.pub = nullptr;
    da.pub_flag = nullptr;
    da.stamp = da.epoch + 1;
    cudaError_t e = cudaSuccess;
    // A planner kernel publishes the call's plan only when the previous fused call is still running:
    // then it plans while that call streams.  A call made alone plans faster in its own CTAs (the
    // planner's few global round trips are on the critical path either way).
    bool in_flight = false;
    if (!x_host && planner && c->use_planner && c->dec_ev_used) {
        const cudaError_t q = cudaEventQuery(c->dec_ev);
        in_flight = q == cudaErrorNotReady;
        if (q != cudaSuccess) cudaGetLastError();  // not-ready is not an error of this call
    }
    if (in_flight) {
        PubPlan* pub = reinterpret_cast<PubPlan*>(reinterpret_cast<char*>(c->d_pub) + (da.epoch & 3) * pub_plan_bytes());
        uint32_t* flag = c->d_pub_flag + (da.epoch & 3);
        e = launch_planner(da, dgrid, pub, flag, da.stamp, st);
        if (e != cudaSuccess) return fail(MOE_ECUDA, "planner launch: %s", cudaGetErrorString(e));
        c->launches += 1;
        da.pub = pub;
        da.pub_flag = flag;
    }
    if (marks) cudaEventRecord(marks[1], st);
    e = launch_decode(da, dgrid, dsmem, st);
    c->launches += 1;
    if (e != cudaSuccess) return fail(MOE_ECUDA, "decode launch: %s", cudaGetErrorString(e));
    if (c->use_planner) {  // the next call asks whether this one still runs
        if (cudaEventRecord(c->dec_ev, st) == cudaSuccess) c->dec_ev_used = true;
        else cudaGetLastError();
    }
    if (marks)
        for (int i = 2; i < kProfMarks; i++) cudaEventRecord(marks[i], st);
    return MOE_OK;
}

// True when the grouped tensor-core GEMMs take a T-token call of this layer: batches of at least
// prefill_min_t tokens, every local expert of the layer bf16, a supported shape.  They read each
// routed expert once, while the fused decode kernel streams an expert once per token group of at
// most 4 tokens; the default threshold, 10, is the measured crossover on B200 (Solar layer: fused
// faster at 8 tokens, 171.6 against 185.6 us; tensor cores faster at 10, 204.3 against 214.4 us).
bool prefill_applies(moe_ctx* c, int layer, int T) {
    const int H = c->cfg.hidden, F = c->cfg.inter, E = c->cfg.n_experts;
    if (!c->prefill || !c->prefill_tc || T < c->prefill_min_t || !tc_available() || F % 128 || H % 256 || E > kMaxExperts)
        return false;
    for (int e = 0; e < E; e++)
        if (c->h_desc[(size_t)layer * E + e].kind == kKindQ8) return false;
    return true;
}

// Prefill: after the router has grouped the pairs (d_jobs, d_ptok, d_pw, combine lists), the expert
// FFN runs as two grouped GEMMs on the tcgen05 tensor cores over the context's unit tables, read in
// place (fp32 accumulation; g, u and y kept in fp32 like the decode paths):
//   gate/up  tiles of 256 pairs x 128 f: act = SwiGLU(gate . x, up . x) fused in the epilogue
//   down     tiles of 256 pairs x 256 h: y = down . act, the down columns as an MN-major operand
// Sets *done when it ran (every local job bf16, shape supported); the caller runs the CUDA-core path
// otherwise.
int run_prefill(moe_ctx* c, int layer, int T, const uint16_t* x, float* o, int accumulate, cudaStream_t st, bool* done) {
    *done = false;
    const int H = c->cfg.hidden, F = c->cfg.inter, E = c->cfg.n_experts;
    const size_t NP = (size_t)c->cfg.max_tokens * c->cfg.top_k;
    const bool tc = c->prefill_tc && tc_available() && F % 128 == 0 && H % 256 == 0 && E <= kMaxExperts;
    if (tc) {  // tile lists built on the device from the permutation's job list: no host round trip
        for (int e = 0; e < E; e++)
            if (c->h_desc[(size_t)layer * E + e].kind == kKindQ8) return MOE_OK;  // int8 tables: CUDA cores
        const int mt_max = (int)(NP / 256) + E;  // 256-pair tiles: every job adds at most one partial tile
        const int cap_gu = mt_max * (F / 128), cap_dn = mt_max * (H / 256);
        if (!c->d_pf_x) {
            int st2 = dalloc(&c->d_pf_x, NP * H);
            if (!st2) st2 = dalloc(&c->d_pf_yf, NP * H);
            if (!st2) st2 = dalloc(&c->d_tc_sched, 4);
            if (!st2 && cudaMemset(c->d_tc_sched, 0, 4 * sizeof(uint32_t)) != cudaSuccess) st2 = fail(MOE_ECUDA, "memset");
            if (st2) return st2;
        }
        if (!c->d_tc_items) {
            int st2 = dalloc(&c->d_tc_items, (size_t)cap_gu + cap_dn);
            if (!st2) st2 = dalloc(&c->d_tc_cnt, 4);
            if (!st2) st2 = dalloc(&c->d_tc_mtdone, (size_t)mt_max);
            if (st2) return st2;
        }
        TcItem* items_dn = c->d_tc_items + cap_gu;
        const int n_slots = c->arena_slots[layer];
        CUDA_TRY(launch_tc_items(c->d_jobs, c->d_nlj, E, c->arena[layer], c->stride, F, H, c->d_tc_items, cap_gu, items_dn,
                                 cap_dn, c->d_tc_cnt, c->d_err, c->d_tc_mtdone, st));
        CUDA_TRY(launch_gather_rows(x, c->d_ptok, (int)NP, H, c->d_pf_x, c->sm_count, st, c->d_tc_cnt + 2));
        CUDA_TRY(launch_gateup_tc(c->d_pf_x, (int)NP, c->arena[layer], n_slots, c->stride, c->d_tc_items, 0, c->d_tc_cnt,
                                  H, F, c->d_act, c->d_tc_sched, c->d_err, c->timeout_ns, c->sm_count, c->d_tc_mtdone,
                                  st));
        CUDA_TRY(launch_down_tc(c->d_act, (int)NP, c->arena[layer], n_slots, c->stride, items_dn, 0, c->d_tc_cnt + 1, H, F,
                                c->d_pf_yf, c->d_tc_sched + 2, c->d_err, c->timeout_ns, c->sm_count, c->d_tc_mtdone,
                                st));
        CUDA_TRY(launch_combine_rows(c->d_pf_yf, c->d_pw, c->d_comb_off, c->d_comb_p, T, H, accumulate, o, st));
        c->launches += 5;
        *done = true;
        return MOE_OK;
    }
    return MOE_OK;  // tcgen05 kernels unavailable for this shape: the CUDA-core path runs
}

// Host buffers on the fused path.  Pinned host memory is device-accessible under unified addressing,
// so the kernel uses it in place: every decode CTA copies a slice of the pinned hidden states and
// logits into the context's device buffers and routes once all slices are there, writes its part of
// the output over the bus and CTA 0 leaves the error bits in a pinned word.  No copy is issued on
// the stream.  Unpinned (or, for the output, unaligned) buffers go through the context's pinned
// staging.  One stream synchronisation ends the call.
// Waits for a fused call launched with err_host = h_errsnap: the CTA that finishes last stores the
// call's completion tag there, in pinned memory, after every output, so the call can return once it
// is there (a stream synchronisation costs several microseconds more).  False when the stream ran
// dry without the tag (a bounded wait gave up): the caller synchronises and reads the error word.
bool wait_tag(moe_ctx* c, cudaStream_t st, uint32_t tag) {
    volatile uint32_t* snap = c->h_errsnap;
    bool tagged = false;
    for (uint32_t spin = 1;; spin++) {
        if (snap[1] == tag) {
            tagged = true;
            break;
        }
        if ((spin & 1023u) == 0) {
            const cudaError_t q = cudaStreamQuery(st);
            if (q != cudaErrorNotReady) break;  // done (or failed): the caller's synchronisation tells
            cudaGetLastError();
        }
    }
    std::atomic_thread_fence(std::memory_order_acquire);
    return tagged;
}

// Error bits of a call that reported through h_errsnap (tagged or after a synchronisation): clears
// the sticky device word and, after a timeout, the grid counters.
int snap_status(moe_ctx* c, cudaStream_t st, bool tagged) {
    uint32_t bits = c->h_errsnap[0] | c->latched;
    c->latched = 0;
    if (bits) {
        if (tagged) CUDA_TRY(cudaStreamSynchronize(st));
        CUDA_TRY(cudaMemset(c->d_err, 0, sizeof(uint32_t)));
        if (bits & kErrTimeout) {
            int r = reset_counters(c);
            if (r) return r;
        }
    }
    return map_err(bits);
}

int forward_host_fused(moe_ctx* c, int layer, int T, const uint16_t* hidden, const float* logits, float* out,
                       int32_t* topk_idx, float* topk_w, int flags, cudaStream_t st, DecodeArgs& da, size_t dsmem) {
    const int H = c->cfg.hidden, E = c->cfg.n_experts, K = c->cfg.top_k;
    const size_t hb = (size_t)T * H * 2, lb = (size_t)T * E * 4, ob = (size_t)T * H * 4;
    const bool pin_x = device_mapped(hidden) && ((uintptr_t)hidden & 15u) == 0;
    const bool pin_l = device_mapped(logits) && ((uintptr_t)logits & 15u) == 0;  // the kernel reads it by 16 bytes
    const bool pin_o = device_mapped(out) && ((uintptr_t)out & 15u) == 0;
    int s;
    const float* lg = logits;
    const uint16_t* xs = hidden;  // pinned source the decode kernel copies to the device
    if (!pin_x || !pin_l) {
        if ((s = c->in_stage.reserve(align_up(hb, 256) + lb))) return s;
        if (!pin_l) {
            memcpy((char*)c->in_stage.host + align_up(hb, 256), logits, lb);
            lg = reinterpret_cast<const float*>((char*)c->in_stage.host + align_up(hb, 256));
        }
        if (!pin_x) {
            memcpy(c->in_stage.host, hidden, hb);
            xs = static_cast<const uint16_t*>(c->in_stage.host);
        }
    }
    float* o = out;
    if (!pin_o) {
        if ((s = c->out_stage.reserve(ob))) return s;
        o = static_cast<float*>(c->out_stage.host);
        if (flags & MOE_F_ACCUMULATE) memcpy(o, out, ob);
    }
    volatile uint32_t* snap = c->h_errsnap;
    snap[0] = 0;
    da.x = c->d_hidden;
    da.out = o;
    da.err_host = c->h_errsnap;
    if ((s = launch_fused(c, layer, lg, da, dsmem, st, nullptr, xs))) return s;
    if (!pin_x || !pin_l) c->in_stage.mark(st);
    if (topk_idx) CUDA_TRY(cudaMemcpyAsync(topk_idx, c->d_idx, sizeof(int32_t) * T * K, cudaMemcpyDeviceToHost, st));
    if (topk_w) CUDA_TRY(cudaMemcpyAsync(topk_w, c->d_w, sizeof(float) * T * K, cudaMemcpyDeviceToHost, st));
    // Top-k copies, and kernels that end without a completion tag, take the stream synchronisation.
    const bool tagged = !topk_idx && !topk_w && wait_tag(c, st, da.epoch + 1u);
    if (!tagged) CUDA_TRY(cudaStreamSynchronize(st));
    const int r = snap_status(c, st, tagged);
    if (!pin_o) memcpy(out, o, ob);
    return r;
}

}  // namespace

extern "C" {

int moe_abi_version(void) { return MOE_DP_ABI_VERSION; }

const char* moe_last_error(void) { return g_err.c_str(); }

int moe_create(const moe_config* cfg, moe_ctx** out) {
    if (!cfg || !out) return fail(MOE_EINVAL, "null argument");
    *out = nullptr;
    const moe_config& k = *cfg;
    if (k.hidden <= 0 || k.hidden % 64 != 0 || k.hidden > 16384)
        return fail(MOE_EINVAL, "hidden %d must be a positive multiple of 64, <= 16384", k.hidden);
    if (k.inter <= 0 || k.inter % 64 != 0 || k.inter > 2048)
        return fail(MOE_EINVAL, "inter %d must be a positive multiple of 64, <= 2048", k.inter);
    if (k.n_experts < 1 || k.n_experts > kMaxExperts) return fail(MOE_EINVAL, "n_experts %d not in [1,%d]", k.n_experts, kMaxExperts);
    if (k.top_k < 1 || k.top_k > kMaxTopK || k.top_k > k.n_experts)
        return fail(MOE_EINVAL, "top_k %d not in [1,min(%d,E)]", k.top_k, kMaxTopK);
    if (k.n_layers < 1) return fail(MOE_EINVAL, "n_layers %d < 1", k.n_layers);
    if (k.max_tokens < 1 || k.max_tokens > kMaxTokens) return fail(MOE_EINVAL, "max_tokens %d not in [1,%d]", k.max_tokens, kMaxTokens);
    if (k.scoring != MOE_SCORING_SOFTMAX && k.scoring != MOE_SCORING_SIGMOID) return fail(MOE_EINVAL, "unknown scoring %d", k.scoring);
    if (k.ep_world < 1 || k.ep_rank < 0 || k.ep_rank >= k.ep_world) return fail(MOE_EINVAL, "bad ep rank %d / world %d", k.ep_rank, k.ep_world);
    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev == 0) {
        cudaGetLastError();
        return fail(MOE_ECUDA, "no CUDA device available");
    }
    if (k.device < 0 || k.device >= ndev) return fail(MOE_EINVAL, "device %d not in [0,%d)", k.device, ndev);
    DeviceGuard dg(k.device);
    moe_ctx* c = new moe_ctx;
    c->cfg = k;
    // expert-parallel ranks plan in their own CTAs: their layers stream for a fraction of a
    // one-GPU layer, less than the planner kernel needs under load (measured on two B200: 29.6 us
    // per unit-sharded Solar layer without it, 37.6 us with it)
    c->use_planner = kPlannerDefault && k.ep_world <= 1;
    c->late_bytes = k.ep_world > 1 ? kLateBytesDefaultEp : kLateBytesDefault;
    // eight ranks: each layer streams a few microseconds per GPU; more reducers shorten the
    // reduction + exchange (measured on eight B200, unit-sharded Solar layers: 22.2 us per layer with
    // 96 reducers, 24.1 us with 48)
    if (k.ep_world >= 8) c->reducers = kReducersDefaultEp8;
    c->cfg.shard_map = nullptr;
    c->dev = k.device;
    cudaDeviceGetAttribute(&c->sm_count, cudaDevAttrMultiProcessorCount, k.device);
    const int L = k.n_layers, E = k.n_experts;
    c->owner.assign((size_t)L * E, 0);
    c->slot.assign((size_t)L * E, -1);
    c->n_local.assign(L, 0);
    for (int l = 0; l < L; l++)
        for (int e = 0; e < E; e++) {
            int r = k.shard_map ? k.shard_map[(size_t)l * E + e] : (k.ep_world == 1 ? 0 : e % k.ep_world);
            if (r < 0 || r >= k.ep_world) {
                delete c;
                return fail(MOE_EINVAL, "shard_map[%d][%d] = %d not in [0,%d)", l, e, r, k.ep_world);
            }
            c->owner[(size_t)l * E + e] = r;
            if (r == k.ep_rank) c->slot[(size_t)l * E + e] = c->n_local[l]++;
        }
    c->res = c->slot;
    c->arena_slots.assign(c->n_local.begin(), c->n_local.end());
    c->arena.assign(L, nullptr);
    c->stride = align_up((size_t)3 * k.inter * k.hidden * 2, 256);
    c->h_desc.assign((size_t)L * E, ExpDesc{nullptr, nullptr, nullptr, kKindNone, 0});
    for (size_t i = 0; i < c->h_desc.size(); i++)
        if (c->slot[i] < 0) c->h_desc[i].kind = kKindRemote;
    c->has_bias.assign(L, 0);
    const size_t NP = (size_t)k.max_tokens * k.top_k;
    int st = MOE_OK;
    if (!st) st = dalloc(&c->d_desc, (size_t)L * E);
    if (!st) st = dalloc(&c->d_route_scratch, route_scratch_ints(k.max_tokens, E));
    if (!st) st = dalloc(&c->d_bias, (size_t)L * E);
    if (!st) st = dalloc(&c->d_idx, NP);
    if (!st) st = dalloc(&c->d_w, NP);
    if (!st) st = dalloc(&c->d_counts, E);
    if (!st) st = dalloc(&c->d_offsets, E + 1);
    if (!st) st = dalloc(&c->d_perm, NP);
    if (!st) st = dalloc(&c->d_jobord, E);
    if (!st) st = dalloc(&c->d_nj, 1);
    if (!st) st = dalloc(&c->d_nlj, 1);
    if (!st) st = dalloc(&c->d_ptok, NP);
    if (!st) st = dalloc(&c->d_pw, NP);
    if (!st) st = dalloc(&c->d_pairpos, NP);
    if (!st) st = dalloc(&c->d_comb_off, (size_t)k.max_tokens + 1);
    if (!st) st = dalloc(&c->d_comb_p, NP);
    if (!st) st = dalloc(&c->d_jobs, E);
    if (!st) st = dalloc(&c->d_act, NP * k.inter);
    if (!st) st = dalloc(&c->d_y, NP * k.hidden);
    if (!st) st = dalloc(&c->d_err, 1);
    if (!st) st = dalloc(&c->d_hidden, (size_t)k.max_tokens * k.hidden);
    if (!st) st = dalloc(&c->d_logits, (size_t)k.max_tokens * E);
    if (!st) st = dalloc(&c->d_out, (size_t)k.max_tokens * k.hidden);
    if (!st) st = dalloc(&c->d_cnt, 4);
    if (!st) st = dalloc(&c->d_decide, 4);
    if (!st && cudaMemset(c->d_decide, 0, 4 * sizeof(unsigned long long)) != cudaSuccess) st = fail(MOE_ECUDA, "memset failed");
    if (!st) st = dalloc(&c->d_part, 2 * decode_part_floats(k.hidden, c->sm_count));
    if (!st) st = dalloc(&c->d_hctr, 2);
    if (!st) st = dalloc(reinterpret_cast<char**>(&c->d_pub), 4 * pub_plan_bytes());
    if (!st) st = dalloc(&c->d_pub_flag, 4);
    if (!st && cudaMemset(c->d_pub_flag, 0, 4 * sizeof(uint32_t)) != cudaSuccess) st = fail(MOE_ECUDA, "memset failed");
    if (!st && cudaMemset(c->d_hctr, 0, 2 * sizeof(uint32_t)) != cudaSuccess) st = fail(MOE_ECUDA, "memset failed");
    if (!st && cudaMemset(c->d_cnt, 0, sizeof(unsigned long long) * 4) != cudaSuccess)
        st = fail(MOE_ECUDA, "memset failed");
    if (!st && cudaMallocHost((void**)&c->h_err, sizeof(uint32_t)) != cudaSuccess) st = fail(MOE_ENOMEM, "pinned error word");
    if (!st && cudaMallocHost((void**)&c->h_errsnap, 16) != cudaSuccess) st = fail(MOE_ENOMEM, "pinned error word");
    if (!st && (cudaEventCreateWithFlags(&c->dec_ev, cudaEventDisableTiming) != cudaSuccess ||
                cudaEventCreateWithFlags(&c->in_stage.ev, cudaEventDisableTiming) != cudaSuccess ||
                cudaEventCreateWithFlags(&c->out_stage.ev, cudaEventDisableTiming) != cudaSuccess ||
                cudaEventCreateWithFlags(&c->job_stage.ev, cudaEventDisableTiming) != cudaSuccess))
        st = fail(MOE_ECUDA, "event creation failed");
    if (!st && cudaMemcpy(c->d_desc, c->h_desc.data(), sizeof(ExpDesc) * c->h_desc.size(), cudaMemcpyHostToDevice) != cudaSuccess)
        st = fail(MOE_ECUDA, "descriptor upload failed");
    if (!st && cudaMemset(c->d_err, 0, sizeof(uint32_t)) != cudaSuccess) st = fail(MOE_ECUDA, "memset failed");
    if (!st && cudaMemset(c->d_bias, 0, sizeof(float) * (size_t)L * E) != cudaSuccess) st = fail(MOE_ECUDA, "memset failed");
    if (!st) {
        cudaError_t e = decode_set_smem_limit();
        if (e != cudaSuccess) st = fail(MOE_ECUDA, "kernel attribute: %s", cudaGetErrorString(e));
    }
    if (!st && !decode_register_split_fits()) c->fused = false;  // this build cannot run the fused kernel
    if (!st) {
        cudaError_t e = tc_set_smem_limit();
        if (e != cudaSuccess) st = fail(MOE_ECUDA, "kernel attribute: %s", cudaGetErrorString(e));
    }
    if (!st) {
        cudaError_t e = route_set_smem_limits();
        if (e != cudaSuccess) st = fail(MOE_ECUDA, "kernel attribute: %s", cudaGetErrorString(e));
    }
    if (st) {
        moe_destroy(c);
        return st;
    }
    *out = c;
    return MOE_OK;
}

int moe_destroy(moe_ctx* c) {
    if (!c) return MOE_OK;
    DeviceGuard dg(c->dev);
    cudaDeviceSynchronize();
    if (c->shared) moe_destroy(c->shared);
    if (c->d_down_stage) cudaFree(c->d_down_stage);
    for (uint16_t* r : c->d_router) cudaFree(r);
    for (void* q : {(void*)c->d_blk_zero, (void*)c->d_blk_logits, (void*)c->d_blk_shared, (void*)c->d_blk_moe,
                    (void*)c->d_blk_y, (void*)c->d_blk_io, (void*)c->d_blk_extra})
        if (q) cudaFree(q);
    for (void* p : c->arena) cudaFree(p);
    if (c->d_timeline) cudaFree(c->d_timeline);
    void* ps[] = {c->d_desc, c->d_bias, c->d_idx, c->d_w, c->d_counts, c->d_offsets, c->d_perm, c->d_jobord,
                  c->d_nj, c->d_nlj, c->d_ptok, c->d_pw, c->d_pairpos, c->d_comb_off, c->d_comb_p, c->d_jobs,
                  c->d_act, c->d_y, c->d_err, c->d_hidden, c->d_logits, c->d_out, c->d_cnt, c->d_hctr,
                  c->d_part, c->d_route_scratch, c->d_pub, c->d_pub_flag, c->d_decide};
    for (void* p : ps) cudaFree(p);
    for (void* q : {(void*)c->d_pf_x, (void*)c->d_pf_yf, (void*)c->d_tc_sched,
                    (void*)c->d_tc_items, (void*)c->d_tc_cnt, (void*)c->d_tc_mtdone})
        if (q) cudaFree(q);
    for (void* q : c->ipc_opened) cudaIpcCloseMemHandle(q);
    for (void* q : {(void*)c->d_xbuf, (void*)c->d_peer_x, (void*)c->d_xpart})
        if (q) cudaFree(q);
    if (c->h_err) cudaFreeHost(c->h_err);
    if (c->h_errsnap) cudaFreeHost(c->h_errsnap);
    for (cudaEvent_t ev : c->prof_ev) cudaEventDestroy(ev);
    if (c->dec_ev) cudaEventDestroy(c->dec_ev);
    for (Staging* s : {&c->in_stage, &c->out_stage, &c->job_stage}) {
        if (s->host) cudaFreeHost(s->host);
        if (s->ev) cudaEventDestroy(s->ev);
    }
    delete c;
    return MOE_OK;
}

int moe_load_expert_bf16(moe_ctx* c, int layer, int expert, const uint16_t* gate, const uint16_t* up,
                         const uint16_t* down, int flags) {
    int st = check_layer_expert(c, layer, expert);
    if (st) return st;
    if (!gate || !up || !down) return fail(MOE_EINVAL, "null weight pointer");
    DeviceGuard dg(c->dev);
    if ((st = ensure_arena(c, layer))) return st;
    if ((st = acquire_slot(c, layer, expert))) return st;
    const size_t H = c->cfg.hidden, F = c->cfg.inter, P = unit_pitch(kKindBF16, (int)H);
    char* base = slot_ptr(c, layer, expert);
    const bool host = flags & MOE_F_HOST;
    const cudaMemcpyKind kind = host ? cudaMemcpyHostToDevice : cudaMemcpyDeviceToDevice;
    // unit table: [gate row f | up row f | down column f] per f
    CUDA_TRY(cudaMemcpy2DAsync(base, 2 * P, gate, 2 * H, 2 * H, F, kind, 0));
    CUDA_TRY(cudaMemcpy2DAsync(base + 2 * H, 2 * P, up, 2 * H, 2 * H, F, kind, 0));
    if ((st = load_down_columns(c, base + 4 * H, down, P, 2, host))) return st;
    return upload_desc(c, layer, expert, ExpDesc{base, base + 4 * H, nullptr, kKindBF16, kLayoutUnit});
}

int moe_load_expert_q8(moe_ctx* c, int layer, int expert, const int8_t* q, const float* scales, int flags) {
    int st = check_layer_expert(c, layer, expert);
    if (st) return st;
    if (!q || !scales) return fail(MOE_EINVAL, "null weight pointer");
    DeviceGuard dg(c->dev);
    if ((st = ensure_arena(c, layer))) return st;
    if ((st = acquire_slot(c, layer, expert))) return st;
    const size_t H = c->cfg.hidden, F = c->cfg.inter, P = unit_pitch(kKindQ8, (int)H);
    char* base = slot_ptr(c, layer, expert);
    const bool host = flags & MOE_F_HOST;
    const cudaMemcpyKind kind = host ? cudaMemcpyHostToDevice : cudaMemcpyDeviceToDevice;
    // reference layout [F gate][F up][H down] rows -> unit table [gate | up | down column | sc_g, sc_u, 0, 0]
    CUDA_TRY(cudaMemcpy2DAsync(base, P, q, H, H, F, kind, 0));
    CUDA_TRY(cudaMemcpy2DAsync(base + H, P, q + F * H, H, H, F, kind, 0));
    CUDA_TRY(cudaMemcpy2DAsync(base + 3 * H, P, scales, 4, 4, F, kind, 0));
    CUDA_TRY(cudaMemcpy2DAsync(base + 3 * H + 4, P, scales + F, 4, 4, F, kind, 0));
    CUDA_TRY(cudaMemset2DAsync(base + 3 * H + 8, P, 0, 8, F, 0));
    if ((st = copy_in(base + q8_scale_off(c), scales, (2 * F + H) * 4, host, 0))) return st;
    if ((st = load_down_columns(c, base + 2 * H, q + 2 * F * H, P, 1, host))) return st;
    return upload_desc(c, layer, expert,
                       ExpDesc{base, base + 2 * H, (const float*)(base + q8_scale_off(c)), kKindQ8, kLayoutUnit});
}

int moe_quantize_expert_q8(moe_ctx* c, int layer, int expert) {
    int st = check_layer_expert(c, layer, expert);
    if (st) return st;
    const size_t i = (size_t)layer * c->cfg.n_experts + expert;
    if (c->h_desc[i].kind != kKindBF16) return fail(MOE_ESTATE, "expert (%d,%d) is not a loaded bf16 expert", layer, expert);
    DeviceGuard dg(c->dev);
    const size_t H = c->cfg.hidden, F = c->cfg.inter;
    char* base = slot_ptr(c, layer, expert);
    char* tmp = nullptr;
    const size_t bytes = q8_scale_off(c) + (2 * F + H) * 4;
    if (cudaMalloc(&tmp, bytes) != cudaSuccess) {
        cudaGetLastError();
        return fail(MOE_ENOMEM, "quantisation scratch");
    }
    int n = 0;
    // bf16 unit table in, int8 unit table (with per-unit scale trailers) out
    cudaError_t e = launch_quantize_q8(quant_geom_unit((const uint16_t*)base, (int)H, (int)F, (int8_t*)tmp), (int)H,
                                       (int)F, (float*)(tmp + q8_scale_off(c)), nullptr, 0, &n);
    c->launches += n;
    if (e == cudaSuccess) e = cudaMemcpyAsync(base, tmp, bytes, cudaMemcpyDeviceToDevice, 0);
    if (e == cudaSuccess) e = cudaStreamSynchronize(0);
    cudaFree(tmp);
    if (e != cudaSuccess) return fail(MOE_ECUDA, "quantise: %s", cudaGetErrorString(e));
    return upload_desc(c, layer, expert,
                       ExpDesc{base, base + 2 * H, (const float*)(base + q8_scale_off(c)), kKindQ8, kLayoutUnit});
}

int moe_evict_expert(moe_ctx* c, int layer, int expert) {
    int st = check_layer_expert(c, layer, expert);
    if (st) return st;
    const size_t i = (size_t)layer * c->cfg.n_experts + expert;
    if (c->res[i] < 0) return MOE_OK;
    DeviceGuard dg(c->dev);
    c->res[i] = -1;  // the slot is free for the next load; routing to this expert now reports MOE_ESTATE
    return upload_desc(c, layer, expert, ExpDesc{nullptr, nullptr, nullptr, kKindNone, 0});
}

int moe_expert_kind(moe_ctx* c, int layer, int expert) {
    if (!c || layer < 0 || layer >= c->cfg.n_layers || expert < 0 || expert >= c->cfg.n_experts) return -1;
    int k = c->h_desc[(size_t)layer * c->cfg.n_experts + expert].kind;
    return k == kKindRemote ? MOE_KIND_NONE : k;
}

int moe_set_bias(moe_ctx* c, int layer, const float* bias, int flags) {
    if (!c || layer < 0 || layer >= c->cfg.n_layers) return fail(MOE_EINVAL, "bad context or layer");
    DeviceGuard dg(c->dev);
    if (!bias) {
        CUDA_TRY(cudaMemset(c->d_bias + (size_t)layer * c->cfg.n_experts, 0, sizeof(float) * c->cfg.n_experts));
        c->has_bias[layer] = 0;
        return MOE_OK;
    }
    CUDA_TRY(cudaMemcpy(c->d_bias + (size_t)layer * c->cfg.n_experts, bias, sizeof(float) * c->cfg.n_experts,
                        (flags & MOE_F_HOST) ? cudaMemcpyHostToDevice : cudaMemcpyDeviceToDevice));
    c->has_bias[layer] = 1;
    return MOE_OK;
}

static RouteArgs route_args(moe_ctx* c, int T, const float* logits, const float* bias) {
    RouteArgs a{};
    a.logits = logits;
    a.bias = bias;
    a.T = T;
    a.E = c->cfg.n_experts;
    a.K = c->cfg.top_k;
    a.scoring = c->cfg.scoring;
    a.idx = c->d_idx;
    a.w = c->d_w;
    a.counts = c->d_counts;
    a.offsets = c->d_offsets;
    a.perm = c->d_perm;
    a.job_order = c->d_jobord;
    a.n_jobs = c->d_nj;
    a.ptok = c->d_ptok;
    a.pw = c->d_pw;
    a.pairpos = c->d_pairpos;
    a.comb_off = c->d_comb_off;
    a.comb_p = c->d_comb_p;
    a.jobs = c->d_jobs;
    a.n_ljobs = c->d_nlj;
    a.err = c->d_err;
    a.scratch = c->d_route_scratch;
    return a;
}

int moe_forward(moe_ctx* c, int layer, int T, const uint16_t* hidden, const float* logits, float* out,
                int32_t* topk_idx, float* topk_w, int flags, void* stream) {
    if (!c) return fail(MOE_EINVAL, "null context");
    if (layer < 0 || layer >= c->cfg.n_layers) return fail(MOE_EINVAL, "layer %d out of range [0,%d)", layer, c->cfg.n_layers);
    if (T < 0 || T > c->cfg.max_tokens) return fail(MOE_EINVAL, "T=%d not in [0,%d]", T, c->cfg.max_tokens);
    if (T > 0 && (!hidden || !logits || !out)) return fail(MOE_EINVAL, "null hidden/logits/out");
    if (!(flags & MOE_F_HOST) && (((uintptr_t)hidden | (uintptr_t)logits | (uintptr_t)out) & 15u))
        return fail(MOE_EINVAL, "hidden/logits/out must be 16-byte aligned");
    DeviceGuard dg(c->dev);
    cudaStream_t st = (cudaStream_t)stream;
    const bool host = flags & MOE_F_HOST;
    const int H = c->cfg.hidden, E = c->cfg.n_experts, K = c->cfg.top_k;
    const uint16_t* x = hidden;
    const float* lg = logits;
    float* o = out;
    int s;
    DecodeArgs da{};
    size_t dsmem = 0;
    const bool use_fused = !prefill_applies(c, layer, T) && prepare_fused(c, T, flags, da, &dsmem);
    if (host && use_fused && !c->prof_on)
        return forward_host_fused(c, layer, T, hidden, logits, out, topk_idx, topk_w, flags, st, da, dsmem);
    if (host && T > 0) {
        const size_t hb = (size_t)T * H * 2, lb = (size_t)T * E * 4;
        if (is_pinned_host(hidden) && is_pinned_host(logits)) {
            CUDA_TRY(cudaMemcpyAsync(c->d_hidden, hidden, hb, cudaMemcpyHostToDevice, st));
            CUDA_TRY(cudaMemcpyAsync(c->d_logits, logits, lb, cudaMemcpyHostToDevice, st));
        } else {
            if ((s = c->in_stage.reserve(hb + lb))) return s;
            memcpy(c->in_stage.host, hidden, hb);
            memcpy((char*)c->in_stage.host + hb, logits, lb);
            CUDA_TRY(cudaMemcpyAsync(c->d_hidden, c->in_stage.host, hb, cudaMemcpyHostToDevice, st));
            CUDA_TRY(cudaMemcpyAsync(c->d_logits, (char*)c->in_stage.host + hb, lb, cudaMemcpyHostToDevice, st));
            c->in_stage.mark(st);
        }
        x = c->d_hidden;
        lg = c->d_logits;
        o = c->d_out;
        if (flags & MOE_F_ACCUMULATE) CUDA_TRY(cudaMemcpyAsync(o, out, (size_t)T * H * 4, cudaMemcpyHostToDevice, st));
    }
    int n = 0;
    cudaEvent_t* marks = nullptr;
    if (c->prof_on && T > 0) {
        const size_t need = (c->prof_calls + 1) * kProfMarks;
        while (c->prof_ev.size() < need) {
            cudaEvent_t ev;
            CUDA_TRY(cudaEventCreate(&ev));
            c->prof_ev.push_back(ev);
        }
        marks = &c->prof_ev[c->prof_calls * kProfMarks];
        c->prof_calls++;
        CUDA_TRY(cudaEventRecord(marks[0], st));
    }
    // a synchronous fused call on device buffers waits for its completion tag like a host call
    const bool sync_tag = use_fused && !host && (flags & MOE_F_SYNC) && !topk_idx && !topk_w && !marks;
    if (use_fused) {
        da.x = x;
        da.out = o;
        if (sync_tag) {
            c->h_errsnap[0] = 0;
            da.err_host = c->h_errsnap;
        }
        if ((s = launch_fused(c, layer, lg, da, dsmem, st, marks))) return s;
        if (sync_tag) {
            const bool tagged = wait_tag(c, st, da.epoch + 1u);
            if (!tagged) CUDA_TRY(cudaStreamSynchronize(st));
            return snap_status(c, st, tagged);
        }
    }
    if (T > 0 && !use_fused) {
        RouteArgs ra = route_args(c, T, lg, c->has_bias[layer] ? c->d_bias + (size_t)layer * E : nullptr);
        ra.desc = c->d_desc + (size_t)layer * E;
        cudaError_t e = launch_route(ra, st, &n);
        if (marks) cudaEventRecord(marks[1], st);
        if (e != cudaSuccess) return fail(MOE_ECUDA, "route launch: %s", cudaGetErrorString(e));
        ExpertArgs ea{};
        ea.x = x;
        ea.T = T;
        ea.H = H;
        ea.F = c->cfg.inter;
        ea.jobs = c->d_jobs;
        ea.n_jobs = c->d_nlj;
        ea.n_jobs_host = -1;
        ea.n_jobs_max = std::min(E, T * K);
        ea.max_pairs = T;
        ea.ptok = c->d_ptok;
        ea.pw = c->d_pw;
        ea.act = c->d_act;
        ea.y = c->d_y;
        ea.comb_off = c->d_comb_off;
        ea.comb_p = c->d_comb_p;
        const bool acc = (flags & MOE_F_ACCUMULATE) != 0;
        // expert parallel: the local partial goes to scratch, the exchange adds every rank's into out
        ea.out = c->ep_attached ? c->d_xpart : o;
        ea.accumulate = (acc && !c->ep_attached) ? 1 : 0;
        ea.err = c->d_err;
        ea.unit_layout = 1;  // context tables
        bool done = false;
        c->launches += n;
        n = 0;
        if (prefill_applies(c, layer, T) && !marks) {
            int r = run_prefill(c, layer, T, x, ea.out, ea.accumulate, st, &done);
            if (r) return r;
        }
        if (!done) {
            e = launch_experts(ea, c->sm_count, st, &n, marks ? marks + 2 : nullptr);
            c->launches += n;
            if (e != cudaSuccess) return fail(MOE_ECUDA, "expert launch: %s", cudaGetErrorString(e));
        }
        if (c->ep_attached)
            for (int t0 = 0; t0 < T; t0 += c->ep_tcap) {  // one exchange unless T exceeds the buffer
                const int tc = std::min(c->ep_tcap, T - t0);
                e = launch_ep_exchange(next_ep(c), c->d_xpart + (size_t)t0 * H, o + (size_t)t0 * H, tc, H, acc ? 1 : 0,
                                       c->d_err, c->timeout_ns, c->sm_count - 1, st);
                c->launches += 1;
                if (e != cudaSuccess) return fail(MOE_ECUDA, "exchange launch: %s", cudaGetErrorString(e));
            }
    }
    if (T > 0) {
        const cudaMemcpyKind dk = host ? cudaMemcpyDeviceToHost : cudaMemcpyDeviceToDevice;
        if (topk_idx) CUDA_TRY(cudaMemcpyAsync(topk_idx, c->d_idx, sizeof(int32_t) * T * K, dk, st));
        if (topk_w) CUDA_TRY(cudaMemcpyAsync(topk_w, c->d_w, sizeof(float) * T * K, dk, st));
    }
    if (host) {
        if (T > 0) {
            const size_t ob = (size_t)T * H * 4;
            if (is_pinned_host(out)) {
                CUDA_TRY(cudaMemcpyAsync(out, o, ob, cudaMemcpyDeviceToHost, st));
                return finish_sync(c, st);
            }
            if ((s = c->out_stage.reserve(ob))) return s;
            CUDA_TRY(cudaMemcpyAsync(c->out_stage.host, o, ob, cudaMemcpyDeviceToHost, st));
            int r = finish_sync(c, st);
            memcpy(out, c->out_stage.host, ob);
            return r;
        }
        return finish_sync(c, st);
    }
    if (flags & MOE_F_SYNC) return finish_sync(c, st);
    return MOE_OK;
}

int moe_forward_layers(moe_ctx* c, int n, const int32_t* layers, int T, const uint16_t* const* hidden,
                       const float* const* logits, float* const* out, int flags, void* stream) {
    if (!c) return fail(MOE_EINVAL, "null context");
    if (n < 0) return fail(MOE_EINVAL, "n=%d < 0", n);
    if (n > 0 && (!layers || !hidden || !logits || !out)) return fail(MOE_EINVAL, "null layer or buffer array");
    if (flags & MOE_F_HOST) return fail(MOE_EINVAL, "moe_forward_layers takes device buffers (MOE_F_HOST: call moe_forward)");
    for (int i = 0; i < n; i++) {
        const int st = moe_forward(c, layers[i], T, hidden[i], logits[i], out[i], nullptr, nullptr,
                                   flags & ~MOE_F_SYNC, stream);
        if (st) return st;
    }
    if (flags & MOE_F_SYNC) {
        DeviceGuard dg(c->dev);
        return finish_sync(c, (cudaStream_t)stream);
    }
    return MOE_OK;
}

int moe_route(moe_ctx* c, int T, const float* logits, const float* bias, int32_t* topk_idx, float* topk_w,
              int32_t* counts, int32_t* offsets, int32_t* perm, int32_t* job_order, int32_t* n_jobs, int flags,
              void* stream) {
    if (!c) return fail(MOE_EINVAL, "null context");
    if (T < 0 || T > c->cfg.max_tokens) return fail(MOE_EINVAL, "T=%d not in [0,%d]", T, c->cfg.max_tokens);
    if (T > 0 && !logits) return fail(MOE_EINVAL, "null logits");
    DeviceGuard dg(c->dev);
    cudaStream_t st = (cudaStream_t)stream;
    const bool host = flags & MOE_F_HOST;
    const int E = c->cfg.n_experts, K = c->cfg.top_k;
    const float* lg = logits;
    const float* b = bias;
    if (host) {
        if (T > 0) CUDA_TRY(cudaMemcpyAsync(c->d_logits, logits, sizeof(float) * T * E, cudaMemcpyHostToDevice, st));
        lg = c->d_logits;
        if (bias) {
            CUDA_TRY(cudaMemcpyAsync(c->d_out, bias, sizeof(float) * E, cudaMemcpyHostToDevice, st));
            b = c->d_out;
        }
    }
    RouteArgs ra = route_args(c, T, lg, b);
    ra.desc = nullptr;
    ra.jobs = nullptr;
    ra.n_ljobs = nullptr;
    int n = 0;
    cudaError_t e = launch_route(ra, st, &n);
    c->launches += n;
    if (e != cudaSuccess) return fail(MOE_ECUDA, "route launch: %s", cudaGetErrorString(e));
    const cudaMemcpyKind dk = host ? cudaMemcpyDeviceToHost : cudaMemcpyDeviceToDevice;
    const size_t NP = (size_t)T * K;
    if (topk_idx && NP) CUDA_TRY(cudaMemcpyAsync(topk_idx, c->d_idx, 4 * NP, dk, st));
    if (topk_w && NP) CUDA_TRY(cudaMemcpyAsync(topk_w, c->d_w, 4 * NP, dk, st));
    if (counts) CUDA_TRY(cudaMemcpyAsync(counts, c->d_counts, 4 * E, dk, st));
    if (offsets) CUDA_TRY(cudaMemcpyAsync(offsets, c->d_offsets, 4 * (E + 1), dk, st));
    if (perm && NP) CUDA_TRY(cudaMemcpyAsync(perm, c->d_perm, 4 * NP, dk, st));
    if (job_order) CUDA_TRY(cudaMemcpyAsync(job_order, c->d_jobord, 4 * E, dk, st));
    if (n_jobs) CUDA_TRY(cudaMemcpyAsync(n_jobs, c->d_nj, 4, dk, st));
    if (host || (flags & MOE_F_SYNC)) return finish_sync(c, st);
    return MOE_OK;
}

// Shared body of the explicit-job surfaces (cpu_moe, ck_moe3, ck_moe_q8w).
static int run_jobs(moe_ctx* c, int T, const uint16_t* x, const std::vector<Job>& jobs,
                    const std::vector<int32_t>& ptok, const float* pw_src, bool pw_host, const std::vector<int32_t>& comb_off,
                    const std::vector<int32_t>& comb_p, float* out, int flags, cudaStream_t st) {
    const int H = c->cfg.hidden;
    const size_t NP = ptok.size();
    if (jobs.size() > (size_t)c->cfg.n_experts)
        return fail(MOE_EINVAL, "%zu expert jobs exceed the context capacity n_experts=%d", jobs.size(), c->cfg.n_experts);
    for (const Job& j : jobs)
        if (((uintptr_t)j.ex.w1 | (uintptr_t)j.ex.w2 | (uintptr_t)j.ex.sc) & 15u)
            return fail(MOE_EINVAL, "expert weight pointers must be 16-byte aligned");
    if (((uintptr_t)x | (uintptr_t)out) & 15u) return fail(MOE_EINVAL, "x/out must be 16-byte aligned");
    if (NP > (size_t)c->cfg.max_tokens * c->cfg.top_k)
        return fail(MOE_EINVAL, "%zu routed pairs exceed the context capacity %d (max_tokens * top_k)", NP,
                    c->cfg.max_tokens * c->cfg.top_k);
    if ((size_t)T > (size_t)c->cfg.max_tokens) return fail(MOE_EINVAL, "T=%d exceeds max_tokens", T);
    const bool host = flags & MOE_F_HOST;
    const size_t jb = jobs.size() * sizeof(Job), pb = NP * 4, cb = comb_off.size() * 4, qb = comb_p.size() * 4;
    int s;
    if ((s = c->job_stage.reserve(jb + pb + cb + qb + (pw_host ? pb : 0) + 64))) return s;
    char* hp = (char*)c->job_stage.host;
    memcpy(hp, jobs.data(), jb);
    memcpy(hp + jb, ptok.data(), pb);
    memcpy(hp + jb + pb, comb_off.data(), cb);
    memcpy(hp + jb + pb + cb, comb_p.data(), qb);
    if (jb) CUDA_TRY(cudaMemcpyAsync(c->d_jobs, hp, jb, cudaMemcpyHostToDevice, st));
    if (pb) CUDA_TRY(cudaMemcpyAsync(c->d_ptok, hp + jb, pb, cudaMemcpyHostToDevice, st));
    CUDA_TRY(cudaMemcpyAsync(c->d_comb_off, hp + jb + pb, cb, cudaMemcpyHostToDevice, st));
    if (qb) CUDA_TRY(cudaMemcpyAsync(c->d_comb_p, hp + jb + pb + cb, qb, cudaMemcpyHostToDevice, st));
    if (pb) {
        if (pw_host) {
            memcpy(hp + jb + pb + cb + qb, pw_src, pb);
            CUDA_TRY(cudaMemcpyAsync(c->d_pw, hp + jb + pb + cb + qb, pb, cudaMemcpyHostToDevice, st));
        } else {
            CUDA_TRY(cudaMemcpyAsync(c->d_pw, pw_src, pb, cudaMemcpyDeviceToDevice, st));
        }
    }
    c->job_stage.mark(st);
    const uint16_t* xd = x;
    float* od = out;
    if (host) {
        CUDA_TRY(cudaMemcpyAsync(c->d_hidden, x, (size_t)T * H * 2, cudaMemcpyHostToDevice, st));
        xd = c->d_hidden;
        od = c->d_out;
        if (flags & MOE_F_ACCUMULATE) CUDA_TRY(cudaMemcpyAsync(od, out, (size_t)T * H * 4, cudaMemcpyHostToDevice, st));
    }
    ExpertArgs ea{};
    ea.x = xd;
    ea.T = T;
    ea.H = H;
    ea.F = c->cfg.inter;
    ea.jobs = c->d_jobs;
    ea.n_jobs = nullptr;
    ea.n_jobs_host = (int)jobs.size();
    ea.n_jobs_max = (int)jobs.size();
    int mp = 0;
    for (const Job& j : jobs) mp = std::max(mp, j.n);
    ea.max_pairs = mp;
    ea.ptok = c->d_ptok;
    ea.pw = c->d_pw;
    ea.act = c->d_act;
    ea.y = c->d_y;
    ea.comb_off = c->d_comb_off;
    ea.comb_p = c->d_comb_p;
    ea.out = od;
    ea.accumulate = (flags & MOE_F_ACCUMULATE) ? 1 : 0;
    ea.err = c->d_err;
    int n = 0;
    cudaError_t e = launch_experts(ea, c->sm_count, st, &n, nullptr);
    c->launches += n;
    if (e != cudaSuccess) return fail(MOE_ECUDA, "expert launch: %s", cudaGetErrorString(e));
    if (host) {
        CUDA_TRY(cudaMemcpyAsync(out, od, (size_t)T * H * 4, cudaMemcpyDeviceToHost, st));
        return finish_sync(c, st);
    }
    if (flags & MOE_F_SYNC) return finish_sync(c, st);
    return MOE_OK;
}

int moe_experts(moe_ctx* c, int T, const uint16_t* x, int n_jobs, const uint16_t* const* gu, const uint16_t* const* d,
                const int64_t* tok_off, const int64_t* toks, const float* ws, float* out, int flags, void* stream) {
    if (!c) return fail(MOE_EINVAL, "null context");
    if (T < 0 || n_jobs < 0) return fail(MOE_EINVAL, "negative T or n_jobs");
    if (T > 0 && (!x || !out)) return fail(MOE_EINVAL, "null x/out");
    if (n_jobs > 0 && (!gu || !d || !tok_off || !toks || !ws)) return fail(MOE_EINVAL, "null job arrays");
    DeviceGuard dg(c->dev);
    const int F = c->cfg.inter;
    std::vector<Job> jobs(n_jobs);
    std::vector<int32_t> ptok;
    std::vector<std::vector<int32_t>> per_tok(T);
    if (n_jobs > 0 && tok_off[0] != 0) return fail(MOE_EINVAL, "tok_off[0] must be 0");
    for (int j = 0; j < n_jobs; j++) {
        if (!gu[j] || !d[j]) return fail(MOE_EINVAL, "null weights for job %d", j);
        const int64_t a = tok_off[j], b = tok_off[j + 1];
        if (b < a) return fail(MOE_EINVAL, "tok_off not monotone at job %d", j);
        jobs[j] = Job{ExpDesc{gu[j], d[j], nullptr, kKindBF16, 0}, (int32_t)a, (int32_t)(b - a)};
        for (int64_t i = a; i < b; i++) {
            if (toks[i] < 0 || toks[i] >= T) return fail(MOE_EINVAL, "token %lld of job %d out of range [0,%d)", (long long)toks[i], j, T);
            per_tok[toks[i]].push_back((int32_t)i);
            ptok.push_back((int32_t)toks[i]);
        }
    }
    (void)F;
    std::vector<int32_t> comb_off(T + 1, 0), comb_p;
    for (int t = 0; t < T; t++) {
        comb_off[t + 1] = comb_off[t] + (int32_t)per_tok[t].size();
        comb_p.insert(comb_p.end(), per_tok[t].begin(), per_tok[t].end());
    }
    return run_jobs(c, T, x, jobs, ptok, ws, true, comb_off, comb_p, out, flags, (cudaStream_t)stream);
}

static int single_token_jobs(moe_ctx* c, int E, std::vector<Job>& jobs, std::vector<int32_t>& ptok,
                             std::vector<int32_t>& comb_off, std::vector<int32_t>& comb_p) {
    (void)c;
    jobs.resize(E);
    ptok.assign(E, 0);
    comb_off = {0, E};
    comb_p.resize(E);
    for (int e = 0; e < E; e++) comb_p[e] = e;
    return MOE_OK;
}

int moe_ck_moe3(moe_ctx* c, int E, const uint16_t* const* base, const float* w, const uint16_t* x, float* out, int flags,
                void* stream) {
    if (!c) return fail(MOE_EINVAL, "null context");
    if (E <= 0) return MOE_OK;  // cpu_kern.c:142: no experts, nothing to add
    if (!base || !w || !x || !out) return fail(MOE_EINVAL, "null argument");
    DeviceGuard dg(c->dev);
    const size_t FH = (size_t)c->cfg.inter * c->cfg.hidden;
    std::vector<Job> jobs;
    std::vector<int32_t> ptok, co, cp;
    single_token_jobs(c, E, jobs, ptok, co, cp);
    for (int e = 0; e < E; e++) {
        if (!base[e]) return fail(MOE_EINVAL, "null base[%d]", e);
        jobs[e] = Job{ExpDesc{base[e], base[e] + 2 * FH, nullptr, kKindBF16, 0}, e, 1};
    }
    return run_jobs(c, 1, x, jobs, ptok, w, (flags & MOE_F_HOST) != 0, co, cp, out, flags | MOE_F_ACCUMULATE,
                    (cudaStream_t)stream);
}

int moe_ck_moe_q8w(moe_ctx* c, int E, const int8_t* const* q, const float* const* sc, const float* w, const uint16_t* x,
                   float* out, int flags, void* stream) {
    if (!c) return fail(MOE_EINVAL, "null context");
    if (E <= 0) return MOE_OK;  // cpu_kern.c:307
    if (!q || !sc || !w || !x || !out) return fail(MOE_EINVAL, "null argument");
    DeviceGuard dg(c->dev);
    const size_t FH = (size_t)c->cfg.inter * c->cfg.hidden;
    std::vector<Job> jobs;
    std::vector<int32_t> ptok, co, cp;
    single_token_jobs(c, E, jobs, ptok, co, cp);
    for (int e = 0; e < E; e++) {
        if (!q[e] || !sc[e]) return fail(MOE_EINVAL, "null q/sc[%d]", e);
        jobs[e] = Job{ExpDesc{q[e], q[e] + 2 * FH, sc[e], kKindQ8, 0}, e, 1};
    }
    return run_jobs(c, 1, x, jobs, ptok, w, (flags & MOE_F_HOST) != 0, co, cp, out, flags | MOE_F_ACCUMULATE,
                    (cudaStream_t)stream);
}

int moe_place_expert_q8(moe_ctx* c, const uint16_t* g, const uint16_t* u, const uint16_t* d, int8_t* q, float* sc,
                        int32_t* rs, int flags, void* stream) {
    if (!c) return fail(MOE_EINVAL, "null context");
    if (!g || !u || !d || !q || !sc) return fail(MOE_EINVAL, "null argument");
    DeviceGuard dg(c->dev);
    cudaStream_t st = (cudaStream_t)stream;
    const size_t H = c->cfg.hidden, F = c->cfg.inter, FH = F * H, R = 2 * F + H;
    int n = 0;
    if (!(flags & MOE_F_HOST)) {
        cudaError_t e = launch_quantize_q8(quant_geom_split(g, u, d, (int)H, (int)F, q), (int)H, (int)F, sc, rs, st, &n);
        c->launches += n;
        if (e != cudaSuccess) return fail(MOE_ECUDA, "quantise launch: %s", cudaGetErrorString(e));
        if (flags & MOE_F_SYNC) return finish_sync(c, st);
        return MOE_OK;
    }
    char* tmp = nullptr;
    const size_t bytes = FH * 2 * 3 + 3 * FH + R * 8;
    if (cudaMalloc(&tmp, bytes) != cudaSuccess) {
        cudaGetLastError();
        return fail(MOE_ENOMEM, "quantisation scratch");
    }
    uint16_t* dg_ = (uint16_t*)tmp;
    int8_t* dq = (int8_t*)(tmp + FH * 6);
    float* dsc = (float*)(tmp + FH * 6 + 3 * FH);
    int32_t* drs = (int32_t*)(tmp + FH * 6 + 3 * FH + R * 4);
    cudaError_t e = cudaMemcpyAsync(dg_, g, FH * 2, cudaMemcpyHostToDevice, st);
    if (e == cudaSuccess) e = cudaMemcpyAsync(dg_ + FH, u, FH * 2, cudaMemcpyHostToDevice, st);
    if (e == cudaSuccess) e = cudaMemcpyAsync(dg_ + 2 * FH, d, FH * 2, cudaMemcpyHostToDevice, st);
    if (e == cudaSuccess)
        e = launch_quantize_q8(quant_geom_split(dg_, dg_ + FH, dg_ + 2 * FH, (int)H, (int)F, dq), (int)H, (int)F, dsc,
                               drs, st, &n);
    c->launches += n;
    if (e == cudaSuccess) e = cudaMemcpyAsync(q, dq, 3 * FH, cudaMemcpyDeviceToHost, st);
    if (e == cudaSuccess) e = cudaMemcpyAsync(sc, dsc, R * 4, cudaMemcpyDeviceToHost, st);
    if (e == cudaSuccess && rs) e = cudaMemcpyAsync(rs, drs, R * 4, cudaMemcpyDeviceToHost, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    cudaFree(tmp);
    if (e != cudaSuccess) return fail(MOE_ECUDA, "quantise: %s", cudaGetErrorString(e));
    return MOE_OK;
}

// ---- expert-parallel peer exchange ----
namespace {
constexpr uint32_t kEpMagic = 0x4D4F4550u;  // "MOEP"
struct EpBlob {
    uint32_t magic, sm_count, world, rank;
    cudaIpcMemHandle_t x;
};
}  // namespace

int moe_ep_export(moe_ctx* c, void* out, int cap) {
    if (!c) return fail(MOE_EINVAL, "null context");
    if (c->cfg.ep_world < 2 || c->cfg.ep_world > kEpMaxWorld)
        return fail(MOE_EINVAL, "peer exchange needs 2..%d ranks (ep_world = %d)", kEpMaxWorld, c->cfg.ep_world);
    static_assert(sizeof(EpBlob) <= MOE_EP_RECORD_BYTES, "record size");
    if (!out || cap < MOE_EP_RECORD_BYTES) return fail(MOE_EINVAL, "handle buffer needs %d bytes", MOE_EP_RECORD_BYTES);
    DeviceGuard dg(c->dev);
    const int W = c->cfg.ep_world, H = c->cfg.hidden;
    int st = MOE_OK;
    if (!c->d_xbuf) {
        // a slot holds a whole call of up to max_tokens tokens (2048 at most), so a call exchanges once
        c->ep_tcap = std::max(kEpMaxT, std::min(kEpMaxTcap, c->cfg.max_tokens));
        if (!st) st = dalloc(&c->d_xbuf, (size_t)2 * W * c->ep_tcap * H);
        if (!st) st = dalloc(&c->d_peer_x, (size_t)kEpMaxWorld);
        if (!st) st = dalloc(&c->d_xpart, (size_t)kEpMaxT * H * ((c->cfg.max_tokens + kEpMaxT - 1) / kEpMaxT));
        if (st) return st;
    }
    // No word may carry an epoch of an earlier attachment (epochs restart at 1 on import).  Every rank
    // exports before the records are exchanged and imports after, so clearing here precedes every
    // rank's first call.
    CUDA_TRY(cudaMemset(c->d_xbuf, 0, sizeof(uint64_t) * 2 * (size_t)W * c->ep_tcap * H));
    CUDA_TRY(cudaDeviceSynchronize());
    EpBlob b{};
    b.magic = kEpMagic;
    b.sm_count = (uint32_t)c->sm_count;
    b.world = (uint32_t)W;
    b.rank = (uint32_t)c->cfg.ep_rank;
    CUDA_TRY(cudaIpcGetMemHandle(&b.x, c->d_xbuf));
    memset(out, 0, MOE_EP_RECORD_BYTES);
    memcpy(out, &b, sizeof(b));
    return MOE_OK;
}

int moe_ep_import(moe_ctx* c, const void* blobs, int world) {
    if (!c || !blobs) return fail(MOE_EINVAL, "null argument");
    if (!c->d_xbuf) return fail(MOE_ESTATE, "moe_ep_export must come first");
    if (world != c->cfg.ep_world) return fail(MOE_EINVAL, "world %d != ep_world %d", world, c->cfg.ep_world);
    DeviceGuard dg(c->dev);
    std::vector<uint64_t*> px(kEpMaxWorld, nullptr);
    for (int r = 0; r < world; r++) {
        EpBlob b;
        memcpy(&b, (const char*)blobs + (size_t)r * MOE_EP_RECORD_BYTES, sizeof(b));
        if (b.magic != kEpMagic || (int)b.world != world || (int)b.rank != r)
            return fail(MOE_EINVAL, "peer handle %d is not rank %d of %d", r, r, world);
        if ((int)b.sm_count != c->sm_count)
            return fail(MOE_EINVAL, "rank %d has %u SMs, this GPU %d (the output slicing must agree)", r, b.sm_count, c->sm_count);
        if (r == c->cfg.ep_rank) {
            px[r] = c->d_xbuf;
            continue;
        }
        void* x = nullptr;
        cudaError_t e = cudaIpcOpenMemHandle(&x, b.x, cudaIpcMemLazyEnablePeerAccess);
        if (e != cudaSuccess) {
            cudaGetLastError();
            return fail(MOE_ECOMM, "opening rank %d's exchange buffer: %s", r, cudaGetErrorString(e));
        }
        c->ipc_opened.push_back(x);
        px[r] = static_cast<uint64_t*>(x);
    }
    CUDA_TRY(cudaMemcpy(c->d_peer_x, px.data(), sizeof(uint64_t*) * kEpMaxWorld, cudaMemcpyHostToDevice));
    c->ep_attached = true;
    c->xepoch = 0;
    return MOE_OK;
}

// ---------------- MoE-block calls: the steps either side of the routed experts ----------------

static int ensure_shared(moe_ctx* c) {
    if (c->shared) return MOE_OK;
    moe_config k = c->cfg;
    if (c->shared_inter > 0) k.inter = c->shared_inter;  // a unit-sharded context still holds the whole shared expert
    k.n_experts = 1;  // softmax over one zero logit: weight exactly 1 for every token
    k.top_k = 1;
    k.scoring = MOE_SCORING_SOFTMAX;
    k.ep_rank = 0;
    k.ep_world = 1;   // replicated on every expert-parallel rank: identical y everywhere
    k.shard_map = nullptr;
    int st = moe_create(&k, &c->shared);
    if (st) return st;
    moe_ctx* s = c->shared;
    s->fused = c->fused;
    s->timeout_ns = c->timeout_ns;
    s->prefill = c->prefill;
    s->prefill_min_t = c->prefill_min_t;
    s->prefill_tc = c->prefill_tc;
    s->ns_cap = c->ns_cap;
    s->stage_target = c->stage_target;
    s->q8_cost_pm = c->q8_cost_pm;
    s->reducers = c->reducers;
    s->use_planner = c->use_planner;
    s->late_bytes = c->late_bytes;
    const size_t NT = c->cfg.max_tokens, H = c->cfg.hidden, E = c->cfg.n_experts;
    if (!st) st = dalloc(&c->d_blk_zero, NT);
    if (!st) st = dalloc(&c->d_blk_logits, NT * E);
    if (!st) st = dalloc(&c->d_blk_shared, NT * H);
    if (!st) st = dalloc(&c->d_blk_moe, NT * H);
    if (!st) st = dalloc(&c->d_blk_y, NT * H);
    if (!st) st = dalloc(&c->d_blk_io, 3 * NT * H);
    if (!st) st = dalloc(&c->d_blk_extra, NT * H);
    if (!st && cudaMemset(c->d_blk_zero, 0, NT * sizeof(float)) != cudaSuccess) st = fail(MOE_ECUDA, "memset");
    if (!st) c->d_router.assign(c->cfg.n_layers, nullptr);
    return st;
}

int moe_load_shared(moe_ctx* c, int layer, const uint16_t* gate, const uint16_t* up, const uint16_t* down,
                    const uint16_t* router, int flags) {
    if (!c) return fail(MOE_EINVAL, "null context");
    if (layer < 0 || layer >= c->cfg.n_layers) return fail(MOE_EINVAL, "layer %d out of range [0,%d)", layer, c->cfg.n_layers);
    if (!gate != !up || !gate != !down) return fail(MOE_EINVAL, "the shared expert needs gate, up and down together");
    DeviceGuard dg(c->dev);
    int st = ensure_shared(c);
    if (st) return st;
    if (gate && (st = moe_load_expert_bf16(c->shared, layer, 0, gate, up, down, flags))) return st;
    if (router) {
        const size_t n = (size_t)c->cfg.n_experts * c->cfg.hidden;
        if (!c->d_router[layer] && (st = dalloc(&c->d_router[layer], n))) return st;
        CUDA_TRY(cudaMemcpy(c->d_router[layer], router, n * 2,
                            (flags & MOE_F_HOST) ? cudaMemcpyHostToDevice : cudaMemcpyDeviceToDevice));
    }
    return MOE_OK;
}

static int block_checks(moe_ctx* c, int layer, int T) {
    if (!c) return fail(MOE_EINVAL, "null context");
    if (layer < 0 || layer >= c->cfg.n_layers) return fail(MOE_EINVAL, "layer %d out of range [0,%d)", layer, c->cfg.n_layers);
    if (T < 0 || T > c->cfg.max_tokens) return fail(MOE_EINVAL, "T=%d not in [0,%d]", T, c->cfg.max_tokens);
    return MOE_OK;
}

static bool aligned16(const void* p) { return ((uintptr_t)p & 15u) == 0; }

// Both contexts' latched device status (the shared context's calls run without MOE_F_SYNC).
static int block_sync(moe_ctx* c, cudaStream_t st) {
    const int a = finish_sync(c, st);
    const int b = c->shared ? finish_sync(c->shared, st) : MOE_OK;
    return a ? a : b;
}

int moe_shared_router(moe_ctx* c, int layer, int T, const uint16_t* h2, const uint16_t* x2, uint16_t* y_out,
                      float* logits, int flags, void* stream) {
    int st = block_checks(c, layer, T);
    if (st) return st;
    if (flags & MOE_F_HOST) return fail(MOE_EINVAL, "moe_shared_router takes device pointers");
    if (T == 0) return MOE_OK;
    if (!h2 || (y_out && !x2)) return fail(MOE_EINVAL, "null h2 / x2");
    if (!aligned16(h2) || !aligned16(x2) || !aligned16(y_out)) return fail(MOE_EINVAL, "buffers must be 16-byte aligned");
    DeviceGuard dg(c->dev);
    cudaStream_t s = (cudaStream_t)stream;
    const int H = c->cfg.hidden, E = c->cfg.n_experts;
    if (logits) {
        if (c->d_router.empty() || !c->d_router[layer]) return fail(MOE_ESTATE, "no router weights loaded for layer %d", layer);
        CUDA_TRY(launch_router_gemv(c->d_router[layer], h2, T, E, H, logits, s));
        c->launches++;
    }
    if (y_out) {
        if (!c->shared || moe_expert_kind(c->shared, layer, 0) != kKindBF16)
            return fail(MOE_ESTATE, "no shared expert loaded for layer %d", layer);
        if ((st = moe_forward(c->shared, layer, T, h2, c->d_blk_zero, c->d_blk_shared, nullptr, nullptr, 0, s))) return st;
        CUDA_TRY(launch_residual(nullptr, x2, c->d_blk_shared, nullptr, nullptr, (long)T * H, y_out, nullptr, c->sm_count, s));
        c->launches++;
    }
    return (flags & MOE_F_SYNC) ? block_sync(c, s) : MOE_OK;
}

int moe_combine_residual(moe_ctx* c, int T, const uint16_t* y, const float* extra, const float* moe_out,
                         uint16_t* x_next, int flags, void* stream) {
    if (!c) return fail(MOE_EINVAL, "null context");
    if (T < 0 || T > c->cfg.max_tokens) return fail(MOE_EINVAL, "T=%d not in [0,%d]", T, c->cfg.max_tokens);
    if (flags & MOE_F_HOST) return fail(MOE_EINVAL, "moe_combine_residual takes device pointers");
    if (T == 0) return MOE_OK;
    if (!y || !moe_out || !x_next) return fail(MOE_EINVAL, "null y / moe_out / x_next");
    if (!aligned16(y) || !aligned16(extra) || !aligned16(moe_out) || !aligned16(x_next))
        return fail(MOE_EINVAL, "buffers must be 16-byte aligned");
    DeviceGuard dg(c->dev);
    cudaStream_t s = (cudaStream_t)stream;
    CUDA_TRY(launch_residual(y, nullptr, nullptr, extra, moe_out, (long)T * c->cfg.hidden, nullptr, x_next, c->sm_count, s));
    c->launches++;
    return (flags & MOE_F_SYNC) ? finish_sync(c, s) : MOE_OK;
}

int moe_block_forward(moe_ctx* c, int layer, int T, const uint16_t* h2, const uint16_t* x2, const float* extra,
                      uint16_t* x_next, uint16_t* y_out, float* logits_out, int flags, void* stream) {
    int st = block_checks(c, layer, T);
    if (st) return st;
    if (T > 0 && (!h2 || !x2 || !x_next)) return fail(MOE_EINVAL, "null h2 / x2 / x_next");
    if (c->cfg.ep_world > 1 && !c->ep_attached)
        return fail(MOE_ESTATE, "expert-parallel block calls need the peer exchange (moe_ep_import)");
    if (!c->shared || moe_expert_kind(c->shared, layer, 0) != kKindBF16 || !c->d_router[layer])
        return fail(MOE_ESTATE, "layer %d needs its shared expert and router weights (moe_load_shared)", layer);
    const bool host = flags & MOE_F_HOST;
    if (!host && (!aligned16(h2) || !aligned16(x2) || !aligned16(extra) || !aligned16(x_next) || !aligned16(y_out) ||
                  !aligned16(logits_out)))
        return fail(MOE_EINVAL, "buffers must be 16-byte aligned");
    if (T == 0) return MOE_OK;
    DeviceGuard dg(c->dev);
    cudaStream_t s = (cudaStream_t)stream;
    const int H = c->cfg.hidden, E = c->cfg.n_experts;
    const size_t NT = c->cfg.max_tokens, n = (size_t)T * H;
    const uint16_t* dh = h2;
    const uint16_t* dx = x2;
    const float* de = extra;
    uint16_t* dn = x_next;
    if (host) {  // inputs to the device, outputs back, one synchronisation at the end
        uint16_t* io = c->d_blk_io;
        CUDA_TRY(cudaMemcpyAsync(io, h2, n * 2, cudaMemcpyHostToDevice, s));
        CUDA_TRY(cudaMemcpyAsync(io + NT * H, x2, n * 2, cudaMemcpyHostToDevice, s));
        if (extra) CUDA_TRY(cudaMemcpyAsync(c->d_blk_extra, extra, n * 4, cudaMemcpyHostToDevice, s));
        dh = io;
        dx = io + NT * H;
        de = extra ? c->d_blk_extra : nullptr;
        dn = io + 2 * NT * H;
    }
    float* lg = (logits_out && !host) ? logits_out : c->d_blk_logits;
    uint16_t* y = (y_out && !host) ? y_out : c->d_blk_y;
    const int K = c->cfg.top_k;
    CUDA_TRY(launch_router_gemv(c->d_router[layer], dh, T, E, H, lg, s));  // router-logit producer
    c->launches++;
    DecodeArgs da{};
    size_t dsmem = 0;
    // fused: the shared expert is one more job of the routed unit stream, and the decode kernel's
    // reduction writes y and x_next (one plan, one decode grid)
    const bool fused = c->cfg.ep_world == 1 && !c->prof_on && c->shared->cfg.inter == c->cfg.inter &&
                       !prefill_applies(c, layer, T) &&
                       T * (K + 1) <= kDecodeMaxPairs &&
                       c->sm_count - 1 + T * (K + 1) <= kMaxSegTotal && prepare_fused(c, T, 0, da, &dsmem);
    if (fused) {
        da.x = dh;
        da.out = c->d_blk_moe;
        da.block = 1;
        da.x2 = dx;
        da.extra = de;
        da.x_next = dn;
        da.y_out = y;
        // the logits come from the GEMV just launched: a planner could never get ahead, only add a hop
        if ((st = launch_fused(c, layer, lg, da, dsmem, s, nullptr, nullptr, c->shared->d_desc + layer, false))) return st;
    } else {
        // routed experts (their plan runs as soon as the logits exist), shared expert (its plan
        // overlaps the routed stream), then one element-wise pass for y and x_next
        if ((st = moe_forward(c, layer, T, dh, lg, c->d_blk_moe, nullptr, nullptr, 0, s))) return st;
        if ((st = moe_forward(c->shared, layer, T, dh, c->d_blk_zero, c->d_blk_shared, nullptr, nullptr, 0, s))) return st;
        CUDA_TRY(launch_residual(nullptr, dx, c->d_blk_shared, de, c->d_blk_moe, (long)n, y, dn, c->sm_count, s));
        c->launches++;
    }
    if (host) {
        CUDA_TRY(cudaMemcpyAsync(x_next, dn, n * 2, cudaMemcpyDeviceToHost, s));
        if (y_out) CUDA_TRY(cudaMemcpyAsync(y_out, y, n * 2, cudaMemcpyDeviceToHost, s));
        if (logits_out) CUDA_TRY(cudaMemcpyAsync(logits_out, lg, (size_t)T * E * 4, cudaMemcpyDeviceToHost, s));
    }
    return (host || (flags & MOE_F_SYNC)) ? block_sync(c, s) : MOE_OK;
}

int moe_router_exp(const float* x, float* y, int64_t n, void* stream) {
    if (n < 0) return fail(MOE_EINVAL, "negative n");
    if (n == 0) return MOE_OK;
    if (!x || !y) return fail(MOE_EINVAL, "null x / y");
    int dev = 0, sms = 0;
    CUDA_TRY(cudaGetDevice(&dev));
    CUDA_TRY(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    CUDA_TRY(launch_router_exp(x, y, (long long)n, sms, (cudaStream_t)stream));
    return MOE_OK;
}

int moe_status(moe_ctx* c, void* stream) {
    if (!c) return fail(MOE_EINVAL, "null context");
    DeviceGuard dg(c->dev);
    return finish_sync(c, (cudaStream_t)stream);
}

int64_t moe_launch_count(moe_ctx* c) { return c ? c->launches + (c->shared ? c->shared->launches : 0) : -1; }

static int set_option_one(moe_ctx* c, int option, int64_t value);

int moe_set_option(moe_ctx* c, int option, int64_t value) {
    if (!c) return fail(MOE_EINVAL, "null context");
    const int st = set_option_one(c, option, value);
    // the shared-expert context follows the path options (not the test hook, not instrumentation)
    if (st == MOE_OK && c->shared && option != MOE_OPT_INJECT_WAIT_TIMEOUT && option != MOE_OPT_TIMELINE &&
        option != MOE_OPT_SHARED_INTER)
        return set_option_one(c->shared, option, value);
    return st;
}

static int set_option_one(moe_ctx* c, int option, int64_t value) {
    switch (option) {
        case MOE_OPT_FUSED_DECODE:
            c->fused = value != 0;
            return MOE_OK;
        case MOE_OPT_WAIT_TIMEOUT_US:
            if (value < 1000 || value > 60000000) return fail(MOE_EINVAL, "wait timeout %lld us not in [1e3, 6e7]", (long long)value);
            c->timeout_ns = (uint64_t)value * 1000ull;
            return MOE_OK;
        case MOE_OPT_INJECT_WAIT_TIMEOUT:
            c->inject_timeout = value != 0;
            return MOE_OK;
        case MOE_OPT_RING_STAGES:
            if (value < 0 || value > 16) return fail(MOE_EINVAL, "ring stages %lld not in [0,16]", (long long)value);
            c->ns_cap = (int)value;
            return MOE_OK;
        case MOE_OPT_PREFILL_MIN_T:
            if (value < 0 || value > kMaxTokens) return fail(MOE_EINVAL, "prefill batch %lld not in [0,%d]", (long long)value, kMaxTokens);
            c->prefill = value > 0;
            c->prefill_min_t = (int)std::max<int64_t>(1, value);
            return MOE_OK;
        case MOE_OPT_PREFILL_TC:
            c->prefill_tc = value != 0;
            return MOE_OK;
        case MOE_OPT_LAYER_SLOTS:
            if (value < 0 || value > c->cfg.n_experts)
                return fail(MOE_EINVAL, "layer slots %lld not in [0,%d]", (long long)value, c->cfg.n_experts);
            c->slot_budget = (int)value;
            return MOE_OK;
        case MOE_OPT_SHARED_INTER: {
            const int64_t v = value ? value : c->cfg.inter;
            if (v < 64 || v % 64 || v > 2048) return fail(MOE_EINVAL, "shared inter %lld must be a multiple of 64 in [64, 2048]", (long long)v);
            if (c->shared && c->shared->cfg.inter != v)
                return fail(MOE_ESTATE, "the shared expert is already loaded with inter %d", c->shared->cfg.inter);
            c->shared_inter = (int)v;
            return MOE_OK;
        }
        case MOE_OPT_STAGE_BYTES:
            if (value < 0 || value > 196608) return fail(MOE_EINVAL, "stage bytes %lld not in [0,196608]", (long long)value);
            c->stage_target = (uint32_t)value;
            return MOE_OK;
        case MOE_OPT_Q8_UNIT_COST:
            if (value != 0 && (value < 500 || value > 4000))
                return fail(MOE_EINVAL, "int8 unit cost %lld not 0 or in [500,4000] per mille", (long long)value);
            c->q8_cost_pm = (int)value;
            return MOE_OK;
        case MOE_OPT_PLANNER:
            c->use_planner = value != 0;
            return MOE_OK;
        case MOE_OPT_REDUCERS:
            if (value < 0 || value > kPlanMaxGrid) return fail(MOE_EINVAL, "reducers %lld not in [0,%d]", (long long)value, kPlanMaxGrid);
            c->reducers = (int)value;
            return MOE_OK;
        case MOE_OPT_LATE_BYTES:
            if (value < 0 || value > (64ll << 20)) return fail(MOE_EINVAL, "late bytes %lld not in [0, 64 MiB]", (long long)value);
            c->late_bytes = value;
            return MOE_OK;
        case MOE_OPT_TIMELINE: {
            DeviceGuard dg(c->dev);
            if (value && !c->d_timeline) {
                int st = dalloc(&c->d_timeline, (size_t)c->sm_count * kTimelineSlots + 3 * kStageLogMax);
                if (st) return st;
                CUDA_TRY(cudaMemset(c->d_timeline, 0, sizeof(uint64_t) * ((size_t)c->sm_count * kTimelineSlots + 3 * kStageLogMax)));
            } else if (!value && c->d_timeline) {
                cudaDeviceSynchronize();
                cudaFree(c->d_timeline);
                c->d_timeline = nullptr;
            }
            return MOE_OK;
        }
        default:
            return fail(MOE_EINVAL, "unknown option %d", option);
    }
}

int moe_timeline_read(moe_ctx* c, uint64_t* out, int cap) {
    if (!c || !out) return fail(MOE_EINVAL, "bad argument");
    if (!c->d_timeline) return fail(MOE_ESTATE, "timeline recording is off (MOE_OPT_TIMELINE)");
    DeviceGuard dg(c->dev);
    const int n = std::min(cap, c->sm_count * kTimelineSlots + 3 * kStageLogMax);
    CUDA_TRY(cudaDeviceSynchronize());
    CUDA_TRY(cudaMemcpy(out, c->d_timeline, sizeof(uint64_t) * n, cudaMemcpyDeviceToHost));
    return MOE_OK;
}

int moe_profile(moe_ctx* c, int enable) {
    if (!c) return fail(MOE_EINVAL, "null context");
    c->prof_on = enable != 0;
    c->prof_calls = 0;
    return MOE_OK;
}

int moe_profile_read(moe_ctx* c, double* stage_ms, int n_stages, int64_t* n_calls) {
    if (!c || !stage_ms || n_stages < 1) return fail(MOE_EINVAL, "bad argument");
    DeviceGuard dg(c->dev);
    for (int i = 0; i < n_stages; i++) stage_ms[i] = 0.0;
    for (size_t k = 0; k < c->prof_calls; k++) {
        cudaEvent_t* m = &c->prof_ev[k * kProfMarks];
        CUDA_TRY(cudaEventSynchronize(m[kProfMarks - 1]));
        for (int i = 0; i < n_stages && i < kProfMarks - 1; i++) {
            float ms = 0.f;
            CUDA_TRY(cudaEventElapsedTime(&ms, m[i], m[i + 1]));
            stage_ms[i] += ms;
        }
    }
    if (n_calls) *n_calls = (int64_t)c->prof_calls;
    c->prof_calls = 0;
    return MOE_OK;
}

}  // extern "C"
