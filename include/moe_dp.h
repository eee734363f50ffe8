/*
 * moe_dp.h -- C ABI of the B200 routed-expert MoE data plane (libmoe_dp.so).
 *
 * One call per layer per step takes hidden states, router logits and a layer id and returns the
 * combined routed-expert output, the surface of npu-offload's
 *   Model::moe_phase(l, logits, h2)          track2_opt/solar_engine/src/main.rs:149-209
 *   Runtime._moe(l, h2, Tb, T)               solar_hybrid/runtime.py:338-423
 * It also exports the reference's lower-level CPU-kernel surfaces so a caller of those can switch
 * without reshaping its data:
 *   cpu_moe(x, gus, ds, toks, ws)            solar_hybrid/cpu_moe.cpp:38-96   -> moe_experts()
 *   ck_moe3(E, base, w, x, out, H, F)        track2_opt/solar_engine/csrc/cpu_kern.c:141-172 -> moe_ck_moe3()
 *   ck_moe_q8w(E, q, sc, w, x, out, H, F)    cpu_kern.c:306-333               -> moe_ck_moe_q8w()
 *   ck_place_expert_q8(g, u, d, q, sc, rs)   cpu_kern.c:227-241               -> moe_place_expert_q8()
 *
 * Conventions
 *  - bf16 values are raw uint16_t bits; all matrices are row-major.
 *  - Every entry point returns 0 (MOE_OK) or a positive MOE_E* status; moe_last_error() gives the
 *    calling thread's message for its last failing call.  Unlike the reference's void C kernels,
 *    nothing aborts the process.
 *  - Pointers are device pointers unless the call takes MOE_F_HOST, in which case hidden / logits /
 *    x / out / topk / w pointers are host memory and the call returns with the result in place.
 *    Pinned (cudaMallocHost / cudaHostAlloc) buffers are used directly: on the fused decode path the
 *    kernels read pinned logits and write a 16-byte-aligned pinned output over the bus; any other
 *    host buffer goes through the library's own pinned staging.
 *  - Device-pointer calls are asynchronous on `stream` (a cudaStream_t; NULL = legacy default
 *    stream).  Device-side errors (non-finite router input, a bounded wait that gave up) are
 *    latched in the context and returned by the next MOE_F_SYNC call or by moe_status().
 *  - One context per GPU per process.  Calls on one context must be serialised by the caller
 *    (like the reference engine's single caller thread, main.rs:149); distinct contexts are
 *    independent.
 */
#ifndef MOE_DP_H
#define MOE_DP_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define MOE_API __attribute__((visibility("default")))
#else
#define MOE_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define MOE_DP_ABI_VERSION 1

/* status codes */
#define MOE_OK 0
#define MOE_EINVAL 1      /* bad argument: null pointer, layer/expert/T out of range, shape limits */
#define MOE_ENONFINITE 2  /* a router probability was NaN (NaN or +inf logit, or all -inf): the
                             reference panics here (partial_cmp().unwrap(), host.rs.tpl:259) */
#define MOE_ECUDA 3       /* CUDA runtime error (message has the CUDA error string) */
#define MOE_ENOMEM 4      /* device or pinned-host allocation failed */
#define MOE_ESTATE 5      /* context state: routed expert not loaded, expert not local to this rank */
#define MOE_ETIMEOUT 6    /* a device-side bounded wait gave up (the kernel returned, nothing hung) */
#define MOE_ECOMM 7       /* expert-parallel exchange failed */

/* router scoring */
#define MOE_SCORING_SOFTMAX 0 /* host.rs.tpl:247-268: softmax, top-k by p (ties -> lower index), w = p/sum p */
#define MOE_SCORING_SIGMOID 1 /* host.rs:119-128: sigmoid + correction bias, w = s/(sum s + 1e-20) */

/* flags */
#define MOE_F_HOST 0x1       /* data pointers are host memory; call is synchronous */
#define MOE_F_ACCUMULATE 0x2 /* out += result (ck_moe3 semantics, cpu_kern.c:141) instead of out = result */
#define MOE_F_SYNC 0x4       /* synchronise `stream` before returning and report device-side status */

/* expert storage kinds */
#define MOE_KIND_NONE 0
#define MOE_KIND_BF16 1
#define MOE_KIND_Q8 2

typedef struct moe_config {
    int32_t hidden;           /* H (multiple of 64, <= 16384; the fused decode path takes H <= 8192) */
    int32_t inter;            /* F (multiple of 64) */
    int32_t n_experts;        /* E, 1..256 */
    int32_t top_k;            /* K, 1..16, <= E */
    int32_t n_layers;         /* layers held by this context */
    int32_t max_tokens;       /* largest T per call, 1..4096 */
    int32_t scoring;          /* MOE_SCORING_* */
    int32_t device;           /* CUDA device ordinal */
    int32_t ep_rank;          /* expert-parallel rank of this context (0 when unsharded) */
    int32_t ep_world;         /* expert-parallel world size (1 when unsharded) */
    const int32_t* shard_map; /* optional host array [n_layers * n_experts]: owner rank of each
                                 (layer, expert); NULL with ep_world == 1 means all local */
} moe_config;

typedef struct moe_ctx moe_ctx;

MOE_API int moe_abi_version(void);
MOE_API const char* moe_last_error(void);

/* Create / destroy a context on cfg->device.  Replaces the engine start-up that permutes and
 * uploads expert tables (track2_opt/solar_engine/src/chip.rs:208-233). */
MOE_API int moe_create(const moe_config* cfg, moe_ctx** out);
MOE_API int moe_destroy(moe_ctx* ctx);

/* Load one bf16 expert: gate [F,H], up [F,H], down [H,F] -- the tensors of
 * Weights::expert (track2_opt/solar_engine/src/host.rs:112-116).  The library stores them in its
 * own HBM table (one contiguous unit per intermediate index f: gate row f, up row f, down column f);
 * the caller keeps ownership of its buffers.  flags: MOE_F_HOST if host pointers. */
MOE_API int moe_load_expert_bf16(moe_ctx* ctx, int layer, int expert, const uint16_t* gate, const uint16_t* up,
                         const uint16_t* down, int flags);

/* Load one int8 weight-only expert in the ck_place_expert_q8 layout (cpu_kern.c:227-241):
 * q = [2F rows of H (gate rows, then up rows)][H rows of F (down)], scales = [2F + H] fp32. */
MOE_API int moe_load_expert_q8(moe_ctx* ctx, int layer, int expert, const int8_t* q, const float* scales, int flags);

/* Re-store an already loaded bf16 expert as int8 weight-only, quantising on the GPU with the
 * reference's per-row rule (quant_row, cpu_kern.c:218-224) -- bit-identical tables. */
MOE_API int moe_quantize_expert_q8(moe_ctx* ctx, int layer, int expert);

/* Kind (MOE_KIND_*) of a stored expert, or -1 on bad arguments. */
MOE_API int moe_expert_kind(moe_ctx* ctx, int layer, int expert);

/* HBM-hot / host-cold expert tier (the reference's swap of a device table slot,
 * track2_opt/solar_engine/src/experts_b.rs:162-186, driven by the LFU-decay `follow` of
 * solar_hybrid/runtime.py:287-311).  With MOE_OPT_LAYER_SLOTS = S set before a layer's first load,
 * that layer's HBM table holds S experts; a load takes a free slot, and moe_evict_expert frees one
 * (the expert then reads as MOE_KIND_NONE and routing a token to it makes moe_forward report
 * MOE_ESTATE).  Evicting or loading must not overlap a forward call of the same layer on the GPU:
 * loads run on the legacy default stream; callers on other streams synchronise first.
 * npu_offload_b200.cache.ExpertCache keeps the host copies and makes the choices. */
MOE_API int moe_evict_expert(moe_ctx* ctx, int layer, int expert);

/* Sigmoid-scoring correction bias for a layer ([E] fp32; e_score_correction_bias, host.rs:120). */
MOE_API int moe_set_bias(moe_ctx* ctx, int layer, const float* bias, int flags);

/* The hot path.  hidden [T,H] bf16, router_logits [T,E] fp32 -> out [T,H] fp32
 *   out[t] = sum_k w[t,k] * expert_{idx[t,k]}(hidden[t])
 * with idx/w from the configured router.  topk_idx [T,K] int32 and topk_w [T,K] fp32 are
 * optional outputs (NULL to skip).  Replaces moe_phase's route + dispatch + cold CPU experts +
 * combine (main.rs:150-207) and Runtime._moe (runtime.py:340-423).  Under expert parallelism
 * (ep_world > 1) every rank passes the same hidden/logits and receives the full combined output. */
MOE_API int moe_forward(moe_ctx* ctx, int layer, int T, const uint16_t* hidden, const float* router_logits, float* out,
                int32_t* topk_idx, float* topk_w, int flags, void* stream);

/* n moe_forward calls enqueued by one call, in order: call i is layer layers[i] on hidden[i],
 * router_logits[i] -> out[i] (device buffers, T tokens each; MOE_F_ACCUMULATE applies to every call,
 * MOE_F_SYNC synchronises once after the last).  For a caller that issues several layers' MoE work
 * back to back -- the engine's layer loop issuing moe_phase per layer (main.rs:267-289, moe_phase
 * main.rs:149-209) with its inputs ready -- it keeps the caller's language off the per-layer path.
 * Stops at the first failing call and returns its status. */
MOE_API int moe_forward_layers(moe_ctx* ctx, int n, const int32_t* layers, int T, const uint16_t* const* hidden,
                               const float* const* router_logits, float* const* out, int flags, void* stream);

/* Router + token permutation alone (device pointers unless MOE_F_HOST; bias may be NULL):
 *   topk_idx/topk_w [T,K]; counts [E]; offsets [E+1] (expert-id order); perm [T*K] pair ids
 *   t*K+k grouped by expert, tokens ascending (runtime.py:343-347); job_order [E] experts in
 *   first-appearance order (the cpu_moe job list, runtime.py:352-354); n_jobs [1]. */
MOE_API int moe_route(moe_ctx* ctx, int T, const float* router_logits, const float* bias, int32_t* topk_idx, float* topk_w,
              int32_t* counts, int32_t* offsets, int32_t* perm, int32_t* job_order, int32_t* n_jobs, int flags,
              void* stream);

/* cpu_moe surface (cpu_moe.cpp:38-39) with caller-owned expert weights in device memory:
 *   x [T,H] bf16; job j uses gu[j] = [2F,H] (gate rows then up rows) and d[j] = [H,F];
 *   its tokens are toks[tok_off[j] .. tok_off[j+1]) with weights ws[...] (host arrays).
 * out [T,H] fp32 = sum over jobs (zero-filled first unless MOE_F_ACCUMULATE).  n_jobs == 0
 * gives zeros, like the reference. */
MOE_API int moe_experts(moe_ctx* ctx, int T, const uint16_t* x, int n_jobs, const uint16_t* const* gu,
                const uint16_t* const* d, const int64_t* tok_off, const int64_t* toks, const float* ws, float* out,
                int flags, void* stream);

/* ck_moe3 surface (cpu_kern.c:141-172): one token, base[e] = device pointer to an expert in the
 * [g F*H][u F*H][d H*F] layout, w [E]; out [H] += sum_e w[e] * expert_e(x).  Always accumulates. */
MOE_API int moe_ck_moe3(moe_ctx* ctx, int E, const uint16_t* const* base, const float* w, const uint16_t* x, float* out,
                int flags, void* stream);

/* ck_moe_q8w surface (cpu_kern.c:306-333): int8 weight-only experts q[e] / sc[e] (device
 * pointers, ck_place_expert_q8 layout), one token, out [H] += sum_e w[e] * expert_e(x). */
MOE_API int moe_ck_moe_q8w(moe_ctx* ctx, int E, const int8_t* const* q, const float* const* sc, const float* w,
                   const uint16_t* x, float* out, int flags, void* stream);

/* ck_place_expert_q8 (cpu_kern.c:227-241) on the GPU: g/u [F,H], d [H,F] bf16 -> q, sc [2F+H],
 * rs [2F+H] row sums (rs may be NULL).  Device pointers unless MOE_F_HOST. */
MOE_API int moe_place_expert_q8(moe_ctx* ctx, const uint16_t* g, const uint16_t* u, const uint16_t* d, int8_t* q, float* sc,
                        int32_t* rs, int flags, void* stream);

/* ---- The steps either side of the routed experts in one Solar MoE block
 * (track2_opt/solar_engine/src/layer.rs:1-6: combine -> attention -> shared expert + router). ----
 *
 * moe_load_shared: layer `layer`'s shared expert (gate [Fs*H], up [Fs*H] rows, down [H*Fs] row-major,
 * the routed experts' layout; Fs = MOE_OPT_SHARED_INTER, by default the context's F) and router
 * weights Wr [E*H] row-major, bf16.  Either part may be NULL
 * (then left as loaded before).  Copied; host pointers with MOE_F_HOST.  Replaces the host-side
 * placement of dense/shared.rs's WG / WD / WR tables (shared.rs:5-31).
 *
 * moe_shared_router: the router-logit producer + shared expert, dense/shared.rs:1-3, :192-210
 * (`shared_router`), T tokens, device pointers:
 *   logits [T,E] f32  = h2 . Wr^T (fp32 accumulate)                        (skipped if NULL)
 *   y_out  [T,H] bf16 = bf16(x2 + down . (silu(gate . h2) * (up . h2)))    (skipped if NULL)
 * The shared expert uses cpu_moe's rounding points (g, u fp32, act bf16); the reference's device
 * kernel also rounds g and u to bf16 (its host checker expert_ref, solar_engine/src/host_util.rs:35-46).
 *
 * moe_combine_residual: the next layer's input, dense/combine.rs:1-77 (`combine`) and layer.rs:4:
 *   x_next [T,H] bf16 = bf16((y + extra) + moe_out), fp32 math, one rounding; extra may be NULL.
 *   moe_out is the combined routed-expert output (what moe_forward returns: sum_k w_k expert_k).
 *
 * moe_block_forward: all three around moe_forward in one call (no host round trip):
 *   logits = h2 . Wr^T; moe_out = routed experts on (h2, logits); y = bf16(x2 + shared(h2));
 *   x_next = bf16((y + extra) + moe_out).
 * y_out / logits_out may be NULL (kept in the context).  Device pointers, or host pointers with
 * MOE_F_HOST (then synchronous).  Expert-parallel contexts need moe_ep_import first (every rank
 * computes the shared expert itself and returns the same x_next). */
MOE_API int moe_load_shared(moe_ctx* ctx, int layer, const uint16_t* gate, const uint16_t* up, const uint16_t* down,
                            const uint16_t* router, int flags);
MOE_API int moe_shared_router(moe_ctx* ctx, int layer, int T, const uint16_t* h2, const uint16_t* x2,
                              uint16_t* y_out, float* logits, int flags, void* stream);
MOE_API int moe_combine_residual(moe_ctx* ctx, int T, const uint16_t* y, const float* extra, const float* moe_out,
                                 uint16_t* x_next, int flags, void* stream);
MOE_API int moe_block_forward(moe_ctx* ctx, int layer, int T, const uint16_t* h2, const uint16_t* x2,
                              const float* extra, uint16_t* x_next, uint16_t* y_out, float* logits_out, int flags,
                              void* stream);

/* Expert-parallel combine over NVLink peer memory (no counterpart in the reference, whose chips
 * return partial sums to one host).  Collective set-up, once per context, every rank of the box:
 *   moe_ep_export(ctx, buf, cap)      writes this rank's MOE_EP_RECORD_BYTES handle record into buf;
 *   (the caller all-gathers the records in rank order, e.g. torch.distributed.all_gather_object)
 *   moe_ep_import(ctx, records, world) maps every other rank's exchange buffer.
 * Afterwards moe_forward on every rank returns the full combined output (all ranks' experts),
 * identical on all ranks; every rank must make the same sequence of moe_forward calls.  A rank that
 * stops calling makes the others' calls fail with MOE_ETIMEOUT after the wait bound. */
#define MOE_EP_RECORD_BYTES 256
MOE_API int moe_ep_export(moe_ctx* ctx, void* buf, int cap);
MOE_API int moe_ep_import(moe_ctx* ctx, const void* records, int world);

/* The router's exponential, y[i] = exp(x[i]) rounded once to fp32 (correctly rounded), on the
 * calling thread's current device, asynchronously on `stream`; x and y are device pointers.  It is
 * the exp of the softmax numerators (host.rs.tpl:249, `(v - m).exp()`) and of the sigmoid
 * denominators (track2_opt/solar_engine/src/host.rs:121) as every router kernel evaluates it,
 * exported so a caller (and the tests) can compare it with a host libm over the whole domain. */
MOE_API int moe_router_exp(const float* x, float* y, int64_t n, void* stream);

/* Synchronise `stream`, then return (and clear) the latched device-side status. */
MOE_API int moe_status(moe_ctx* ctx, void* stream);

/* Number of kernels this context has launched since creation (instrumentation for benchmarks). */
MOE_API int64_t moe_launch_count(moe_ctx* ctx);

/* Context options (moe_set_option):
 *   MOE_OPT_FUSED_DECODE        1 (default): batches of T <= 16 below the tensor-core threshold run as one
 *                               fused persistent kernel (routing + expert GEMV + combine); 0: the
 *                               multi-kernel path.
 *   MOE_OPT_WAIT_TIMEOUT_US     bound on every device-side wait of the fused kernel (default 1 s);
 *                               a wait that runs out makes the call report MOE_ETIMEOUT.
 *   MOE_OPT_INJECT_WAIT_TIMEOUT test hook: 1 makes the fused kernel's grid-wide arrival wait for one
 *                               CTA more than the grid has, so the bounded-wait error path can be
 *                               tested without faulting or hanging the GPU.
 *   MOE_OPT_RING_STAGES         tuning: cap on the fused kernel's shared-memory ring depth (2..16;
 *                               0 = as deep as shared memory allows, the default).
 *   MOE_OPT_STAGE_BYTES         tuning: target bytes per ring stage of the fused kernel (a stage holds
 *                               max(1, target / unit bytes) units; 0 = the default, 48 KiB).
 *   MOE_OPT_PREFILL_MIN_T       batches of at least this many tokens (default 10) run the expert FFN as
 *                               grouped tensor-core GEMMs (each routed expert read once) when every
 *                               local expert of the layer is bf16; smaller batches, and layers holding
 *                               int8 experts, take the fused decode kernel (T <= 16) or the CUDA-core
 *                               path; 0 keeps every batch off the tensor-core path.
 *   MOE_OPT_PREFILL_TC          1 (default): prefill batches run the gate/up and down GEMMs on the
 *                               library's persistent tcgen05 kernels (SwiGLU fused, g / u / y kept in
 *                               fp32); 0: they stay on the CUDA-core multi-kernel path.
 *   MOE_OPT_LAYER_SLOTS         HBM expert slots per layer for layers not yet loaded (0, the default:
 *                               one per local expert); see moe_evict_expert.
 *   MOE_OPT_TIMELINE            instrumentation: 1 records, per CTA of the latest fused launch, 24
 *                               globaltimer / cycle slots (0 start, 1 plan share loaded, 2 all stages
 *                               issued, 3 all segments done, 4 grid-wide arrival seen, 5 reduction
 *                               done; for consumer warp 0, SM cycles (8) waiting for ring stages,
 *                               (9) working on them, (10) of which in the cross-warp exchange; when
 *                               the CTA plans: 16 plan decision made, 17 logits and expert table
 *                               loaded, 18 top-k chosen, 6 routed, 7 jobs, 15 pairs and share; when
 *                               it reduces: 19 partial sums staged, 20 cross-rank exchange begun), the
 *                               planner kernel's stamps in the row after the grid's (0 start,
 *                               1 planned, 2 published, 3 predecessor complete) and CTA 0's per-stage
 *                               stamps; read them with moe_timeline_read.
 *   MOE_OPT_SHARED_INTER        intermediate size of the shared expert (moe_load_shared), set before its
 *                               first load; 0 (the default) = the context's inter.  A context holding a
 *                               slice of every routed expert's units (inter = the slice) still loads the
 *                               whole shared expert: set this to its full width.
 *   MOE_OPT_Q8_UNIT_COST        tuning: how much of the fused kernel's stream one int8 unit counts for
 *                               when a call's units are cut into per-CTA shares, per mille of its bytes
 *                               (500..4000; 0 = the default, 2500).  Shares are balanced by this cost
 *                               rather than by bytes, because dequantising an int8 unit takes longer
 *                               per byte than streaming it.
 *   MOE_OPT_REDUCERS            tuning: in a stream of fused calls (a device-buffer call planned while
 *                               the previous call on the context still runs), how many CTAs (the last to
 *                               finish their share) reduce the partial sums into the output; the others
 *                               leave at once and the next call's CTAs take their SMs.  Raised as
 *                               needed so that a reducer's slice of the partial sums fits on chip
 *                               (default 48; 96 on expert-parallel contexts of eight or more ranks).  Calls made alone, host-buffer calls and block calls use
 *                               every CTA.  0: every call uses every CTA and even shares, so output
 *                               bits never depend on timing (otherwise a streamed call's shares, and
 *                               with them the fp32 summation order, differ from a lone call's).
 *   MOE_OPT_PLANNER             1: a device-buffer fused call made while the previous one still runs is
 *                               planned by a one-CTA planner kernel on the SM the decode grid leaves
 *                               free; 0: every CTA plans for itself.  Default 1 on single-GPU
 *                               contexts, 0 on expert-parallel ones (ep_world > 1).
 *   MOE_OPT_LATE_BYTES          tuning: in a stream of fused calls, the last CTAs by index (as many as
 *                               reduce), which start only when the previous call's reducers leave
 *                               their SMs, get shares smaller by this many bytes of the bf16 stream
 *                               (default 688128, 28 Solar units; 1376256 on expert-parallel contexts). */
#define MOE_OPT_FUSED_DECODE 1
#define MOE_OPT_WAIT_TIMEOUT_US 2
#define MOE_OPT_INJECT_WAIT_TIMEOUT 3
#define MOE_OPT_TIMELINE 4
#define MOE_OPT_RING_STAGES 5
#define MOE_OPT_STAGE_BYTES 6
#define MOE_OPT_PREFILL_MIN_T 7
#define MOE_OPT_PREFILL_TC 8
#define MOE_OPT_LAYER_SLOTS 9
#define MOE_OPT_SHARED_INTER 10
#define MOE_OPT_Q8_UNIT_COST 11
#define MOE_OPT_REDUCERS 12
#define MOE_OPT_LATE_BYTES 13
#define MOE_OPT_PLANNER 14
MOE_API int moe_set_option(moe_ctx* ctx, int option, int64_t value);

/* Copies up to cap stamps to host memory (synchronises): [SM count][24] per-CTA stamps (see
 * MOE_OPT_TIMELINE) followed by CTA 0's per-stage issue / landed / released stamps ([3][1024]). */
MOE_API int moe_timeline_read(moe_ctx* ctx, uint64_t* out, int cap);

/* Stage timing of moe_forward with CUDA events on the caller's stream (instrumentation; off by
 * default).  moe_profile(ctx, 1) starts a fresh record; moe_profile_read synchronises and returns
 * the summed milliseconds per stage (0 router+permutation, 1 gate/up+SwiGLU kernel, 2 down kernel,
 * 3 combine kernel; with the fused decode kernel everything is stage 1) over the calls made since,
 * and the number of calls; it then clears the record. */
MOE_API int moe_profile(moe_ctx* ctx, int enable);
MOE_API int moe_profile_read(moe_ctx* ctx, double* stage_ms, int n_stages, int64_t* n_calls);

/* ck_moe3 without any allocation, for callers that may not call cudaMalloc (for example a server
 * whose own allocator already owns all of HBM, or code running where an allocation could block or
 * fail): it needs no moe_ctx (whose creation allocates) and allocates nothing, neither device nor
 * pinned host memory.  No counterpart in the reference: it is the ck_moe3 surface above
 * (out [H] += sum_e w[e] * expert_e(x), base[e] in the [g F*H][u F*H][d H*F] layout; base is a host
 * array of device pointers, w / x / out are device pointers) with its working memory held in a
 * 1 MiB file-scope device array inside libmoe_dp.so, which every GPU that loads the library keeps
 * until the process exits.  Limits: E <= 16 and E * (2F + 4H) bytes plus tables within the 1 MiB
 * (H = 4096, F = 1280 fits 16 experts); larger calls return MOE_EINVAL.  Runs on the calling
 * thread's current device, asynchronously on `stream`.  All calls on a device share that array:
 * calls that overlap on the GPU race, so keep them on one stream or synchronise between them.  The
 * first call on each device looks the array's address up (cudaGetSymbolAddress) and should be made
 * before any stream capture. */
MOE_API int moe_ck_moe3_noalloc(int E, const uint16_t* const* base, const float* w, const uint16_t* x, float* out,
                                int H, int F, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* MOE_DP_H */
