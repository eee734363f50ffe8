/*
 * moe_oracle.c -- CPU restatement of npu-offload's routed-expert MoE data plane.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the checker, never the product: only tests/,
 * __graft_entry__.smoke() and bench.py's cpu_baseline / reference legs load it.  The product
 * path (npu_offload_b200) never calls into it and fails loudly when its CUDA library is missing.
 *
 * Every function names the reference lines it restates (paths are relative to the
 * ai-computing/npu-offload project root).  Arithmetic is plain scalar C with fp32 accumulation;
 * the rounding points (where a value is rounded to bf16, which sums are sequential) follow the
 * reference exactly.  Dot products are summed left to right, which differs from the reference's
 * 32-lane AVX-512 reduction order only in the last bits (the oracle is pinned against the compiled
 * reference in tests/test_oracle.py).
 *
 * Build: oracle/build.py (gcc -O2 -fopenmp -shared -fPIC; no -ffast-math, no FMA contraction).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define OR_OK 0
#define OR_EINVAL 1
#define OR_ENONFINITE 2

/* bf16 <-> f32, round-to-nearest-even without NaN special-casing: solar_hybrid/cpu_moe.cpp:30-34,
 * track2_opt/solar_engine/csrc/cpu_kern.c:21-27. */
static inline float bf2f(uint16_t b) {
    uint32_t u = (uint32_t)b << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}
static inline uint16_t f2bf(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    u += 0x7FFFu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}

uint16_t or_f2bf(float f) { return f2bf(f); }
float or_bf2f(uint16_t b) { return bf2f(b); }

void or_set_threads(int n) {
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
#else
    (void)n;
#endif
}

int or_max_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

/* The routers' exponential: exp evaluated in double and rounded once to fp32, i.e. a correctly
 * rounded expf.  The reference calls f32::exp (host.rs.tpl:249, host.rs:121), which goes to the
 * platform libm; glibc 2.39's expf is not correctly rounded -- it is one ulp off on 97,052 of the
 * 1,120,927,745 floats in [-104, 0], the domain of the softmax's exp(v - max).  The GPU routers and
 * this oracle both use the correctly rounded value (tests compare them over that whole domain), so
 * top-k ties and weights agree bit for bit between them. */
static inline float router_exp(float x) { return (float)exp((double)x); }

/* router_exp over n consecutive float bit patterns starting at first_bits (test support). */
void or_router_exp_range(uint32_t first_bits, int64_t n, float* out) {
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < n; i++) {
        const uint32_t b = first_bits + (uint32_t)i;
        float x;
        memcpy(&x, &b, 4);
        out[i] = router_exp(x);
    }
}

/* Count of floats among bit patterns first_bits, first_bits + stride, ... (n of them) where router_exp
 * differs from the long-double exp rounded to fp32 (a correctly-rounded check; test support). */
int64_t or_router_exp_vs_long_double(uint32_t first_bits, int64_t n, int32_t stride) {
    int64_t bad = 0;
#pragma omp parallel for schedule(static) reduction(+ : bad)
    for (int64_t i = 0; i < n; i++) {
        const uint32_t b = first_bits + (uint32_t)(i * stride);
        float x;
        memcpy(&x, &b, 4);
        const float a = (float)expl((long double)x), c = router_exp(x);
        if (memcmp(&a, &c, 4) != 0) bad++;
    }
    return bad;
}

/* Count of floats (bit patterns first_bits .. first_bits + n - 1) where the host libm's expf differs
 * from router_exp, and the largest difference in ulps (test support). */
int64_t or_libm_expf_mismatches(uint32_t first_bits, int64_t n, int32_t* max_ulp) {
    int64_t bad = 0;
    int32_t worst = 0;
#pragma omp parallel for schedule(static) reduction(+ : bad) reduction(max : worst)
    for (int64_t i = 0; i < n; i++) {
        const uint32_t b = first_bits + (uint32_t)i;
        float x;
        memcpy(&x, &b, 4);
        const float a = expf(x), c = router_exp(x);
        int32_t ua, uc;
        memcpy(&ua, &a, 4);
        memcpy(&uc, &c, 4);
        if (ua != uc) {
            bad++;
            const int32_t d = ua > uc ? ua - uc : uc - ua;
            if (d > worst) worst = d;
        }
    }
    if (max_ulp) *max_ulp = worst;
    return bad;
}

/* Top-k selection shared by both scoring modes: repeatedly take the largest key, ties to the lower
 * index.  Equivalent to the first k entries of the reference's stable descending sort
 * (npu-kernels/npu_kernels/rngd/layer_template/src/host.rs.tpl:256-260; Rust sort_by is stable, so
 * track2_opt/solar_engine/src/host.rs:123-124 breaks ties the same way). */
static void topk_desc(const float* key, int E, int K, int32_t* out) {
    unsigned char taken[1024];
    memset(taken, 0, (size_t)E);
    for (int k = 0; k < K; k++) {
        int best = -1;
        for (int i = 0; i < E; i++) {
            if (taken[i]) continue;
            if (best < 0 || key[i] > key[best]) best = i;
        }
        taken[best] = 1;
        out[k] = best;
    }
}

/*
 * Softmax router, npu-kernels/npu_kernels/rngd/layer_template/src/host.rs.tpl:247-268:
 *   m = max(logits); e_i = exp(v_i - m) (router_exp); z = sum_i e_i (sequential, index order); p_i = e_i / z;
 *   order p descending, ties -> lower index; take K; w_k = p_k / sum_k p_k (sequential, no epsilon).
 * Returns OR_ENONFINITE where the reference would panic (a NaN reaching partial_cmp().unwrap()).
 */
int or_route_softmax(int T, int E, int K, const float* logits, int32_t* idx, float* w) {
    if (T < 0 || E <= 0 || E > 1024 || K <= 0 || K > E) return OR_EINVAL;
    int status = OR_OK;
    float p[1024];
    for (int t = 0; t < T; t++) {
        const float* v = logits + (size_t)t * E;
        float m = -INFINITY;
        for (int i = 0; i < E; i++) m = (v[i] > m || m != m) ? v[i] : m; /* f32::max fold */
        float z = 0.f;
        for (int i = 0; i < E; i++) {
            p[i] = router_exp(v[i] - m);
            z += p[i];
        }
        int bad = 0;
        for (int i = 0; i < E; i++) {
            p[i] = p[i] / z;
            if (p[i] != p[i]) bad = 1;
        }
        if (bad) status = OR_ENONFINITE;
        int32_t* it = idx + (size_t)t * K;
        float* wt = w + (size_t)t * K;
        topk_desc(p, E, K, it);
        float tot = 0.f;
        for (int k = 0; k < K; k++) tot += p[it[k]];
        for (int k = 0; k < K; k++) wt[k] = p[it[k]] / tot;
    }
    return status;
}

/*
 * Sigmoid + correction-bias router, track2_opt/solar_engine/src/host.rs:119-128 (also the template's
 * non-softmax branch, host.rs.tpl:254-265):
 *   s_i = 1/(1+exp(-v_i)) (router_exp); key_i = s_i + bias_i; top K by key (ties -> lower index);
 *   w_k = s_k / (sum_k s_k + 1e-20).   bias may be NULL (all zero).
 */
int or_route_sigmoid(int T, int E, int K, const float* logits, const float* bias, int32_t* idx, float* w) {
    if (T < 0 || E <= 0 || E > 1024 || K <= 0 || K > E) return OR_EINVAL;
    int status = OR_OK;
    float s[1024], key[1024];
    for (int t = 0; t < T; t++) {
        const float* v = logits + (size_t)t * E;
        int bad = 0;
        for (int i = 0; i < E; i++) {
            s[i] = 1.0f / (1.0f + router_exp(-v[i]));
            key[i] = s[i] + (bias ? bias[i] : 0.0f);
            if (key[i] != key[i]) bad = 1;
        }
        if (bad) status = OR_ENONFINITE;
        int32_t* it = idx + (size_t)t * K;
        float* wt = w + (size_t)t * K;
        topk_desc(key, E, K, it);
        float tot = 0.f;
        for (int k = 0; k < K; k++) tot += s[it[k]];
        tot += 1e-20f;
        for (int k = 0; k < K; k++) wt[k] = s[it[k]] / tot;
    }
    return status;
}

/*
 * Token -> expert grouping, solar_hybrid/runtime.py:343-354 (per = {e: [(t, w)]}, t-major, k-minor
 * insertion; jobs in first-appearance order) and the expert-major CSR the device path uses.
 * Outputs:
 *   counts[E]         pairs per expert
 *   offsets[E+1]      exclusive prefix of counts (expert-id order)
 *   perm[T*K]         pair ids (t*K + k), grouped by expert id ascending, tokens ascending in a group
 *   job_order[E]      experts with count > 0 in first-appearance order (the cpu_moe job list)
 *   *n_jobs           number of such experts
 * Returns OR_EINVAL if an index is out of range or repeats within a token.
 */
int or_permute(int T, int K, int E, const int32_t* idx, int32_t* counts, int32_t* offsets, int32_t* perm,
               int32_t* job_order, int32_t* n_jobs) {
    if (T < 0 || K <= 0 || E <= 0) return OR_EINVAL;
    memset(counts, 0, sizeof(int32_t) * (size_t)E);
    int nj = 0;
    for (int t = 0; t < T; t++)
        for (int k = 0; k < K; k++) {
            int e = idx[(size_t)t * K + k];
            if (e < 0 || e >= E) return OR_EINVAL;
            for (int k2 = 0; k2 < k; k2++)
                if (idx[(size_t)t * K + k2] == e) return OR_EINVAL;
            if (counts[e] == 0) job_order[nj++] = e;
            counts[e]++;
        }
    offsets[0] = 0;
    for (int e = 0; e < E; e++) offsets[e + 1] = offsets[e] + counts[e];
    int32_t* fill = (int32_t*)calloc((size_t)E, sizeof(int32_t));
    for (int t = 0; t < T; t++)
        for (int k = 0; k < K; k++) {
            int e = idx[(size_t)t * K + k];
            perm[offsets[e] + fill[e]++] = t * K + k;
        }
    free(fill);
    *n_jobs = nj;
    return OR_OK;
}

/* fp32 dot of two bf16 vectors, sequential. */
static inline float dot_bf16(const uint16_t* a, const uint16_t* b, int n) {
    float s = 0.f;
    for (int i = 0; i < n; i++) s += bf2f(a[i]) * bf2f(b[i]);
    return s;
}
/* fp32 dot of bf16 x with int8 weights widened exactly: cpu_kern.c:292-305. */
static inline float dot_bf16_i8(const uint16_t* x, const int8_t* q, int n) {
    float s = 0.f;
    for (int i = 0; i < n; i++) s += bf2f(x[i]) * (float)q[i];
    return s;
}

/* SwiGLU activation rounded to bf16: cpu_moe.cpp:70-77 (act = f2bf(g / (1 + exp(-g)) * u)). */
static inline uint16_t swiglu_bf16(float g, float u) { return f2bf(g / (1.f + expf(-g)) * u); }

/*
 * One expert job of the fused decode MoE, cpu_moe.cpp:38-96 semantics for tokens toks[0..nt):
 *   g,u  = rows of gu (gate rows 0..F-1, up rows F..2F-1) . x_t   (fp32, not rounded)  :63-66
 *   act  = bf16(silu(g) * u)                                                           :70-77
 *   out[t,h] += w_j * dot(d[h,:], act)                                                 :81-93
 * gu: [2F, H] bf16 row-major; d: [H, F] bf16 row-major.
 */
static void expert_job_bf16(int H, int F, const uint16_t* x, const uint16_t* gu, const uint16_t* d, int nt,
                            const int64_t* toks, const float* ws, float* out, uint16_t* act) {
    #pragma omp parallel for schedule(static)
    for (int f = 0; f < F; f++) {
        const uint16_t* rg = gu + (size_t)f * H;
        const uint16_t* ru = gu + (size_t)(F + f) * H;
        for (int j = 0; j < nt; j++) {
            const uint16_t* xt = x + (size_t)toks[j] * H;
            act[(size_t)j * F + f] = swiglu_bf16(dot_bf16(rg, xt, H), dot_bf16(ru, xt, H));
        }
    }
    #pragma omp parallel for schedule(static)
    for (int h = 0; h < H; h++) {
        const uint16_t* row = d + (size_t)h * F;
        for (int j = 0; j < nt; j++)
            out[(size_t)toks[j] * H + h] += ws[j] * dot_bf16(row, act + (size_t)j * F, F);
    }
}

/*
 * Weight-only int8 expert job, ck_moe_q8w semantics (cpu_kern.c:306-333) applied to each token:
 *   g_r = dot(x, q_r) * sc[r]; act = bf16(silu(g) * u); out[h] += w * dot(act, qd_h) * sc[2F+h].
 * q: [(2F) rows of H][H rows of F] int8 (ck_place_expert_q8 layout, cpu_kern.c:227-241); sc: [2F+H].
 */
static void expert_job_q8(int H, int F, const uint16_t* x, const int8_t* q, const float* sc, int nt,
                          const int64_t* toks, const float* ws, float* out, uint16_t* act) {
    #pragma omp parallel for schedule(static)
    for (int f = 0; f < F; f++) {
        for (int j = 0; j < nt; j++) {
            const uint16_t* xt = x + (size_t)toks[j] * H;
            float g = dot_bf16_i8(xt, q + (size_t)f * H, H) * sc[f];
            float u = dot_bf16_i8(xt, q + (size_t)(F + f) * H, H) * sc[F + f];
            act[(size_t)j * F + f] = swiglu_bf16(g, u);
        }
    }
    const int8_t* qd = q + (size_t)2 * F * H;
    #pragma omp parallel for schedule(static)
    for (int h = 0; h < H; h++)
        for (int j = 0; j < nt; j++)
            out[(size_t)toks[j] * H + h] += ws[j] * dot_bf16_i8(act + (size_t)j * F, qd + (size_t)h * F, F) * sc[2 * F + h];
}

/*
 * cpu_moe surface (cpu_moe.cpp:38-39): x [T,H] bf16, per job j: gu[j] [2F,H], d[j] [H,F],
 * tokens toks[tok_off[j] .. tok_off[j+1]) with routing weights ws[...].  out [T,H] fp32 is
 * zero-filled first unless `accumulate` is set (ck_moe3 accumulates, cpu_kern.c:141).
 * Jobs are applied in order, so each out[t,h] sums its experts in job order like the reference.
 * q8[j] != NULL selects the int8 weight-only form for job j (then gu[j]/d[j] are ignored and
 * sc[j] holds its scales).
 */
int or_cpu_moe(int T, int H, int F, int n_jobs, const uint16_t* x, const uint16_t* const* gu,
               const uint16_t* const* d, const int8_t* const* q8, const float* const* sc, const int64_t* tok_off,
               const int64_t* toks, const float* ws, float* out, int accumulate) {
    if (T < 0 || H <= 0 || F <= 0 || n_jobs < 0) return OR_EINVAL;
    if (!accumulate) memset(out, 0, sizeof(float) * (size_t)T * H);
    if (n_jobs == 0) return OR_OK;
    int maxnt = 0;
    for (int j = 0; j < n_jobs; j++) {
        int nt = (int)(tok_off[j + 1] - tok_off[j]);
        if (nt < 0) return OR_EINVAL;
        if (nt > maxnt) maxnt = nt;
        for (int64_t i = tok_off[j]; i < tok_off[j + 1]; i++)
            if (toks[i] < 0 || toks[i] >= T) return OR_EINVAL;
    }
    uint16_t* act = (uint16_t*)malloc(sizeof(uint16_t) * (size_t)(maxnt > 0 ? maxnt : 1) * F);
    for (int j = 0; j < n_jobs; j++) {
        int nt = (int)(tok_off[j + 1] - tok_off[j]);
        if (nt == 0) continue;
        if (q8 && q8[j])
            expert_job_q8(H, F, x, q8[j], sc[j], nt, toks + tok_off[j], ws + tok_off[j], out, act);
        else
            expert_job_bf16(H, F, x, gu[j], d[j], nt, toks + tok_off[j], ws + tok_off[j], out, act);
    }
    free(act);
    return OR_OK;
}

/*
 * Per-row symmetric int8 quantisation, cpu_kern.c:218-224 (quant_row):
 *   m = max |w|; s = m > 0 ? m / 127 : 1; inv = 1 / s; q = clamp(lrintf(w * inv), -127, 127); rs = sum q.
 */
static void quant_row(const uint16_t* src, int n, int8_t* dst, float* sc, int32_t* rs) {
    float m = 0.f;
    for (int i = 0; i < n; i++) {
        float v = fabsf(bf2f(src[i]));
        if (v > m) m = v;
    }
    float s = m > 0 ? m / 127.f : 1.f, inv = 1.f / s;
    int32_t sum = 0;
    for (int i = 0; i < n; i++) {
        int q = (int)lrintf(bf2f(src[i]) * inv);
        q = q > 127 ? 127 : (q < -127 ? -127 : q);
        dst[i] = (int8_t)q;
        sum += q;
    }
    *sc = s;
    *rs = sum;
}

/* ck_place_expert_q8 layout (cpu_kern.c:227-241): rows 0..2F-1 = gate|up rows (len H), then H down rows
 * (len F); sc/rs hold one entry per row.  rs may be NULL. */
void or_place_expert_q8(const uint16_t* g, const uint16_t* u, const uint16_t* d, int8_t* q, float* sc, int32_t* rs,
                        int H, int F) {
    #pragma omp parallel for schedule(static)
    for (int r = 0; r < 2 * F + H; r++) {
        int32_t dummy;
        int32_t* rsp = rs ? &rs[r] : &dummy;
        if (r < F)
            quant_row(g + (size_t)r * H, H, q + (size_t)r * H, &sc[r], rsp);
        else if (r < 2 * F)
            quant_row(u + (size_t)(r - F) * H, H, q + (size_t)r * H, &sc[r], rsp);
        else {
            int h = r - 2 * F;
            quant_row(d + (size_t)h * F, F, q + (size_t)2 * F * H + (size_t)h * F, &sc[r], rsp);
        }
    }
}

/*
 * Whole MoE layer as the reference's host path composes it (solar_hybrid/runtime.py:338-423 with
 * mode="cpu": route -> group -> cpu_moe over the job list -> fp32 output):
 *   scoring 0 = softmax router (host.rs.tpl:247-268), 1 = sigmoid + bias (host.rs:119-128).
 * Expert e's weights: gu[e], d[e] (bf16) or q8[e]/sc[e] (int8, when q8 && q8[e]).
 * Also returns idx/w (may be NULL).
 */
int or_moe_layer(int T, int H, int F, int E, int K, int scoring, const uint16_t* x, const float* logits,
                 const float* bias, const uint16_t* const* gu, const uint16_t* const* d, const int8_t* const* q8,
                 const float* const* sc, float* out, int32_t* idx_out, float* w_out) {
    if (T < 0 || E <= 0 || K <= 0 || K > E) return OR_EINVAL;
    int32_t* idx = (int32_t*)malloc(sizeof(int32_t) * (size_t)(T > 0 ? T : 1) * K);
    float* w = (float*)malloc(sizeof(float) * (size_t)(T > 0 ? T : 1) * K);
    int st = scoring == 0 ? or_route_softmax(T, E, K, logits, idx, w) : or_route_sigmoid(T, E, K, logits, bias, idx, w);
    int32_t* counts = (int32_t*)malloc(sizeof(int32_t) * (size_t)E);
    int32_t* offsets = (int32_t*)malloc(sizeof(int32_t) * (size_t)(E + 1));
    int32_t* perm = (int32_t*)malloc(sizeof(int32_t) * (size_t)(T > 0 ? T : 1) * K);
    int32_t* job_order = (int32_t*)malloc(sizeof(int32_t) * (size_t)E);
    int32_t nj = 0;
    int st2 = or_permute(T, K, E, idx, counts, offsets, perm, job_order, &nj);
    if (st2 != OR_OK) st = st2;
    const uint16_t** jgu = (const uint16_t**)malloc(sizeof(void*) * (size_t)E);
    const uint16_t** jd = (const uint16_t**)malloc(sizeof(void*) * (size_t)E);
    const int8_t** jq = (const int8_t**)malloc(sizeof(void*) * (size_t)E);
    const float** jsc = (const float**)malloc(sizeof(void*) * (size_t)E);
    int64_t* toff = (int64_t*)malloc(sizeof(int64_t) * (size_t)(E + 1));
    int64_t* toks = (int64_t*)malloc(sizeof(int64_t) * (size_t)(T > 0 ? T : 1) * K);
    float* ws = (float*)malloc(sizeof(float) * (size_t)(T > 0 ? T : 1) * K);
    toff[0] = 0;
    for (int j = 0; j < nj; j++) {
        int e = job_order[j];
        jgu[j] = gu ? gu[e] : NULL;
        jd[j] = d ? d[e] : NULL;
        jq[j] = q8 ? q8[e] : NULL;
        jsc[j] = sc ? sc[e] : NULL;
        int n = 0;
        for (int i = offsets[e]; i < offsets[e + 1]; i++, n++) {
            int p = perm[i];
            toks[toff[j] + n] = p / K;
            ws[toff[j] + n] = w[p];
        }
        toff[j + 1] = toff[j] + n;
    }
    if (st2 == OR_OK) {
        int st3 = or_cpu_moe(T, H, F, nj, x, jgu, jd, q8 ? jq : NULL, jsc, toff, toks, ws, out, 0);
        if (st3 != OR_OK) st = st3;
    }
    if (idx_out) memcpy(idx_out, idx, sizeof(int32_t) * (size_t)T * K);
    if (w_out) memcpy(w_out, w, sizeof(float) * (size_t)T * K);
    free(idx); free(w); free(counts); free(offsets); free(perm); free(job_order);
    free(jgu); free(jd); free(jq); free(jsc); free(toff); free(toks); free(ws);
    return st;
}

/*
 * Router-logit producer, track2_opt/solar_engine/src/dense/shared.rs:1-3 (`shared_router`):
 *   logits[t, e] = h2_t . Wr[e, :]   fp32 accumulate, fp32 out.  Wr: [E, H] bf16 row-major.
 */
void or_router_logits(int T, int E, int H, const uint16_t* h2, const uint16_t* wr, float* logits) {
    #pragma omp parallel for schedule(static)
    for (int e = 0; e < E; e++)
        for (int t = 0; t < T; t++) logits[(size_t)t * E + e] = dot_bf16(wr + (size_t)e * H, h2 + (size_t)t * H, H);
}

/*
 * Shared expert + residual of shared.rs:1-3:  y = bf16(x2 + Wsd @ (silu(Wsg h2) * (Wsu h2))), fp32 add
 * before the one rounding.  device_rounding = 0: the expert in cpu_moe's rounding points (g, u fp32,
 * act bf16; cpu_moe.cpp:63-93), the form the B200 kernels compute.  device_rounding = 1: the
 * reference's own host checker of its device kernels, expert_ref (solar_engine/src/host_util.rs:35-46:
 * g and u rounded to bf16 before SwiGLU).  gu: [2F, H] (gate rows, then up rows); d: [H, F].
 * shared_out (optional) receives the fp32 expert output before the residual.
 */
void or_shared_expert(int T, int H, int F, const uint16_t* h2, const uint16_t* x2, const uint16_t* gu,
                      const uint16_t* d, int device_rounding, float* shared_out, uint16_t* y) {
    uint16_t* act = (uint16_t*)malloc(sizeof(uint16_t) * (size_t)(T > 0 ? T : 1) * F);
    float* s = (float*)malloc(sizeof(float) * (size_t)(T > 0 ? T : 1) * H);
    #pragma omp parallel for schedule(static)
    for (int f = 0; f < F; f++)
        for (int t = 0; t < T; t++) {
            const uint16_t* xt = h2 + (size_t)t * H;
            float g = dot_bf16(gu + (size_t)f * H, xt, H), u = dot_bf16(gu + (size_t)(F + f) * H, xt, H);
            if (device_rounding) {
                g = bf2f(f2bf(g));
                u = bf2f(f2bf(u));
            }
            act[(size_t)t * F + f] = swiglu_bf16(g, u);
        }
    #pragma omp parallel for schedule(static)
    for (int h = 0; h < H; h++)
        for (int t = 0; t < T; t++) s[(size_t)t * H + h] = dot_bf16(d + (size_t)h * F, act + (size_t)t * F, F);
    for (size_t i = 0; i < (size_t)T * H; i++) {
        if (shared_out) shared_out[i] = s[i];
        if (y) y[i] = f2bf(bf2f(x2[i]) + s[i]);
    }
    free(act);
    free(s);
}

/*
 * Residual combine into the next layer's input, solar_engine/src/dense/combine.rs:1 and
 * layer.rs:4:  x_next = bf16((y + extra) + moe), fp32 math, one rounding.  moe is the combined
 * routed-expert sum (sum_k g_k e_k); extra may be NULL (then x_next = bf16(y + moe)).
 */
void or_combine_residual(long n, const uint16_t* y, const float* extra, const float* moe, uint16_t* x_next) {
    for (long i = 0; i < n; i++) {
        const float s = extra ? bf2f(y[i]) + extra[i] : bf2f(y[i]);
        x_next[i] = f2bf(s + moe[i]);
    }
}
