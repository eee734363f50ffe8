// Router / permutation launch interface (device pointers).
#pragma once
#include "common.cuh"

namespace moe {

struct RouteArgs {
    const float* logits;  // [T, E]
    const float* bias;    // [E] or null (sigmoid scoring)
    int T, E, K, scoring;
    int32_t* idx;         // [T*K] out (required)
    float* w;             // [T*K] out (required)
    int32_t* counts;      // [E] out, optional
    int32_t* offsets;     // [E+1] out, optional
    int32_t* perm;        // [T*K] out, optional: pair ids grouped by expert
    int32_t* job_order;   // [E] out, optional
    int32_t* n_jobs;      // [1] out, optional
    int32_t* ptok;        // [T*K] out, optional: token of each grouped pair
    float* pw;            // [T*K] out, optional: routing weight of each grouped pair
    int32_t* pairpos;     // [T*K] out, required when comb_p is set: grouped position of pair t*K+k
    int32_t* comb_off;    // [T+1] out, optional: per-token CSR into comb_p
    int32_t* comb_p;      // [T*K] out, optional: grouped positions of a token's pairs in job order
    Job* jobs;            // [E] out, optional: local expert jobs in job order
    int32_t* n_ljobs;     // [1] out, optional
    const ExpDesc* desc;  // [E] expert table of the layer, or null
    uint32_t* err;        // latched error bits
    int32_t* scratch;     // optional [permute_scratch_ints(T, E)]: batches above 64 tokens then place
                          // their pairs over many CTAs (null: one block does everything)
};

// Ints of RouteArgs::scratch for T tokens and E experts.
constexpr size_t route_scratch_ints(int T, int E) { return (size_t)(T + 31) / 32 * E + 3 * (size_t)E; }

cudaError_t launch_route(const RouteArgs& a, cudaStream_t st, int* launches);
cudaError_t route_set_smem_limits();
// y[i] = router_exp(x[i]) for i < n (device pointers).
cudaError_t launch_router_exp(const float* x, float* y, long long n, int sms, cudaStream_t st);

}  // namespace moe
