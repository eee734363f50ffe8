// Expert FFN launch interface (device pointers).
#pragma once
#include "common.cuh"

namespace moe {

struct ExpertArgs {
    const uint16_t* x;        // [T, H] bf16 hidden states
    int T, H, F;
    const Job* jobs;          // local expert jobs
    const int32_t* n_jobs;    // device count of jobs (used when n_jobs_host < 0)
    int n_jobs_host;          // job count when the host knows it, else -1
    int n_jobs_max;           // host upper bound on the job count (grid sizing)
    int max_pairs;            // host upper bound on the pairs of one job
    const int32_t* ptok;      // [NP] token of each grouped pair
    const float* pw;          // [NP] routing weight of each grouped pair
    uint16_t* act;            // [NP, F] bf16 scratch: SwiGLU activations
    float* y;                 // [NP, H] fp32 scratch: weighted expert outputs
    const int32_t* comb_off;  // [T+1]
    const int32_t* comb_p;    // grouped pair positions per token, in job order (-1 = skip)
    float* out;               // [T, H] fp32
    int accumulate;           // out += instead of out =
    uint32_t* err;
};

// Launches the decode expert pipeline (gate/up+SwiGLU, down, combine); adds the launch count.
// marks (nullable): three events recorded after the gate/up, down and combine stages.
cudaError_t launch_experts(const ExpertArgs& a, int sm_count, cudaStream_t st, int* launches, cudaEvent_t* marks);

// ck_place_expert_q8 on the device: quant_row applied to the 2F gate/up rows and H down rows.
// interleaved = 0: g/u are separate [F,H] arrays and q gets the reference layout
// ([F gate][F up][H down] rows); 1: g/u are the rows of an interleaved [F][gate|up] table
// (u = g + H) and q gets the same interleaved layout followed by the H down rows.
cudaError_t launch_quantize_q8(const uint16_t* g, const uint16_t* u, const uint16_t* d, int H, int F, int8_t* q,
                               float* sc, int32_t* rs, cudaStream_t st, int* launches, int interleaved);

}  // namespace moe
