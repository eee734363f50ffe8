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
    int unit_layout;          // 1: every job's expert is a kLayoutUnit table; 0: kLayoutSplit
    const float* comb_w;      // combine: null when y already carries the routing weights, else the
                              // weight of each pair (y[p] is multiplied by comb_w[p])
};

// out[t, :] = (accumulate ? out : 0) + sum over the token's pairs (comb_off / comb_p, job order) of
// y[p, :] (times comb_w[p] when set).
cudaError_t launch_combine(const ExpertArgs& a, cudaStream_t st, int* launches);

// Prefill helpers (prefill.cu): token-row gather before the grouped GEMMs, weighted combine after.
cudaError_t launch_gather_rows(const uint16_t* x, const int32_t* ptok, int n, int H, uint16_t* xg, int sm_count,
                               cudaStream_t st, const int* n_dev = nullptr);
cudaError_t launch_combine_rows(const float* y, const float* w, const int32_t* comb_off, const int32_t* comb_p, int T,
                                int H, int accumulate, float* out, cudaStream_t st);

// Launches the decode expert pipeline (gate/up+SwiGLU, down, combine); adds the launch count.
// marks (nullable): three events recorded after the gate/up, down and combine stages.
cudaError_t launch_experts(const ExpertArgs& a, int sm_count, cudaStream_t st, int* launches, cudaEvent_t* marks);

// Row geometry of quantize_q8_kernel (element offsets / steps; bf16 in, int8 out).
struct QuantGeom {
    const uint16_t* g;        // gate row f at g + f * gu_pitch
    const uint16_t* u;        // up row f at u + f * gu_pitch
    const uint16_t* d;        // down row h, element i at d + h * d_row_step + i * d_elem_step
    size_t gu_pitch, d_row_step, d_elem_step;
    int8_t* q;                // gate row f at q + f * q_pitch, up row f at + q_up_off
    size_t q_pitch, q_up_off;
    size_t q_down_off, q_down_row_step, q_down_elem_step;  // down row h element i
    int trailer;              // 1: also write (sc_gate f, sc_up f, 0, 0) at q + f * q_pitch + 3H
};

// Reference layout in and out: [F gate][F up] rows of H, down [H, F] ([F gate][F up][H down] rows).
QuantGeom quant_geom_split(const uint16_t* g, const uint16_t* u, const uint16_t* d, int H, int F, int8_t* q);
// A bf16 unit table in, an int8 unit table out (kLayoutUnit).
QuantGeom quant_geom_unit(const uint16_t* unit_bf16, int H, int F, int8_t* q_unit);

// ck_place_expert_q8 on the device: quant_row applied to the 2F gate/up rows and H down rows;
// scales / row sums (nullable) in the reference's row order.
cudaError_t launch_quantize_q8(const QuantGeom& q, int H, int F, float* sc, int32_t* rs, cudaStream_t st,
                               int* launches);

// Scatters a row-major [H, F] down matrix (element size esize: 2 = bf16, 1 = int8) into the down
// columns of a unit table: dst[f * pitch + h] = src[h * F + f] (pitch in elements).
cudaError_t launch_scatter_down(const void* src, void* dst, size_t pitch, int H, int F, int esize, cudaStream_t st,
                                int* launches);

}  // namespace moe
