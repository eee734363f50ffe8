// Fused persistent decode kernel: launch interface.
#pragma once
#include "common.cuh"

namespace moe {

constexpr int kDecodeMaxT = 16;  // largest batch the fused decode kernel takes
constexpr int kDecodeMaxPairs = kDecodeMaxT * kMaxTopK;
constexpr int kDecodePlanJobs = 128;  // local jobs of one fused call (<= min(E, T*K))
constexpr int kTimelineSlots = 16;  // per-CTA stamps recorded when DecodeArgs::timeline is set
constexpr int kStageLogMax = 1024;  // stages of CTA 0 recorded in DecodeArgs::stage_log
constexpr int kPlanMaxGrid = 256;   // decode CTAs a plan can describe
constexpr int kSegPerCta = 16;      // gate/up segments (runs of one job's units) per decode CTA

// Routing result and job list of one fused call, identical for every decode CTA.  The plan structs
// are copied with 16-byte vector loads, hence the 16-byte alignment (sizes are multiples of 16).
struct __align__(16) PlanShared {
    int nj, np, T, pad;
    int jexp[kDecodePlanJobs];
    int jkind[kDecodePlanJobs];
    int jlayout[kDecodePlanJobs];
    const unsigned char* jw1[kDecodePlanJobs];  // job's gate/up rows
    const unsigned char* jw2[kDecodePlanJobs];  // job's down rows
    const float* jsc[kDecodePlanJobs];          // job's int8 row scales
    int jp0[kDecodePlanJobs + 1];               // pair offsets (job-major)
    int ptok[kDecodeMaxPairs];                  // token of each pair
    float pw[kDecodeMaxPairs];                  // routing weight of each pair
    int tpn[kDecodeMaxT];                       // local pairs per token
    int tpair[kDecodeMaxT][kMaxTopK];           // a token's pairs in job order
};

// One decode CTA's static share: gate/up units [u_first, u_end) as segments, down rows [h0, h1).
struct __align__(16) PlanCta {
    int u_first, u_end, n1, n2, h0, h1, nseg, pad;
    int seg_j[kSegPerCta], seg_f0[kSegPerCta], seg_fend[kSegPerCta], seg_ups[kSegPerCta];
    int seg_stage[kSegPerCta + 1];
    int pad2[3];
};

struct __align__(16) DecodePlan {
    PlanShared sh;
    PlanCta cta[kPlanMaxGrid];
};
static_assert(sizeof(PlanShared) % 16 == 0 && sizeof(PlanCta) % 16 == 0 && sizeof(DecodePlan) % 16 == 0,
              "plan structs are copied as int4");
static_assert(alignof(PlanShared) == 16 && alignof(PlanCta) == 16, "plan structs are copied as int4");

struct PlanArgs {
    const float* logits;   // [T, E]
    const float* bias;     // [E] or null
    const ExpDesc* desc;   // [E] expert table of the layer
    DecodePlan* plan;      // this call's plan (parity buffer)
    uint32_t* flag;        // this call's plan flag: set to stamp once the plan is written
    uint32_t stamp;
    int32_t* idx_out;      // [T, K] router indices
    float* w_out;          // [T, K] router weights
    uint32_t* err;
    int T, E, K, H, F, scoring;
    int G;                 // decode grid size
    uint32_t slot_bytes;
    int rs_bf16, rs_q8;
};

struct DecodeArgs {
    const DecodePlan* plan;    // written by plan_kernel for this call
    const uint32_t* flag;      // plan flag; the plan is valid once *flag == stamp
    uint32_t stamp;
    const uint16_t* x;     // [T, H] bf16
    float* out;            // [T, H] fp32
    uint16_t* act;         // [kDecodeMaxPairs, F] bf16 scratch
    uint32_t* ctr;         // [2, kDecodeMaxPairs] readiness counters (parity double-buffered)
    uint32_t* err;
    int T, E, K, H, F, scoring, accumulate;
    uint32_t epoch;        // call counter: selects the counter parity
    int NS;                // ring stages
    int nwc;               // consumer warps that take ring stages round-robin
    uint32_t slot_bytes;   // bytes per ring stage
    int rs_bf16, rs_q8;    // down rows per phase-2 stage
    int act_resident;      // 1: all activations staged in shared memory at once; 0: two rolling slots
    int x_f32;             // 1: x widened to fp32 in shared memory (small batches); 0: bf16 x
    uint32_t off_ring, off_x, off_ybuf;  // dynamic shared-memory offsets
    int hr_max;            // max output rows per CTA (ybuf row pitch)
    uint64_t timeout_ns;   // bound on every device-side wait
    int inject_timeout;    // test hook: wait for a readiness count that never arrives
    uint64_t* timeline;    // optional [grid][kTimelineSlots] per-CTA phase stamps (globaltimer ns), else null
    int ns_cap;            // tuning: cap on ring stages (0 = as many as shared memory allows)
    uint64_t* stage_log;   // optional [3][kStageLogMax] issue / landed / released stamps of CTA 0's stages
};

// Host-side planning: shared-memory size and stage geometry for (T, H, F, K) on `grid` CTAs.
// Returns false when the shape does not fit the fused kernel.
bool plan_decode(DecodeArgs& a, int grid, size_t* smem_bytes);

// Both launches use programmatic dependent launch: the plan kernel (one CTA) runs beside the
// previous decode grid on the SM that grid leaves free.
cudaError_t launch_plan(const PlanArgs& p, cudaStream_t st);
cudaError_t launch_decode(const DecodeArgs& a, int grid, size_t smem, cudaStream_t st);

cudaError_t decode_set_smem_limit();
cudaError_t plan_set_smem_limit();

}  // namespace moe
