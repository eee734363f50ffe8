// Fused decode path: one persistent decode kernel per call (routing, expert GEMV, combine), launch interface.
#pragma once
#include "common.cuh"

namespace moe {

constexpr int kDecodeMaxT = 16;  // largest batch the fused decode path takes
constexpr int kDecodeMaxPairs = kDecodeMaxT * kMaxTopK;
constexpr int kGroupMax = 4;     // tokens of one token group (their x / y slices live in registers)
constexpr int kMaxGroups = kDecodeMaxPairs;
constexpr int kPlanMaxGrid = 256;  // largest decode grid
constexpr int kSegPerCta = 8;      // segments (runs of one token group's units) per decode CTA
constexpr int kMaxSegTotal = kPlanMaxGrid + kMaxGroups;  // segments of one call: <= grid + groups
// Fused decode defaults: reducing CTAs (0 = every CTA) and how much smaller (in bf16 stream bytes)
// the shares of the CTAs that start when the previous call's reducers leave their SMs are.  Measured
// on B200 at the Solar shape, back-to-back layers: batch 1 49.5 -> 43.8 us per layer against every
// CTA reducing (flat within 1 us for 32-64 reducers and 24-40 units), batch 4 124 -> 98 us.
constexpr int kReducersDefault = 48;
constexpr int kReducersDefaultEp8 = 96;  // expert-parallel contexts of eight or more ranks
constexpr bool kPlannerDefault = true;
constexpr long long kLateBytesDefault = 28 * 24576;
// expert-parallel contexts: the reducers also exchange with the other ranks, so the late CTAs start
// later (measured on two B200, unit-sharded Solar layers: 29.7 us per layer at 56 units, 33.0 at 28)
constexpr long long kLateBytesDefaultEp = 56 * 24576;
constexpr int kTimelineSlots = 24;  // per-CTA stamps recorded when DecodeArgs::timeline is set
constexpr int kStageLogMax = 1024;  // stages of CTA 0 recorded in DecodeArgs::stage_log

// One segment: units [f0, f0 + nu) of one token group's expert, a contiguous run of the unit table.
struct __align__(16) Seg {
    const unsigned char* src;  // unit f0
    const float* sc;           // int8 scales [2F + H] of the expert (down scales at 2F), null for bf16
    int kind, f0, nu, nt;      // expert kind, first unit, units, tokens of the group (1..kGroupMax)
    int gidx, grp, pad0, pad1; // partial-sum slot (share * kSegPerCta + k), token group
    int tok[kGroupMax];        // the group's token rows of x
};

// One decode CTA's share: its segments (in stream order) and the output quads it reduces.
struct __align__(16) PlanCta {
    int nseg, nstage, q0, q1;          // segments, ring stages, output quads [q0, q1) of H/4
    int seg_stage[kSegPerCta + 1];     // first ring stage of each segment
    int nred;                          // the call's reducing CTAs (the last nred to arrive)
    int pad[2];
    Seg seg[kSegPerCta];
};

// Reduction tables of one call (built inside every decode CTA).
struct __align__(16) PlanShared {
    int T, np, ngrp, nsegtot;
    int sp0, pad_[3];                        // block calls: first pair of the shared expert (pair sp0 + t = token t)
    int gvs0[kMaxGroups], gvs1[kMaxGroups];  // call-wide segment range [gvs0, gvs1) of each token group
    int pgrp[kDecodeMaxPairs];               // token group of pair p (pairs job-major)
    int prow[kDecodeMaxPairs];               // row of pair p inside its group
    float pw[kDecodeMaxPairs];               // routing weight of pair p
    int tpn[kDecodeMaxT];                    // local pairs of token t
    int tpair[kDecodeMaxT][kMaxTopK];        // token t's pairs in job order
    int segrows[kMaxSegTotal];               // rows (tokens) of each call-wide segment's partial sums
    int srow0[kMaxSegTotal + 1];             // first staged row of each call-wide segment (prefix of segrows)
};
static_assert(sizeof(Seg) == 64, "Seg layout");
static_assert(sizeof(PlanShared) % 16 == 0 && sizeof(PlanCta) % 16 == 0, "plan structs are 16-byte multiples");

// Expert-parallel combine over NVLink peer memory.  Every rank owns an exchange buffer
// x[2][world][tstride][H] of 64-bit words (call parity, source rank, token, element).  For each
// output slice (the quads one reducing CTA owns, the same slicing on every rank) a rank stores every
// value of its partial into every rank's buffer as one word {epoch, fp32 bits} -- an aligned 64-bit
// store is single-copy atomic, so a reader polls each word until it carries the call's epoch, with no
// fence and no flag (the low-latency protocol of NCCL's LL transport) -- and adds the ranks' values
// in rank order: every rank ends with the same full output, bit for bit.  Buffers alternate by call
// parity, so a rank one call ahead never overwrites words a slower rank still reads.
constexpr int kEpMaxT = 64;      // the exchange buffer holds at least this many tokens per slot
constexpr int kEpMaxTcap = 2048; // and at most this many (longer calls exchange in chunks of it)
constexpr int kEpMaxWorld = 8;  // ranks of one box
struct EpExchange {
    uint64_t* const* peer_x;       // [world] every rank's exchange buffer (peer pointers; own = local)
    const uint64_t* x_local;       // this rank's exchange buffer
    int rank, world;
    uint32_t epoch;                // this call's exchange number (same on all ranks), >= 1
    int tstride;                   // tokens per (parity, rank) slot of the buffers
};

struct PubPlan;

struct DecodeArgs {
    // a plan published by the call's planner kernel (null: none); a CTA that finds pub_flag == stamp
    // when it starts copies its share from it instead of planning itself
    const PubPlan* pub;
    const uint32_t* pub_flag;
    uint32_t stamp;
    // routing inputs (every CTA routes the call itself unless the published plan is ready)
    const float* logits;   // [T, E] fp32 device memory (host calls: the device copy the kernel makes)
    const float* bias;     // [E] or null (sigmoid scoring)
    const ExpDesc* desc;   // [E] expert table of the layer
    const ExpDesc* shared; // block calls: the layer's shared expert, appended as one more job whose
                           //   pairs are every token with weight 1 (kept out of the routed sum)
    int32_t* idx_out;      // [T, K] router indices (written by CTA 0), or null
    float* w_out;          // [T, K] router weights, or null
    // host calls: pinned host sources copied into x / logits on the device.  hctr[0] counts, over the
    // context's host calls, the CTAs whose slice of x is in place (this call's are all in once it
    // reaches hbase + G); hctr[1] holds the number (hidx + 1) of the latest host call whose logits CTA 0
    // copied (wrapping 32-bit arithmetic for both)
    const uint16_t* x_src;
    const float* lg_src;
    uint32_t* hctr;
    uint32_t hbase;
    uint32_t hidx;
    const uint16_t* x;     // [T, H] bf16
    float* out;            // [T, H] fp32, 16-byte aligned (device or device-accessible pinned host memory)
    float* part;           // [grid * kSegPerCta, kGroupMax, H] fp32 partial sums of this call (one of two
                           //   buffers, by call parity): block s * kSegPerCta + k holds the k-th segment
                           //   of CTA s's share
    unsigned long long* cnt; // [4] monotonic over the context's fused calls: [0] / [3] CTAs arrived (even /
                             //   odd calls; call e owns [(e/2) * G, (e/2 + 1) * G) of its counter),
                             //   [1] CTAs finished (outputs written, or none to write), [2] CTAs past their
                             //   partial-sum reads.  Call e on G CTAs owns [e * G, (e + 1) * G) of [1] and
                             //   [2].  Its CTAs write partial sums once call e - 2 staged its own
                             //   (cnt[2] >= (e - 1) * G), and its reducers write outputs once call e - 1
                             //   finished (cnt[1] >= e * G), so a call streams while the previous one
                             //   reduces and exchanges, and no grid waits for a planner
    unsigned long long* decide; // [4] calls planned in every CTA: word e % 4 holds (e << 8) | streamed, set by
                                //   the first CTA of call e (compare-and-swap) from whether call e - 1 was still
                                //   running, so every CTA cuts the same shares
    int nred;              // streamed calls' reducing CTAs: the last nred CTAs to arrive reduce one output
                           //   slice each, the others exit at once, freeing their SMs for the next call.
                           //   The planner applies it (PlanCta::nred) when it finds the previous call
                           //   still running; every other call reduces on all CTAs
    int nlate;             // streamed calls: the last nlate CTAs (by index) get shares smaller by
                           //   late_cost: they start when the previous call's reducers leave their SMs
    long long late_cost;   // (unit_cost units)
    uint32_t* err;
    uint32_t* err_host;    // optional host-mapped words: [0] the call's error bits, [1] its completion tag
                           //   (epoch + 1), stored (release, system scope) by the CTA that finishes last
    int T, E, K, H, F, scoring, accumulate;
    uint32_t epoch;        // call counter: selects the counter parity
    int NS;                // ring stages
    int ch;                // 256-element chunks per lane and row (H <= 2048 * ch)
    int gmax;              // tokens per token group
    int ups_bf16, ups_q8;  // units per ring stage of each kind
    uint32_t slot_bytes;   // bytes per ring stage
    uint32_t off_ring;     // dynamic shared-memory offset of the ring
    uint64_t timeout_ns;   // bound on every device-side wait
    int inject_timeout;    // test hook: the grid barrier waits for one CTA more than the grid
    uint64_t* timeline;    // optional [grid][kTimelineSlots] per-CTA stamps, else null
    uint64_t* stage_log;   // optional [3][kStageLogMax] issue / landed / released stamps of CTA 0's stages
    int ns_cap;            // tuning: cap on ring stages (0 = as many as shared memory allows)
    uint32_t stage_target; // tuning: target bytes per ring stage (0 = default)
    int q8_cost;           // planning cost of one int8 unit in bf16-stream bytes (0 = default,
                           //   kQ8CostDefault per mille of the unit's bytes)
    EpExchange ep;         // cross-rank combine (ep.world > 1 with peers attached), else world = 0
    // block calls (plan with a shared expert): instead of out, x_next = bf16((y + extra) + routed)
    // with y = bf16(x2 + shared); y_out (optional) receives y; extra may be null
    int block;
    const uint16_t* x2;
    const float* extra;
    uint16_t* x_next;
    uint16_t* y_out;
};

// Host-side planning: shared-memory size and stage geometry for (T, H, F) on `grid` CTAs.
// Returns false when the shape does not fit the fused path.
bool plan_decode(DecodeArgs& a, int grid, size_t* smem_bytes);

// Per call: the planner kernel (one CTA, published plan) and the decode grid, both with programmatic
// dependent launch.  The planner runs on the SM the decode grid leaves free, so for back-to-back
// calls the next plan is usually ready before its decode CTAs start; a decode CTA that finds it not
// ready plans itself (the same code, the same bits).
cudaError_t launch_planner(const DecodeArgs& a, int grid, PubPlan* out, uint32_t* flag, uint32_t stamp, cudaStream_t st);
cudaError_t launch_decode(const DecodeArgs& a, int grid, size_t smem, cudaStream_t st);
size_t pub_plan_bytes();

cudaError_t decode_set_smem_limit();
// True when every decode kernel instantiation is launched with enough registers per thread for its
// producer / consumer register split (otherwise the fused path must not be used).
bool decode_register_split_fits();

// Cross-rank combine of out[t0 .. t0+T) for a T <= ep.tstride chunk already holding this rank's
// partial (multi-kernel and prefill paths): `part` is the local partial [T, H], `out` receives base
// (accumulate) + the sum over ranks; grid = the decode grid size G (same output slicing on every
// rank).  One launch pushes every value of the chunk to every rank, then collects: one round of
// exchange latency per call however many tokens it has.
cudaError_t launch_ep_exchange(const EpExchange& ep, const float* part, float* out, int T, int H, int accumulate,
                               uint32_t* err, uint64_t timeout_ns, int grid, cudaStream_t st);

// Partial-sum floats the decode path needs for hidden size H on a grid of G CTAs.
// Floats of one partial-sum buffer (a context holds two, used by alternate calls).
inline size_t decode_part_floats(int H, int G) { return (size_t)G * kSegPerCta * kGroupMax * H; }

}  // namespace moe
