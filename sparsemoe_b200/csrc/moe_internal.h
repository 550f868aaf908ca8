// Internal interfaces between the orchestration (moe.cu) and the kernels.
#pragma once

#include <cstddef>
#include <cstdint>
#include <cuda_runtime.h>
#include "../../include/sparsemoe_b200.h"

namespace moe {

// Routes per dispatch chunk: the unit of the deterministic slot scan.
constexpr int kChunkRoutes = 1024;

// Experts from which the router switches to its register-tiled kernel and
// the sequential-j logit order (the oracle follows the same rule).
constexpr int kRouterTiledMinExperts = 64;
// Below this many tokens, many-expert routers split the experts over CTAs
// so that small batches fill the GPU.
constexpr int64_t kRouterSliceMaxT = 2048;
// Many-expert routers cut d into blocks of this many j's: each block is one
// fmaf chain (a CTA's work), and the blocks are summed by a fixed tree in a
// separate fold + top-k pass (the oracle follows the same order).
constexpr int kRouterBlockJ = 512;

// Error codes the kernels write to the device status word.
constexpr int kDevErrTimeout = 1;

struct Shape {
    int B, N, d, f, E, k, cap;
    int dtype;         // MOE_DTYPE_*
    int router_dtype;  // MOE_ROUTER_*
    bool act_bf16;     // x (and the 16-bit output copy) are bf16 rather than f16
    int64_t T() const { return (int64_t)B * N; }
    int chunks() const { return (int)(((int64_t)N * k + kChunkRoutes - 1) / kChunkRoutes); }
    int64_t rows_capacity() const { return (int64_t)E * B * cap; }  // rows of the per-expert buffers
};

// Most row groups one grouped-GEMM launch takes (experts, or (sender, expert)
// blocks under expert parallelism).
constexpr int kMaxGroups = 1024;

// Device scratch owned by the library (one block per device, grown on demand).
// A fixed-size header (status word, GEMM group table) comes first, so calls
// with different shapes never move it; the routing tables follow.
struct Workspace {
    int* status;        // [1]       device error word (kDevErrTimeout, ...)
    int* grp_rows;      // [kMaxGroups] rows of each GEMM group (expert-parallel calls)
    int* grp_start;     // [kMaxGroups] first row of each group
    int* grp_weight;    // [kMaxGroups] expert weight index of each group
    int* grp_out_rank;  // [kMaxGroups] peer that receives each group's output rows
    int* grp_out_row;   // [kMaxGroups] first output row of each group there
    int* route_slot;    // [B*N*k]   slot of each route, -1 if dropped / no expert
    int* chunk_count;   // [B, chunks, E] routes per (batch, chunk, expert)
    int* chunk_base;    // [B, chunks, E] exclusive prefix over chunks
    int* row_base;      // [B, E]    first row of (b, e) inside expert e's block
    int* expert_rows;   // [E]       kept rows of expert e over all batches
    int* expert_start;  // [E]       first row of expert e: exclusive prefix of expert_rows
    float* a_scale;     // FP8: [E*B*CAP, d/128] activation block scales; INT8_CHANNEL: [E*B*CAP] row scales
    float* h_scale;     // FP8 / INT8_CHANNEL: [E*B*CAP, f/128] h block scales
    float* router_logits;  // [ceil(d/512), T, E] per-block partial logits of the many-expert routers
};
size_t workspace_header_bytes();

// Row groups of one grouped GEMM: group g has rows[g] rows starting at row
// start[g] of the A/H/Y buffers (capacity rows_capacity) and multiplies expert
// weight[g] (weight == nullptr: group g uses expert g).  Device arrays.
constexpr int kMaxPeers = 8;
// Optional redirect of the down GEMM's output rows (expert parallelism over
// peer memory): group g's rows go to bases[rank[g]] from row row0[g] on (rows
// of out_ld f32), instead of the local Y at the group's start row.  The
// epilogue then ends with a system-scope fence.
struct OutRedirect {
    const int* rank = nullptr;   // [G] device
    const int* row0 = nullptr;   // [G] device
    float* bases[kMaxPeers] = {};
};

// Destination of the gathered rows: the local buffers (rows[0], scales[0],
// row = expert_start[e] + ...) or, under expert parallelism over peer memory,
// expert e's owner: rows[rank[e]] / scales[rank[e]] from row row0[e] + the
// (batch, slot) offset on.  rank / row0 are device arrays of E.
struct GatherDst {
    void* rows[kMaxPeers] = {};
    float* scales[kMaxPeers] = {};
    const int* rank = nullptr;
    const int* row0 = nullptr;
};

struct GroupTable {
    const int* rows;
    const int* start;
    const int* weight;
    int G;
    int64_t rows_capacity;
    OutRedirect redirect = {};
};
size_t workspace_bytes(const Shape& s);
void carve_workspace(void* base, const Shape& s, Workspace* ws);

// Per-tensor scales of the int8 path (MoEArgs scale_* fields).
struct GemmScales {
    float s_in = 1.0f, s_gate = 1.0f, s_up = 1.0f, s_mid = 1.0f, s_down = 1.0f;
};

// router.cu: logits (+bias), warp-shuffle top-k, softmax.
// True when the router runs expert-sliced (E >= 64, E % 32 == 0, T < kRouterSliceMaxT).
bool router_sliced(const Shape& s);
// True for the many-expert routers (E >= 64, E % 32 == 0): per-block partials + fold.
bool router_blocked(const Shape& s);
cudaError_t launch_router_topk(const void* x, const void* wr, const float* bias, const Shape& s,
                               float* logits_scratch,
                               float* logits, int* idx, float* w, cudaStream_t st);
// dispatch.cu: deterministic capacity slots + 16-byte row gather.
// a_rows receives 16-bit rows, or int8 rows quantised with 1/s_in (int8 path).
// Two phases (a batch split over expert-parallel ranks needs the totals of
// every shard in between): route histogram (+ the shard's raw per-(batch,
// expert) totals), then slots with the earlier shards' slot_base, drops,
// tables and (unless skipped) the gather.
cudaError_t launch_dispatch_count(const int* idx, const Shape& s, const Workspace& ws, int* counts, int* raw,
                                  cudaStream_t st);
cudaError_t launch_dispatch_finish(const void* x, const int* idx, const float* w, const Shape& s,
                                   const Workspace& ws, const GemmScales& sc, const int* slot_base, int* counts,
                                   int* token_ids, float* token_weights, void* a_rows, cudaStream_t st,
                                   bool skip_gather);
cudaError_t launch_ep_plan(const int* table, int P, int E, int me, int strided, int* plan, cudaStream_t st);
cudaError_t launch_dispatch_gather(const void* x, const int* idx, const Shape& s, const Workspace& ws,
                                   const GemmScales& sc, const GatherDst& gd, cudaStream_t st);
// expert_gemm.cu: grouped tcgen05 GEMMs.
cudaError_t launch_expert_up_gate(const void* a_rows, const void* w_gate, const void* w_up,
                                  const Shape& s, const GroupTable& gt, int* status, const GemmScales& sc,
                                  void* h_rows, cudaStream_t st, int num_sms);
cudaError_t launch_expert_down(const void* h_rows, const void* w_down, const Shape& s,
                               const GroupTable& gt, int* status, const GemmScales& sc, float* y_rows,
                               cudaStream_t st, int num_sms);
// expert_gemm_fp8.cu: block-scaled e4m3 GEMMs.
cudaError_t launch_fp8_up_gate(const void* a_rows, const float* a_scale, const void* w_gate, const void* w_up,
                               const float* s_gate, const float* s_up, const Shape& s, const GroupTable& gt,
                               int* status, void* h_rows, float* h_scale, cudaStream_t st, int num_sms);
cudaError_t launch_fp8_down(const void* h_rows, const float* h_scale, const void* w_down, const float* s_down,
                            const Shape& s, const GroupTable& gt, int* status, float* y_rows, cudaStream_t st,
                            int num_sms);
// expert_gemm_fp8.cu, int8 form: per-output-channel weight scales, per-row x
// scales, per-(row, 128-feature block) h scales.
cudaError_t launch_i8c_up_gate(const void* a_rows, const float* a_scale, const void* w_gate, const void* w_up,
                               const float* s_gate, const float* s_up, const Shape& s, const GroupTable& gt,
                               int* status, void* h_rows, float* h_scale, cudaStream_t st, int num_sms);
cudaError_t launch_i8c_down(const void* h_rows, const float* h_scale, const void* w_down, const float* s_down,
                            const Shape& s, const GroupTable& gt, int* status, float* y_rows, cudaStream_t st,
                            int num_sms);

// selftest.cu: one CTA whose bounded mbarrier wait runs out after timeout_ns
// (nothing arrives) and records kDevErrTimeout in *status.
cudaError_t launch_wait_selftest(int* status, uint64_t timeout_ns, cudaStream_t st);

// expert_gemm_i4.cu: the reference's packed-transposed int4 format (int4
// values in int8 A rows, weights as packed pairs [E * N/2, K] bytes), exact
// kind::i8 MMAs on nibbles sign-extended in shared memory.
cudaError_t launch_i4_up_gate(const void* a_rows, const void* w_gate, const void* w_up, const Shape& s,
                              const GroupTable& gt, int* status, const GemmScales& sc, void* h_rows, cudaStream_t st,
                              int num_sms);
cudaError_t launch_i4_down(const void* h_rows, const void* w_down, const Shape& s, const GroupTable& gt, int* status,
                           const GemmScales& sc, float* y_rows, cudaStream_t st, int num_sms);

// expert_gemm_w4.cu: 4-bit weights dequantised to bf16 in shared memory.
cudaError_t launch_w4_up_gate(const void* a_rows, const void* w_gate, const void* w_up, const void* s_gate,
                              const void* s_up, const void* z_gate, const void* z_up, const Shape& s,
                              const GroupTable& gt, int* status, void* h_rows, cudaStream_t st, int num_sms);
cudaError_t launch_w4_down(const void* h_rows, const void* w_down, const void* s_down, const void* z_down,
                           const Shape& s, const GroupTable& gt, int* status, float* y_rows, cudaStream_t st,
                           int num_sms);
// expert_gemm_w4.cu, NVFP4 form: e2m1 nibbles, e4m3 scales per 16 K-rows, f32
// global scale per expert matrix.
cudaError_t launch_fp4_up_gate(const void* a_rows, const void* w_gate, const void* w_up, const void* s_gate,
                               const void* s_up, const float* g_gate, const float* g_up, const Shape& s,
                               const GroupTable& gt, int* status, void* h_rows, cudaStream_t st, int num_sms);
cudaError_t launch_fp4_down(const void* h_rows, const void* w_down, const void* s_down, const float* g_down,
                            const Shape& s, const GroupTable& gt, int* status, float* y_rows, cudaStream_t st,
                            int num_sms);

// combine.cu: gate-weighted gather-sum into [B, N, d].
cudaError_t launch_combine(const float* y_rows, const int* idx, const float* w, const Shape& s,
                           const Workspace& ws, float* out, void* out16, cudaStream_t st,
                           const void* residual = nullptr);
// norm.cu: RMSNorm of the [T, d] input rows into out (MoeDims.norm_* semantics).
cudaError_t launch_rmsnorm(const void* x, const void* g, const Shape& s, float eps, void* out, cudaStream_t st);

void set_error(const char* fmt, ...);

// moe.cu: shared pieces of the layer entry points.
int make_shape_checked(const MoeDims* dims, Shape* s);
int check_args_16(const MoEArgs* a);
int check_args(const MoEArgs* a, int dtype);
int check_norm(const MoeDims* dims);
int current_device(int* dev, int* num_sms);           // sm_100 check, cached SM count
void note_status_word(int dev, int* status);            // read by moe_check_device_status
int enqueue_layer(const MoEArgs* a, const MoeDims* dims, const Shape& s, const Workspace& ws, int num_sms,
                  cudaStream_t stream);

}  // namespace moe
