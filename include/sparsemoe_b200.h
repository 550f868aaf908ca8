// C ABI of the B200 capacity-routed MoE layer (libsparsemoe_b200.so).
//
// Plain pointers, sizes and a cudaStream_t only.  Each entry point names the
// reference interface it replaces (paths are within MattJBorowski1991/SparseMoE).
#pragma once

#include <stddef.h>
#include <stdint.h>
#include "moe_args.h"

#ifdef __cplusplus
extern "C" {
#endif

// ---- status codes (moe_solve_v2 and friends) ------------------------------
#define MOE_OK                 0
#define MOE_ERR_INVALID_ARG   -1   // null pointer / bad shape
#define MOE_ERR_UNSUPPORTED   -2   // shape or dtype this build has no kernel for
#define MOE_ERR_CUDA          -3   // a CUDA runtime/driver call failed
#define MOE_ERR_TIMEOUT       -4   // a device-side bounded wait gave up
#define MOE_ERR_NO_KERNEL     -5   // the sm_100a kernels cannot run on this device

// ---- activation / weight formats ------------------------------------------
#define MOE_DTYPE_F16   0   // fp16 weights/activations (reference kernels/capacity.cu)
#define MOE_DTYPE_BF16  1   // bf16 bit patterns in the same `half*` fields
#define MOE_DTYPE_INT8  2   // per-tensor int8 weights/activations, s32 accumulate, f16 x and router
                            // (reference kernels/capacity_int8_ptx.cu; MoEArgs *_int8 fields + scales)
#define MOE_DTYPE_FP8_BLOCK 3  // e4m3 weights with f32 scales per 128x128 block (MoeDims.w_scale_*),
                               // activations and h quantised on the fly per 1x128 block, bf16 x and
                               // router, f32 accumulate; MoEArgs *_fp8 fields
#define MOE_DTYPE_W4A16 4      // 4-bit weights: INT4 asymmetric, group 128 along K, fp16 scale and
                               // zero per (group, column) (MoeDims.w4_*), nibble-packed [E, K, N/2]
                               // (pair-interleaved words, see moe_quantize_int4_g128)
                               // in the MoEArgs *_int4 fields; bf16 x, router and h
#define MOE_DTYPE_NVFP4 6   // NVFP4 weights: e2m1 nibbles packed as for MOE_DTYPE_W4A16 in the *_int4
                            // fields, one e4m3 scale per (16 K-rows, column) (MoeDims.w4_scale_*:
                            // gate/up [E, d/16, f], down [E, f/16, d]) and one f32 global scale per
                            // expert matrix (MoeDims.fp4_global_*); w = e2m1 * scale * global;
                            // bf16 x, router and h
#define MOE_DTYPE_INT4_PTX 7   // the reference's int4 format (kernels/capacity_int4_ptx.cu:166-307,396-486,
                               // 586-675; inputs/data.cu:89-140): per-tensor int4 weights (max/7) packed
                               // transposed, per expert [N/2][K] bytes, columns 2p (low nibble) and 2p+1
                               // (high) of row k at byte (p, k), in the MoEArgs *_int4 fields; f16 x and
                               // router; x and h quantised per tensor to int4 values rn(clamp(v/s, -7, 7)),
                               // kept one per byte in per_expert_wmma_inputs_int8 and
                               // hidden_mlp_layer_1_out_int8; s32 accumulate; the MoEArgs scales.
                               // The GEMMs read the packed weights as they are (nibbles are
                               // sign-extended in shared memory).
#define MOE_DTYPE_FP8 8        // the reference's fp8 format (kernels/capacity_fp8_ptx.cu:98-220,330-395,
                               // 566-670; inputs/data.cu:142-150): e4m3 weights in the MoEArgs *_fp8
                               // fields with per-tensor scales (the builder's are 1.0); f16 x and router;
                               // x and h quantised as e4m3(clamp(v/s, -448, 448)); f32 accumulate
#define MOE_DTYPE_INT8_CHANNEL 5   // int8 weights with one f32 scale per output channel (MoeDims.w_scale_*:
                                   // gate/up [E, f], down [E, d]); x quantised per token (amax / 127) on
                                   // the fly, h per token and 128-feature block; s32 accumulate; bf16 x
                                   // and router; MoEArgs *_int8 fields

// ---- router formats --------------------------------------------------------
#define MOE_ROUTER_SAME 0   // router_weights have the activation dtype
#define MOE_ROUTER_F32  1   // router_weights point to f32 [d, E]

// Runtime shape of one layer call.  The reference fixes these at compile time
// (include/config.h:6-38); here they travel with the call.
typedef struct MoeDims {
    int   num_batches;      // B: independent routing groups (blockIdx.z in the reference)
    int   tokens;           // N: tokens per batch
    int   d_model;          // d  (multiple of 256)
    int   d_ff;             // f  (multiple of 128)
    int   num_experts;      // E  (multiple of 8, <= 256)
    int   top_k;            // k  (1..32, <= E)
    float capacity_factor;  // cf
    int   cap;              // >0: use this CAP;  0: CAP = moe_capacity(N,k,E,cf);  -1: no drop (CAP = N)
    int   dtype;            // MOE_DTYPE_*
    int   router_dtype;     // MOE_ROUTER_*
    const float* router_bias;  // optional device [E] f32 added to every logit (Zipf popularity bias)
    void* output_16;        // optional device [B, N, d] copy of the output in the 16-bit dtype
    void* scratch;          // optional caller device memory for the library's routing tables
    size_t scratch_bytes;   //   (>= moe_workspace_bytes(dims)); NULL: the library's own block
    // weight scales (device f32).  MOE_DTYPE_FP8_BLOCK: gate/up [E, d/128, f/128], down [E, f/128, d/128];
    // MOE_DTYPE_INT8_CHANNEL: gate/up [E, f], down [E, d]
    const float* w_scale_gate;
    const float* w_scale_up;
    const float* w_scale_down;
    // MOE_DTYPE_W4A16 group scales and zeros (device fp16): gate/up [E, d/128, f], down [E, f/128, d];
    // MOE_DTYPE_NVFP4 uses w4_scale_* for its e4m3 block scales (see above)
    const void* w4_scale_gate;
    const void* w4_scale_up;
    const void* w4_scale_down;
    const void* w4_zero_gate;
    const void* w4_zero_up;
    const void* w4_zero_down;
    // MOE_DTYPE_NVFP4 per-expert global scales (device f32 [E] each)
    const float* fp4_global_gate;
    const float* fp4_global_up;
    const float* fp4_global_down;
    // Expert parallelism over a batch split across ranks (global capacity).
    // Optional device int32 [B, E]: for each (batch, expert) the slots that the
    // routes of earlier shards of the same batch already took; this call keeps
    // a route iff slot_base + its slot within this shard < cap.  NULL: 0.
    const int* slot_base;
    // Optional device f32 buffer for the per-row activation scales of the
    // dynamically quantised formats (FP8_BLOCK [rows, d/128], INT8_CHANNEL
    // [rows]): written by the gather, read by the up/gate GEMM.  NULL: scratch.
    float* act_scale;
    // Non-zero: the routing stages stop before the gather (expert parallelism
    // over peer memory, where moe_stage_dispatch_peer gathers into the owners).
    int skip_gather;
    // The stages either side of the layer (no reference counterpart; a
    // transformer block's pre-MoE norm and residual connection).  Optional:
    // norm_weight (device [d], the activation dtype) turns on an RMSNorm of
    // the input rows before the router, written to norm_out (device [B, N, d],
    // the activation dtype; required with norm_weight), which the router and
    // the gather then read:  xn = round16((x * g) / sqrt(sum(x^2) / d + eps)).
    // residual (device [B, N, d], the activation dtype) is added to every
    // output row in the combine (out = residual + sum_l w_l y_l, the sum in
    // route order), usually the un-normalised input.
    const void* norm_weight;
    float norm_eps;
    void* norm_out;
    const void* residual;
} MoeDims;

// Reference: kernels/launcher.h:21 `extern "C" void solve(MoEArgs args)`.
// Runs the whole layer for the dims set by moe_set_solve_dims (defaults: the
// reference's include/config.h), synchronises the device, prints
// "Total duration via cudaEventRecord: %.3f ms" and exits(1) on any error,
// exactly as the reference launcher does.  The format path is chosen from the
// non-null weight fields, as the reference's allocators fill them
// (drivers/main.cu:84-106): fp16 weights -> `capacity` (or the bf16 / other
// 16-bit-field formats set by moe_set_solve_dims); *_int4 weights ->
// `capacity_int4_ptx` (MOE_DTYPE_INT4_PTX); *_int8 weights alone ->
// `capacity_int8_ptx` (MOE_DTYPE_INT8); *_fp8 weights -> `capacity_fp8_ptx`
// (MOE_DTYPE_FP8).
void solve(struct MoEArgs args);

// Status-returning, stream-ordered form of solve() with runtime dims.
// Asynchronous: returns once the layer is enqueued on `stream`.
int moe_solve_v2(const struct MoEArgs* args, const MoeDims* dims, cudaStream_t stream);

// No reference counterpart.  Same as moe_solve_v2, but the library allocates
// nothing: its scratch lives in a static device array of
// moe_noalloc_scratch_bytes() (4 MiB) per GPU, held until process exit.  For
// callers that cannot let the library call cudaMalloc (engines that own all
// device memory through a pre-planned pool; serving loops that cannot take
// the device synchronisation of cudaMalloc/cudaFree).  Calls needing more
// scratch than the array (moe_workspace_bytes) fail with MOE_ERR_UNSUPPORTED.
// All calls on a device share the array: calls that overlap on the GPU race.
// The first call on a device resolves the array's address (cudaGetSymbolAddress)
// and caches it for the life of the CUDA context (stale after cudaDeviceReset);
// make it before any stream capture.  dims->act_scale is honoured as in
// moe_solve_v2; dims->scratch must be null (MOE_ERR_INVALID_ARG otherwise).
int moe_solve_v2_noalloc(const struct MoEArgs* args, const MoeDims* dims, cudaStream_t stream);
size_t moe_noalloc_scratch_bytes(void);

// ---- expert-parallel building blocks (no reference counterpart: the reference
//      is single-GPU).  One layer call = moe_stage_route -> (exchange rows) ->
//      moe_stage_expert_ffn on the owner -> (exchange rows back) ->
//      moe_stage_combine, with the same dims for route and combine, on one
//      device and host thread.
// Router, top-k, capacity slots (kept iff slot < CAP, route-id order within a
// batch) and the gather of the kept token rows into per_expert_wmma_inputs in
// the dense expert-major layout: expert e's rows start at
// sum_{e'<e} sum_b expert_counts[b, e'], batch 0's slots first.
int moe_stage_route(const struct MoEArgs* args, const MoeDims* dims, cudaStream_t stream);
// The same stage in two phases, for a batch split across ranks: phase 1
// (router, top-k, per-(batch, expert) route totals of this shard before any
// drop, written to raw_counts: device int32 [B, E]); the caller exchanges the
// totals and sets dims.slot_base; phase 2 (slots, drops, gather) on the same
// dims and scratch.
int moe_stage_route_counts(const struct MoEArgs* args, const MoeDims* dims, int* raw_counts,
                           cudaStream_t stream);
int moe_stage_route_finish(const struct MoEArgs* args, const MoeDims* dims, cudaStream_t stream);
// SwiGLU FFN over row groups: group g has group_rows[g] rows starting at row
// group_start[g] of per_expert_wmma_inputs (A), hidden_mlp_layer_1_out_fp16
// (H) and hidden_mlp_layer_2_out (Y, f32), all with rows_capacity rows, and
// uses expert group_expert[g] (NULL: g) of the dims.num_experts experts whose
// weights args holds.  The three arrays are host memory (copied on `stream`).
int moe_stage_expert_ffn(const struct MoEArgs* args, const MoeDims* dims, const int* group_rows,
                         const int* group_start, const int* group_expert, int num_groups,
                         int64_t rows_capacity, cudaStream_t stream);
// The FFN stage with its output rows sent to peers: group g's rows of Y go to
// out_bases[group_out_rank[g]] from row group_out_row[g] on (f32 rows of
// d_model), written by the down GEMM's epilogue (NVLink stores from inside the
// GEMM, so the return transfer overlaps it) instead of hidden_mlp_layer_2_out.
// out_bases are device pointers valid in this process (moe_peer_open), at most
// 8.  The caller orders the peers' later reads after this stage (a barrier).
int moe_stage_expert_ffn_peer(const struct MoEArgs* args, const MoeDims* dims, const int* group_rows,
                              const int* group_start, const int* group_expert, const int* group_out_rank,
                              const int* group_out_row, int num_groups, int64_t rows_capacity,
                              float* const* out_bases, int num_bases, cudaStream_t stream);
// Combine: final_output[t] = sum over kept routes in route order of
// w * Y[row], Y = hidden_mlp_layer_2_out in the layout moe_stage_route made.
int moe_stage_combine(const struct MoEArgs* args, const MoeDims* dims, cudaStream_t stream);
// Scratch (MoeDims.scratch) that moe_stage_expert_ffn needs for rows_capacity
// rows with these dims: the group table, plus the h scales of FP8_BLOCK and
// INT8_CHANNEL (for which caller scratch is required; the row scales of A
// come in MoeDims.act_scale).
size_t moe_ffn_scratch_bytes(const MoeDims* dims, int64_t rows_capacity);

// Expert parallelism over peer memory without host synchronisation.
// moe_ep_plan: from the all-gathered kept-row table [world, E] (device int32,
// rows each rank routes to each expert), writes the device plan of this rank
// (7*E int32) for contiguous ownership (strided == 0: rank q holds experts
// q*E/world .. (q+1)*E/world - 1) or strided ownership (rank q holds experts
// q, q + world, q + 2*world, ...; local index e / world): per expert e the
// owner rank and the first row of this rank's
// block in the owner's receive buffer, then the owner-side row groups
// (local expert j x sender s, g = j*world + s): rows, start row in the
// receive buffer, local expert, sender, and the first row of the group's
// results in the sender's return buffer.
int moe_ep_plan(const int* table, int world, int rank, int num_experts, int strided, int* plan,
                cudaStream_t stream);
// Gathers this rank's kept rows (quantised for the 8-bit formats, with their
// row scales) straight into the owners' receive buffers row_bases[owner]
// (scale_bases[owner]) as the plan places them; the routing tables come from
// moe_stage_route / _finish with dims.skip_gather on the same dims and scratch.
int moe_stage_dispatch_peer(const struct MoEArgs* args, const MoeDims* dims, const int* plan,
                            void* const* row_bases, float* const* scale_bases, int num_bases, cudaStream_t stream);
// The owner FFN over the plan's row groups (device arrays; num_groups =
// E_global), result rows stored into out_bases[sender] by the down GEMM.
// dims.num_experts is the owner's local expert count.
int moe_stage_expert_ffn_planned(const struct MoEArgs* args, const MoeDims* dims, const int* plan,
                                 int num_groups, int64_t rows_capacity, float* const* out_bases, int num_bases,
                                 cudaStream_t stream);

// ---- expert weight files (.bin): a layer's router and expert weights in the
//      formats the kernels read (no repacking on load).  The reference's
//      driver names a cache file it never writes (drivers/main.cu:27-31).
#define MOE_WFILE_MAX_ARRAYS 16
typedef struct MoeWeightArray {
    char name[24];          // "wr", "bias", "wg", "wu", "wd", "wg_q", "sg", "wg_s", "wg_z", "wg_g", ...
    int32_t elem_bytes;     // 1, 2 or 4
    int32_t kind;           // 0 unsigned integer (or 16-bit float bit patterns), 1 signed integer, 2 float
    int32_t ndim;           // 1..4
    int32_t reserved;
    int64_t shape[4];
    uint64_t offset;        // byte offset in the file (256-aligned); set by moe_weights_write
    uint64_t bytes;         // elements x elem_bytes; set by moe_weights_write
} MoeWeightArray;
typedef struct MoeWeightFile {
    char magic[8];          // "SMOEW001"
    int32_t dtype;          // MOE_DTYPE_* of the expert weights
    int32_t router_dtype;   // MOE_ROUTER_*
    int32_t num_experts, d_model, d_ff;
    int32_t num_arrays;
    int32_t reserved;
    MoeWeightArray arrays[MOE_WFILE_MAX_ARRAYS];
} MoeWeightFile;
// Writes the header (magic, offsets and sizes filled in) and data[i] (host
// memory) for each of header->num_arrays arrays.
int moe_weights_write(const char* path, const MoeWeightFile* header, const void* const* data);
// Reads and checks the header (magic, descriptors, sizes within the file).
int moe_weights_read_header(const char* path, MoeWeightFile* header);
// Copies array `index` into dst (host memory of at least its bytes).
int moe_weights_read_array(const char* path, const MoeWeightFile* header, int index, void* dst,
                           size_t dst_bytes);

// Peer memory for expert parallelism (CUDA IPC within a node): allocate a
// device buffer and its 64-byte handle; map a peer's handle in this process;
// unmap; free.  moe_memcpy_async copies between any device pointers
// (a peer's included) on `stream` with the copy engines.
int moe_peer_alloc(size_t bytes, void** ptr, void* handle64);
int moe_peer_open(const void* handle64, void** ptr);
int moe_peer_close(void* ptr);
int moe_peer_free(void* ptr);
int moe_memcpy_async(void* dst, const void* src, size_t bytes, cudaStream_t stream);

// Synchronises `stream` and reports a device-side failure (MOE_ERR_TIMEOUT) of
// the last moe_solve_v2 on this device, MOE_OK otherwise.
int moe_check_device_status(cudaStream_t stream);

// Dims used by solve() and by the input builder (inputs/data.h functions).
int moe_set_solve_dims(const MoeDims* dims);
int moe_get_solve_dims(MoeDims* dims);

// Reference: inputs/data.cu:392-398 and kernels/capacity.cu:502-503:
// CAP = round_up((int)ceilf((float)N*(float)k/(float)E*cf), 16).
int moe_capacity(int tokens, int top_k, int num_experts, float capacity_factor);

// Bytes of device scratch the library keeps for a call with these dims
// (routing tables; the caller's MoEArgs buffers hold everything else).
size_t moe_workspace_bytes(const MoeDims* dims);

// Instrumentation (no reference counterpart; the reference times the whole
// launch only, kernels/launcher.h:23-45).  With 6 cudaEvent_t handles set,
// each later moe_solve_v2 on this host thread records events[i] on its stream
// before stage i (0 router+top-k, 1 dispatch, 2 up/gate GEMM, 3 down GEMM,
// 4 combine) and events[5] after the last one.  count = 0 turns it off.
int moe_set_stage_events(void* const* events, int count);

// Frees the library's cached device scratch on the current device.
void moe_release(void);

// No reference counterpart (the reference has no failure detection).
// Self-test of the bounded device waits every kernel here uses: enqueues one
// CTA that waits on an mbarrier nothing arrives on, for at most timeout_ns
// (0 < timeout_ns <= 10 s); the wait gives up, records a timeout in this
// device's status word and the kernel returns, so the context stays usable.
// A following moe_check_device_status(stream) returns MOE_ERR_TIMEOUT; the
// next layer call clears the word.
int moe_selftest_wait_timeout(int64_t timeout_ns, cudaStream_t stream);

// Text of the last error recorded on this host thread ("" if none).
const char* moe_last_error(void);

// Reference inputs/data.cu:13-57: per-tensor symmetric quantiser of n fp16
// values, scale = max|x| / qmax (1 if all zero), q = nearbyint(clamp(x/scale,
// -qmax, qmax)).  qmax = 127 (int8) or 7 (int4 values).  Returns the scale.
float moe_quantize_per_tensor(const uint16_t* src_f16, size_t n, int8_t* dst, float qmax);

// Reference inputs/data.cu:89-140 (quantize_symmetric_per_tensor_int4_packed_transposed,
// its packing step): int4 values of E row-major [K, N] matrices -> per expert
// [N/2][K] bytes, column 2p in the low and 2p+1 in the high nibble of byte (p, k).
void moe_pack_int4_transposed(const int8_t* q, int E, int K, int N, uint8_t* out);

// Reference inputs/data.cu:142-150 (quantize_per_tensor_fp8_e4m3): n fp16
// values cast to e4m3 (nearest even, saturating to +-448).
void moe_cast_e4m3(const uint16_t* src_f16, size_t n, uint8_t* dst);

// FP8 block quantiser for weights [E, K, N] (16-bit, bf16 != 0: bf16):
// per expert and 128x128 block, s = amax / 448 (1 if the block is zero),
// q = e4m3(x / s) rounded to nearest even, saturating at +-448.
// Writes q [E, K, N] (e4m3 bytes) and scales [E, K/128, N/128].
void moe_quantize_fp8_blocks(const uint16_t* src, int E, int K, int N, int bf16, uint8_t* q, float* scales);

// Per-output-channel int8 quantiser for weights [E, K, N] (16-bit, bf16 != 0:
// bf16): per expert and column n, s = max_k |w| / 127 (1 if the column is
// zero), q = clamp(nearbyint(w / s), -127, 127).  Writes q [E, K, N] and
// scales [E, N].
void moe_quantize_int8_channel(const uint16_t* src, int E, int K, int N, int bf16, int8_t* q, float* scales);

// NVFP4 quantiser for weights [E, K, N] (16-bit, bf16 != 0: bf16): per expert
// g = amax / (448 * 6) (1 if the matrix is zero); per column and group of 16
// along K, s = e4m3(amax_group / (6 * g)) (round to nearest even, saturating;
// a zero group gets s = 1.0), and q = e2m1(w / (s * g)) rounded to the nearest
// of {0, 0.5, 1, 1.5, 2, 3, 4, 6} (ties to the even code), sign in bit 3.
// Writes packed [E, K, N/2] (same pair-interleaved words as
// moe_quantize_int4_g128), e4m3 scales [E, K/16, N] and globals [E].
void moe_quantize_nvfp4(const uint16_t* src, int E, int K, int N, int bf16, uint8_t* packed, uint8_t* scales,
                        float* globals);

// Device twins of the four quantisers above (int8 per channel, FP8 blocks,
// INT4 g128 -- declared below -- and NVFP4): same formats, bit-identical
// outputs, for weights already in device memory; asynchronous on `stream`.
// src must be 16-byte aligned; N a multiple of 8 (FP8: K, N multiples of 128;
// INT4: K of 128; NVFP4: K of 16).  Return MOE_OK or an error code.
int moe_quantize_int8_channel_device(const void* src, int E, int K, int N, int bf16, int8_t* q, float* scales,
                                     cudaStream_t stream);
int moe_quantize_fp8_blocks_device(const void* src, int E, int K, int N, int bf16, uint8_t* q, float* scales,
                                   cudaStream_t stream);
int moe_quantize_int4_g128_device(const void* src, int E, int K, int N, int bf16, uint8_t* packed,
                                  uint16_t* scales, uint16_t* zeros, cudaStream_t stream);
int moe_quantize_nvfp4_device(const void* src, int E, int K, int N, int bf16, uint8_t* packed, uint8_t* scales,
                              float* globals, cudaStream_t stream);

// 4-bit asymmetric group quantiser for weights [E, K, N] (16-bit, bf16 != 0:
// bf16): per expert, column n and group of 128 along K, s = (max - min) / 15
// (1 if max == min), z = -min / s, both rounded to fp16; q = clamp(rint(w /
// s + z), 0, 15) with the fp16 values; w is represented as (q - z) * s.
// Writes packed [E, K, N/2] -- each little-endian 32-bit word holds 8
// consecutive columns, column pair (2p, 2p+1) at bits 4p and 16 + 4p -- and
// fp16 bit patterns of scales / zeros [E, K/128, N].
void moe_quantize_int4_g128(const uint16_t* src, int E, int K, int N, int bf16, uint8_t* packed,
                            uint16_t* scales, uint16_t* zeros);

// ---- seeded input generator (the reference has none: inputs/data.cu:164-177
//      zero-fills everything).  Counter-based, thread-count independent:
//      value i of (seed, stream) depends only on (seed, stream, i). ----------
// Normal(0, std) values written as fp16 (bf16 != 0: bf16) bit patterns.
void moe_fill_normal_16(uint16_t* dst, size_t n, uint64_t seed, uint64_t stream, float std, int bf16);
void moe_fill_normal_f32(float* dst, size_t n, uint64_t seed, uint64_t stream, float std);
// Zipf(s) expert-popularity bias: bias[e] = -scale * s * ln(1 + rank(e)),
// rank a seeded permutation of 0..E-1 (seed 0 = identity).
void moe_zipf_bias(float* dst, int num_experts, float s, float scale, uint64_t seed);

#ifdef __cplusplus
}
#endif
