// MoEArgs: the by-value argument block of the capacity-routed MoE layer.
//
// Byte-compatible with the reference's struct (include/moe_args.h:8-55 of
// MattJBorowski1991/SparseMoE): same field order, same types, so a driver
// built against the reference header (drivers/main.cu) links against this
// library unchanged.  Every pointer is device memory owned by the caller.
//
// Layouts used by this implementation (B = num_batches, N = tokens per batch,
// E = experts, CAP = per-batch per-expert capacity, d = d_model, f = d_ff):
//   input                         [B, N, d]                 f16 (or bf16 bits)
//   router_weights                [d, E]                    f16 (or bf16 bits)
//   expert_{up,gate}_proj_weights [E, d, f] row-major       f16 (or bf16 bits)
//   expert_down_proj_weights      [E, f, d] row-major       f16 (or bf16 bits)
//   expert_logits                 [B, N, E]                 f32
//   selected_expert_indices       [B, N, k]                 i32 (-1 = none)
//   selected_expert_weights       [B, N, k]                 f32
//   expert_counts                 [B, E]                    i32, min(routes, CAP)
//   expert_token_ids              [B, E, CAP]               i32
//   expert_token_weights          [B, E, CAP]               f32
//   per_expert_wmma_inputs        [B*E*CAP, d]  kept rows, dense expert-major
//   hidden_mlp_layer_1_out_fp16   [B*E*CAP, f]  SwiGLU output (same rows)
//   hidden_mlp_layer_2_out        [B*E*CAP, d]  f32 down-projection output
//   final_output                  [B, N, d]                 f32
// The three per-expert scratch buffers have the reference's byte size
// (B*E*CAP rows) but hold only the kept rows, expert by expert: expert e's
// rows start after all kept rows of experts < e, batch 0's slots first, so
// one expert is one contiguous GEMM operand (the int8 path uses the *_int8
// fields the same way).  hidden_mlp_layer_1_out / hidden_mlp_gate_out
// (f32 up/gate) are not used: SwiGLU is fused into the up/gate GEMM epilogue.
#pragma once

#include <stdint.h>
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>

struct MoEArgs {
    const half* input;
    const half* router_weights;
    const half* expert_up_proj_weights;
    const half* expert_gate_proj_weights;
    const half* expert_down_proj_weights;
    const int8_t* expert_up_proj_weights_int8;
    const int8_t* expert_gate_proj_weights_int8;
    const int8_t* expert_down_proj_weights_int8;
    const uint8_t* expert_up_proj_weights_int4;     // [E, f/2, d] packed-transposed (int4_ptx layout)
    const uint8_t* expert_gate_proj_weights_int4;
    const uint8_t* expert_down_proj_weights_int4;   // [E, d/2, f]
    const __nv_fp8_e4m3* expert_up_proj_weights_fp8;
    const __nv_fp8_e4m3* expert_gate_proj_weights_fp8;
    const __nv_fp8_e4m3* expert_down_proj_weights_fp8;
    float scale_up_w;
    float scale_gate_w;
    float scale_down_w;
    float scale_input_act;
    float scale_mid_act;
    float*  expert_logits;
    int*    selected_expert_indices;
    float*  selected_expert_weights;
    int*    expert_counts;
    int*    expert_token_ids;
    float*  expert_token_weights;
    half* per_expert_wmma_inputs;
    int8_t* per_expert_wmma_inputs_int8;
    uint8_t* per_expert_wmma_inputs_int4;
    __nv_fp8_e4m3* per_expert_wmma_inputs_fp8;
    float* hidden_mlp_layer_1_out;
    float* hidden_mlp_gate_out;
    half* hidden_mlp_layer_1_out_fp16;
    int8_t* hidden_mlp_layer_1_out_int8;
    uint8_t* hidden_mlp_layer_1_out_int4;
    __nv_fp8_e4m3* hidden_mlp_layer_1_out_fp8;
    float* hidden_mlp_layer_2_out;
    float* final_output;
    int num_batches;
    bool use_capacity;
    int cap;
};
