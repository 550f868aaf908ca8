// Host input builder: C++ API of the reference's inputs/data.h
// (MattJBorowski1991/SparseMoE inputs/data.h:7-62), same signatures, plus a
// seeded generator.  Shapes come from the solve() dims (moe_get_solve_dims;
// defaults = include/config.h), so the vectors a driver sizes from config.h
// match what these functions expect.
#pragma once

#include <vector>
#include <cstdint>
#include <cuda_fp16.h>
#include "moe_args.h"

// Reference inputs/data.cu:164-177: zero-fill every host vector.
void initialize_host_data(
    std::vector<half>& h_input,
    std::vector<float>& h_final_output,
    std::vector<half>& h_expert_up_proj_weights,
    std::vector<half>& h_expert_gate_proj_weights,
    std::vector<half>& h_expert_down_proj_weights);

// New: x ~ N(0,1); up/gate ~ N(0, 1/sqrt(d)); down ~ N(0, 1/sqrt(f)), from `seed`.
// Also makes the allocators below draw router weights ~ N(0, 0.02) from the
// same seed instead of the reference's cudaMemset(0) (inputs/data.cu:237-243).
void initialize_host_data_seeded(
    std::vector<half>& h_input,
    std::vector<float>& h_final_output,
    std::vector<half>& h_expert_up_proj_weights,
    std::vector<half>& h_expert_gate_proj_weights,
    std::vector<half>& h_expert_down_proj_weights,
    uint64_t seed);

// Reference inputs/data.cu:179-197 (fp16 `capacity` path).
MoEArgs allocate_and_copy_to_device(
    const std::vector<half>& h_input,
    const std::vector<half>& h_expert_up_proj_weights,
    const std::vector<half>& h_expert_gate_proj_weights,
    const std::vector<half>& h_expert_down_proj_weights,
    bool use_capacity);

// Reference inputs/data.cu:526-544 (per-tensor int8 weights + scales).
MoEArgs allocate_and_copy_to_device_int8(
    const std::vector<half>& h_input,
    const std::vector<half>& h_expert_up_proj_weights,
    const std::vector<half>& h_expert_gate_proj_weights,
    const std::vector<half>& h_expert_down_proj_weights,
    bool use_capacity);

// Reference inputs/data.cu:546-564 (int4 values, plain nibble packing).
MoEArgs allocate_and_copy_to_device_int4(
    const std::vector<half>& h_input,
    const std::vector<half>& h_expert_up_proj_weights,
    const std::vector<half>& h_expert_gate_proj_weights,
    const std::vector<half>& h_expert_down_proj_weights,
    bool use_capacity);

// Reference inputs/data.cu:566-584 (int4 packed-transposed [E][n/2][K]).
MoEArgs allocate_and_copy_to_device_int4_ptx(
    const std::vector<half>& h_input,
    const std::vector<half>& h_expert_up_proj_weights,
    const std::vector<half>& h_expert_gate_proj_weights,
    const std::vector<half>& h_expert_down_proj_weights,
    bool use_capacity);

// Reference inputs/data.cu:586-604 (fp8 e4m3 cast weights).
MoEArgs allocate_and_copy_to_device_fp8(
    const std::vector<half>& h_input,
    const std::vector<half>& h_expert_up_proj_weights,
    const std::vector<half>& h_expert_gate_proj_weights,
    const std::vector<half>& h_expert_down_proj_weights,
    bool use_capacity);

// Reference inputs/data.cu:606-640: frees every non-null device pointer.
void cleanup_device_data(MoEArgs& args);
