// Default layer shape: the values of the reference's compile-time config
// (include/config.h:6-38 of MattJBorowski1991/SparseMoE), under the same
// names so that the reference driver (drivers/main.cu) sizes its host vectors
// from this header unchanged.  This library reads them only as the initial
// value of the runtime dims used by solve() (moe_set_solve_dims overrides).
#ifndef CONFIG_H
#define CONFIG_H

constexpr int N = 256;             // tokens per batch
constexpr int d_model = 4096;
constexpr int h = 32;              // unused (kept for source compatibility)
constexpr int num_batches = 4;
constexpr int num_experts = 32;
constexpr int k = 4;               // top-k
constexpr int THREADS_PER_WARP = 32;
constexpr int up_proj_dim = 4;     // d_ff = up_proj_dim * d_model
constexpr float capacity_factor = 0.8f;
constexpr int NSTREAMS = 4;        // unused

#endif  // CONFIG_H
