// Compile-time shape for building the reference's kernels (kernels/unfused.cu
// as a golden-vector generator, the fused kernels for the pin harness) as test
// infrastructure.  It shadows the reference's
// own include/config.h through the include path: same names (the reference
// sources use them), values chosen by -D at build time.
#include <math.h>

#ifndef CONFIG_H
#define CONFIG_H

#ifndef REF_N
#define REF_N 256
#endif
#ifndef REF_D
#define REF_D 512
#endif
#ifndef REF_B
#define REF_B 2
#endif
#ifndef REF_E
#define REF_E 16
#endif
#ifndef REF_K
#define REF_K 2
#endif
#ifndef REF_UP
#define REF_UP 2
#endif
#ifndef REF_CF
#define REF_CF 0.8f
#endif

constexpr int N = REF_N;
constexpr int d_model = REF_D;
constexpr int h = 32;
constexpr int num_batches = REF_B;
constexpr int num_experts = REF_E;
constexpr int k = REF_K;
constexpr int THREADS_PER_WARP = 32;

#define WMMA_M 16
#define WMMA_N 16
#define WMMA_K 16
#define WMMA_K_FP16 16
#define PAD 0

#define WARP_TILES_X 4
#define WARP_TILES_Y 2
#define WARPS_PER_BLOCK (WARP_TILES_X * WARP_TILES_Y)

constexpr int up_proj_dim = REF_UP;
constexpr float capacity_factor = REF_CF;
constexpr int NSTREAMS = 4;

#endif  // CONFIG_H
