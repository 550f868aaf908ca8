// Weight repacking for the reference's int4 format (MOE_DTYPE_INT4_PTX).
//
// The reference stores each expert's int4 weight matrix [K, N] "packed
// transposed" (inputs/data.cu:89-140): [N/2][K] bytes, byte (p, k) holding
// column 2p in its low nibble and column 2p+1 in its high nibble, the layout
// its mma.m16n8k64.s4 fragments read (kernels/capacity_int4_ptx.cu:171-307).
// The tcgen05 int8 GEMM here reads row-major [K, N] int8 (N contiguous, an
// MN-major operand), so each call first unpacks the three matrices into the
// library's scratch: values are sign-extended nibbles in [-8, 7] (the
// quantiser only produces [-7, 7]), so the int8 GEMM is exact.
//
// One CTA transposes a tile of 64 byte-rows (128 columns) x 32 K: coalesced
// 4-byte loads along K into shared memory, coalesced 4-byte stores along N.
// Experts that kept no rows in this call are skipped.  HBM-bound: per expert
// used, K*N/2 bytes read and K*N written per matrix.
#include "moe_internal.h"

namespace moe {
namespace {

constexpr int kTileP = 64;   // byte rows (column pairs) per tile = 128 output columns
constexpr int kTileK = 32;   // K rows per tile

__device__ __forceinline__ uint32_t sext_nibble(uint32_t v) { return (uint32_t)(((int32_t)(v << 28)) >> 28) & 0xFFu; }

__global__ void __launch_bounds__(256) unpack_int4_ptx_kernel(const uint8_t* __restrict__ packed, int K, int N,
                                                             const int* __restrict__ expert_rows,
                                                             int8_t* __restrict__ out) {
    __shared__ uint32_t tile[kTileP][kTileK / 4 + 1];   // [p][k/4] words of 4 K-bytes (+1: no bank conflicts)
    const int e = blockIdx.z;
    if (expert_rows && expert_rows[e] == 0) return;     // no kept rows: the GEMM never reads this expert
    const int p0 = blockIdx.x * kTileP, k0 = blockIdx.y * kTileK;
    const uint8_t* src = packed + (size_t)e * (N / 2) * K;
    int8_t* dst = out + (size_t)e * K * N;
    // load: 64 rows x 8 words
    for (int i = threadIdx.x; i < kTileP * (kTileK / 4); i += blockDim.x) {
        const int r = i / (kTileK / 4), w = i % (kTileK / 4);
        tile[r][w] = __ldg(reinterpret_cast<const uint32_t*>(src + (size_t)(p0 + r) * K + k0) + w);
    }
    __syncthreads();
    // store: 32 K rows x 32 words (each word = columns 4w..4w+3 = byte rows 2w, 2w+1)
    for (int i = threadIdx.x; i < kTileK * (2 * kTileP / 4); i += blockDim.x) {
        const int kr = i / (2 * kTileP / 4), w = i % (2 * kTileP / 4);
        const int sh = 8 * (kr & 3);
        const uint32_t b0 = (tile[2 * w][kr >> 2] >> sh) & 0xFFu;
        const uint32_t b1 = (tile[2 * w + 1][kr >> 2] >> sh) & 0xFFu;
        const uint32_t word = sext_nibble(b0) | (sext_nibble(b0 >> 4) << 8) | (sext_nibble(b1) << 16) |
                              (sext_nibble(b1 >> 4) << 24);
        reinterpret_cast<uint32_t*>(dst + (size_t)(k0 + kr) * N + 2 * p0)[w] = word;
    }
}

}  // namespace

cudaError_t launch_unpack_int4_ptx(const uint8_t* packed, int E, int K, int N, const int* expert_rows, int8_t* out,
                                   cudaStream_t st) {
    if (E <= 0 || K <= 0 || N <= 0) return cudaSuccess;
    if (K % kTileK != 0 || N % (2 * kTileP) != 0) return cudaErrorInvalidValue;
    const dim3 grid(N / (2 * kTileP), K / kTileK, E);
    unpack_int4_ptx_kernel<<<grid, 256, 0, st>>>(packed, K, N, expert_rows, out);
    return cudaGetLastError();
}

}  // namespace moe
