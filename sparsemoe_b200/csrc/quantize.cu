// Device weight quantisers: the same formats and the same arithmetic as the
// host quantisers in data.cu (moe_quantize_int8_channel, _fp8_blocks,
// _int4_g128, _nvfp4), for weights already on the GPU -- a checkpoint loaded
// in bf16, or the large synthetic weights of the DeepSeek-V3-shape workloads.
// Each output is bit-identical to its host twin (same expressions, IEEE
// division, round-to-nearest conversions), which the GPU tests check.
//
// All weights are [E, K, N] 16-bit (bf16 != 0: bf16, else fp16), row-major.
#include "moe_internal.h"
#include "common.cuh"

#include <cuda_fp16.h>
#include <cuda_fp8.h>

#include <algorithm>

namespace moe {
namespace {

template <bool kBf16>
__device__ __forceinline__ float ld16(const uint16_t* p, size_t i) {
    const uint16_t u = p[i];
    if (kBf16) return __uint_as_float((uint32_t)u << 16);
    return __half2float(__ushort_as_half(u));
}

// Loads 8 consecutive 16-bit values (16-byte aligned) as f32.
template <bool kBf16>
__device__ __forceinline__ void ld16x8(const uint16_t* p, float (&v)[8]) {
    const uint4 raw = *reinterpret_cast<const uint4*>(p);
    const uint32_t* u = reinterpret_cast<const uint32_t*>(&raw);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        if (kBf16) {
            v[2 * q] = __uint_as_float(u[q] << 16);
            v[2 * q + 1] = __uint_as_float(u[q] & 0xFFFF0000u);
        } else {
            v[2 * q] = __half2float(__ushort_as_half((uint16_t)(u[q] & 0xFFFFu)));
            v[2 * q + 1] = __half2float(__ushort_as_half((uint16_t)(u[q] >> 16)));
        }
    }
}

// ---- int8, one scale per output channel ----------------------------------------
template <bool kBf16>
__global__ void q_int8_channel_kernel(const uint16_t* __restrict__ src, int E, int K, int N, int8_t* __restrict__ q,
                                      float* __restrict__ scales) {
    const int64_t id = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (id >= (int64_t)E * N) return;
    const int e = (int)(id / N), n = (int)(id - (int64_t)e * N);
    const uint16_t* col = src + (size_t)e * K * N + n;
    float m = 0.0f;
    for (int r = 0; r < K; ++r) m = fmaxf(m, fabsf(ld16<kBf16>(col, (size_t)r * N)));
    const float s = m > 0.0f ? m / 127.0f : 1.0f;
    scales[id] = s;
    int8_t* qc = q + (size_t)e * K * N + n;
    for (int r = 0; r < K; ++r) {
        const float v = nearbyintf(ld16<kBf16>(col, (size_t)r * N) / s);
        qc[(size_t)r * N] = (int8_t)(int)fminf(fmaxf(v, -127.0f), 127.0f);
    }
}

// ---- e4m3, one scale per 128 x 128 block ---------------------------------------
// One CTA (128 threads, one column each) per block.
template <bool kBf16>
__global__ void __launch_bounds__(128) q_fp8_blocks_kernel(const uint16_t* __restrict__ src, int K, int N,
                                                           uint8_t* __restrict__ q, float* __restrict__ scales) {
    __shared__ float red[4];
    const int bn = blockIdx.x, bk = blockIdx.y, e = blockIdx.z;
    const int kb = K / 128, nb = N / 128;
    const size_t base = ((size_t)e * K + (size_t)bk * 128) * N + (size_t)bn * 128 + threadIdx.x;
    float m = 0.0f;
    for (int i = 0; i < 128; ++i) m = fmaxf(m, fabsf(ld16<kBf16>(src, base + (size_t)i * N)));
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
    __syncthreads();
    m = fmaxf(fmaxf(red[0], red[1]), fmaxf(red[2], red[3]));
    const float sc = m > 0.0f ? m / 448.0f : 1.0f;
    if (threadIdx.x == 0) scales[((size_t)e * kb + bk) * nb + bn] = sc;
    for (int i = 0; i < 128; ++i)
        q[base + (size_t)i * N] =
            (uint8_t)__nv_cvt_float_to_fp8(ld16<kBf16>(src, base + (size_t)i * N) / sc, __NV_SATFINITE, __NV_E4M3);
}

// The 4-bit formats pack 8 consecutive columns per little-endian 32-bit word,
// column pair (2p, 2p+1) at bits 4p and 16 + 4p.
__device__ __forceinline__ uint32_t pack8(const int (&q)[8]) {
    uint32_t w = 0;
#pragma unroll
    for (int p = 0; p < 4; ++p) w |= ((uint32_t)q[2 * p] << (4 * p)) | ((uint32_t)q[2 * p + 1] << (16 + 4 * p));
    return w;
}

// ---- INT4 asymmetric, group 128 along K, fp16 scale and zero -------------------
// Thread per (expert, group, 8-column word).
template <bool kBf16>
__global__ void q_int4_g128_kernel(const uint16_t* __restrict__ src, int E, int K, int N,
                                   uint32_t* __restrict__ packed, __half* __restrict__ scales,
                                   __half* __restrict__ zeros) {
    const int W = N / 8, G = K / 128;
    const int64_t id = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (id >= (int64_t)E * G * W) return;
    const int w = (int)(id % W);
    const int g = (int)((id / W) % G);
    const int e = (int)(id / ((int64_t)W * G));
    const uint16_t* blk = src + ((size_t)e * K + (size_t)g * 128) * N + 8 * w;
    float mn[8], mx[8];
#pragma unroll
    for (int c = 0; c < 8; ++c) { mn[c] = INFINITY; mx[c] = -INFINITY; }
    for (int i = 0; i < 128; ++i) {
        float v[8];
        ld16x8<kBf16>(blk + (size_t)i * N, v);
#pragma unroll
        for (int c = 0; c < 8; ++c) { mn[c] = fminf(mn[c], v[c]); mx[c] = fmaxf(mx[c], v[c]); }
    }
    float sf[8], zf[8];
#pragma unroll
    for (int c = 0; c < 8; ++c) {
        float sc = (mx[c] - mn[c]) / 15.0f;
        if (!(sc > 0.0f)) sc = 1.0f;
        const __half sh = __float2half_rn(sc);
        const __half zh = __float2half_rn(-mn[c] / __half2float(sh));
        sf[c] = __half2float(sh);
        zf[c] = __half2float(zh);
        const size_t o = ((size_t)e * G + g) * N + 8 * w + c;
        scales[o] = sh;
        zeros[o] = zh;
    }
    for (int i = 0; i < 128; ++i) {
        float v[8];
        ld16x8<kBf16>(blk + (size_t)i * N, v);
        int qv[8];
#pragma unroll
        for (int c = 0; c < 8; ++c) qv[c] = max(0, min(15, (int)rintf(v[c] / sf[c] + zf[c])));
        packed[((size_t)e * K + (size_t)g * 128 + i) * W + w] = pack8(qv);
    }
}

// ---- NVFP4: e2m1, e4m3 scale per 16 K-rows, f32 global per matrix -------------
template <bool kBf16>
__global__ void q_amax_kernel(const uint16_t* __restrict__ src, int64_t per_expert, unsigned int* __restrict__ amax) {
    const int e = blockIdx.y;
    const uint16_t* m = src + (size_t)e * per_expert;
    float a = 0.0f;
    for (int64_t i = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) * 8; i < per_expert;
         i += (int64_t)gridDim.x * blockDim.x * 8) {
        float v[8];
        ld16x8<kBf16>(m + i, v);
#pragma unroll
        for (int c = 0; c < 8; ++c) a = fmaxf(a, fabsf(v[c]));
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, off));
    if ((threadIdx.x & 31) == 0) atomicMax(amax + e, __float_as_uint(a));   // a >= 0: bit order = value order
}

__global__ void q_global_kernel(float* __restrict__ g, int E) {
    const int e = blockIdx.x * blockDim.x + threadIdx.x;
    if (e >= E) return;
    const float amax = g[e];   // written as the bits of a non-negative float by q_amax_kernel
    g[e] = amax > 0.0f ? amax / (448.0f * 6.0f) : 1.0f;
}

__device__ __forceinline__ int e2m1_code(float v) {
    const float kMag[8] = {0.0f, 0.5f, 1.0f, 1.5f, 2.0f, 3.0f, 4.0f, 6.0f};
    const int sign = v < 0.0f ? 8 : 0;
    const float a = fabsf(v);
    int best = 7;
    if (a < 6.0f) {
        best = 0;
        for (int c = 1; c < 8; ++c) {
            const float dc = fabsf(a - kMag[c]), db = fabsf(a - kMag[best]);
            if (dc < db || (dc == db && (c & 1) == 0)) best = c;
        }
    }
    return sign | best;
}

// Thread per (expert, 16-row group, 8-column word).
template <bool kBf16>
__global__ void q_nvfp4_kernel(const uint16_t* __restrict__ src, int E, int K, int N, const float* __restrict__ glob,
                               uint32_t* __restrict__ packed, uint8_t* __restrict__ scales) {
    const int W = N / 8, G = K / 16;
    const int64_t id = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (id >= (int64_t)E * G * W) return;
    const int w = (int)(id % W);
    const int gr = (int)((id / W) % G);
    const int e = (int)(id / ((int64_t)W * G));
    const float g = glob[e];
    const uint16_t* blk = src + ((size_t)e * K + (size_t)gr * 16) * N + 8 * w;
    float m[8];
#pragma unroll
    for (int c = 0; c < 8; ++c) m[c] = 0.0f;
    for (int i = 0; i < 16; ++i) {
        float v[8];
        ld16x8<kBf16>(blk + (size_t)i * N, v);
#pragma unroll
        for (int c = 0; c < 8; ++c) m[c] = fmaxf(m[c], fabsf(v[c]));
    }
    float div[8];
    uint32_t sc_lo = 0, sc_hi = 0;
#pragma unroll
    for (int c = 0; c < 8; ++c) {
        uint8_t sc = 0x38;   // 1.0
        if (m[c] > 0.0f) {
            sc = (uint8_t)__nv_cvt_float_to_fp8(m[c] / (6.0f * g), __NV_SATFINITE, __NV_E4M3);
            if ((sc & 0x7F) == 0) sc = 0x01;   // smallest positive subnormal, never zero
        }
        if (c < 4) sc_lo |= (uint32_t)sc << (8 * c); else sc_hi |= (uint32_t)sc << (8 * (c - 4));
        div[c] = __half2float(__half(__nv_cvt_fp8_to_halfraw(sc, __NV_E4M3))) * g;
    }
    *reinterpret_cast<uint2*>(scales + ((size_t)e * G + gr) * N + 8 * w) = make_uint2(sc_lo, sc_hi);
    for (int i = 0; i < 16; ++i) {
        float v[8];
        ld16x8<kBf16>(blk + (size_t)i * N, v);
        int qv[8];
#pragma unroll
        for (int c = 0; c < 8; ++c) qv[c] = e2m1_code(v[c] / div[c]);
        packed[((size_t)e * K + (size_t)gr * 16 + i) * W + w] = pack8(qv);
    }
}

int q_fail(cudaError_t e) { return e == cudaSuccess ? MOE_OK : MOE_ERR_CUDA; }

bool q_shape_ok(const void* src, int E, int K, int N, int kmul) {
    return src && E > 0 && K > 0 && N > 0 && K % kmul == 0 && N % 8 == 0 &&
           reinterpret_cast<uintptr_t>(src) % 16 == 0;
}

}  // namespace
}  // namespace moe

using namespace moe;

extern "C" int moe_quantize_int8_channel_device(const void* src, int E, int K, int N, int bf16, int8_t* q,
                                                float* scales, cudaStream_t st) {
    if (!q_shape_ok(src, E, K, N, 1) || !q || !scales) return MOE_ERR_INVALID_ARG;
    const int64_t n = (int64_t)E * N;
    const unsigned blocks = (unsigned)((n + 255) / 256);
    if (bf16) q_int8_channel_kernel<true><<<blocks, 256, 0, st>>>((const uint16_t*)src, E, K, N, q, scales);
    else q_int8_channel_kernel<false><<<blocks, 256, 0, st>>>((const uint16_t*)src, E, K, N, q, scales);
    return q_fail(cudaGetLastError());
}

extern "C" int moe_quantize_fp8_blocks_device(const void* src, int E, int K, int N, int bf16, uint8_t* q,
                                              float* scales, cudaStream_t st) {
    if (!q_shape_ok(src, E, K, N, 128) || N % 128 != 0 || !q || !scales) return MOE_ERR_INVALID_ARG;
    const dim3 grid(N / 128, K / 128, E);
    if (bf16) q_fp8_blocks_kernel<true><<<grid, 128, 0, st>>>((const uint16_t*)src, K, N, q, scales);
    else q_fp8_blocks_kernel<false><<<grid, 128, 0, st>>>((const uint16_t*)src, K, N, q, scales);
    return q_fail(cudaGetLastError());
}

extern "C" int moe_quantize_int4_g128_device(const void* src, int E, int K, int N, int bf16, uint8_t* packed,
                                             uint16_t* scales, uint16_t* zeros, cudaStream_t st) {
    if (!q_shape_ok(src, E, K, N, 128) || !packed || !scales || !zeros) return MOE_ERR_INVALID_ARG;
    const int64_t n = (int64_t)E * (K / 128) * (N / 8);
    const unsigned blocks = (unsigned)((n + 255) / 256);
    if (bf16)
        q_int4_g128_kernel<true><<<blocks, 256, 0, st>>>((const uint16_t*)src, E, K, N, (uint32_t*)packed,
                                                         (__half*)scales, (__half*)zeros);
    else
        q_int4_g128_kernel<false><<<blocks, 256, 0, st>>>((const uint16_t*)src, E, K, N, (uint32_t*)packed,
                                                          (__half*)scales, (__half*)zeros);
    return q_fail(cudaGetLastError());
}

extern "C" int moe_quantize_nvfp4_device(const void* src, int E, int K, int N, int bf16, uint8_t* packed,
                                         uint8_t* scales, float* globals, cudaStream_t st) {
    if (!q_shape_ok(src, E, K, N, 16) || !packed || !scales || !globals) return MOE_ERR_INVALID_ARG;
    cudaError_t err = cudaMemsetAsync(globals, 0, sizeof(float) * E, st);
    if (err != cudaSuccess) return MOE_ERR_CUDA;
    const int64_t per = (int64_t)K * N;
    const dim3 agrid((unsigned)std::min<int64_t>(1024, (per / 8 + 255) / 256), E);
    if (bf16) q_amax_kernel<true><<<agrid, 256, 0, st>>>((const uint16_t*)src, per, (unsigned int*)globals);
    else q_amax_kernel<false><<<agrid, 256, 0, st>>>((const uint16_t*)src, per, (unsigned int*)globals);
    q_global_kernel<<<(E + 255) / 256, 256, 0, st>>>(globals, E);
    const int64_t n = (int64_t)E * (K / 16) * (N / 8);
    const unsigned blocks = (unsigned)((n + 255) / 256);
    if (bf16)
        q_nvfp4_kernel<true><<<blocks, 256, 0, st>>>((const uint16_t*)src, E, K, N, globals, (uint32_t*)packed,
                                                     scales);
    else
        q_nvfp4_kernel<false><<<blocks, 256, 0, st>>>((const uint16_t*)src, E, K, N, globals, (uint32_t*)packed,
                                                      scales);
    return q_fail(cudaGetLastError());
}
