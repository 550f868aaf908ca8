// Shared device helpers: 16-bit conversions and small vector types.
#pragma once

#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <cstdint>

#include <atomic>

#include "moe_internal.h"

namespace moe {

// First output row of group g of a down GEMM: the local Y at the group's
// start row, or the redirected peer rows (expert parallelism).
__device__ __forceinline__ float* down_rows(const OutRedirect& r, float* local, int g, int start, int ld) {
    if (r.rank) return r.bases[__ldg(r.rank + g)] + (int64_t)__ldg(r.row0 + g) * ld;
    return local + (int64_t)start * ld;
}

template <typename T> struct F16Traits;
template <> struct F16Traits<__half> {
    static __device__ __forceinline__ float to_f32(__half v) { return __half2float(v); }
    static __device__ __forceinline__ __half from_f32(float v) { return __float2half_rn(v); }
    static __device__ __forceinline__ uint32_t pack2(float a, float b) {
        __half2 h = __floats2half2_rn(a, b);
        return *reinterpret_cast<uint32_t*>(&h);
    }
    static __device__ __forceinline__ float2 unpack2(uint32_t u) {
        __half2 h = *reinterpret_cast<__half2*>(&u);
        return __half22float2(h);
    }
};
template <> struct F16Traits<__nv_bfloat16> {
    static __device__ __forceinline__ float to_f32(__nv_bfloat16 v) { return __bfloat162float(v); }
    static __device__ __forceinline__ __nv_bfloat16 from_f32(float v) { return __float2bfloat16_rn(v); }
    static __device__ __forceinline__ uint32_t pack2(float a, float b) {
        __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
        return *reinterpret_cast<uint32_t*>(&h);
    }
    static __device__ __forceinline__ float2 unpack2(uint32_t u) {
        __nv_bfloat162 h = *reinterpret_cast<__nv_bfloat162*>(&u);
        return __bfloat1622float2(h);
    }
};

// Coalesced store of one warp's 32-row x 16-column f32 block: lane l holds
// row l's 16 values v[0..15] (an epilogue thread owns one TMEM lane = one
// row).  Storing from that layout directly would make every vector store
// touch 32 rows; instead the block goes through a 2 KB shared-memory stage
// (16-byte slots XOR-swizzled by (row >> 1) & 3, conflict-free both ways) and
// each store instruction then writes 8 rows x 64 contiguous bytes.  Rows
// >= nrows are not written.  Must be called by all 32 lanes.
__device__ __forceinline__ void warp_store_rows16(float4* stage, const float* v, float* g, int64_t ld, int nrows,
                                                  int lane) {
    const int sw = (lane >> 1) & 3;
#pragma unroll
    for (int j = 0; j < 4; ++j) stage[lane * 4 + (j ^ sw)] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
    __syncwarp();
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int r = 8 * i + (lane >> 2), c = lane & 3;
        const float4 val = stage[r * 4 + (c ^ ((r >> 1) & 3))];
        if (r < nrows) *reinterpret_cast<float4*>(g + (int64_t)r * ld + 4 * c) = val;
    }
    __syncwarp();
}

// Packed f32x2 FMA (sm_100): a0 = fma(p0, s, a0), a1 = fma(p1, s, a1), each
// rounded once exactly as fmaf -- one instruction for two accumulators.
__device__ __forceinline__ void ffma2(float& a0, float& a1, float p0, float p1, float s) {
    unsigned long long acc, pp, ss;
    float2 av = make_float2(a0, a1), pv = make_float2(p0, p1), sv = make_float2(s, s);
    acc = *reinterpret_cast<unsigned long long*>(&av);
    pp = *reinterpret_cast<unsigned long long*>(&pv);
    ss = *reinterpret_cast<unsigned long long*>(&sv);
    asm("fma.rn.f32x2 %0, %1, %2, %0;" : "+l"(acc) : "l"(pp), "l"(ss));
    const float2 r = *reinterpret_cast<float2*>(&acc);
    a0 = r.x;
    a1 = r.y;
}

// Raises a kernel's dynamic shared-memory limit once per device (again only
// when a launch needs more), so that launches recorded inside a CUDA-graph
// capture make no attribute call.  One SmemAttr per kernel instantiation.
struct SmemAttr {
    std::atomic<int> bytes[64];
};
template <typename Kernel>
inline cudaError_t ensure_smem(Kernel kern, size_t bytes, SmemAttr& a) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    std::atomic<int>& have = a.bytes[dev & 63];
    if (have.load(std::memory_order_acquire) >= (int)bytes) return cudaSuccess;
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
    if (e == cudaSuccess) {
        int cur = have.load();
        while (cur < (int)bytes && !have.compare_exchange_weak(cur, (int)bytes)) {
        }
    }
    return e;
}

}  // namespace moe
