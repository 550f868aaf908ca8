// The stage before the layer: pre-MoE RMSNorm of the tokens (a transformer
// block's norm ahead of its MoE FFN; the reference has none), written once
// to MoeDims.norm_out so that the router and the gather both read the
// normalised rows.  One warp per token, in a fixed order the CPU oracle
// restates:
//   ss   = sum x_j^2: lane l accumulates the 8-element chunks c = l, l+32, ..
//          (elements 8c..8c+7 in ascending j) with fmaf from 0.0f, then the
//          xor butterfly p[l] = p[l] + p[l ^ off], off = 16..1;
//   r    = sqrt(ss / d + eps)           (IEEE division, add and square root)
//   xn_j = round16((x_j * g_j) / r)     (IEEE multiply and division)
// so every lane ends with the same r and the result is bit-reproducible.
// HBM-bound: T*d*2 bytes read, T*d*2 written.
#include "moe_internal.h"
#include "common.cuh"

namespace moe {
namespace {

template <typename T16>
__global__ void __launch_bounds__(256) rmsnorm_kernel(const T16* __restrict__ x, const T16* __restrict__ g,
                                                     int64_t T, int d, float eps, T16* __restrict__ out) {
    const int64_t t = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (t >= T) return;
    const uint4* row = reinterpret_cast<const uint4*>(x + t * d);
    const int nvec = d / 8;
    float acc = 0.0f;
    for (int c = lane; c < nvec; c += 32) {
        const uint4 raw = __ldg(row + c);
        const uint32_t* u = reinterpret_cast<const uint32_t*>(&raw);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const float2 f = F16Traits<T16>::unpack2(u[q]);
            acc = fmaf(f.x, f.x, acc);
            acc = fmaf(f.y, f.y, acc);
        }
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) acc = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, off));
    const float r = __fsqrt_rn(__fadd_rn(__fdiv_rn(acc, (float)d), eps));
    const uint4* grow = reinterpret_cast<const uint4*>(g);
    uint4* orow = reinterpret_cast<uint4*>(out + t * d);
    for (int c = lane; c < nvec; c += 32) {
        const uint4 raw = __ldg(row + c), graw = __ldg(grow + c);
        const uint32_t* u = reinterpret_cast<const uint32_t*>(&raw);
        const uint32_t* gu = reinterpret_cast<const uint32_t*>(&graw);
        uint4 o;
        uint32_t* ou = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const float2 f = F16Traits<T16>::unpack2(u[q]), gf = F16Traits<T16>::unpack2(gu[q]);
            ou[q] = F16Traits<T16>::pack2(__fdiv_rn(__fmul_rn(f.x, gf.x), r), __fdiv_rn(__fmul_rn(f.y, gf.y), r));
        }
        orow[c] = o;
    }
}

}  // namespace

cudaError_t launch_rmsnorm(const void* x, const void* g, const Shape& s, float eps, void* out, cudaStream_t st) {
    if (s.T() == 0) return cudaSuccess;
    const unsigned blocks = (unsigned)((s.T() + 7) / 8);
    if (s.act_bf16)
        rmsnorm_kernel<__nv_bfloat16><<<blocks, 256, 0, st>>>((const __nv_bfloat16*)x, (const __nv_bfloat16*)g,
                                                               s.T(), s.d, eps, (__nv_bfloat16*)out);
    else
        rmsnorm_kernel<__half><<<blocks, 256, 0, st>>>((const __half*)x, (const __half*)g, s.T(), s.d, eps,
                                                        (__half*)out);
    return cudaGetLastError();
}

}  // namespace moe
