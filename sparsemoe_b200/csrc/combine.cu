// Stage 5: gate-weighted combine back to [B, N, d].
//
// Reference semantics: kernels/capacity.cu:380-423 -- out[b,t,:] is the sum of
// w * Y_e[slot,:] over the token's kept routes, no renormalisation after
// drops, tokens with no kept route get 0.  The reference scatters with f32
// atomicAdd (order = arrival order); here each CTA gathers one token's k rows
// and sums them in l = 0..k-1 order with separately rounded multiply and add
// (out = ((0 + w0*y0) + w1*y1) + ...), which is deterministic and is the order
// the CPU oracle uses.  With a residual (MoeDims.residual) the sum starts from
// the residual row instead of 0: out = ((r + w0*y0) + w1*y1) + ....  No atomics, no zero-fill pass: every output element is
// written exactly once.  HBM-bound: reads R_kept*d*4 bytes, writes T*d*4.
#include "moe_internal.h"
#include "common.cuh"

namespace moe {
namespace {

constexpr int kThreads = 256;

template <typename T16>
__global__ void __launch_bounds__(kThreads) combine_kernel(
    const float* __restrict__ y_rows, const int* __restrict__ idx, const float* __restrict__ w,
    const int* __restrict__ route_slot, const int* __restrict__ row_base, const int* __restrict__ expert_start,
    int N, int d, int E, int k, const T16* __restrict__ residual, float* __restrict__ out, T16* __restrict__ out16) {
    __shared__ int64_t s_row[32];
    __shared__ float s_w[32];
    const int64_t t = blockIdx.x;  // flattened token b*N + n
    const int b = (int)(t / N);
    if (threadIdx.x < k) {
        const int64_t r = t * k + threadIdx.x;
        const int slot = route_slot[r];
        int64_t row = -1;
        if (slot >= 0) {
            const int e = idx[r];
            row = (int64_t)expert_start[e] + row_base[b * E + e] + slot;
        }
        s_row[threadIdx.x] = row;
        s_w[threadIdx.x] = w[r];
    }
    __syncthreads();
    const int nvec = d / 4;
    for (int v = threadIdx.x; v < nvec; v += kThreads) {
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
        if (residual != nullptr) {
            const uint2 rr = __ldg(reinterpret_cast<const uint2*>(residual + t * d) + v);
            const float2 r01 = F16Traits<T16>::unpack2(rr.x), r23 = F16Traits<T16>::unpack2(rr.y);
            acc = make_float4(r01.x, r01.y, r23.x, r23.y);
        }
        for (int l = 0; l < k; ++l) {
            const int64_t row = s_row[l];
            if (row < 0) continue;
            const float wl = s_w[l];
            const float4 y = __ldg(reinterpret_cast<const float4*>(y_rows + row * d) + v);
            acc.x = __fadd_rn(acc.x, __fmul_rn(wl, y.x));
            acc.y = __fadd_rn(acc.y, __fmul_rn(wl, y.y));
            acc.z = __fadd_rn(acc.z, __fmul_rn(wl, y.z));
            acc.w = __fadd_rn(acc.w, __fmul_rn(wl, y.w));
        }
        reinterpret_cast<float4*>(out + t * d)[v] = acc;
        if (out16 != nullptr) {
            uint2 pk;
            pk.x = F16Traits<T16>::pack2(acc.x, acc.y);
            pk.y = F16Traits<T16>::pack2(acc.z, acc.w);
            reinterpret_cast<uint2*>(out16 + t * d)[v] = pk;
        }
    }
}

}  // namespace

cudaError_t launch_combine(const float* y_rows, const int* idx, const float* w, const Shape& s,
                           const Workspace& ws, float* out, void* out16, cudaStream_t st, const void* residual) {
    if (s.T() == 0) return cudaSuccess;
    if (s.act_bf16)
        combine_kernel<__nv_bfloat16><<<(unsigned)s.T(), kThreads, 0, st>>>(
            y_rows, idx, w, ws.route_slot, ws.row_base, ws.expert_start, s.N, s.d, s.E, s.k,
            (const __nv_bfloat16*)residual, out, (__nv_bfloat16*)out16);
    else
        combine_kernel<__half><<<(unsigned)s.T(), kThreads, 0, st>>>(
            y_rows, idx, w, ws.route_slot, ws.row_base, ws.expert_start, s.N, s.d, s.E, s.k,
            (const __half*)residual, out, (__half*)out16);
    return cudaGetLastError();
}

}  // namespace moe
