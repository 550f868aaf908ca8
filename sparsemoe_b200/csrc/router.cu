// Stage 1+2: router logits, warp-shuffle top-k and gated softmax, one kernel.
//
// Reference semantics: kernels/capacity.cu:13-142 (router GEMM, fp32 result)
// and :171-238 (top_k_gating).  Differences by design:
//  * logits use a fixed fp32 order -- for each (token, expert) a sequential
//    fmaf chain over j = 0..d-1 starting at 0.0f, then + bias[e] -- so the CPU
//    oracle reproduces them bit for bit (the reference's WMMA order is
//    unspecified);
//  * top-k is a k-round warp argmax over (value desc, index asc), the same
//    selection as the reference's insertion sort with strict '>' (ties go to
//    the lower expert index; values <= -1e20 and NaN are never selected;
//    unfilled slots keep (-1e20, -1)).
//
// Layout: one CTA = 32*TPT tokens x all E experts.  Warp g owns experts
// [8g, 8g+8); lane l owns tokens l, l+32, ... of the tile.  x and Wr are
// staged through shared memory in K-chunks (x transposed so lanes read
// consecutive words).  The kernel is HBM-bound on reading x once.
#include "moe_internal.h"
#include "common.cuh"
#include <algorithm>

namespace moe {
namespace {

constexpr int kTPT = 2;               // tokens per thread
constexpr int kTM = 32 * kTPT;        // tokens per CTA
constexpr int kKC = 64;               // K chunk staged in shared memory

template <typename TX, typename TW>
__global__ void __launch_bounds__(1024) router_topk_kernel(
    const TX* __restrict__ x, const TW* __restrict__ wr, const float* __restrict__ bias,
    int64_t T, int d, int E, int k, float* __restrict__ logits, int* __restrict__ idx,
    float* __restrict__ wts) {
    extern __shared__ float smem[];
    float* xs = smem;                   // [kKC][kTM]
    float* ws = xs + kKC * kTM;         // [kKC][E]
    float* lg = ws;                     // reused after the K loop: [kTM][E]
    const int G = E / 8;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nthr = blockDim.x;
    const int64_t t0 = (int64_t)blockIdx.x * kTM;

    float acc[kTPT][8];
#pragma unroll
    for (int i = 0; i < kTPT; ++i)
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[i][e] = 0.0f;

    for (int j0 = 0; j0 < d; j0 += kKC) {
        // x tile: kTM tokens x kKC columns as 16-byte vectors, stored transposed.
        for (int v = threadIdx.x; v < kTM * (kKC / 8); v += nthr) {
            const int tt = v / (kKC / 8), jv = v % (kKC / 8);
            const int64_t t = t0 + tt;
            float f8[8];
            if (t < T) {
                const uint4 raw = *reinterpret_cast<const uint4*>(x + t * d + j0 + jv * 8);
                const uint32_t* u = reinterpret_cast<const uint32_t*>(&raw);
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    float2 p = F16Traits<TX>::unpack2(u[q]);
                    f8[2 * q] = p.x;
                    f8[2 * q + 1] = p.y;
                }
            } else {
#pragma unroll
                for (int q = 0; q < 8; ++q) f8[q] = 0.0f;
            }
#pragma unroll
            for (int q = 0; q < 8; ++q) xs[(jv * 8 + q) * kTM + tt] = f8[q];
        }
        // Wr rows j0..j0+kKC, all experts.
        for (int v = threadIdx.x; v < kKC * E; v += nthr) {
            const int jj = v / E, e = v % E;
            if constexpr (sizeof(TW) == 4) {
                ws[v] = wr[(int64_t)(j0 + jj) * E + e];
            } else {
                ws[v] = F16Traits<TW>::to_f32(wr[(int64_t)(j0 + jj) * E + e]);
            }
        }
        __syncthreads();
#pragma unroll 4
        for (int jj = 0; jj < kKC; ++jj) {
            const float4 w0 = *reinterpret_cast<const float4*>(&ws[jj * E + warp * 8]);
            const float4 w1 = *reinterpret_cast<const float4*>(&ws[jj * E + warp * 8 + 4]);
            const float wv[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
            for (int i = 0; i < kTPT; ++i) {
                const float xv = xs[jj * kTM + i * 32 + lane];
#pragma unroll
                for (int e = 0; e < 8; ++e) acc[i][e] = fmaf(xv, wv[e], acc[i][e]);
            }
        }
        __syncthreads();
    }

    // Logits (+bias) to shared memory and (optionally) global.
#pragma unroll
    for (int i = 0; i < kTPT; ++i) {
        const int tt = i * 32 + lane;
        const int64_t t = t0 + tt;
#pragma unroll
        for (int e = 0; e < 8; ++e) {
            const int ee = warp * 8 + e;
            const float v = bias ? __fadd_rn(acc[i][e], bias[ee]) : acc[i][e];
            lg[tt * E + ee] = v;
            if (logits != nullptr && t < T) logits[t * E + ee] = v;
        }
    }
    __syncthreads();

    // Top-k: warp g handles tokens g, g+G, ...  Lane l owns experts l, l+32, ...
    const int per_lane = (E + 31) / 32;  // <= 8
    for (int tt = warp; tt < kTM; tt += G) {
        const int64_t t = t0 + tt;
        if (t >= T) break;
        uint32_t taken = 0;
        float my_v = -1e20f;
        int my_i = -1;
        for (int l = 0; l < k; ++l) {
            float bv = 0.0f;
            int bi = -1;
            for (int q = 0; q < per_lane; ++q) {
                const int e = lane + 32 * q;
                if (e < E && !(taken & (1u << q))) {
                    const float v = lg[tt * E + e];
                    if (v > -1e20f && (bi < 0 || v > bv)) { bv = v; bi = e; }
                }
            }
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) {
                const float ov = __shfl_xor_sync(0xffffffffu, bv, off);
                const int oi = __shfl_xor_sync(0xffffffffu, bi, off);
                if (oi >= 0 && (bi < 0 || ov > bv || (ov == bv && oi < bi))) { bv = ov; bi = oi; }
            }
            if (bi < 0) break;  // fewer than k selectable experts: rest keep the sentinel
            if ((bi & 31) == lane) taken |= 1u << (bi >> 5);
            if (lane == l) { my_v = bv; my_i = bi; }
        }
        // Softmax over the k kept values: w_l = exp(v_l - v_0) / (sum + 1e-10).
        const float mx = __shfl_sync(0xffffffffu, my_v, 0);
        const float ex = (lane < k) ? expf(my_v - mx) : 0.0f;
        float sum = 0.0f;
        for (int l = 0; l < k; ++l) sum += __shfl_sync(0xffffffffu, ex, l);
        if (lane < k) {
            idx[t * k + lane] = my_i;
            wts[t * k + lane] = ex / (sum + 1e-10f);
        }
    }
}

template <typename TX, typename TW>
cudaError_t launch_typed(const void* x, const void* wr, const float* bias, const Shape& s,
                         float* logits, int* idx, float* w, cudaStream_t st) {
    const int threads = 32 * (s.E / 8);
    const size_t smem = sizeof(float) * ((size_t)kKC * kTM + (size_t)std::max(kKC, kTM) * s.E);
    auto kern = router_topk_kernel<TX, TW>;
    cudaError_t err = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (err != cudaSuccess) return err;
    const int64_t blocks = (s.T() + kTM - 1) / kTM;
    kern<<<(unsigned)blocks, threads, smem, st>>>((const TX*)x, (const TW*)wr, bias, s.T(), s.d, s.E,
                                                  s.k, logits, idx, w);
    return cudaGetLastError();
}

}  // namespace

cudaError_t launch_router_topk(const void* x, const void* wr, const float* bias, const Shape& s,
                               float* logits, int* idx, float* w, cudaStream_t st) {
    if (s.T() == 0) return cudaSuccess;
    const bool bf = s.dtype == MOE_DTYPE_BF16;
    if (s.router_dtype == MOE_ROUTER_F32) {
        return bf ? launch_typed<__nv_bfloat16, float>(x, wr, bias, s, logits, idx, w, st)
                  : launch_typed<__half, float>(x, wr, bias, s, logits, idx, w, st);
    }
    return bf ? launch_typed<__nv_bfloat16, __nv_bfloat16>(x, wr, bias, s, logits, idx, w, st)
              : launch_typed<__half, __half>(x, wr, bias, s, logits, idx, w, st);
}

}  // namespace moe
