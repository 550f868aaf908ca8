// Stage 1+2: router logits, warp-shuffle top-k and gated softmax, one kernel.
//
// Reference semantics: kernels/capacity.cu:13-142 (router GEMM, fp32 result)
// and :171-238 (top_k_gating).  Differences by design:
//  * logits use a fixed fp32 order (the reference's WMMA order is
//    unspecified) that the CPU oracle reproduces bit for bit.  For E < 64 (or
//    E not a multiple of 32):
//      lane l (0..31) owns the 8-element chunks c = l, l+32, l+64, ... of the
//      d-dimension (elements 8c..8c+7) and accumulates them in ascending j
//      with fmaf, starting at 0.0f;  the 32 partial sums are then combined by
//      an xor butterfly  p[l] = p[l] + p[l ^ off]  for off = 16, 8, 4, 2, 1;
//      logit = p[0] (+ bias[e], one rounded add);
//    for E >= 64 and a multiple of 32 (router_tiled_kernel, then
//    fold_topk_kernel): d is cut into blocks of kRouterBlockJ = 512 j's; per (token, expert)
//    each block is one sequential fmaf chain over its j's from 0.0f (one CTA's work, written
//    as a partial logit), and fold_topk_kernel sums the nb blocks by the fixed tree
//      tree(a, 1) = b_a,  tree(a, n) = tree(a, h) + tree(a + h, n - h),  h = largest power of
//      two below n,
//    then + bias[e];
//  * top-k is a k-round warp argmax over (value desc, index asc), the same
//    selection as the reference's insertion sort with strict '>' (ties go to
//    the lower expert index; values <= -1e20 and NaN are never selected;
//    unfilled slots keep (-1e20, -1)).
//
// Layout: 8 warps per CTA; a work item is TT consecutive tokens x one group
// of 8 experts.  Lanes read x as 16-byte vectors (one 512-byte
// coalesced segment per warp load) and the matching 8 router rows x 8
// experts; all lanes end the butterfly with the same sums.  Logits go to
// shared memory, then each warp runs the top-k of one token at a time.  The
// kernel reads x once from HBM (the router weights stay in L1/L2).
#include "moe_internal.h"
#include "common.cuh"
#include <algorithm>

namespace moe {
namespace {

constexpr int kWarps = 8;

template <typename TW>
__device__ __forceinline__ void load_wr8(const TW* __restrict__ p, float (&w)[8]) {
    if constexpr (sizeof(TW) == 4) {
        const float4 a = *reinterpret_cast<const float4*>(p);
        const float4 b = *reinterpret_cast<const float4*>(p + 4);
        w[0] = a.x; w[1] = a.y; w[2] = a.z; w[3] = a.w; w[4] = b.x; w[5] = b.y; w[6] = b.z; w[7] = b.w;
    } else {
        const uint4 raw = __ldg(reinterpret_cast<const uint4*>(p));
        const uint32_t* u = reinterpret_cast<const uint32_t*>(&raw);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const float2 f = F16Traits<TW>::unpack2(u[q]);
            w[2 * q] = f.x;
            w[2 * q + 1] = f.y;
        }
    }
}


// Order-preserving key of a float: a larger key is a larger value, -0 maps
// to +0's key (the two compare equal, so the lower index must win the tie).
__device__ __forceinline__ uint32_t order_key(float v) {
    const uint32_t u = __float_as_uint(v + 0.0f);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float key_value(uint32_t key) {
    return __uint_as_float((key & 0x80000000u) ? (key & 0x7FFFFFFFu) : ~key);
}

// k-round warp argmax over (value desc, index asc) -- the reference's
// insertion top-k with strict '>' -- then the softmax over the k kept values,
// w_l = exp(v_l - v_0) / (sum + 1e-10).  Lane l holds the logits of experts
// l, l+32, ... in v[0..8).  A round is two warp reductions (redux.sync): the
// largest key, then the lowest expert index among the lanes holding it; only
// the winning lane rescans its candidates.
__device__ __forceinline__ void topk_softmax_regs(const float (&v)[8], int E, int k, int64_t t,
                                                  int* __restrict__ idx, float* __restrict__ wts, int lane) {
    uint32_t avail = 0;
#pragma unroll
    for (int q = 0; q < 8; ++q)
        if (lane + 32 * q < E && v[q] > -1e20f) avail |= 1u << q;   // NaN and the sentinel never selectable
    uint32_t bk = 0;
    int be = -1;
    auto lane_best = [&]() {
        bk = 0;
        be = -1;
#pragma unroll
        for (int q = 0; q < 8; ++q) {
            if (avail & (1u << q)) {
                const uint32_t kq = order_key(v[q]);
                if (kq > bk) { bk = kq; be = lane + 32 * q; }   // strict: the lower index keeps a tie
            }
        }
    };
    lane_best();
    float my_v = -1e20f;
    int my_i = -1;
    for (int l = 0; l < k; ++l) {
        const uint32_t m = __reduce_max_sync(0xffffffffu, bk);
        if (m == 0) break;  // fewer than k selectable experts: the rest keep the sentinel
        const int bi = (int)__reduce_min_sync(0xffffffffu, bk == m ? (uint32_t)be : 0xFFFFFFFFu);
        if (lane == l) { my_v = key_value(m); my_i = bi; }
        if ((bi & 31) == lane) {
            avail &= ~(1u << (bi >> 5));
            lane_best();
        }
    }
    const float mx = __shfl_sync(0xffffffffu, my_v, 0);
    const float ex = (lane < k) ? expf(my_v - mx) : 0.0f;
    float sum = 0.0f;
    for (int l = 0; l < k; ++l) sum += __shfl_sync(0xffffffffu, ex, l);
    if (lane < k) {
        idx[t * k + lane] = my_i;
        wts[t * k + lane] = ex / (sum + 1e-10f);
    }
}

// The same over a row of E logits in shared memory.
__device__ __forceinline__ void topk_softmax_warp(const float* row, int E, int k, int64_t t, int* __restrict__ idx,
                                                  float* __restrict__ wts, int lane) {
    float v[8];
#pragma unroll
    for (int q = 0; q < 8; ++q) v[q] = lane + 32 * q < E ? row[lane + 32 * q] : -1e20f;
    topk_softmax_regs(v, E, k, t, idx, wts, lane);
}

// Work item = (TT tokens, one group of 8 experts); a CTA holds CT tokens
// (CT a multiple of TT) and its warps take the CT/TT x E/8 items in turn, so
// small token counts still spread over many warps (TT = 1) while large ones
// reuse each router row for 4 or 8 tokens.
template <typename TX, typename TW, int TT>
__global__ void __launch_bounds__(kWarps * 32) router_topk_kernel(
    const TX* __restrict__ x, const TW* __restrict__ wr, const float* __restrict__ bias,
    int64_t T, int d, int E, int k, int CT, float* __restrict__ logits, int* __restrict__ idx,
    float* __restrict__ wts) {
    extern __shared__ float lg_all[];  // [CT][E]
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t cta_t0 = (int64_t)blockIdx.x * CT;
    const int nchunks = d / 256;
    const int G = E / 8;
    const int items = (CT / TT) * G;

    for (int item = warp; item < items; item += kWarps) {
        const int quad = item / G, g = item - quad * G;
        const int64_t t0 = cta_t0 + (int64_t)quad * TT;
        float acc[TT][8];
#pragma unroll
        for (int tt = 0; tt < TT; ++tt)
#pragma unroll
            for (int e = 0; e < 8; ++e) acc[tt][e] = 0.0f;
        for (int i = 0; i < nchunks; ++i) {
            const int j0 = 8 * (lane + 32 * i);
            float xv[TT][8];
#pragma unroll
            for (int tt = 0; tt < TT; ++tt) {
                const int64_t t = t0 + tt;
                if (t < T) {
                    const uint4 raw = __ldg(reinterpret_cast<const uint4*>(x + t * d + j0));
                    const uint32_t* u = reinterpret_cast<const uint32_t*>(&raw);
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        const float2 f = F16Traits<TX>::unpack2(u[q]);
                        xv[tt][2 * q] = f.x;
                        xv[tt][2 * q + 1] = f.y;
                    }
                } else {
#pragma unroll
                    for (int q = 0; q < 8; ++q) xv[tt][q] = 0.0f;
                }
            }
#pragma unroll
            for (int jj = 0; jj < 8; ++jj) {
                float wv[8];
                load_wr8(wr + (int64_t)(j0 + jj) * E + 8 * g, wv);
#pragma unroll
                for (int tt = 0; tt < TT; ++tt)
#pragma unroll
                    for (int e = 0; e < 8; ++e) acc[tt][e] = fmaf(xv[tt][jj], wv[e], acc[tt][e]);
            }
        }
#pragma unroll
        for (int tt = 0; tt < TT; ++tt)
#pragma unroll
            for (int e = 0; e < 8; ++e)
#pragma unroll
                for (int off = 16; off > 0; off >>= 1)
                    acc[tt][e] = acc[tt][e] + __shfl_xor_sync(0xffffffffu, acc[tt][e], off);
        if (lane == 0) {
#pragma unroll
            for (int tt = 0; tt < TT; ++tt)
#pragma unroll
                for (int e = 0; e < 8; ++e) {
                    const int ee = 8 * g + e;
                    lg_all[(quad * TT + tt) * E + ee] = bias ? __fadd_rn(acc[tt][e], bias[ee]) : acc[tt][e];
                }
        }
    }
    __syncthreads();

    for (int tt = warp; tt < CT; tt += kWarps) {
        const int64_t t = cta_t0 + tt;
        if (t >= T) break;
        const float* row = lg_all + tt * E;
        if (logits != nullptr)
            for (int e = lane; e < E; e += 32) logits[t * E + e] = row[e];
        topk_softmax_warp(row, E, k, t, idx, wts, lane);
    }
}

// Many experts (E >= kRouterTiledMinExperts, E % 32 == 0): a register-tiled
// CUDA-core GEMM over one 512-j block of d per CTA (grid.y = block), written
// as partial logits part[block][t][e] for fold_topk_kernel.  CTA = 16*MT
// tokens x an expert slice of EC experts (grid.z; EC = E, or 32 for small
// batches), 2EC threads; thread (r, c) owns tokens MT*r.. and
// experts 8c..8c+7 (4 vector shared loads per MT*8 FMAs); x and Wr K-slices
// of 32 are staged in shared memory as f32 (x transposed), double-buffered:
// the next slice is loaded into registers during the FMAs.  Splitting d into
// blocks multiplies the CTAs by ceil(d/512), so even 64-expert routers keep
// every SM busy.
constexpr int kTiledKC = 32;

template <typename TX, typename TW, int MT>
__global__ void __launch_bounds__(MT == 8 ? 256 : 512) router_tiled_kernel(
    const TX* __restrict__ x, const TW* __restrict__ wr, int64_t T, int d, int E, float* __restrict__ part) {
    constexpr int kTiledTM = 16 * MT;
    extern __shared__ float sm[];
    const int nthr = blockDim.x;
    const int EC = nthr / 2;                     // experts of this CTA's slice (a multiple of 32)
    const int e0 = blockIdx.z * EC;
    float* xs = sm;                              // [2][kTiledKC][kTiledTM]
    float* ws = xs + 2 * kTiledKC * kTiledTM;    // [2][kTiledKC][EC]
    const int cgroups = EC / 8;
    const int xvecs = kTiledTM * (kTiledKC / 8);   // x vectors per slice (8 tokens of 16 B each per j-row)
    // a warp covers 8 token rows x 4 expert groups, so its shared-memory
    // loads touch 8 x-rows (256 B) and 4 router groups (128 B) per K step
    const int warp_id = threadIdx.x >> 5, lane_id = threadIdx.x & 31;
    const int wpr = cgroups / 4;   // warps per 8-row block
    const int r = (warp_id / wpr) * 8 + (lane_id & 7), c = (warp_id % wpr) * 4 + (lane_id >> 3);
    const int64_t t0 = (int64_t)blockIdx.x * kTiledTM;
    const int jbeg = blockIdx.y * kRouterBlockJ, jend = min(d, jbeg + kRouterBlockJ);
    float acc[MT][8];
#pragma unroll
    for (int i = 0; i < MT; ++i)
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[i][e] = 0.0f;

    // The next K slice is loaded into registers while the current one is
    // multiplied out of shared memory (double-buffered, one barrier per slice).
    constexpr int kXVec = kTiledTM * (kTiledKC / 8) / 64;   // x vectors per thread (>= 64 threads)
    uint4 xr[kXVec];
    float wreg[2][8];
    auto load_slice = [&](int j0) {
#pragma unroll
        for (int v = 0; v < kXVec; ++v) {
            const int vi = threadIdx.x + v * nthr;
            xr[v] = make_uint4(0u, 0u, 0u, 0u);
            if (vi < xvecs) {
                const int tt = vi / (kTiledKC / 8), jv = vi - tt * (kTiledKC / 8);
                const int64_t t = t0 + tt;
                if (t < T) xr[v] = __ldg(reinterpret_cast<const uint4*>(x + t * d + j0 + jv * 8));
            }
        }
#pragma unroll
        for (int v = 0; v < 2; ++v) {   // kTiledKC * EC/8 vectors = 2 per thread
            const int vi = threadIdx.x + v * nthr;
            const int jj = vi / cgroups, cc = vi - jj * cgroups;
            load_wr8(wr + (int64_t)(j0 + jj) * E + e0 + 8 * cc, wreg[v]);
        }
    };
    auto store_slice = [&](int buf) {
        float* xb = xs + buf * kTiledKC * kTiledTM;
        float* wb = ws + buf * kTiledKC * EC;
#pragma unroll
        for (int v = 0; v < kXVec; ++v) {
            const int vi = threadIdx.x + v * nthr;
            if (vi < xvecs) {
                const int tt = vi / (kTiledKC / 8), jv = vi - tt * (kTiledKC / 8);
                const uint32_t* u = reinterpret_cast<const uint32_t*>(&xr[v]);
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    const float2 p = F16Traits<TX>::unpack2(u[q]);
                    xb[(jv * 8 + 2 * q) * kTiledTM + tt] = p.x;
                    xb[(jv * 8 + 2 * q + 1) * kTiledTM + tt] = p.y;
                }
            }
        }
#pragma unroll
        for (int v = 0; v < 2; ++v) {
            const int vi = threadIdx.x + v * nthr;
            const int jj = vi / cgroups, cc = vi - jj * cgroups;
            float4* dst = reinterpret_cast<float4*>(wb + jj * EC + 8 * cc);
            dst[0] = make_float4(wreg[v][0], wreg[v][1], wreg[v][2], wreg[v][3]);
            dst[1] = make_float4(wreg[v][4], wreg[v][5], wreg[v][6], wreg[v][7]);
        }
    };
    const int nslices = (jend - jbeg) / kTiledKC;
    load_slice(jbeg);
    store_slice(0);
    __syncthreads();
    for (int sl = 0; sl < nslices; ++sl) {
        const int buf = sl & 1;
        if (sl + 1 < nslices) load_slice(jbeg + (sl + 1) * kTiledKC);
        const float* xb = xs + buf * kTiledKC * kTiledTM;
        const float* wb = ws + buf * kTiledKC * EC;
#pragma unroll 4
        for (int jj = 0; jj < kTiledKC; ++jj) {
            const float4 wa = *reinterpret_cast<const float4*>(wb + jj * EC + 8 * c);
            const float4 wc = *reinterpret_cast<const float4*>(wb + jj * EC + 8 * c + 4);
            const float wv[8] = {wa.x, wa.y, wa.z, wa.w, wc.x, wc.y, wc.z, wc.w};
            float xv[MT];
#pragma unroll
            for (int i = 0; i < MT; i += 4) {
                const float4 xa = *reinterpret_cast<const float4*>(xb + jj * kTiledTM + MT * r + i);
                xv[i] = xa.x; xv[i + 1] = xa.y; xv[i + 2] = xa.z; xv[i + 3] = xa.w;
            }
#pragma unroll
            for (int i = 0; i < MT; ++i)
#pragma unroll
                for (int e = 0; e < 8; e += 2) ffma2(acc[i][e], acc[i][e + 1], wv[e], wv[e + 1], xv[i]);
        }
        if (sl + 1 < nslices) store_slice(buf ^ 1);
        __syncthreads();
    }
    float* pb = part + (int64_t)blockIdx.y * T * E;
#pragma unroll
    for (int i = 0; i < MT; ++i) {
        const int64_t t = t0 + MT * r + i;
        if (t < T) {
            float4* dst = reinterpret_cast<float4*>(pb + t * E + e0 + 8 * c);
            dst[0] = make_float4(acc[i][0], acc[i][1], acc[i][2], acc[i][3]);
            dst[1] = make_float4(acc[i][4], acc[i][5], acc[i][6], acc[i][7]);
        }
    }
}

// One warp per token: the nb partial logits of each expert summed by the
// block tree (a binary-counter stack: leaf b closes one pair per trailing 1
// bit of b, the left operand first; the remaining stack is folded from the
// top, each entry added on the left), + bias, then top-k + softmax on the
// lane's logits in registers.
constexpr int kFoldMaxLevels = 8;   // nb <= 255 blocks (d <= 130560)
constexpr int kFoldUnrolled = 16;   // d <= 8192: every partial of an expert loaded before the fold
__global__ void __launch_bounds__(128) fold_topk_kernel(const float* __restrict__ part, int nb, int64_t T, int E,
                                                       int k, const float* __restrict__ bias,
                                                       float* __restrict__ logits, int* __restrict__ idx,
                                                       float* __restrict__ wts) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t t = (int64_t)blockIdx.x * 4 + warp;
    if (t >= T) return;
    float vals[8];
#pragma unroll
    for (int q = 0; q < 8; ++q) {
        const int e = lane + 32 * q;
        vals[q] = -1e20f;
        if (e >= E) continue;
        float st[kFoldMaxLevels];
        int top = 0;
        if (nb <= kFoldUnrolled) {
            // all of this expert's partials in flight at once, then the fold
            float pv[kFoldUnrolled];
#pragma unroll
            for (int b = 0; b < kFoldUnrolled; ++b)
                if (b < nb) pv[b] = __ldg(part + ((int64_t)b * T + t) * E + e);
#pragma unroll
            for (int b = 0; b < kFoldUnrolled; ++b) {
                if (b >= nb) break;
                float v = pv[b];
                for (int i = b; i & 1; i >>= 1) v = st[--top] + v;
                st[top++] = v;
            }
        } else {
            for (int b = 0; b < nb; ++b) {
                float v = part[((int64_t)b * T + t) * E + e];
                for (int i = b; i & 1; i >>= 1) v = st[--top] + v;
                st[top++] = v;
            }
        }
        float v = st[--top];
        while (top > 0) v = st[--top] + v;
        if (bias) v = __fadd_rn(v, bias[e]);
        vals[q] = v;
        if (logits != nullptr) logits[t * E + e] = v;
    }
    topk_softmax_regs(vals, E, k, t, idx, wts, lane);
}

template <typename TX, typename TW>
cudaError_t launch_blocked(const void* x, const void* wr, const float* bias, const Shape& s, float* logits,
                           float* part, int* idx, float* w, cudaStream_t st) {
    const int nb = (s.d + kRouterBlockJ - 1) / kRouterBlockJ;
    // Tokens x experts x blocks: every expert in one CTA when the tokens alone
    // fill the GPU (x read once per block), else 32-expert slices so that
    // decode-sized batches still spread over every SM.
    constexpr int MT = 4, kTiledTM = 16 * MT;
    const int EC = router_sliced(s) ? 32 : s.E;
    const size_t smem = sizeof(float) * 2 * (size_t)kTiledKC * (kTiledTM + (size_t)EC);
    auto kern = router_tiled_kernel<TX, TW, MT>;
    static SmemAttr attr;
    cudaError_t err = ensure_smem(kern, 2 * (size_t)kTiledKC * (kTiledTM + 256) * sizeof(float), attr);
    if (err != cudaSuccess) return err;
    const dim3 grid((unsigned)((s.T() + kTiledTM - 1) / kTiledTM), nb, s.E / EC);
    kern<<<grid, 2 * EC, smem, st>>>((const TX*)x, (const TW*)wr, s.T(), s.d, s.E, part);
    fold_topk_kernel<<<(unsigned)((s.T() + 3) / 4), 128, 0, st>>>(part, nb, s.T(), s.E, s.k, bias, logits, idx, w);
    return cudaGetLastError();
}

template <typename TX, typename TW, int TT>
cudaError_t launch_items(const void* x, const void* wr, const float* bias, const Shape& s, int CT, float* logits,
                         int* idx, float* w, cudaStream_t st) {
    const size_t smem = sizeof(float) * (size_t)CT * s.E;
    const int64_t blocks = (s.T() + CT - 1) / CT;
    auto kern = router_topk_kernel<TX, TW, TT>;
    static SmemAttr attr;
    cudaError_t err = ensure_smem(kern, smem, attr);
    if (err != cudaSuccess) return err;
    kern<<<(unsigned)blocks, kWarps * 32, smem, st>>>((const TX*)x, (const TW*)wr, bias, s.T(), s.d, s.E, s.k, CT,
                                                      logits, idx, w);
    return cudaGetLastError();
}

template <typename TX, typename TW>
cudaError_t launch_typed(const void* x, const void* wr, const float* bias, const Shape& s,
                         float* logits, int* idx, float* w, cudaStream_t st) {
    // Tokens per item TT: the largest of 8, 4, 1 that still leaves two CTAs of
    // work items per SM (each router row read from L2 serves TT tokens);
    // tokens per CTA CT: one item per warp.
    const int G = s.E / 8;
    const int64_t want = 2 * 148 * kWarps;
    const int TT = s.T() * G / 8 >= want ? 8 : (s.T() * G / 4 >= want ? 4 : 1);
    const int CT = TT * std::max(1, kWarps / G);
    if (TT == 8) return launch_items<TX, TW, 8>(x, wr, bias, s, CT, logits, idx, w, st);
    if (TT == 4) return launch_items<TX, TW, 4>(x, wr, bias, s, CT, logits, idx, w, st);
    return launch_items<TX, TW, 1>(x, wr, bias, s, CT, logits, idx, w, st);
}

template <typename TX, typename TW>
cudaError_t launch_any(const void* x, const void* wr, const float* bias, const Shape& s, float* logits,
                       float* logits_scratch, int* idx, float* w, cudaStream_t st) {
    if (!router_blocked(s)) return launch_typed<TX, TW>(x, wr, bias, s, logits, idx, w, st);
    return launch_blocked<TX, TW>(x, wr, bias, s, logits, logits_scratch, idx, w, st);
}

}  // namespace

bool router_blocked(const Shape& s) { return s.E >= kRouterTiledMinExperts && s.E % 32 == 0; }

bool router_sliced(const Shape& s) { return router_blocked(s) && s.T() < kRouterSliceMaxT; }

cudaError_t launch_router_topk(const void* x, const void* wr, const float* bias, const Shape& s,
                               float* logits_scratch, float* logits, int* idx, float* w, cudaStream_t st) {
    if (s.T() == 0) return cudaSuccess;
    const bool bf = s.act_bf16;
    if (s.router_dtype == MOE_ROUTER_F32) {
        return bf ? launch_any<__nv_bfloat16, float>(x, wr, bias, s, logits, logits_scratch, idx, w, st)
                  : launch_any<__half, float>(x, wr, bias, s, logits, logits_scratch, idx, w, st);
    }
    return bf ? launch_any<__nv_bfloat16, __nv_bfloat16>(x, wr, bias, s, logits, logits_scratch, idx, w, st)
              : launch_any<__half, __half>(x, wr, bias, s, logits, logits_scratch, idx, w, st);
}

}  // namespace moe
