// Stage 3: deterministic capacity dispatch and the 16-byte row gather.
//
// Reference semantics: kernels/capacity.cu:245-309 (build_per_expert_buffers,
// clamp_expert_counts) and :312-377 (assign_per_expert_wmma_inputs), with the
// slot of route r = t*k + l defined as the number of earlier routes (route-id
// order) of the same batch to the same expert -- the serial execution of the
// reference loop.  Kept iff slot < CAP; no renormalisation of the kept
// weights; counts[b,e] = min(routes, CAP).
//
// Four launches:
//   count   grid (chunks, B): per-(chunk, expert) route histogram
//   scan    1 CTA:            exclusive prefix over chunks; counts; per-expert
//                             row bases of the compact expert-major layout
//   assign  grid (chunks, B): warp-aggregated ranking (__match_any_sync +
//                             popc), in-order prefix across warps, writes the
//                             slot tables (token ids / weights / route slots)
//   scatter one warp per token: reads the token's row once (quantising it
//                             for the 8-bit formats) and writes it to the
//                             compact-block row of each kept route with
//                             16-byte vector stores (HBM-bound: T*d*2 B read,
//                             R_kept*d*s_a B written).
// Dense expert-major row layout: expert e's kept rows start at
// expert_start[e] = sum of the kept rows of experts < e; within it batch b's
// slots start at row_base[b,e].  Row of (b, e, slot) = expert_start[e] +
// row_base[b,e] + slot.
#include "moe_internal.h"
#include <algorithm>
#include <cstdint>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <cuda_fp8.h>

namespace moe {
namespace {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;

// Row of slot (b, e, s) and the peer (0: local) that receives it.
__device__ __forceinline__ int64_t gather_row(const GatherDst& g, const int* expert_start, const int* row_base,
                                              int e, int be, int s, int& q) {
    if (g.rank) {
        q = g.rank[e];
        return (int64_t)g.row0[e] + row_base[be] + s;
    }
    q = 0;
    return (int64_t)expert_start[e] + row_base[be] + s;
}
constexpr int kRounds = kChunkRoutes / kThreads;

__global__ void __launch_bounds__(kThreads) dispatch_count_kernel(const int* __restrict__ idx, int N,
                                                                  int k, int E, int chunks,
                                                                  int* __restrict__ chunk_count) {
    __shared__ int hist[256];
    const int c = blockIdx.x, b = blockIdx.y;
    for (int e = threadIdx.x; e < E; e += kThreads) hist[e] = 0;
    __syncthreads();
    const int64_t routes = (int64_t)N * k;
    const int* idx_b = idx + (int64_t)b * routes;
    for (int i = 0; i < kRounds; ++i) {
        const int64_t r = (int64_t)c * kChunkRoutes + i * kThreads + threadIdx.x;
        if (r < routes) {
            const int e = idx_b[r];
            if (e >= 0 && e < E) atomicAdd(&hist[e], 1);
        }
    }
    __syncthreads();
    int* out = chunk_count + ((int64_t)b * chunks + c) * E;
    for (int e = threadIdx.x; e < E; e += kThreads) out[e] = hist[e];
}

// slot_base (optional, [B, E]): slots already taken by earlier shards of the
// same batch (expert parallelism over a split batch); raw (optional, [B, E]):
// the shard's route totals before any drop.
__global__ void __launch_bounds__(256) dispatch_scan_kernel(const int* __restrict__ chunk_count,
                                                            int B, int E, int chunks, int cap,
                                                            const int* __restrict__ slot_base,
                                                            int* __restrict__ raw,
                                                            int* __restrict__ chunk_base,
                                                            int* __restrict__ counts,
                                                            int* __restrict__ row_base,
                                                            int* __restrict__ expert_rows,
                                                            int* __restrict__ expert_start) {
    __shared__ int s_rows[256];
    const int e = threadIdx.x;
    int rows = 0;
    if (e < E) {
    for (int b = 0; b < B; ++b) {
        int run = 0;
        for (int c = 0; c < chunks; ++c) {
            const int64_t o = ((int64_t)b * chunks + c) * E + e;
            chunk_base[o] = run;
            run += chunk_count[o];
        }
        if (raw) raw[b * E + e] = run;
        const int room = slot_base ? max(0, cap - slot_base[b * E + e]) : cap;
        const int kept = run < room ? run : room;
        counts[b * E + e] = kept;
        row_base[b * E + e] = rows;
        rows += kept;
    }
    expert_rows[e] = rows;
    s_rows[e] = rows;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        int acc = 0;
        for (int q = 0; q < E; ++q) { expert_start[q] = acc; acc += s_rows[q]; }
    }
}

__global__ void __launch_bounds__(kThreads) dispatch_assign_kernel(
    const int* __restrict__ idx, const float* __restrict__ w, int N, int k, int E, int cap, int chunks,
    const int* __restrict__ chunk_base, const int* __restrict__ slot_base, int* __restrict__ token_ids,
    float* __restrict__ token_weights, int* __restrict__ route_slot) {
    __shared__ int base[256];
    __shared__ int room[256];   // slots this shard may still fill per expert
    __shared__ int wcnt[kWarps][256];
    const int c = blockIdx.x, b = blockIdx.y;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int e = threadIdx.x; e < E; e += kThreads) {
        base[e] = chunk_base[((int64_t)b * chunks + c) * E + e];
        room[e] = slot_base ? max(0, cap - slot_base[b * E + e]) : cap;
#pragma unroll
        for (int q = 0; q < kWarps; ++q) wcnt[q][e] = 0;
    }
    __syncthreads();
    const int64_t routes = (int64_t)N * k;
    const int64_t rb = (int64_t)b * routes;
    const unsigned lt_mask = (1u << lane) - 1u;
    for (int i = 0; i < kRounds; ++i) {
        const int64_t r = (int64_t)c * kChunkRoutes + i * kThreads + threadIdx.x;
        int e = -1;
        if (r < routes) {
            e = idx[rb + r];
            if (e < 0 || e >= E) e = -1;
        }
        const unsigned peers = __match_any_sync(0xffffffffu, e);
        const int rank = __popc(peers & lt_mask);
        if (e >= 0 && rank == 0) wcnt[warp][e] = __popc(peers);
        __syncthreads();
        int slot = -1;
        if (e >= 0) {
            int s = base[e] + rank;
            for (int q = 0; q < warp; ++q) s += wcnt[q][e];
            slot = s;
        }
        __syncthreads();
        for (int ee = threadIdx.x; ee < E; ee += kThreads) {
            int add = 0;
#pragma unroll
            for (int q = 0; q < kWarps; ++q) { add += wcnt[q][ee]; wcnt[q][ee] = 0; }
            base[ee] += add;
        }
        // Slot tables.
        const bool kept = e >= 0 && slot < room[e];
        if (r < routes) {
            route_slot[rb + r] = kept ? slot : -1;
            if (kept) {
                const int64_t o = ((int64_t)b * E + e) * cap + slot;
                token_ids[o] = (int)(r / k);
                token_weights[o] = w[rb + r];
            }
        }
        __syncthreads();
    }
}

// The row copy ("gather" of the reference, assign_per_expert_wmma_inputs)
// runs token-major: one warp per token (b, t) reads the token's row once,
// quantises it once (every format's row quantisation depends on the token
// alone) and writes it to the destination row of each of its kept routes, so
// x is read once instead of once per route (k times).  Lane l < k holds
// route l's destination (row, peer); -1 = dropped.
struct RouteDst {
    int64_t row;
    int q;
};
__device__ __forceinline__ RouteDst route_dst(const int* __restrict__ idx, const int* __restrict__ route_slot,
                                              const int* row_base, const int* expert_start, const GatherDst& gd,
                                              int E, int k, int64_t r0, int b, int lane) {
    RouteDst d{-1, 0};
    if (lane < k) {
        const int slot = route_slot[r0 + lane];
        if (slot >= 0) {
            const int e = idx[r0 + lane];
            d.row = gather_row(gd, expert_start, row_base, e, b * E + e, slot, d.q);
        }
    }
    return d;
}

// Warp w handles part w % split of token w / split's row (split > 1 only when
// there are too few tokens to fill the GPU, e.g. decode batches).
__device__ __forceinline__ bool token_of_warp(int N, int B, int split, int64_t& bt, int& b, int& part) {
    const int64_t w = (int64_t)blockIdx.x * kWarps + (threadIdx.x >> 5);
    if (w >= (int64_t)B * N * split) return false;
    bt = w / split;
    part = (int)(w - bt * split);
    b = (int)(bt / N);
    return true;
}
// [begin, end) of part `part` of n units, cut in multiples of `unit`.
__device__ __forceinline__ void part_range(int n, int unit, int split, int part, int& begin, int& end) {
    const int per = (n + split * unit - 1) / (split * unit) * unit;
    begin = min(n, part * per);
    end = min(n, begin + per);
}

// 16-bit rows: a plain copy, 4 x 16 B per lane in flight.
__global__ void __launch_bounds__(kThreads) dispatch_scatter_kernel(
    const uint4* __restrict__ x, const int* __restrict__ idx, const int* __restrict__ route_slot,
    const int* __restrict__ row_base, const int* __restrict__ expert_start, int N, int E, int B, int k,
    int vec_per_row, int split, const GatherDst gd) {
    const int lane = threadIdx.x & 31;
    int64_t bt;
    int b, part, vb, ve;
    if (!token_of_warp(N, B, split, bt, b, part)) return;
    const RouteDst my = route_dst(idx, route_slot, row_base, expert_start, gd, E, k, bt * k, b, lane);
    if (!__any_sync(0xffffffffu, my.row >= 0)) return;
    part_range(vec_per_row, 128, split, part, vb, ve);
    const uint4* src = x + bt * vec_per_row;
    for (int v0 = vb; v0 < ve; v0 += 128) {
        uint4 a[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int v = v0 + 32 * i + lane;
            if (v < ve) a[i] = __ldg(src + v);
        }
        for (int l = 0; l < k; ++l) {
            const int64_t row = __shfl_sync(0xffffffffu, my.row, l);
            if (row < 0) continue;
            uint4* dst = static_cast<uint4*>(gd.rows[__shfl_sync(0xffffffffu, my.q, l)]) + row * vec_per_row;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const int v = v0 + 32 * i + lane;
                if (v < ve) dst[v] = a[i];
            }
        }
    }
}

// The per-tensor formats: the token's f16 row quantised with the MoEArgs
// scale s_in, 8 values per 16-byte load, one byte each:
//   kQ = 0  int8  rn(clamp(x / s_in, -128, 127))  (reference capacity_int8_ptx.cu:391-432)
//   kQ = 1  int4  rn(clamp(x / s_in, -7, 7))      (capacity_int4_ptx.cu:396-441; kept one value per
//                                                  byte, not nibble-packed: the GEMM reads int8)
//   kQ = 2  e4m3  e4m3(clamp(x / s_in, -448, 448)) (capacity_fp8_ptx.cu:330-352, nearest even)
template <int kQ>
__device__ __forceinline__ uint32_t quant_pair(float a, float b, float s_in) {
    if (kQ == 2) {
        const float qa = fminf(fmaxf(a / s_in, -448.f), 448.f), qb = fminf(fmaxf(b / s_in, -448.f), 448.f);
        return (uint32_t)__nv_cvt_float2_to_fp8x2(make_float2(qa, qb), __NV_SATFINITE, __NV_E4M3);
    }
    constexpr float lo = kQ == 0 ? -128.f : -7.f, hi = kQ == 0 ? 127.f : 7.f;
    const int q0 = __float2int_rn(fminf(fmaxf(a / s_in, lo), hi));
    const int q1 = __float2int_rn(fminf(fmaxf(b / s_in, lo), hi));
    return (uint32_t)(q0 & 0xFF) | ((uint32_t)(q1 & 0xFF) << 8);
}

template <int kQ>
__global__ void __launch_bounds__(kThreads) dispatch_scatter_q8_kernel(
    const uint4* __restrict__ x, const int* __restrict__ idx, const int* __restrict__ route_slot,
    const int* __restrict__ row_base, const int* __restrict__ expert_start, int N, int E, int B, int k,
    int vec_per_row, int split, float s_in, const GatherDst gd) {
    const int lane = threadIdx.x & 31;
    int64_t bt;
    int b, part, vb, ve;
    if (!token_of_warp(N, B, split, bt, b, part)) return;
    const RouteDst my = route_dst(idx, route_slot, row_base, expert_start, gd, E, k, bt * k, b, lane);
    if (!__any_sync(0xffffffffu, my.row >= 0)) return;
    part_range(vec_per_row, 64, split, part, vb, ve);
    const uint4* src = x + bt * vec_per_row;
    for (int v0 = vb; v0 < ve; v0 += 64) {
        uint2 w[2];
#pragma unroll
        for (int i = 0; i < 2; ++i) {
            const int v = v0 + 32 * i + lane;
            w[i] = make_uint2(0u, 0u);
            if (v < ve) {
                const uint4 raw = __ldg(src + v);
                const __half2* h2 = reinterpret_cast<const __half2*>(&raw);
                uint32_t p[2] = {0u, 0u};
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const float2 f = __half22float2(h2[j]);
                    p[j >> 1] |= quant_pair<kQ>(f.x, f.y, s_in) << (16 * (j & 1));
                }
                w[i] = make_uint2(p[0], p[1]);
            }
        }
        for (int l = 0; l < k; ++l) {
            const int64_t row = __shfl_sync(0xffffffffu, my.row, l);
            if (row < 0) continue;
            uint2* dst = static_cast<uint2*>(gd.rows[__shfl_sync(0xffffffffu, my.q, l)]) + row * vec_per_row;
#pragma unroll
            for (int i = 0; i < 2; ++i) {
                const int v = v0 + 32 * i + lane;
                if (v < ve) dst[v] = w[i];
            }
        }
    }
}

// FP8 block path: the token's bf16 row quantised per 1x128 block,
// s = amax / 448 (1 for an all-zero block), q = e4m3(x / s) (nearest even,
// saturating); lane l handles elements 4l..4l+3 of each block.
__global__ void __launch_bounds__(kThreads) dispatch_scatter_fp8_kernel(
    const __nv_bfloat16* __restrict__ x, const int* __restrict__ idx, const int* __restrict__ route_slot,
    const int* __restrict__ row_base, const int* __restrict__ expert_start, int N, int E, int B, int k, int d,
    int split, const GatherDst gd) {
    const int lane = threadIdx.x & 31;
    int64_t bt;
    int b, part, kb0, kb1;
    if (!token_of_warp(N, B, split, bt, b, part)) return;
    const RouteDst my = route_dst(idx, route_slot, row_base, expert_start, gd, E, k, bt * k, b, lane);
    if (!__any_sync(0xffffffffu, my.row >= 0)) return;
    const __nv_bfloat16* src = x + bt * d;
    const int nblk = d / 128;   // a multiple of 2 (d % 256 == 0)
    part_range(nblk, 8, split, part, kb0, kb1);
    // 8 blocks' loads in flight per round (lane: 4 elements of each block)
    for (int b0 = kb0; b0 < kb1; b0 += 8) {
        const int nb = min(8, kb1 - b0);
        uint2 raw[8];
#pragma unroll
        for (int i = 0; i < 8; ++i)
            if (i < nb) raw[i] = __ldg(reinterpret_cast<const uint2*>(src + (b0 + i) * 128) + lane);
        uint32_t code[8];
        float scale[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            if (i >= nb) break;
            const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&raw[i]);
            const float2 v0 = __bfloat1622float2(h2[0]), v1 = __bfloat1622float2(h2[1]);
            float amax = fmaxf(fmaxf(fabsf(v0.x), fabsf(v0.y)), fmaxf(fabsf(v1.x), fabsf(v1.y)));
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
            const float sc = amax > 0.0f ? amax / 448.0f : 1.0f;
            const uint32_t lo =
                __nv_cvt_float2_to_fp8x2(make_float2(v0.x / sc, v0.y / sc), __NV_SATFINITE, __NV_E4M3);
            const uint32_t hi =
                __nv_cvt_float2_to_fp8x2(make_float2(v1.x / sc, v1.y / sc), __NV_SATFINITE, __NV_E4M3);
            code[i] = lo | (hi << 16);
            scale[i] = sc;
        }
        for (int l = 0; l < k; ++l) {
            const int64_t row = __shfl_sync(0xffffffffu, my.row, l);
            if (row < 0) continue;
            const int q = __shfl_sync(0xffffffffu, my.q, l);
            uint8_t* dst = static_cast<uint8_t*>(gd.rows[q]) + row * d;
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                if (i >= nb) break;
                reinterpret_cast<uint32_t*>(dst + (b0 + i) * 128)[lane] = code[i];
            }
            // lane i writes block b0+i's scale
            if (lane < nb) {
                float sc = scale[0];
#pragma unroll
                for (int i = 1; i < 8; ++i)
                    if (lane == i) sc = scale[i];
                gd.scales[q][row * nblk + b0 + lane] = sc;
            }
        }
    }
}

// INT8_CHANNEL: the row is quantised per token, s = amax / 127 (1 for a zero
// row), q = clamp(rn(x / s), -127, 127).  Pass 1 reduces amax over the row,
// pass 2 re-reads it (L1/L2 hits) and writes 8 int8 per 16-byte load to
// every kept route's row.
__global__ void __launch_bounds__(kThreads) dispatch_scatter_q8tok_kernel(
    const uint4* __restrict__ x, const int* __restrict__ idx, const int* __restrict__ route_slot,
    const int* __restrict__ row_base, const int* __restrict__ expert_start, int N, int E, int B, int k, int vecs,
    const GatherDst gd) {
    const int lane = threadIdx.x & 31;
    int64_t bt;
    int b, part;
    if (!token_of_warp(N, B, 1, bt, b, part)) return;
    const RouteDst my = route_dst(idx, route_slot, row_base, expert_start, gd, E, k, bt * k, b, lane);
    if (!__any_sync(0xffffffffu, my.row >= 0)) return;
    const uint4* src = x + bt * vecs;
    float amax = 0.0f;
    for (int v = lane; v < vecs; v += 32) {
        const uint4 raw = __ldg(src + v);
        const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float2 f = __bfloat1622float2(h2[i]);
            amax = fmaxf(amax, fmaxf(fabsf(f.x), fabsf(f.y)));
        }
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
    const float sc = amax > 0.0f ? amax / 127.0f : 1.0f;
    for (int v = lane; v < vecs; v += 32) {
        const uint4 raw = __ldg(src + v);
        const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&raw);
        uint32_t w[2] = {0u, 0u};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float2 f = __bfloat1622float2(h2[i]);
            const int q0 = max(-127, min(127, __float2int_rn(f.x / sc)));
            const int q1 = max(-127, min(127, __float2int_rn(f.y / sc)));
            w[i >> 1] |= ((uint32_t)(q0 & 0xff) | ((uint32_t)(q1 & 0xff) << 8)) << (16 * (i & 1));
        }
        for (int l = 0; l < k; ++l) {
            const int64_t row = __shfl_sync(0xffffffffu, my.row, l);
            if (row < 0) continue;
            uint2* dst = static_cast<uint2*>(gd.rows[__shfl_sync(0xffffffffu, my.q, l)]) + row * vecs;
            dst[v] = make_uint2(w[0], w[1]);
        }
    }
    if (lane < k && my.row >= 0) gd.scales[my.q][my.row] = sc;
}

// Expert-parallel plan of rank `me` from the kept-row table [P, E] (one CTA).
// Ownership: contiguous (expert e on rank e / (E/P), local index e % (E/P)) or
// strided (rank e % P, local index e / P -- spreads popular low-index experts
// over the ranks).  Layout (7E ints): owner[E] | row0[E] | g_rows[G] |
// g_start[G] | g_expert[G] | g_sender[G] | g_out_row[G], G = E, g = j * P + s.
__global__ void __launch_bounds__(256) ep_plan_kernel(const int* __restrict__ table, int P, int E, int me,
                                                      int strided, int* __restrict__ plan) {
    const int el = E / P;
    auto gexp = [&](int q, int j) { return strided ? j * P + q : q * el + j; };   // owner q's j-th expert
    auto to_owner = [&](int s, int q) {
        int n = 0;
        for (int j = 0; j < el; ++j) n += table[s * E + gexp(q, j)];
        return n;
    };
    auto recv_off = [&](int s, int q) {   // rows of senders < s in q's receive buffer
        int n = 0;
        for (int s2 = 0; s2 < s; ++s2) n += to_owner(s2, q);
        return n;
    };
    for (int e = threadIdx.x; e < E; e += blockDim.x) {
        const int q = strided ? e % P : e / el, lj = strided ? e / P : e % el;
        int within = 0;
        for (int j2 = 0; j2 < lj; ++j2) within += table[me * E + gexp(q, j2)];
        plan[e] = q;
        plan[E + e] = recv_off(me, q) + within;
    }
    for (int g = threadIdx.x; g < E; g += blockDim.x) {
        const int j = g / P, s = g - j * P;
        const int ge = gexp(me, j);
        int within = 0;
        for (int j2 = 0; j2 < j; ++j2) within += table[s * E + gexp(me, j2)];
        int start_in_sender = 0;   // first row of expert ge in sender s's dense expert-major layout
        for (int e2 = 0; e2 < ge; ++e2) start_in_sender += table[s * E + e2];
        plan[2 * E + g] = table[s * E + ge];
        plan[3 * E + g] = recv_off(s, me) + within;
        plan[4 * E + g] = j;
        plan[5 * E + g] = s;
        plan[6 * E + g] = start_in_sender;
    }
}

}  // namespace

cudaError_t launch_ep_plan(const int* table, int P, int E, int me, int strided, int* plan, cudaStream_t st) {
    ep_plan_kernel<<<1, 256, 0, st>>>(table, P, E, me, strided, plan);
    return cudaGetLastError();
}

// Route totals per (chunk, batch, expert); with `raw` also the shard's
// per-(batch, expert) totals.
cudaError_t launch_dispatch_count(const int* idx, const Shape& s, const Workspace& ws, int* counts, int* raw,
                                  cudaStream_t st) {
    if (s.T() == 0) {
        if (raw && s.B > 0) return cudaMemsetAsync(raw, 0, sizeof(int) * s.B * s.E, st);
        return cudaSuccess;
    }
    const dim3 grid(s.chunks(), s.B);
    dispatch_count_kernel<<<grid, kThreads, 0, st>>>(idx, s.N, s.k, s.E, s.chunks(), ws.chunk_count);
    if (raw)
        dispatch_scan_kernel<<<1, 256, 0, st>>>(ws.chunk_count, s.B, s.E, s.chunks(), s.cap, nullptr, raw,
                                                ws.chunk_base, counts, ws.row_base, ws.expert_rows,
                                                ws.expert_start);
    return cudaGetLastError();
}

// Slots (with the optional slot_base of earlier shards), drops, slot tables
// and the gather; needs launch_dispatch_count's histogram in ws.
cudaError_t launch_dispatch_finish(const void* x, const int* idx, const float* w, const Shape& s,
                                   const Workspace& ws, const GemmScales& sc, const int* slot_base, int* counts,
                                   int* token_ids, float* token_weights, void* a_rows, cudaStream_t st,
                                   bool skip_gather) {
    if (s.T() == 0) {
        cudaError_t e = cudaMemsetAsync(ws.expert_rows, 0, sizeof(int) * s.E, st);
        if (e == cudaSuccess) e = cudaMemsetAsync(ws.expert_start, 0, sizeof(int) * s.E, st);
        if (e == cudaSuccess && s.B > 0) e = cudaMemsetAsync(counts, 0, sizeof(int) * s.B * s.E, st);
        return e;
    }
    const dim3 grid(s.chunks(), s.B);
    dispatch_scan_kernel<<<1, 256, 0, st>>>(ws.chunk_count, s.B, s.E, s.chunks(), s.cap, slot_base, nullptr,
                                            ws.chunk_base, counts, ws.row_base, ws.expert_rows, ws.expert_start);
    dispatch_assign_kernel<<<grid, kThreads, 0, st>>>(idx, w, s.N, s.k, s.E, s.cap, s.chunks(), ws.chunk_base,
                                                      slot_base, token_ids, token_weights, ws.route_slot);
    return skip_gather ? cudaGetLastError()
                       : launch_dispatch_gather(x, idx, s, ws, sc, GatherDst{{a_rows}, {ws.a_scale}}, st);
}

// The row copy alone: every kept route's token row (quantised for the 8-bit
// formats) into its destination row; needs the route slots of the assign.
cudaError_t launch_dispatch_gather(const void* x, const int* idx, const Shape& s, const Workspace& ws,
                                   const GemmScales& sc, const GatherDst& gd, cudaStream_t st) {
    // 16-bit activations: rows of d elements = d/8 16-byte vectors.
    const int64_t tokens = (int64_t)s.B * s.N;
    if (tokens <= 0) return cudaSuccess;
    // split rows over several warps when the tokens alone leave the GPU
    // under-filled (32 warps per SM wanted); the per-token INT8 form needs
    // the whole row in one warp for its amax
    constexpr int64_t kWantWarps = 148 * 32;
    auto split_for = [&](int units) {
        const int64_t want = (kWantWarps + tokens - 1) / tokens;
        return (int)std::max<int64_t>(1, std::min<int64_t>(want, units));
    };
    const int split = s.dtype == MOE_DTYPE_INT8_CHANNEL ? 1
                      : s.dtype == MOE_DTYPE_FP8_BLOCK  ? split_for((s.d / 128 + 7) / 8)
                      : (s.dtype == MOE_DTYPE_INT8 || s.dtype == MOE_DTYPE_INT4_PTX || s.dtype == MOE_DTYPE_FP8)
                          ? split_for((s.d / 8 + 63) / 64)
                          : split_for((s.d / 8 + 127) / 128);
    const unsigned blocks = (unsigned)((tokens * split + kWarps - 1) / kWarps);
    const int* rs = ws.route_slot;
    if (s.dtype == MOE_DTYPE_FP8_BLOCK)
        dispatch_scatter_fp8_kernel<<<blocks, kThreads, 0, st>>>((const __nv_bfloat16*)x, idx, rs, ws.row_base,
                                                                 ws.expert_start, s.N, s.E, s.B, s.k, s.d, split, gd);
    else if (s.dtype == MOE_DTYPE_INT8_CHANNEL)
        dispatch_scatter_q8tok_kernel<<<blocks, kThreads, 0, st>>>((const uint4*)x, idx, rs, ws.row_base,
                                                                   ws.expert_start, s.N, s.E, s.B, s.k, s.d / 8, gd);
    else if (s.dtype == MOE_DTYPE_INT8)
        dispatch_scatter_q8_kernel<0><<<blocks, kThreads, 0, st>>>((const uint4*)x, idx, rs, ws.row_base,
                                                                   ws.expert_start, s.N, s.E, s.B, s.k, s.d / 8,
                                                                   split, sc.s_in, gd);
    else if (s.dtype == MOE_DTYPE_INT4_PTX)
        dispatch_scatter_q8_kernel<1><<<blocks, kThreads, 0, st>>>((const uint4*)x, idx, rs, ws.row_base,
                                                                   ws.expert_start, s.N, s.E, s.B, s.k, s.d / 8,
                                                                   split, sc.s_in, gd);
    else if (s.dtype == MOE_DTYPE_FP8)
        dispatch_scatter_q8_kernel<2><<<blocks, kThreads, 0, st>>>((const uint4*)x, idx, rs, ws.row_base,
                                                                   ws.expert_start, s.N, s.E, s.B, s.k, s.d / 8,
                                                                   split, sc.s_in, gd);
    else
        dispatch_scatter_kernel<<<blocks, kThreads, 0, st>>>((const uint4*)x, idx, rs, ws.row_base, ws.expert_start,
                                                             s.N, s.E, s.B, s.k, s.d / 8, split, gd);
    return cudaGetLastError();
}


}  // namespace moe
