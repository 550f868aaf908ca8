// Stage 4 with 4-bit weights (BASELINE config 5 format): INT4 asymmetric,
// group 128 along K, fp16 scale and zero per (group, output column),
// nibble-packed along N ([E, K, N/2] bytes; each 32-bit word holds 8
// consecutive columns interleaved so that column pair (2p, 2p+1) sits at bits
// 4p and 16+4p); bf16 activations; f32 accumulate.
//
//   w(k, n) = (q(k, n) - z(k/128, n)) * s(k/128, n)
//
// The weights travel from HBM as nibbles (a quarter of bf16's bytes) and are
// dequantised in shared memory by a converter warpgroup: each 64-row K stage
// of packed nibbles becomes bf16 w = fma(q, s, -z*s) in packed bf16x2 math
// (q from the magic constant 0x4300|q = 128+q, one shift + LOP3 per column
// pair) written straight into the 128B-swizzled MN-major layout the MMA
// reads, so the tensor cores run plain kind::f16 bf16 MMAs into TMEM with no
// per-group promotion.  (Dequantising to e4m3 instead would round every
// weight to a 3-bit mantissa -- ~6% relative error per weight -- which the
// 6e-2 bar of this format cannot absorb; bf16 keeps 2^-9.)
//
// kFmt = 1 runs NVFP4 weights through the same pipeline: e2m1 nibbles in the
// same packing, one e4m3 scale per (16 K-rows, column) and one f32 global
// scale per expert matrix, w = e2m1 * s * g.  The converter places the nibble's
// magnitude in bf16 bits 6..8 and its sign in bit 15, which as a bf16 value is
// exactly e2m1 * 2^-126 (code 1 lands on the subnormal 2^-127), and multiplies
// by the bf16 s * 2^118, so the staged weight is e2m1 * s * 2^-8 -- exact,
// since the product has at most 6 significant bits.  The epilogue applies
// g * 2^8 in f32 (the accumulators of one tile share one expert matrix).
//
// Warps (448 threads, persistent, one CTA per SM):
//   0      TMA: bf16 A tile (128 x 64, K-major SW128), packed B (64 K-rows x
//          256 columns / 2), the stage's 256 fp16 scales and zeros.
//   1      MMA: 4 x tcgen05.mma kind::f16 M128 N256 K16 per stage, double-
//          buffered TMEM accumulators.
//   2-5    epilogue (SwiGLU -> bf16 h, or f32 y), as the 16-bit kernel.
//   6-13   converter: nibbles -> bf16 into the stage's B buffer, then
//          fence.proxy.async and arrive on the stage's converted barrier.
#include "moe_internal.h"
#include "common.cuh"
#include "sm100.cuh"

#include <cuda.h>
#include <cuda_fp8.h>
#include <cudaTypedefs.h>

namespace moe {

bool make_map_box(CUtensorMap* map, const void* base, CUtensorMapDataType dt, int elem_bytes, uint64_t inner,
                  uint64_t outer, uint32_t box_inner, uint32_t box_outer, bool swizzle128);

namespace {

using namespace sm100;

constexpr int kBM = 128;
constexpr int kBK = 64;
constexpr int kStages = 3;
constexpr int kThreads = 448;   // 2 + 4 epilogue + 8 converter warps
constexpr int kConvThreads = 256;
constexpr int kABytes = kBM * 128;        // 16 KB
constexpr int kBBytes = 64 * 256 * 2;     // 32 KB bf16: 4 chunks of 64 columns x 64 K-rows
constexpr int kChunkBytes = 64 * 128;     // 8 KB
constexpr int kPBytes = 64 * 128;         // 8 KB packed nibbles
constexpr int kSZBytes = 512;             // 256 fp16 scales (and as many zeros)
constexpr int kStageBytes = kABytes + kBBytes + kPBytes + 2 * kSZBytes;   // 57 KB
constexpr int kTxBytes = kABytes + kPBytes + 2 * kSZBytes;
constexpr int kTmemCols = 512;
constexpr size_t kSmemBytes = 1024 + (size_t)kStages * kStageBytes + 256 + 4 * 2048;

struct W4Params {
    const int* g_rows;
    const int* g_start;
    const int* g_weight;
    int G;
    int K;
    int n_tiles;
    int out_ld;
    void* out;          // bf16 h (up/gate) or f32 y (down)
    const float* gs0;   // NVFP4: per-expert global scales (gate or down)
    const float* gs1;   // NVFP4: up
    int* status;
    uint32_t idesc;
};

struct W4Maps {
    CUtensorMap a;          // bf16 activations [rows, K]
    CUtensorMap p0, p1;     // packed weights [E*K, N/2] (gate, up; down uses p0)
    CUtensorMap s0, s1;     // fp16 scales [E*K/128, N]  (NVFP4: e4m3 scales [E*K/16, N])
    CUtensorMap z0, z1;     // fp16 zeros (unused by NVFP4)
};

__device__ __forceinline__ void decode_tile(int t, const int* pre, const int* mt, int G, int& g, int& m, int& n) {
    int lo = 0, hi = G - 1;
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (pre[mid] <= t) lo = mid; else hi = mid - 1;
    }
    g = lo;
    const int local = t - pre[g];
    n = local / mt[g];
    m = local - n * mt[g];
}

__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// kMode 0: up/gate + SwiGLU -> bf16 h;  1: down -> f32 y.
// kFmt 0: INT4 asymmetric g128;  1: NVFP4.
template <int kMode, int kFmt>
__global__ void __launch_bounds__(kThreads, 1)
    w4_gemm_kernel(const __grid_constant__ W4Maps mp, const W4Params p) {
    extern __shared__ uint8_t smem_raw[];
    __shared__ int s_pre[kMaxGroups + 1];
    __shared__ int s_mt[kMaxGroups];
    __shared__ int s_rows[kMaxGroups];
    __shared__ int s_start[kMaxGroups];
    __shared__ int s_wt[kMaxGroups];

    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* stage0 = smem;  // per stage: A | B | packed | scales | zeros
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + kStages * kStageBytes);
    uint64_t* conv = full + kStages;
    uint64_t* empty = conv + kStages;
    uint64_t* tfull = empty + kStages;
    uint64_t* tempty = tfull + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
    float4* sStage = reinterpret_cast<float4*>(smem + kStages * kStageBytes + 256);   // 4 epilogue warps x 2 KB
    auto sA = [&](int s) { return stage0 + s * kStageBytes; };
    auto sB = [&](int s) { return stage0 + s * kStageBytes + kABytes; };
    auto sP = [&](int s) { return stage0 + s * kStageBytes + kABytes + kBBytes; };
    auto sS = [&](int s) { return stage0 + s * kStageBytes + kABytes + kBBytes + kPBytes; };
    auto sZ = [&](int s) { return stage0 + s * kStageBytes + kABytes + kBBytes + kPBytes + kSZBytes; };

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&conv[s], kConvThreads);
            mbar_init(&empty[s], 1);
        }
        for (int a = 0; a < 2; ++a) { mbar_init(&tfull[a], 1); mbar_init(&tempty[a], 128); }
        fence_mbar_init();
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, kTmemCols);
        tmem_relinquish();
    }
    for (int g = threadIdx.x; g < p.G; g += kThreads) {
        const int r = p.g_rows[g];
        s_rows[g] = r;
        s_mt[g] = (r + kBM - 1) / kBM;
        s_start[g] = p.g_start[g];
        s_wt[g] = p.g_weight ? p.g_weight[g] : g;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        int acc = 0;
        for (int g = 0; g < p.G; ++g) { s_pre[g] = acc; acc += s_mt[g] * p.n_tiles; }
        s_pre[p.G] = acc;
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    const int total = s_pre[p.G];
    const int kblocks = p.K / kBK;
    const int groups_k = p.K / 128;

    if (warp == 0) {
        if (lane == 0) {
            int s = 0;
            uint32_t ph = 0;
            for (int t = blockIdx.x; t < total; t += gridDim.x) {
                int g, m, n;
                decode_tile(t, s_pre, s_mt, p.G, g, m, n);
                const int a_row = s_start[g] + m * kBM;
                const int b_row = s_wt[g] * p.K;
                const int sz_row0 = s_wt[g] * groups_k;
                const int fp4_row0 = s_wt[g] * (p.K / 16);
                for (int kb = 0; kb < kblocks; ++kb) {
                    if (!mbar_wait(&empty[s], ph ^ 1u, p.status, kDevErrTimeout)) goto producer_done;
                    mbar_arrive_expect_tx(&full[s], kTxBytes);
                    const int k0 = kb * kBK;
                    tma_load_2d(sA(s), &mp.a, &full[s], k0, a_row);
                    if (kMode == 0) {
                        tma_load_2d(sP(s), &mp.p0, &full[s], n * 64, b_row + k0);
                        tma_load_2d(sP(s) + kPBytes / 2, &mp.p1, &full[s], n * 64, b_row + k0);
                        if (kFmt == 0) {
                            tma_load_2d(sS(s), &mp.s0, &full[s], n * 128, sz_row0 + k0 / 128);
                            tma_load_2d(sS(s) + kSZBytes / 2, &mp.s1, &full[s], n * 128, sz_row0 + k0 / 128);
                            tma_load_2d(sZ(s), &mp.z0, &full[s], n * 128, sz_row0 + k0 / 128);
                            tma_load_2d(sZ(s) + kSZBytes / 2, &mp.z1, &full[s], n * 128, sz_row0 + k0 / 128);
                        } else {   // 4 groups of 16 K-rows x 128 columns of e4m3 scales each
                            tma_load_2d(sS(s), &mp.s0, &full[s], n * 128, fp4_row0 + k0 / 16);
                            tma_load_2d(sS(s) + kSZBytes, &mp.s1, &full[s], n * 128, fp4_row0 + k0 / 16);
                        }
                    } else {
                        tma_load_2d(sP(s), &mp.p0, &full[s], n * 128, b_row + k0);
                        if (kFmt == 0) {
                            tma_load_2d(sS(s), &mp.s0, &full[s], n * 256, sz_row0 + k0 / 128);
                            tma_load_2d(sZ(s), &mp.z0, &full[s], n * 256, sz_row0 + k0 / 128);
                        } else {   // 4 x 256 e4m3 scales
                            tma_load_2d(sS(s), &mp.s0, &full[s], n * 256, fp4_row0 + k0 / 16);
                        }
                    }
                    if (++s == kStages) { s = 0; ph ^= 1u; }
                }
            }
        producer_done:;
        }
    } else if (warp == 1) {
        if (lane == 0) {
            int s = 0, acc = 0;
            uint32_t ph = 0, aph = 0;
            for (int t = blockIdx.x; t < total; t += gridDim.x) {
                if (!mbar_wait(&tempty[acc], aph ^ 1u, p.status, kDevErrTimeout)) break;
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + acc * 256;
                bool ok = true;
                for (int kb = 0; kb < kblocks; ++kb) {
                    if (!mbar_wait(&conv[s], ph, p.status, kDevErrTimeout)) { ok = false; break; }
                    tc_fence_after();
                    const uint32_t a_base = smem_u32(sA(s));
                    const uint32_t b_base = smem_u32(sB(s));
#pragma unroll
                    for (int kk = 0; kk < 4; ++kk) {
                        const uint64_t adesc = smem_desc_sw128(a_base + kk * 32, 16, 1024);
                        const uint64_t bdesc = smem_desc_sw128(b_base + kk * 16 * 128, kChunkBytes, 1024);
                        mma_f16_ss(d_tmem, adesc, bdesc, p.idesc, (kb | kk) != 0 ? 1u : 0u);
                    }
                    mma_commit(&empty[s]);
                    if (++s == kStages) { s = 0; ph ^= 1u; }
                }
                if (!ok) break;
                mma_commit(&tfull[acc]);
                acc ^= 1;
                if (acc == 0) aph ^= 1u;
            }
        }
    } else if (warp < 6) {
        // ---------------- epilogue (warps 2..5) ----------------
        const int q = warp & 3;
        const int row_in_tile = q * 32 + lane;
        int acc = 0;
        uint32_t aph = 0;
        for (int t = blockIdx.x; t < total; t += gridDim.x) {
            int g, m, n;
            decode_tile(t, s_pre, s_mt, p.G, g, m, n);
            if (!mbar_wait_warp(&tfull[acc], aph, p.status, kDevErrTimeout)) break;
            tc_fence_after();
            const int row_local = m * kBM + row_in_tile;
            const bool valid = row_local < s_rows[g];
            const int64_t out_row = (int64_t)s_start[g] + row_local;
            const uint32_t taddr = tmem_base + ((uint32_t)(q * 32) << 16) + acc * 256;
            // NVFP4: the global scale times 2^8 (the staged weights carry 2^-8)
            const float gsa = kFmt == 1 ? p.gs0[s_wt[g]] * 256.0f : 1.0f;
            const float gsb = (kFmt == 1 && kMode == 0) ? p.gs1[s_wt[g]] * 256.0f : 1.0f;
            if (kMode == 0) {
                __nv_bfloat16* h = reinterpret_cast<__nv_bfloat16*>(p.out) + out_row * p.out_ld + n * 128;
#pragma unroll 1
                for (int c = 0; c < 128; c += 32) {
                    uint32_t gr[32], ur[32];
                    tmem_ld_32x32b_x32(taddr + c, gr);
                    tmem_ld_32x32b_x32(taddr + 128 + c, ur);
                    tmem_wait_ld();
                    if (c == 96) { tc_fence_before(); mbar_arrive(&tempty[acc]); }
                    uint32_t packed[16];
#pragma unroll
                    for (int i = 0; i < 16; ++i) {
                        float hv[2];
#pragma unroll
                        for (int j = 0; j < 2; ++j) {
                            const float gv = __uint_as_float(gr[2 * i + j]) * gsa;
                            const float uv = __uint_as_float(ur[2 * i + j]) * gsb;
                            hv[j] = uv * (gv / (1.0f + __expf(-gv)));
                        }
                        packed[i] = F16Traits<__nv_bfloat16>::pack2(hv[0], hv[1]);
                    }
                    if (valid) {
                        uint4* o = reinterpret_cast<uint4*>(h + c);
#pragma unroll
                        for (int v = 0; v < 4; ++v)
                            o[v] = make_uint4(packed[4 * v], packed[4 * v + 1], packed[4 * v + 2], packed[4 * v + 3]);
                    }
                }
            } else {
                const int warp_row0 = m * kBM + q * 32;
                const int nrows = s_rows[g] - warp_row0;
                float* y = reinterpret_cast<float*>(p.out) + ((int64_t)s_start[g] + warp_row0) * p.out_ld + n * 256;
                float4* stage = sStage + (warp - 2) * 128;
#pragma unroll 1
                for (int c = 0; c < 256; c += 32) {
                    uint32_t r[32];
                    tmem_ld_32x32b_x32(taddr + c, r);
                    tmem_wait_ld();
                    if (c == 224) { tc_fence_before(); mbar_arrive(&tempty[acc]); }
                    float v[32];
#pragma unroll
                    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]) * gsa;
                    warp_store_rows16(stage, v, y + c, p.out_ld, nrows, lane);
                    warp_store_rows16(stage, v + 16, y + c + 16, p.out_ld, nrows, lane);
                }
            }
            acc ^= 1;
            if (acc == 0) aph ^= 1u;
        }
    } else {
        // ---------------- converter (warps 6..13) ----------------
        // thread: 8-column unit u (columns 8u..8u+7) of K-rows rg, rg+8, ...
        const int ct = threadIdx.x - 192;
        const int u = ct & 31, rg = ct >> 5;
        const int chunk = u >> 3, uc = u & 7;
        const __nv_bfloat162 k128 = __floats2bfloat162_rn(128.0f, 128.0f);
        int s = 0;
        uint32_t ph = 0;
        bool ok = true;
        for (int t = blockIdx.x; t < total && ok; t += gridDim.x) {
            for (int kb = 0; kb < kblocks; ++kb) {
                if (!mbar_wait(&full[s], ph, p.status, kDevErrTimeout)) { ok = false; break; }
                if (kFmt == 0) {
                    __nv_bfloat162 sc[4], cc[4];
                    {
                        const uint4 s8 = *reinterpret_cast<const uint4*>(sS(s) + u * 16);
                        const uint4 z8 = *reinterpret_cast<const uint4*>(sZ(s) + u * 16);
                        const __half2* sh = reinterpret_cast<const __half2*>(&s8);
                        const __half2* zh = reinterpret_cast<const __half2*>(&z8);
    #pragma unroll
                        for (int i = 0; i < 4; ++i) {
                            const float2 sf = __half22float2(sh[i]), zf = __half22float2(zh[i]);
                            sc[i] = __floats2bfloat162_rn(sf.x, sf.y);
                            cc[i] = __floats2bfloat162_rn(-(zf.x * sf.x), -(zf.y * sf.y));
                        }
                    }
                    const uint8_t* src = sP(s);
                    uint8_t* dst = sB(s) + chunk * kChunkBytes;
    #pragma unroll 4
                    for (int j = 0; j < 8; ++j) {
                        const int k = rg + 8 * j;
                        const int off = kMode == 0 ? (u < 16 ? k * 64 + u * 4 : kPBytes / 2 + k * 64 + (u - 16) * 4)
                                                   : k * 128 + u * 4;
                        const uint32_t w = *reinterpret_cast<const uint32_t*>(src + off);
                        uint32_t o[4];
    #pragma unroll
                        for (int i = 0; i < 4; ++i) {
                            const uint32_t biased = ((w >> (4 * i)) & 0x000F000Fu) | 0x43004300u;   // bf16x2 128+q
                            const __nv_bfloat162 q = __hsub2(*reinterpret_cast<const __nv_bfloat162*>(&biased), k128);
                            const __nv_bfloat162 v = __hfma2(q, sc[i], cc[i]);
                            o[i] = *reinterpret_cast<const uint32_t*>(&v);
                        }
                        *reinterpret_cast<uint4*>(dst + k * 128 + ((uc ^ (k & 7)) << 4)) = make_uint4(o[0], o[1], o[2], o[3]);
                    }
                } else {
                    // e4m3 scales of this thread's 8 columns for the stage's 4 groups, as bf16 s * 2^118
                    __nv_bfloat162 sc[4][4];
#pragma unroll
                    for (int gi = 0; gi < 4; ++gi) {
                        const uint8_t* sp = kMode == 0 ? (u < 16 ? sS(s) + gi * 128 + 8 * u
                                                                 : sS(s) + 512 + gi * 128 + 8 * (u - 16))
                                                       : sS(s) + gi * 256 + 8 * u;
                        const uint2 raw = *reinterpret_cast<const uint2*>(sp);
#pragma unroll
                        for (int i = 0; i < 4; ++i) {
                            const uint32_t word = i < 2 ? raw.x : raw.y;
                            const __nv_fp8x2_storage_t pr = (__nv_fp8x2_storage_t)((word >> (16 * (i & 1))) & 0xFFFFu);
                            const float2 f = __half22float2(__half2(__nv_cvt_fp8x2_to_halfraw2(pr, __NV_E4M3)));
                            sc[gi][i] = __floats2bfloat162_rn(f.x * 0x1p118f, f.y * 0x1p118f);
                        }
                    }
                    const uint8_t* src = sP(s);
                    uint8_t* dst = sB(s) + chunk * kChunkBytes;
#pragma unroll
                    for (int j = 0; j < 8; ++j) {
                        const int k = rg + 8 * j;   // K-row k of the stage is in group j / 2
                        const int off = kMode == 0 ? (u < 16 ? k * 64 + u * 4 : kPBytes / 2 + k * 64 + (u - 16) * 4)
                                                   : k * 128 + u * 4;
                        const uint32_t w = *reinterpret_cast<const uint32_t*>(src + off);
                        uint32_t o[4];
#pragma unroll
                        for (int i = 0; i < 4; ++i) {
                            const uint32_t sh = w >> (4 * i);
                            const uint32_t bits = ((sh << 6) & 0x01C001C0u) | ((sh << 12) & 0x80008000u);
                            const __nv_bfloat162 v =
                                __hmul2(*reinterpret_cast<const __nv_bfloat162*>(&bits), sc[j >> 1][i]);
                            o[i] = *reinterpret_cast<const uint32_t*>(&v);
                        }
                        *reinterpret_cast<uint4*>(dst + k * 128 + ((uc ^ (k & 7)) << 4)) =
                            make_uint4(o[0], o[1], o[2], o[3]);
                    }
                }
                fence_proxy_async_smem();
                mbar_arrive(&conv[s]);
                if (++s == kStages) { s = 0; ph ^= 1u; }
            }
        }
    }
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, kTmemCols);
    }
}

template <int kMode, int kFmt>
cudaError_t launch(const W4Maps& mp, const W4Params& p, cudaStream_t st, int num_sms) {
    auto kern = w4_gemm_kernel<kMode, kFmt>;
    cudaError_t err = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemBytes);
    if (err != cudaSuccess) return err;
    kern<<<num_sms, kThreads, kSmemBytes, st>>>(mp, p);
    return cudaGetLastError();
}

bool packed_map(CUtensorMap* m, const void* w, uint64_t rows, uint64_t n_cols, uint32_t box_cols) {
    return make_map_box(m, w, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, n_cols / 2, rows, box_cols / 2, kBK, false);
}
bool sz_map(CUtensorMap* m, const void* sz, uint64_t rows, uint64_t n_cols, uint32_t box_cols) {
    return make_map_box(m, sz, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, n_cols, rows, box_cols, 1, false);
}
// NVFP4 e4m3 scales [E*K/16, N]: 4 group rows (one 64-row stage) per box
bool fp4_scale_map(CUtensorMap* m, const void* sc, uint64_t rows, uint64_t n_cols, uint32_t box_cols) {
    return make_map_box(m, sc, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, n_cols, rows, box_cols, kBK / 16, false);
}

}  // namespace

cudaError_t launch_w4_up_gate(const void* a_rows, const void* w_gate, const void* w_up, const void* s_gate,
                              const void* s_up, const void* z_gate, const void* z_up, const Shape& s,
                              const GroupTable& gt, int* status, void* h_rows, cudaStream_t st, int num_sms) {
    if (gt.G <= 0 || gt.rows_capacity <= 0) return cudaSuccess;
    W4Maps mp;
    const uint64_t wrows = (uint64_t)s.E * s.d, grows = (uint64_t)s.E * (s.d / 128);
    if (!make_map_box(&mp.a, a_rows, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, s.d, gt.rows_capacity, 64, kBM, true) ||
        !packed_map(&mp.p0, w_gate, wrows, s.f, 128) || !packed_map(&mp.p1, w_up, wrows, s.f, 128) ||
        !sz_map(&mp.s0, s_gate, grows, s.f, 128) || !sz_map(&mp.s1, s_up, grows, s.f, 128) ||
        !sz_map(&mp.z0, z_gate, grows, s.f, 128) || !sz_map(&mp.z1, z_up, grows, s.f, 128))
        return cudaErrorInvalidValue;
    W4Params p{};
    p.g_rows = gt.rows;
    p.g_start = gt.start;
    p.g_weight = gt.weight;
    p.G = gt.G;
    p.K = s.d;
    p.n_tiles = s.f / 128;
    p.out_ld = s.f;
    p.out = h_rows;
    p.status = status;
    p.idesc = idesc_f16(true, kBM, 256, false, true);
    return launch<0, 0>(mp, p, st, num_sms);
}

cudaError_t launch_w4_down(const void* h_rows, const void* w_down, const void* s_down, const void* z_down,
                           const Shape& s, const GroupTable& gt, int* status, float* y_rows, cudaStream_t st,
                           int num_sms) {
    if (gt.G <= 0 || gt.rows_capacity <= 0) return cudaSuccess;
    W4Maps mp;
    const uint64_t wrows = (uint64_t)s.E * s.f, grows = (uint64_t)s.E * (s.f / 128);
    if (!make_map_box(&mp.a, h_rows, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, s.f, gt.rows_capacity, 64, kBM, true) ||
        !packed_map(&mp.p0, w_down, wrows, s.d, 256) || !sz_map(&mp.s0, s_down, grows, s.d, 256) ||
        !sz_map(&mp.z0, z_down, grows, s.d, 256))
        return cudaErrorInvalidValue;
    mp.p1 = mp.p0;
    mp.s1 = mp.s0;
    mp.z1 = mp.z0;
    W4Params p{};
    p.g_rows = gt.rows;
    p.g_start = gt.start;
    p.g_weight = gt.weight;
    p.G = gt.G;
    p.K = s.f;
    p.n_tiles = s.d / 256;
    p.out_ld = s.d;
    p.out = y_rows;
    p.status = status;
    p.idesc = idesc_f16(true, kBM, 256, false, true);
    return launch<1, 0>(mp, p, st, num_sms);
}

cudaError_t launch_fp4_up_gate(const void* a_rows, const void* w_gate, const void* w_up, const void* s_gate,
                               const void* s_up, const float* g_gate, const float* g_up, const Shape& s,
                               const GroupTable& gt, int* status, void* h_rows, cudaStream_t st, int num_sms) {
    if (gt.G <= 0 || gt.rows_capacity <= 0) return cudaSuccess;
    W4Maps mp;
    const uint64_t wrows = (uint64_t)s.E * s.d, grows = (uint64_t)s.E * (s.d / 16);
    if (!make_map_box(&mp.a, a_rows, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, s.d, gt.rows_capacity, 64, kBM, true) ||
        !packed_map(&mp.p0, w_gate, wrows, s.f, 128) || !packed_map(&mp.p1, w_up, wrows, s.f, 128) ||
        !fp4_scale_map(&mp.s0, s_gate, grows, s.f, 128) || !fp4_scale_map(&mp.s1, s_up, grows, s.f, 128))
        return cudaErrorInvalidValue;
    mp.z0 = mp.s0;
    mp.z1 = mp.s1;
    W4Params p{};
    p.g_rows = gt.rows;
    p.g_start = gt.start;
    p.g_weight = gt.weight;
    p.G = gt.G;
    p.K = s.d;
    p.n_tiles = s.f / 128;
    p.out_ld = s.f;
    p.out = h_rows;
    p.gs0 = g_gate;
    p.gs1 = g_up;
    p.status = status;
    p.idesc = idesc_f16(true, kBM, 256, false, true);
    return launch<0, 1>(mp, p, st, num_sms);
}

cudaError_t launch_fp4_down(const void* h_rows, const void* w_down, const void* s_down, const float* g_down,
                            const Shape& s, const GroupTable& gt, int* status, float* y_rows, cudaStream_t st,
                            int num_sms) {
    if (gt.G <= 0 || gt.rows_capacity <= 0) return cudaSuccess;
    W4Maps mp;
    const uint64_t wrows = (uint64_t)s.E * s.f, grows = (uint64_t)s.E * (s.f / 16);
    if (!make_map_box(&mp.a, h_rows, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, s.f, gt.rows_capacity, 64, kBM, true) ||
        !packed_map(&mp.p0, w_down, wrows, s.d, 256) || !fp4_scale_map(&mp.s0, s_down, grows, s.d, 256))
        return cudaErrorInvalidValue;
    mp.p1 = mp.p0;
    mp.s1 = mp.s0;
    mp.z0 = mp.s0;
    mp.z1 = mp.s0;
    W4Params p{};
    p.g_rows = gt.rows;
    p.g_start = gt.start;
    p.g_weight = gt.weight;
    p.G = gt.G;
    p.K = s.f;
    p.n_tiles = s.d / 256;
    p.out_ld = s.d;
    p.out = y_rows;
    p.gs0 = g_down;
    p.gs1 = g_down;
    p.status = status;
    p.idesc = idesc_f16(true, kBM, 256, false, true);
    return launch<1, 1>(mp, p, st, num_sms);
}

}  // namespace moe
