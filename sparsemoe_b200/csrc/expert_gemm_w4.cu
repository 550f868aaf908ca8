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
// Tile: 256 rows x 128 columns (up/gate: 64 gate + 64 up columns of the same
// 64 h features).  Both 128-row halves multiply the same converted B stage,
// so each dequantised weight serves 256 rows -- the converter's work per
// FLOP is half that of a 128-row tile.
//
// Warps (448 threads, persistent, one CTA per SM):
//   0      TMA: bf16 A tile (256 x 64, K-major SW128), packed B (64 K-rows x
//          128 columns / 2), the stage's scales (and INT4 zeros).
//   1      MMA: per K16 step 2 x tcgen05.mma kind::f16 M128 N128 (one per row
//          half) into a 256-column TMEM accumulator, double-buffered.
//   2-5    epilogue (SwiGLU -> bf16 h, or f32 y rows stored coalesced).
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

// Tile shapes (kBM x kBN = 32768): 256 x 128 when experts hold many rows (each
// converted B stage then feeds two M128 MMAs), 128 x 256 when they hold few
// (decode: fewer N tiles, so the activations are re-read fewer times).
template <int kBM>
struct Tile {
    static constexpr int BM = kBM;
    static constexpr int BN = 32768 / kBM;
    static constexpr int kHalves = kBM / 128;            // M128 MMAs per K step
    static constexpr int kABytes = kBM * 128;            // kBM rows x 64 bf16
    static constexpr int kBBytes = 64 * BN * 2;          // bf16 B: BN/64 chunks of 64 columns x 64 K-rows
    static constexpr int kPBytes = 64 * BN / 2;          // packed nibbles
    static constexpr int kSZBytes = 4 * BN;              // INT4: BN fp16 scales + BN zeros; NVFP4: 4 x BN e4m3
    // Two rings: kRaw TMA stages (A, packed weights, scales) and kBSt converted
    // bf16 B stages, so loads, conversion and MMAs overlap across stages;
    // every A and B buffer sits on a 1024-byte boundary (128B swizzle atoms).
    // 4 + 3 stages fill 230.7 KB of the 232 KB a CTA may use for both tiles.
    static constexpr int kRawBytes = (kABytes + kPBytes + kSZBytes + 1023) / 1024 * 1024;
    static constexpr int kRaw = 4;
    static constexpr int kBSt = 3;   // the converter runs up to two stages ahead of the MMA
    static constexpr int kTxBytes = kABytes + kPBytes + kSZBytes;
    static constexpr size_t kSmemBytes = 1024 + (size_t)kRaw * kRawBytes + (size_t)kBSt * kBBytes + 256 + 4 * 2048;
    // dynamic + the kernel's static group tables (5 x kMaxGroups ints + 1) within a CTA's 227 KB
    static_assert(kSmemBytes + sizeof(int) * (5 * kMaxGroups + 1) <= 232448, "shared memory per CTA");
    static constexpr int kUnits = BN / 8;                 // converter: 8-column units
    static constexpr int kRowGroups = 256 / kUnits;       // converter threads per unit
    static constexpr int kRowsPerThread = 64 / kRowGroups;
};
constexpr int kBK = 64;
constexpr int kThreads = 448;             // 2 + 4 epilogue + 8 converter warps
constexpr int kConvThreads = 256;
constexpr int kChunkBytes = 64 * 128;     // 8 KB
constexpr int kTmemCols = 512;            // 2 accumulators x 256 columns

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
    OutRedirect red;    // down: optional peer destination of each group's rows
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
// kFmt 0: INT4 asymmetric g128;  1: NVFP4.  kBM: tile rows (128 or 256).
template <int kMode, int kFmt, int kBM>
__global__ void __launch_bounds__(kThreads, 1)
    w4_gemm_kernel(const __grid_constant__ W4Maps mp, const W4Params p) {
    using TL = Tile<kBM>;
    constexpr int kBN = TL::BN;
    constexpr int kABytes = TL::kABytes, kBBytes = TL::kBBytes, kPBytes = TL::kPBytes;
    constexpr int kRaw = TL::kRaw, kBSt = TL::kBSt, kRawBytes = TL::kRawBytes;
    extern __shared__ uint8_t smem_raw[];
    __shared__ int s_pre[kMaxGroups + 1];
    __shared__ int s_mt[kMaxGroups];
    __shared__ int s_rows[kMaxGroups];
    __shared__ int s_start[kMaxGroups];
    __shared__ int s_wt[kMaxGroups];

    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* raw0 = smem;                                  // kRaw x [A | packed | scales (| zeros)]
    uint8_t* bst0 = smem + kRaw * kRawBytes;               // kBSt x converted bf16 B
    uint64_t* full = reinterpret_cast<uint64_t*>(bst0 + kBSt * kBBytes);   // raw stage loaded
    uint64_t* empty = full + kRaw;                         // raw stage consumed (MMA done)
    uint64_t* conv = empty + kRaw;                         // B stage converted
    uint64_t* bfree = conv + kBSt;                         // B stage consumed (MMA done)
    uint64_t* tfull = bfree + kBSt;
    uint64_t* tempty = tfull + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
    float4* sStage = reinterpret_cast<float4*>(bst0 + kBSt * kBBytes + 256);   // 4 epilogue warps x 2 KB
    auto sA = [&](int s) { return raw0 + s * kRawBytes; };
    auto sP = [&](int s) { return raw0 + s * kRawBytes + kABytes; };
    auto sS = [&](int s) { return raw0 + s * kRawBytes + kABytes + kPBytes; };
    auto sB = [&](int b) { return bst0 + b * kBBytes; };

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int s = 0; s < kRaw; ++s) { mbar_init(&full[s], 1); mbar_init(&empty[s], 1); }
        for (int b = 0; b < kBSt; ++b) { mbar_init(&conv[b], kConvThreads); mbar_init(&bfree[b], 1); }
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
                    mbar_arrive_expect_tx(&full[s], TL::kTxBytes);
                    const int k0 = kb * kBK;
                    tma_load_2d(sA(s), &mp.a, &full[s], k0, a_row);
                    if (kMode == 0) {   // kBN/2 gate + kBN/2 up columns = n * kBN/4 bytes of nibbles
                        tma_load_2d(sP(s), &mp.p0, &full[s], n * (kBN / 4), b_row + k0);
                        tma_load_2d(sP(s) + kPBytes / 2, &mp.p1, &full[s], n * (kBN / 4), b_row + k0);
                        if (kFmt == 0) {   // scales [gate | up], then zeros [gate | up], kBN/2 fp16 each
                            tma_load_2d(sS(s), &mp.s0, &full[s], n * (kBN / 2), sz_row0 + k0 / 128);
                            tma_load_2d(sS(s) + kBN, &mp.s1, &full[s], n * (kBN / 2), sz_row0 + k0 / 128);
                            tma_load_2d(sS(s) + 2 * kBN, &mp.z0, &full[s], n * (kBN / 2), sz_row0 + k0 / 128);
                            tma_load_2d(sS(s) + 3 * kBN, &mp.z1, &full[s], n * (kBN / 2), sz_row0 + k0 / 128);
                        } else {   // [gate: 4 groups x kBN/2] [up: 4 groups x kBN/2] e4m3
                            tma_load_2d(sS(s), &mp.s0, &full[s], n * (kBN / 2), fp4_row0 + k0 / 16);
                            tma_load_2d(sS(s) + 2 * kBN, &mp.s1, &full[s], n * (kBN / 2), fp4_row0 + k0 / 16);
                        }
                    } else {
                        tma_load_2d(sP(s), &mp.p0, &full[s], n * (kBN / 2), b_row + k0);
                        if (kFmt == 0) {
                            tma_load_2d(sS(s), &mp.s0, &full[s], n * kBN, sz_row0 + k0 / 128);
                            tma_load_2d(sS(s) + 2 * kBN, &mp.z0, &full[s], n * kBN, sz_row0 + k0 / 128);
                        } else {   // 4 groups x kBN e4m3 scales
                            tma_load_2d(sS(s), &mp.s0, &full[s], n * kBN, fp4_row0 + k0 / 16);
                        }
                    }
                    if (++s == kRaw) { s = 0; ph ^= 1u; }
                }
            }
        producer_done:;
        }
    } else if (warp == 1) {
        if (lane == 0) {
            int s = 0, b = 0, acc = 0;
            uint32_t ph = 0, bph = 0, aph = 0;
            for (int t = blockIdx.x; t < total; t += gridDim.x) {
                if (!mbar_wait(&tempty[acc], aph ^ 1u, p.status, kDevErrTimeout)) break;
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + acc * 256;   // kHalves x kBN columns
                bool ok = true;
                for (int kb = 0; kb < kblocks; ++kb) {
                    // the converter finished B[b], so raw stage s (same K step) has landed too
                    if (!mbar_wait(&conv[b], bph, p.status, kDevErrTimeout)) { ok = false; break; }
                    tc_fence_after();
                    const uint32_t a_base = smem_u32(sA(s));
                    const uint32_t b_base = smem_u32(sB(b));
#pragma unroll
                    for (int kk = 0; kk < 4; ++kk) {
                        const uint64_t bdesc = smem_desc_sw128(b_base + kk * 16 * 128, kChunkBytes, 1024);
                        const uint32_t accum = (kb | kk) != 0 ? 1u : 0u;
#pragma unroll
                        for (int hm = 0; hm < TL::kHalves; ++hm) {   // row halves: A rows 128*hm.. at 16 KB * hm
                            const uint64_t adesc = smem_desc_sw128(a_base + hm * 16384 + kk * 32, 16, 1024);
                            mma_f16_ss(d_tmem + hm * kBN, adesc, bdesc, p.idesc, accum);
                        }
                    }
                    mma_commit(&empty[s]);
                    mma_commit(&bfree[b]);
                    if (++s == kRaw) { s = 0; ph ^= 1u; }
                    if (++b == kBSt) { b = 0; bph ^= 1u; }
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
        int acc = 0;
        uint32_t aph = 0;
        float4* stage = sStage + (warp - 2) * 128;
        for (int t = blockIdx.x; t < total; t += gridDim.x) {
            int g, m, n;
            decode_tile(t, s_pre, s_mt, p.G, g, m, n);
            if (!mbar_wait_warp(&tfull[acc], aph, p.status, kDevErrTimeout)) break;
            tc_fence_after();
            // NVFP4: the global scale times 2^8 (the staged weights carry 2^-8)
            const float gsa = kFmt == 1 ? p.gs0[s_wt[g]] * 256.0f : 1.0f;
            const float gsb = (kFmt == 1 && kMode == 0) ? p.gs1[s_wt[g]] * 256.0f : 1.0f;
#pragma unroll 1
            for (int hm = 0; hm < TL::kHalves; ++hm) {
                const int warp_row0 = m * kBM + hm * 128 + q * 32;
                const int row_local = warp_row0 + lane;
                const bool valid = row_local < s_rows[g];
                const uint32_t taddr = tmem_base + ((uint32_t)(q * 32) << 16) + acc * 256 + hm * kBN;
                const bool last_half = hm == TL::kHalves - 1;
                if (kMode == 0) {
                    __nv_bfloat16* h = reinterpret_cast<__nv_bfloat16*>(p.out) +
                                       ((int64_t)s_start[g] + row_local) * p.out_ld + n * (kBN / 2);
#pragma unroll 1
                    for (int c = 0; c < kBN / 2; c += 32) {
                        uint32_t gr[32], ur[32];
                        tmem_ld_32x32b_x32(taddr + c, gr);
                        tmem_ld_32x32b_x32(taddr + kBN / 2 + c, ur);
                        tmem_wait_ld();
                        if (last_half && c == kBN / 2 - 32) { tc_fence_before(); mbar_arrive(&tempty[acc]); }
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
                    const int nrows = s_rows[g] - warp_row0;
                    float* y = down_rows(p.red, reinterpret_cast<float*>(p.out), g, s_start[g], p.out_ld) +
                               (int64_t)warp_row0 * p.out_ld + n * kBN;
#pragma unroll 1
                    for (int c = 0; c < kBN; c += 32) {
                        uint32_t r[32];
                        tmem_ld_32x32b_x32(taddr + c, r);
                        tmem_wait_ld();
                        if (last_half && c == kBN - 32) { tc_fence_before(); mbar_arrive(&tempty[acc]); }
                        float v[32];
#pragma unroll
                        for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]) * gsa;
                        warp_store_rows16(stage, v, y + c, p.out_ld, nrows, lane);
                        warp_store_rows16(stage, v + 16, y + c + 16, p.out_ld, nrows, lane);
                    }
                }
            }
            acc ^= 1;
            if (acc == 0) aph ^= 1u;
        }
        if (kMode == 1 && p.red.rank) __threadfence_system();   // peer rows visible before the kernel ends
    } else {
        // ---------------- converter (warps 6..13) ----------------
        // thread: 8-column unit u of the kBN columns, K rows krow0 + kRowGroups*j.
        // Up/gate: the first kUnits/2 units are gate columns, the rest up; the
        // up units take K rows rg ^ (32 / kUnits), so one warp's gate and up
        // nibble loads land in distinct shared-memory bank ranges.
        constexpr int kU = TL::kUnits, kRG = TL::kRowGroups;
        constexpr int kPRow = kMode == 0 ? kBN / 4 : kBN / 2;   // packed bytes per K row (per half)
        const int ct = threadIdx.x - 192;
        const int u = ct % kU, rg = ct / kU;
        const int chunk = u >> 3, uc = u & 7;
        const bool up_unit = kMode == 0 && u >= kU / 2;
        const int ul = up_unit ? u - kU / 2 : u;          // unit within its half
        const int krow0 = up_unit ? (rg ^ (32 / kU)) : rg;
        const int p_base = up_unit ? kPBytes / 2 : 0;
        const __nv_bfloat162 k128 = __floats2bfloat162_rn(128.0f, 128.0f);
        int s = 0, b = 0;
        uint32_t ph = 0, bph = 0;
        bool ok = true;
        for (int t = blockIdx.x; t < total && ok; t += gridDim.x) {
            for (int kb = 0; kb < kblocks; ++kb) {
                if (!mbar_wait(&full[s], ph, p.status, kDevErrTimeout) ||
                    !mbar_wait(&bfree[b], bph ^ 1u, p.status, kDevErrTimeout)) {
                    ok = false;
                    break;
                }
                const uint8_t* src = sP(s) + p_base;
                uint8_t* dst = sB(b) + chunk * kChunkBytes;
                if (kFmt == 0) {
                    __nv_bfloat162 sc[4], cc[4];
                    {
                        // fp16 scales at [0, 2 kBN) bytes, zeros at [2 kBN, 4 kBN); gate | up halves
                        const int so = (up_unit ? kBN : 0) + ul * 16;
                        const uint4 s8 = *reinterpret_cast<const uint4*>(sS(s) + so);
                        const uint4 z8 = *reinterpret_cast<const uint4*>(sS(s) + 2 * kBN + so);
                        const __half2* sh = reinterpret_cast<const __half2*>(&s8);
                        const __half2* zh = reinterpret_cast<const __half2*>(&z8);
#pragma unroll
                        for (int i = 0; i < 4; ++i) {
                            const float2 sf = __half22float2(sh[i]), zf = __half22float2(zh[i]);
                            sc[i] = __floats2bfloat162_rn(sf.x, sf.y);
                            cc[i] = __floats2bfloat162_rn(-(zf.x * sf.x), -(zf.y * sf.y));
                        }
                    }
#pragma unroll
                    for (int j = 0; j < TL::kRowsPerThread; ++j) {
                        const int k = krow0 + kRG * j;
                        const uint32_t w = *reinterpret_cast<const uint32_t*>(src + k * kPRow + ul * 4);
                        uint32_t o[4];
#pragma unroll
                        for (int i = 0; i < 4; ++i) {
                            const uint32_t biased = ((w >> (4 * i)) & 0x000F000Fu) | 0x43004300u;   // bf16x2 128+q
                            const __nv_bfloat162 qv =
                                __hsub2(*reinterpret_cast<const __nv_bfloat162*>(&biased), k128);
                            const __nv_bfloat162 v = __hfma2(qv, sc[i], cc[i]);
                            o[i] = *reinterpret_cast<const uint32_t*>(&v);
                        }
                        *reinterpret_cast<uint4*>(dst + k * 128 + ((uc ^ (k & 7)) << 4)) =
                            make_uint4(o[0], o[1], o[2], o[3]);
                    }
                } else {
                    // e4m3 scales: up/gate [gate: 4 x kBN/2 | up: 4 x kBN/2], down 4 x kBN; K row k of
                    // the stage is in group k / 16; scales become bf16 s * 2^118
                    constexpr int kSRow = kMode == 0 ? kBN / 2 : kBN;
                    const uint8_t* sbase = sS(s) + (up_unit ? 2 * kBN : 0) + 8 * ul;
                    __nv_bfloat162 sc[4][4];   // [group][column pair]
#pragma unroll
                    for (int gi = 0; gi < 4; ++gi) {
                        const uint2 raw = *reinterpret_cast<const uint2*>(sbase + gi * kSRow);
#pragma unroll
                        for (int i = 0; i < 4; ++i) {
                            const uint32_t word = i < 2 ? raw.x : raw.y;
                            const __nv_fp8x2_storage_t pr =
                                (__nv_fp8x2_storage_t)((word >> (16 * (i & 1))) & 0xFFFFu);
                            const float2 f = __half22float2(__half2(__nv_cvt_fp8x2_to_halfraw2(pr, __NV_E4M3)));
                            sc[gi][i] = __floats2bfloat162_rn(f.x * 0x1p118f, f.y * 0x1p118f);
                        }
                    }
#pragma unroll
                    for (int j = 0; j < TL::kRowsPerThread; ++j) {
                        const int k = krow0 + kRG * j;   // krow0 < kRG <= 16: group (kRG * j) / 16
                        const uint32_t w = *reinterpret_cast<const uint32_t*>(src + k * kPRow + ul * 4);
                        uint32_t o[4];
#pragma unroll
                        for (int i = 0; i < 4; ++i) {
                            const uint32_t sh = w >> (4 * i);
                            const uint32_t bits = ((sh << 6) & 0x01C001C0u) | ((sh << 12) & 0x80008000u);
                            const __nv_bfloat162 v = __hmul2(*reinterpret_cast<const __nv_bfloat162*>(&bits),
                                                             sc[(kRG * j) >> 4][i]);
                            o[i] = *reinterpret_cast<const uint32_t*>(&v);
                        }
                        *reinterpret_cast<uint4*>(dst + k * 128 + ((uc ^ (k & 7)) << 4)) =
                            make_uint4(o[0], o[1], o[2], o[3]);
                    }
                }
                fence_proxy_async_smem();
                mbar_arrive(&conv[b]);
                if (++s == kRaw) { s = 0; ph ^= 1u; }
                if (++b == kBSt) { b = 0; bph ^= 1u; }
            }
        }
    }
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, kTmemCols);
    }
}

template <int kMode, int kFmt, int kBM>
cudaError_t launch_bm(const W4Maps& mp, const W4Params& p, cudaStream_t st, int num_sms) {
    auto kern = w4_gemm_kernel<kMode, kFmt, kBM>;
    constexpr size_t smem = Tile<kBM>::kSmemBytes;
    static SmemAttr attr;
    cudaError_t err = ensure_smem(kern, smem, attr);
    if (err != cudaSuccess) return err;
    kern<<<num_sms, kThreads, smem, st>>>(mp, p);
    return cudaGetLastError();
}

// 256-row tiles when the groups average at least 256 rows of capacity
bool tall_tiles(const GroupTable& gt) { return gt.rows_capacity / gt.G >= 256; }



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

// One GEMM of the 4-bit path.  kMode 0: w0/w1 = gate/up [E, d, f/2], output
// h [rows, f]; kMode 1: w0 = down [E, f, d/2], output f32 y [rows, d].
// INT4 (kFmt 0): s/z fp16 [E, K/128, N]; NVFP4: s e4m3 [E, K/16, N], g f32 [E].
template <int kMode, int kFmt, int kBM>
cudaError_t launch_fmt(const void* a_rows, const void* w0, const void* w1, const void* s0, const void* s1,
                       const void* z0, const void* z1, const float* g0, const float* g1, const Shape& s,
                       const GroupTable& gt, int* status, void* out, cudaStream_t st, int num_sms) {
    constexpr int kBN = Tile<kBM>::BN;
    const int K = kMode == 0 ? s.d : s.f, N = kMode == 0 ? s.f : s.d;
    const uint32_t box = kMode == 0 ? kBN / 2 : kBN;   // weight columns per operand per tile
    const uint64_t wrows = (uint64_t)s.E * K;
    const uint64_t srows = (uint64_t)s.E * (kFmt == 0 ? K / 128 : K / 16);
    W4Maps mp;
    bool ok = make_map_box(&mp.a, a_rows, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, K, gt.rows_capacity, 64, kBM, true) &&
              packed_map(&mp.p0, w0, wrows, N, box) && packed_map(&mp.p1, kMode == 0 ? w1 : w0, wrows, N, box);
    if (kFmt == 0)
        ok = ok && sz_map(&mp.s0, s0, srows, N, box) && sz_map(&mp.s1, kMode == 0 ? s1 : s0, srows, N, box) &&
             sz_map(&mp.z0, z0, srows, N, box) && sz_map(&mp.z1, kMode == 0 ? z1 : z0, srows, N, box);
    else {
        ok = ok && fp4_scale_map(&mp.s0, s0, srows, N, box) &&
             fp4_scale_map(&mp.s1, kMode == 0 ? s1 : s0, srows, N, box);
        mp.z0 = mp.s0;
        mp.z1 = mp.s1;
    }
    if (!ok) return cudaErrorInvalidValue;
    W4Params p{};
    p.g_rows = gt.rows;
    p.g_start = gt.start;
    p.g_weight = gt.weight;
    p.G = gt.G;
    p.status = status;
    p.idesc = idesc_f16(true, 128, kBN, false, true);
    p.K = K;
    p.n_tiles = kMode == 0 ? N / (kBN / 2) : N / kBN;
    p.out_ld = N;
    p.out = out;
    p.gs0 = g0;
    p.gs1 = kMode == 0 ? g1 : g0;
    if (kMode == 1) p.red = gt.redirect;
    return launch_bm<kMode, kFmt, kBM>(mp, p, st, num_sms);
}

template <int kMode, int kFmt>
cudaError_t launch_any(const void* a_rows, const void* w0, const void* w1, const void* s0, const void* s1,
                       const void* z0, const void* z1, const float* g0, const float* g1, const Shape& s,
                       const GroupTable& gt, int* status, void* out, cudaStream_t st, int num_sms) {
    if (gt.G <= 0 || gt.rows_capacity <= 0) return cudaSuccess;
    return tall_tiles(gt)
               ? launch_fmt<kMode, kFmt, 256>(a_rows, w0, w1, s0, s1, z0, z1, g0, g1, s, gt, status, out, st, num_sms)
               : launch_fmt<kMode, kFmt, 128>(a_rows, w0, w1, s0, s1, z0, z1, g0, g1, s, gt, status, out, st,
                                              num_sms);
}

}  // namespace

cudaError_t launch_w4_up_gate(const void* a_rows, const void* w_gate, const void* w_up, const void* s_gate,
                              const void* s_up, const void* z_gate, const void* z_up, const Shape& s,
                              const GroupTable& gt, int* status, void* h_rows, cudaStream_t st, int num_sms) {
    return launch_any<0, 0>(a_rows, w_gate, w_up, s_gate, s_up, z_gate, z_up, nullptr, nullptr, s, gt, status, h_rows,
                            st, num_sms);
}

cudaError_t launch_w4_down(const void* h_rows, const void* w_down, const void* s_down, const void* z_down,
                           const Shape& s, const GroupTable& gt, int* status, float* y_rows, cudaStream_t st,
                           int num_sms) {
    return launch_any<1, 0>(h_rows, w_down, nullptr, s_down, nullptr, z_down, nullptr, nullptr, nullptr, s, gt,
                            status, y_rows, st, num_sms);
}

cudaError_t launch_fp4_up_gate(const void* a_rows, const void* w_gate, const void* w_up, const void* s_gate,
                               const void* s_up, const float* g_gate, const float* g_up, const Shape& s,
                               const GroupTable& gt, int* status, void* h_rows, cudaStream_t st, int num_sms) {
    return launch_any<0, 1>(a_rows, w_gate, w_up, s_gate, s_up, nullptr, nullptr, g_gate, g_up, s, gt, status,
                            h_rows, st, num_sms);
}

cudaError_t launch_fp4_down(const void* h_rows, const void* w_down, const void* s_down, const float* g_down,
                            const Shape& s, const GroupTable& gt, int* status, float* y_rows, cudaStream_t st,
                            int num_sms) {
    return launch_any<1, 1>(h_rows, w_down, nullptr, s_down, nullptr, nullptr, nullptr, g_down, nullptr, s, gt,
                            status, y_rows, st, num_sms);
}

}  // namespace moe
