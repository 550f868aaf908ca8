// Stage 4, FP8 block-scaled form: e4m3 operands with f32 scales per 1x128
// activation block and per 128x128 weight block (amax / 448), f32 accumulate.
//
//   U[r, n] = sum_kb  s_a[r, kb] * s_w[kb, n/128] * sum_{k in kb} qa[r, k] qw[k, n]
//
// The scales are arbitrary f32 (not powers of two), so the tensor core's MX
// block scaling cannot apply them.  Each 128-wide K block is instead MMA'd
// into its own TMEM partial (double-buffered, 2 x 256 columns) and promoted by
// the epilogue warps into register accumulators with one packed f32x2 FMA per
// two columns: acc += P_kb * (s_a * s_w).
//
// Warp roles (640 threads = 5 warpgroups, one persistent CTA per SM):
//   warp 0      TMA producer: A 128 rows x 128 B (one K block, K-major, 128B
//               swizzle) + B 128 K-rows x 256 columns from the row-major
//               [K, N] e4m3 weights (MN-major, 128B swizzle); 3-stage ring.
//   warp 1      MMA issuer: per K block 4 x tcgen05.mma kind::f8f6f4 M128
//               N256 K32 into TMEM partial P[kb & 1].
//   warps 2-3   idle (they complete warpgroup 0, which hands its registers
//               to the promotion warpgroups through setmaxnreg).
//   warps 4-19  promotion + epilogue, four per SM sub-partition so that one
//               warp's TMEM-load latency hides behind the others' FMAs: warp
//               w reads TMEM lanes 32*(w%4).. and quarter (w-4)/4 of the
//               columns, one 32-column TMEM load in flight per wait (112
//               registers per thread: 64 accumulators plus 32 loaded values):
//                 up/gate: gate cols [32qt, 32qt+32) and up cols 128+[32qt, ..)
//                 of the same 32 output features, so SwiGLU is local; the
//                 row block of 128 features (the tile) gets its 1x128 scale
//                 from the four quarters' amax (exchanged through shared
//                 memory) and is written as e4m3(h * (1/s)) plus its f32
//                 scale s (SiLU as g * fast-reciprocal(1 + e^-g));
//                 down: cols [64qt, 64qt+64), written as f32 rows of Y.
// Quantisation (host weights, device activations and h) rounds x / s to the
// nearest e4m3, saturating at +-448.
//
// The same kernel, kKind = 1, runs the INT8_CHANNEL format (s8 x s8 -> s32,
// tcgen05.mma kind::i8): per-output-channel weight scales s_w[n] and per-row
// activation scales (x: one per row; h: one per row and 128-feature block, the
// up/gate tile), both amax / 127.
//   up/gate: the row and column scales are constant along K, so all K blocks
//            accumulate into one s32 TMEM tile and the epilogue reads it once:
//            g = (float)G_s32 * (s_x[r] * s_g[n]); h = silu(g) * u is
//            requantised per 128-feature block, q = clamp(rn(h / s_h), +-127).
//   down:    s_h varies along K, so each K block is promoted as in the FP8 form
//            (acc += (float)P_kb * s_h[r, kb]) and the epilogue multiplies the
//            sum by s_d[n].
#include "moe_internal.h"
#include "common.cuh"
#include "sm100.cuh"

#include <cuda.h>
#include <cuda_fp8.h>
#include <cudaTypedefs.h>

namespace moe {

bool make_map_u8(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer, uint32_t box_outer);

namespace {

using namespace sm100;

constexpr int kBM = 128;
constexpr int kStages = 3;
// 20 warps = 5 warpgroups: warpgroup 0 (TMA, MMA, two idle warps) gives up
// registers with setmaxnreg, the four promotion warpgroups take them.  The
// launch holds 96 registers per thread (65536 / 640 rounded down to the
// allocation unit of 8); the split must not exceed that total, or the
// setmaxnreg.inc would wait forever -- the host checks the compiled count
// before the first launch.
constexpr int kThreads = 640;
constexpr int kPromoWarps = 16;
constexpr int kPromoWarp0 = 4;
constexpr int kRegsLaunch = 96;
constexpr int kRegsCtrl = 32, kRegsPromo = 112;
static_assert(kRegsCtrl * 128 + kRegsPromo * 128 * (kPromoWarps / 4) <= kRegsLaunch * kThreads,
              "register split must fit the launch total");
constexpr int kABytes = kBM * 128;
constexpr int kBBytes = 128 * 256;
constexpr int kStageBytes = kABytes + kBBytes;
constexpr int kChunkBytes = 128 * 128;   // 128 K-rows x 128 columns (one swizzle span)
constexpr int kTmemCols = 512;
constexpr size_t kStageOutBytes = kPromoWarps * 2048;   // per-warp 32x16 f32 staging for coalesced Y stores
constexpr size_t kSmemBytes = 1024 + (size_t)kStages * kStageBytes + 256 + kStageOutBytes;

struct Fp8Params {
    const int* g_rows;
    const int* g_start;
    const int* g_weight;
    int G;
    int K;               // reduction length
    int n_tiles;         // output tiles per group
    int out_ld;          // output row length (f or d)
    void* out;           // e4m3 h rows (up/gate) or f32 y rows (down)
    float* out_scale;    // up/gate: [rows, f/128] h block scales
    const float* a_scale;    // [rows, K/128] activation block scales
    const float* w_scale0;   // up/gate: gate [Ew, K/128, f/128]; down: [Ew, f/128, d/128]
    const float* w_scale1;   // up/gate: up scales
    int* status;
    uint32_t idesc;
    OutRedirect red;         // down: optional peer destination of each group's rows
};

// m-tiles of a group come from its row count (no per-group table: shared
// memory is at its limit in this kernel)
__device__ __forceinline__ void decode_tile(int t, const int* pre, const int* rows, int G, int& g, int& m, int& n) {
    int lo = 0, hi = G - 1;
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (pre[mid] <= t) lo = mid; else hi = mid - 1;
    }
    g = lo;
    const int local = t - pre[g];
    const int mt = (rows[g] + kBM - 1) / kBM;
    n = local / mt;
    m = local - n * mt;
}

__device__ __forceinline__ uint32_t e4m3x4(float a, float b, float c, float d) {
    const uint32_t lo = __nv_cvt_float2_to_fp8x2(make_float2(a, b), __NV_SATFINITE, __NV_E4M3);
    const uint32_t hi = __nv_cvt_float2_to_fp8x2(make_float2(c, d), __NV_SATFINITE, __NV_E4M3);
    return lo | (hi << 16);
}

__device__ __forceinline__ uint32_t s8x4(float a, float b, float c, float d) {
    auto q = [](float v) { return (uint32_t)(max(-127, min(127, __float2int_rn(v))) & 0xff); };
    return q(a) | (q(b) << 8) | (q(c) << 16) | (q(d) << 24);
}

// kMode 0: up/gate + SwiGLU -> 8-bit h + scales;  1: down -> f32 y.
// kKind 0: e4m3 with block scales;  1: int8 with channel scales.
template <int kMode, int kKind>
__global__ void __launch_bounds__(kThreads, 1)
    fp8_gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB0,
                    const __grid_constant__ CUtensorMap tmB1, const Fp8Params p) {
    extern __shared__ uint8_t smem_raw[];
    __shared__ int s_pre[kMaxGroups + 1];
    __shared__ int s_rows[kMaxGroups];
    __shared__ int s_start[kMaxGroups];
    __shared__ int s_wt[kMaxGroups];
    __shared__ float s_amax[4][kBM];

    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sA = smem;
    uint8_t* sB = smem + kStages * kABytes;
    uint64_t* full = reinterpret_cast<uint64_t*>(sB + kStages * kBBytes);
    uint64_t* empty = full + kStages;
    uint64_t* pfull = empty + kStages;
    uint64_t* pempty = pfull + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(pempty + 2);
    float4* sStage = reinterpret_cast<float4*>(sB + kStages * kBBytes + 256);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) { mbar_init(&full[s], 1); mbar_init(&empty[s], 1); }
        for (int a = 0; a < 2; ++a) { mbar_init(&pfull[a], 1); mbar_init(&pempty[a], kPromoWarps * 32); }
        fence_mbar_init();
        tma_prefetch_desc(&tmA);
        tma_prefetch_desc(&tmB0);
        if (kMode == 0) tma_prefetch_desc(&tmB1);
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, kTmemCols);
        tmem_relinquish();
    }
    for (int g = threadIdx.x; g < p.G; g += kThreads) {
        const int r = p.g_rows[g];
        s_rows[g] = r;
        s_start[g] = p.g_start[g];
        s_wt[g] = p.g_weight ? p.g_weight[g] : g;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        int acc = 0;
        for (int g = 0; g < p.G; ++g) { s_pre[g] = acc; acc += (s_rows[g] + kBM - 1) / kBM * p.n_tiles; }
        s_pre[p.G] = acc;
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    const int total = s_pre[p.G];
    const int kblocks = p.K / 128;
    // warp-uniform warpgroup index (the shuffle makes the uniformity explicit)
    const int wgroup = __shfl_sync(0xffffffffu, (int)(threadIdx.x >> 7), 0);

    if (wgroup == 0) {
        asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kRegsCtrl));
        if (warp == 0) {
            if (lane == 0) {
                int s = 0;
                uint32_t ph = 0;
                for (int t = blockIdx.x; t < total; t += gridDim.x) {
                    int g, m, n;
                    decode_tile(t, s_pre, s_rows, p.G, g, m, n);
                    const int a_row = s_start[g] + m * kBM;
                    const int b_row = s_wt[g] * p.K;
                    for (int kb = 0; kb < kblocks; ++kb) {
                        if (!mbar_wait(&empty[s], ph ^ 1u, p.status, kDevErrTimeout)) goto producer_done;
                        mbar_arrive_expect_tx(&full[s], kStageBytes);
                        uint8_t* a_dst = sA + s * kABytes;
                        uint8_t* b_dst = sB + s * kBBytes;
                        tma_load_2d(a_dst, &tmA, &full[s], kb * 128, a_row);
                        if (kMode == 0) {
                            tma_load_2d(b_dst, &tmB0, &full[s], n * 128, b_row + kb * 128);
                            tma_load_2d(b_dst + kChunkBytes, &tmB1, &full[s], n * 128, b_row + kb * 128);
                        } else {
                            tma_load_2d(b_dst, &tmB0, &full[s], n * 256, b_row + kb * 128);
                            tma_load_2d(b_dst + kChunkBytes, &tmB0, &full[s], n * 256 + 128, b_row + kb * 128);
                        }
                        if (++s == kStages) { s = 0; ph ^= 1u; }
                    }
                }
            producer_done:;
            }
        } else if (warp == 1) {
            if (lane == 0) {
                int s = 0, pb = 0;
                uint32_t ph = 0, pph = 0;
                bool ok = true;
                // kWhole: one TMEM accumulator over all K blocks (int8 up/gate)
                constexpr bool kWhole = kKind == 1 && kMode == 0;
                for (int t = blockIdx.x; t < total && ok; t += gridDim.x) {
                    for (int kb = 0; kb < kblocks; ++kb) {
                        if (((!kWhole || kb == 0) && !mbar_wait(&pempty[pb], pph ^ 1u, p.status, kDevErrTimeout)) ||
                            !mbar_wait(&full[s], ph, p.status, kDevErrTimeout)) {
                            ok = false;
                            break;
                        }
                        tc_fence_after();
                        const uint32_t a_base = smem_u32(sA + s * kABytes);
                        const uint32_t b_base = smem_u32(sB + s * kBBytes);
                        const uint32_t d_tmem = tmem_base + pb * 256;
#pragma unroll
                        for (int kk = 0; kk < 4; ++kk) {
                            const uint64_t adesc = smem_desc_sw128(a_base + kk * 32, 16, 1024);
                            const uint64_t bdesc = smem_desc_sw128(b_base + kk * 32 * 128, kChunkBytes, 1024);
                            const uint32_t accum = (kk != 0 || (kWhole && kb != 0)) ? 1u : 0u;
                            if (kKind == 0) mma_f8_ss(d_tmem, adesc, bdesc, p.idesc, accum);
                            else mma_i8_ss(d_tmem, adesc, bdesc, p.idesc, accum);
                        }
                        mma_commit(&empty[s]);
                        if (++s == kStages) { s = 0; ph ^= 1u; }
                        if (!kWhole || kb == kblocks - 1) {
                            mma_commit(&pfull[pb]);
                            pb ^= 1;
                            if (pb == 0) pph ^= 1u;
                        }
                    }
                }
            }
        }   // warps 2, 3: idle
    } else {
        asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kRegsPromo));
        // ---------------- promotion + epilogue (warps 4..19) ----------------
        const int q = warp & 3;
        const int qt = (warp - kPromoWarp0) >> 2;   // column quarter
        const int row_in_tile = q * 32 + lane;
        const int nkb = kblocks;
        const int nblk = p.out_ld / 128;
        // TMEM column of round rnd (32 columns each): up/gate reads 32 gate
        // then the same 32 features' up columns; down reads 64 adjacent columns
        auto rcol = [&](int rnd) { return kMode == 0 ? 128 * rnd + 32 * qt : 64 * qt + 32 * rnd; };
        int pb = 0;
        uint32_t pph = 0;
        for (int t = blockIdx.x; t < total; t += gridDim.x) {
            int g, m, n;
            decode_tile(t, s_pre, s_rows, p.G, g, m, n);
            const int row_local = m * kBM + row_in_tile;
            const bool valid = row_local < s_rows[g];
            const int64_t row = (int64_t)s_start[g] + row_local;
            // rows past the group's end read the group's first row's (finite) scales; never stored
            const float* arow = p.a_scale + (valid ? row : (int64_t)s_start[g]) * nkb;
            const int wexp = s_wt[g];
            float acc[64];
#pragma unroll
            for (int i = 0; i < 64; ++i) acc[i] = 0.0f;
            bool ok = true;
            // scales of K block kb+1 are loaded while block kb is promoted
            auto wscale = [&](const float* base, int kb, int col) {
                return base[((int64_t)wexp * nkb + kb) * nblk + col];
            };
            const int wcol = kMode == 0 ? n : 2 * n + (qt >> 1);
            if (kKind == 1 && kMode == 0) {
                // int8 up/gate: one s32 accumulator, scaled by s_x[r] * s_w[n]
                const float sx = p.a_scale[valid ? row : (int64_t)s_start[g]];
                const float* sg = p.w_scale0 + (int64_t)wexp * p.out_ld + n * 128 + 32 * qt;
                const float* su = p.w_scale1 + (int64_t)wexp * p.out_ld + n * 128 + 32 * qt;
                if (!mbar_wait_warp(&pfull[pb], pph, p.status, kDevErrTimeout)) break;
                tc_fence_after();
                const uint32_t tbase = tmem_base + ((uint32_t)(q * 32) << 16) + pb * 256;
#pragma unroll
                for (int rnd = 0; rnd < 2; ++rnd) {
                    uint32_t r[32];
                    tmem_ld_32x32b_x32(tbase + rcol(rnd), r);
                    tmem_wait_ld();
                    if (rnd == 1) { tc_fence_before(); mbar_arrive(&pempty[pb]); }
                    const float4* ws4 = reinterpret_cast<const float4*>(rnd == 0 ? sg : su);
#pragma unroll
                    for (int v = 0; v < 8; ++v) {
                        const float4 w4 = __ldg(ws4 + v);
                        acc[32 * rnd + 4 * v + 0] = (float)(int)r[4 * v + 0] * (sx * w4.x);
                        acc[32 * rnd + 4 * v + 1] = (float)(int)r[4 * v + 1] * (sx * w4.y);
                        acc[32 * rnd + 4 * v + 2] = (float)(int)r[4 * v + 2] * (sx * w4.z);
                        acc[32 * rnd + 4 * v + 3] = (float)(int)r[4 * v + 3] * (sx * w4.w);
                    }
                }
                pb ^= 1;
                if (pb == 0) pph ^= 1u;
            } else {
                float sa_n = arow[0];
                float sw0_n = kKind == 0 ? wscale(p.w_scale0, 0, wcol) : 1.0f;
                float sw1_n = (kKind == 0 && kMode == 0) ? wscale(p.w_scale1, 0, wcol) : sw0_n;
                for (int kb = 0; kb < nkb; ++kb) {
                    const float sa = sa_n, sw0 = sw0_n, sw1 = sw1_n;
                    if (kb + 1 < nkb) {
                        sa_n = arow[kb + 1];
                        if (kKind == 0) {
                            sw0_n = wscale(p.w_scale0, kb + 1, wcol);
                            sw1_n = kMode == 0 ? wscale(p.w_scale1, kb + 1, wcol) : sw0_n;
                        }
                    }
                    if (!mbar_wait_warp(&pfull[pb], pph, p.status, kDevErrTimeout)) { ok = false; break; }
                    tc_fence_after();
                    const uint32_t tbase = tmem_base + ((uint32_t)(q * 32) << 16) + pb * 256;
                    const float sc0 = sa * sw0, sc1 = sa * sw1;
#pragma unroll
                    for (int rnd = 0; rnd < 2; ++rnd) {
                        uint32_t r[32];
                        tmem_ld_32x32b_x32(tbase + rcol(rnd), r);
                        tmem_wait_ld();
                        if (rnd == 1) { tc_fence_before(); mbar_arrive(&pempty[pb]); }
                        const float sc = (kMode == 0 && rnd == 1) ? sc1 : sc0;
#pragma unroll
                        for (int i = 0; i < 32; i += 2) {
                            const float p0 = kKind == 0 ? __uint_as_float(r[i]) : (float)(int)r[i];
                            const float p1 = kKind == 0 ? __uint_as_float(r[i + 1]) : (float)(int)r[i + 1];
                            ffma2(acc[32 * rnd + i], acc[32 * rnd + i + 1], p0, p1, sc);
                        }
                    }
                    pb ^= 1;
                    if (pb == 0) pph ^= 1u;
                }
                if (!ok) break;
            }
            if (kMode == 0) {
                float amax = 0.0f;
#pragma unroll
                for (int i = 0; i < 32; ++i) {
                    const float gv = acc[i], uv = acc[32 + i];
                    const float h = uv * __fdividef(gv, 1.0f + __expf(-gv));
                    acc[i] = h;
                    amax = fmaxf(amax, fabsf(h));
                }
                // the 1x128 block of h = the four quarters of this row
                asm volatile("bar.sync %0, 128;" ::"r"(1 + q) : "memory");
                s_amax[qt][row_in_tile] = amax;
                asm volatile("bar.sync %0, 128;" ::"r"(1 + q) : "memory");
                const float bmax = fmaxf(fmaxf(s_amax[0][row_in_tile], s_amax[1][row_in_tile]),
                                         fmaxf(s_amax[2][row_in_tile], s_amax[3][row_in_tile]));
                const float sh = bmax > 0.0f ? bmax / (kKind == 0 ? 448.0f : 127.0f) : 1.0f;
                const float inv = 1.0f / sh;   // q = rn(h * (1/s)): one division per row, not per element
                if (valid) {
                    uint8_t* h8 = reinterpret_cast<uint8_t*>(p.out) + row * p.out_ld + n * 128 + 32 * qt;
                    uint4* o = reinterpret_cast<uint4*>(h8);
#pragma unroll
                    for (int v = 0; v < 2; ++v) {
                        uint32_t w4[4];
#pragma unroll
                        for (int j = 0; j < 4; ++j) {
                            const int i = 16 * v + 4 * j;
                            w4[j] = kKind == 0 ? e4m3x4(acc[i] * inv, acc[i + 1] * inv, acc[i + 2] * inv, acc[i + 3] * inv)
                                               : s8x4(acc[i] * inv, acc[i + 1] * inv, acc[i + 2] * inv, acc[i + 3] * inv);
                        }
                        o[v] = make_uint4(w4[0], w4[1], w4[2], w4[3]);
                    }
                    if (qt == 0) p.out_scale[row * nblk + n] = sh;
                }
            } else {
                if (kKind == 1) {
                    const float4* wd = reinterpret_cast<const float4*>(p.w_scale0 + (int64_t)wexp * p.out_ld +
                                                                       n * 256 + 64 * qt);
#pragma unroll
                    for (int v = 0; v < 16; ++v) {
                        const float4 w4 = __ldg(wd + v);
                        acc[4 * v] *= w4.x;
                        acc[4 * v + 1] *= w4.y;
                        acc[4 * v + 2] *= w4.z;
                        acc[4 * v + 3] *= w4.w;
                    }
                }
                // this warp's 32 rows x 64 columns, coalesced through shared memory
                const int warp_row0 = m * kBM + q * 32;
                const int nrows = s_rows[g] - warp_row0;
                float* y = down_rows(p.red, reinterpret_cast<float*>(p.out), g, s_start[g], p.out_ld) +
                           (int64_t)warp_row0 * p.out_ld + n * 256 + 64 * qt;
                float4* stage = sStage + (warp - kPromoWarp0) * 128;
#pragma unroll
                for (int c = 0; c < 4; ++c) warp_store_rows16(stage, acc + 16 * c, y + 16 * c, p.out_ld, nrows, lane);
            }
        }
        if (kMode == 1 && p.red.rank) __threadfence_system();   // peer rows visible before the kernel ends
    }
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, kTmemCols);
    }
}

template <int kMode, int kKind>
cudaError_t launch(const CUtensorMap& a, const CUtensorMap& b0, const CUtensorMap& b1, const Fp8Params& p,
                   cudaStream_t st, int num_sms) {
    auto kern = fp8_gemm_kernel<kMode, kKind>;
    static SmemAttr attr;
    cudaError_t err = ensure_smem(kern, kSmemBytes, attr);
    if (err != cudaSuccess) return err;
    // the setmaxnreg split draws on the registers the launch holds; a build
    // that compiled to fewer would make the promotion warps wait forever
    static int regs = -1;
    if (regs < 0) {
        cudaFuncAttributes fa{};
        err = cudaFuncGetAttributes(&fa, kern);
        if (err != cudaSuccess) return err;
        regs = fa.numRegs;
    }
    if (regs < kRegsLaunch) return cudaErrorInvalidConfiguration;
    kern<<<num_sms, kThreads, kSmemBytes, st>>>(a, b0, b1, p);
    return cudaGetLastError();
}

}  // namespace

cudaError_t launch_fp8_up_gate(const void* a_rows, const float* a_scale, const void* w_gate, const void* w_up,
                               const float* s_gate, const float* s_up, const Shape& s, const GroupTable& gt,
                               int* status, void* h_rows, float* h_scale, cudaStream_t st, int num_sms) {
    if (gt.G <= 0 || gt.rows_capacity <= 0) return cudaSuccess;
    CUtensorMap ta, tg, tu;
    if (!make_map_u8(&ta, a_rows, s.d, gt.rows_capacity, kBM) ||
        !make_map_u8(&tg, w_gate, s.f, (uint64_t)s.E * s.d, 128) ||
        !make_map_u8(&tu, w_up, s.f, (uint64_t)s.E * s.d, 128))
        return cudaErrorInvalidValue;
    Fp8Params p{};
    p.g_rows = gt.rows;
    p.g_start = gt.start;
    p.g_weight = gt.weight;
    p.G = gt.G;
    p.K = s.d;
    p.n_tiles = s.f / 128;
    p.out_ld = s.f;
    p.out = h_rows;
    p.out_scale = h_scale;
    p.a_scale = a_scale;
    p.w_scale0 = s_gate;
    p.w_scale1 = s_up;
    p.status = status;
    p.idesc = idesc_e4m3(kBM, 256, true);
    return launch<0, 0>(ta, tg, tu, p, st, num_sms);
}

cudaError_t launch_fp8_down(const void* h_rows, const float* h_scale, const void* w_down, const float* s_down,
                            const Shape& s, const GroupTable& gt, int* status, float* y_rows, cudaStream_t st,
                            int num_sms) {
    if (gt.G <= 0 || gt.rows_capacity <= 0) return cudaSuccess;
    CUtensorMap th, td;
    if (!make_map_u8(&th, h_rows, s.f, gt.rows_capacity, kBM) ||
        !make_map_u8(&td, w_down, s.d, (uint64_t)s.E * s.f, 128))
        return cudaErrorInvalidValue;
    Fp8Params p{};
    p.g_rows = gt.rows;
    p.g_start = gt.start;
    p.g_weight = gt.weight;
    p.G = gt.G;
    p.K = s.f;
    p.n_tiles = s.d / 256;
    p.out_ld = s.d;
    p.out = y_rows;
    p.a_scale = h_scale;
    p.w_scale0 = s_down;
    p.status = status;
    p.idesc = idesc_e4m3(kBM, 256, true);
    p.red = gt.redirect;
    return launch<1, 0>(th, td, td, p, st, num_sms);
}

cudaError_t launch_i8c_up_gate(const void* a_rows, const float* a_scale, const void* w_gate, const void* w_up,
                               const float* s_gate, const float* s_up, const Shape& s, const GroupTable& gt,
                               int* status, void* h_rows, float* h_scale, cudaStream_t st, int num_sms) {
    if (gt.G <= 0 || gt.rows_capacity <= 0) return cudaSuccess;
    CUtensorMap ta, tg, tu;
    if (!make_map_u8(&ta, a_rows, s.d, gt.rows_capacity, kBM) ||
        !make_map_u8(&tg, w_gate, s.f, (uint64_t)s.E * s.d, 128) ||
        !make_map_u8(&tu, w_up, s.f, (uint64_t)s.E * s.d, 128))
        return cudaErrorInvalidValue;
    Fp8Params p{};
    p.g_rows = gt.rows;
    p.g_start = gt.start;
    p.g_weight = gt.weight;
    p.G = gt.G;
    p.K = s.d;
    p.n_tiles = s.f / 128;
    p.out_ld = s.f;
    p.out = h_rows;
    p.out_scale = h_scale;
    p.a_scale = a_scale;
    p.w_scale0 = s_gate;
    p.w_scale1 = s_up;
    p.status = status;
    p.idesc = idesc_i8(kBM, 256, true);
    return launch<0, 1>(ta, tg, tu, p, st, num_sms);
}

cudaError_t launch_i8c_down(const void* h_rows, const float* h_scale, const void* w_down, const float* s_down,
                            const Shape& s, const GroupTable& gt, int* status, float* y_rows, cudaStream_t st,
                            int num_sms) {
    if (gt.G <= 0 || gt.rows_capacity <= 0) return cudaSuccess;
    CUtensorMap th, td;
    if (!make_map_u8(&th, h_rows, s.f, gt.rows_capacity, kBM) ||
        !make_map_u8(&td, w_down, s.d, (uint64_t)s.E * s.f, 128))
        return cudaErrorInvalidValue;
    Fp8Params p{};
    p.g_rows = gt.rows;
    p.g_start = gt.start;
    p.g_weight = gt.weight;
    p.G = gt.G;
    p.K = s.f;
    p.n_tiles = s.d / 256;
    p.out_ld = s.d;
    p.out = y_rows;
    p.a_scale = h_scale;
    p.w_scale0 = s_down;
    p.status = status;
    p.idesc = idesc_i8(kBM, 256, true);
    p.red = gt.redirect;
    return launch<1, 1>(th, td, td, p, st, num_sms);
}

}  // namespace moe
