// Stage 4: the expert SwiGLU FFN as two grouped GEMMs on tcgen05 tensor cores.
//
// Reference semantics:
//   16-bit  kernels/capacity.cu:505-511 -- U = A_e Wup_e, G = A_e Wgate_e in
//           f32, h = U * G / (1 + exp(-G)) rounded to the 16-bit type
//           (capacity.cu:144-168), then Y = h_e Wdown_e in f32.
//   int8    kernels/capacity_int8_ptx.cu:445-476 and :578-619 -- s32 GEMMs on
//           per-tensor quantised operands; U*s_in*s_up, G*s_in*s_gate, SiLU*mul,
//           requantised h = rn(clamp(x / s_mid, -128, 127)); the down GEMM's
//           s32 result is dequantised by s_mid*s_down.
//
// Design (one persistent CTA per SM, warp-specialised, 192 threads):
//   warp 0      TMA producer: A tile 128 rows x 128 bytes of K (K-major, 128B
//               swizzle) and the B tile of 128 bytes of K rows x 256 columns
//               straight from the reference's row-major [K, N] weights
//               (N-contiguous = MN-major, 128B swizzle), into a 4-stage smem
//               ring guarded by full/empty mbarriers.
//   warp 1      MMA issuer: one thread issues tcgen05.mma M=128 N=256 (4 per
//               K block) into a double-buffered TMEM accumulator (2 x 256
//               columns), commits to the ring's empty barrier and, per tile,
//               to the accumulator-full barrier.
//   warps 2-5   epilogue: tcgen05.ld rows out of TMEM, releases the buffer,
//               then
//                 up/gate mode: columns [0,128) = gate, [128,256) = up of the
//                 same 128 output features (the B tile holds Wgate | Wup), so
//                 SwiGLU (and the int8 requantisation) happens in registers
//                 and only h is written;
//                 down mode: writes the f32 rows of Y (int8: dequantised).
// The operand format is a trait (Fmt16 / FmtI8): both keep 128-byte swizzle
// rows, so only the K block (64 vs 128 elements), the B chunk width (64 vs
// 128 columns), the MMA kind and the epilogue arithmetic differ.
// Tiles: a row group (an expert's kept rows on one GPU; a (sender, expert)
// block under expert parallelism) owns ceil(rows / 128) M-tiles, with the row
// counts read on the device -- empty capacity slots cost no MMA work.  Tile
// order is group-major, then N-tile, then M-tile, so the CTAs in flight share
// one expert's weights and activations in L2.
#include "moe_internal.h"
#include "common.cuh"
#include "sm100.cuh"

#include <cudaTypedefs.h>
#include <cuda.h>
#include <mutex>

namespace moe {
namespace {

using namespace sm100;

constexpr int kBM = 128;
constexpr int kUmmaN = 256;
constexpr int kStages = 4;
constexpr int kThreads = 192;
constexpr int kABytes = kBM * 128;                  // 16 KB: 128 rows x 128 bytes of K
constexpr int kBBytes = 128 * kUmmaN;               // 32 KB: 128 bytes of K rows x 256 columns
constexpr int kStageBytes = kABytes + kBBytes;
constexpr int kAccCols = kUmmaN;
constexpr int kTmemCols = 2 * kAccCols;
constexpr size_t kSmemBytes = 1024 + (size_t)kStages * kStageBytes + 256 + 4 * 2048;

struct GemmParams {
    const int* g_rows;       // [G] rows of each group
    const int* g_start;      // [G] first row of each group in A and in the output
    const int* g_weight;     // [G] expert weight index of each group (null: g)
    int G;
    int K;                   // reduction length (d for up/gate, f for down)
    int n_tiles;             // output tiles along N per expert
    int out_ld;              // output row length in elements (f or d)
    void* out;               // h rows (up/gate) or f32 y rows (down)
    int* status;
    uint32_t idesc;
    // int8 per-tensor scales (capacity_int8_ptx.cu:455-457, 596)
    float deq_gate, deq_up;  // s_in*s_gate, s_in*s_up
    float inv_mid;           // 1 / s_mid
    float deq_down;          // s_mid*s_down
    OutRedirect red;         // down: optional peer destination of each group's rows
};

// ---- operand formats -----------------------------------------------------------
template <typename T16>
struct Fmt16 {
    static constexpr int kElemBytes = 2;
    static constexpr int kBK = 64;           // K elements per stage (128 bytes)
    static constexpr int kChunkN = 64;       // B columns per 128-byte swizzle span
    static constexpr int kUmmaK = 16;
    static __device__ __forceinline__ void mma(uint32_t d, uint64_t a, uint64_t b, uint32_t id, uint32_t acc) {
        mma_f16_ss(d, a, b, id, acc);
    }
    // 32 columns of gate/up accumulators -> 32 h values (16-bit) at dst.
    static __device__ __forceinline__ void swiglu_store(const uint32_t (&g)[32], const uint32_t (&u)[32],
                                                        const GemmParams&, void* dst, bool valid) {
        uint32_t packed[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
            float hv[2];
#pragma unroll
            for (int j = 0; j < 2; ++j) {
                const float gv = __uint_as_float(g[2 * i + j]);
                const float uv = __uint_as_float(u[2 * i + j]);
                hv[j] = uv * (gv / (1.0f + __expf(-gv)));
            }
            packed[i] = F16Traits<T16>::pack2(hv[0], hv[1]);
        }
        if (valid) {
            uint4* o = reinterpret_cast<uint4*>(dst);
#pragma unroll
            for (int v = 0; v < 4; ++v)
                o[v] = make_uint4(packed[4 * v], packed[4 * v + 1], packed[4 * v + 2], packed[4 * v + 3]);
        }
    }
    static __device__ __forceinline__ float down_value(uint32_t r, const GemmParams&) { return __uint_as_float(r); }
};

// Per-tensor int8 (capacity_int8_ptx.cu): clamp [-128, 127].
template <int kQMax>
struct FmtI8T {
    static constexpr int kElemBytes = 1;
    static constexpr int kBK = 128;
    static constexpr int kChunkN = 128;
    static constexpr int kUmmaK = 32;
    static __device__ __forceinline__ void mma(uint32_t d, uint64_t a, uint64_t b, uint32_t id, uint32_t acc) {
        mma_i8_ss(d, a, b, id, acc);
    }
    // capacity_int8_ptx.cu:465-474: dequant, SiLU(gate)*up, requant.
    static __device__ __forceinline__ void swiglu_store(const uint32_t (&g)[32], const uint32_t (&u)[32],
                                                        const GemmParams& p, void* dst, bool valid) {
        uint32_t packed[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            uint32_t word = 0;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const float uf = (float)(int)u[4 * i + j] * p.deq_up;
                const float gf = (float)(int)g[4 * i + j] * p.deq_gate;
                const float silu = gf / (1.0f + __expf(-gf));
                const float fused = uf * silu;
                constexpr float lo = kQMax == 127 ? -128.f : -(float)kQMax;
                const int q = __float2int_rn(fminf(fmaxf(fused * p.inv_mid, lo), (float)kQMax));
                word |= (uint32_t)(q & 0xFF) << (8 * j);
            }
            packed[i] = word;
        }
        if (valid) {
            uint4* o = reinterpret_cast<uint4*>(dst);
            o[0] = make_uint4(packed[0], packed[1], packed[2], packed[3]);
            o[1] = make_uint4(packed[4], packed[5], packed[6], packed[7]);
        }
    }
    // capacity_int8_ptx.cu:615: (float)int32 * (s_mid * s_down)
    static __device__ __forceinline__ float down_value(uint32_t r, const GemmParams& p) {
        return (float)(int)r * p.deq_down;
    }
};
using FmtI8 = FmtI8T<127>;

// The reference's per-tensor fp8 format (capacity_fp8_ptx.cu:362-395, :566-600):
// e4m3 x e4m3 with f32 accumulation (kind::f8f6f4); up*s_in*s_up and
// gate*s_in*s_gate, SiLU*mul, h = e4m3(clamp(fused / s_mid, -448, 448));
// the down result is dequantised by s_mid*s_down.
struct FmtE4 {
    static constexpr int kElemBytes = 1;
    static constexpr int kBK = 128;
    static constexpr int kChunkN = 128;
    static constexpr int kUmmaK = 32;
    static __device__ __forceinline__ void mma(uint32_t d, uint64_t a, uint64_t b, uint32_t id, uint32_t acc) {
        mma_f8_ss(d, a, b, id, acc);
    }
    static __device__ __forceinline__ void swiglu_store(const uint32_t (&g)[32], const uint32_t (&u)[32],
                                                        const GemmParams& p, void* dst, bool valid) {
        uint32_t packed[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            float v[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const float uf = __uint_as_float(u[4 * i + j]) * p.deq_up;
                const float gf = __uint_as_float(g[4 * i + j]) * p.deq_gate;
                const float silu = gf / (1.0f + __expf(-gf));
                v[j] = fminf(fmaxf(uf * silu * p.inv_mid, -448.f), 448.f);
            }
            packed[i] = (uint32_t)__nv_cvt_float2_to_fp8x2(make_float2(v[0], v[1]), __NV_SATFINITE, __NV_E4M3) |
                        ((uint32_t)__nv_cvt_float2_to_fp8x2(make_float2(v[2], v[3]), __NV_SATFINITE, __NV_E4M3)
                         << 16);
        }
        if (valid) {
            uint4* o = reinterpret_cast<uint4*>(dst);
            o[0] = make_uint4(packed[0], packed[1], packed[2], packed[3]);
            o[1] = make_uint4(packed[4], packed[5], packed[6], packed[7]);
        }
    }
    static __device__ __forceinline__ float down_value(uint32_t r, const GemmParams& p) {
        return __uint_as_float(r) * p.deq_down;
    }
};

__device__ __forceinline__ void decode_tile(int t, const int* pre, const int* mt, int G, int& e,
                                            int& m, int& n) {
    int lo = 0, hi = G - 1;
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (pre[mid] <= t) lo = mid; else hi = mid - 1;
    }
    e = lo;
    const int local = t - pre[e];
    n = local / mt[e];
    m = local - n * mt[e];
}

template <int kMode, class Fmt>  // kMode 0: up/gate + SwiGLU -> h;  1: down -> f32 y
__global__ void __launch_bounds__(kThreads, 1)
    expert_gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB0,
                       const __grid_constant__ CUtensorMap tmB1, const GemmParams p) {
    constexpr int kBK = Fmt::kBK;
    constexpr int kChunkN = Fmt::kChunkN;
    constexpr int kChunkBytes = kBK * 128;            // K rows x 128 bytes
    constexpr int kChunks = kUmmaN / kChunkN;         // B chunks per stage
    constexpr int kKSteps = kBK / Fmt::kUmmaK;        // MMAs per stage
    constexpr int kOutN = kMode == 0 ? 128 : 256;     // output columns per tile
    extern __shared__ uint8_t smem_raw[];
    __shared__ int s_pre[kMaxGroups + 1];
    __shared__ int s_mt[kMaxGroups];
    __shared__ int s_rows[kMaxGroups];
    __shared__ int s_start[kMaxGroups];
    __shared__ int s_wt[kMaxGroups];

    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sA = smem;
    uint8_t* sB = smem + kStages * kABytes;
    uint64_t* full = reinterpret_cast<uint64_t*>(sB + kStages * kBBytes);
    uint64_t* empty = full + kStages;
    uint64_t* tfull = empty + kStages;
    uint64_t* tempty = tfull + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
    uint8_t* sStage = sB + kStages * kBBytes + 256;   // 4 epilogue warps x 2 KB

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) { mbar_init(&full[s], 1); mbar_init(&empty[s], 1); }
        for (int a = 0; a < 2; ++a) { mbar_init(&tfull[a], 1); mbar_init(&tempty[a], 128); }
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

    if (warp == 0) {
        if (lane == 0) {
            // ---------------- TMA producer ----------------
            int s = 0;
            uint32_t ph = 0;
            for (int t = blockIdx.x; t < total; t += gridDim.x) {
                int e, m, n;
                decode_tile(t, s_pre, s_mt, p.G, e, m, n);
                const int a_row = s_start[e] + m * kBM;
                const int b_row = s_wt[e] * p.K;
                for (int kb = 0; kb < kblocks; ++kb) {
                    if (!mbar_wait(&empty[s], ph ^ 1u, p.status, kDevErrTimeout)) goto producer_done;
                    mbar_arrive_expect_tx(&full[s], kStageBytes);
                    uint8_t* a_dst = sA + s * kABytes;
                    uint8_t* b_dst = sB + s * kBBytes;
                    const int k0 = kb * kBK;
                    tma_load_2d(a_dst, &tmA, &full[s], k0, a_row);
                    if (kMode == 0) {
                        // [Wgate cols n0..n0+127 | Wup cols n0..n0+127]
                        const int n0 = n * 128;
#pragma unroll
                        for (int j = 0; j < kChunks / 2; ++j) {
                            tma_load_2d(b_dst + j * kChunkBytes, &tmB0, &full[s], n0 + j * kChunkN, b_row + k0);
                            tma_load_2d(b_dst + (kChunks / 2 + j) * kChunkBytes, &tmB1, &full[s], n0 + j * kChunkN,
                                        b_row + k0);
                        }
                    } else {
                        const int n0 = n * 256;
#pragma unroll
                        for (int j = 0; j < kChunks; ++j)
                            tma_load_2d(b_dst + j * kChunkBytes, &tmB0, &full[s], n0 + j * kChunkN, b_row + k0);
                    }
                    if (++s == kStages) { s = 0; ph ^= 1u; }
                }
            }
        producer_done:;
        }
    } else if (warp == 1) {
        if (lane == 0) {
            // ---------------- MMA issuer ----------------
            int s = 0;
            uint32_t ph = 0;
            int acc = 0;
            uint32_t aph = 0;
            for (int t = blockIdx.x; t < total; t += gridDim.x) {
                if (!mbar_wait(&tempty[acc], aph ^ 1u, p.status, kDevErrTimeout)) break;
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + acc * kAccCols;
                bool ok = true;
                for (int kb = 0; kb < kblocks; ++kb) {
                    if (!mbar_wait(&full[s], ph, p.status, kDevErrTimeout)) { ok = false; break; }
                    tc_fence_after();
                    const uint32_t a_base = smem_u32(sA + s * kABytes);
                    const uint32_t b_base = smem_u32(sB + s * kBBytes);
#pragma unroll
                    for (int kk = 0; kk < kKSteps; ++kk) {
                        // A: K-major SW128, 8-row groups 1024 B apart; K step = 32 bytes.
                        const uint64_t adesc = smem_desc_sw128(a_base + kk * 32, 16, 1024);
                        // B: MN-major SW128; column chunks kChunkBytes apart (LBO), 8-row K
                        // groups 1024 B apart (SBO); K step = kUmmaK rows of 128 bytes.
                        const uint64_t bdesc =
                            smem_desc_sw128(b_base + kk * Fmt::kUmmaK * 128, kChunkBytes, 1024);
                        Fmt::mma(d_tmem, adesc, bdesc, p.idesc, (kb | kk) != 0 ? 1u : 0u);
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
    } else {
        // ---------------- epilogue (warps 2..5) ----------------
        const int q = warp & 3;                // TMEM lane quarter this warp may access
        const int row_in_tile = q * 32 + lane;
        int acc = 0;
        uint32_t aph = 0;
        for (int t = blockIdx.x; t < total; t += gridDim.x) {
            int e, m, n;
            decode_tile(t, s_pre, s_mt, p.G, e, m, n);
            if (!mbar_wait_warp(&tfull[acc], aph, p.status, kDevErrTimeout)) break;
            tc_fence_after();
            const int row_local = m * kBM + row_in_tile;
            const bool valid = row_local < s_rows[e];
            const int64_t out_row = (int64_t)s_start[e] + row_local;
            const uint32_t taddr = tmem_base + ((uint32_t)(q * 32) << 16) + acc * kAccCols;
            if (kMode == 0) {
                uint8_t* h = reinterpret_cast<uint8_t*>(p.out) +
                             (out_row * p.out_ld + (int64_t)n * kOutN) * Fmt::kElemBytes;
#pragma unroll 1
                for (int c = 0; c < 128; c += 32) {
                    uint32_t g[32], u[32];
                    tmem_ld_32x32b_x32(taddr + c, g);
                    tmem_ld_32x32b_x32(taddr + 128 + c, u);
                    tmem_wait_ld();
                    if (c == 96) { tc_fence_before(); mbar_arrive(&tempty[acc]); }
                    Fmt::swiglu_store(g, u, p, h + c * Fmt::kElemBytes, valid);
                }
            } else {
                // rows of this warp's quarter: [warp_row0, warp_row0 + 32), coalesced through smem
                const int warp_row0 = m * kBM + q * 32;
                const int nrows = s_rows[e] - warp_row0;
                float* y = down_rows(p.red, reinterpret_cast<float*>(p.out), e, s_start[e], p.out_ld) +
                           (int64_t)warp_row0 * p.out_ld + n * kOutN;
                float4* stage = reinterpret_cast<float4*>(sStage) + (warp - 2) * 128;
#pragma unroll 1
                for (int c = 0; c < 256; c += 32) {
                    uint32_t r[32];
                    tmem_ld_32x32b_x32(taddr + c, r);
                    tmem_wait_ld();
                    if (c == 224) { tc_fence_before(); mbar_arrive(&tempty[acc]); }
                    float v[32];
#pragma unroll
                    for (int i = 0; i < 32; ++i) v[i] = Fmt::down_value(r[i], p);
                    warp_store_rows16(stage, v, y + c, p.out_ld, nrows, lane);
                    warp_store_rows16(stage, v + 16, y + c + 16, p.out_ld, nrows, lane);
                }
            }
            acc ^= 1;
            if (acc == 0) aph ^= 1u;
        }
        if (kMode == 1 && p.red.rank) __threadfence_system();   // peer rows visible before the kernel ends
    }
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, kTmemCols);
    }
}

// ---- host side ----------------------------------------------------------------
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, []() {
        cudaDriverEntryPointQueryResult q;
        void* ptr = nullptr;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
    });
    return fn;
}

// 2-D row-major tensor [outer, inner] of `elem_bytes`-byte elements, boxes of
// 128 bytes x box_outer rows with the 128-byte swizzle.
bool make_map(CUtensorMap* map, const void* base, CUtensorMapDataType dt, int elem_bytes, uint64_t inner,
              uint64_t outer, uint32_t box_outer) {
    auto fn = encode_fn();
    if (!fn) { set_error("cuTensorMapEncodeTiled unavailable"); return false; }
    cuuint64_t dims[2] = {inner, outer};
    cuuint64_t strides[1] = {inner * (uint64_t)elem_bytes};
    cuuint32_t box[2] = {(cuuint32_t)(128 / elem_bytes), box_outer};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(map, dt, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                    CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        set_error("cuTensorMapEncodeTiled failed (%d) for [%llu, %llu] box [%u, %u]", (int)r,
                  (unsigned long long)outer, (unsigned long long)inner, box_outer, box[0]);
        return false;
    }
    return true;
}

template <int kMode, class Fmt>
cudaError_t launch_gemm(const CUtensorMap& a, const CUtensorMap& b0, const CUtensorMap& b1,
                        const GemmParams& p, cudaStream_t st, int num_sms) {
    auto kern = expert_gemm_kernel<kMode, Fmt>;
    static SmemAttr attr;
    cudaError_t err = ensure_smem(kern, kSmemBytes, attr);
    if (err != cudaSuccess) return err;
    kern<<<num_sms, kThreads, kSmemBytes, st>>>(a, b0, b1, p);
    return cudaGetLastError();
}

struct FmtDesc {
    CUtensorMapDataType dt;
    int elem_bytes;
    int bk;
    int chunk_n;
};
FmtDesc fmt_desc(int dtype) {
    switch (dtype) {
        case MOE_DTYPE_BF16: return {CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, 64, 64};
        case MOE_DTYPE_INT8:
        case MOE_DTYPE_FP8: return {CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, 128, 128};
        default: return {CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, 64, 64};
    }
}

GemmParams base_params(const GroupTable& gt, int* status, const GemmScales& sc) {
    GemmParams p{};
    p.g_rows = gt.rows;
    p.g_start = gt.start;
    p.g_weight = gt.weight;
    p.G = gt.G;
    p.status = status;
    p.deq_gate = sc.s_in * sc.s_gate;
    p.deq_up = sc.s_in * sc.s_up;
    p.inv_mid = 1.0f / sc.s_mid;
    p.deq_down = sc.s_mid * sc.s_down;
    p.red = gt.redirect;   // used by the down GEMM only
    return p;
}

}  // namespace

bool make_map_u8(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer, uint32_t box_outer) {
    return make_map(map, base, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, inner, outer, box_outer);
}

// General 2-D row-major map with an explicit box and swizzle mode.
bool make_map_box(CUtensorMap* map, const void* base, CUtensorMapDataType dt, int elem_bytes, uint64_t inner,
                  uint64_t outer, uint32_t box_inner, uint32_t box_outer, bool swizzle128) {
    auto fn = encode_fn();
    if (!fn) { set_error("cuTensorMapEncodeTiled unavailable"); return false; }
    cuuint64_t dims[2] = {inner, outer};
    cuuint64_t strides[1] = {inner * (uint64_t)elem_bytes};
    cuuint32_t box[2] = {box_inner, box_outer};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(map, dt, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                    swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        set_error("cuTensorMapEncodeTiled failed (%d) for [%llu, %llu] box [%u, %u]", (int)r,
                  (unsigned long long)outer, (unsigned long long)inner, box_outer, box_inner);
        return false;
    }
    return true;
}

cudaError_t launch_expert_up_gate(const void* a_rows, const void* w_gate, const void* w_up, const Shape& s,
                                  const GroupTable& gt, int* status, const GemmScales& sc, void* h_rows,
                                  cudaStream_t st, int num_sms) {
    if (gt.G <= 0 || gt.rows_capacity <= 0) return cudaSuccess;
    const FmtDesc fd = fmt_desc(s.dtype);
    const uint64_t rows = (uint64_t)gt.rows_capacity;
    CUtensorMap ta, tg, tu;
    if (!make_map(&ta, a_rows, fd.dt, fd.elem_bytes, s.d, rows, kBM) ||
        !make_map(&tg, w_gate, fd.dt, fd.elem_bytes, s.f, (uint64_t)s.E * s.d, fd.bk) ||
        !make_map(&tu, w_up, fd.dt, fd.elem_bytes, s.f, (uint64_t)s.E * s.d, fd.bk))
        return cudaErrorInvalidValue;
    GemmParams p = base_params(gt, status, sc);
    p.K = s.d;
    p.n_tiles = s.f / 128;
    p.out_ld = s.f;
    p.out = h_rows;
    switch (s.dtype) {
        case MOE_DTYPE_INT8:
            p.idesc = idesc_i8(kBM, kUmmaN, true);
            return launch_gemm<0, FmtI8>(ta, tg, tu, p, st, num_sms);
        case MOE_DTYPE_FP8:
            p.idesc = idesc_e4m3(kBM, kUmmaN, true);
            return launch_gemm<0, FmtE4>(ta, tg, tu, p, st, num_sms);
        case MOE_DTYPE_BF16:
            p.idesc = idesc_f16(true, kBM, kUmmaN, false, true);
            return launch_gemm<0, Fmt16<__nv_bfloat16>>(ta, tg, tu, p, st, num_sms);
        default:
            p.idesc = idesc_f16(false, kBM, kUmmaN, false, true);
            return launch_gemm<0, Fmt16<__half>>(ta, tg, tu, p, st, num_sms);
    }
}

cudaError_t launch_expert_down(const void* h_rows, const void* w_down, const Shape& s, const GroupTable& gt,
                               int* status, const GemmScales& sc, float* y_rows, cudaStream_t st, int num_sms) {
    if (gt.G <= 0 || gt.rows_capacity <= 0) return cudaSuccess;
    const FmtDesc fd = fmt_desc(s.dtype);
    const uint64_t rows = (uint64_t)gt.rows_capacity;
    CUtensorMap th, td;
    if (!make_map(&th, h_rows, fd.dt, fd.elem_bytes, s.f, rows, kBM) ||
        !make_map(&td, w_down, fd.dt, fd.elem_bytes, s.d, (uint64_t)s.E * s.f, fd.bk))
        return cudaErrorInvalidValue;
    GemmParams p = base_params(gt, status, sc);
    p.K = s.f;
    p.n_tiles = s.d / 256;
    p.out_ld = s.d;
    p.out = y_rows;
    switch (s.dtype) {
        case MOE_DTYPE_INT8:
            p.idesc = idesc_i8(kBM, kUmmaN, true);
            return launch_gemm<1, FmtI8>(th, td, td, p, st, num_sms);
        case MOE_DTYPE_FP8:
            p.idesc = idesc_e4m3(kBM, kUmmaN, true);
            return launch_gemm<1, FmtE4>(th, td, td, p, st, num_sms);
        case MOE_DTYPE_BF16:
            p.idesc = idesc_f16(true, kBM, kUmmaN, false, true);
            return launch_gemm<1, Fmt16<__nv_bfloat16>>(th, td, td, p, st, num_sms);
        default:
            p.idesc = idesc_f16(false, kBM, kUmmaN, false, true);
            return launch_gemm<1, Fmt16<__half>>(th, td, td, p, st, num_sms);
    }
}

}  // namespace moe
