// Stage 4 for the reference's int4 format (MOE_DTYPE_INT4_PTX,
// kernels/capacity_int4_ptx.cu): per-tensor int4 weights stored packed
// transposed (inputs/data.cu:89-140: per expert [N/2][K] bytes, byte (p, k)
// holds column 2p in its low nibble and column 2p+1 in its high nibble),
// activations and h as int4 values one per byte, s32 accumulation, the
// reference's per-tensor dequant / SiLU / requant (clamp +-7) and down
// dequant in the epilogue.
//
// The packed-transposed bytes are already K-contiguous per column pair, so a
// TMA box of 64 pair rows x 128 K bytes holds 128 weight columns x 128 K; a
// converter warpgroup sign-extends each byte's two nibbles into rows 2p and
// 2p+1 of a K-major int8 B tile (128B swizzle, the layout of the A tile), and
// the tensor core runs exact tcgen05.mma kind::i8 M128 N256 K32 on it.  The
// weights cross HBM once as nibbles, with no unpacked copy.
//
// Warps (448 threads, persistent, one CTA per SM):
//   0      TMA: int8 A tile (128 rows x 128 K bytes) and the packed B tile
//          (2 boxes of 64 pair rows x 128 K bytes) per K block, 3-stage ring.
//   1      MMA: 4 x kind::i8 M128 N256 K32 per K block into a double-buffered
//          256-column TMEM accumulator.
//   2-5    epilogue: up/gate -> h = requant(silu(G s_in s_gate) U s_in s_up / s_mid)
//          as int4 values in int8 (TMEM columns [0,128) gate, [128,256) up of
//          the same 128 features); down -> f32 rows Y * s_mid s_down.
//   6-13   converter: nibbles -> K-major int8 B (3-stage ring).
#include "moe_internal.h"
#include "common.cuh"
#include "sm100.cuh"

#include <cuda.h>

namespace moe {

bool make_map_u8(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer, uint32_t box_outer);

namespace {

using namespace sm100;

constexpr int kBM = 128, kBN = 256, kBK = 128;   // K block = 128 int8 = one 128-byte swizzle row
constexpr int kABytes = kBM * kBK;               // 16 KB
constexpr int kPBytes = (kBN / 2) * kBK;         // 16 KB of packed pairs
constexpr int kBBytes = kBN * kBK;               // 32 KB of K-major int8
constexpr int kRaw = 3, kBSt = 3;
constexpr int kRawBytes = kABytes + kPBytes;
constexpr int kThreads = 448;
constexpr int kConvThreads = 256;
constexpr int kTmemCols = 512;
constexpr size_t kSmemBytes = 1024 + (size_t)kRaw * kRawBytes + (size_t)kBSt * kBBytes + 256 + 4 * 2048;
static_assert(kSmemBytes + sizeof(int) * (5 * kMaxGroups + 1) <= 232448, "shared memory per CTA");

struct I4Params {
    const int* g_rows;
    const int* g_start;
    const int* g_weight;
    int G;
    int K;
    int n_tiles;
    int out_ld;
    int pairs;          // N / 2: packed pair rows per expert matrix
    void* out;          // int8 h rows (up/gate) or f32 y rows (down)
    int* status;
    uint32_t idesc;
    float deq_gate, deq_up, inv_mid, deq_down;   // capacity_int4_ptx.cu:455-457, 596
    OutRedirect red;
};

struct I4Maps {
    CUtensorMap a;        // int8 rows [rows, K]
    CUtensorMap p0, p1;   // packed pairs [E * N/2, K] (gate, up; down uses p0)
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

// The four low (high) nibbles of a word's bytes, each sign-extended to a byte.
__device__ __forceinline__ uint32_t sext_lo4(uint32_t w) { return __vsub4((w & 0x0F0F0F0Fu) ^ 0x08080808u, 0x08080808u); }
__device__ __forceinline__ uint32_t sext_hi4(uint32_t w) {
    return __vsub4(((w >> 4) & 0x0F0F0F0Fu) ^ 0x08080808u, 0x08080808u);
}

__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// kMode 0: up/gate + SwiGLU -> int4-valued h;  1: down -> f32 y.
template <int kMode>
__global__ void __launch_bounds__(kThreads, 1)
    i4_gemm_kernel(const __grid_constant__ I4Maps mp, const I4Params p) {
    extern __shared__ uint8_t smem_raw[];
    __shared__ int s_pre[kMaxGroups + 1];
    __shared__ int s_mt[kMaxGroups];
    __shared__ int s_rows[kMaxGroups];
    __shared__ int s_start[kMaxGroups];
    __shared__ int s_wt[kMaxGroups];

    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* raw0 = smem;
    uint8_t* bst0 = smem + kRaw * kRawBytes;
    uint64_t* full = reinterpret_cast<uint64_t*>(bst0 + kBSt * kBBytes);
    uint64_t* empty = full + kRaw;
    uint64_t* conv = empty + kRaw;
    uint64_t* bfree = conv + kBSt;
    uint64_t* tfull = bfree + kBSt;
    uint64_t* tempty = tfull + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
    float4* sStage = reinterpret_cast<float4*>(bst0 + kBSt * kBBytes + 256);
    auto sA = [&](int s) { return raw0 + s * kRawBytes; };
    auto sP = [&](int s) { return raw0 + s * kRawBytes + kABytes; };
    auto sB = [&](int b) { return bst0 + b * kBBytes; };

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int s = 0; s < kRaw; ++s) { mbar_init(&full[s], 1); mbar_init(&empty[s], 1); }
        for (int b = 0; b < kBSt; ++b) { mbar_init(&conv[b], kConvThreads); mbar_init(&bfree[b], 1); }
        for (int a = 0; a < 2; ++a) { mbar_init(&tfull[a], 1); mbar_init(&tempty[a], 128); }
        fence_mbar_init();
        tma_prefetch_desc(&mp.a);
        tma_prefetch_desc(&mp.p0);
        if (kMode == 0) tma_prefetch_desc(&mp.p1);
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
            int s = 0;
            uint32_t ph = 0;
            for (int t = blockIdx.x; t < total; t += gridDim.x) {
                int g, m, n;
                decode_tile(t, s_pre, s_mt, p.G, g, m, n);
                const int a_row = s_start[g] + m * kBM;
                // packed pair rows of this tile: up/gate 64 gate + 64 up pairs (128 features), down 128 pairs
                const int prow = s_wt[g] * p.pairs + n * (kMode == 0 ? 64 : 128);
                for (int kb = 0; kb < kblocks; ++kb) {
                    if (!mbar_wait(&empty[s], ph ^ 1u, p.status, kDevErrTimeout)) goto producer_done;
                    mbar_arrive_expect_tx(&full[s], kRawBytes);
                    const int k0 = kb * kBK;
                    tma_load_2d(sA(s), &mp.a, &full[s], k0, a_row);
                    if (kMode == 0) {
                        tma_load_2d(sP(s), &mp.p0, &full[s], k0, prow);
                        tma_load_2d(sP(s) + kPBytes / 2, &mp.p1, &full[s], k0, prow);
                    } else {
                        tma_load_2d(sP(s), &mp.p0, &full[s], k0, prow);
                        tma_load_2d(sP(s) + kPBytes / 2, &mp.p0, &full[s], k0, prow + 64);
                    }
                    if (++s == kRaw) { s = 0; ph ^= 1u; }
                }
            }
        producer_done:;
        }
    } else if (warp == 1) {
        if (lane == 0) {
            int s = 0, b = 0, acc = 0;
            uint32_t bph = 0, aph = 0;
            for (int t = blockIdx.x; t < total; t += gridDim.x) {
                if (!mbar_wait(&tempty[acc], aph ^ 1u, p.status, kDevErrTimeout)) break;
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + acc * kBN;
                bool ok = true;
                for (int kb = 0; kb < kblocks; ++kb) {
                    // the converter finished B[b] after its raw stage (A included) had landed
                    if (!mbar_wait(&conv[b], bph, p.status, kDevErrTimeout)) { ok = false; break; }
                    tc_fence_after();
                    const uint32_t a_base = smem_u32(sA(s));
                    const uint32_t b_base = smem_u32(sB(b));
#pragma unroll
                    for (int kk = 0; kk < 4; ++kk) {
                        // both operands K-major SW128: 8-row groups 1024 B apart, K step 32 bytes
                        const uint64_t adesc = smem_desc_sw128(a_base + kk * 32, 16, 1024);
                        const uint64_t bdesc = smem_desc_sw128(b_base + kk * 32, 16, 1024);
                        mma_i8_ss(d_tmem, adesc, bdesc, p.idesc, (kb | kk) != 0 ? 1u : 0u);
                    }
                    mma_commit(&empty[s]);
                    mma_commit(&bfree[b]);
                    if (++s == kRaw) s = 0;
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
        const int row_in_tile = q * 32 + lane;
        int acc = 0;
        uint32_t aph = 0;
        float4* stage = sStage + (warp - 2) * 128;
        for (int t = blockIdx.x; t < total; t += gridDim.x) {
            int g, m, n;
            decode_tile(t, s_pre, s_mt, p.G, g, m, n);
            if (!mbar_wait_warp(&tfull[acc], aph, p.status, kDevErrTimeout)) break;
            tc_fence_after();
            const int row_local = m * kBM + row_in_tile;
            const bool valid = row_local < s_rows[g];
            const uint32_t taddr = tmem_base + ((uint32_t)(q * 32) << 16) + acc * kBN;
            if (kMode == 0) {
                int8_t* h = reinterpret_cast<int8_t*>(p.out) + ((int64_t)s_start[g] + row_local) * p.out_ld + n * 128;
#pragma unroll 1
                for (int c = 0; c < 128; c += 32) {
                    uint32_t gr[32], ur[32];
                    tmem_ld_32x32b_x32(taddr + c, gr);
                    tmem_ld_32x32b_x32(taddr + 128 + c, ur);
                    tmem_wait_ld();
                    if (c == 96) { tc_fence_before(); mbar_arrive(&tempty[acc]); }
                    // capacity_int4_ptx.cu:470-477: dequant, SiLU(gate) * up, requant to [-7, 7]
                    uint32_t packed[8];
#pragma unroll
                    for (int i = 0; i < 8; ++i) {
                        uint32_t word = 0;
#pragma unroll
                        for (int j = 0; j < 4; ++j) {
                            const float uf = (float)(int)ur[4 * i + j] * p.deq_up;
                            const float gf = (float)(int)gr[4 * i + j] * p.deq_gate;
                            const float silu = gf / (1.0f + __expf(-gf));
                            const float fused = uf * silu;
                            const int qv = __float2int_rn(fminf(fmaxf(fused * p.inv_mid, -7.f), 7.f));
                            word |= (uint32_t)(qv & 0xFF) << (8 * j);
                        }
                        packed[i] = word;
                    }
                    if (valid) {
                        uint4* o = reinterpret_cast<uint4*>(h + c);
                        o[0] = make_uint4(packed[0], packed[1], packed[2], packed[3]);
                        o[1] = make_uint4(packed[4], packed[5], packed[6], packed[7]);
                    }
                }
            } else {
                const int warp_row0 = m * kBM + q * 32;
                const int nrows = s_rows[g] - warp_row0;
                float* y = down_rows(p.red, reinterpret_cast<float*>(p.out), g, s_start[g], p.out_ld) +
                           (int64_t)warp_row0 * p.out_ld + n * kBN;
#pragma unroll 1
                for (int c = 0; c < kBN; c += 32) {
                    uint32_t r[32];
                    tmem_ld_32x32b_x32(taddr + c, r);
                    tmem_wait_ld();
                    if (c == kBN - 32) { tc_fence_before(); mbar_arrive(&tempty[acc]); }
                    float v[32];
#pragma unroll
                    for (int i = 0; i < 32; ++i) v[i] = (float)(int)r[i] * p.deq_down;   // :615
                    warp_store_rows16(stage, v, y + c, p.out_ld, nrows, lane);
                    warp_store_rows16(stage, v + 16, y + c + 16, p.out_ld, nrows, lane);
                }
            }
            acc ^= 1;
            if (acc == 0) aph ^= 1u;
        }
        if (kMode == 1 && p.red.rank) __threadfence_system();
    } else {
        // ---------------- converter (warps 6..13) ----------------
        // 16-byte chunk id = packed row pr (0..127) x chunk c (0..7); the TMA
        // wrote row pr's chunk c at chunk c ^ (pr & 7); B rows 2pr (low
        // nibbles) and 2pr+1 (high nibbles) take their chunk c at c ^ (row & 7).
        const int ct = threadIdx.x - 192;
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
                const uint8_t* src = sP(s);
                uint8_t* dst = sB(b);
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const int id = ct + i * kConvThreads;
                    const int pr = id >> 3, c = id & 7;
                    const uint4 w = *reinterpret_cast<const uint4*>(src + pr * 128 + ((c ^ (pr & 7)) << 4));
                    const int r0 = 2 * pr, r1 = r0 + 1;
                    *reinterpret_cast<uint4*>(dst + r0 * 128 + ((c ^ (r0 & 7)) << 4)) =
                        make_uint4(sext_lo4(w.x), sext_lo4(w.y), sext_lo4(w.z), sext_lo4(w.w));
                    *reinterpret_cast<uint4*>(dst + r1 * 128 + ((c ^ (r1 & 7)) << 4)) =
                        make_uint4(sext_hi4(w.x), sext_hi4(w.y), sext_hi4(w.z), sext_hi4(w.w));
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

template <int kMode>
cudaError_t launch_i4(const I4Maps& mp, const I4Params& p, cudaStream_t st, int num_sms) {
    auto kern = i4_gemm_kernel<kMode>;
    static SmemAttr attr;
    cudaError_t err = ensure_smem(kern, kSmemBytes, attr);
    if (err != cudaSuccess) return err;
    kern<<<num_sms, kThreads, kSmemBytes, st>>>(mp, p);
    return cudaGetLastError();
}

I4Params base_params(const GroupTable& gt, int* status, const GemmScales& sc) {
    I4Params p{};
    p.g_rows = gt.rows;
    p.g_start = gt.start;
    p.g_weight = gt.weight;
    p.G = gt.G;
    p.status = status;
    p.idesc = idesc_i8(kBM, kBN, /*b_mn_major=*/false);
    p.deq_gate = sc.s_in * sc.s_gate;
    p.deq_up = sc.s_in * sc.s_up;
    p.inv_mid = 1.0f / sc.s_mid;
    p.deq_down = sc.s_mid * sc.s_down;
    p.red = gt.redirect;
    return p;
}

}  // namespace

cudaError_t launch_i4_up_gate(const void* a_rows, const void* w_gate, const void* w_up, const Shape& s,
                              const GroupTable& gt, int* status, const GemmScales& sc, void* h_rows, cudaStream_t st,
                              int num_sms) {
    if (gt.G <= 0 || gt.rows_capacity <= 0) return cudaSuccess;
    I4Maps mp;
    if (!make_map_u8(&mp.a, a_rows, s.d, gt.rows_capacity, kBM) ||
        !make_map_u8(&mp.p0, w_gate, s.d, (uint64_t)s.E * (s.f / 2), 64) ||
        !make_map_u8(&mp.p1, w_up, s.d, (uint64_t)s.E * (s.f / 2), 64))
        return cudaErrorInvalidValue;
    I4Params p = base_params(gt, status, sc);
    p.red = OutRedirect{};
    p.K = s.d;
    p.n_tiles = s.f / 128;
    p.out_ld = s.f;
    p.pairs = s.f / 2;
    p.out = h_rows;
    return launch_i4<0>(mp, p, st, num_sms);
}

cudaError_t launch_i4_down(const void* h_rows, const void* w_down, const Shape& s, const GroupTable& gt, int* status,
                           const GemmScales& sc, float* y_rows, cudaStream_t st, int num_sms) {
    if (gt.G <= 0 || gt.rows_capacity <= 0) return cudaSuccess;
    I4Maps mp;
    if (!make_map_u8(&mp.a, h_rows, s.f, gt.rows_capacity, kBM) ||
        !make_map_u8(&mp.p0, w_down, s.f, (uint64_t)s.E * (s.d / 2), 64))
        return cudaErrorInvalidValue;
    mp.p1 = mp.p0;
    I4Params p = base_params(gt, status, sc);
    p.K = s.f;
    p.n_tiles = s.d / 256;
    p.out_ld = s.d;
    p.pairs = s.d / 2;
    p.out = y_rows;
    return launch_i4<1>(mp, p, st, num_sms);
}

}  // namespace moe
