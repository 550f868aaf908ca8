// Host input builder: the reference's inputs/data.h API (inputs/data.cu:13-640
// of MattJBorowski1991/SparseMoE), rewritten, with shapes taken from the
// runtime solve() dims instead of config.h constants, plus a seeded variant.
//
// Buffer sizes follow the reference (inputs/data.cu:400-521): every
// intermediate is [B, E, CAP, .]-sized, CAP = moe_capacity(...) when
// use_capacity else N; only the buffers of the chosen weight format are
// allocated; unused pointers stay null (memset 0, inputs/data.cu:211).
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <vector>
#include <cuda_fp8.h>

#include "../../include/data.h"
#include "../../include/sparsemoe_b200.h"

namespace {

#define BUILDER_CHECK(call)                                                                   \
    do {                                                                                      \
        cudaError_t err_ = (call);                                                            \
        if (err_ != cudaSuccess) {                                                            \
            fprintf(stderr, "CUDA Error at: %s: %d: %s \n", __FILE__, __LINE__,              \
                    cudaGetErrorString(err_));                                                \
            exit(1);                                                                          \
        }                                                                                     \
    } while (0)

struct BuilderState {
    bool seeded = false;
    uint64_t seed = 0;
};
BuilderState g_builder;

float h2f(half v) { return __half2float(v); }

// inputs/data.cu:13-34 / 36-57: per-tensor symmetric, scale = max|x| / qmax,
// q = nearbyint(clamp(x / scale, -qmax, qmax)).
float quant_symmetric(const std::vector<half>& src, std::vector<int8_t>& dst, float qmax);

}  // namespace

extern "C" float moe_quantize_per_tensor(const uint16_t* src, size_t n, int8_t* dst, float qmax) {
    float m = 0.0f;
    for (size_t i = 0; i < n; ++i) {
        half h;
        std::memcpy(&h, &src[i], 2);
        m = std::fmax(m, std::fabs(__half2float(h)));
    }
    const float scale = m > 0.0f ? m / qmax : 1.0f;
    for (size_t i = 0; i < n; ++i) {
        half h;
        std::memcpy(&h, &src[i], 2);
        const float c = std::fmin(qmax, std::fmax(-qmax, __half2float(h) / scale));
        dst[i] = (int8_t)(int)nearbyintf(c);
    }
    return scale;
}

extern "C" void moe_quantize_fp8_blocks(const uint16_t* src, int E, int K, int N, int bf16, uint8_t* q,
                                        float* scales) {
    auto val = [&](size_t i) -> float {
        if (bf16) {
            uint32_t u = (uint32_t)src[i] << 16;
            float f;
            std::memcpy(&f, &u, 4);
            return f;
        }
        half h;
        std::memcpy(&h, &src[i], 2);
        return __half2float(h);
    };
    const int kb = K / 128, nb = N / 128;
    for (int e = 0; e < E; ++e)
        for (int bk = 0; bk < kb; ++bk)
            for (int bn = 0; bn < nb; ++bn) {
                float m = 0.0f;
                for (int i = 0; i < 128; ++i)
                    for (int j = 0; j < 128; ++j)
                        m = std::fmax(m, std::fabs(val(((size_t)e * K + bk * 128 + i) * N + bn * 128 + j)));
                const float sc = m > 0.0f ? m / 448.0f : 1.0f;
                scales[((size_t)e * kb + bk) * nb + bn] = sc;
                for (int i = 0; i < 128; ++i)
                    for (int j = 0; j < 128; ++j) {
                        const size_t idx = ((size_t)e * K + bk * 128 + i) * N + bn * 128 + j;
                        q[idx] = (uint8_t)__nv_cvt_float_to_fp8(val(idx) / sc, __NV_SATFINITE, __NV_E4M3);
                    }
            }
}

extern "C" void moe_quantize_int8_channel(const uint16_t* src, int E, int K, int N, int bf16, int8_t* q,
                                          float* scales) {
    auto val = [&](size_t i) -> float {
        if (bf16) {
            uint32_t u = (uint32_t)src[i] << 16;
            float f;
            std::memcpy(&f, &u, 4);
            return f;
        }
        half h;
        std::memcpy(&h, &src[i], 2);
        return __half2float(h);
    };
    std::vector<float> m((size_t)N);
    for (int e = 0; e < E; ++e) {
        std::fill(m.begin(), m.end(), 0.0f);
        for (int r = 0; r < K; ++r)
            for (int c = 0; c < N; ++c) m[c] = std::fmax(m[c], std::fabs(val(((size_t)e * K + r) * N + c)));
        for (int c = 0; c < N; ++c) scales[(size_t)e * N + c] = m[c] > 0.0f ? m[c] / 127.0f : 1.0f;
        for (int r = 0; r < K; ++r)
            for (int c = 0; c < N; ++c) {
                const size_t i = ((size_t)e * K + r) * N + c;
                const float v = nearbyintf(val(i) / scales[(size_t)e * N + c]);
                q[i] = (int8_t)(int)std::fmin(std::fmax(v, -127.0f), 127.0f);
            }
    }
}

namespace {
// e2m1 magnitudes by code 0..7
constexpr float kE2m1[8] = {0.0f, 0.5f, 1.0f, 1.5f, 2.0f, 3.0f, 4.0f, 6.0f};

// Nearest e2m1 code of v (ties to the even code, saturating at 6), sign in bit 3.
uint8_t e2m1_code(float v) {
    const uint8_t sign = v < 0.0f ? 8 : 0;
    const float a = std::fabs(v);
    int best = 7;
    if (a < 6.0f) {
        best = 0;
        for (int c = 1; c < 8; ++c) {
            const float dc = std::fabs(a - kE2m1[c]), db = std::fabs(a - kE2m1[best]);
            if (dc < db || (dc == db && (c & 1) == 0)) best = c;
        }
    }
    return (uint8_t)(sign | best);
}

float e4m3_value(uint8_t code) {
    const __half_raw r = __nv_cvt_fp8_to_halfraw(code, __NV_E4M3);
    return __half2float(__half(r));
}
}  // namespace

extern "C" void moe_quantize_nvfp4(const uint16_t* src, int E, int K, int N, int bf16, uint8_t* packed,
                                   uint8_t* scales, float* globals) {
    auto val = [&](size_t i) -> float {
        if (bf16) {
            uint32_t u = (uint32_t)src[i] << 16;
            float f;
            std::memcpy(&f, &u, 4);
            return f;
        }
        half h;
        std::memcpy(&h, &src[i], 2);
        return __half2float(h);
    };
    const int G = K / 16;
    std::memset(packed, 0, (size_t)E * K * (N / 2));
    for (int e = 0; e < E; ++e) {
        float amax = 0.0f;
        for (size_t i = 0; i < (size_t)K * N; ++i) amax = std::fmax(amax, std::fabs(val((size_t)e * K * N + i)));
        const float g = amax > 0.0f ? amax / (448.0f * 6.0f) : 1.0f;
        globals[e] = g;
        for (int gr = 0; gr < G; ++gr)
            for (int n = 0; n < N; ++n) {
                float m = 0.0f;
                for (int i = 0; i < 16; ++i) m = std::fmax(m, std::fabs(val(((size_t)e * K + gr * 16 + i) * N + n)));
                uint8_t sc = 0x38;   // 1.0
                if (m > 0.0f) {
                    sc = (uint8_t)__nv_cvt_float_to_fp8(m / (6.0f * g), __NV_SATFINITE, __NV_E4M3);
                    if ((sc & 0x7F) == 0) sc = 0x01;   // smallest positive subnormal, never zero
                }
                scales[((size_t)e * G + gr) * N + n] = sc;
                const float div = e4m3_value(sc) * g;
                for (int i = 0; i < 16; ++i) {
                    const size_t k = (size_t)gr * 16 + i;
                    const uint8_t q = e2m1_code(val(((size_t)e * K + k) * N + n) / div);
                    const int pcol = n & 7, bit = 4 * (pcol >> 1) + 16 * (pcol & 1);
                    uint8_t* word = packed + ((size_t)e * K + k) * (N / 2) + (n >> 3) * 4;
                    word[bit >> 3] |= (uint8_t)(q << (bit & 7));
                }
            }
    }
}

extern "C" void moe_quantize_int4_g128(const uint16_t* src, int E, int K, int N, int bf16, uint8_t* packed,
                                       uint16_t* scales, uint16_t* zeros) {
    auto val = [&](size_t i) -> float {
        if (bf16) {
            uint32_t u = (uint32_t)src[i] << 16;
            float f;
            std::memcpy(&f, &u, 4);
            return f;
        }
        half h;
        std::memcpy(&h, &src[i], 2);
        return __half2float(h);
    };
    const int G = K / 128;
    std::memset(packed, 0, (size_t)E * K * (N / 2));
    for (int e = 0; e < E; ++e)
        for (int g = 0; g < G; ++g)
            for (int n = 0; n < N; ++n) {
                float mn = INFINITY, mx = -INFINITY;
                for (int i = 0; i < 128; ++i) {
                    const float v = val(((size_t)e * K + g * 128 + i) * N + n);
                    mn = std::fmin(mn, v);
                    mx = std::fmax(mx, v);
                }
                float sc = (mx - mn) / 15.0f;
                if (!(sc > 0.0f)) sc = 1.0f;
                const half sh = __float2half_rn(sc);
                const half zh = __float2half_rn(-mn / __half2float(sh));
                const float sf = __half2float(sh), zf = __half2float(zh);
                std::memcpy(&scales[((size_t)e * G + g) * N + n], &sh, 2);
                std::memcpy(&zeros[((size_t)e * G + g) * N + n], &zh, 2);
                for (int i = 0; i < 128; ++i) {
                    const size_t k = (size_t)g * 128 + i;
                    const float v = val(((size_t)e * K + k) * N + n);
                    int q = (int)rintf(v / sf + zf);
                    q = q < 0 ? 0 : (q > 15 ? 15 : q);
                    // 8 columns per 32-bit word, pair (2p, 2p+1) at bits 4p and 16 + 4p
                    const int pcol = n & 7, bit = 4 * (pcol >> 1) + 16 * (pcol & 1);
                    uint8_t* word = packed + ((size_t)e * K + k) * (N / 2) + (n >> 3) * 4;
                    word[bit >> 3] |= (uint8_t)(q << (bit & 7));
                }
            }
}

// inputs/data.cu:89-140: int4 values (int8 in [-8, 7]) of E row-major [K, N]
// matrices -> per expert [N/2][K] bytes, column 2p in the low nibble and 2p+1
// in the high nibble of byte (p, k).
extern "C" void moe_pack_int4_transposed(const int8_t* q, int E, int K, int N, uint8_t* out) {
    const size_t per = (size_t)K * N, bytes_per = (size_t)(N / 2) * K;
    std::memset(out, 0, (size_t)E * bytes_per);
    for (int e = 0; e < E; ++e)
        for (int kk = 0; kk < K; ++kk)
            for (int n = 0; n < N; ++n) {
                const uint8_t nib = (uint8_t)(q[(size_t)e * per + (size_t)kk * N + n] & 0xF);
                out[(size_t)e * bytes_per + (size_t)(n / 2) * K + kk] |= (n & 1) ? (uint8_t)(nib << 4) : nib;
            }
}

// inputs/data.cu:142-150: fp16 -> e4m3 by direct conversion (nearest even,
// saturating to +-448).
extern "C" void moe_cast_e4m3(const uint16_t* src, size_t n, uint8_t* dst) {
    for (size_t i = 0; i < n; ++i) {
        half h;
        std::memcpy(&h, &src[i], 2);
        dst[i] = (uint8_t)__nv_cvt_float_to_fp8(__half2float(h), __NV_SATFINITE, __NV_E4M3);
    }
}

namespace {

float quant_symmetric(const std::vector<half>& src, std::vector<int8_t>& dst, float qmax) {
    dst.resize(src.size());
    return moe_quantize_per_tensor(reinterpret_cast<const uint16_t*>(src.data()), src.size(), dst.data(), qmax);
}

// inputs/data.cu:59-87: int4 values, two per byte, even index in the low nibble.
void pack_int4(const std::vector<int8_t>& q, std::vector<uint8_t>& out) {
    out.assign((q.size() + 1) / 2, 0);
    for (size_t i = 0; i < q.size(); ++i) {
        const uint8_t nib = (uint8_t)(q[i] & 0xF);
        out[i >> 1] |= (i & 1) ? (uint8_t)(nib << 4) : nib;
    }
}

// inputs/data.cu:89-140: per expert, [K, Ncols] -> bytes [Ncols/2][K]; byte
// (n/2, kk) holds columns n (low nibble, even) and n+1 (high nibble).
void pack_int4_transposed(const std::vector<int8_t>& q, std::vector<uint8_t>& out, int experts, int K,
                          int Ncols) {
    const size_t per = (size_t)K * Ncols;
    const size_t bytes_per = (size_t)(Ncols / 2) * K;
    out.assign((size_t)experts * bytes_per, 0);
    for (int e = 0; e < experts; ++e)
        for (int kk = 0; kk < K; ++kk)
            for (int n = 0; n < Ncols; ++n) {
                const uint8_t nib = (uint8_t)(q[(size_t)e * per + (size_t)kk * Ncols + n] & 0xF);
                uint8_t& b = out[(size_t)e * bytes_per + (size_t)(n / 2) * K + kk];
                b |= (n & 1) ? (uint8_t)(nib << 4) : nib;
            }
}

template <class T>
T* upload(const T* host, size_t count) {
    T* d = nullptr;
    BUILDER_CHECK(cudaMalloc(&d, count * sizeof(T)));
    BUILDER_CHECK(cudaMemcpy(d, host, count * sizeof(T), cudaMemcpyHostToDevice));
    return d;
}
template <class T>
T* alloc(size_t count) {
    T* d = nullptr;
    BUILDER_CHECK(cudaMalloc(&d, count * sizeof(T)));
    return d;
}

enum class Fmt { F16, INT8, INT4, INT4_PTX, FP8 };

MoEArgs build(const std::vector<half>& x, const std::vector<half>& wu, const std::vector<half>& wg,
              const std::vector<half>& wd, bool use_capacity, Fmt fmt) {
    MoeDims dims;
    moe_get_solve_dims(&dims);
    const int B = dims.num_batches, Nt = dims.tokens, d = dims.d_model, f = dims.d_ff, E = dims.num_experts,
              kk = dims.top_k;
    MoEArgs a;
    std::memset(&a, 0, sizeof(a));
    a.num_batches = B;
    a.use_capacity = use_capacity;
    a.input = upload(x.data(), (size_t)B * Nt * d);
    // Router weights: zero (reference inputs/data.cu:237-243) or seeded N(0, 0.02).
    {
        const size_t n = (size_t)d * E;
        half* r = alloc<half>(n);
        if (g_builder.seeded) {
            std::vector<uint16_t> h(n);
            moe_fill_normal_16(h.data(), n, g_builder.seed, 1, 0.02f, 0);
            BUILDER_CHECK(cudaMemcpy(r, h.data(), n * 2, cudaMemcpyHostToDevice));
        } else {
            BUILDER_CHECK(cudaMemset(r, 0, n * 2));
        }
        a.router_weights = r;
    }
    const size_t nw = (size_t)E * d * f;
    if (fmt == Fmt::F16) {
        a.expert_up_proj_weights = upload(wu.data(), nw);
        a.expert_gate_proj_weights = upload(wg.data(), nw);
        a.expert_down_proj_weights = upload(wd.data(), nw);
    } else if (fmt == Fmt::INT8 || fmt == Fmt::INT4 || fmt == Fmt::INT4_PTX) {
        const float qmax = fmt == Fmt::INT8 ? 127.0f : 7.0f;
        std::vector<int8_t> qu, qg, qd;
        a.scale_up_w = quant_symmetric(wu, qu, qmax);
        a.scale_gate_w = quant_symmetric(wg, qg, qmax);
        a.scale_down_w = quant_symmetric(wd, qd, qmax);
        a.scale_input_act = 1.0f;  // placeholder activation scales (inputs/data.cu:320-322)
        a.scale_mid_act = 1.0f;
        a.expert_up_proj_weights_int8 = upload(qu.data(), qu.size());
        a.expert_gate_proj_weights_int8 = upload(qg.data(), qg.size());
        a.expert_down_proj_weights_int8 = upload(qd.data(), qd.size());
        if (fmt != Fmt::INT8) {
            std::vector<uint8_t> pu, pg, pd;
            if (fmt == Fmt::INT4_PTX) {
                pack_int4_transposed(qu, pu, E, d, f);
                pack_int4_transposed(qg, pg, E, d, f);
                pack_int4_transposed(qd, pd, E, f, d);
            } else {
                pack_int4(qu, pu);
                pack_int4(qg, pg);
                pack_int4(qd, pd);
            }
            a.expert_up_proj_weights_int4 = upload(pu.data(), pu.size());
            a.expert_gate_proj_weights_int4 = upload(pg.data(), pg.size());
            a.expert_down_proj_weights_int4 = upload(pd.data(), pd.size());
        }
    } else {  // FP8: direct e4m3 cast, unit scales (inputs/data.cu:142-150, 359-390)
        auto cast = [&](const std::vector<half>& src) {
            std::vector<__nv_fp8_e4m3> q(src.size());
            for (size_t i = 0; i < src.size(); ++i) q[i] = __nv_fp8_e4m3(h2f(src[i]));
            return upload(q.data(), q.size());
        };
        a.expert_up_proj_weights_fp8 = cast(wu);
        a.expert_gate_proj_weights_fp8 = cast(wg);
        a.expert_down_proj_weights_fp8 = cast(wd);
        a.scale_up_w = a.scale_gate_w = a.scale_down_w = a.scale_input_act = a.scale_mid_act = 1.0f;
    }
    const int cap = use_capacity ? moe_capacity(Nt, kk, E, dims.capacity_factor) : Nt;
    a.cap = cap;
    const size_t rows = (size_t)B * E * cap;
    a.expert_logits = alloc<float>((size_t)B * Nt * E);
    a.selected_expert_indices = alloc<int>((size_t)B * Nt * kk);
    a.selected_expert_weights = alloc<float>((size_t)B * Nt * kk);
    a.expert_counts = alloc<int>((size_t)B * E);
    a.expert_token_ids = alloc<int>(rows);
    a.expert_token_weights = alloc<float>(rows);
    if (fmt == Fmt::F16) a.per_expert_wmma_inputs = alloc<half>(rows * d);
    if (fmt == Fmt::INT8 || fmt == Fmt::INT4 || fmt == Fmt::INT4_PTX)
        a.per_expert_wmma_inputs_int8 = alloc<int8_t>(rows * d);
    if (fmt == Fmt::INT4 || fmt == Fmt::INT4_PTX) a.per_expert_wmma_inputs_int4 = alloc<uint8_t>(rows * d / 2);
    if (fmt == Fmt::FP8) a.per_expert_wmma_inputs_fp8 = alloc<__nv_fp8_e4m3>(rows * d);
    a.hidden_mlp_layer_1_out = alloc<float>(rows * f);
    a.hidden_mlp_gate_out = alloc<float>(rows * f);
    if (fmt == Fmt::F16) a.hidden_mlp_layer_1_out_fp16 = alloc<half>(rows * f);
    if (fmt == Fmt::INT8 || fmt == Fmt::INT4 || fmt == Fmt::INT4_PTX)
        a.hidden_mlp_layer_1_out_int8 = alloc<int8_t>(rows * f);
    if (fmt == Fmt::INT4 || fmt == Fmt::INT4_PTX) a.hidden_mlp_layer_1_out_int4 = alloc<uint8_t>(rows * f / 2);
    if (fmt == Fmt::FP8) a.hidden_mlp_layer_1_out_fp8 = alloc<__nv_fp8_e4m3>(rows * f);
    a.hidden_mlp_layer_2_out = alloc<float>(rows * d);
    a.final_output = alloc<float>((size_t)B * Nt * d);
    return a;
}

}  // namespace

void initialize_host_data(std::vector<half>& h_input, std::vector<float>& h_final_output,
                          std::vector<half>& h_expert_up_proj_weights,
                          std::vector<half>& h_expert_gate_proj_weights,
                          std::vector<half>& h_expert_down_proj_weights) {
    g_builder.seeded = false;
    const half z = __float2half(0.0f);
    std::fill(h_input.begin(), h_input.end(), z);
    std::fill(h_final_output.begin(), h_final_output.end(), 0.0f);
    std::fill(h_expert_up_proj_weights.begin(), h_expert_up_proj_weights.end(), z);
    std::fill(h_expert_gate_proj_weights.begin(), h_expert_gate_proj_weights.end(), z);
    std::fill(h_expert_down_proj_weights.begin(), h_expert_down_proj_weights.end(), z);
}

void initialize_host_data_seeded(std::vector<half>& h_input, std::vector<float>& h_final_output,
                                 std::vector<half>& h_expert_up_proj_weights,
                                 std::vector<half>& h_expert_gate_proj_weights,
                                 std::vector<half>& h_expert_down_proj_weights, uint64_t seed) {
    MoeDims dims;
    moe_get_solve_dims(&dims);
    g_builder.seeded = true;
    g_builder.seed = seed;
    auto fill = [&](std::vector<half>& v, uint64_t stream, float stdv) {
        moe_fill_normal_16(reinterpret_cast<uint16_t*>(v.data()), v.size(), seed, stream, stdv, 0);
    };
    fill(h_input, 0, 1.0f);
    fill(h_expert_gate_proj_weights, 2, 1.0f / std::sqrt((float)dims.d_model));
    fill(h_expert_up_proj_weights, 3, 1.0f / std::sqrt((float)dims.d_model));
    fill(h_expert_down_proj_weights, 4, 1.0f / std::sqrt((float)dims.d_ff));
    std::fill(h_final_output.begin(), h_final_output.end(), 0.0f);
}

MoEArgs allocate_and_copy_to_device(const std::vector<half>& x, const std::vector<half>& wu,
                                    const std::vector<half>& wg, const std::vector<half>& wd, bool use_capacity) {
    return build(x, wu, wg, wd, use_capacity, Fmt::F16);
}
MoEArgs allocate_and_copy_to_device_int8(const std::vector<half>& x, const std::vector<half>& wu,
                                         const std::vector<half>& wg, const std::vector<half>& wd,
                                         bool use_capacity) {
    return build(x, wu, wg, wd, use_capacity, Fmt::INT8);
}
MoEArgs allocate_and_copy_to_device_int4(const std::vector<half>& x, const std::vector<half>& wu,
                                         const std::vector<half>& wg, const std::vector<half>& wd,
                                         bool use_capacity) {
    return build(x, wu, wg, wd, use_capacity, Fmt::INT4);
}
MoEArgs allocate_and_copy_to_device_int4_ptx(const std::vector<half>& x, const std::vector<half>& wu,
                                             const std::vector<half>& wg, const std::vector<half>& wd,
                                             bool use_capacity) {
    return build(x, wu, wg, wd, use_capacity, Fmt::INT4_PTX);
}
MoEArgs allocate_and_copy_to_device_fp8(const std::vector<half>& x, const std::vector<half>& wu,
                                        const std::vector<half>& wg, const std::vector<half>& wd,
                                        bool use_capacity) {
    return build(x, wu, wg, wd, use_capacity, Fmt::FP8);
}

void cleanup_device_data(MoEArgs& a) {
    const void* ptrs[] = {a.input, a.router_weights, a.expert_up_proj_weights, a.expert_gate_proj_weights,
                          a.expert_down_proj_weights, a.expert_up_proj_weights_int8,
                          a.expert_gate_proj_weights_int8, a.expert_down_proj_weights_int8,
                          a.expert_up_proj_weights_int4, a.expert_gate_proj_weights_int4,
                          a.expert_down_proj_weights_int4, a.expert_up_proj_weights_fp8,
                          a.expert_gate_proj_weights_fp8, a.expert_down_proj_weights_fp8, a.expert_logits,
                          a.selected_expert_indices, a.selected_expert_weights, a.expert_counts,
                          a.expert_token_ids, a.expert_token_weights, a.per_expert_wmma_inputs,
                          a.per_expert_wmma_inputs_int8, a.per_expert_wmma_inputs_int4,
                          a.per_expert_wmma_inputs_fp8, a.hidden_mlp_layer_1_out, a.hidden_mlp_gate_out,
                          a.hidden_mlp_layer_1_out_fp16, a.hidden_mlp_layer_1_out_int8,
                          a.hidden_mlp_layer_1_out_int4, a.hidden_mlp_layer_1_out_fp8,
                          a.hidden_mlp_layer_2_out, a.final_output};
    for (const void* p : ptrs)
        if (p) BUILDER_CHECK(cudaFree(const_cast<void*>(p)));
}
