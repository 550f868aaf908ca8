// Seeded, counter-based input generator (the reference has none: its
// inputs/data.cu:164-177 zero-fills, and the router weights are memset to 0).
//
// Value i of stream (seed, stream):
//   key  = splitmix64(seed ^ splitmix64(stream + 0x5851F42D4C957F2D))
//   u(j) = ((splitmix64(key + j * 0x9E3779B97F4A7C15) >> 11) + 0.5) * 2^-53   in (0, 1)
//   pair p = i / 2 uses u(2p), u(2p+1) in the Box-Muller transform
//   z0 = sqrt(-2 ln u(2p)) cos(2 pi u(2p+1)),  z1 = ... sin(...)
//   value i = std * (i even ? z0 : z1), computed in double, rounded once.
// It depends only on (seed, stream, i): any thread split gives the same data.
#include <cmath>
#include <cstdint>
#include <cstring>
#include <thread>
#include <vector>
#include <algorithm>

#include "../../include/sparsemoe_b200.h"

namespace {

inline uint64_t splitmix64(uint64_t z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}
inline uint64_t stream_key(uint64_t seed, uint64_t stream) {
    return splitmix64(seed ^ splitmix64(stream + 0x5851F42D4C957F2Dull));
}
inline double uniform01(uint64_t key, uint64_t j) {
    const uint64_t h = splitmix64(key + j * 0x9E3779B97F4A7C15ull);
    return ((double)(h >> 11) + 0.5) * (1.0 / 9007199254740992.0);
}
inline double normal_at(uint64_t key, uint64_t i) {
    const uint64_t p = i >> 1;
    const double u1 = uniform01(key, 2 * p), u2 = uniform01(key, 2 * p + 1);
    const double r = std::sqrt(-2.0 * std::log(u1));
    const double a = 6.283185307179586 * u2;
    return (i & 1) ? r * std::sin(a) : r * std::cos(a);
}

uint16_t f32_to_f16_rn(float f) {
    uint32_t x;
    std::memcpy(&x, &f, 4);
    const uint32_t sign = (x >> 16) & 0x8000u;
    const uint32_t ax = x & 0x7fffffffu;
    if (ax >= 0x7f800000u) return (uint16_t)(sign | 0x7c00u | (ax > 0x7f800000u ? 0x200u : 0u));
    if (ax >= 0x477ff000u) return (uint16_t)(sign | 0x7c00u);  // rounds to >= 65520 -> inf
    if (ax < 0x38800000u) {                                   // subnormal half (or zero)
        if (ax < 0x33000000u) return (uint16_t)sign;          // < 2^-25: rounds to 0
        const uint32_t e = ax >> 23;
        const uint32_t m = (ax & 0x7fffffu) | 0x800000u;
        const uint32_t shift = 126 - e;                        // 14 + (113 - e) - ... -> mantissa shift
        const uint32_t q = m >> shift;
        const uint32_t rem = m & ((1u << shift) - 1u);
        const uint32_t half = 1u << (shift - 1);
        uint32_t r = q + ((rem > half || (rem == half && (q & 1u))) ? 1u : 0u);
        return (uint16_t)(sign | r);
    }
    uint32_t r = ((ax - 0x38000000u) >> 13);
    const uint32_t rem = ax & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (r & 1u))) ++r;
    return (uint16_t)(sign | r);
}
uint16_t f32_to_bf16_rn(float f) {
    uint32_t u;
    std::memcpy(&u, &f, 4);
    if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40u);
    u += 0x7fffu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}

template <class F>
void parallel_range(size_t n, F&& fn) {
    unsigned nt = std::max(1u, std::min(16u, std::thread::hardware_concurrency()));
    if (n < (1u << 16)) nt = 1;
    std::vector<std::thread> pool;
    const size_t per = (n + nt - 1) / nt;
    for (unsigned t = 0; t < nt; ++t) {
        const size_t b = t * per, e = std::min(n, b + per);
        if (b >= e) break;
        pool.emplace_back([=, &fn]() { fn(b, e); });
    }
    for (auto& th : pool) th.join();
}

}  // namespace

extern "C" void moe_fill_normal_16(uint16_t* dst, size_t n, uint64_t seed, uint64_t stream, float stdv,
                                   int bf16) {
    const uint64_t key = stream_key(seed, stream);
    parallel_range(n, [&](size_t b, size_t e) {
        for (size_t i = b; i < e; ++i) {
            const float v = (float)(stdv * normal_at(key, i));
            dst[i] = bf16 ? f32_to_bf16_rn(v) : f32_to_f16_rn(v);
        }
    });
}

extern "C" void moe_fill_normal_f32(float* dst, size_t n, uint64_t seed, uint64_t stream, float stdv) {
    const uint64_t key = stream_key(seed, stream);
    parallel_range(n, [&](size_t b, size_t e) {
        for (size_t i = b; i < e; ++i) dst[i] = (float)(stdv * normal_at(key, i));
    });
}

extern "C" void moe_zipf_bias(float* dst, int E, float s, float scale, uint64_t seed) {
    std::vector<int> rank(E);
    for (int e = 0; e < E; ++e) rank[e] = e;
    if (seed != 0) {  // Fisher-Yates with the counter-based stream
        const uint64_t key = stream_key(seed, 0x7A1Full);
        for (int i = E - 1; i > 0; --i) {
            const int j = (int)(uniform01(key, (uint64_t)i) * (i + 1));
            std::swap(rank[i], rank[std::min(j, i)]);
        }
    }
    for (int e = 0; e < E; ++e) dst[e] = (float)(-(double)scale * s * std::log(1.0 + rank[e]));
}
