// synth.cpp -- seeded synthetic weights in the on-disk layout of the reference's
// gpt_int8.safetensors (crates/core/src/models/gpt.rs:229-250, 477-515).
//
// The reference ships no weights here; its benchmark configs call for
// random-init N(0, 0.02) weights quantized MLX-style (affine, group 64, 8 bit,
// fp16 scales/biases).  This generator is the build's own quantizer:
//   per group of 64 weights: s = (max - min) / 255, b = min,
//   q = clamp(round((w - b) / s), 0, 255), packed little-endian 4 per u32.
// Every value is a pure function of (seed, tensor tag, element index), so any
// thread count gives the same bytes.
#include <cmath>
#include <cstdint>
#include <cstring>

namespace {

inline uint64_t mix64(uint64_t z) {
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
    return z ^ (z >> 31);
}

// Standard normal for element `i` of the stream (seed, tag): Box-Muller on two
// 32-bit halves of one 64-bit hash.
inline double normal_at(uint64_t seed, uint64_t tag, uint64_t i) {
    uint64_t h = mix64(mix64(seed ^ 0x5851F42D4C957F2DULL) ^ tag ^ mix64(i + 0x9E3779B97F4A7C15ULL));
    double u1 = ((double)(h >> 32) + 0.5) * (1.0 / 4294967296.0);
    double u2 = (double)(h & 0xFFFFFFFFULL) * (1.0 / 4294967296.0);
    return std::sqrt(-2.0 * std::log(u1)) * std::cos(6.283185307179586 * u2);
}

// float -> IEEE half bits, round to nearest even (own implementation).
inline uint16_t f2h(float f) {
    uint32_t x;
    std::memcpy(&x, &f, 4);
    uint32_t sign = (x >> 16) & 0x8000u;
    uint32_t ax = x & 0x7FFFFFFFu;
    if (ax >= 0x7F800000u) return (uint16_t)(sign | 0x7C00u | (ax > 0x7F800000u ? 0x200u : 0));
    if (ax >= 0x477FF000u) return (uint16_t)(sign | 0x7C00u);  // rounds to inf
    if (ax < 0x38800000u) {                                      // subnormal half
        if (ax < 0x33000000u) return (uint16_t)sign;             // < 2^-25 -> 0
        // value = m * 2^(e-150); in units of the half subnormal step 2^-24 that
        // is m >> (126 - e), rounded to nearest even.
        uint32_t e = ax >> 23, m = (ax & 0x7FFFFFu) | 0x800000u;
        uint32_t shift = 126 - e;  // 14..24
        uint32_t hq = m >> shift;
        uint32_t rem = m & ((1u << shift) - 1);
        uint32_t half = 1u << (shift - 1);
        if (rem > half || (rem == half && (hq & 1))) ++hq;
        return (uint16_t)(sign | hq);
    }
    uint32_t e = (ax >> 23) - 112, m = ax & 0x7FFFFFu;
    uint32_t h = (e << 10) | (m >> 13);
    uint32_t rem = m & 0x1FFFu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1))) ++h;
    return (uint16_t)(sign | h);
}

inline float h2f(uint16_t h) {
    uint32_t sign = (uint32_t)(h >> 15) << 31, e = (h >> 10) & 0x1F, m = h & 0x3FF, bits;
    if (e == 0) {
        float v = (float)m * 5.9604644775390625e-8f;
        return (h >> 15) ? -v : v;
    }
    if (e == 31) bits = sign | 0x7F800000u | (m << 13);
    else bits = sign | ((e + 112) << 23) | (m << 13);
    float f;
    std::memcpy(&f, &bits, 4);
    return f;
}

}  // namespace

extern "C" {

// FNV-1a of a tensor name: the per-tensor stream tag.
uint64_t itts_synth_tag(const char *name) {
    uint64_t h = 0xCBF29CE484222325ULL;
    for (const unsigned char *p = (const unsigned char *)name; *p; ++p) {
        h ^= *p;
        h *= 0x100000001B3ULL;
    }
    return h;
}

void itts_synth_normal_f32(uint64_t seed, uint64_t tag, float *dst, int64_t n, float mean,
                           float stdev) {
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < n; ++i) dst[i] = (float)(mean + stdev * normal_at(seed, tag, (uint64_t)i));
}

// N(mean, std) values rounded through fp16 (the benchmark's fp16 conditioning
// latents), stored as f32 because the decoder interface takes f32 conds.
void itts_synth_normal_f16_as_f32(uint64_t seed, uint64_t tag, float *dst, int64_t n, float mean,
                                  float stdev) {
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < n; ++i)
        dst[i] = h2f(f2h((float)(mean + stdev * normal_at(seed, tag, (uint64_t)i))));
}

// Quantized linear [out, in]: w u32 [out, in/4], scales/biases [out, in/64]
// (uint16 fp16 bits when sb_half, else f32).  Weights ~ N(0, std).
int itts_synth_quant_linear(uint64_t seed, uint64_t tag, int out, int in, float stdev, int sb_half,
                            uint32_t *w, void *scales, void *biases) {
    if (in % 64 != 0 || out <= 0) return 1;
    const int groups = in / 64;
#pragma omp parallel for schedule(static)
    for (int o = 0; o < out; ++o) {
        float vals[64];
        uint8_t *qrow = (uint8_t *)(w + (size_t)o * (in / 4));
        for (int g = 0; g < groups; ++g) {
            float mn = INFINITY, mx = -INFINITY;
            for (int i = 0; i < 64; ++i) {
                uint64_t idx = (uint64_t)o * (uint64_t)in + (uint64_t)(g * 64 + i);
                vals[i] = (float)(stdev * normal_at(seed, tag, idx));
                mn = vals[i] < mn ? vals[i] : mn;
                mx = vals[i] > mx ? vals[i] : mx;
            }
            float s = (mx - mn) / 255.0f;
            if (!(s > 0.0f)) s = 1e-8f;
            float b = mn;
            size_t si = (size_t)o * groups + g;
            if (sb_half) {
                uint16_t sh = f2h(s), bh = f2h(b);
                ((uint16_t *)scales)[si] = sh;
                ((uint16_t *)biases)[si] = bh;
                s = h2f(sh);
                b = h2f(bh);
                if (!(s > 0.0f)) s = 1e-8f;
            } else {
                ((float *)scales)[si] = s;
                ((float *)biases)[si] = b;
            }
            for (int i = 0; i < 64; ++i) {
                float qf = std::nearbyint((vals[i] - b) / s);
                qf = qf < 0.0f ? 0.0f : (qf > 255.0f ? 255.0f : qf);
                qrow[g * 64 + i] = (uint8_t)qf;
            }
        }
    }
    return 0;
}

}  // extern "C"
