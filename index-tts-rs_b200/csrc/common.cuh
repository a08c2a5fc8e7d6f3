// common.cuh -- device-side data layout shared by the decoder kernels.
//
// HBM layout (one itts_gpt per device):
//   quantized linear: tiled int8 weights + (scale, offset) pairs, see mk.h; bias f32 [out]
//   LayerNorm weight/bias, embedding tables: f32 as in the checkpoint.
//   KV cache (itts_kv): K and V each fp16 [layer][slot][head][max_seq][64], so one
//   head's keys are contiguous 128-byte rows for the split-K decode attention.
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace itts {

constexpr int kHeadDim = 64;
constexpr int kGroup = 64;
constexpr int kBitsetWords = 129;
constexpr int kStartMel = 8192;
constexpr int kStopMel = 8193;
constexpr int kStartText = 0;
constexpr int kStopText = 1;
constexpr float kAttnScale = 0.125f;  // 64^-0.5 (gpt.rs:67)
constexpr float kNormEps = 1e-5f;     // gpt.rs:42

// Per-request decode state, resident in HBM so a captured decode-step graph can
// replay unchanged: the sampler kernel writes the next token / position here and
// the next replay's embedding kernel reads them.
struct SlotState {
    int32_t tok;        // mel token fed at the next decode step
    int32_t pos;        // its mel position index (prior + step + 2, sampler.rs:386)
    int32_t valid_len;  // KV positions filled
    int32_t active;     // 1 while generating
    int32_t n_codes;    // codes emitted
    int32_t max_steps;  // samples allowed (sampler.rs:348-349)
    int32_t min_codes;  // STOP masked while n_codes < min_codes (sampler.rs:372-376)
    int32_t step;       // samples drawn so far
    int32_t n_prior;
    int32_t error;      // nonzero: KV capacity exceeded (gpt.rs:157-165)
    int32_t greedy;
    uint32_t top_k;
    float top_p;
    float temperature;
    float rep_penalty;
    int32_t max_seq;
    uint64_t rng;                 // SamplerRng state (sampler.rs:24-26)
    uint64_t seen[kBitsetWords];  // SeenTokenBitSet (sampler.rs:67-69)
};

// Streaming 128-bit load of weights read once per step (no L1 allocation).
__device__ __forceinline__ uint4 ld_stream(const void *p) {
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
    return r;
}

// Exact u8 -> f32: the byte is placed in the low mantissa bits of 2^23, and
// 2^23 is subtracted (both steps exact).
__device__ __forceinline__ float byte_to_float(uint32_t word, int k) {
    uint32_t bits = __byte_perm(word, 0x4B000000u, 0x7440u + (uint32_t)k);
    return __uint_as_float(bits) - 8388608.0f;
}

__device__ __forceinline__ float gelu_tanh(float x) {
    const float k = 0.7978845608028654f;  // sqrt(2/pi)
    return 0.5f * x * (1.0f + tanhf(k * (x + 0.044715f * x * x * x)));
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ size_t kv_index(int layer, int slot, int head, int pos, int n_slots,
                                           int n_heads, int max_seq) {
    return ((((size_t)layer * n_slots + slot) * n_heads + head) * max_seq + pos) * kHeadDim;
}

}  // namespace itts
