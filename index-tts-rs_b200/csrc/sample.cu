// sample.cu -- on-device sampler kernels and decode-loop bookkeeping: the general kernel
// (any top-k, full sort of the candidates) and the small-k kernel around the routine of
// sample_small.cuh.  Both restate crates/core/src/models/sampler.rs:191-284 bit for bit in
// IEEE fp32 (the helpers, the exact order of operations and the tie order are in
// sample_small.cuh).
#include <cstdint>

#include "itts_gpt.h"
#include "kernels.h"
#include "sample_small.cuh"

namespace itts {

constexpr int kSampleThreads = 1024;
constexpr int kMaxSampleLogits = 16384;
static_assert(kMaxSampleLogits == kSmallMaxLogits, "one logit limit for both sampler kernels");

__global__ void __launch_bounds__(kSampleThreads) sample_kernel(SampleArgs a) {
    extern __shared__ __align__(16) unsigned char sm_raw[];
    __shared__ uint32_t hist[256];
    __shared__ uint32_t s_bin, s_above, s_count;
    __shared__ float s_bestv[32];
    __shared__ int s_besti[32];
    __shared__ int s_token;
    __shared__ float s_max;

    const int col = blockIdx.x;
    SlotState &st = a.slots[a.batch_slot[col]];
    if (!st.active) return;
    const int n = a.n_logits, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    float *lg = reinterpret_cast<float *>(sm_raw);
    uint64_t *keys = reinterpret_cast<uint64_t *>(sm_raw + ((size_t)((n + 1) & ~1) * 4));
    float *row = a.logits + (size_t)col * a.ld_logits;

    const int n_codes = st.n_codes;
    const bool mask_stop = n_codes < st.min_codes && kStopMel < n;
    for (int i = tid; i < n; i += kSampleThreads) lg[i] = (mask_stop && i == kStopMel) ? -INFINITY : row[i];
    __syncthreads();

    // repetition penalty (sampler.rs:138-157)
    const float pen = st.rep_penalty;
    if (fabsf(__fsub_rn(pen, 1.0f)) > 1.1920929e-7f) {
        for (int i = tid; i < n && i < kBitsetWords * 64; i += kSampleThreads) {
            if ((st.seen[i >> 6] >> (i & 63)) & 1ULL) {
                const float v = lg[i];
                lg[i] = v < 0.0f ? __fmul_rn(v, pen) : __fdiv_rn(v, pen);
            }
        }
    }
    __syncthreads();
    if (a.write_back)
        for (int i = tid; i < n; i += kSampleThreads) row[i] = lg[i];

    if (st.greedy) {  // argmax_finite (sampler.rs:395-405)
        float bv = -INFINITY;
        int bi = 0x7FFFFFFF;
        for (int i = tid; i < n; i += kSampleThreads) {
            const float v = lg[i];
            if (isfinite(v) && (bi == 0x7FFFFFFF || v > bv)) { bv = v; bi = i; }
        }
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, off);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, off);
            if (oi != 0x7FFFFFFF && (bi == 0x7FFFFFFF || ov > bv || (ov == bv && oi < bi))) { bv = ov; bi = oi; }
        }
        if (lane == 0) { s_bestv[warp] = bv; s_besti[warp] = bi; }
        __syncthreads();
        if (tid == 0) {
            float v = -INFINITY;
            int id = 0x7FFFFFFF;
            for (int w = 0; w < kSampleThreads / 32; ++w) {
                const int oi = s_besti[w];
                const float ov = s_bestv[w];
                if (oi != 0x7FFFFFFF && (id == 0x7FFFFFFF || ov > v || (ov == v && oi < id))) { v = ov; id = oi; }
            }
            s_token = id == 0x7FFFFFFF ? 0 : id;
        }
        __syncthreads();
    } else {
        const float inv_temp = __fdiv_rn(1.0f, st.temperature);  // sampler.rs:210
        for (int i = tid; i < n; i += kSampleThreads) {
            const float v = lg[i];
            lg[i] = isfinite(v) ? __fmul_rn(v, inv_temp) : -INFINITY;
        }
        const uint32_t raw_k = st.top_k;
        const int k = (raw_k == 0 || raw_k >= (uint32_t)n) ? n : (int)raw_k;  // :221-226
        int P = 1;
        while (P < k) P <<= 1;
        __syncthreads();

        // radix-select the k-th largest key (keys are unique: value, then id)
        uint64_t prefix = 0, pmask = 0;
        if (k < n) {
            uint32_t remaining = (uint32_t)k;
            const int n_iter = (n + kSampleThreads - 1) / kSampleThreads;
            for (int digit = 7; digit >= 0; --digit) {
                const int shift = digit * 8;
                if (tid < 256) hist[tid] = 0;
                __syncthreads();
                for (int it = 0; it < n_iter; ++it) {
                    const int i = tid + it * kSampleThreads;
                    uint64_t key = 0;
                    bool match = false;
                    if (i < n) {
                        key = cand_key(lg[i], i);
                        match = (key & pmask) == prefix;
                    }
                    const uint32_t bin = (uint32_t)(key >> shift) & 0xFFu;
                    const unsigned act = __ballot_sync(0xffffffffu, match);
                    if (match) {
                        const unsigned peers = __match_any_sync(act, bin);
                        if (lane == __ffs(peers) - 1) atomicAdd(&hist[bin], (uint32_t)__popc(peers));
                    }
                }
                __syncthreads();
                if (warp == 0) {
                    // lane L holds bins 255-8L .. 248-8L (top-down order)
                    uint32_t c[8], tot = 0;
#pragma unroll
                    for (int j = 0; j < 8; ++j) { c[j] = hist[255 - 8 * lane - j]; tot += c[j]; }
                    uint32_t incl = tot;
#pragma unroll
                    for (int off = 1; off < 32; off <<= 1) {
                        const uint32_t o = __shfl_up_sync(0xffffffffu, incl, off);
                        if (lane >= off) incl += o;
                    }
                    const uint32_t excl = incl - tot;
                    if (excl < remaining && remaining <= incl) {
                        uint32_t cum = excl;
#pragma unroll
                        for (int j = 0; j < 8; ++j) {
                            if (cum + c[j] >= remaining) { s_bin = 255 - 8 * lane - j; s_above = cum; break; }
                            cum += c[j];
                        }
                    }
                }
                __syncthreads();
                prefix |= (uint64_t)s_bin << shift;
                pmask |= 0xFFULL << shift;
                remaining -= s_above;
                __syncthreads();
            }
        }
        // gather the k candidates (key >= k-th key), pad to P with 0 keys
        if (tid == 0) s_count = 0;
        __syncthreads();
        {
            const int n_iter = (n + kSampleThreads - 1) / kSampleThreads;
            for (int it = 0; it < n_iter; ++it) {
                const int i = tid + it * kSampleThreads;
                uint64_t key = 0;
                bool take = false;
                if (i < n) {
                    key = cand_key(lg[i], i);
                    take = k == n || key >= prefix;
                }
                const unsigned bal = __ballot_sync(0xffffffffu, take);
                uint32_t base = 0;
                if (lane == 0 && bal) base = atomicAdd(&s_count, (uint32_t)__popc(bal));
                base = __shfl_sync(0xffffffffu, base, 0);
                if (take) keys[base + __popc(bal & ((1u << lane) - 1))] = key;
            }
        }
        __syncthreads();
        for (int i = k + tid; i < P; i += kSampleThreads) keys[i] = 0;
        // bitonic sort, descending
        for (int size = 2; size <= P; size <<= 1) {
            for (int stride = size >> 1; stride > 0; stride >>= 1) {
                __syncthreads();
                for (int i = tid; i < (P >> 1); i += kSampleThreads) {
                    const int pos = 2 * i - (i & (stride - 1));
                    const int j = pos + stride;
                    const bool desc = (pos & size) == 0;
                    const uint64_t x = keys[pos], y = keys[j];
                    if ((x < y) == desc) { keys[pos] = y; keys[j] = x; }
                }
            }
        }
        __syncthreads();
        // ids / numerators (sampler.rs:233-248), reusing the key storage
        int my_id[kMaxSampleLogits / kSampleThreads];
        float my_v[kMaxSampleLogits / kSampleThreads];
#pragma unroll
        for (int r = 0; r < kMaxSampleLogits / kSampleThreads; ++r) {
            const int i = tid + r * kSampleThreads;
            my_id[r] = 0;
            my_v[r] = 0.f;
            if (i < k) { my_id[r] = key_id(keys[i]); my_v[r] = lg[my_id[r]]; }
        }
        if (tid == 0) {
            const float v0 = lg[key_id(keys[0])];
            s_max = isfinite(v0) ? v0 : 0.0f;
        }
        __syncthreads();
        int *ids = reinterpret_cast<int *>(keys);
        float *probs = reinterpret_cast<float *>(ids + P);
        const float mx = s_max;
#pragma unroll
        for (int r = 0; r < kMaxSampleLogits / kSampleThreads; ++r) {
            const int i = tid + r * kSampleThreads;
            if (i < k) {
                ids[i] = my_id[r];
                probs[i] = isfinite(my_v[r]) ? exp_cr(__fsub_rn(my_v[r], mx)) : 0.0f;
            }
        }
        __syncthreads();
        if (tid == 0) s_token = draw_candidate(st, ids, probs, k);
        __syncthreads();
    }

    if (tid == 0) loop_step(a, st, col, s_token, n_codes);
}

// The standalone kernel of the small-k sampler (sample_small.cuh), one CTA per column.
constexpr int kSmallThreads = 1024;

__global__ void __launch_bounds__(kSmallThreads) sample_small_kernel(SampleArgs a) {
    extern __shared__ __align__(16) float lgs[];  // [n] logits, [n] order keys, [n] keys of one bin
    __shared__ SmallSampleSmem sm;
    sample_small_body<kSmallThreads>(a, blockIdx.x, sm, lgs, threadIdx.x, [] { __syncthreads(); });
}

bool sample_small_ok(const itts_sampling_params &p, int n_logits) {
    return p.greedy || (p.top_k >= 1 && p.top_k <= (uint32_t)kSmallK && p.top_k < (uint32_t)n_logits);
}

static size_t sample_smem_bytes(int n) {
    int P = 1;
    while (P < n) P <<= 1;
    return (size_t)((n + 1) & ~1) * 4 + (size_t)P * 8;
}

void launch_sample(const SampleArgs &a, cudaStream_t st) {
    if (a.small_k)
        sample_small_kernel<<<a.nb, kSmallThreads, (size_t)a.n_logits * 3 * sizeof(float), st>>>(a);
    else
        sample_kernel<<<a.nb, kSampleThreads, sample_smem_bytes(a.n_logits), st>>>(a);
}

void kernels_init_sample() {
    // the largest shared-memory carve-out, like the decode step's other kernels
    cudaFuncSetAttribute(sample_kernel, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
    cudaFuncSetAttribute(sample_small_kernel, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
    cudaFuncSetAttribute(sample_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)sample_smem_bytes(kMaxSampleLogits));
    cudaFuncSetAttribute(sample_small_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)(kMaxSampleLogits * 3 * sizeof(float)));
}

}  // namespace itts
