// sample.cu -- on-device sampler and decode-loop bookkeeping.
//
// Restates crates/core/src/models/sampler.rs bit for bit in IEEE fp32:
//   repetition penalty over the seen bitset (:138-157), greedy argmax_finite
//   (:395-405), multiply by 1/temperature (:210-219), top-k (:221-231), descending
//   sort, softmax numerators exp(l - max) (:233-248), top-p cut (:254-264),
//   draw = u * active_sum and first draw <= acc (:274-283), and the loop step of
//   generate_codes_after (:371-389).  All arithmetic uses the _rn intrinsics so no
//   multiply-add is contracted; sums are sequential in candidate order.
// Order among equal scaled logits: lower token id first (the reference's unstable
// select/sort leaves it unspecified).  exp() is the correctly rounded
// (float)exp((double)x).
#include <cstdint>

#include "itts_gpt.h"
#include "kernels.h"

namespace itts {

constexpr int kSampleThreads = 1024;
constexpr int kMaxSampleLogits = 16384;

__device__ __forceinline__ uint64_t rng_next_u64(uint64_t &s) {  // sampler.rs:48-54
    s += 0x9E3779B97F4A7C15ULL;
    uint64_t z = s;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
    return z ^ (z >> 31);
}

__device__ __forceinline__ float rng_next_f32(uint64_t &s) {  // sampler.rs:58-61
    const uint32_t upper = (uint32_t)(rng_next_u64(s) >> 40);
    return __fmul_rn(__uint2float_rn(upper), 1.0f / 16777216.0f);
}

// Total order used for candidate selection: larger key = earlier candidate.
// +0 and -0 compare equal in the reference, so zero is canonicalized.
__device__ __forceinline__ uint64_t cand_key(float v, int i) {
    uint32_t b = v == 0.0f ? 0u : __float_as_uint(v);
    const uint32_t o = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
    return ((uint64_t)o << 32) | (uint64_t)(0xFFFFFFFFu - (uint32_t)i);
}
__device__ __forceinline__ int key_id(uint64_t k) { return (int)(0xFFFFFFFFu - (uint32_t)k); }

__device__ __forceinline__ float exp_cr(float x) { return (float)exp((double)x); }

// The sequential part of sample_next_token after the sorted candidates (ids) and their
// softmax numerators (probs, k of them): sum in candidate order, top-p cut, multinomial
// draw (sampler.rs:250-283).  Advances st.rng when it draws.
__device__ int draw_candidate(SlotState &st, const int *ids, const float *probs, int k) {
    float prob_sum = 0.0f;
    for (int i = 0; i < k; ++i) prob_sum = __fadd_rn(prob_sum, probs[i]);
    if (prob_sum <= 0.0f || !isfinite(prob_sum)) return ids[0];  // :250-252
    const float top_p = st.top_p;
    float cum = 0.0f;
    int active = k;
    for (int i = 0; i < k; ++i) {  // :254-264
        const float norm_p = __fdiv_rn(probs[i], prob_sum);
        if (i > 0 && cum > top_p) { active = i; break; }
        cum = __fadd_rn(cum, norm_p);
    }
    float active_sum = 0.0f;
    for (int i = 0; i < active; ++i) active_sum = __fadd_rn(active_sum, probs[i]);
    if (active_sum <= 0.0f || !isfinite(active_sum)) return ids[0];  // :270-272
    uint64_t rs = st.rng;
    const float draw = __fmul_rn(rng_next_f32(rs), active_sum);  // :274
    st.rng = rs;
    int token = ids[active - 1];  // :283
    float acc = 0.0f;
    for (int i = 0; i < active; ++i) {
        acc = __fadd_rn(acc, probs[i]);
        if (draw <= acc) { token = ids[i]; break; }
    }
    return token;
}

// generate_codes_after's loop step after a sample (sampler.rs:371-389).
__device__ void loop_step(const SampleArgs &a, SlotState &st, int col, int tok, int n_codes) {
    if (a.token_out) a.token_out[col] = tok;
    if (a.after_forward) st.valid_len += 1;
    const int step = st.step;
    st.step = step + 1;
    if (tok == kStopMel) {
        st.active = 0;
    } else {
        if (a.codes) a.codes[(size_t)a.batch_slot[col] * a.codes_stride + n_codes] = tok;
        st.n_codes = n_codes + 1;
        if (tok >= 0 && tok < kBitsetWords * 64) st.seen[tok >> 6] |= 1ULL << (tok & 63);
        if (step + 1 >= st.max_steps) {
            st.active = 0;
        } else if (st.valid_len + 1 > st.max_seq) {  // gpt.rs:157-165 on the next step
            st.error = 1;
            st.active = 0;
        } else {
            st.tok = tok;
            st.pos = st.n_prior + step + 2;  // sampler.rs:386
        }
    }
}

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

// ---------------------------------------------------------------------------
// The same sampler for top_k in 1..kSmallK (and greedy columns), 1,024 threads.  The k-th
// largest scaled logit is found by a 4-pass radix select over 32-bit order keys (kept in
// shared memory; one histogram, updated once per distinct bin of a warp); the candidates are
// the keys above it and the ties at it, the lowest ids first (when a tie group straddles the k-th place, one warp scans
// the ids in order); one warp sorts the candidates (bitonic, in registers) into the
// reference's order (value descending, id ascending).  The tail is the general kernel's.
// The code is kept small (plain loops): it runs once per decode step from cold
// instruction memory.
// ---------------------------------------------------------------------------
constexpr int kSmallK = 64;
constexpr int kSmallThreads = 1024;

__device__ __forceinline__ uint32_t order_key(float v) {
    const uint32_t b = v == 0.0f ? 0u : __float_as_uint(v);
    return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

__global__ void __launch_bounds__(kSmallThreads) sample_small_kernel(SampleArgs a) {
    extern __shared__ __align__(16) float lgs[];  // [n] logits, then [n] order keys
    __shared__ uint32_t hist[256];
    __shared__ uint32_t s_bin, s_above, s_count, s_eq;
    __shared__ uint64_t cand[kSmallK];
    __shared__ int s_ids[kSmallK];
    __shared__ float s_probs[kSmallK];
    __shared__ float s_bestv[kSmallThreads / 32];
    __shared__ int s_besti[kSmallThreads / 32];
    __shared__ int s_token;

    const int col = blockIdx.x;
    SlotState &st = a.slots[a.batch_slot[col]];
    if (!st.active) return;
    const int n = a.n_logits, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    uint32_t *keys = reinterpret_cast<uint32_t *>(lgs + n);
    float *row = a.logits + (size_t)col * a.ld_logits;
    const int n_codes = st.n_codes;
    const bool mask_stop = n_codes < st.min_codes && kStopMel < n;
    const float pen = st.rep_penalty;
    const bool do_pen = fabsf(__fsub_rn(pen, 1.0f)) > 1.1920929e-7f;
#pragma unroll 4
    for (int i = tid; i < n; i += kSmallThreads) {  // STOP mask, repetition penalty (sampler.rs:138-157)
        float v = (mask_stop && i == kStopMel) ? -INFINITY : row[i];
        if (do_pen && i < kBitsetWords * 64 && ((st.seen[i >> 6] >> (i & 63)) & 1ULL))
            v = v < 0.0f ? __fmul_rn(v, pen) : __fdiv_rn(v, pen);
        lgs[i] = v;
        if (a.write_back) row[i] = v;
    }
    __syncthreads();

    if (st.greedy) {  // argmax_finite (sampler.rs:395-405)
        float bv = -INFINITY;
        int bi = 0x7FFFFFFF;
        for (int i = tid; i < n; i += kSmallThreads) {
            const float v = lgs[i];
            if (isfinite(v) && (bi == 0x7FFFFFFF || v > bv)) { bv = v; bi = i; }
        }
        for (int off = 16; off > 0; off >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, off);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, off);
            if (oi != 0x7FFFFFFF && (bi == 0x7FFFFFFF || ov > bv || (ov == bv && oi < bi))) { bv = ov; bi = oi; }
        }
        if (lane == 0) { s_bestv[warp] = bv; s_besti[warp] = bi; }
        __syncthreads();
        if (tid == 0) {
            float val = -INFINITY;
            int id = 0x7FFFFFFF;
            for (int w = 0; w < kSmallThreads / 32; ++w) {
                const int oi = s_besti[w];
                const float ov = s_bestv[w];
                if (oi != 0x7FFFFFFF && (id == 0x7FFFFFFF || ov > val || (ov == val && oi < id))) { val = ov; id = oi; }
            }
            s_token = id == 0x7FFFFFFF ? 0 : id;
        }
        __syncthreads();
    } else {
        const float inv_temp = __fdiv_rn(1.0f, st.temperature);  // sampler.rs:210
        for (int i = tid; i < n; i += kSmallThreads) {
            const float v = lgs[i];
            const float sv = isfinite(v) ? __fmul_rn(v, inv_temp) : -INFINITY;
            lgs[i] = sv;
            keys[i] = order_key(sv);
        }
        const uint32_t raw_k = st.top_k;
        const int k = min(kSmallK, (raw_k == 0 || raw_k >= (uint32_t)n) ? n : (int)raw_k);  // :221-226
        uint32_t prefix = 0, pmask = 0, remaining = (uint32_t)k;
        for (int shift = 24; shift >= 0; shift -= 8) {  // radix select of the k-th largest key
            if (tid < 256) hist[tid] = 0;
            __syncthreads();  // also: keys written / the previous pass's s_bin read
            for (int i0 = 0; i0 < n; i0 += kSmallThreads) {  // (uniform trip count: warp-wide match)
                const int i = i0 + tid;
                uint32_t bin = 0x100u;  // no bin: out of range or outside the prefix
                if (i < n) {
                    const uint32_t key = keys[i];
                    if ((key & pmask) == prefix) bin = (key >> shift) & 0xFFu;
                }
                // one shared-memory atomic per distinct bin of the warp (most keys share a few
                // bins in the first passes)
                const unsigned peers = __match_any_sync(0xffffffffu, bin);
                if (bin != 0x100u && lane == __ffs(peers) - 1) atomicAdd(&hist[bin], (uint32_t)__popc(peers));
            }
            __syncthreads();
            if (warp == 0) {  // lane L holds bins 255-8L .. 248-8L (top-down order)
                uint32_t c[8], sum = 0;
#pragma unroll
                for (int j = 0; j < 8; ++j) { c[j] = hist[255 - 8 * lane - j]; sum += c[j]; }
                uint32_t incl = sum;
                for (int off = 1; off < 32; off <<= 1) {
                    const uint32_t o = __shfl_up_sync(0xffffffffu, incl, off);
                    if (lane >= off) incl += o;
                }
                const uint32_t excl = incl - sum;
                if (excl < remaining && remaining <= incl) {
                    uint32_t cum = excl;
                    for (int j = 0; j < 8; ++j) {
                        if (cum + c[j] >= remaining) {
                            s_bin = 255 - 8 * lane - j;
                            s_above = cum;
                            s_eq = c[j];
                            break;
                        }
                        cum += c[j];
                    }
                }
            }
            __syncthreads();
            prefix |= s_bin << shift;
            pmask |= 0xFFu << shift;
            remaining -= s_above;
        }
        // after the last pass s_eq counts the keys equal to the threshold; all of them are
        // candidates unless the group straddles the k-th place
        const bool all_ties = remaining == s_eq;
        if (tid == 0) s_count = 0;
        __syncthreads();
        for (int i = tid; i < n; i += kSmallThreads) {
            const uint32_t key = keys[i];
            if (key > prefix || (all_ties && key == prefix)) cand[atomicAdd(&s_count, 1u)] = cand_key(lgs[i], i);
        }
        __syncthreads();
        if (!all_ties && warp == 0) {  // the `remaining` lowest ids among the ties, in id order
            uint32_t base = s_count, left = remaining;
            for (int i0 = 0; i0 < n && left > 0; i0 += 32) {
                const int i = i0 + lane;
                const bool tie = i < n && keys[i] == prefix;
                const unsigned m = __ballot_sync(0xffffffffu, tie);
                const uint32_t rank = __popc(m & ((1u << lane) - 1u));
                if (tie && rank < left) cand[base + rank] = cand_key(lgs[i], i);
                const uint32_t took = min((uint32_t)__popc(m), left);
                base += took;
                left -= took;
            }
        }
        __syncthreads();
        if (warp == 0) {  // bitonic sort of the k candidates, descending: element e = lane + 32 r
            uint64_t x[2];
            for (int r = 0; r < 2; ++r) x[r] = lane + 32 * r < k ? cand[lane + 32 * r] : 0ULL;
            for (int size = 2; size <= 64; size <<= 1)
                for (int stride = size >> 1; stride > 0; stride >>= 1) {
                    const uint64_t y0 = stride == 32 ? x[1] : __shfl_xor_sync(0xffffffffu, x[0], stride);
                    const uint64_t y1 = stride == 32 ? x[0] : __shfl_xor_sync(0xffffffffu, x[1], stride);
                    const uint64_t yy[2] = {y0, y1};
                    for (int r = 0; r < 2; ++r) {
                        const int e = lane + 32 * r;
                        const bool desc = (e & size) == 0, lower = (e & stride) == 0;
                        const uint64_t hi = x[r] > yy[r] ? x[r] : yy[r], lo = x[r] > yy[r] ? yy[r] : x[r];
                        x[r] = desc == lower ? hi : lo;
                    }
                }
            // ids and softmax numerators (sampler.rs:233-248)
            const float v0 = lgs[key_id(__shfl_sync(0xffffffffu, x[0], 0))];
            const float mx = isfinite(v0) ? v0 : 0.0f;
            for (int r = 0; r < 2; ++r) {
                const int e = lane + 32 * r;
                if (e < k) {
                    const int id = key_id(x[r]);
                    const float vv = lgs[id];
                    s_ids[e] = id;
                    s_probs[e] = isfinite(vv) ? exp_cr(__fsub_rn(vv, mx)) : 0.0f;
                }
            }
            __syncwarp();
            if (lane == 0) s_token = draw_candidate(st, s_ids, s_probs, k);
        }
        __syncthreads();
    }
    if (tid == 0) loop_step(a, st, col, s_token, n_codes);
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
        sample_small_kernel<<<a.nb, kSmallThreads, (size_t)a.n_logits * 2 * sizeof(float), st>>>(a);
    else
        sample_kernel<<<a.nb, kSampleThreads, sample_smem_bytes(a.n_logits), st>>>(a);
}

void kernels_init_sample() {
    cudaFuncSetAttribute(sample_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)sample_smem_bytes(kMaxSampleLogits));
    cudaFuncSetAttribute(sample_small_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)(kMaxSampleLogits * 2 * sizeof(float)));
}

}  // namespace itts
