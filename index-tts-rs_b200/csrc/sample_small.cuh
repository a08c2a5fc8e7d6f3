// sample_small.cuh -- the sampler of sample_next_token for greedy or top-k <= 64 columns,
// as a device routine shared by the standalone sampler kernel (sample.cu) and the batch-1
// decode-step kernel, which runs it in its last CTA after the logits head (xk_decode.cu).
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
#pragma once
#include <cstdint>

#include "kernels.h"

namespace itts {

static __device__ __forceinline__ uint64_t rng_next_u64(uint64_t &s) {  // sampler.rs:48-54
    s += 0x9E3779B97F4A7C15ULL;
    uint64_t z = s;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
    return z ^ (z >> 31);
}

static __device__ __forceinline__ float rng_next_f32(uint64_t &s) {  // sampler.rs:58-61
    const uint32_t upper = (uint32_t)(rng_next_u64(s) >> 40);
    return __fmul_rn(__uint2float_rn(upper), 1.0f / 16777216.0f);
}

// Total order used for candidate selection: larger key = earlier candidate.
// +0 and -0 compare equal in the reference, so zero is canonicalized.
static __device__ __forceinline__ uint64_t cand_key(float v, int i) {
    uint32_t b = v == 0.0f ? 0u : __float_as_uint(v);
    const uint32_t o = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
    return ((uint64_t)o << 32) | (uint64_t)(0xFFFFFFFFu - (uint32_t)i);
}
static __device__ __forceinline__ int key_id(uint64_t k) { return (int)(0xFFFFFFFFu - (uint32_t)k); }

static __device__ __forceinline__ float exp_cr(float x) { return (float)exp((double)x); }

// The sequential part of sample_next_token after the sorted candidates (ids) and their
// softmax numerators (probs, k of them): sum in candidate order, top-p cut, multinomial
// draw (sampler.rs:250-283).  Advances st.rng when it draws.
static __device__ int draw_candidate(SlotState &st, const int *ids, const float *probs, int k) {
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

// The same by one warp (all 32 lanes call it; lane 0's result is returned to every lane):
// the top-p divisions run on the lanes in parallel (they do not depend on the running sum);
// the sequential sums stay in candidate order on lane 0, reading the candidates in blocks
// of 8 so that the loads are not in the chain of adds.  probs, norm and ids hold kSmallK
// entries (those past k are read but not used); norm is scratch.
static __device__ int draw_candidate_warp(SlotState &st, const int *ids, const float *probs, float *norm, int k,
                                          int lane) {
    float prob_sum = 0.0f;
    if (lane == 0) {
        for (int i0 = 0; i0 < k; i0 += 8) {
            float q[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) q[u] = probs[i0 + u];
#pragma unroll
            for (int u = 0; u < 8; ++u)
                if (i0 + u < k) prob_sum = __fadd_rn(prob_sum, q[u]);
        }
    }
    prob_sum = __shfl_sync(0xffffffffu, prob_sum, 0);
    if (prob_sum <= 0.0f || !isfinite(prob_sum)) return ids[0];  // :250-252
    for (int i = lane; i < k; i += 32) norm[i] = __fdiv_rn(probs[i], prob_sum);
    __syncwarp();
    int token = 0;
    if (lane == 0) {
        const float top_p = st.top_p;
        float cum = 0.0f;
        int active = k;
        bool cut = false;
        for (int i0 = 0; i0 < k && !cut; i0 += 8) {  // :254-264
            float q[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) q[u] = norm[i0 + u];
#pragma unroll
            for (int u = 0; u < 8; ++u) {
                const int i = i0 + u;
                if (i < k && !cut) {
                    if (i > 0 && cum > top_p) {
                        active = i;
                        cut = true;
                    } else {
                        cum = __fadd_rn(cum, q[u]);
                    }
                }
            }
        }
        float active_sum = 0.0f;
        for (int i0 = 0; i0 < active; i0 += 8) {
            float q[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) q[u] = probs[i0 + u];
#pragma unroll
            for (int u = 0; u < 8; ++u)
                if (i0 + u < active) active_sum = __fadd_rn(active_sum, q[u]);
        }
        if (active_sum <= 0.0f || !isfinite(active_sum)) {  // :270-272
            token = ids[0];
        } else {
            uint64_t rs = st.rng;
            const float draw = __fmul_rn(rng_next_f32(rs), active_sum);  // :274
            st.rng = rs;
            int pick = active - 1;  // :283
            float acc = 0.0f;
            bool found = false;
            for (int i0 = 0; i0 < active && !found; i0 += 8) {
                float q[8];
#pragma unroll
                for (int u = 0; u < 8; ++u) q[u] = probs[i0 + u];
#pragma unroll
                for (int u = 0; u < 8; ++u) {
                    const int i = i0 + u;
                    if (i < active && !found) {
                        acc = __fadd_rn(acc, q[u]);
                        if (draw <= acc) {
                            pick = i;
                            found = true;
                        }
                    }
                }
            }
            token = ids[pick];
        }
    }
    return __shfl_sync(0xffffffffu, token, 0);
}

// generate_codes_after's loop step after a sample (sampler.rs:371-389).
static __device__ void loop_step(const SampleArgs &a, SlotState &st, int col, int tok, int n_codes) {
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

// ---------------------------------------------------------------------------
// The sampler for top_k in 1..kSmallK (and greedy columns).  The k-th
// largest scaled logit is found by a 4-pass radix select over 32-bit order keys (kept in
// shared memory; one histogram, updated once per distinct bin of a warp); the candidates are
// the keys above it and the ties at it, the lowest ids first (when a tie group straddles the k-th place, one warp scans
// the ids in order); one warp sorts the candidates (bitonic, in registers) into the
// reference's order (value descending, id ascending).  The tail is the general kernel's.
// The code is kept small (plain loops): it runs once per decode step from cold
// instruction memory.
// ---------------------------------------------------------------------------
constexpr int kSmallK = 64;
constexpr int kSmallMaxLogits = 16384;  // logits per column (one register set of NTH threads)

static __device__ __forceinline__ uint32_t order_key(float v) {
    const uint32_t b = v == 0.0f ? 0u : __float_as_uint(v);
    return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

// Shared memory of the routine besides the logits and keys ([n] floats, then [n] keys).
struct SmallSampleSmem {
    SlotState st;  // the column's slot state, copied in at the start and out at the end
    uint32_t hist[256];
    uint32_t bin, above, count, eq;
    uint64_t cand[kSmallK];
    int ids[kSmallK];
    float probs[kSmallK], norm[kSmallK];
    float bestv[32];
    int besti[32];
    int token;
};

// Samples batch column `col` with NTH threads (tid 0..NTH-1, a multiple of 32, at least
// 256); sync() is a barrier over exactly those threads.  lgs holds 3 n_logits words: the
// scaled logits, their order keys, and the keys of the first radix pass's selected bin.
template <int NTH, class Sync>
static __device__ void sample_small_body(const SampleArgs &a, int col, SmallSampleSmem &sm, float *lgs, int tid,
                                         Sync sync) {
    uint32_t *hist = sm.hist;
    uint32_t &s_bin = sm.bin, &s_above = sm.above, &s_count = sm.count, &s_eq = sm.eq;
    uint64_t *cand = sm.cand;
    int *s_ids = sm.ids;
    float *s_probs = sm.probs, *s_norm = sm.norm, *s_bestv = sm.bestv;
    int *s_besti = sm.besti;
    int &s_token = sm.token;
    SlotState &gst = a.slots[a.batch_slot[col]];
    if (!gst.active) return;  // (every thread reads the same flag)
    const int n = a.n_logits, lane = tid & 31, warp = tid >> 5;
    uint32_t *keys = reinterpret_cast<uint32_t *>(lgs + n), *bin_keys = keys + n;
    float *row = a.logits + (size_t)col * a.ld_logits;
    // this thread's logits i = tid + NTH j, all loads in flight at once; the slot state into
    // shared memory meanwhile
    constexpr int E = (kSmallMaxLogits + NTH - 1) / NTH;
    float v[E];
#pragma unroll
    for (int j = 0; j < E; ++j) {
        const int i = tid + NTH * j;
        v[j] = i < n ? row[i] : 0.0f;
    }
    constexpr int SW = (int)(sizeof(SlotState) / 8);
    static_assert(sizeof(SlotState) % 8 == 0, "slot state copied in 8-byte words");
    if (tid < SW) reinterpret_cast<uint64_t *>(&sm.st)[tid] = reinterpret_cast<const uint64_t *>(&gst)[tid];
    sync();
    SlotState &st = sm.st;
    const int n_codes = st.n_codes;
    const bool mask_stop = n_codes < st.min_codes && kStopMel < n;
    const float pen = st.rep_penalty;
    const bool do_pen = fabsf(__fsub_rn(pen, 1.0f)) > 1.1920929e-7f;
#pragma unroll
    for (int j = 0; j < E; ++j) {  // STOP mask, repetition penalty (sampler.rs:138-157)
        const int i = tid + NTH * j;
        if (i < n) {
            float x = (mask_stop && i == kStopMel) ? -INFINITY : v[j];
            if (do_pen && i < kBitsetWords * 64 && ((st.seen[i >> 6] >> (i & 63)) & 1ULL))
                x = x < 0.0f ? __fmul_rn(x, pen) : __fdiv_rn(x, pen);
            v[j] = x;
            if (a.write_back) row[i] = x;
        }
    }

    if (st.greedy) {  // argmax_finite (sampler.rs:395-405)
        float bv = -INFINITY;
        int bi = 0x7FFFFFFF;
#pragma unroll
        for (int j = 0; j < E; ++j) {
            const int i = tid + NTH * j;
            if (i < n && isfinite(v[j]) && (bi == 0x7FFFFFFF || v[j] > bv)) { bv = v[j]; bi = i; }
        }
        for (int off = 16; off > 0; off >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, off);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, off);
            if (oi != 0x7FFFFFFF && (bi == 0x7FFFFFFF || ov > bv || (ov == bv && oi < bi))) { bv = ov; bi = oi; }
        }
        if (lane == 0) { s_bestv[warp] = bv; s_besti[warp] = bi; }
        sync();
        if (tid == 0) {
            float val = -INFINITY;
            int id = 0x7FFFFFFF;
            for (int w = 0; w < NTH / 32; ++w) {
                const int oi = s_besti[w];
                const float ov = s_bestv[w];
                if (oi != 0x7FFFFFFF && (id == 0x7FFFFFFF || ov > val || (ov == val && oi < id))) { val = ov; id = oi; }
            }
            s_token = id == 0x7FFFFFFF ? 0 : id;
        }
        sync();
    } else {
        const float inv_temp = __fdiv_rn(1.0f, st.temperature);  // sampler.rs:210
        uint32_t kr[E];  // this thread's order keys (registers; 0 past n, below every key in use)
#pragma unroll
        for (int j = 0; j < E; ++j) {
            const int i = tid + NTH * j;
            kr[j] = 0u;
            if (i < n) {
                const float sv = isfinite(v[j]) ? __fmul_rn(v[j], inv_temp) : -INFINITY;
                lgs[i] = sv;
                kr[j] = order_key(sv);
                keys[i] = kr[j];
            }
        }
        const uint32_t raw_k = st.top_k;
        const int k = min(kSmallK, (raw_k == 0 || raw_k >= (uint32_t)n) ? n : (int)raw_k);  // :221-226
        uint32_t prefix = 0, pmask = 0, remaining = (uint32_t)k;
        // the bin holding the k-th largest key among the keys matching (prefix, pmask) at this
        // digit: s_bin, s_above (keys in higher bins) and s_eq (keys in the bin)
        auto pick_bin = [&]() {
            sync();
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
            sync();
        };
        // one shared-memory atomic per distinct bin of the warp (most keys share a few bins)
        auto count = [&](uint32_t key, bool in, int shift) {
            const uint32_t bin = in && (key & pmask) == prefix ? (key >> shift) & 0xFFu : 0x100u;
            const unsigned peers = __match_any_sync(0xffffffffu, bin);
            if (bin != 0x100u && lane == __ffs(peers) - 1) atomicAdd(&hist[bin], (uint32_t)__popc(peers));
        };
        // radix select of the k-th largest key: the first digit over every key (registers),
        // then the keys of its bin are gathered and the other three digits run over them only
        if (tid < 256) hist[tid] = 0;
        if (tid == 0) s_count = 0;
        sync();
#pragma unroll
        for (int j = 0; j < E; ++j)
            if (j * NTH < n) count(kr[j], tid + NTH * j < n, 24);  // (uniform trip count)
        pick_bin();
        prefix = s_bin << 24;
        pmask = 0xFF000000u;
        remaining -= s_above;
        const int m = (int)s_eq;  // keys in the selected bin
#pragma unroll
        for (int j = 0; j < E; ++j) {  // gather them (any order: only their digits are counted)
            if (j * NTH >= n) break;
            const bool in = tid + NTH * j < n && (kr[j] & pmask) == prefix;
            const unsigned bal = __ballot_sync(0xffffffffu, in);
            uint32_t base = 0;
            if (lane == 0 && bal) base = atomicAdd(&s_count, (uint32_t)__popc(bal));
            base = __shfl_sync(0xffffffffu, base, 0);
            if (in) bin_keys[base + __popc(bal & ((1u << lane) - 1u))] = kr[j];
        }
        for (int shift = 16; shift >= 0; shift -= 8) {
            if (tid < 256) hist[tid] = 0;
            sync();  // also: the gathered keys written / the previous pass's s_bin read
            for (int t0 = 0; t0 < m; t0 += NTH) count(t0 + tid < m ? bin_keys[t0 + tid] : 0u, t0 + tid < m, shift);
            pick_bin();
            prefix |= s_bin << shift;
            pmask |= 0xFFu << shift;
            remaining -= s_above;
        }
        // after the last pass s_eq counts the keys equal to the threshold; all of them are
        // candidates unless the group straddles the k-th place
        const bool all_ties = remaining == s_eq;
        if (tid == 0) s_count = 0;
        sync();
        for (int i = tid; i < n; i += NTH) {
            const uint32_t key = keys[i];
            if (key > prefix || (all_ties && key == prefix)) cand[atomicAdd(&s_count, 1u)] = cand_key(lgs[i], i);
        }
        sync();
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
        sync();
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
            const int tok = draw_candidate_warp(st, s_ids, s_probs, s_norm, k, lane);
            if (lane == 0) s_token = tok;
        }
        sync();
    }
    if (tid == 0) loop_step(a, st, col, s_token, n_codes);
    sync();
    if (tid < SW) reinterpret_cast<uint64_t *>(&gst)[tid] = reinterpret_cast<const uint64_t *>(&sm.st)[tid];
}

}  // namespace itts
