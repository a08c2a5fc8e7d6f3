// decode.cu -- decode-step kernels: int8 group-64 affine GEMV with fused
// LayerNorm prologue and bias / GELU / residual / KV-scatter epilogues, split-K
// flash-decode attention over the fp16 KV cache, and the step embedding.
//
// Reference semantics: Gpt2Block::forward (crates/core/src/models/gpt.rs:325-384),
// QuantizedLinear::forward (gpt.rs:252-263, MLX quantized_matmul affine g64/8-bit),
// Gpt::step (gpt.rs:706-754).
#include <cstdio>

#include "kernels.h"

namespace itts {

// ---------------------------------------------------------------------------
// GEMV: y[b, o] = sum_i xn[b, i] * (s[o,g] * q[o,i] + z[o,g]) + bias[o]
// computed per 16-byte chunk c of a row as  s * (x . q) + z * (sum x)  with the
// chunk sums of x precomputed once per CTA.  One warp owns two adjacent rows;
// lanes stride over 16-byte chunks (coalesced 512 B per warp load).
// ---------------------------------------------------------------------------
struct GemvParams {
    QLinear W;
    bool sb_half;
    const float *x;
    float *y;
    int ncols;  // batch columns (<= NB)
    int col0;   // first batch column of this launch
    int ln_mode;
    const float *ln_w, *ln_b, *ln2_w, *ln2_b;
    // EPI_QKV
    float *q_out;
    __half *k_cache, *v_cache;
    const SlotState *slots;
    const int *batch_slot;
    int n_slots, n_heads, max_seq, layer, d;
};

template <int NB>
__device__ void block_layernorm_rows(float *xs, int K, int ncols, const float *w, const float *b) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nwarps = blockDim.x >> 5;
    for (int r = warp; r < ncols; r += nwarps) {
        float *row = xs + (size_t)r * K;
        float s = 0.f;
        for (int i = lane; i < K; i += 32) s += row[i];
        s = warp_sum(s);
        const float mean = s / (float)K;
        float v = 0.f;
        for (int i = lane; i < K; i += 32) {
            float c = row[i] - mean;
            v += c * c;
        }
        v = warp_sum(v);
        const float rstd = 1.0f / sqrtf(v / (float)K + kNormEps);
        for (int i = lane; i < K; i += 32) row[i] = (row[i] - mean) * rstd * w[i] + b[i];
    }
}

template <int NB, int EPI>
__global__ void __launch_bounds__(256) gemv_kernel(GemvParams p) {
    extern __shared__ __align__(16) float smem[];
    const int K = p.W.in, OUT = p.W.out, C = K >> 4, G = K >> 6;
    float *xs = smem;               // [NB][K]
    float *sx = smem + NB * K;      // [NB][C] chunk sums
    for (int i = threadIdx.x; i < NB * K; i += blockDim.x) {
        const int b = i / K;
        xs[i] = b < p.ncols ? p.x[(size_t)(p.col0 + b) * K + (i - b * K)] : 0.f;
    }
    __syncthreads();
    if (p.ln_mode >= 1) {
        block_layernorm_rows<NB>(xs, K, p.ncols, p.ln_w, p.ln_b);
        __syncthreads();
        if (p.ln_mode == 2) {
            block_layernorm_rows<NB>(xs, K, p.ncols, p.ln2_w, p.ln2_b);
            __syncthreads();
        }
    }
    for (int i = threadIdx.x; i < NB * C; i += blockDim.x) {
        const float4 *v = reinterpret_cast<const float4 *>(xs + (size_t)i * 16);
        float s = 0.f;
#pragma unroll
        for (int j = 0; j < 4; ++j) s += (v[j].x + v[j].y) + (v[j].z + v[j].w);
        sx[i] = s;
    }
    __syncthreads();

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nwarps = blockDim.x >> 5;
    for (int r0 = (blockIdx.x * nwarps + warp) * 2; r0 < OUT; r0 += gridDim.x * nwarps * 2) {
        const bool has1 = r0 + 1 < OUT;
        float acc0[NB], acc1[NB];
#pragma unroll
        for (int b = 0; b < NB; ++b) acc0[b] = acc1[b] = 0.f;
        const uint8_t *w0 = p.W.q + (size_t)r0 * K;
        const uint8_t *w1 = w0 + (has1 ? K : 0);
#pragma unroll 2
        for (int c = lane; c < C; c += 32) {
            const uint4 a = ld_stream(w0 + (size_t)c * 16);
            const uint4 bq = ld_stream(w1 + (size_t)c * 16);
            const int g = c >> 2;
            const float s0 = load_sb(p.W.scales, p.sb_half, (size_t)r0 * G + g);
            const float z0 = load_sb(p.W.biases, p.sb_half, (size_t)r0 * G + g);
            const float s1 = load_sb(p.W.scales, p.sb_half, (size_t)(r0 + (has1 ? 1 : 0)) * G + g);
            const float z1 = load_sb(p.W.biases, p.sb_half, (size_t)(r0 + (has1 ? 1 : 0)) * G + g);
            float qa[16], qb[16];
            const uint32_t wa[4] = {a.x, a.y, a.z, a.w}, wb[4] = {bq.x, bq.y, bq.z, bq.w};
#pragma unroll
            for (int j = 0; j < 16; ++j) {
                qa[j] = byte_to_float(wa[j >> 2], j & 3);
                qb[j] = byte_to_float(wb[j >> 2], j & 3);
            }
#pragma unroll
            for (int b = 0; b < NB; ++b) {
                const float4 *xv = reinterpret_cast<const float4 *>(xs + (size_t)b * K + c * 16);
                float xr[16];
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const float4 t = xv[j];
                    xr[4 * j] = t.x; xr[4 * j + 1] = t.y; xr[4 * j + 2] = t.z; xr[4 * j + 3] = t.w;
                }
                float d0 = 0.f, d1 = 0.f;
#pragma unroll
                for (int j = 0; j < 16; ++j) {
                    d0 = fmaf(xr[j], qa[j], d0);
                    d1 = fmaf(xr[j], qb[j], d1);
                }
                const float scs = sx[b * C + c];
                acc0[b] += s0 * d0 + z0 * scs;
                acc1[b] += s1 * d1 + z1 * scs;
            }
        }
#pragma unroll
        for (int b = 0; b < NB; ++b) {
            acc0[b] = warp_sum(acc0[b]);
            acc1[b] = warp_sum(acc1[b]);
        }
        // Lanes 0..2*NB-1 each finish one (row, column) output.
        if (lane < 2 * NB) {
            const int b = lane >> 1, r = r0 + (lane & 1);
            float v = 0.f;
#pragma unroll
            for (int bb = 0; bb < NB; ++bb)
                if (bb == b) v = (lane & 1) ? acc1[bb] : acc0[bb];
            if (b < p.ncols && r < OUT) {
                v += p.W.bias[r];
                const int col = p.col0 + b;
                if (EPI == EPI_PLAIN) {
                    p.y[(size_t)col * OUT + r] = v;
                } else if (EPI == EPI_GELU) {
                    p.y[(size_t)col * OUT + r] = gelu_tanh(v);
                } else if (EPI == EPI_RESID) {
                    p.y[(size_t)col * OUT + r] += v;
                } else {  // EPI_QKV: q to q_out, k/v into the cache at valid_len
                    const int d = p.d;
                    if (r < d) {
                        p.q_out[(size_t)col * d + r] = v;
                    } else {
                        const int slot = p.batch_slot[col];
                        const SlotState &st = p.slots[slot];
                        if (st.active && st.valid_len < p.max_seq) {
                            const int rr = r - d, which = rr / d, o = rr - which * d;
                            const int h = o >> 6, e = o & 63;
                            __half *cache = which == 0 ? p.k_cache : p.v_cache;
                            cache[kv_index(p.layer, slot, h, st.valid_len, p.n_slots, p.n_heads,
                                           p.max_seq) + e] = __float2half_rn(v);
                        }
                    }
                }
            }
        }
    }
}

static int g_num_sms = 148;

template <int NB, int EPI>
static void gemv_launch_t(const GemvParams &p, cudaStream_t st) {
    const int K = p.W.in;
    const size_t smem = (size_t)NB * K * 4 + (size_t)NB * (K / 16) * 4;
    const int rows_per_cta = 8 * 2;
    int grid = (p.W.out + rows_per_cta - 1) / rows_per_cta;
    gemv_kernel<NB, EPI><<<grid, 256, smem, st>>>(p);
}

template <int NB>
static void gemv_launch_epi(int epi, const GemvParams &p, cudaStream_t st) {
    switch (epi) {
    case EPI_PLAIN: gemv_launch_t<NB, EPI_PLAIN>(p, st); break;
    case EPI_GELU: gemv_launch_t<NB, EPI_GELU>(p, st); break;
    case EPI_RESID: gemv_launch_t<NB, EPI_RESID>(p, st); break;
    default: gemv_launch_t<NB, EPI_QKV>(p, st); break;
    }
}

template <int NB, int EPI>
static void set_gemv_attr() {
    cudaFuncSetAttribute(gemv_kernel<NB, EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         NB * 5120 * 4 + NB * 320 * 4);
}
template <int NB>
static void set_gemv_attrs() {
    set_gemv_attr<NB, EPI_PLAIN>();
    set_gemv_attr<NB, EPI_GELU>();
    set_gemv_attr<NB, EPI_RESID>();
    set_gemv_attr<NB, EPI_QKV>();
}

void launch_gemv(const QLinear &W, bool sb_half, int epi, int ln_mode, const float *ln_w,
                 const float *ln_b, const float *ln2_w, const float *ln2_b, const float *x,
                 float *y, int nb, const DecodeView *dv, int layer, cudaStream_t st) {
    GemvParams p{};
    p.W = W;
    p.sb_half = sb_half;
    p.x = x;
    p.y = y;
    p.ln_mode = ln_mode;
    p.ln_w = ln_w; p.ln_b = ln_b; p.ln2_w = ln2_w; p.ln2_b = ln2_b;
    if (dv) {
        p.q_out = y;
        p.k_cache = dv->k_cache;
        p.v_cache = dv->v_cache;
        p.slots = dv->slots;
        p.batch_slot = dv->batch_slot;
        p.n_slots = dv->n_slots;
        p.n_heads = dv->n_heads;
        p.max_seq = dv->max_seq;
        p.d = dv->d;
    }
    p.layer = layer;
    for (int c0 = 0; c0 < nb; c0 += 8) {
        p.col0 = c0;
        p.ncols = nb - c0 < 8 ? nb - c0 : 8;
        if (p.ncols == 1) gemv_launch_epi<1>(epi, p, st);
        else if (p.ncols == 2) gemv_launch_epi<2>(epi, p, st);
        else if (p.ncols <= 4) gemv_launch_epi<4>(epi, p, st);
        else gemv_launch_epi<8>(epi, p, st);
    }
}

// ---------------------------------------------------------------------------
// Step embedding: x[b] = mel_emb[tok] + mel_pos[pos]  (gpt.rs:720-725)
// ---------------------------------------------------------------------------
__global__ void embed_step_kernel(const float *mel_emb, const float *mel_pos, const SlotState *slots,
                                  const int *batch_slot, int d, int mel_vocab, int mel_pos_len,
                                  float *x) {
    const int b = blockIdx.x;
    const SlotState &st = slots[batch_slot[b]];
    int tok = st.tok, pos = st.pos;
    tok = tok < 0 ? 0 : (tok >= mel_vocab ? mel_vocab - 1 : tok);
    pos = pos < 0 ? 0 : (pos >= mel_pos_len ? mel_pos_len - 1 : pos);
    for (int i = threadIdx.x; i < d; i += blockDim.x)
        x[(size_t)b * d + i] = mel_emb[(size_t)tok * d + i] + mel_pos[(size_t)pos * d + i];
}

void launch_embed_step(const ModelView &m, const DecodeView &dv, float *x, cudaStream_t st) {
    embed_step_kernel<<<dv.nb, 256, 0, st>>>(m.mel_emb, m.mel_pos, dv.slots, dv.batch_slot, m.d,
                                             m.mel_vocab, m.mel_pos_len, x);
}

// ---------------------------------------------------------------------------
// Split-K flash-decode attention: one query per (column, head) against the slot's
// K/V positions [0, valid_len] (the new position was written by the QKV epilogue).
// Grid (split, head, column); each split covers split_len positions, 8 lanes per
// position (16 B of the 128-B fp16 row each); the last split CTA to finish merges
// the partial (max, sum, acc[64]) triples in split order.
// ---------------------------------------------------------------------------
struct AttnParams {
    const float *q;
    float *out;
    const __half *k_cache, *v_cache;
    const SlotState *slots;
    const int *batch_slot;
    int n_slots, n_heads, max_seq, layer, d;
    float *partials;
    int *counters;
    int split_len, max_splits;
};

struct SoftmaxPart {
    float m, l, acc[8];
};

__device__ __forceinline__ void merge_part(SoftmaxPart &a, float m2, float l2, const float *acc2) {
    const float M = fmaxf(a.m, m2);
    if (M == -INFINITY) return;
    const float fa = a.m == -INFINITY ? 0.f : expf(a.m - M);
    const float fb = m2 == -INFINITY ? 0.f : expf(m2 - M);
    a.l = a.l * fa + l2 * fb;
#pragma unroll
    for (int e = 0; e < 8; ++e) a.acc[e] = a.acc[e] * fa + acc2[e] * fb;
    a.m = M;
}

__global__ void __launch_bounds__(128) attn_decode_kernel(AttnParams p) {
    const int split = blockIdx.x, h = blockIdx.y, col = blockIdx.z;
    const int slot = p.batch_slot[col];
    const SlotState &st = p.slots[slot];
    if (!st.active) return;
    const int L = min(st.valid_len + 1, p.max_seq);
    const int n_used = (L + p.split_len - 1) / p.split_len;
    if (split >= n_used) return;
    const int s0 = split * p.split_len, s1 = min(L, s0 + p.split_len);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, grp = lane >> 3, d8 = lane & 7;

    float qv[8];
    const float *qp = p.q + (size_t)col * p.d + h * kHeadDim + d8 * 8;
#pragma unroll
    for (int e = 0; e < 8; ++e) qv[e] = qp[e] * kAttnScale;
    const size_t base = kv_index(p.layer, slot, h, 0, p.n_slots, p.n_heads, p.max_seq);
    const __half *Kb = p.k_cache + base;
    const __half *Vb = p.v_cache + base;

    SoftmaxPart part;
    part.m = -INFINITY;
    part.l = 0.f;
#pragma unroll
    for (int e = 0; e < 8; ++e) part.acc[e] = 0.f;
    for (int j0 = s0 + warp * 4; j0 < s1; j0 += 16) {
        const int j = j0 + grp;
        const bool ok = j < s1;
        float s = 0.f;
        uint4 kr = make_uint4(0, 0, 0, 0), vr = make_uint4(0, 0, 0, 0);
        if (ok) {
            kr = *reinterpret_cast<const uint4 *>(Kb + (size_t)j * kHeadDim + d8 * 8);
            vr = *reinterpret_cast<const uint4 *>(Vb + (size_t)j * kHeadDim + d8 * 8);
        }
        const __half2 *k2 = reinterpret_cast<const __half2 *>(&kr);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const float2 kf = __half22float2(k2[e]);
            s = fmaf(qv[2 * e], kf.x, s);
            s = fmaf(qv[2 * e + 1], kf.y, s);
        }
        s += __shfl_xor_sync(0xffffffffu, s, 1);
        s += __shfl_xor_sync(0xffffffffu, s, 2);
        s += __shfl_xor_sync(0xffffffffu, s, 4);
        if (ok) {
            const float mn = fmaxf(part.m, s);
            const float corr = part.m == -INFINITY ? 0.f : expf(part.m - mn);
            const float pj = expf(s - mn);
            part.l = part.l * corr + pj;
            const __half2 *v2 = reinterpret_cast<const __half2 *>(&vr);
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const float2 vf = __half22float2(v2[e]);
                part.acc[2 * e] = part.acc[2 * e] * corr + pj * vf.x;
                part.acc[2 * e + 1] = part.acc[2 * e + 1] * corr + pj * vf.y;
            }
            part.m = mn;
        }
    }
    // merge the 4 position groups of the warp (lanes with equal d8)
#pragma unroll
    for (int off = 8; off <= 16; off <<= 1) {
        const float m2 = __shfl_xor_sync(0xffffffffu, part.m, off);
        const float l2 = __shfl_xor_sync(0xffffffffu, part.l, off);
        float a2[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) a2[e] = __shfl_xor_sync(0xffffffffu, part.acc[e], off);
        merge_part(part, m2, l2, a2);
    }
    __shared__ float sm_m[4], sm_l[4], sm_acc[4][64];
    if (grp == 0) {
        if (d8 == 0) { sm_m[warp] = part.m; sm_l[warp] = part.l; }
#pragma unroll
        for (int e = 0; e < 8; ++e) sm_acc[warp][d8 * 8 + e] = part.acc[e];
    }
    __syncthreads();
    float *part_out = p.partials + (((size_t)col * p.n_heads + h) * p.max_splits + split) * 66;
    if (threadIdx.x < 64) {
        const int e = threadIdx.x;
        float M = -INFINITY;
        for (int w = 0; w < 4; ++w) M = fmaxf(M, sm_m[w]);
        float l = 0.f, a = 0.f;
        for (int w = 0; w < 4; ++w) {
            const float f = sm_m[w] == -INFINITY ? 0.f : expf(sm_m[w] - M);
            l += sm_l[w] * f;
            a += sm_acc[w][e] * f;
        }
        if (n_used == 1) {
            p.out[(size_t)col * p.d + h * kHeadDim + e] = a / l;
        } else {
            part_out[2 + e] = a;
            if (e == 0) { part_out[0] = M; part_out[1] = l; }
        }
    }
    if (n_used == 1) return;
    __threadfence();
    __syncthreads();
    __shared__ int is_last;
    if (threadIdx.x == 0) {
        const int prev = atomicAdd(&p.counters[col * p.n_heads + h], 1);
        is_last = prev == n_used - 1;
    }
    __syncthreads();
    if (!is_last) return;
    __threadfence();
    if (threadIdx.x < 64) {
        const int e = threadIdx.x;
        const float *pp = p.partials + ((size_t)col * p.n_heads + h) * p.max_splits * 66;
        float M = -INFINITY;
        for (int s = 0; s < n_used; ++s) M = fmaxf(M, __ldcg(pp + s * 66));
        float l = 0.f, a = 0.f;
        for (int s = 0; s < n_used; ++s) {
            const float ms = __ldcg(pp + s * 66);
            const float f = ms == -INFINITY ? 0.f : expf(ms - M);
            l += __ldcg(pp + s * 66 + 1) * f;
            a += __ldcg(pp + s * 66 + 2 + e) * f;
        }
        p.out[(size_t)col * p.d + h * kHeadDim + e] = a / l;
        if (e == 0) p.counters[col * p.n_heads + h] = 0;
    }
}

void launch_attn_decode(const DecodeView &dv, int layer, const float *q, DecodeBufs &b,
                        cudaStream_t st) {
    AttnParams p{};
    p.q = q;
    p.out = b.attn;
    p.k_cache = dv.k_cache;
    p.v_cache = dv.v_cache;
    p.slots = dv.slots;
    p.batch_slot = dv.batch_slot;
    p.n_slots = dv.n_slots;
    p.n_heads = dv.n_heads;
    p.max_seq = dv.max_seq;
    p.layer = layer;
    p.d = dv.d;
    p.partials = b.partials;
    p.counters = b.counters;
    p.split_len = b.split_len;
    p.max_splits = b.max_splits;
    dim3 grid(b.max_splits, dv.n_heads, dv.nb);
    attn_decode_kernel<<<grid, 128, 0, st>>>(p);
}

void decode_forward(const ModelView &m, const DecodeView &dv, DecodeBufs &b, cudaStream_t st) {
    launch_embed_step(m, dv, b.x, st);
    for (int l = 0; l < m.n_layers; ++l) {
        const LayerW &L = m.layers[l];
        launch_gemv(L.c_attn, m.sb_half, EPI_QKV, 1, L.ln1_w, L.ln1_b, nullptr, nullptr, b.x, b.q,
                    dv.nb, &dv, l, st);
        launch_attn_decode(dv, l, b.q, b, st);
        launch_gemv(L.c_proj, m.sb_half, EPI_RESID, 0, nullptr, nullptr, nullptr, nullptr, b.attn,
                    b.x, dv.nb, nullptr, l, st);
        launch_gemv(L.c_fc, m.sb_half, EPI_GELU, 1, L.ln2_w, L.ln2_b, nullptr, nullptr, b.x, b.u,
                    dv.nb, nullptr, l, st);
        launch_gemv(L.mlp_proj, m.sb_half, EPI_RESID, 0, nullptr, nullptr, nullptr, nullptr, b.u,
                    b.x, dv.nb, nullptr, l, st);
    }
    launch_gemv(m.mel_head, m.sb_half, EPI_PLAIN, 2, m.ln_f_w, m.ln_f_b, m.final_w, m.final_b, b.x,
                b.logits, dv.nb, nullptr, 0, st);
}

void kernels_init_decode() {
    set_gemv_attrs<1>();
    set_gemv_attrs<2>();
    set_gemv_attrs<4>();
    set_gemv_attrs<8>();
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&g_num_sms, cudaDevAttrMultiProcessorCount, dev);
}

}  // namespace itts
