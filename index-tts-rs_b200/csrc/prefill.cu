// prefill.cu -- prompt (prefill) kernels: sequence embedding, row LayerNorm,
// int8 group-64 dequant GEMM with bias / GELU / residual / KV-scatter epilogues,
// and causal attention.
//
// Reference semantics: Gpt::prefix_embedding / sequence_embedding
// (crates/core/src/models/gpt.rs:535-627), Gpt::prefill_after (gpt.rs:655-696),
// Gpt2Block::forward with the causal mask (gpt.rs:325-384).
#include "gemm.cuh"

namespace itts {

// Row r of [conds(n_conds), text_emb[0,t..,1] + lang_emb[lang] + text_pos[i],
//           mel_emb[8192] + mel_pos[0], mel_emb[prior[c]] + mel_pos[c + 2]]
__global__ void embed_prefix_kernel(ModelView m, const int *full_text, int n_full,
                                    const float *conds, int n_conds, int lang, const int *prior,
                                    int n_prior, float *x) {
    const int r = blockIdx.x, d = m.d;
    float *out = x + (size_t)r * d;
    if (r < n_conds) {
        for (int i = threadIdx.x; i < d; i += blockDim.x) out[i] = conds[(size_t)r * d + i];
    } else if (r < n_conds + n_full) {
        const int t = r - n_conds, tok = full_text[t];
        for (int i = threadIdx.x; i < d; i += blockDim.x)
            out[i] = (m.text_emb[(size_t)tok * d + i] + m.lang_emb[(size_t)lang * d + i]) +
                     m.text_pos[(size_t)t * d + i];
    } else if (r == n_conds + n_full) {
        for (int i = threadIdx.x; i < d; i += blockDim.x)
            out[i] = m.mel_emb[(size_t)kStartMel * d + i] + m.mel_pos[i];
    } else {
        const int c = r - (n_conds + n_full + 1), tok = prior[c];
        for (int i = threadIdx.x; i < d; i += blockDim.x)
            out[i] = m.mel_emb[(size_t)tok * d + i] + m.mel_pos[(size_t)(c + 2) * d + i];
    }
}

void launch_embed_prefix(const ModelView &m, const int *full_text, int n_full, const float *conds,
                         int n_conds, int lang, const int *prior, int n_prior, float *x,
                         cudaStream_t st) {
    const int T = n_conds + n_full + 1 + n_prior;
    embed_prefix_kernel<<<T, 256, 0, st>>>(m, full_text, n_full, conds, n_conds, lang, prior,
                                            n_prior, x);
}

// y[t] = LayerNorm(x[t]) * w + b, one CTA per row, two-pass statistics.
template <typename TY>
__global__ void __launch_bounds__(256) layernorm_rows_kernel(const float *x, const float *w,
                                                             const float *b, int d, TY *y) {
    const int t = blockIdx.x;
    const float *row = x + (size_t)t * d;
    __shared__ float red[8];
    __shared__ float stat;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    float s = 0.f;
    for (int i = threadIdx.x; i < d; i += blockDim.x) s += row[i];
    s = warp_sum(s);
    if (lane == 0) red[warp] = s;
    __syncthreads();
    if (threadIdx.x == 0) {
        float a = 0.f;
        for (int i = 0; i < (int)(blockDim.x >> 5); ++i) a += red[i];
        stat = a / (float)d;
    }
    __syncthreads();
    const float mean = stat;
    float v = 0.f;
    for (int i = threadIdx.x; i < d; i += blockDim.x) {
        const float c = row[i] - mean;
        v += c * c;
    }
    v = warp_sum(v);
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    if (threadIdx.x == 0) {
        float a = 0.f;
        for (int i = 0; i < (int)(blockDim.x >> 5); ++i) a += red[i];
        stat = 1.0f / sqrtf(a / (float)d + kNormEps);
    }
    __syncthreads();
    const float rstd = stat;
    for (int i = threadIdx.x; i < d; i += blockDim.x) {
        const float v = (row[i] - mean) * rstd * w[i] + b[i];
        if constexpr (sizeof(TY) == 2) y[(size_t)t * d + i] = __float2half_rn(v);
        else y[(size_t)t * d + i] = v;
    }
}

// The same with one warp per row (d a multiple of 128, at most 128 * LNW_CH): the row
// stays in registers (float4 chunks c * 128 + 4 lane), two-pass statistics over them.
constexpr int LNW_CH = 16;
template <typename TY>
__global__ void __launch_bounds__(256) layernorm_rows_warp_kernel(const float *x, const float *w,
                                                                  const float *b, int rows, int d, TY *y) {
    const int t = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (t >= rows) return;
    const int nch = d / 128;
    const float4 *row = reinterpret_cast<const float4 *>(x + (size_t)t * d);
    float4 v[LNW_CH];
    float s = 0.f;
#pragma unroll
    for (int c = 0; c < LNW_CH; ++c)  // every load issued before the first use (no early exit)
        v[c] = c < nch ? row[c * 32 + lane] : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int c = 0; c < LNW_CH; ++c) s += (v[c].x + v[c].y) + (v[c].z + v[c].w);
    const float mean = warp_sum(s) / (float)d;
    float q = 0.f;
#pragma unroll
    for (int c = 0; c < LNW_CH; ++c) {
        if (c >= nch) break;
        const float a0 = v[c].x - mean, a1 = v[c].y - mean, a2 = v[c].z - mean, a3 = v[c].w - mean;
        q += (a0 * a0 + a1 * a1) + (a2 * a2 + a3 * a3);
    }
    const float rstd = 1.0f / sqrtf(warp_sum(q) / (float)d + kNormEps);
#pragma unroll
    for (int c = 0; c < LNW_CH; ++c) {
        if (c >= nch) break;
        const int k = c * 128 + 4 * lane;
        const float4 ww = *reinterpret_cast<const float4 *>(w + k), bb = *reinterpret_cast<const float4 *>(b + k);
        const float o0 = (v[c].x - mean) * rstd * ww.x + bb.x, o1 = (v[c].y - mean) * rstd * ww.y + bb.y;
        const float o2 = (v[c].z - mean) * rstd * ww.z + bb.z, o3 = (v[c].w - mean) * rstd * ww.w + bb.w;
        if constexpr (sizeof(TY) == 2) {
            const __half2 h01 = __floats2half2_rn(o0, o1), h23 = __floats2half2_rn(o2, o3);
            uint2 hv;
            hv.x = *reinterpret_cast<const uint32_t *>(&h01);
            hv.y = *reinterpret_cast<const uint32_t *>(&h23);
            *reinterpret_cast<uint2 *>(y + (size_t)t * d + k) = hv;
        } else {
            *reinterpret_cast<float4 *>(y + (size_t)t * d + k) = make_float4(o0, o1, o2, o3);
        }
    }
}

template <typename TY>
static void launch_ln(const float *x, const float *w, const float *b, int rows, int d, TY *y, cudaStream_t st) {
    const bool aligned = ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(y) |
                           reinterpret_cast<uintptr_t>(w) | reinterpret_cast<uintptr_t>(b)) & 15) == 0;
    if (d % 128 == 0 && d <= 128 * LNW_CH && aligned)
        layernorm_rows_warp_kernel<TY><<<(rows + 7) / 8, 256, 0, st>>>(x, w, b, rows, d, y);
    else
        layernorm_rows_kernel<TY><<<rows, 256, 0, st>>>(x, w, b, d, y);
}
void launch_layernorm_rows(const float *x, const float *w, const float *b, int rows, int d,
                           float *y, cudaStream_t st) {
    launch_ln<float>(x, w, b, rows, d, y, st);
}
void launch_layernorm_rows_h(const float *x, const float *w, const float *b, int rows, int d,
                             __half *y, cudaStream_t st) {
    launch_ln<__half>(x, w, b, rows, d, y, st);
}

// ---------------------------------------------------------------------------
// GEMM: y[t, o] = x[t, :] . W[o, :] + bias[o] for T prompt positions.
// CTA tile 64 positions x 64 outputs, K step = one quantization group (64);
// the weight tile is dequantized once into shared memory (fp32) and reused by
// all 64 positions.  Thread tile 4 x 4.
// ---------------------------------------------------------------------------

template <int EPI>
__global__ void __launch_bounds__(256) gemm_q8_kernel(GemmParams p) {
    constexpr int BM = 64, BN = 64, BK = 64, PAD = 4;
    __shared__ __align__(16) float Xs[BK][BM + PAD];
    __shared__ __align__(16) float Ws[BK][BN + PAD];
    const int K = p.W.in, OUT = p.W.out;
    const int t0 = blockIdx.y * BM, o0 = blockIdx.x * BN;
    const int tid = threadIdx.x, ty = tid >> 4, tx = tid & 15;
    float acc[4][4] = {};
    for (int k0 = 0; k0 < K; k0 += BK) {
        {  // X tile: thread loads 16 consecutive k of one position
            const int t = tid >> 2, kq = (tid & 3) * 16;
            const int tt = t0 + t;
#pragma unroll
            for (int j = 0; j < 16; j += 4) {
                float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
                if (tt < p.T) {
                    const uint2 h = *reinterpret_cast<const uint2 *>(p.x + (size_t)tt * K + k0 + kq + j);
                    const float2 a = __half22float2(*reinterpret_cast<const __half2 *>(&h.x));
                    const float2 b = __half22float2(*reinterpret_cast<const __half2 *>(&h.y));
                    v = make_float4(a.x, a.y, b.x, b.y);
                }
                Xs[kq + j][t] = v.x;
                Xs[kq + j + 1][t] = v.y;
                Xs[kq + j + 2][t] = v.z;
                Xs[kq + j + 3][t] = v.w;
            }
        }
        {  // W tile: thread dequantizes the 16 bytes (fragment order) at [16c, 16c+16)
            // of one row's quantization group
            const int r = tid >> 2, c = tid & 3;
            const int o = o0 + r;
            float s = 0.f, z = 0.f;
            uint4 w = make_uint4(0, 0, 0, 0);
            if (o < OUT) {
                w = ld_stream(p.W.tiles + mk_q_offset(p.W, o, k0) + c * 16);
                const uint8_t *sb = p.W.tiles + mk_sb_offset(p.W, o, k0);
                if (p.W.sbb == 4) {
                    const float2 f = __half22float2(*reinterpret_cast<const __half2 *>(sb));
                    s = f.x; z = f.y;
                } else {
                    const float2 f = *reinterpret_cast<const float2 *>(sb);
                    s = f.x; z = f.y;
                }
            }
            const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
            for (int pb = 0; pb < 16; ++pb) {
                const int k = (pb >> 2) * 16 + ((pb >> 1) & 1) * 8 + 2 * c + (pb & 1);
                Ws[k][r] = s * byte_to_float(ww[pb >> 2], pb & 3) + z;
            }
        }
        __syncthreads();
#pragma unroll 8
        for (int kk = 0; kk < BK; ++kk) {
            const float4 a = *reinterpret_cast<const float4 *>(&Xs[kk][ty * 4]);
            const float4 b = *reinterpret_cast<const float4 *>(&Ws[kk][tx * 4]);
            const float av[4] = {a.x, a.y, a.z, a.w}, bv[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int t = t0 + ty * 4 + i;
        if (t >= p.T) continue;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int o = o0 + tx * 4 + j;
            if (o >= OUT) continue;
            gemm_store<EPI>(p, t, o, acc[i][j] + p.W.bias[o], qkv_dest(p, t));
        }
    }
}

// Row counts from which the tensor-core GEMM is used (below it the CUDA-core tile wastes
// less of a 128-row MMA tile).
constexpr int kGemmTcMinRows = 16;

void launch_gemm(int epi, const MkLin &W, const __half *x, void *y, int T, const DecodeView *dv,
                 __half *k_cache, __half *v_cache, int kv_slot, int n_slots, int n_heads,
                 int max_seq, int layer, int d, cudaStream_t st, float *ws, int ws_splits) {
    GemmParams p{};
    p.W = W;
    p.x = x;
    p.y = static_cast<float *>(y);
    p.T = T;
    p.k_cache = k_cache;
    p.v_cache = v_cache;
    p.kv_slot = kv_slot;
    p.n_slots = n_slots;
    p.n_heads = n_heads;
    p.max_seq = max_seq;
    p.layer = layer;
    p.d = d;
    if (dv) {
        p.slots = dv->slots;
        p.batch_slot = dv->batch_slot;
    }
    p.ws = ws;
    p.ws_splits = ws_splits;
    if (W.w16 && (T >= kGemmF16MinRows || (ws && T >= kGemmTcMinRows)) && launch_gemm_f16(epi, p, W.w16, st)) return;
    if (T >= kGemmTcMinRows && launch_gemm_tc(epi, p, st)) return;
    dim3 grid((W.out + 63) / 64, (T + 63) / 64);
    switch (epi) {
    case EPI_PLAIN: gemm_q8_kernel<EPI_PLAIN><<<grid, 256, 0, st>>>(p); break;
    case EPI_GELU: gemm_q8_kernel<EPI_GELU><<<grid, 256, 0, st>>>(p); break;
    case EPI_RESID: gemm_q8_kernel<EPI_RESID><<<grid, 256, 0, st>>>(p); break;
    default: gemm_q8_kernel<EPI_QKV><<<grid, 256, 0, st>>>(p); break;
    }
}

void launch_gemm_rows(int epi, const MkLin &W, const __half *x, void *y, int T, const int *row_slot,
                      const int *row_pos, __half *k_cache, __half *v_cache, int n_slots, int n_heads,
                      int max_seq, int layer, int d, cudaStream_t st) {
    GemmParams p{};
    p.W = W;
    p.x = x;
    p.y = static_cast<float *>(y);
    p.T = T;
    p.k_cache = k_cache;
    p.v_cache = v_cache;
    p.row_slot = row_slot;
    p.row_pos = row_pos;
    p.kv_slot = -1;
    p.n_slots = n_slots;
    p.n_heads = n_heads;
    p.max_seq = max_seq;
    p.layer = layer;
    p.d = d;
    if (T >= kGemmF16MinRows && W.w16 && launch_gemm_f16(epi, p, W.w16, st)) return;
    if (T >= kGemmTcMinRows && launch_gemm_tc(epi, p, st)) return;
    dim3 grid((W.out + 63) / 64, (T + 63) / 64);
    switch (epi) {
    case EPI_PLAIN: gemm_q8_kernel<EPI_PLAIN><<<grid, 256, 0, st>>>(p); break;
    case EPI_GELU: gemm_q8_kernel<EPI_GELU><<<grid, 256, 0, st>>>(p); break;
    case EPI_RESID: gemm_q8_kernel<EPI_RESID><<<grid, 256, 0, st>>>(p); break;
    default: gemm_q8_kernel<EPI_QKV><<<grid, 256, 0, st>>>(p); break;
    }
}

// Gpt2Block::head_attention (gpt.rs:391-427) on the prefill's QKV of one layer: for
// query row t = q0 + blockIdx.x, softmax over keys 0..t of head `head` at scale 0.125
// (the prefix and the Mel positions up to the query), keeping key columns [k0, k1).
// accumulate: maps = (maps + p) / 2, the mean of two heads' maps.
__global__ void __launch_bounds__(128) head_probs_kernel(const float *qkv, int T, int d, int head, int q0,
                                                         int k0, int k1, float *maps, int accumulate) {
    extern __shared__ float hp_sc[];  // [t + 1] scores, then [32] reduction scratch
    __shared__ float q[64];
    __shared__ float red[4];
    const int t = q0 + blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    if (tid < 64) q[tid] = qkv[(size_t)t * 3 * d + head * 64 + tid];
    __syncthreads();
    float mx = -INFINITY;
    for (int j = tid; j <= t; j += blockDim.x) {
        const float *k = qkv + (size_t)j * 3 * d + d + head * 64;
        float s = 0.f;
        for (int e = 0; e < 64; ++e) s = fmaf(q[e], k[e], s);
        s *= kAttnScale;
        hp_sc[j] = s;
        mx = fmaxf(mx, s);
    }
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if (lane == 0) red[warp] = mx;
    __syncthreads();
    mx = fmaxf(fmaxf(red[0], red[1]), fmaxf(red[2], red[3]));
    __syncthreads();
    float den = 0.f;
    for (int j = tid; j <= t; j += blockDim.x) {
        const float e = expf(hp_sc[j] - mx);
        hp_sc[j] = e;
        den += e;
    }
    den = warp_sum(den);
    if (lane == 0) red[warp] = den;
    __syncthreads();
    den = (red[0] + red[1]) + (red[2] + red[3]);
    const int nk = k1 - k0;
    float *row = maps + (size_t)blockIdx.x * nk;
    for (int j = k0 + tid; j < k1; j += blockDim.x) {
        const float pj = j <= t ? hp_sc[j] / den : 0.f;
        row[j - k0] = accumulate ? (row[j - k0] + pj) / 2.0f : pj;
    }
}

// log_softmax of each logits row, taken at the row's target (gpt.rs:850-852).
__global__ void __launch_bounds__(256) log_softmax_pick_kernel(const float *logits, int V, const int *targets,
                                                               float *out) {
    __shared__ float red[8];
    const float *row = logits + (size_t)blockIdx.x * V;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    float mx = -INFINITY;
    for (int v = tid; v < V; v += blockDim.x) mx = fmaxf(mx, row[v]);
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if (lane == 0) red[warp] = mx;
    __syncthreads();
    mx = red[0];
    for (int w = 1; w < 8; ++w) mx = fmaxf(mx, red[w]);
    __syncthreads();
    float s = 0.f;
    for (int v = tid; v < V; v += blockDim.x) s += expf(row[v] - mx);
    s = warp_sum(s);
    if (lane == 0) red[warp] = s;
    __syncthreads();
    if (tid == 0) {
        float tot = 0.f;
        for (int w = 0; w < 8; ++w) tot += red[w];
        out[blockIdx.x] = (row[targets[blockIdx.x]] - mx) - logf(tot);
    }
}

void prefill_forward(const ModelView &m, const DecodeView &dv, int slot, int T, PrefillBufs &pb,
                     float *logits_row, cudaStream_t st, const PrefillHooks *hk) {
    const int d = m.d;
    int map_done = 0;
    for (int l = 0; l < m.n_layers; ++l) {
        const MkLayer &L = m.layers[l];
        __half *n16 = reinterpret_cast<__half *>(pb.n), *attn16 = reinterpret_cast<__half *>(pb.attn),
               *u16 = reinterpret_cast<__half *>(pb.u);
        launch_layernorm_rows_h(pb.x, L.ln1_w, L.ln1_b, T, d, n16, st);
        launch_gemm(EPI_QKV, L.qkv, n16, pb.qkv, T, nullptr, dv.k_cache, dv.v_cache, slot,
                    dv.n_slots, dv.n_heads, dv.max_seq, l, d, st);
        if (hk && hk->maps && (l == hk->map_layers[0] || l == hk->map_layers[1])) {
            const int rows = T - hk->map_q0;
            head_probs_kernel<<<rows, 128, (size_t)T * sizeof(float), st>>>(
                pb.qkv, T, d, hk->map_head, hk->map_q0, hk->map_k0, hk->map_k1, hk->maps, map_done++ > 0);
        }
        if (hk && l == hk->stop_layer) return;
        launch_attn_prefill_fa(pb.qkv, T, slot, dv, l, d, attn16, st);
        launch_gemm(EPI_RESID, L.proj, attn16, pb.x, T, nullptr, nullptr, nullptr, -1, 0, 0, 0, l,
                    d, st);
        launch_layernorm_rows_h(pb.x, L.ln2_w, L.ln2_b, T, d, n16, st);
        launch_gemm(EPI_GELU, L.fc, n16, pb.u, T, nullptr, nullptr, nullptr, -1, 0, 0, 0, l, d, st);
        launch_gemm(EPI_RESID, L.mlp, u16, pb.x, T, nullptr, nullptr, nullptr, -1, 0, 0, 0, l, d,
                    st);
    }
    if (hk && hk->lp_q0 >= 0) {
        // every row from lp_q0: ln_f, final_norm, mel_head, log_softmax at its target
        const int rows = T - hk->lp_q0;
        launch_layernorm_rows(pb.x + (size_t)hk->lp_q0 * d, m.ln_f_w, m.ln_f_b, rows, d, pb.n, st);
        launch_layernorm_rows_h(pb.n, m.final_w, m.final_b, rows, d, reinterpret_cast<__half *>(pb.attn), st);
        launch_gemm(EPI_PLAIN, m.mel_head, reinterpret_cast<const __half *>(pb.attn), hk->lp_logits, rows, nullptr, nullptr, nullptr, -1, 0, 0, 0,
                    0, d, st);
        log_softmax_pick_kernel<<<rows, 256, 0, st>>>(hk->lp_logits, m.mel_vocab, hk->lp_targets, hk->lp_out);
        return;
    }
    // ln_f then final_norm on the last row, then mel_head (gpt.rs:673-692)
    const float *last = pb.x + (size_t)(T - 1) * d;
    launch_layernorm_rows(last, m.ln_f_w, m.ln_f_b, 1, d, pb.n, st);
    __half *fin16 = reinterpret_cast<__half *>(pb.n + d);
    launch_layernorm_rows_h(pb.n, m.final_w, m.final_b, 1, d, fin16, st);
    launch_gemm(EPI_PLAIN, m.mel_head, fin16, logits_row, 1, nullptr, nullptr, nullptr, -1, 0, 0,
                0, 0, d, st);
}

// The largest shared-memory carve-out for the LayerNorms that run between the decode step's
// big kernels (see kernels_init_decode).
void kernels_init_prefill() {
    cudaFuncSetAttribute(layernorm_rows_warp_kernel<float>, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
    cudaFuncSetAttribute(layernorm_rows_warp_kernel<__half>, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
    cudaGetLastError();
}

}  // namespace itts
