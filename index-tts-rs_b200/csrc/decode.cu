// decode.cu -- decode-step dispatch: the persistent decode-step kernel for up to
// MK_MAX_NB batch columns (mk_decode.cu), and for larger batches a GEMM path
// (prefill.cu's int8 GEMM with batch columns as rows) around a split-K flash-decode
// attention over the fp16 KV cache.
//
// Reference semantics: Gpt::step (crates/core/src/models/gpt.rs:706-754),
// Gpt2Block::forward (gpt.rs:325-384).
#include <cstdio>

#include "kernels.h"

namespace itts {

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
    int q_stride;
    __half *out;  // [nb][d] fp16 (the input of the c_proj GEMM)
    const __half *k_cache, *v_cache;
    const SlotState *slots;
    const int *batch_slot;
    int n_slots, n_heads, max_seq, layer, d;
    float *partials;
    int *counters;
    int split_len, max_splits;
    int frag;  // write the output in fragment order (the skinny GEMM's activation layout)
};

// position of head element e (0..63) in the attention output: natural, or fragment order
__device__ __forceinline__ int attn_out_pos(int e, int frag) {
    if (!frag) return e;
    const int b = e >> 4, kk = e & 15, c = (kk & 7) >> 1, hi = kk >> 3, lo = kk & 1;
    return c * 16 + b * 4 + hi * 2 + lo;
}

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
    const float *qp = p.q + (size_t)col * p.q_stride + h * kHeadDim + d8 * 8;
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
    // each trip: positions j0 + grp and j0 + 16 + grp (two 16-position rows of the warp's
    // range); all four K/V loads are issued before the first is used
    for (int j0 = s0 + warp * 4; j0 < s1; j0 += 32) {
        uint4 kr[2], vr[2];
        bool ok[2];
#pragma unroll
        for (int u = 0; u < 2; ++u) {
            const int j = j0 + 16 * u + grp;
            ok[u] = j < s1;
            kr[u] = make_uint4(0, 0, 0, 0);
            vr[u] = kr[u];
            if (ok[u]) {
                kr[u] = *reinterpret_cast<const uint4 *>(Kb + (size_t)j * kHeadDim + d8 * 8);
                vr[u] = *reinterpret_cast<const uint4 *>(Vb + (size_t)j * kHeadDim + d8 * 8);
            }
        }
#pragma unroll
        for (int u = 0; u < 2; ++u) {
            float s = 0.f;
            const __half2 *k2 = reinterpret_cast<const __half2 *>(&kr[u]);
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const float2 kf = __half22float2(k2[e]);
                s = fmaf(qv[2 * e], kf.x, s);
                s = fmaf(qv[2 * e + 1], kf.y, s);
            }
            s += __shfl_xor_sync(0xffffffffu, s, 1);
            s += __shfl_xor_sync(0xffffffffu, s, 2);
            s += __shfl_xor_sync(0xffffffffu, s, 4);
            if (ok[u]) {
                const float mn = fmaxf(part.m, s);
                const float corr = part.m == -INFINITY ? 0.f : expf(part.m - mn);
                const float pj = expf(s - mn);
                part.l = part.l * corr + pj;
                const __half2 *v2 = reinterpret_cast<const __half2 *>(&vr[u]);
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const float2 vf = __half22float2(v2[e]);
                    part.acc[2 * e] = part.acc[2 * e] * corr + pj * vf.x;
                    part.acc[2 * e + 1] = part.acc[2 * e + 1] * corr + pj * vf.y;
                }
                part.m = mn;
            }
        }
    }
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
            p.out[(size_t)col * p.d + h * kHeadDim + attn_out_pos(e, p.frag)] = __float2half_rn(a / l);
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
        p.out[(size_t)col * p.d + h * kHeadDim + attn_out_pos(e, p.frag)] = __float2half_rn(a / l);
        if (e == 0) p.counters[col * p.n_heads + h] = 0;
    }
}

void launch_attn_decode(const DecodeView &dv, int layer, const float *q, int q_stride,
                        DecodeBufs &b, cudaStream_t st, int frag) {
    AttnParams p{};
    p.frag = frag;
    p.q = q;
    p.q_stride = q_stride;
    p.out = reinterpret_cast<__half *>(b.attn);
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

static MkParams mk_params(const ModelView &m, const DecodeView &dv, DecodeBufs &b) {
    MkParams p{};
    p.n_layers = m.n_layers;
    p.d = m.d;
    p.H = m.n_heads;
    p.ff = m.ff;
    p.mel_vocab = m.mel_vocab;
    p.mel_pos_len = m.mel_pos_len;
    p.nb = dv.nb;
    p.grid = b.mk_grid;
    p.nslot = b.mk_nslot[dv.nb];
    p.xsk = m.ff > m.d ? m.ff : m.d;
    p.sbb = m.sb_half ? 4 : 8;
    p.layers = m.d_layers;
    p.head = m.mel_head;
    p.lnf_w = m.ln_f_w; p.lnf_b = m.ln_f_b; p.fin_w = m.final_w; p.fin_b = m.final_b;
    p.mel_emb = m.mel_emb;
    p.mel_pos = m.mel_pos;
    p.slots = dv.slots;
    p.batch_slot = dv.batch_slot;
    p.n_slots = dv.n_slots;
    p.max_seq = dv.max_seq;
    p.kc = dv.k_cache;
    p.vc = dv.v_cache;
    p.qkv_ll = b.qkv_ll;
    p.attn_ll = b.attn_ll;
    p.ao_ll = b.ao_ll;
    p.h_ll = b.h_ll;
    p.u_ll = b.u_ll;
    p.x_ll = b.x_ll;
    p.logits = b.logits;
    p.epoch = b.epoch;
    p.err = b.err;
    p.trace = b.trace;
    p.stall = b.stall;
    return p;
}

static bool use_mk(const DecodeBufs &b, int nb) {
    return nb <= MK_MAX_NB && b.mk_grid > 0 && b.mk_nslot[nb] >= 2;
}

static bool use_wide(const ModelView &m, const DecodeBufs &b, int nb) {
    if (!b.wide_int8 || nb > SK_MAX_NB || m.d > MK_MAX_D || m.d % 128 || m.ff % 64) return false;
    const MkLayer &L = m.layers[0];
    return skinny_ok(L.qkv, nb) && skinny_ok(L.proj, nb) && skinny_ok(L.fc, nb) && skinny_ok(L.mlp, nb) &&
           skinny_ok(m.mel_head, nb);
}

// Steps of up to XK_SEQ_MAX_NB columns run the batch-1 cluster kernel once per column (each
// launch streams the weights again, but a column costs less than in the grid-wide kernel).
static bool use_xk(const DecodeBufs &b, int nb) { return b.xk.grid > 0 && nb <= XK_SEQ_MAX_NB; }

int decode_forward_launches(const ModelView &m, const DecodeBufs &b, int nb) {
    if (use_xk(b, nb)) return nb;
    if (use_mk(b, nb)) return 1;
    if (use_wide(m, b, nb)) return 1 + 6 * m.n_layers + 3;
    return 1 + 7 * m.n_layers + 3;
}

bool decode_uses_f16_weights(const ModelView &m, const DecodeBufs &b, int nb) {
    return !(use_xk(b, nb) || use_mk(b, nb) || use_wide(m, b, nb));
}

// Steps of 5..SK_MAX_NB columns: LayerNorms into fragment order, the skinny int8 GEMMs, the
// split-K flash-decode attention with fragment-order output (6 launches per layer).
static cudaError_t decode_forward_wide(const ModelView &m, const DecodeView &dv, DecodeBufs &b, cudaStream_t st) {
    const int d = m.d, nb = dv.nb;
    launch_embed_step(m, dv, b.x, st);
    __half *n16 = reinterpret_cast<__half *>(b.n), *attn16 = reinterpret_cast<__half *>(b.attn),
           *u16 = reinterpret_cast<__half *>(b.u), *fin16 = reinterpret_cast<__half *>(b.n2);
    cudaError_t e = cudaSuccess;
    auto ok = [&](cudaError_t r) { if (e == cudaSuccess) e = r; };
    for (int l = 0; l < m.n_layers; ++l) {
        const MkLayer &L = m.layers[l];
        launch_ln_frag(b.x, L.ln1_w, L.ln1_b, nb, d, n16, st);
        ok(launch_skinny(EPI_QKV, L.qkv, n16, nb, b.q, &dv, l, d, b.ws, b.sk_counters, st));
        launch_attn_decode(dv, l, b.q, 3 * d, b, st, 1);
        ok(launch_skinny(EPI_RESID, L.proj, attn16, nb, b.x, nullptr, l, d, b.ws, b.sk_counters, st));
        launch_ln_frag(b.x, L.ln2_w, L.ln2_b, nb, d, n16, st);
        ok(launch_skinny(EPI_GELU, L.fc, n16, nb, b.u, nullptr, l, d, b.ws, b.sk_counters, st, L.mlp.kc));
        ok(launch_skinny(EPI_RESID, L.mlp, u16, nb, b.x, nullptr, l, d, b.ws, b.sk_counters, st));
    }
    launch_layernorm_rows(b.x, m.ln_f_w, m.ln_f_b, nb, d, b.n, st);   // gpt.ln_f, then final_norm
    launch_ln_frag(b.n, m.final_w, m.final_b, nb, d, fin16, st);
    ok(launch_skinny(EPI_PLAIN, m.mel_head, fin16, nb, b.logits, nullptr, 0, d, b.ws, b.sk_counters, st));
    return e != cudaSuccess ? e : cudaGetLastError();
}

cudaError_t decode_forward(const ModelView &m, const DecodeView &dv, DecodeBufs &b,
                           cudaStream_t st) {
    if (use_xk(b, dv.nb)) {
        for (int col = 0; col < dv.nb; ++col) {
            MkParams p = mk_params(m, dv, b);
            p.batch_slot = dv.batch_slot + col;
            p.nb = 1;
            p.logits = b.logits + (size_t)col * m.mel_vocab;
            const cudaError_t e = xk_launch(p, b.xk, b.xkb, st);
            if (e != cudaSuccess) return e;
        }
        return cudaSuccess;
    }
    if (use_mk(b, dv.nb)) return mk_launch(mk_params(m, dv, b), st);
    if (use_wide(m, b, dv.nb)) return decode_forward_wide(m, dv, b, st);
    const int d = m.d;
    launch_embed_step(m, dv, b.x, st);
    __half *n16 = reinterpret_cast<__half *>(b.n), *attn16 = reinterpret_cast<__half *>(b.attn),
           *u16 = reinterpret_cast<__half *>(b.u), *fin16 = reinterpret_cast<__half *>(b.n2);
    for (int l = 0; l < m.n_layers; ++l) {
        const MkLayer &L = m.layers[l];
        launch_layernorm_rows_h(b.x, L.ln1_w, L.ln1_b, dv.nb, d, n16, st);
        launch_gemm(EPI_QKV, L.qkv, n16, b.q, dv.nb, &dv, dv.k_cache, dv.v_cache, -1, dv.n_slots,
                    dv.n_heads, dv.max_seq, l, d, st, b.ws, b.ws_splits);
        launch_attn_decode(dv, l, b.q, 3 * d, b, st, 0);
        launch_gemm(EPI_RESID, L.proj, attn16, b.x, dv.nb, nullptr, nullptr, nullptr, -1, 0, 0, 0, l,
                    d, st, b.ws, b.ws_splits);
        launch_layernorm_rows_h(b.x, L.ln2_w, L.ln2_b, dv.nb, d, n16, st);
        launch_gemm(EPI_GELU, L.fc, n16, b.u, dv.nb, nullptr, nullptr, nullptr, -1, 0, 0, 0, l, d, st, b.ws,
                    b.ws_splits);
        launch_gemm(EPI_RESID, L.mlp, u16, b.x, dv.nb, nullptr, nullptr, nullptr, -1, 0, 0, 0, l, d,
                    st, b.ws, b.ws_splits);
    }
    launch_layernorm_rows(b.x, m.ln_f_w, m.ln_f_b, dv.nb, d, b.n, st);
    launch_layernorm_rows_h(b.n, m.final_w, m.final_b, dv.nb, d, fin16, st);
    launch_gemm(EPI_PLAIN, m.mel_head, fin16, b.logits, dv.nb, nullptr, nullptr, nullptr, -1, 0, 0, 0,
                0, d, st);
    return cudaGetLastError();
}

// Every kernel of a decode step asks for the largest shared-memory carve-out: the step's
// big kernels (the batch-1 cluster kernel, the skinny GEMMs) need it, and an SM whose next
// kernel prefers another L1 / shared split has to drain and reconfigure between launches.
void kernels_init_decode() {
    cudaFuncSetAttribute(embed_step_kernel, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
    cudaFuncSetAttribute(attn_decode_kernel, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
    cudaGetLastError();
}

}  // namespace itts
