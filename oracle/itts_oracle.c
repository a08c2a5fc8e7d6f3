/*
 * itts_oracle.c -- CPU restatement of the index-tts-rs Stage-1 GPT decoder hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  Nothing in the shipped library links, loads or calls
 * this file; only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg
 * use it, and there only as the checker (or as the timed CPU stand-in for the
 * reference, which is Rust + MLX/Metal and cannot be built in this container).
 *
 * What it restates (paths relative to the tyrchen/index-tts-rs project):
 *   crates/core/src/models/gpt.rs      -- decoder, KV cache, prefill / step
 *   crates/core/src/models/sampler.rs  -- SamplerRng, SeenTokenBitSet,
 *                                         sample_next_token, generate_codes_after
 * The per-op arithmetic lives in the third-party crate mlx-rs 0.33.0 / mlx-sys
 * 0.7.0 (Apple MLX, not vendored in the reference).  The ops are restated from
 * MLX's published semantics:
 *   quantized_matmul(transpose=true, group_size=64, bits=8), affine format:
 *       W[o,i] = scales[o,i/64] * q[o,i] + biases[o,i/64],  q = byte (i%4) of
 *       the little-endian u32 weight[o, i/4]
 *   fast::layer_norm(eps=1e-5), gelu_approximate (tanh form),
 *   fast::scaled_dot_product_attention(scale=0.125, causal iff T>1).
 * All arithmetic is IEEE fp32 like the reference's fp32 MLX path.
 *
 * Parity pinning: the sampler is pinned by the reference's own known-answer
 * tests (sampler.rs:177-189, 430-454, 98-107, 456-485).  The decoder arithmetic
 * (the MLX boundary) is UNPINNED against reference outputs in this container:
 * the reference's golden logits (crates/core/fixtures/golden_ref.safetensors,
 * CP-10/CP-11) need the real 867 MB checkpoint, which is absent.  The decoder
 * restatement is instead cross-checked against an independent GPT-2
 * implementation (HuggingFace transformers GPT2Model, fp32) on the same
 * dequantized weights.
 *
 * Tie-break: the reference's top-k uses select_nth_unstable_by + sort_unstable_by
 * (sampler.rs:228,231), whose order among equal scaled logits is unspecified.
 * This restatement (and the CUDA sampler) define it as "lower token id first".
 *
 * exp(): the reference calls f32::exp (the platform libm expf).  This restatement
 * uses the correctly rounded value (float)exp((double)x); a test records how
 * often glibc's expf differs from it.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#include <stdio.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define ORC_OK 0
#define ORC_E_VALIDATION 1
#define ORC_E_ALLOC 2

#define MEL_VOCAB_REF 8194
#define START_TEXT 0      /* gpt.rs:57 */
#define STOP_TEXT 1       /* gpt.rs:59 */
#define START_MEL 8192    /* gpt.rs:61 */
#define STOP_MEL 8193     /* gpt.rs:63 */
#define GROUP 64          /* gpt.rs:65 */
#define HEAD_DIM 64       /* gpt.rs:36 */
#define NORM_EPS 1e-5f    /* gpt.rs:42 */
#define ATTN_SCALE 0.125f /* gpt.rs:67 */
#define BITSET_WORDS 129  /* sampler.rs:19 */

static char g_err[512];
const char *orc_last_error(void) { return g_err; }
static int fail(int code, const char *msg) {
    snprintf(g_err, sizeof g_err, "%s", msg);
    return code;
}

/* ------------------------------------------------------------------ */
/* SamplerRng (sampler.rs:24-62)                                       */
/* ------------------------------------------------------------------ */
uint64_t orc_rng_new(uint64_t seed) { return seed ^ 0x9E3779B97F4A7C15ULL; } /* :41-45 */

uint64_t orc_rng_next_u64(uint64_t *state) { /* :48-54 */
    *state += 0x9E3779B97F4A7C15ULL;
    uint64_t z = *state;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
    return z ^ (z >> 31);
}

float orc_rng_next_f32(uint64_t *state) { /* :58-61 */
    uint32_t upper24 = (uint32_t)(orc_rng_next_u64(state) >> 40);
    return (float)upper24 * (1.0f / (float)(1u << 24));
}

/* ------------------------------------------------------------------ */
/* SeenTokenBitSet (sampler.rs:67-158)                                 */
/* ------------------------------------------------------------------ */
void orc_seen_empty(uint64_t *w) { memset(w, 0, BITSET_WORDS * sizeof(uint64_t)); }
void orc_seen_insert(uint64_t *w, int64_t tok) { /* :118-124 */
    if (tok < 0) return;
    uint64_t wi = (uint64_t)tok / 64, bi = (uint64_t)tok % 64;
    if (wi < BITSET_WORDS) w[wi] |= 1ULL << bi;
}
int orc_seen_contains(const uint64_t *w, int64_t tok) { /* :128-134 */
    if (tok < 0) return 0;
    uint64_t wi = (uint64_t)tok / 64, bi = (uint64_t)tok % 64;
    return wi < BITSET_WORDS && ((w[wi] >> bi) & 1ULL);
}
void orc_seen_initial(uint64_t *w) { /* :110-115 */
    orc_seen_empty(w);
    orc_seen_insert(w, STOP_TEXT);
    orc_seen_insert(w, START_MEL);
}
void orc_apply_repetition_penalty(const uint64_t *w, float *logits, int64_t n, float penalty) {
    /* :138-157 */
    if (fabsf(penalty - 1.0f) <= 1.1920929e-7f) return; /* f32::EPSILON */
    for (int wi = 0; wi < BITSET_WORDS; ++wi) {
        uint64_t word = w[wi];
        while (word) {
            int bit = __builtin_ctzll(word);
            int64_t tid = (int64_t)wi * 64 + bit;
            if (tid < n) {
                if (logits[tid] < 0.0f) logits[tid] *= penalty;
                else logits[tid] /= penalty;
            }
            word &= word - 1;
        }
    }
}

/* ------------------------------------------------------------------ */
/* sample_next_token (sampler.rs:191-284)                              */
/* ------------------------------------------------------------------ */
typedef struct {
    int32_t greedy;
    uint32_t top_k;
    float top_p;
    float temperature;
    float repetition_penalty;
    uint32_t max_mel_tokens;
} orc_params; /* config.rs:1283-1320 */

int orc_argmax_finite(const float *l, int64_t n) { /* sampler.rs:395-405 */
    int best = 0;
    float bv = -INFINITY;
    for (int64_t i = 0; i < n; ++i)
        if (isfinite(l[i]) && l[i] > bv) { bv = l[i]; best = (int)i; }
    return best;
}

float orc_expf(float x) { return (float)exp((double)x); }

typedef struct { int32_t id; float v; } cand_t;

/* Descending by value (sampler.rs:407-414; candidates are never NaN because
 * non-finite logits become -inf at :213-217), ties: lower id first. */
static int cand_cmp(const void *a, const void *b) {
    const cand_t *x = (const cand_t *)a, *y = (const cand_t *)b;
    if (x->v > y->v) return -1;
    if (x->v < y->v) return 1;
    return (x->id < y->id) ? -1 : (x->id > y->id);
}

int orc_sample_next_token(float *logits, int64_t n, const uint64_t *seen, const orc_params *p,
                          uint64_t *rng, int32_t *tok_out) {
    if (n <= 0) return fail(ORC_E_VALIDATION, "logits: logits slice must not be empty");
    orc_apply_repetition_penalty(seen, logits, n, p->repetition_penalty); /* :204 */
    if (p->greedy) { *tok_out = orc_argmax_finite(logits, n); return ORC_OK; } /* :206-208 */
    float inv_temp = 1.0f / p->temperature; /* :210 */
    cand_t *c = (cand_t *)malloc((size_t)n * sizeof(cand_t));
    float *probs = (float *)malloc((size_t)n * sizeof(float));
    if (!c || !probs) { free(c); free(probs); return fail(ORC_E_ALLOC, "oom"); }
    for (int64_t i = 0; i < n; ++i) { /* :212-219 */
        float v = logits[i];
        c[i].id = (int32_t)i;
        c[i].v = isfinite(v) ? v * inv_temp : -INFINITY;
    }
    int64_t k = p->top_k == 0 ? n : (p->top_k < (uint64_t)n ? (int64_t)p->top_k : n); /* :221-226 */
    /* select_nth + truncate + sort (:227-231) == full sort then truncate, under
     * the fixed tie-break. */
    qsort(c, (size_t)n, sizeof(cand_t), cand_cmp);
    int64_t len = k;
    float max_logit = isfinite(c[0].v) ? c[0].v : 0.0f; /* :233-235 */
    float prob_sum = 0.0f;
    for (int64_t i = 0; i < len; ++i) { /* :238-248 */
        float pr = isfinite(c[i].v) ? orc_expf(c[i].v - max_logit) : 0.0f;
        probs[i] = pr;
        prob_sum += pr;
    }
    if (prob_sum <= 0.0f || !isfinite(prob_sum)) { /* :250-252 */
        *tok_out = c[0].id; free(c); free(probs); return ORC_OK;
    }
    float top_p = p->top_p, cum = 0.0f;
    int64_t active = len;
    for (int64_t i = 0; i < len; ++i) { /* :254-264 */
        float norm_p = probs[i] / prob_sum;
        if (i > 0 && cum > top_p) { active = i; break; }
        cum += norm_p;
    }
    float active_sum = 0.0f; /* :269 */
    for (int64_t i = 0; i < active; ++i) active_sum += probs[i];
    if (active_sum <= 0.0f || !isfinite(active_sum)) { /* :270-272 */
        *tok_out = c[0].id; free(c); free(probs); return ORC_OK;
    }
    float draw = orc_rng_next_f32(rng) * active_sum; /* :274 */
    float acc = 0.0f;
    for (int64_t i = 0; i < active; ++i) { /* :275-281 */
        acc += probs[i];
        if (draw <= acc) { *tok_out = c[i].id; free(c); free(probs); return ORC_OK; }
    }
    *tok_out = c[active - 1].id; /* :283 */
    free(c); free(probs);
    return ORC_OK;
}

/* ------------------------------------------------------------------ */
/* Model                                                               */
/* ------------------------------------------------------------------ */
typedef struct {
    const uint32_t *w;      /* [out, in/4] packed u8 (little endian) */
    const void *scales;     /* [out, in/64] f32 or f16 bits */
    const void *biases;     /* [out, in/64] */
    const float *bias;      /* [out] */
    int out, in;
} orc_linear;

typedef struct {
    const float *ln1_w, *ln1_b, *ln2_w, *ln2_b;
    orc_linear c_attn, c_proj, c_fc, mlp_proj;
} orc_layer;

typedef struct {
    int n_layers, d, n_heads, ff, mel_vocab, text_vocab, lang_vocab, mel_pos_len, text_pos_len;
    int sb_half;
    const float *text_emb, *lang_emb, *mel_emb, *mel_pos, *text_pos;
    const float *ln_f_w, *ln_f_b, *final_w, *final_b;
    orc_linear mel_head;
    orc_layer *layers;
} orc_model;

static float half_to_float(uint16_t h) {
    uint32_t sign = (uint32_t)(h >> 15) << 31, exp = (h >> 10) & 0x1F, man = h & 0x3FF, bits;
    if (exp == 0) {
        if (man == 0) bits = sign;
        else { /* subnormal: value = man * 2^-24 */
            float f = (float)man * 5.9604644775390625e-8f;
            return (h >> 15) ? -f : f;
        }
    } else if (exp == 31) bits = sign | 0x7F800000u | (man << 13);
    else bits = sign | ((exp + 112) << 23) | (man << 13);
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

static inline float sb_get(const void *p, int half, int64_t idx) {
    return half ? half_to_float(((const uint16_t *)p)[idx]) : ((const float *)p)[idx];
}

orc_model *orc_model_new(int n_layers, int d, int n_heads, int ff, int mel_vocab, int text_vocab,
                         int lang_vocab, int mel_pos_len, int text_pos_len, int sb_half) {
    orc_model *m = (orc_model *)calloc(1, sizeof(orc_model));
    if (!m) return NULL;
    m->n_layers = n_layers; m->d = d; m->n_heads = n_heads; m->ff = ff;
    m->mel_vocab = mel_vocab; m->text_vocab = text_vocab; m->lang_vocab = lang_vocab;
    m->mel_pos_len = mel_pos_len; m->text_pos_len = text_pos_len; m->sb_half = sb_half;
    m->layers = (orc_layer *)calloc((size_t)n_layers, sizeof(orc_layer));
    return m;
}
void orc_model_free(orc_model *m) { if (m) { free(m->layers); free(m); } }

/* Binds one linear (gpt.rs:229-250 names: <prefix>.weight/.scales/.biases/.bias). */
static void bind_linear(orc_linear *l, const void *w, const void *s, const void *b, const void *bias,
                        int out, int in) {
    l->w = (const uint32_t *)w; l->scales = s; l->biases = b; l->bias = (const float *)bias;
    l->out = out; l->in = in;
}

/* which: 0=c_attn 1=c_proj 2=c_fc 3=mlp_proj 4=mel_head */
void orc_model_set_linear(orc_model *m, int layer, int which, const void *w, const void *s,
                          const void *b, const void *bias) {
    int d = m->d, ff = m->ff;
    if (which == 4) { bind_linear(&m->mel_head, w, s, b, bias, m->mel_vocab, d); return; }
    orc_layer *L = &m->layers[layer];
    switch (which) {
    case 0: bind_linear(&L->c_attn, w, s, b, bias, 3 * d, d); break;
    case 1: bind_linear(&L->c_proj, w, s, b, bias, d, d); break;
    case 2: bind_linear(&L->c_fc, w, s, b, bias, ff, d); break;
    case 3: bind_linear(&L->mlp_proj, w, s, b, bias, d, ff); break;
    }
}
void orc_model_set_layer_norms(orc_model *m, int layer, const float *ln1_w, const float *ln1_b,
                               const float *ln2_w, const float *ln2_b) {
    orc_layer *L = &m->layers[layer];
    L->ln1_w = ln1_w; L->ln1_b = ln1_b; L->ln2_w = ln2_w; L->ln2_b = ln2_b;
}
void orc_model_set_globals(orc_model *m, const float *text_emb, const float *lang_emb,
                           const float *mel_emb, const float *mel_pos, const float *text_pos,
                           const float *ln_f_w, const float *ln_f_b, const float *final_w,
                           const float *final_b) {
    m->text_emb = text_emb; m->lang_emb = lang_emb; m->mel_emb = mel_emb; m->mel_pos = mel_pos;
    m->text_pos = text_pos; m->ln_f_w = ln_f_w; m->ln_f_b = ln_f_b; m->final_w = final_w;
    m->final_b = final_b;
}

/* QuantizedLinear::forward (gpt.rs:252-263): y[t,o] = sum_i x[t,i] * W[o,i] + bias[o] */
static void linear_fwd(const orc_model *m, const orc_linear *l, const float *x, int T, float *y) {
    const int in = l->in, out = l->out, groups = in / GROUP;
#pragma omp parallel
    {
        float *row = (float *)malloc((size_t)in * sizeof(float));
#pragma omp for schedule(static)
        for (int o = 0; o < out; ++o) {
            const uint8_t *q = (const uint8_t *)(l->w + (size_t)o * (in / 4));
            for (int g = 0; g < groups; ++g) {
                float s = sb_get(l->scales, m->sb_half, (int64_t)o * groups + g);
                float b = sb_get(l->biases, m->sb_half, (int64_t)o * groups + g);
                for (int i = 0; i < GROUP; ++i) row[g * GROUP + i] = s * (float)q[g * GROUP + i] + b;
            }
            for (int t = 0; t < T; ++t) {
                const float *xt = x + (size_t)t * in;
                float acc = 0.0f;
                for (int i = 0; i < in; ++i) acc += xt[i] * row[i];
                y[(size_t)t * out + o] = acc + l->bias[o];
            }
        }
        free(row);
    }
}

/* fast::layer_norm(x, w, b, 1e-5) over the last axis */
static void layer_norm(const float *x, const float *w, const float *b, int T, int d, float *y) {
    for (int t = 0; t < T; ++t) {
        const float *xt = x + (size_t)t * d;
        float mean = 0.0f, var = 0.0f;
        for (int i = 0; i < d; ++i) mean += xt[i];
        mean /= (float)d;
        for (int i = 0; i < d; ++i) { float c = xt[i] - mean; var += c * c; }
        var /= (float)d;
        float rstd = 1.0f / sqrtf(var + NORM_EPS);
        for (int i = 0; i < d; ++i) y[(size_t)t * d + i] = (xt[i] - mean) * rstd * w[i] + b[i];
    }
}

static float gelu_tanh(float x) { /* nn::gelu_approximate (gpt.rs:381) */
    const float k = 0.7978845608028654f; /* sqrt(2/pi) */
    return 0.5f * x * (1.0f + tanhf(k * (x + 0.044715f * x * x * x)));
}

/* KvCache (gpt.rs:74-217): fp32 [layer][head][max_seq][64], preallocated to
 * max_seq (the reference grows in 256-position steps up to max_seq; the
 * contents and the overflow error are the same). */
typedef struct {
    float *k, *v;
    int n_layers, n_heads, max_seq, valid_len;
} orc_kv;

orc_kv *orc_kv_new(const orc_model *m, int max_seq) {
    if (max_seq <= 0) { fail(ORC_E_VALIDATION, "max_seq: KV cache max_seq must be >= 1"); return NULL; }
    orc_kv *kv = (orc_kv *)calloc(1, sizeof(orc_kv));
    size_t n = (size_t)m->n_layers * m->n_heads * max_seq * HEAD_DIM;
    kv->k = (float *)calloc(n, sizeof(float));
    kv->v = (float *)calloc(n, sizeof(float));
    kv->n_layers = m->n_layers; kv->n_heads = m->n_heads; kv->max_seq = max_seq; kv->valid_len = 0;
    if (!kv->k || !kv->v) { free(kv->k); free(kv->v); free(kv); fail(ORC_E_ALLOC, "oom"); return NULL; }
    return kv;
}
void orc_kv_free(orc_kv *kv) { if (kv) { free(kv->k); free(kv->v); free(kv); } }
void orc_kv_reset(orc_kv *kv) { kv->valid_len = 0; }
int orc_kv_valid_len(const orc_kv *kv) { return kv->valid_len; }

static inline float *kv_ptr(float *base, const orc_kv *kv, int layer, int head, int pos);

/* Timing aid for the CPU baseline (no reference counterpart): extends every layer's
 * cache from valid_len to n positions by repeating the filled positions cyclically, so a
 * following orc_step costs what a step at KV length n costs (the work of a step depends
 * only on the length).  Needs valid_len >= 1 and n <= max_seq. */
int orc_kv_fill(orc_kv *kv, int n) {
    if (kv->valid_len < 1 || n > kv->max_seq || n < kv->valid_len)
        return fail(ORC_E_VALIDATION, "kv_fill: need 1 <= valid_len <= n <= max_seq");
    const int v0 = kv->valid_len;
    for (int l = 0; l < kv->n_layers; ++l)
        for (int h = 0; h < kv->n_heads; ++h)
            for (int p = v0; p < n; ++p) {
                memcpy(kv_ptr(kv->k, kv, l, h, p), kv_ptr(kv->k, kv, l, h, p % v0), HEAD_DIM * sizeof(float));
                memcpy(kv_ptr(kv->v, kv, l, h, p), kv_ptr(kv->v, kv, l, h, p % v0), HEAD_DIM * sizeof(float));
            }
    kv->valid_len = n;
    return ORC_OK;
}

static inline float *kv_ptr(float *base, const orc_kv *kv, int layer, int head, int pos) {
    return base + (((size_t)layer * kv->n_heads + head) * kv->max_seq + pos) * HEAD_DIM;
}

/* Gpt2Block::forward (gpt.rs:325-384).  x: [T, d] updated in place. */
static int block_fwd(const orc_model *m, int li, orc_kv *kv, float *x, int T, int new_valid,
                     int causal) {
    const orc_layer *L = &m->layers[li];
    const int d = m->d, H = m->n_heads, ff = m->ff;
    if (new_valid > kv->max_seq) { /* gpt.rs:157-165 */
        char buf[160];
        snprintf(buf, sizeof buf, "kv_cache: sequence length %d exceeds KV cache capacity %d",
                 new_valid, kv->max_seq);
        return fail(ORC_E_VALIDATION, buf);
    }
    const int prev = new_valid - T;
    float *n1 = (float *)malloc((size_t)T * d * sizeof(float));
    float *qkv = (float *)malloc((size_t)T * 3 * d * sizeof(float));
    float *attn = (float *)malloc((size_t)T * d * sizeof(float));
    float *tmp = (float *)malloc((size_t)T * d * sizeof(float));
    float *hid = (float *)malloc((size_t)T * ff * sizeof(float));
    layer_norm(x, L->ln1_w, L->ln1_b, T, d, n1);          /* :339-344 */
    linear_fwd(m, &L->c_attn, n1, T, qkv);                /* :345 */
    /* split q|k|v, heads (:346-360); cache update at prev..new_valid (:362) */
    for (int t = 0; t < T; ++t)
        for (int h = 0; h < H; ++h) {
            memcpy(kv_ptr(kv->k, kv, li, h, prev + t), qkv + (size_t)t * 3 * d + d + h * HEAD_DIM,
                   HEAD_DIM * sizeof(float));
            memcpy(kv_ptr(kv->v, kv, li, h, prev + t),
                   qkv + (size_t)t * 3 * d + 2 * d + h * HEAD_DIM, HEAD_DIM * sizeof(float));
        }
    /* scaled_dot_product_attention(scale 0.125, causal iff T>1) (:363-368).
     * Causal with T queries over new_valid keys: query t sees keys
     * 0..=prev+t (bottom-right aligned). */
    const int use_mask = causal && T > 1;
#pragma omp parallel
    {
        float *sc = (float *)malloc((size_t)new_valid * sizeof(float));
#pragma omp for collapse(2) schedule(static)
        for (int t = 0; t < T; ++t)
            for (int h = 0; h < H; ++h) {
                const float *q = qkv + (size_t)t * 3 * d + h * HEAD_DIM;
                int nk = use_mask ? prev + t + 1 : new_valid;
                float mx = -INFINITY;
                for (int j = 0; j < nk; ++j) {
                    const float *kj = kv_ptr(kv->k, kv, li, h, j);
                    float s = 0.0f;
                    for (int e = 0; e < HEAD_DIM; ++e) s += (q[e] * ATTN_SCALE) * kj[e];
                    sc[j] = s;
                    if (s > mx) mx = s;
                }
                float den = 0.0f;
                for (int j = 0; j < nk; ++j) { sc[j] = expf(sc[j] - mx); den += sc[j]; }
                float *o = attn + (size_t)t * d + h * HEAD_DIM;
                for (int e = 0; e < HEAD_DIM; ++e) o[e] = 0.0f;
                for (int j = 0; j < nk; ++j) {
                    const float *vj = kv_ptr(kv->v, kv, li, h, j);
                    float pj = sc[j] / den;
                    for (int e = 0; e < HEAD_DIM; ++e) o[e] += pj * vj[e];
                }
            }
        free(sc);
    }
    linear_fwd(m, &L->c_proj, attn, T, tmp);              /* :372 */
    for (size_t i = 0; i < (size_t)T * d; ++i) x[i] += tmp[i];
    layer_norm(x, L->ln2_w, L->ln2_b, T, d, n1);          /* :375-380 */
    linear_fwd(m, &L->c_fc, n1, T, hid);                  /* :381 */
    for (size_t i = 0; i < (size_t)T * ff; ++i) hid[i] = gelu_tanh(hid[i]);
    linear_fwd(m, &L->mlp_proj, hid, T, tmp);             /* :382 */
    for (size_t i = 0; i < (size_t)T * d; ++i) x[i] += tmp[i]; /* :383 */
    free(n1); free(qkv); free(attn); free(tmp); free(hid);
    return ORC_OK;
}

/* ln_f then final_norm on one row, then mel_head (gpt.rs:673-692, 734-750) */
static void head_fwd(const orc_model *m, const float *h, float *logits) {
    const int d = m->d;
    float *a = (float *)malloc((size_t)d * sizeof(float));
    float *b = (float *)malloc((size_t)d * sizeof(float));
    layer_norm(h, m->ln_f_w, m->ln_f_b, 1, d, a);
    layer_norm(a, m->final_w, m->final_b, 1, d, b);
    linear_fwd(m, &m->mel_head, b, 1, logits);
    free(a); free(b);
}

/* sequence_embedding / prefix_embedding (gpt.rs:535-627):
 * [conds(n_conds), text_emb[0,toks..,1] + lang_emb[lang] + text_pos[0..L+2),
 *  mel_emb[8192] + mel_pos[0], mel_emb[prior[i]] + mel_pos[2+i] ...] */
int orc_sequence_embedding(const orc_model *m, const int32_t *text, int n_text, const float *conds,
                           int n_conds, int lang, const int32_t *codes, int n_codes, float *out,
                           int *seq_len_out) {
    const int d = m->d;
    if (n_text <= 0) return fail(ORC_E_VALIDATION, "text_tokens: text_tokens must not be empty");
    if (n_codes + 3 > m->mel_pos_len)
        return fail(ORC_E_VALIDATION, "codes: codes exceed the Mel positional capacity");
    int full = n_text + 2;
    if (full > m->text_pos_len) return fail(ORC_E_VALIDATION, "text_tokens: text sequence too long");
    if (n_conds <= 0) return fail(ORC_E_VALIDATION, "conds: expected at least one conditioning row");
    if (lang < 0 || lang >= m->lang_vocab) return fail(ORC_E_VALIDATION, "lang_id: out of range");
    for (int i = 0; i < n_text; ++i)
        if (text[i] < 0 || text[i] >= m->text_vocab)
            return fail(ORC_E_VALIDATION, "text_tokens: token id out of range");
    for (int i = 0; i < n_codes; ++i)
        if (codes[i] < 0 || codes[i] >= m->mel_vocab)
            return fail(ORC_E_VALIDATION, "codes: token id out of range");
    if (!out) { *seq_len_out = n_conds + full + 1 + n_codes; return ORC_OK; }
    int r = 0;
    memcpy(out, conds, (size_t)n_conds * d * sizeof(float));
    r += n_conds;
    for (int t = 0; t < full; ++t, ++r) {
        int tok = t == 0 ? START_TEXT : (t == full - 1 ? STOP_TEXT : text[t - 1]);
        for (int i = 0; i < d; ++i)
            out[(size_t)r * d + i] = (m->text_emb[(size_t)tok * d + i] + m->lang_emb[(size_t)lang * d + i]) +
                                     m->text_pos[(size_t)t * d + i];
    }
    for (int i = 0; i < d; ++i)
        out[(size_t)r * d + i] = m->mel_emb[(size_t)START_MEL * d + i] + m->mel_pos[i];
    ++r;
    for (int c = 0; c < n_codes; ++c, ++r)
        for (int i = 0; i < d; ++i)
            out[(size_t)r * d + i] = m->mel_emb[(size_t)codes[c] * d + i] + m->mel_pos[(size_t)(c + 2) * d + i];
    *seq_len_out = r;
    return ORC_OK;
}

/* Gpt::prefill_after (gpt.rs:655-696) */
int orc_prefill(const orc_model *m, orc_kv *kv, const int32_t *text, int n_text, const float *conds,
                int n_conds, int lang, const int32_t *prior, int n_prior, float *logits) {
    int T = 0, rc = orc_sequence_embedding(m, text, n_text, conds, n_conds, lang, prior, n_prior, NULL, &T);
    if (rc) return rc;
    float *x = (float *)malloc((size_t)T * m->d * sizeof(float));
    orc_sequence_embedding(m, text, n_text, conds, n_conds, lang, prior, n_prior, x, &T);
    orc_kv_reset(kv);
    for (int l = 0; l < m->n_layers; ++l) {
        rc = block_fwd(m, l, kv, x, T, T, 1);
        if (rc) { free(x); return rc; }
    }
    kv->valid_len = T;
    head_fwd(m, x + (size_t)(T - 1) * m->d, logits);
    free(x);
    return ORC_OK;
}

/* Alignment heads and the number of leading layers alignment replays
 * (crates/core/src/align/mod.rs:37-40). */
static const int ALIGN_HEADS[2][2] = {{4, 10}, {5, 10}};
#define ALIGN_LAYERS 6
#define MASK_FILL 1e9f /* gpt.rs:72 */

/* Gpt2Block::head_attention (gpt.rs:391-427): softmax attention of one head of the layer
 * whose input is x [T, d] (LN1 -> c_attn), for query rows qs..T-1, each seeing the
 * whole prefix 0..qs-1 and the positions qs..itself; keeps key columns klo..khi-1.
 * out: [T - qs][khi - klo]. */
static void head_attention(const orc_model *m, int li, const float *x, int T, int head, int qs,
                           int klo, int khi, float *out) {
    const orc_layer *L = &m->layers[li];
    const int d = m->d, nk = khi - klo;
    float *n1 = (float *)malloc((size_t)T * d * sizeof(float));
    float *qkv = (float *)malloc((size_t)T * 3 * d * sizeof(float));
    layer_norm(x, L->ln1_w, L->ln1_b, T, d, n1);
    linear_fwd(m, &L->c_attn, n1, T, qkv);
#pragma omp parallel
    {
        float *sc = (float *)malloc((size_t)T * sizeof(float));
#pragma omp for schedule(static)
        for (int t = qs; t < T; ++t) {
            const float *q = qkv + (size_t)t * 3 * d + head * HEAD_DIM;
            float mx = -INFINITY;
            for (int j = 0; j < T; ++j) {
                const float *k = qkv + (size_t)j * 3 * d + d + head * HEAD_DIM;
                float s = 0.0f;
                for (int e = 0; e < HEAD_DIM; ++e) s += q[e] * k[e];
                s *= ATTN_SCALE;
                if (j > t) s += -MASK_FILL; /* (tri - 1) * MASK_FILL on the Mel part */
                sc[j] = s;
                if (s > mx) mx = s;
            }
            float den = 0.0f;
            for (int j = 0; j < T; ++j) { sc[j] = expf(sc[j] - mx); den += sc[j]; }
            for (int j = klo; j < khi; ++j) out[(size_t)(t - qs) * nk + (j - klo)] = sc[j] / den;
        }
        free(sc);
    }
    free(n1); free(qkv);
}

/* Gpt::replay (gpt.rs:800-861) and Gpt::alignment_attention (gpt.rs:875-915).
 * fed: the codes fed after <START_MEL> (codes[..n-1], or prior ++ codes[..n-1]).
 * mode 0: all layers; log_probs[i] = log_softmax(head(row qs + i))[targets[i]] for i < n_targets
 *         (log_probs may be NULL); maps (may be NULL) = alignment attention from rows qs..
 * mode 1: alignment only, the first ALIGN_LAYERS layers (the last one not run past its
 *         attention map).  maps: [T - qs][n_text + 2], averaged over ALIGN_HEADS. */
int orc_replay(const orc_model *m, orc_kv *kv, const int32_t *text, int n_text, const float *conds,
               int n_conds, int lang, const int32_t *fed, int n_fed, int qs, int mode,
               const int32_t *targets, int n_targets, float *log_probs, float *maps) {
    int T = 0, rc = orc_sequence_embedding(m, text, n_text, conds, n_conds, lang, fed, n_fed, NULL, &T);
    if (rc) return rc;
    if (qs < 0 || qs >= T) return fail(ORC_E_VALIDATION, "codes: query start out of range");
    const int want_maps = maps != NULL;
    if (want_maps && (m->n_layers < ALIGN_LAYERS || m->n_heads <= ALIGN_HEADS[0][1]))
        return fail(ORC_E_VALIDATION, "attention: the model has no alignment heads");
    const int d = m->d, klo = n_conds, khi = n_conds + n_text + 2, rows = T - qs, nk = khi - klo;
    float *x = (float *)malloc((size_t)T * d * sizeof(float));
    orc_sequence_embedding(m, text, n_text, conds, n_conds, lang, fed, n_fed, x, &T);
    orc_kv_reset(kv);
    float *map_b = want_maps ? (float *)malloc((size_t)rows * nk * sizeof(float)) : NULL;
    const int n_run = mode == 1 ? ALIGN_LAYERS : m->n_layers;
    for (int l = 0; l < n_run; ++l) {
        if (want_maps)
            for (int a = 0; a < 2; ++a)
                if (ALIGN_HEADS[a][0] == l)
                    head_attention(m, l, x, T, ALIGN_HEADS[a][1], qs, klo, khi, a == 0 ? maps : map_b);
        if (mode == 1 && l + 1 >= ALIGN_LAYERS) break;
        rc = block_fwd(m, l, kv, x, T, T, 1);
        if (rc) { free(x); free(map_b); return rc; }
    }
    orc_kv_reset(kv);
    if (want_maps) /* stack(maps).mean(0) */
        for (size_t i = 0; i < (size_t)rows * nk; ++i) maps[i] = (maps[i] + map_b[i]) / 2.0f;
    if (mode == 0 && log_probs) {
        float *lg = (float *)malloc((size_t)m->mel_vocab * sizeof(float));
        for (int i = 0; i < n_targets && qs + i < T; ++i) {
            head_fwd(m, x + (size_t)(qs + i) * d, lg);
            float mx = -INFINITY;
            for (int v = 0; v < m->mel_vocab; ++v) if (lg[v] > mx) mx = lg[v];
            double den = 0.0;
            for (int v = 0; v < m->mel_vocab; ++v) den += exp((double)(lg[v] - mx));
            log_probs[i] = (lg[targets[i]] - mx) - (float)log(den); /* log_softmax, take_along_axis */
        }
        free(lg);
    }
    free(x); free(map_b);
    return ORC_OK;
}

/* Gpt::step (gpt.rs:706-754) */
int orc_step(const orc_model *m, orc_kv *kv, int tok, int pos, float *logits) {
    if (tok < 0 || tok >= m->mel_vocab) return fail(ORC_E_VALIDATION, "mel_token_id: out of range");
    if (pos < 0 || pos >= m->mel_pos_len) return fail(ORC_E_VALIDATION, "pos_idx: out of range");
    const int d = m->d;
    float *x = (float *)malloc((size_t)d * sizeof(float));
    for (int i = 0; i < d; ++i) x[i] = m->mel_emb[(size_t)tok * d + i] + m->mel_pos[(size_t)pos * d + i];
    int nv = kv->valid_len + 1;
    for (int l = 0; l < m->n_layers; ++l) {
        int rc = block_fwd(m, l, kv, x, 1, nv, 0);
        if (rc) { free(x); return rc; }
    }
    kv->valid_len = nv;
    head_fwd(m, x, logits);
    free(x);
    return ORC_OK;
}

/* generate_codes_after (sampler.rs:340-392).  codes_out must hold max_steps. */
int orc_generate(const orc_model *m, orc_kv *kv, const int32_t *text, int n_text, const float *conds,
                 int n_conds, int lang, const int32_t *prior, int n_prior, int min_codes,
                 const orc_params *p, uint64_t *rng, int32_t *codes_out, int max_out, int *n_out) {
    int max_steps = (int)p->max_mel_tokens;
    int cap = m->mel_pos_len - 3 - n_prior;
    if (cap < 0) cap = 0;
    if (max_steps > cap) max_steps = cap; /* :348-349 */
    if (max_steps == 0)
        return fail(ORC_E_VALIDATION, "max_mel_tokens: no Mel positions left to generate");
    if (max_out < max_steps) return fail(ORC_E_VALIDATION, "codes_out: buffer too small");
    float *logits = (float *)malloc((size_t)m->mel_vocab * sizeof(float));
    int rc = orc_prefill(m, kv, text, n_text, conds, n_conds, lang, prior, n_prior, logits);
    if (rc) { free(logits); return rc; }
    uint64_t seen[BITSET_WORDS];
    orc_seen_initial(seen); /* :368 */
    int n = 0;
    for (int step = 0; step < max_steps; ++step) {
        if (n < min_codes) logits[STOP_MEL] = -INFINITY; /* :372-376 */
        int32_t tok = 0;
        rc = orc_sample_next_token(logits, m->mel_vocab, seen, p, rng, &tok);
        if (rc) break;
        if (tok == STOP_MEL) break; /* :378 */
        codes_out[n++] = tok;
        if (tok >= 0 && tok < m->mel_vocab) orc_seen_insert(seen, tok);
        if (step + 1 < max_steps) {
            rc = orc_step(m, kv, tok, n_prior + step + 2, logits); /* :385-388 */
            if (rc) break;
        }
    }
    free(logits);
    *n_out = n;
    return rc;
}

int orc_num_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}
void orc_set_num_threads(int n) {
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
#else
    (void)n;
#endif
}

/* ---------------------------------------------------------------------------------------
 * SemanticCodec decode (crates/core/src/models/codec.rs:202-239, the Vocos backbone
 * codec.rs:83-102, the ConvNeXt block crates/core/src/models/convnext.rs:66-73), fp32.
 * MLX conv weights are channels-last [C_out, K, C_in]; conv1d is a cross-correlation:
 * y[t, o] = b[o] + sum_k sum_i x[t + k - pad, i] w[o, k, i] (zero outside the sequence).
 * --------------------------------------------------------------------------------------- */
typedef struct {
    const float *dw_w, *dw_b, *norm_w, *norm_b, *pw1_w, *pw1_b, *pw2_w, *pw2_b, *gamma;
} orc_codec_block;

typedef struct {
    int n_layers, hidden, dim, inter, cdim, n_codes, embed_k, dw_k, up_k;
    const float *codebook, *out_w, *out_b, *embed_w, *embed_b, *norm_w, *norm_b, *fnorm_w, *fnorm_b;
    const float *proj_w, *proj_b, *up_w, *up_b;
    orc_codec_block *blocks;
} orc_codec;

orc_codec *orc_codec_new(int n_layers, int hidden, int dim, int inter, int cdim, int n_codes, int embed_k,
                         int dw_k, int up_k) {
    orc_codec *c = (orc_codec *)calloc(1, sizeof(orc_codec));
    c->n_layers = n_layers; c->hidden = hidden; c->dim = dim; c->inter = inter; c->cdim = cdim;
    c->n_codes = n_codes; c->embed_k = embed_k; c->dw_k = dw_k; c->up_k = up_k;
    c->blocks = (orc_codec_block *)calloc((size_t)n_layers, sizeof(orc_codec_block));
    return c;
}
void orc_codec_free(orc_codec *c) { if (c) { free(c->blocks); free(c); } }
void orc_codec_set_globals(orc_codec *c, const float *codebook, const float *out_w, const float *out_b,
                           const float *embed_w, const float *embed_b, const float *norm_w, const float *norm_b,
                           const float *fnorm_w, const float *fnorm_b, const float *proj_w, const float *proj_b,
                           const float *up_w, const float *up_b) {
    c->codebook = codebook; c->out_w = out_w; c->out_b = out_b; c->embed_w = embed_w; c->embed_b = embed_b;
    c->norm_w = norm_w; c->norm_b = norm_b; c->fnorm_w = fnorm_w; c->fnorm_b = fnorm_b;
    c->proj_w = proj_w; c->proj_b = proj_b; c->up_w = up_w; c->up_b = up_b;
}
void orc_codec_set_block(orc_codec *c, int l, const float *dw_w, const float *dw_b, const float *norm_w,
                         const float *norm_b, const float *pw1_w, const float *pw1_b, const float *pw2_w,
                         const float *pw2_b, const float *gamma) {
    orc_codec_block *b = &c->blocks[l];
    b->dw_w = dw_w; b->dw_b = dw_b; b->norm_w = norm_w; b->norm_b = norm_b; b->pw1_w = pw1_w;
    b->pw1_b = pw1_b; b->pw2_w = pw2_w; b->pw2_b = pw2_b; b->gamma = gamma;
}

/* conv1d over `rows` output rows of x [src_rows][cin] (optionally the x`rep` nearest
 * repetition of it), kernel k, pad (k-1)/2, weight [cout][k][cin] */
static void codec_conv(const float *x, int src_rows, int rep, int cin, const float *w, const float *b, int k,
                       int cout, float *y) {
    const int pad = (k - 1) / 2, rows = src_rows * rep;
#pragma omp parallel for schedule(static)
    for (int t = 0; t < rows; ++t)
        for (int o = 0; o < cout; ++o) {
            float acc = 0.f;
            for (int kk = 0; kk < k; ++kk) {
                const int r = t + kk - pad;
                if (r < 0 || r >= rows) continue;
                const float *xr = x + (size_t)(r / rep) * cin;
                const float *wr = w + ((size_t)o * k + kk) * cin;
                for (int i = 0; i < cin; ++i) acc += xr[i] * wr[i];
            }
            y[(size_t)t * cout + o] = acc + b[o];
        }
}

static void codec_ln(float *x, int rows, int c, const float *w, const float *b) { /* fast::layer_norm, eps 1e-6 */
    for (int t = 0; t < rows; ++t) {
        float *xr = x + (size_t)t * c;
        float mean = 0.f, var = 0.f;
        for (int i = 0; i < c; ++i) mean += xr[i];
        mean /= (float)c;
        for (int i = 0; i < c; ++i) { const float d = xr[i] - mean; var += d * d; }
        var /= (float)c;
        const float rstd = 1.0f / sqrtf(var + 1e-6f);
        for (int i = 0; i < c; ++i) xr[i] = (xr[i] - mean) * rstd * w[i] + b[i];
    }
}

int orc_codec_decode(const orc_codec *c, const int32_t *codes, int T, float *out) {
    if (T <= 0) return fail(ORC_E_VALIDATION, "codes: token sequence length T must be >= 1");
    for (int t = 0; t < T; ++t)
        if (codes[t] < 0 || codes[t] >= c->n_codes) return fail(ORC_E_VALIDATION, "codes: out of range");
    const int H = c->hidden, D = c->dim, F = c->inter;
    float *x = (float *)malloc((size_t)T * H * sizeof(float));
    float *h = (float *)malloc((size_t)T * D * sizeof(float));
    float *t1 = (float *)malloc((size_t)T * D * sizeof(float));
    float *u = (float *)malloc((size_t)T * F * sizeof(float));
    for (int t = 0; t < T; ++t) /* codebook lookup + out_project Conv1d(k=1) (codec.rs:219-221) */
        for (int o = 0; o < H; ++o) {
            float acc = 0.f;
            for (int j = 0; j < c->cdim; ++j) acc += c->codebook[(size_t)codes[t] * c->cdim + j] * c->out_w[(size_t)o * c->cdim + j];
            x[(size_t)t * H + o] = acc + c->out_b[o];
        }
    codec_conv(x, T, 1, H, c->embed_w, c->embed_b, c->embed_k, D, h); /* backbone embed + norm (codec.rs:84-91) */
    codec_ln(h, T, D, c->norm_w, c->norm_b);
    for (int l = 0; l < c->n_layers; ++l) { /* ConvNeXt blocks (convnext.rs:66-73) */
        const orc_codec_block *b = &c->blocks[l];
        const int K = c->dw_k, pad = (K - 1) / 2;
        for (int t = 0; t < T; ++t)
            for (int ch = 0; ch < D; ++ch) {
                float acc = 0.f;
                for (int k = 0; k < K; ++k) {
                    const int r = t + k - pad;
                    if (r >= 0 && r < T) acc += h[(size_t)r * D + ch] * b->dw_w[(size_t)ch * K + k];
                }
                t1[(size_t)t * D + ch] = acc + b->dw_b[ch];
            }
        codec_ln(t1, T, D, b->norm_w, b->norm_b);
        codec_conv(t1, T, 1, D, b->pw1_w, b->pw1_b, 1, F, u);
        for (size_t i = 0; i < (size_t)T * F; ++i) /* nn::gelu: x * (1 + erf(x / sqrt 2)) / 2 */
            u[i] = 0.5f * u[i] * (1.0f + erff(u[i] * 0.70710678118654752f));
        codec_conv(u, T, 1, F, b->pw2_w, b->pw2_b, 1, D, t1);
        for (int t = 0; t < T; ++t)
            for (int ch = 0; ch < D; ++ch) h[(size_t)t * D + ch] += b->gamma[ch] * t1[(size_t)t * D + ch];
    }
    codec_ln(h, T, D, c->fnorm_w, c->fnorm_b);
    codec_conv(h, T, 1, D, c->proj_w, c->proj_b, 1, H, x); /* decoder.1 (codec.rs:224-230) */
    codec_conv(x, T, 2, H, c->up_w, c->up_b, c->up_k, H, out); /* x2 repeat + up conv (codec.rs:233-235) */
    free(x); free(h); free(t1); free(u);
    return ORC_OK;
}
