// kernels.h -- host launchers of the decoder kernels (all on one CUDA stream).
#pragma once
#include "common.cuh"

namespace itts {

enum Epilogue : int { EPI_PLAIN = 0, EPI_GELU = 1, EPI_RESID = 2, EPI_QKV = 3 };

// Where a decode step reads and writes its per-request state.
struct DecodeView {
    SlotState *slots;      // [n_slots]
    const int *batch_slot; // batch column -> slot
    int nb;                // batch columns
    int n_slots, n_heads, max_seq, d;
    __half *k_cache, *v_cache;
};

struct ModelView {
    int n_layers, d, n_heads, ff, mel_vocab, text_vocab, lang_vocab, mel_pos_len, text_pos_len;
    bool sb_half;
    const float *text_emb, *lang_emb, *mel_emb, *mel_pos, *text_pos;
    const float *ln_f_w, *ln_f_b, *final_w, *final_b;
    QLinear mel_head;
    const LayerW *layers;  // host array [n_layers]
};

// Decode-step scratch (sized for max_batch columns).
struct DecodeBufs {
    float *x, *q, *attn, *u, *logits;
    float *partials;  // [max_batch][H][max_splits][2 + 64]
    int *counters;    // [max_batch][H], zero between launches
    int max_splits, split_len;
};

// Prefill scratch for one request of up to max_tokens positions.
struct PrefillBufs {
    float *x, *n, *qkv, *attn, *u;
    int max_tokens;
};

void kernels_init();  // one-time function attributes (dynamic shared memory)

// y/x rows are batch columns 0..nb-1 (stride = in / out features).
void launch_gemv(const QLinear &W, bool sb_half, int epi, int ln_mode, const float *ln_w,
                 const float *ln_b, const float *ln2_w, const float *ln2_b, const float *x,
                 float *y, int nb, const DecodeView *dv, int layer, cudaStream_t st);

void launch_embed_step(const ModelView &m, const DecodeView &dv, float *x, cudaStream_t st);

void launch_attn_decode(const DecodeView &dv, int layer, const float *q, DecodeBufs &b,
                        cudaStream_t st);

// Whole decode forward for dv.nb columns: embedding, all layers, double LN + head.
void decode_forward(const ModelView &m, const DecodeView &dv, DecodeBufs &b, cudaStream_t st);

// Prefill of one request already embedded in pb.x[0..T): all layers; K/V of every
// position written to `slot`; logits of position T-1 into logits_row.
void prefill_forward(const ModelView &m, const DecodeView &dv, int slot, int T, PrefillBufs &pb,
                     float *logits_row, cudaStream_t st);

void launch_embed_prefix(const ModelView &m, const int *full_text, int n_full, const float *conds,
                         int n_conds, int lang, const int *prior, int n_prior, float *x,
                         cudaStream_t st);

// Sampler over batch columns 0..nb-1 (logits row b for column b).
struct SampleArgs {
    SlotState *slots;
    const int *batch_slot;
    int nb;
    float *logits;
    int ld_logits;
    int n_logits;
    int after_forward;  // the logits follow a decode step: valid_len += 1 first
    int write_back;     // store the penalized logits back (standalone API)
    int32_t *codes;     // [n_slots][codes_stride]
    int codes_stride;
    int32_t *token_out; // optional [nb]
};
void launch_sample(const SampleArgs &a, cudaStream_t st);

}  // namespace itts
