// kernels.h -- host launchers of the decoder kernels (all on one CUDA stream).
#pragma once
#include <cuda.h>

#include "common.cuh"
#include "mk.h"

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
    MkLin mel_head;
    const MkLayer *layers;    // host array [n_layers]
    const MkLayer *d_layers;  // the same, in device memory (persistent kernel)
};

// The clustered all-SM decode step of one column (xk_decode.cu): launch shape and its
// global exchange buffers (counted fixed-point accumulator words, by step parity).
struct XkConfig {
    int grid = 0, rt = 0, coop = 0;
};
struct XkBufs {  // one allocation: [2][L][d] accumulator words for h and for x, then [grid] launch counters
    unsigned long long *hacc = nullptr;  // counted fixed-point sums of the heads' c_proj partials, by step parity
    unsigned long long *xacc = nullptr;  // the same for the clusters' mlp partials (the next x)
    uint32_t *epoch = nullptr;
    // the K and V caches as 5-D tensors {64, max_seq, heads, slots, layers} for tiled loads of
    // 84 positions x 64 values with the 128-byte swizzle
    alignas(64) CUtensorMap kmap, vmap;
};

// Decode-step scratch (sized for max_batch columns).
struct DecodeBufs {
    float *x, *n, *n2, *q, *attn, *u, *logits;  // q holds [max_batch][3d] (QKV output)
    float *partials;  // [max_batch][H][max_splits][2 + 64]
    int *counters;    // [max_batch][H], zero between launches
    int max_splits, split_len;
    // persistent decode-step kernel state (LL activation buffers, see mk.h)
    uint64_t *qkv_ll, *attn_ll, *ao_ll, *h_ll, *u_ll, *x_ll;
    uint32_t *epoch;  // [grid] launch counters, never reset
    int *err;
    unsigned long long *trace;  // optional per-CTA stage timestamps
    int mk_grid, mk_nslot[MK_MAX_NB + 1];
    float *ws;      // split-K partial sums of the fp16 GEMM: [ws_splits][max_batch][max(3d, ff)]
    int ws_splits;
    XkConfig xk;    // grid > 0: batch-1 steps run on the clustered all-SM kernel (xk_decode.cu)
    XkBufs xkb;
    int *sk_counters;  // split-K counters of the skinny decode GEMMs (zero between launches)
    bool wide_int8;    // steps of 5..SK_MAX_NB columns run the skinny int8 GEMMs
    int stall;         // test hook copied into MkParams::stall (itts_test_stall)
};

// Prefill scratch for one request of up to max_tokens positions.
struct PrefillBufs {
    float *x, *n, *qkv, *attn, *u;
    int max_tokens;
};

// One 64-query tile of the packed prefill attention.
struct AttnTile {
    int row0;  // the request's first row in the packed buffers
    int q0;    // first query (position) of the tile
    int T;     // the request's positions
    int slot;  // its KV-cache slot
};

// Scratch of a packed prefill of several requests (rows = all their positions).
struct PrefillBatch {
    float *x = nullptr, *n = nullptr, *qkv = nullptr, *attn = nullptr, *u = nullptr;
    int *row_slot = nullptr, *row_pos = nullptr;  // [rows] KV destination of each row
    AttnTile *tiles = nullptr;                     // [n_tiles]
    int *last_row = nullptr;                       // [requests] row of each request's last position
    int n_tiles = 0;
    size_t cap_rows = 0, cap_tiles = 0, cap_req = 0;
};

void kernels_init();  // one-time function attributes (dynamic shared memory)

void launch_embed_step(const ModelView &m, const DecodeView &dv, float *x, cudaStream_t st);

void launch_attn_decode(const DecodeView &dv, int layer, const float *q, int q_stride,
                        DecodeBufs &b, cudaStream_t st, int frag);

void launch_layernorm_rows(const float *x, const float *w, const float *b, int rows, int d,
                           float *y, cudaStream_t st);
// The same with an fp16 output (the input of a GEMM).
void launch_layernorm_rows_h(const float *x, const float *w, const float *b, int rows, int d,
                             __half *y, cudaStream_t st);

// y[t, :] = x[t, :] . W^T + bias with an epilogue, for t < T; x is fp16, y is fp32 (fp16
// for EPI_GELU).  In decode mode (dv != null) the QKV epilogue appends row t's K/V to slot
// batch_slot[t] at its valid_len; in prefill mode (dv == null, kv_slot >= 0) row t's K/V go
// to position t of kv_slot.
// ws / ws_splits: split-K workspace for the fp16 GEMM on few rows (decode steps of many
// columns), used when the weight's fp16 copy exists.
void launch_gemm(int epi, const MkLin &W, const __half *x, void *y, int T, const DecodeView *dv,
                 __half *k_cache, __half *v_cache, int kv_slot, int n_slots, int n_heads,
                 int max_seq, int layer, int d, cudaStream_t st, float *ws = nullptr, int ws_splits = 0);

// Decode forward for dv.nb columns: the persistent kernel when nb <= MK_MAX_NB (one
// launch), else the GEMM path (embedding, 7 launches per layer, head).
cudaError_t decode_forward(const ModelView &m, const DecodeView &dv, DecodeBufs &b,
                           cudaStream_t st);
// Decode step of one column on one 6-CTA cluster per attention head (120 CTAs for 20 heads);
// each stage's input is gathered once per cluster (default for batch 1; ITTS_XK=0 at cache
// creation turns it off).
// Fills `out` and returns the grid size, or -1 when the model or the device does not fit it.
int xk_config(const ModelView &m, XkConfig *out);
constexpr int XK_SEQ_MAX_NB = 4;  // steps of up to this many columns: one cluster-kernel launch per column
// The K/V tensor maps of a cache (XkBufs::kmap / vmap).
cudaError_t xk_make_kv_maps(const ModelView &m, __half *k_cache, __half *v_cache, int n_slots, int max_seq,
                            XkBufs &b);
// cuTensorMapEncodeTiled from the driver (null when the driver does not provide it).
using EncodeTiledFn = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                   const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiledFn encode_tiled();
cudaError_t xk_launch(const MkParams &p, const XkConfig &xc, const XkBufs &b, cudaStream_t st);
// The head-major copy of a c_proj (MkLayer::proj_h) from its tiles: n_heads * n_rb chunks.
cudaError_t make_proj_by_head(const MkLin &W, int n_heads, uint8_t *dst, cudaStream_t st);
// The copy of an mlp projection sliced by input (MkLayer::mlp_k): whether the shape allows it,
// its size, and the copy itself.
bool mlp_slice_ok(const MkLin &W, int n_heads);
size_t mlp_slice_bytes(const MkLin &W, int n_heads);
cudaError_t make_mlp_by_slice(const MkLin &W, int n_heads, uint8_t *dst, cudaStream_t st);
// Decode steps of 5..SK_MAX_NB columns on the int8 tiles (decode_wide.cu): the skinny GEMM
// of one linear for nb columns whose activations x are fp16 [n_kc][nb][kc] (K chunk-major,
// [nb][in] for one chunk) in fragment order (each group of 64 inputs permuted like the weight
// bytes); epilogue as launch_gemm's, except EPI_GELU, whose fp16 output is written in that
// layout for the next GEMM, whose K chunk is y_kc.  ws /
// counters: partial sums of linears with several K chunks ([n_kc][nb][out] floats, and
// n_rb counters that are zero between launches).
constexpr int SK_MAX_NB = 64;
bool skinny_ok(const MkLin &W, int nb);
cudaError_t launch_skinny(int epi, const MkLin &W, const __half *x, int nb, void *y, const DecodeView *dv,
                          int layer, int d, float *ws, int *counters, cudaStream_t st, int y_kc = 0);
// LayerNorm of rows into fp16 fragment order (the skinny GEMM's input).
void launch_ln_frag(const float *x, const float *w, const float *b, int rows, int d, __half *y, cudaStream_t st);
void kernels_init_wide();
void kernels_init_decode();   // shared-memory carve-out of the decode step's small kernels
void kernels_init_prefill();
// Whether a step of nb columns reads the fp16 weight copies (made before its first launch).
bool decode_uses_f16_weights(const ModelView &m, const DecodeBufs &b, int nb);
// Number of kernels decode_forward launches for nb columns.
int decode_forward_launches(const ModelView &m, const DecodeBufs &b, int nb);


// Optional extras of a prefill for the teacher-forced replay (gpt.rs:800-915).
struct PrefillHooks {
    int stop_layer = -1;      // >= 0: run layers below it, then only its LN1 + QKV
    int map_layers[2] = {-1, -1}, map_head = 0;  // alignment heads (layer, head)
    int map_q0 = 0, map_k0 = 0, map_k1 = 0;  // query rows map_q0.., key columns [k0, k1)
    float *maps = nullptr;    // [T - map_q0][k1 - k0], the mean of the two heads' maps
    int lp_q0 = -1;           // >= 0: log-probabilities of rows lp_q0.. instead of last logits
    const int *lp_targets = nullptr;  // [T - lp_q0] target code of each row
    float *lp_logits = nullptr;       // [T - lp_q0][mel_vocab] scratch
    float *lp_out = nullptr;          // [T - lp_q0]
};

// Prefill of one request already embedded in pb.x[0..T): all layers; K/V of every
// position written to `slot`; logits of position T-1 into logits_row (unless hooks ask
// for per-row log-probabilities instead).
void prefill_forward(const ModelView &m, const DecodeView &dv, int slot, int T, PrefillBufs &pb,
                     float *logits_row, cudaStream_t st, const PrefillHooks *hk = nullptr);

// Packed prefill of n_req requests (pb filled: rows, tables; pb.x embedded): all layers,
// each row's K/V into its request's slot, logits of request r into row r of `logits`.
void prefill_batch_forward(const ModelView &m, const DecodeView &dv, const PrefillBatch &pb, int n_req,
                           int total, float *logits, cudaStream_t st);
// Causal attention of one request's prompt (T positions of QKV rows; K/V from the cache
// slot the QKV epilogue filled): tensor-core flash attention, fp16 output [T][d].
void launch_attn_prefill_fa(const float *qkv, int T, int slot, const DecodeView &dv, int layer, int d,
                            __half *out, cudaStream_t st);
// launch_gemm for a packed prefill: the QKV epilogue writes row t's K/V to
// (row_slot[t], row_pos[t]).
void launch_gemm_rows(int epi, const MkLin &W, const __half *x, void *y, int T, const int *row_slot,
                      const int *row_pos, __half *k_cache, __half *v_cache, int n_slots, int n_heads,
                      int max_seq, int layer, int d, cudaStream_t st);

// fp16 copy of a linear's weights (dequantized exactly as the int8 GEMMs do).
cudaError_t make_weights_f16(const MkLin &W, __half *w16, cudaStream_t st);
// Rows from which prefill GEMMs use the fp16 weight copy (made on the first such prefill).
constexpr int kGemmF16MinRows = 256;

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
    int small_k;        // every column is greedy or has top_k in 1..64 (below n_logits)
};
void launch_sample(const SampleArgs &a, cudaStream_t st);

// SemanticCodec decode (codec.cu; crates/core/src/models/codec.rs:202-239): device
// pointers of the weights (fp32, the checkpoint's layouts) and the work buffers.
struct CodecBlock {
    const float *dw_w, *dw_b, *norm_w, *norm_b, *pw1_w, *pw1_b, *pw2_w, *pw2_b, *gamma;
};
struct CodecView {
    int n_layers, hidden, dim, inter, cdim, n_codes, embed_k, dw_k, up_k;
    float eps;
    const float *codebook, *out_w, *out_b, *embed_w, *embed_b, *norm_w, *norm_b, *fnorm_w, *fnorm_b;
    const float *proj_w, *proj_b, *up_w, *up_b;
    const CodecBlock *blocks;  // host array [n_layers]
};
struct CodecBufs {
    float *x, *t, *h, *u;  // [cap][hidden], [cap][dim] x 2, [cap][inter]
};
// codes (device, [T], each < n_codes) -> d_out [2T][hidden]
cudaError_t codec_decode_forward(const CodecView &c, const int32_t *d_codes, int T, const CodecBufs &b,
                                 float *d_out, cudaStream_t st);

}  // namespace itts
