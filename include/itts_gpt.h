/*
 * itts_gpt.h -- C ABI of the B200 (sm_100a) IndexTTS-2.5 Stage-1 GPT decoder.
 *
 * Drop-in for the decoder / KV-cache / sampler interface of tyrchen/index-tts-rs
 * (crates/core/src/models/mod.rs:41-59 re-exports; the implementations are in
 * crates/core/src/models/gpt.rs and crates/core/src/models/sampler.rs).  Each entry
 * point below names the Rust item it replaces.  A Rust `-sys` crate binds this
 * header one to one.
 *
 * Conventions
 *  - Every call returns an int status: ITTS_OK or one of the ITTS_E_* codes, which
 *    mirror IndexTtsError::{Validation, Mlx (device), WeightLoad, Io}
 *    (crates/core/src/error.rs).  Nothing aborts the process.  The message of the
 *    calling thread's last failure is returned by itts_last_error().
 *  - Handles are opaque.  One host thread owns a handle at a time (the reference keeps
 *    every GPU object on one worker thread, crates/core/src/engine/actor.rs:1-5).
 *    Each itts_gpt owns one CUDA stream on its device; handles on different devices
 *    are independent (no global device state), so one worker per GPU runs in parallel.
 *  - All pointers are host pointers to caller-owned memory unless the name says
 *    otherwise.  Device memory is allocated at load / cache-creation time only.
 */
#ifndef ITTS_GPT_H
#define ITTS_GPT_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes (crates/core/src/error.rs IndexTtsError variants). */
#define ITTS_OK 0
#define ITTS_E_VALIDATION 1 /* IndexTtsError::Validation{field, reason} */
#define ITTS_E_CUDA 2       /* IndexTtsError::Mlx: device execution failure */
#define ITTS_E_WEIGHTLOAD 3 /* IndexTtsError::WeightLoad: missing / mis-shaped tensor */
#define ITTS_E_IO 4         /* IndexTtsError::Io */
#define ITTS_E_TIMEOUT 5    /* a bounded device wait gave up */

/* Tensor dtypes accepted by itts_gpt_from_tensors (safetensors names in parens). */
#define ITTS_DTYPE_F32 0 /* "F32" */
#define ITTS_DTYPE_F16 1 /* "F16" (scales / biases only) */
#define ITTS_DTYPE_U32 2 /* "U32" (packed weights) */
#define ITTS_DTYPE_I32 3 /* "I32" (accepted as packed weights, like loader.rs:919) */

/* Model constants (crates/core/src/models/gpt.rs:31-72, sampler.rs:19). */
#define ITTS_HEAD_DIM 64
#define ITTS_GROUP_SIZE 64
#define ITTS_MEL_VOCAB 8194
#define ITTS_START_TEXT_TOKEN 0
#define ITTS_STOP_TEXT_TOKEN 1
#define ITTS_START_MEL_TOKEN 8192
#define ITTS_STOP_MEL_TOKEN 8193
#define ITTS_BITSET_WORDS 129
#define ITTS_DEFAULT_KV_MAX_SEQ 2048
#define ITTS_MAX_SAMPLE_LOGITS 16384 /* largest logits slice itts_sample_next_token takes */

typedef struct itts_gpt itts_gpt; /* replaces `Gpt` (gpt.rs:436-450) */
typedef struct itts_kv itts_kv;   /* replaces `KvCache` (gpt.rs:74-81), with batch slots */

/* One named host tensor; replaces a `FilteredWeights` entry (loader.rs). */
typedef struct itts_tensor {
    const char *name;   /* reference tensor name, e.g. "gpt.h.0.attn.c_attn.scales" */
    int32_t dtype;      /* ITTS_DTYPE_* */
    int32_t ndim;       /* 1 or 2 */
    int64_t shape[4];
    const void *data;   /* host pointer, row-major */
} itts_tensor;

/* SamplingParams (crates/core/src/config.rs:1283-1320). */
typedef struct itts_sampling_params {
    int32_t greedy;           /* argmax after the repetition penalty */
    uint32_t top_k;           /* 0..=8194, 0 = no top-k filtering (config.rs:614-620) */
    float top_p;              /* 0.01..=1.0 */
    float temperature;        /* 0.05..=2.0 */
    float repetition_penalty; /* 1.0..=50.0 */
    uint32_t max_mel_tokens;  /* 1..=1815 */
} itts_sampling_params;

/* CodePrompt (crates/core/src/models/sampler.rs:287-301); conds is [n_conds, d]. */
typedef struct itts_code_prompt {
    const int32_t *text_tokens;
    int32_t n_text;
    const float *conds;
    int32_t n_conds; /* the reference fixes 3 (gpt.rs:549-553); the benchmark uses 32 */
    int32_t lang_id;
    const int32_t *prior_codes;
    int32_t n_prior;
    int32_t min_codes;
} itts_code_prompt;

/* ---- errors, parameters, host-side sampler state ------------------------------ */

/* Copies the calling thread's last error message (NUL-terminated, truncated to len)
 * and returns its full length. */
size_t itts_last_error(char *buf, size_t len);

/* Range checks of the SamplingParams newtypes (config.rs:454-682, 1309-1310). */
int itts_sampling_params_validate(const itts_sampling_params *params);

/* SamplerRng::new (sampler.rs:41-45): returns the initial state for `seed`. */
uint64_t itts_rng_new(uint64_t seed);
/* SamplerRng::next_f32 (sampler.rs:58-61), advancing *state. */
float itts_rng_next_f32(uint64_t *state);
/* SeenTokenBitSet::new_with_initial_tokens (sampler.rs:110-115): {1, 8192}. */
void itts_seen_initial(uint64_t words[ITTS_BITSET_WORDS]);
/* SeenTokenBitSet::insert (sampler.rs:118-124). */
void itts_seen_insert(uint64_t words[ITTS_BITSET_WORDS], int64_t token_id);

/* ---- model ---------------------------------------------------------------------- */

/* Gpt::load_from_path (gpt.rs:522-525, loader.rs:768-856): reads a gpt_int8
 * safetensors file (F32 or F16 scales/biases) onto `device`. */
int itts_gpt_load(const char *path, int device, itts_gpt **out);
/* Gpt::from_weights (gpt.rs:477-515): the same from caller-owned host tensors. */
int itts_gpt_from_tensors(const itts_tensor *tensors, int32_t n_tensors, int device,
                          itts_gpt **out);
/* Every itts_kv created from `gpt` must be freed before `gpt`. */
void itts_gpt_free(itts_gpt *gpt);
/* Gpt::num_layers (gpt.rs:529-531). */
int32_t itts_gpt_num_layers(const itts_gpt *gpt);
/* Geometry: {n_layers, d, n_heads, ff, mel_vocab, text_vocab, mel_pos_len,
 * text_pos_len, lang_vocab, scales_are_f16}. */
int itts_gpt_dims(const itts_gpt *gpt, int32_t dims[10]);

/* ---- KV cache --------------------------------------------------------------------- */

/* KvCache::new (gpt.rs:102-128) with `max_batch` independent request slots, each of
 * capacity max_seq positions (fp16 K/V in HBM).  max_seq == 0 is a Validation error
 * like gpt.rs:103-108. */
int itts_kv_create(itts_gpt *gpt, int32_t max_seq, int32_t max_batch, itts_kv **out);
void itts_kv_free(itts_kv *kv);
/* KvCache::reset (gpt.rs:131-133) of one slot, or of every slot when slot < 0. */
int itts_kv_reset(itts_kv *kv, int32_t slot);
/* KvCache::valid_len (gpt.rs:137-139). */
int itts_kv_valid_len(const itts_kv *kv, int32_t slot, int32_t *out);
/* KvCache::max_seq (gpt.rs:143-145). */
int32_t itts_kv_max_seq(const itts_kv *kv);
int32_t itts_kv_max_batch(const itts_kv *kv);
/* Which decode-step kernel runs a step of `n_columns` batch columns on this cache:
 * 2 = the persistent grid-wide kernel (up to 4 columns), 3 = the multi-launch GEMM path,
 * 4 = one 6-CTA cluster per attention head, launched once per column for up to 4 columns
 * (the default; ITTS_XK=0 at itts_kv_create turns it off).  No reference counterpart (the
 * reference has one MLX code path); used by tests and the benchmark to name the kernel. */
int32_t itts_kv_decode_kernel(const itts_kv *kv, int32_t n_columns);

/* ---- forward ---------------------------------------------------------------------- */

/* Gpt::prefill_after (gpt.rs:655-696); Gpt::prefill when n_prior == 0 (gpt.rs:636-644).
 * Resets `slot`, runs the causal forward over
 * [conds, <BOS> text <EOS>, <START_MEL>, prior codes] and writes the [mel_vocab] logits
 * of the last position to logits_out (may be NULL). */
int itts_gpt_prefill(itts_gpt *gpt, itts_kv *kv, int32_t slot, const int32_t *text_tokens,
                     int32_t n_text, const float *conds, int32_t n_conds, int32_t lang_id,
                     const int32_t *prior_codes, int32_t n_prior, float *logits_out);

/* Gpt::prefill_after (gpt.rs:655-696) for n requests at once: request r resets slot r
 * and is prefilled from prompts[r] (text, conds, lang, prior codes; min_codes unused),
 * all n in one packed forward (every linear runs once over all positions).  logits_out
 * is [n, mel_vocab] (may be NULL).  The reference prefills one request per call; this
 * entry point gives the same logits and cache contents as n itts_gpt_prefill calls. */
int itts_gpt_prefill_batch(itts_gpt *gpt, itts_kv *kv, int32_t n, const itts_code_prompt *prompts,
                           float *logits_out);

/* Gpt::step (gpt.rs:706-754), batched: for i in 0..n, feeds mel token toks[i] at mel
 * position pos[i] into slot slots[i] (slots distinct), appending one KV position each.
 * logits_out is [n, mel_vocab] (may be NULL). */
int itts_gpt_step(itts_gpt *gpt, itts_kv *kv, int32_t n, const int32_t *slots,
                  const int32_t *toks, const int32_t *pos, float *logits_out);

/* Gpt::teacher_forced / Gpt::code_log_probs (gpt.rs:766-797, replay :800-861): replays
 * `codes` with teacher forcing after the prompt and writes log p(codes[i] | conds, text,
 * codes[..i]) to log_probs_out[i] (may be NULL).  With attention_out != NULL also the text
 * attention of heads (layer 4, head 10) and (5, 10) (align/mod.rs:37) averaged, row-major
 * [n_codes, n_text + 2] (columns <BOS>, text..., <EOS>); the model needs 6 layers and 11
 * heads for it.  `slot` of kv is scratch and is left reset. */
int itts_gpt_teacher_forced(itts_gpt *gpt, itts_kv *kv, int32_t slot, const int32_t *text_tokens,
                            int32_t n_text, const float *conds, int32_t n_conds, int32_t lang_id,
                            const int32_t *codes, int32_t n_codes, float *log_probs_out,
                            float *attention_out);

/* Gpt::alignment_attention (gpt.rs:875-915): the same attention for `codes` generated after
 * prior_codes, replaying only the first 6 layers (align/mod.rs:40); attention_out is
 * [n_codes, n_text + 2].  `slot` of kv is scratch and is left reset. */
int itts_gpt_alignment_attention(itts_gpt *gpt, itts_kv *kv, int32_t slot, const int32_t *text_tokens,
                                 int32_t n_text, const float *conds, int32_t n_conds, int32_t lang_id,
                                 const int32_t *prior_codes, int32_t n_prior, const int32_t *codes,
                                 int32_t n_codes, float *attention_out);

/* ---- sampling and the decode loop --------------------------------------------------- */

/* sample_next_token (sampler.rs:191-284), run by the on-device sampler: applies the
 * repetition penalty to `logits` in place (written back), then greedy argmax or
 * temperature / top-k / top-p / multinomial draw.  *rng_state advances exactly when the
 * reference draws.  1 <= n_logits <= ITTS_MAX_SAMPLE_LOGITS. */
int itts_sample_next_token(itts_gpt *gpt, float *logits, int32_t n_logits,
                           const uint64_t seen_words[ITTS_BITSET_WORDS],
                           const itts_sampling_params *params, uint64_t *rng_state,
                           int32_t *token_out);

/* No counterpart in the reference.  itts_sample_next_token for callers that cannot
 * allocate device memory: a process whose GPU memory belongs to another runtime (a
 * serving framework's allocator, or a fixed budget that must not grow), or a real-time
 * thread, where cudaMalloc / cudaFree would synchronize the device.  It needs no handle
 * and allocates nothing: it runs on the calling thread's current device, on `stream` (a
 * cudaStream_t; NULL is the default stream), and returns once that stream has
 * synchronized.  Its device working set lives in one static array per device (67,072
 * bytes, held by every GPU that loads the library until exit), so
 * 1 <= n_logits <= ITTS_STATIC_SAMPLE_MAX_LOGITS; a longer slice is rejected with
 * ITTS_E_VALIDATION.  The first call on a device does the set-up (it looks up the array's
 * device address and sets the kernel's shared-memory limit); make it before any stream
 * capture.  All calls on one device share the array: calls that overlap on the GPU (from
 * several host threads, or on several streams) race and return wrong results, so
 * serialize them. */
#define ITTS_STATIC_SAMPLE_MAX_LOGITS 16384
int itts_sample_next_token_static(float *logits, int32_t n_logits,
                                  const uint64_t seen_words[ITTS_BITSET_WORDS],
                                  const itts_sampling_params *params, uint64_t *rng_state,
                                  int32_t *token_out, void *stream);

/* generate_codes_after (sampler.rs:340-392); generate_codes (sampler.rs:309-326) is the
 * case n_prior == 0, min_codes == 0.  Prefill, then a CUDA-graph decode step per token
 * with sampling on the device; only the codes return to the host.  codes_out must hold
 * min(max_mel_tokens, 1815 - n_prior) entries (max_codes says how many it holds). */
int itts_generate_codes_after(itts_gpt *gpt, itts_kv *kv, int32_t slot,
                              const itts_code_prompt *prompt,
                              const itts_sampling_params *params, uint64_t *rng_state,
                              int32_t *codes_out, int32_t max_codes, int32_t *n_codes_out);

/* Ragged batched generate: request r runs generate_codes_after in slot r with its own
 * prompt, params[r] and rng_states[r]; all live requests share each decode step and
 * each leaves the batch at its own STOP.  codes_out is [n_req, codes_stride];
 * n_codes_out[r] receives request r's count.  Results equal n_req independent calls. */
int itts_generate_batch(itts_gpt *gpt, itts_kv *kv, int32_t n_req,
                        const itts_code_prompt *prompts, const itts_sampling_params *params,
                        uint64_t *rng_states, int32_t *codes_out, int32_t codes_stride,
                        int32_t *n_codes_out);

/* ---- continuous batching ------------------------------------------------------------ */
/* The reference serves one request at a time on its single engine actor
 * (crates/core/src/engine/actor.rs:1227-1277), each through generate_codes_after
 * (sampler.rs:340-392).  These three calls run that loop for many requests at once on
 * one itts_kv: each of its max_batch slots holds at most one request, requests enter
 * free slots between decode chunks and leave at their own STOP, and every decode step
 * (one CUDA graph over all slots) advances all live requests.  Each request's codes are
 * those of its own generate_codes_after call, within the decoder's tolerances.  A slot
 * holding a live request is rejected by the other slot-taking entry points until it is
 * collected; itts_kv_reset on it cancels the request. */

/* Starts n requests in the given free slots: one packed prefill of their prompts, then
 * each one's first sample (min_codes from the prompt, params[r], rng_states[r]).  The
 * requests already in other slots are not disturbed. */
int itts_batch_admit(itts_gpt *gpt, itts_kv *kv, int32_t n, const int32_t *slots,
                     const itts_code_prompt *prompts, const itts_sampling_params *params,
                     const uint64_t *rng_states);

/* Replays decode steps over all slots, `chunk` at a time, until a live request has
 * finished (STOP, its step limit, or an outgrown KV cache) or max_steps steps ran.
 * finished_out (max_batch entries) receives the slots whose requests finished since the
 * last call, *n_finished their number and *n_live the number still generating.  A
 * request that finished at its first sample (admission) is reported without a step. */
int itts_batch_decode(itts_gpt *gpt, itts_kv *kv, int32_t max_steps, int32_t chunk,
                      int32_t *finished_out, int32_t *n_finished, int32_t *n_live);

/* Takes a finished request out of `slot` and frees the slot: its codes (what
 * generate_codes_after would return; codes_out holds max_codes), the SamplerRng state
 * after its last draw, and *status_out = ITTS_OK or ITTS_E_VALIDATION when the request
 * outgrew the KV cache (gpt.rs:157-165). */
int itts_batch_collect(itts_kv *kv, int32_t slot, int32_t *codes_out, int32_t max_codes,
                       int32_t *n_codes_out, uint64_t *rng_state_out, int32_t *status_out);

/* Device time (CUDA events on the handle's stream) of the last generate call:
 * prefill_ms (all prefills) and decode_ms (first sample through the last step), and the
 * number of decode-step graph launches it made.  After itts_gpt_prefill_batch: prefill_ms
 * is the packed forward (embedded prompts to logits), decode_ms and launches are 0. */
int itts_gpt_last_timing(const itts_gpt *gpt, float *prefill_ms, float *decode_ms,
                         int32_t *decode_launches);

/* ---- SemanticCodec decode (the step after the decoder) -------------------------------- */

typedef struct itts_codec itts_codec; /* replaces `SemanticCodec` (models/codec.rs:104-114) */

/* SemanticCodec::load_from_path (codec.rs:165-175): reads raw/semantic_codec.safetensors
 * (F32 tensors; the encoder's tensors are ignored) onto `device`. */
int itts_codec_load(const char *path, int device, itts_codec **out);
/* SemanticCodec::from_weights (codec.rs:136-162): the same from caller-owned host tensors. */
int itts_codec_from_tensors(const itts_tensor *tensors, int32_t n_tensors, int device,
                            itts_codec **out);
void itts_codec_free(itts_codec *codec);
/* SemanticCodec::num_layers (codec.rs:178-182). */
int32_t itts_codec_num_layers(const itts_codec *codec);
/* Geometry: {n_layers, hidden (1024), backbone dim (384), intermediate (2048), codebook
 * size (8192)} (codec.rs:27-42). */
int itts_codec_dims(const itts_codec *codec, int32_t dims[5]);
/* SemanticCodec::decode (codec.rs:202-239) of one sequence: codes [n_codes] (each in
 * 0..8191) -> out [2 * n_codes][1024] fp32 (row-major), the features the length regulator
 * takes (engine/actor.rs:597-615).  n_codes == 0 is a Validation error like codec.rs:211-216.
 * device_ms (may be NULL) receives the device time of the decode (CUDA events). */
int itts_codec_decode(itts_codec *codec, const int32_t *codes, int32_t n_codes, float *out,
                      float *device_ms);

/* ---- measurement (no reference counterpart) ----------------------------------------- */

/* Replays `iters` times the decode-step forward (everything but the sampler) for slots
 * 0..nb-1 with kv_len cached positions each (the cache contents are whatever the slots
 * hold; the forward appends position kv_len without advancing the slots), and returns
 * the mean device time per step (CUDA events on the handle's stream) and the number of
 * kernel launches per step.  The slots' host-visible state is restored afterwards. */
int itts_bench_decode_forward(itts_gpt *gpt, itts_kv *kv, int32_t nb, int32_t kv_len,
                              int32_t iters, float *ms_per_step, int32_t *launches_per_step);

/* The same for one step of nb <= 4 columns with per-CTA stage timestamps recorded by
 * whichever single-launch decode-step kernel the cache runs for nb (itts_kv_decode_kernel):
 * device globaltimer ns in the grid-wide kernel, SM clock cycles in the cluster kernel.
 * out[cta * events_per_cta + i], 0 where a CTA recorded nothing (the cluster kernel uses fewer
 * CTAs than the reported grid).  out_len must be at least grid * 512.  No reference
 * counterpart (a profiling aid). */
int itts_bench_trace(itts_gpt *gpt, itts_kv *kv, int32_t nb, int32_t kv_len,
                     unsigned long long *out, int32_t out_len, int32_t *grid,
                     int32_t *events_per_cta);

/* ---- test hook (no reference counterpart) ------------------------------------------- */

/* Makes the cache's batch-1 decode steps on the cluster kernel (xk_decode_kernel) start
 * with a bounded wait on a device word that nothing sets: `polls` polls about 1 us apart,
 * after which the step does nothing else and the call returns ITTS_E_TIMEOUT, with the
 * slot's state as before the step.  polls == 0 turns the wait off.  ITTS_E_VALIDATION when
 * polls is outside 0..2^20 or the cache runs another batch-1 kernel. */
int itts_test_stall(itts_gpt *gpt, itts_kv *kv, int32_t polls);

#ifdef __cplusplus
}
#endif
#endif /* ITTS_GPT_H */
