// api.cu -- the C ABI declared in include/itts_gpt.h.
//
// Host orchestration of the decoder: weight upload (Gpt::from_weights,
// crates/core/src/models/gpt.rs:477-515), safetensors reading (loader.rs:768-856),
// the batch-slot KV cache (gpt.rs:74-217), prefill / step (gpt.rs:655-754), the
// sampler (sampler.rs:191-284) and the decode loop (sampler.rs:340-392), which
// replays one captured CUDA graph per decode step.  No CPU fallback: every numeric
// step runs in the kernels of decode.cu / prefill.cu / sample.cu.
#include <cuda_runtime.h>
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <array>
#include <cerrno>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>
#include <thread>
#include <unordered_map>
#include <vector>

#include <nvtx3/nvToolsExt.h>

#include "../../include/itts_gpt.h"
#include "kernels.h"

namespace itts {
void kernels_init_sample();
bool sample_small_ok(const itts_sampling_params &p, int n_logits);  // sample.cu
void kernels_init_gemm_tc();
}  // namespace itts

using namespace itts;

static thread_local std::string t_err;

// Host-side NVTX range over one entry point or decode chunk (profilers show the reference's
// per-stage spans, crates/core/src/engine/stream.rs:20-27, as named ranges; nothing is
// recorded unless a profiler is attached).
struct NvtxRange {
    explicit NvtxRange(const char *name) { nvtxRangePushA(name); }
    ~NvtxRange() { nvtxRangePop(); }
    NvtxRange(const NvtxRange &) = delete;
    NvtxRange &operator=(const NvtxRange &) = delete;
};

static int set_err(int code, const std::string &msg) {
    t_err = msg;
    return code;
}
static int validation(const char *field, const std::string &reason) {
    return set_err(ITTS_E_VALIDATION, std::string("validation error on `") + field + "`: " + reason);
}
static int weight_load(const std::string &artifact, const std::string &msg) {
    return set_err(ITTS_E_WEIGHTLOAD, "weight load error in `" + artifact + "`: " + msg);
}

#define CUDA_TRY(x)                                                                       \
    do {                                                                                  \
        cudaError_t e_ = (x);                                                             \
        if (e_ != cudaSuccess)                                                            \
            return set_err(ITTS_E_CUDA, std::string("device error: ") + #x + ": " +       \
                                            cudaGetErrorString(e_));                      \
    } while (0)

#define TRY(x)                 \
    do {                       \
        int rc_ = (x);         \
        if (rc_ != ITTS_OK)    \
            return rc_;        \
    } while (0)

struct itts_gpt {
    int device = 0;
    ModelView m{};
    std::vector<MkLayer> layers;
    MkLayer *d_layers = nullptr;
    void *arena = nullptr;
    __half *w16_arena = nullptr;  // fp16 copies of the layer weights (long prefills), made once
    void *projh_arena = nullptr;  // head-major c_proj copies (batch-1 cluster decode step)
    void *mlpk_arena = nullptr;   // input-sliced mlp copies (the same step)
    bool w16_tried = false;
    cudaStream_t stream = nullptr;
    cudaEvent_t ev[3] = {nullptr, nullptr, nullptr};
    cudaEvent_t evp[2] = {nullptr, nullptr};  // around the forward of a packed prefill
    float last_prefill_ms = 0.f, last_decode_ms = 0.f;
    int last_launches = 0;
    // standalone sampler scratch
    SlotState *d_sstate = nullptr;
    float *d_slogits = nullptr;
    int *d_sidx = nullptr;  // [0] = batch slot 0, [1] = token out
    SlotState *h_sstate = nullptr;
};

struct itts_kv {
    itts_gpt *gpt = nullptr;
    int max_seq = 0, max_batch = 0;
    __half *k = nullptr, *v = nullptr;
    SlotState *d_slots = nullptr;
    int *d_batch_slot = nullptr;
    DecodeBufs db{};
    PrefillBufs pb{};
    int32_t *d_codes = nullptr;
    int codes_stride = 0;
    int *d_text = nullptr, *d_prior = nullptr;
    float *d_conds = nullptr;
    int max_conds = 0;
    std::vector<SlotState> h_state;  // host mirror (authoritative between calls)
    SlotState *h_pinned = nullptr;   // staging [max_batch]
    int32_t *h_i32 = nullptr;        // staging ints
    float *h_f32 = nullptr;          // staging conds
    size_t h_f32_cap = 0;
    std::vector<cudaGraphExec_t> graphs;  // by batch size
    std::vector<cudaGraph_t> graph_defs;
    std::vector<char> graph_failed;       // capture unsupported: launch directly
    size_t ll_bytes = 0;
    // packed prefill of several requests (grown on demand)
    PrefillBatch pbb{};
    int *d_text_b = nullptr, *d_prior_b = nullptr;
    float *d_conds_b = nullptr;
    size_t cap_text_b = 0, cap_prior_b = 0, cap_conds_b = 0;
    // continuous batching (itts_batch_*): per slot, a request admitted and not yet collected
    // (live) and, among those, finished; the slots of an admission's first sample
    std::vector<char> live, finished;
    int *d_admit = nullptr;
};

static void free_prefill_batch(itts_kv *kv) {
    void *dev[] = {kv->pbb.x, kv->pbb.n, kv->pbb.qkv, kv->pbb.attn, kv->pbb.u, kv->pbb.row_slot,
                   kv->pbb.row_pos, kv->pbb.tiles, kv->pbb.last_row, kv->d_text_b, kv->d_prior_b,
                   kv->d_conds_b};
    for (void *p : dev) cudaFree(p);
    kv->pbb = PrefillBatch{};
    kv->d_text_b = kv->d_prior_b = nullptr;
    kv->d_conds_b = nullptr;
    kv->cap_text_b = kv->cap_prior_b = kv->cap_conds_b = 0;
}

// ------------------------------------------------------------------------------
// errors, params, host-side sampler helpers
// ------------------------------------------------------------------------------
extern "C" size_t itts_last_error(char *buf, size_t len) {
    if (buf && len) {
        size_t n = std::min(len - 1, t_err.size());
        std::memcpy(buf, t_err.data(), n);
        buf[n] = 0;
    }
    return t_err.size();
}

extern "C" int itts_sampling_params_validate(const itts_sampling_params *p) {
    if (!p) return validation("params", "null pointer");
    auto fin = [](float v) { return std::isfinite(v); };
    if (!fin(p->temperature) || !(p->temperature >= 0.05f && p->temperature <= 2.0f))
        return validation("temperature", "must be finite and in 0.05..=2.0, got " + std::to_string(p->temperature));
    if (!fin(p->top_p) || !(p->top_p >= 0.01f && p->top_p <= 1.0f))
        return validation("top_p", "must be finite and in 0.01..=1.0, got " + std::to_string(p->top_p));
    if (p->top_k > (uint32_t)ITTS_MEL_VOCAB)
        return validation("top_k", "must be <= 8194, got " + std::to_string(p->top_k));
    if (!fin(p->repetition_penalty) || !(p->repetition_penalty >= 1.0f && p->repetition_penalty <= 50.0f))
        return validation("repetition_penalty", "must be finite and in 1.0..=50.0, got " + std::to_string(p->repetition_penalty));
    if (p->max_mel_tokens < 1 || p->max_mel_tokens > 1815)
        return validation("max_mel_tokens", "must be in 1..=1815, got " + std::to_string(p->max_mel_tokens));
    return ITTS_OK;
}

extern "C" uint64_t itts_rng_new(uint64_t seed) { return seed ^ 0x9E3779B97F4A7C15ULL; }

extern "C" float itts_rng_next_f32(uint64_t *s) {
    *s += 0x9E3779B97F4A7C15ULL;
    uint64_t z = *s;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
    z ^= z >> 31;
    return (float)(uint32_t)(z >> 40) * (1.0f / 16777216.0f);
}

extern "C" void itts_seen_insert(uint64_t *w, int64_t tok) {
    if (tok < 0) return;
    const uint64_t wi = (uint64_t)tok / 64, bi = (uint64_t)tok % 64;
    if (wi < ITTS_BITSET_WORDS) w[wi] |= 1ULL << bi;
}

extern "C" void itts_seen_initial(uint64_t *w) {
    std::memset(w, 0, ITTS_BITSET_WORDS * sizeof(uint64_t));
    itts_seen_insert(w, ITTS_STOP_TEXT_TOKEN);
    itts_seen_insert(w, ITTS_START_MEL_TOKEN);
}

// ------------------------------------------------------------------------------
// model upload
// ------------------------------------------------------------------------------
namespace {

struct TensorTable {
    std::unordered_map<std::string, const itts_tensor *> by_name;
    const itts_tensor *get(const std::string &n) const {
        auto it = by_name.find(n);
        return it == by_name.end() ? nullptr : it->second;
    }
};

std::string shape_str(const itts_tensor *t) {
    std::string s = "[";
    for (int i = 0; i < t->ndim; ++i) s += (i ? ", " : "") + std::to_string(t->shape[i]);
    return s + "]";
}

// tensor_array_shaped (loader.rs:316-331): presence, rank, extents.
int expect(const TensorTable &tt, const std::string &name, std::vector<int64_t> shape,
           const itts_tensor **out, const char *artifact = "gpt_int8.safetensors") {
    const itts_tensor *t = tt.get(name);
    if (!t) return weight_load(artifact, "missing tensor `" + name + "`");
    bool ok = t->ndim == (int)shape.size();
    for (size_t i = 0; ok && i < shape.size(); ++i) ok = t->shape[i] == shape[i];
    if (!ok) {
        std::string e = "[";
        for (size_t i = 0; i < shape.size(); ++i) e += (i ? ", " : "") + std::to_string(shape[i]);
        return weight_load(name, "shape " + shape_str(t) + " != expected " + e + "]");
    }
    if (!t->data) return weight_load(name, "null data pointer");
    *out = t;
    return ITTS_OK;
}

size_t align256(size_t x) { return (x + 255) & ~(size_t)255; }

}  // namespace

static void gpt_destroy(itts_gpt *g) {
    if (!g) return;
    cudaSetDevice(g->device);
    if (g->stream) cudaStreamSynchronize(g->stream);
    for (auto &e : g->ev)
        if (e) cudaEventDestroy(e);
    for (auto &e : g->evp)
        if (e) cudaEventDestroy(e);
    cudaFree(g->arena);
    cudaFree(g->w16_arena);
    cudaFree(g->projh_arena);
    cudaFree(g->mlpk_arena);
    cudaFree(g->d_layers);
    cudaFree(g->d_sstate);
    cudaFree(g->d_slogits);
    cudaFree(g->d_sidx);
    cudaFreeHost(g->h_sstate);
    if (g->stream) cudaStreamDestroy(g->stream);
    delete g;
}

extern "C" int itts_gpt_from_tensors(const itts_tensor *tensors, int32_t n_tensors, int device,
                                     itts_gpt **out) {
    if (!out) return validation("out", "null pointer");
    *out = nullptr;
    if (!tensors || n_tensors <= 0) return weight_load("gpt_int8.safetensors", "no tensors");
    TensorTable tt;
    for (int i = 0; i < n_tensors; ++i)
        if (tensors[i].name) tt.by_name[tensors[i].name] = &tensors[i];

    const itts_tensor *mel = tt.get("mel_embedding.weight");
    if (!mel || mel->ndim != 2)
        return weight_load("gpt_int8.safetensors", "missing tensor `mel_embedding.weight`");
    const int64_t d = mel->shape[1], mel_vocab = mel->shape[0];
    if (d <= 0 || d % 64 != 0 || d > 5120)
        return weight_load("mel_embedding.weight", "model dim must be a positive multiple of 64, <= 5120");
    if (mel_vocab <= ITTS_STOP_MEL_TOKEN || mel_vocab > ITTS_MAX_SAMPLE_LOGITS)
        return weight_load("mel_embedding.weight", "mel vocabulary must hold the STOP token (8193) and be <= 16384");
    int n_layers = 0;
    while (tt.get("gpt.h." + std::to_string(n_layers) + ".ln_1.weight")) ++n_layers;
    if (n_layers == 0) return weight_load("gpt_int8.safetensors", "missing tensor `gpt.h.0.ln_1.weight`");
    const itts_tensor *fcb = tt.get("gpt.h.0.mlp.c_fc.bias");
    if (!fcb || fcb->ndim != 1) return weight_load("gpt_int8.safetensors", "missing tensor `gpt.h.0.mlp.c_fc.bias`");
    const int64_t ff = fcb->shape[0];
    if (ff <= 0 || ff % 64 != 0 || ff > 5120)
        return weight_load("gpt.h.0.mlp.c_fc.bias", "MLP dim must be a positive multiple of 64, <= 5120");
    const itts_tensor *hs = tt.get("mel_head.scales");
    if (!hs) return weight_load("gpt_int8.safetensors", "missing tensor `mel_head.scales`");
    if (hs->dtype != ITTS_DTYPE_F16 && hs->dtype != ITTS_DTYPE_F32)
        return weight_load("mel_head.scales", "scales must be F32 or F16");
    const bool sb_half = hs->dtype == ITTS_DTYPE_F16;

    const itts_tensor *te = tt.get("text_embedding.weight");
    const itts_tensor *le = tt.get("lang_embedding.weight");
    const itts_tensor *mp = tt.get("mel_pos_embedding.emb.weight");
    const itts_tensor *tp = tt.get("text_pos_embedding.emb.weight");
    for (auto pr : {std::make_pair(te, "text_embedding.weight"), std::make_pair(le, "lang_embedding.weight"),
                    std::make_pair(mp, "mel_pos_embedding.emb.weight"), std::make_pair(tp, "text_pos_embedding.emb.weight")})
        if (!pr.first || pr.first->ndim != 2 || pr.first->shape[1] != d)
            return weight_load(pr.second, pr.first ? "shape " + shape_str(pr.first) + " has the wrong model dim"
                                                   : std::string("missing tensor"));

    if (d % 128 != 0 || ff % 128 != 0)
        return weight_load("gpt_int8.safetensors", "model and MLP dims must be multiples of 128");

    // Host-side plan: f32 tensors are copied as they are; every quantized linear is
    // re-tiled (mk.h) into a staging buffer first.
    struct Up { const void *src; size_t bytes; size_t off; std::vector<uint8_t> staged; };
    std::vector<Up> ups;
    ups.reserve(16 + 13 * n_layers);
    auto add = [&](const void *src, size_t bytes) {
        ups.push_back({src, bytes, 0, {}});
        return (int)ups.size() - 1;
    };
    auto f32 = [&](const std::string &name, std::vector<int64_t> shape, int *idx) -> int {
        const itts_tensor *t;
        TRY(expect(tt, name, shape, &t));
        if (t->dtype != ITTS_DTYPE_F32) return weight_load(name, "expected F32");
        size_t n = 1;
        for (auto sdim : shape) n *= (size_t)sdim;
        *idx = add(t->data, n * 4);
        return ITTS_OK;
    };
    struct LinIdx { int tiles, bias; MkLin lin; };
    auto lin = [&](const std::string &p, int64_t o, int64_t in, LinIdx *li) -> int {
        const itts_tensor *w, *sc, *bi;
        TRY(expect(tt, p + ".weight", {o, in / 4}, &w));
        if (w->dtype != ITTS_DTYPE_U32 && w->dtype != ITTS_DTYPE_I32) return weight_load(p + ".weight", "expected U32");
        TRY(expect(tt, p + ".scales", {o, in / 64}, &sc));
        TRY(expect(tt, p + ".biases", {o, in / 64}, &bi));
        const int want = sb_half ? ITTS_DTYPE_F16 : ITTS_DTYPE_F32;
        if (sc->dtype != want || bi->dtype != want)
            return weight_load(p + ".scales", "scales/biases must all share one dtype (F16 or F32)");
        MkLin L{};
        L.out = (int)o;
        L.in = (int)in;
        L.kc = MK_MAX_KC;
        while (in % L.kc != 0) L.kc -= 128;
        L.n_kc = (int)(in / L.kc);
        L.n_rb = (int)((o + 15) / 16);
        L.sbb = sb_half ? 4 : 8;
        L.tile_bytes = mk_tile_bytes(L.kc, L.sbb);
        const itts_tensor *bt;
        TRY(expect(tt, p + ".bias", {o}, &bt));
        if (bt->dtype != ITTS_DTYPE_F32) return weight_load(p + ".bias", "expected F32");
        const float *bias_src = (const float *)bt->data;
        const size_t total = (size_t)L.n_rb * L.n_kc * L.tile_bytes;
        li->tiles = add(nullptr, total);
        std::vector<uint8_t> &buf = ups[li->tiles].staged;
        buf.assign(total, 0);
        const uint8_t *q = (const uint8_t *)w->data;
        const int G = (int)(in / 64);
        const size_t sb_bytes = sb_half ? 2 : 4;
        const uint8_t *sp = (const uint8_t *)sc->data, *bp = (const uint8_t *)bi->data;
        auto work = [&](int rb0, int rb1) {
            for (int rb = rb0; rb < rb1; ++rb)
                for (int m = 0; m < 16; ++m) {
                    const int64_t row = (int64_t)rb * 16 + m;
                    if (row >= o) break;
                    for (int64_t k = 0; k < in; k += 64) {
                        const size_t qo = mk_q_offset(L, (int)row, (int)k);  // group start
                        const uint8_t *src = q + row * in + k;
                        for (int e = 0; e < 64; ++e) buf[qo + frag_pos_host(e)] = src[e];
                        const size_t so = mk_sb_offset(L, (int)row, (int)k);
                        const size_t gi = (size_t)row * G + (size_t)(k / 64);
                        std::memcpy(&buf[so], sp + gi * sb_bytes, sb_bytes);
                        std::memcpy(&buf[so + sb_bytes], bp + gi * sb_bytes, sb_bytes);
                    }
                    for (int kci = 0; kci < L.n_kc; ++kci) {
                        const size_t tile = (size_t)rb * L.n_kc + kci;
                        std::memcpy(&buf[tile * L.tile_bytes + mk_tile_bias_offset(L.kc, L.sbb) + m * 4],
                                    bias_src + row, 4);
                    }
                }
        };
        const int nt = std::max(1, std::min(16, (int)std::thread::hardware_concurrency()));
        std::vector<std::thread> th;
        const int per = (L.n_rb + nt - 1) / nt;
        for (int i = 0; i < nt; ++i) {
            const int a = i * per, b = std::min(L.n_rb, a + per);
            if (a < b) th.emplace_back(work, a, b);
        }
        for (auto &t : th) t.join();
        TRY(f32(p + ".bias", {o}, &li->bias));
        li->lin = L;
        return ITTS_OK;
    };
    int i_te, i_le, i_me, i_mp, i_tp, i_lfw, i_lfb, i_fnw, i_fnb;
    TRY(f32("text_embedding.weight", {te->shape[0], d}, &i_te));
    TRY(f32("lang_embedding.weight", {le->shape[0], d}, &i_le));
    TRY(f32("mel_embedding.weight", {mel_vocab, d}, &i_me));
    TRY(f32("mel_pos_embedding.emb.weight", {mp->shape[0], d}, &i_mp));
    TRY(f32("text_pos_embedding.emb.weight", {tp->shape[0], d}, &i_tp));
    TRY(f32("gpt.ln_f.weight", {d}, &i_lfw));
    TRY(f32("gpt.ln_f.bias", {d}, &i_lfb));
    TRY(f32("final_norm.weight", {d}, &i_fnw));
    TRY(f32("final_norm.bias", {d}, &i_fnb));
    LinIdx head;
    TRY(lin("mel_head", mel_vocab, d, &head));
    struct LayIdx { int l1w, l1b, l2w, l2b; LinIdx a, p, fc, mp; };
    std::vector<LayIdx> li(n_layers);
    for (int i = 0; i < n_layers; ++i) {
        const std::string p = "gpt.h." + std::to_string(i);
        TRY(f32(p + ".ln_1.weight", {d}, &li[i].l1w));
        TRY(f32(p + ".ln_1.bias", {d}, &li[i].l1b));
        TRY(f32(p + ".ln_2.weight", {d}, &li[i].l2w));
        TRY(f32(p + ".ln_2.bias", {d}, &li[i].l2b));
        TRY(lin(p + ".attn.c_attn", 3 * d, d, &li[i].a));
        TRY(lin(p + ".attn.c_proj", d, d, &li[i].p));
        TRY(lin(p + ".mlp.c_fc", ff, d, &li[i].fc));
        TRY(lin(p + ".mlp.c_proj", d, ff, &li[i].mp));
    }

    itts_gpt *g = new itts_gpt();
    g->device = device;
    {
        cudaError_t e = cudaSetDevice(device);
        if (e != cudaSuccess) { delete g; return set_err(ITTS_E_CUDA, std::string("cudaSetDevice: ") + cudaGetErrorString(e)); }
    }
    static bool inited[64] = {false};
    if (device >= 0 && device < 64 && !inited[device]) {
        kernels_init_sample();
        kernels_init_gemm_tc();
        kernels_init_wide();
        kernels_init_decode();
        kernels_init_prefill();
        inited[device] = true;
    }
    size_t total = 0;
    for (auto &u : ups) { u.off = total; total = align256(total + u.bytes); }
    auto fail = [&](cudaError_t e, const char *what) {
        std::string msg = std::string("device error: ") + what + ": " + cudaGetErrorString(e);
        gpt_destroy(g);
        return set_err(ITTS_E_CUDA, msg);
    };
    cudaError_t e;
    if ((e = cudaStreamCreateWithFlags(&g->stream, cudaStreamNonBlocking)) != cudaSuccess) return fail(e, "stream");
    for (auto &ev : g->ev)
        if ((e = cudaEventCreate(&ev)) != cudaSuccess) return fail(e, "event");
    for (auto &ev : g->evp)
        if ((e = cudaEventCreate(&ev)) != cudaSuccess) return fail(e, "event");
    if ((e = cudaMalloc(&g->arena, total)) != cudaSuccess) return fail(e, "weights");
    char *base = (char *)g->arena;
    for (auto &u : ups) {
        const void *src = u.staged.empty() ? u.src : (const void *)u.staged.data();
        if ((e = cudaMemcpy(base + u.off, src, u.bytes, cudaMemcpyHostToDevice)) != cudaSuccess)
            return fail(e, "weight upload");
    }
    auto F = [&](int idx) { return (const float *)(base + ups[idx].off); };
    auto mk = [&](const LinIdx &x) {
        MkLin L = x.lin;
        L.tiles = (const uint8_t *)(base + ups[x.tiles].off);
        L.bias = F(x.bias);
        return L;
    };
    g->layers.resize(n_layers);
    for (int i = 0; i < n_layers; ++i) {
        MkLayer &L = g->layers[i];
        L.ln1_w = F(li[i].l1w); L.ln1_b = F(li[i].l1b); L.ln2_w = F(li[i].l2w); L.ln2_b = F(li[i].l2b);
        L.qkv = mk(li[i].a); L.proj = mk(li[i].p); L.fc = mk(li[i].fc); L.mlp = mk(li[i].mp);
    }
    // head-major copies of the c_proj weights (batch-1 cluster decode step), made once here
    // (about 42 MB for the IndexTTS-2.5 decoder).  Every layer's c_proj must have layer 0's
    // shape; otherwise, or when the copy cannot be made, no layer gets one and batch-1 steps
    // run on the grid-wide kernel instead (xk_config declines a model without the copies).
    // ITTS_XK=0 at load: neither these nor the sliced mlp copies below are made.
    const char *xk_env = getenv("ITTS_XK");
    const bool want_xk = !(xk_env && xk_env[0] == '0');
    if (want_xk) {
        const MkLin &P0 = g->layers[0].proj;
        const size_t per = (size_t)(d / 64) * P0.n_rb * mk_projh_chunk_bytes(P0.sbb);
        bool fits = d % 64 == 0 && P0.n_kc == 1 && P0.kc == (int)d;
        for (int i = 1; i < n_layers && fits; ++i) {
            const MkLin &Pi = g->layers[i].proj;
            fits = Pi.n_kc == P0.n_kc && Pi.kc == P0.kc && Pi.n_rb == P0.n_rb && Pi.sbb == P0.sbb;
        }
        cudaGetLastError();  // a stale error from an earlier call must not read as this copy failing
        cudaError_t pe = fits ? cudaMalloc(&g->projh_arena, per * n_layers) : cudaErrorInvalidValue;
        for (int i = 0; i < n_layers && pe == cudaSuccess; ++i) {
            uint8_t *dst = (uint8_t *)g->projh_arena + per * i;
            pe = make_proj_by_head(g->layers[i].proj, (int)(d / 64), dst, g->stream);
            g->layers[i].proj_h = dst;
        }
        if (pe == cudaSuccess && fits) pe = cudaStreamSynchronize(g->stream);
        if (pe != cudaSuccess) {
            cudaGetLastError();
            cudaFree(g->projh_arena);
            g->projh_arena = nullptr;
            for (int i = 0; i < n_layers; ++i) g->layers[i].proj_h = nullptr;
        }
    }
    // copies of the mlp projections sliced by input (batch-1 cluster decode step: each cluster
    // applies the rows of its own slice of the c_fc output), made once here (about 167 MB for
    // the IndexTTS-2.5 decoder).  Same all-or-nothing rule as the c_proj copies.
    if (want_xk) {
        const int H = (int)(d / 64);
        const MkLin &M0 = g->layers[0].mlp;
        const size_t per = mlp_slice_bytes(M0, H);
        bool fits = mlp_slice_ok(M0, H);
        for (int i = 1; i < n_layers && fits; ++i) {
            const MkLin &Mi = g->layers[i].mlp;
            fits = Mi.in == M0.in && Mi.kc == M0.kc && Mi.n_rb == M0.n_rb && Mi.sbb == M0.sbb;
        }
        cudaGetLastError();
        cudaError_t pe = fits ? cudaMalloc(&g->mlpk_arena, per * n_layers) : cudaErrorInvalidValue;
        for (int i = 0; i < n_layers && pe == cudaSuccess; ++i) {
            uint8_t *dst = (uint8_t *)g->mlpk_arena + per * i;
            pe = make_mlp_by_slice(g->layers[i].mlp, H, dst, g->stream);
            g->layers[i].mlp_k = dst;
        }
        if (pe == cudaSuccess && fits) pe = cudaStreamSynchronize(g->stream);
        if (pe != cudaSuccess) {
            cudaGetLastError();
            cudaFree(g->mlpk_arena);
            g->mlpk_arena = nullptr;
            for (int i = 0; i < n_layers; ++i) g->layers[i].mlp_k = nullptr;
        }
    }
    if ((e = cudaMalloc(&g->d_layers, sizeof(MkLayer) * n_layers)) != cudaSuccess) return fail(e, "layers");
    if ((e = cudaMemcpy(g->d_layers, g->layers.data(), sizeof(MkLayer) * n_layers, cudaMemcpyHostToDevice)) != cudaSuccess)
        return fail(e, "layers");
    ModelView &m = g->m;
    m.n_layers = n_layers; m.d = (int)d; m.n_heads = (int)(d / 64); m.ff = (int)ff;
    m.mel_vocab = (int)mel_vocab; m.text_vocab = (int)te->shape[0]; m.lang_vocab = (int)le->shape[0];
    m.mel_pos_len = (int)mp->shape[0]; m.text_pos_len = (int)tp->shape[0];
    m.sb_half = sb_half;
    m.text_emb = F(i_te); m.lang_emb = F(i_le); m.mel_emb = F(i_me); m.mel_pos = F(i_mp); m.text_pos = F(i_tp);
    m.ln_f_w = F(i_lfw); m.ln_f_b = F(i_lfb); m.final_w = F(i_fnw); m.final_b = F(i_fnb);
    m.mel_head = mk(head);
    m.layers = g->layers.data();
    m.d_layers = g->d_layers;
    if ((e = cudaMalloc(&g->d_sstate, sizeof(SlotState))) != cudaSuccess) return fail(e, "scratch");
    if ((e = cudaMalloc(&g->d_slogits, ITTS_MAX_SAMPLE_LOGITS * sizeof(float))) != cudaSuccess) return fail(e, "scratch");
    if ((e = cudaMalloc(&g->d_sidx, 2 * sizeof(int))) != cudaSuccess) return fail(e, "scratch");
    if ((e = cudaMallocHost(&g->h_sstate, sizeof(SlotState) + 64)) != cudaSuccess) return fail(e, "pinned");
    *out = g;
    return ITTS_OK;
}

// ------------------------------------------------------------------------------
// safetensors (the format gpt_int8.safetensors uses): u64 header length, JSON
// header {name: {dtype, shape, data_offsets}}, raw little-endian data.
// ------------------------------------------------------------------------------
namespace {
struct JsonCursor {
    const char *p, *e;
    void ws() { while (p < e && (*p == ' ' || *p == '\n' || *p == '\r' || *p == '\t')) ++p; }
    bool lit(char c) { ws(); if (p < e && *p == c) { ++p; return true; } return false; }
    bool str(std::string &s) {
        ws();
        if (p >= e || *p != '"') return false;
        ++p;
        s.clear();
        while (p < e && *p != '"') {
            if (*p == '\\' && p + 1 < e) { s.push_back(p[1]); p += 2; } else s.push_back(*p++);
        }
        if (p >= e) return false;
        ++p;
        return true;
    }
    bool num(int64_t &v) {
        ws();
        char *end = nullptr;
        v = strtoll(p, &end, 10);
        if (end == p) return false;
        p = end;
        return true;
    }
    bool skip() {  // skip any JSON value
        ws();
        if (p >= e) return false;
        if (*p == '"') { std::string s; return str(s); }
        if (*p == '{' || *p == '[') {
            const char open = *p, close = open == '{' ? '}' : ']';
            ++p;
            if (lit(close)) return true;
            for (;;) {
                if (open == '{') { std::string k; if (!str(k) || !lit(':')) return false; }
                if (!skip()) return false;
                if (lit(',')) continue;
                return lit(close);
            }
        }
        while (p < e && *p != ',' && *p != '}' && *p != ']') ++p;
        return true;
    }
};
}  // namespace

// Maps a safetensors file (8-byte header length, JSON header, raw data) and hands its
// tensors (F32 / F16 / U32 / I32; others listed with dtype -1) to `use`, then unmaps it.
template <class Use>
static int read_safetensors(const char *path, Use use) {
    if (!path) return validation("path", "null pointer");
    const int fd = open(path, O_RDONLY);
    if (fd < 0) return set_err(ITTS_E_IO, std::string("I/O error at `") + path + "`: " + strerror(errno));
    struct stat sb;
    if (fstat(fd, &sb) != 0 || sb.st_size < 8) { close(fd); return weight_load(path, "file too small"); }
    const size_t size = (size_t)sb.st_size;
    void *map = mmap(nullptr, size, PROT_READ, MAP_PRIVATE, fd, 0);
    close(fd);
    if (map == MAP_FAILED) return set_err(ITTS_E_IO, std::string("I/O error at `") + path + "`: mmap failed");
    const unsigned char *bytes = (const unsigned char *)map;
    uint64_t hlen = 0;
    std::memcpy(&hlen, bytes, 8);
    int rc = ITTS_OK;
    std::vector<itts_tensor> ts;
    std::vector<std::string> names;
    if (hlen > size - 8) {
        rc = weight_load(path, "invalid header length");
    } else {
        JsonCursor c{(const char *)bytes + 8, (const char *)bytes + 8 + hlen};
        const unsigned char *data = bytes + 8 + hlen;
        const size_t data_len = size - 8 - hlen;
        if (!c.lit('{')) rc = weight_load(path, "invalid header");
        while (rc == ITTS_OK && !c.lit('}')) {
            std::string key;
            if (!c.str(key) || !c.lit(':')) { rc = weight_load(path, "invalid header"); break; }
            if (key == "__metadata__") {
                if (!c.skip()) rc = weight_load(path, "invalid header");
            } else {
                itts_tensor t{};
                std::string dtype;
                int64_t off0 = -1, off1 = -1;
                if (!c.lit('{')) { rc = weight_load(path, "invalid header"); break; }
                while (rc == ITTS_OK && !c.lit('}')) {
                    std::string f;
                    if (!c.str(f) || !c.lit(':')) { rc = weight_load(path, "invalid header"); break; }
                    if (f == "dtype") {
                        if (!c.str(dtype)) rc = weight_load(path, "invalid dtype");
                    } else if (f == "shape") {
                        if (!c.lit('[')) { rc = weight_load(path, "invalid shape"); break; }
                        while (!c.lit(']')) {
                            int64_t v;
                            if (!c.num(v) || t.ndim >= 4) { rc = weight_load(path, "invalid shape"); break; }
                            t.shape[t.ndim++] = v;
                            c.lit(',');
                        }
                    } else if (f == "data_offsets") {
                        if (!c.lit('[') || !c.num(off0) || !c.lit(',') || !c.num(off1) || !c.lit(']'))
                            rc = weight_load(path, "invalid data_offsets");
                    } else if (!c.skip()) {
                        rc = weight_load(path, "invalid header");
                    }
                    c.lit(',');
                }
                if (rc != ITTS_OK) break;
                if (dtype == "F32") t.dtype = ITTS_DTYPE_F32;
                else if (dtype == "F16") t.dtype = ITTS_DTYPE_F16;
                else if (dtype == "U32") t.dtype = ITTS_DTYPE_U32;
                else if (dtype == "I32") t.dtype = ITTS_DTYPE_I32;
                else t.dtype = -1;  // other tensors are ignored unless the decoder needs them
                if (off0 < 0 || off1 < off0 || (size_t)off1 > data_len) { rc = weight_load(key, "data offsets out of range"); break; }
                int64_t n = 1;
                for (int i = 0; i < t.ndim; ++i) n *= t.shape[i];
                const int es = t.dtype == ITTS_DTYPE_F16 ? 2 : 4;
                if (t.dtype >= 0 && n * es != off1 - off0) { rc = weight_load(key, "byte size does not match shape"); break; }
                t.data = data + off0;
                names.push_back(key);
                ts.push_back(t);
            }
            c.lit(',');
        }
    }
    if (rc == ITTS_OK) {
        for (size_t i = 0; i < ts.size(); ++i) ts[i].name = names[i].c_str();
        rc = use(ts.data(), (int32_t)ts.size());
    }
    munmap(map, size);
    return rc;
}

extern "C" int itts_gpt_load(const char *path, int device, itts_gpt **out) {
    if (!out) return validation("out", "null pointer");
    *out = nullptr;
    return read_safetensors(path, [&](const itts_tensor *t, int32_t n) {
        return itts_gpt_from_tensors(t, n, device, out);
    });
}

extern "C" void itts_gpt_free(itts_gpt *g) { gpt_destroy(g); }

extern "C" int32_t itts_gpt_num_layers(const itts_gpt *g) { return g ? g->m.n_layers : 0; }

extern "C" int itts_gpt_dims(const itts_gpt *g, int32_t dims[10]) {
    if (!g || !dims) return validation("gpt", "null pointer");
    const ModelView &m = g->m;
    int32_t v[10] = {m.n_layers, m.d, m.n_heads, m.ff, m.mel_vocab, m.text_vocab, m.mel_pos_len,
                     m.text_pos_len, m.lang_vocab, m.sb_half ? 1 : 0};
    std::memcpy(dims, v, sizeof v);
    return ITTS_OK;
}

// ------------------------------------------------------------------------------
// KV cache
// ------------------------------------------------------------------------------
static void kv_destroy(itts_kv *kv) {
    if (!kv) return;
    cudaSetDevice(kv->gpt->device);
    cudaStreamSynchronize(kv->gpt->stream);
    for (auto g : kv->graphs)
        if (g) cudaGraphExecDestroy(g);
    for (auto g : kv->graph_defs)
        if (g) cudaGraphDestroy(g);
    void *dev[] = {kv->k, kv->v, kv->d_slots, kv->d_batch_slot, kv->db.x, kv->db.n, kv->db.n2,
                   kv->db.q, kv->db.attn, kv->db.u, kv->db.logits, kv->db.partials,
                   kv->db.counters, kv->db.qkv_ll, kv->db.epoch, kv->db.err, kv->db.trace, kv->db.ws,
                   kv->db.xkb.hacc, kv->db.sk_counters,
                   kv->pb.x, kv->pb.n, kv->pb.qkv, kv->pb.attn,
                   kv->pb.u, kv->d_codes, kv->d_text, kv->d_prior, kv->d_conds, kv->d_admit};
    for (void *p : dev) cudaFree(p);
    free_prefill_batch(kv);
    cudaFreeHost(kv->h_pinned);
    cudaFreeHost(kv->h_i32);
    cudaFreeHost(kv->h_f32);
    delete kv;
}

static SlotState blank_slot(int max_seq) {
    SlotState s;
    std::memset(&s, 0, sizeof s);
    s.max_seq = max_seq;
    s.temperature = 0.8f;
    s.top_p = 0.8f;
    s.rep_penalty = 1.0f;
    return s;
}

extern "C" int itts_kv_create(itts_gpt *g, int32_t max_seq, int32_t max_batch, itts_kv **out) {
    if (!out) return validation("out", "null pointer");
    *out = nullptr;
    if (!g) return validation("gpt", "null pointer");
    if (max_seq <= 0) return validation("max_seq", "KV cache max_seq must be >= 1");
    if (max_batch <= 0) return validation("max_batch", "must be >= 1");
    CUDA_TRY(cudaSetDevice(g->device));
    const ModelView &m = g->m;
    itts_kv *kv = new itts_kv();
    kv->gpt = g;
    kv->max_seq = max_seq;
    kv->max_batch = max_batch;
    kv->db.split_len = 128;
    kv->db.max_splits = (max_seq + kv->db.split_len - 1) / kv->db.split_len;
    kv->pb.max_tokens = max_seq;
    kv->codes_stride = m.mel_pos_len;
    kv->max_conds = max_seq;
    const size_t kv_elems = (size_t)m.n_layers * max_batch * m.n_heads * max_seq * kHeadDim;
    cudaError_t e = cudaSuccess;
    auto A = [&](void **p, size_t bytes) { if (e == cudaSuccess) e = cudaMalloc(p, bytes); };
    A((void **)&kv->k, kv_elems * 2);
    A((void **)&kv->v, kv_elems * 2);
    A((void **)&kv->d_slots, sizeof(SlotState) * max_batch);
    A((void **)&kv->d_batch_slot, sizeof(int) * max_batch);
    A((void **)&kv->db.x, sizeof(float) * max_batch * m.d);
    A((void **)&kv->db.n, sizeof(float) * max_batch * m.d);
    A((void **)&kv->db.n2, sizeof(float) * max_batch * m.d);
    A((void **)&kv->db.q, sizeof(float) * max_batch * 3 * m.d);
    A((void **)&kv->db.attn, sizeof(float) * max_batch * m.d);
    A((void **)&kv->db.u, sizeof(float) * max_batch * m.ff);
    A((void **)&kv->db.logits, sizeof(float) * max_batch * m.mel_vocab);
    A((void **)&kv->db.partials, sizeof(float) * max_batch * m.n_heads * kv->db.max_splits * 66);
    A((void **)&kv->db.counters, sizeof(int) * max_batch * m.n_heads);
    kv->db.ws_splits = max_batch > MK_MAX_NB ? 16 : 0;  // split-K partials of the wide steps
    kv->db.sk_counters = nullptr;
    {  // steps of 5..64 columns on the int8 tiles (ITTS_WIDE_F16=1: the fp16-copy GEMMs instead)
        const char *f16 = getenv("ITTS_WIDE_F16");
        kv->db.wide_int8 = !(f16 && f16[0] == '1');
    }
    if (max_batch > MK_MAX_NB) A((void **)&kv->db.sk_counters, sizeof(int) * 4096);
    kv->db.ws = nullptr;
    if (kv->db.ws_splits)
        A((void **)&kv->db.ws, sizeof(float) * kv->db.ws_splits * max_batch * std::max(3 * m.d, m.ff));
    // persistent decode-step kernel
    {
        int nsl = 0, grid = 0;
        kv->db.mk_grid = 0;
        for (int nb = 0; nb <= MK_MAX_NB; ++nb) kv->db.mk_nslot[nb] = 0;
        for (int nb = 1; nb <= MK_MAX_NB && nb <= max_batch; ++nb) {
            grid = mk_config(nb, std::max(m.d, m.ff), m.d, m.n_layers, &nsl);
            if (grid <= 0) break;
            kv->db.mk_grid = grid;
            kv->db.mk_nslot[nb] = nsl;
        }
        const size_t L = m.n_layers, NBM = MK_MAX_NB;
        kv->ll_bytes = sizeof(uint64_t) * L * NBM * (3 * m.d + m.d + m.d + m.ff + m.d) +
                       sizeof(uint64_t) * (L * NBM * m.n_heads * MK_MAX_UNITS * MK_PART_WORDS + NBM * m.d);
        A((void **)&kv->db.qkv_ll, kv->ll_bytes);
        if (e == cudaSuccess) {
            uint64_t *b = kv->db.qkv_ll;
            kv->db.attn_ll = b + L * NBM * 3 * m.d;
            kv->db.ao_ll = kv->db.attn_ll + L * NBM * m.n_heads * MK_MAX_UNITS * MK_PART_WORDS;
            kv->db.h_ll = kv->db.ao_ll + L * NBM * m.d;
            kv->db.u_ll = kv->db.h_ll + L * NBM * m.d;
            kv->db.x_ll = kv->db.u_ll + L * NBM * m.ff;  // L + 1 layers of outputs
            e = cudaMemsetAsync(kv->db.qkv_ll, 0, kv->ll_bytes, g->stream);
        }
        A((void **)&kv->db.epoch, sizeof(uint32_t) * std::max(grid, 1024));
        if (e == cudaSuccess) e = cudaMemsetAsync(kv->db.epoch, 0, sizeof(uint32_t) * std::max(grid, 1024), g->stream);
        A((void **)&kv->db.err, sizeof(int) * 4);
        kv->db.trace = nullptr;
        kv->db.stall = 0;
        kv->db.xk = XkConfig{};
        XkConfig xc;
        if (e == cudaSuccess && xk_config(m, &xc) > 0) {
            const size_t L = m.n_layers;
            const size_t bytes = sizeof(unsigned long long) * 4 * L * m.d + sizeof(uint32_t) * xc.grid;
            A((void **)&kv->db.xkb.hacc, bytes);
            if (e == cudaSuccess) {
                XkBufs &x = kv->db.xkb;
                x.xacc = x.hacc + 2 * L * m.d;
                x.epoch = reinterpret_cast<uint32_t *>(x.xacc + 2 * L * m.d);
                e = cudaMemsetAsync(x.hacc, 0, bytes, g->stream);
                // without the K/V tensor maps batch-1 steps use the grid-wide kernel
                if (e == cudaSuccess && xk_make_kv_maps(m, kv->k, kv->v, max_batch, max_seq, x) == cudaSuccess)
                    kv->db.xk = xc;
            }
        }
    }
    A((void **)&kv->pb.x, sizeof(float) * (size_t)max_seq * m.d);
    A((void **)&kv->pb.n, sizeof(float) * (size_t)max_seq * m.d);
    A((void **)&kv->pb.qkv, sizeof(float) * (size_t)max_seq * 3 * m.d);
    A((void **)&kv->pb.attn, sizeof(float) * (size_t)max_seq * m.d);
    A((void **)&kv->pb.u, sizeof(float) * (size_t)max_seq * m.ff);
    A((void **)&kv->d_codes, sizeof(int32_t) * max_batch * kv->codes_stride);
    A((void **)&kv->d_text, sizeof(int) * (m.text_pos_len + 2));
    A((void **)&kv->d_prior, sizeof(int) * (m.mel_pos_len + 2));
    A((void **)&kv->d_conds, sizeof(float) * (size_t)max_seq * m.d);
    A((void **)&kv->d_admit, sizeof(int) * max_batch);
    if (e == cudaSuccess) e = cudaMallocHost((void **)&kv->h_pinned, sizeof(SlotState) * max_batch);
    if (e == cudaSuccess) e = cudaMallocHost((void **)&kv->h_i32, sizeof(int32_t) * (m.text_pos_len + m.mel_pos_len + 4 * max_batch + 8));
    kv->h_f32_cap = (size_t)max_seq * m.d;
    if (e == cudaSuccess) e = cudaMallocHost((void **)&kv->h_f32, sizeof(float) * kv->h_f32_cap);
    if (e == cudaSuccess) e = cudaMemsetAsync(kv->db.counters, 0, sizeof(int) * max_batch * m.n_heads, g->stream);
    if (e == cudaSuccess && kv->db.sk_counters) e = cudaMemsetAsync(kv->db.sk_counters, 0, sizeof(int) * 4096, g->stream);
    kv->h_state.assign(max_batch, blank_slot(max_seq));
    if (e == cudaSuccess) {
        std::memcpy(kv->h_pinned, kv->h_state.data(), sizeof(SlotState) * max_batch);
        e = cudaMemcpyAsync(kv->d_slots, kv->h_pinned, sizeof(SlotState) * max_batch, cudaMemcpyHostToDevice, g->stream);
    }
    if (e == cudaSuccess) e = cudaStreamSynchronize(g->stream);
    if (e != cudaSuccess) {
        std::string msg = std::string("device error: KV cache allocation: ") + cudaGetErrorString(e);
        kv_destroy(kv);
        return set_err(ITTS_E_CUDA, msg);
    }
    kv->live.assign(max_batch, 0);
    kv->finished.assign(max_batch, 0);
    kv->graphs.assign(2 * (max_batch + 1), nullptr);
    kv->graph_defs.assign(2 * (max_batch + 1), nullptr);
    kv->graph_failed.assign(2 * (max_batch + 1), 0);
    *out = kv;
    return ITTS_OK;
}

extern "C" void itts_kv_free(itts_kv *kv) { kv_destroy(kv); }

static int push_slots(itts_kv *kv, const int *slots, int n);

extern "C" int itts_kv_reset(itts_kv *kv, int32_t slot) {
    if (!kv) return validation("kv", "null pointer");
    if (slot >= kv->max_batch) return validation("slot", "out of range");
    std::vector<int> dropped;  // requests of the continuous batch in these slots are cancelled
    for (int s = 0; s < kv->max_batch; ++s)
        if (slot < 0 || s == slot) {
            kv->h_state[s].valid_len = 0;
            if (kv->live[s]) {
                kv->h_state[s].active = 0;
                kv->live[s] = kv->finished[s] = 0;
                dropped.push_back(s);
            }
        }
    if (!dropped.empty()) {
        CUDA_TRY(cudaSetDevice(kv->gpt->device));
        TRY(push_slots(kv, dropped.data(), (int)dropped.size()));
        CUDA_TRY(cudaStreamSynchronize(kv->gpt->stream));
    }
    return ITTS_OK;
}

extern "C" int itts_kv_valid_len(const itts_kv *kv, int32_t slot, int32_t *out) {
    if (!kv || !out) return validation("kv", "null pointer");
    if (slot < 0 || slot >= kv->max_batch) return validation("slot", "out of range");
    *out = kv->h_state[slot].valid_len;
    return ITTS_OK;
}

extern "C" int32_t itts_kv_max_seq(const itts_kv *kv) { return kv ? kv->max_seq : 0; }
extern "C" int32_t itts_kv_max_batch(const itts_kv *kv) { return kv ? kv->max_batch : 0; }
extern "C" int32_t itts_kv_decode_kernel(const itts_kv *kv, int32_t n_columns) {
    if (!kv || n_columns < 1 || n_columns > kv->max_batch) return 0;
    if (n_columns <= XK_SEQ_MAX_NB && kv->db.xk.grid > 0) return 4;
    if (n_columns <= MK_MAX_NB && kv->db.mk_grid > 0 && kv->db.mk_nslot[n_columns] >= 2) return 2;
    return 3;
}

static DecodeView decode_view(itts_kv *kv, int nb) {
    const ModelView &m = kv->gpt->m;
    DecodeView dv;
    dv.slots = kv->d_slots;
    dv.batch_slot = kv->d_batch_slot;
    dv.nb = nb;
    dv.n_slots = kv->max_batch;
    dv.n_heads = m.n_heads;
    dv.max_seq = kv->max_seq;
    dv.d = m.d;
    dv.k_cache = kv->k;
    dv.v_cache = kv->v;
    return dv;
}

// Pushes the host mirror of `slots` to the device.
static int push_slots(itts_kv *kv, const int *slots, int n) {
    cudaStream_t st = kv->gpt->stream;
    CUDA_TRY(cudaStreamSynchronize(st));  // staging buffer reuse
    for (int i = 0; i < n; ++i) {
        kv->h_pinned[i] = kv->h_state[slots[i]];
    }
    for (int i = 0; i < n; ++i)
        CUDA_TRY(cudaMemcpyAsync(kv->d_slots + slots[i], kv->h_pinned + i, sizeof(SlotState),
                                 cudaMemcpyHostToDevice, st));
    return ITTS_OK;
}

static int pull_slots(itts_kv *kv, const int *slots, int n) {
    cudaStream_t st = kv->gpt->stream;
    for (int i = 0; i < n; ++i)
        CUDA_TRY(cudaMemcpyAsync(kv->h_pinned + i, kv->d_slots + slots[i], sizeof(SlotState),
                                 cudaMemcpyDeviceToHost, st));
    CUDA_TRY(cudaStreamSynchronize(st));
    for (int i = 0; i < n; ++i) kv->h_state[slots[i]] = kv->h_pinned[i];
    return ITTS_OK;
}

static int set_batch_slots(itts_kv *kv, const int *slots, int n) {
    cudaStream_t st = kv->gpt->stream;
    CUDA_TRY(cudaStreamSynchronize(st));
    int32_t *h = kv->h_i32;
    for (int i = 0; i < n; ++i) h[i] = slots[i];
    CUDA_TRY(cudaMemcpyAsync(kv->d_batch_slot, h, sizeof(int) * n, cudaMemcpyHostToDevice, st));
    CUDA_TRY(cudaStreamSynchronize(st));
    return ITTS_OK;
}

// A slot that holds a request of the continuous batch (itts_batch_*) belongs to it until
// the request is collected or the slot is reset.
static int check_not_live(const itts_kv *kv, int slot) {
    if (slot >= 0 && slot < kv->max_batch && kv->live[slot])
        return validation("slot", "slot " + std::to_string(slot) +
                                      " holds a request of the continuous batch (collect it or reset the slot first)");
    return ITTS_OK;
}

// ------------------------------------------------------------------------------
// prefill (gpt.rs:535-627, 655-696)
// ------------------------------------------------------------------------------
static int validate_prompt(const ModelView &m, const int32_t *text, int n_text, const float *conds,
                           int n_conds, int lang, const int32_t *prior, int n_prior, int max_seq,
                           int *T_out) {
    if (!text || n_text <= 0) return validation("text_tokens", "text_tokens must not be empty");
    if (n_prior < 0 || (n_prior > 0 && !prior)) return validation("codes", "invalid prior codes");
    if (n_prior + 3 > m.mel_pos_len)
        return validation("codes", std::to_string(n_prior) + " codes exceed the Mel positional capacity");
    const int full = n_text + 2;
    if (full > m.text_pos_len)
        return validation("text_tokens", "text sequence length " + std::to_string(full) + " exceeds " + std::to_string(m.text_pos_len));
    if (!conds || n_conds <= 0) return validation("conds", "expected at least one conditioning row of width " + std::to_string(m.d));
    if (lang < 0 || lang >= m.lang_vocab)
        return validation("lang_id", "lang_id " + std::to_string(lang) + " out of range 0.." + std::to_string(m.lang_vocab));
    for (int i = 0; i < n_text; ++i)
        if (text[i] < 0 || text[i] >= m.text_vocab)
            return validation("text_tokens", "token id " + std::to_string(text[i]) + " out of range");
    for (int i = 0; i < n_prior; ++i)
        if (prior[i] < 0 || prior[i] >= m.mel_vocab)
            return validation("codes", "code " + std::to_string(prior[i]) + " out of range");
    const int T = n_conds + full + 1 + n_prior;
    if (T > max_seq)
        return validation("kv_cache", "sequence length " + std::to_string(T) + " exceeds KV cache capacity " + std::to_string(max_seq));
    *T_out = T;
    return ITTS_OK;
}

// fp16 copies of the four linears of every layer (not the head, which only ever sees a
// few rows), made once, on the first prefill long enough to use them: a long prompt's
// GEMMs then stream fp16 weights by TMA instead of dequantizing int8 tiles in every CTA.
// They take 2 bytes per weight (0.94 GB for the IndexTTS-2.5 decoder); without memory for
// them the int8 GEMMs run instead.
static void ensure_weights_f16(itts_gpt *g) {
    if (g->w16_tried) return;
    g->w16_tried = true;
    size_t total = 0;
    for (const MkLayer &L : g->layers)
        for (const MkLin *W : {&L.qkv, &L.proj, &L.fc, &L.mlp}) total += (size_t)W->out * W->in;
    __half *a = nullptr;
    if (cudaMalloc(&a, total * sizeof(__half)) != cudaSuccess) {
        cudaGetLastError();
        return;
    }
    size_t off = 0;
    cudaError_t e = cudaSuccess;
    for (MkLayer &L : g->layers)
        for (MkLin *W : {&L.qkv, &L.proj, &L.fc, &L.mlp}) {
            if (e == cudaSuccess) e = make_weights_f16(*W, a + off, g->stream);
            W->w16 = a + off;
            off += (size_t)W->out * W->in;
        }
    if (e == cudaSuccess) e = cudaStreamSynchronize(g->stream);
    if (e != cudaSuccess) {  // keep the int8 path
        cudaGetLastError();
        for (MkLayer &L : g->layers)
            for (MkLin *W : {&L.qkv, &L.proj, &L.fc, &L.mlp}) W->w16 = nullptr;
        cudaFree(a);
        return;
    }
    g->w16_arena = a;
}

static int prefill_impl(itts_gpt *g, itts_kv *kv, int slot, const int32_t *text, int n_text,
                        const float *conds, int n_conds, int lang, const int32_t *prior,
                        int n_prior, float *d_logits_row, const PrefillHooks *hooks = nullptr) {
    const ModelView &m = g->m;
    int T = 0;
    TRY(validate_prompt(m, text, n_text, conds, n_conds, lang, prior, n_prior, kv->max_seq, &T));
    cudaStream_t st = g->stream;
    CUDA_TRY(cudaStreamSynchronize(st));  // staging reuse
    int32_t *h = kv->h_i32;
    h[0] = kStartText;
    for (int i = 0; i < n_text; ++i) h[1 + i] = text[i];
    h[n_text + 1] = kStopText;
    int32_t *hp = h + n_text + 2;
    for (int i = 0; i < n_prior; ++i) hp[i] = prior[i];
    const size_t nc = (size_t)n_conds * m.d;
    if (nc > kv->h_f32_cap) return validation("conds", "too many conditioning rows for this KV cache");
    std::memcpy(kv->h_f32, conds, nc * sizeof(float));
    CUDA_TRY(cudaMemcpyAsync(kv->d_text, h, sizeof(int) * (n_text + 2), cudaMemcpyHostToDevice, st));
    if (n_prior)
        CUDA_TRY(cudaMemcpyAsync(kv->d_prior, hp, sizeof(int) * n_prior, cudaMemcpyHostToDevice, st));
    CUDA_TRY(cudaMemcpyAsync(kv->d_conds, kv->h_f32, nc * sizeof(float), cudaMemcpyHostToDevice, st));
    if (T >= kGemmF16MinRows) ensure_weights_f16(g);
    launch_embed_prefix(m, kv->d_text, n_text + 2, kv->d_conds, n_conds, lang, kv->d_prior, n_prior,
                        kv->pb.x, st);
    DecodeView dv = decode_view(kv, 1);
    prefill_forward(m, dv, slot, T, kv->pb, d_logits_row, st, hooks);
    CUDA_TRY(cudaGetLastError());
    kv->h_state[slot].valid_len = T;
    return ITTS_OK;
}

// Prefill of n requests into their slots in one packed forward (prefill_batch.cu): the
// same results as n calls of prefill_impl, with every linear run once over all positions.
// Prompts must have been validated (Ts[r] = positions of request r).
static int prefill_batch_impl(itts_gpt *g, itts_kv *kv, int n, const int *slots, const itts_code_prompt *prompts,
                              const int *Ts, float *d_logits) {
    const ModelView &m = g->m;
    cudaStream_t st = g->stream;
    size_t total = 0, n_tiles = 0, n_text = 0, n_prior = 0, n_conds = 0;
    for (int r = 0; r < n; ++r) {
        total += Ts[r];
        n_tiles += (Ts[r] + 63) / 64;
        n_text += prompts[r].n_text + 2;
        n_prior += prompts[r].n_prior;
        n_conds += (size_t)prompts[r].n_conds * m.d;
    }
    CUDA_TRY(cudaStreamSynchronize(st));  // the scratch may be reallocated
    if (total >= (size_t)kGemmF16MinRows) ensure_weights_f16(g);
    PrefillBatch &pb = kv->pbb;
    if (total > pb.cap_rows || n_tiles > pb.cap_tiles || (size_t)n > pb.cap_req || n_text > kv->cap_text_b ||
        n_prior > kv->cap_prior_b || n_conds > kv->cap_conds_b) {
        const size_t rows = std::max(total, pb.cap_rows), tiles = std::max(n_tiles, pb.cap_tiles);
        const size_t req = std::max((size_t)n, pb.cap_req), nt = std::max(n_text, kv->cap_text_b);
        const size_t np = std::max(n_prior, kv->cap_prior_b) + 1, nc = std::max(n_conds, kv->cap_conds_b);
        free_prefill_batch(kv);
        cudaError_t e = cudaSuccess;
        auto A = [&](void **p, size_t bytes) { if (e == cudaSuccess) e = cudaMalloc(p, bytes); };
        const size_t qrows = std::max(rows, req);
        A((void **)&pb.x, sizeof(float) * rows * m.d);
        A((void **)&pb.n, sizeof(float) * qrows * m.d);
        A((void **)&pb.qkv, sizeof(float) * qrows * 3 * m.d);
        A((void **)&pb.attn, sizeof(float) * qrows * m.d);
        A((void **)&pb.u, sizeof(float) * rows * m.ff);
        A((void **)&pb.row_slot, sizeof(int) * rows);
        A((void **)&pb.row_pos, sizeof(int) * rows);
        A((void **)&pb.tiles, sizeof(AttnTile) * tiles);
        A((void **)&pb.last_row, sizeof(int) * req);
        A((void **)&kv->d_text_b, sizeof(int) * nt);
        A((void **)&kv->d_prior_b, sizeof(int) * np);
        A((void **)&kv->d_conds_b, sizeof(float) * nc);
        if (e != cudaSuccess) {
            free_prefill_batch(kv);
            cudaGetLastError();
            return set_err(ITTS_E_CUDA, std::string("device error: batched prefill scratch: ") + cudaGetErrorString(e));
        }
        pb.cap_rows = rows;
        pb.cap_tiles = tiles;
        pb.cap_req = req;
        kv->cap_text_b = nt;
        kv->cap_prior_b = np;
        kv->cap_conds_b = nc;
    }
    // host tables: tokens (START, text, STOP), prior codes, conds, row destinations, tiles
    std::vector<int> text(n_text), prior(n_prior + 1), row_slot(total), row_pos(total), last(n);
    std::vector<float> conds(n_conds);
    std::vector<AttnTile> tiles;
    tiles.reserve(n_tiles);
    size_t ot = 0, op = 0, oc = 0, row = 0;
    for (int r = 0; r < n; ++r) {
        const itts_code_prompt &pr = prompts[r];
        text[ot] = kStartText;
        for (int i = 0; i < pr.n_text; ++i) text[ot + 1 + i] = pr.text_tokens[i];
        text[ot + pr.n_text + 1] = kStopText;
        for (int i = 0; i < pr.n_prior; ++i) prior[op + i] = pr.prior_codes[i];
        std::memcpy(conds.data() + oc, pr.conds, sizeof(float) * pr.n_conds * m.d);
        for (int t = 0; t < Ts[r]; ++t) {
            row_slot[row + t] = slots[r];
            row_pos[row + t] = t;
        }
        for (int q0 = 0; q0 < Ts[r]; q0 += 64) tiles.push_back(AttnTile{(int)row, q0, Ts[r], slots[r]});
        last[r] = (int)(row + Ts[r] - 1);
        ot += pr.n_text + 2;
        op += pr.n_prior;
        oc += (size_t)pr.n_conds * m.d;
        row += Ts[r];
    }
    CUDA_TRY(cudaMemcpy(kv->d_text_b, text.data(), sizeof(int) * n_text, cudaMemcpyHostToDevice));
    if (n_prior) CUDA_TRY(cudaMemcpy(kv->d_prior_b, prior.data(), sizeof(int) * n_prior, cudaMemcpyHostToDevice));
    CUDA_TRY(cudaMemcpy(kv->d_conds_b, conds.data(), sizeof(float) * n_conds, cudaMemcpyHostToDevice));
    CUDA_TRY(cudaMemcpy(pb.row_slot, row_slot.data(), sizeof(int) * total, cudaMemcpyHostToDevice));
    CUDA_TRY(cudaMemcpy(pb.row_pos, row_pos.data(), sizeof(int) * total, cudaMemcpyHostToDevice));
    CUDA_TRY(cudaMemcpy(pb.tiles, tiles.data(), sizeof(AttnTile) * tiles.size(), cudaMemcpyHostToDevice));
    CUDA_TRY(cudaMemcpy(pb.last_row, last.data(), sizeof(int) * n, cudaMemcpyHostToDevice));
    pb.n_tiles = (int)tiles.size();
    ot = op = oc = row = 0;
    for (int r = 0; r < n; ++r) {  // embeddings (gpt.rs:535-627), each request at its rows
        const itts_code_prompt &pr = prompts[r];
        launch_embed_prefix(m, kv->d_text_b + ot, pr.n_text + 2, kv->d_conds_b + oc, pr.n_conds, pr.lang_id,
                            kv->d_prior_b + op, pr.n_prior, pb.x + row * m.d, st);
        ot += pr.n_text + 2;
        op += pr.n_prior;
        oc += (size_t)pr.n_conds * m.d;
        row += Ts[r];
    }
    DecodeView dv = decode_view(kv, 1);
    CUDA_TRY(cudaEventRecord(g->evp[0], st));
    prefill_batch_forward(m, dv, pb, n, (int)total, d_logits, st);
    CUDA_TRY(cudaEventRecord(g->evp[1], st));
    CUDA_TRY(cudaGetLastError());
    for (int r = 0; r < n; ++r) kv->h_state[slots[r]].valid_len = Ts[r];
    return ITTS_OK;
}

extern "C" int itts_gpt_prefill(itts_gpt *g, itts_kv *kv, int32_t slot, const int32_t *text,
                                int32_t n_text, const float *conds, int32_t n_conds, int32_t lang,
                                const int32_t *prior, int32_t n_prior, float *logits_out) {
    NvtxRange nvtx("itts prefill");
    if (!g || !kv || kv->gpt != g) return validation("gpt", "null pointer or cache of another model");
    if (slot < 0 || slot >= kv->max_batch) return validation("slot", "out of range");
    TRY(check_not_live(kv, slot));
    CUDA_TRY(cudaSetDevice(g->device));
    kv->h_state[slot].valid_len = 0;  // cache.reset() (gpt.rs:664)
    TRY(prefill_impl(g, kv, slot, text, n_text, conds, n_conds, lang, prior, n_prior,
                     kv->db.logits + (size_t)slot * g->m.mel_vocab));
    TRY(push_slots(kv, &slot, 1));
    if (logits_out)
        CUDA_TRY(cudaMemcpyAsync(logits_out, kv->db.logits + (size_t)slot * g->m.mel_vocab,
                                 sizeof(float) * g->m.mel_vocab, cudaMemcpyDeviceToHost, g->stream));
    CUDA_TRY(cudaStreamSynchronize(g->stream));
    return ITTS_OK;
}

extern "C" int itts_gpt_prefill_batch(itts_gpt *g, itts_kv *kv, int32_t n, const itts_code_prompt *prompts,
                                      float *logits_out) {
    NvtxRange nvtx("itts prefill batch");
    if (!g || !kv || kv->gpt != g) return validation("gpt", "null pointer or cache of another model");
    if (n <= 0 || n > kv->max_batch || !prompts) return validation("n", "batch size out of range");
    const ModelView &m = g->m;
    std::vector<int> Ts(n), slots(n);
    for (int r = 0; r < n; ++r) {
        const itts_code_prompt &pr = prompts[r];
        TRY(validate_prompt(m, pr.text_tokens, pr.n_text, pr.conds, pr.n_conds, pr.lang_id, pr.prior_codes,
                            pr.n_prior, kv->max_seq, &Ts[r]));
        slots[r] = r;
    }
    CUDA_TRY(cudaSetDevice(g->device));
    for (int r = 0; r < n; ++r) kv->h_state[r].valid_len = 0;  // cache.reset() (gpt.rs:664)
    TRY(prefill_batch_impl(g, kv, n, slots.data(), prompts, Ts.data(), kv->db.logits));
    TRY(push_slots(kv, slots.data(), n));
    if (logits_out)
        CUDA_TRY(cudaMemcpyAsync(logits_out, kv->db.logits, sizeof(float) * n * m.mel_vocab, cudaMemcpyDeviceToHost,
                                 g->stream));
    CUDA_TRY(cudaStreamSynchronize(g->stream));
    // device time of the packed forward (embedded prompts to logits)
    CUDA_TRY(cudaEventElapsedTime(&g->last_prefill_ms, g->evp[0], g->evp[1]));
    g->last_decode_ms = 0.f;
    g->last_launches = 0;
    return ITTS_OK;
}

// ------------------------------------------------------------------------------
// teacher-forced replay (gpt.rs:756-915)
// ------------------------------------------------------------------------------
// (layer, head) pairs whose text attention is averaged, and the layers alignment replays
// (crates/core/src/align/mod.rs:37-40).
static const int kAlignHeads[2][2] = {{4, 10}, {5, 10}};
static const int kAlignLayers = 6;

// Gpt::replay (gpt.rs:800-861) when alignment_only is false, Gpt::alignment_attention
// (gpt.rs:875-915) when it is true.  The codes fed after <START_MEL> are prior ++
// codes[..n-1]; query rows start at the <START_MEL> row plus n_prior, and row i scores
// codes[i].  `slot` of the cache is scratch and is left reset.
static int replay_impl(itts_gpt *g, itts_kv *kv, int slot, const int32_t *text, int n_text,
                       const float *conds, int n_conds, int lang, const int32_t *prior, int n_prior,
                       const int32_t *codes, int n_codes, bool alignment_only, float *log_probs_out,
                       float *attention_out) {
    NvtxRange nvtx("itts teacher-forced replay");
    if (!g || !kv || kv->gpt != g) return validation("gpt", "null pointer or cache of another model");
    if (slot < 0 || slot >= kv->max_batch) return validation("slot", "out of range");
    TRY(check_not_live(kv, slot));
    if (!codes || n_codes <= 0) return validation("codes", "codes must not be empty");
    if (n_prior < 0 || (n_prior > 0 && !prior)) return validation("prior_codes", "null pointer");
    const ModelView &m = g->m;
    for (int i = 0; i < n_codes; ++i)
        if (codes[i] < 0 || codes[i] >= m.mel_vocab) return validation("codes", "token id out of range");
    if (attention_out && (m.n_layers < kAlignLayers || m.n_heads <= kAlignHeads[0][1]))
        return validation("attention", "the model has no alignment heads (needs 6 layers and 11 heads)");
    std::vector<int32_t> fed(prior, prior + n_prior);
    fed.insert(fed.end(), codes, codes + n_codes - 1);
    CUDA_TRY(cudaSetDevice(g->device));
    const int text_lo = n_conds, text_hi = n_conds + n_text + 2, q0 = text_hi + n_prior;
    const int nk = n_text + 2;
    int32_t *d_targets = nullptr;
    float *d_lp = nullptr, *d_logits = nullptr, *d_maps = nullptr;
    auto release = [&]() { cudaFree(d_targets); cudaFree(d_lp); cudaFree(d_logits); cudaFree(d_maps); };
    cudaError_t e = cudaSuccess;
    const bool want_lp = !alignment_only && log_probs_out;
    if (want_lp) {
        e = cudaMalloc(&d_targets, sizeof(int32_t) * n_codes);
        if (e == cudaSuccess) e = cudaMalloc(&d_lp, sizeof(float) * n_codes);
        if (e == cudaSuccess) e = cudaMalloc(&d_logits, sizeof(float) * (size_t)n_codes * m.mel_vocab);
        if (e == cudaSuccess)
            e = cudaMemcpyAsync(d_targets, codes, sizeof(int32_t) * n_codes, cudaMemcpyHostToDevice, g->stream);
    }
    if (e == cudaSuccess && attention_out) e = cudaMalloc(&d_maps, sizeof(float) * (size_t)n_codes * nk);
    if (e != cudaSuccess) {
        release();
        return set_err(ITTS_E_CUDA, std::string("device error: replay buffers: ") + cudaGetErrorString(e));
    }
    PrefillHooks hk;
    if (attention_out) {
        hk.map_layers[0] = kAlignHeads[0][0];
        hk.map_layers[1] = kAlignHeads[1][0];
        hk.map_head = kAlignHeads[0][1];
        hk.map_q0 = q0;
        hk.map_k0 = text_lo;
        hk.map_k1 = text_hi;
        hk.maps = d_maps;
    }
    if (alignment_only) hk.stop_layer = kAlignLayers - 1;
    if (want_lp) {
        hk.lp_q0 = q0;
        hk.lp_targets = d_targets;
        hk.lp_logits = d_logits;
        hk.lp_out = d_lp;
    }
    kv->h_state[slot].valid_len = 0;
    const int rc = prefill_impl(g, kv, slot, text, n_text, conds, n_conds, lang, fed.data(), (int)fed.size(),
                                kv->db.logits + (size_t)slot * m.mel_vocab, &hk);
    kv->h_state[slot].valid_len = 0;  // cache.reset() (gpt.rs:839, 912)
    if (rc != ITTS_OK) {
        cudaStreamSynchronize(g->stream);
        release();
        return rc;
    }
    e = cudaSuccess;
    if (want_lp) e = cudaMemcpyAsync(log_probs_out, d_lp, sizeof(float) * n_codes, cudaMemcpyDeviceToHost, g->stream);
    if (e == cudaSuccess && attention_out)
        e = cudaMemcpyAsync(attention_out, d_maps, sizeof(float) * (size_t)n_codes * nk, cudaMemcpyDeviceToHost,
                            g->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(g->stream);
    release();
    if (e != cudaSuccess) return set_err(ITTS_E_CUDA, std::string("device error: replay: ") + cudaGetErrorString(e));
    TRY(push_slots(kv, &slot, 1));
    CUDA_TRY(cudaStreamSynchronize(g->stream));
    return ITTS_OK;
}

extern "C" int itts_gpt_teacher_forced(itts_gpt *g, itts_kv *kv, int32_t slot, const int32_t *text,
                                       int32_t n_text, const float *conds, int32_t n_conds, int32_t lang,
                                       const int32_t *codes, int32_t n_codes, float *log_probs_out,
                                       float *attention_out) {
    return replay_impl(g, kv, slot, text, n_text, conds, n_conds, lang, nullptr, 0, codes, n_codes, false,
                       log_probs_out, attention_out);
}

extern "C" int itts_gpt_alignment_attention(itts_gpt *g, itts_kv *kv, int32_t slot, const int32_t *text,
                                            int32_t n_text, const float *conds, int32_t n_conds, int32_t lang,
                                            const int32_t *prior, int32_t n_prior, const int32_t *codes,
                                            int32_t n_codes, float *attention_out) {
    if (!attention_out) return validation("attention", "null pointer");
    return replay_impl(g, kv, slot, text, n_text, conds, n_conds, lang, prior, n_prior, codes, n_codes, true,
                       nullptr, attention_out);
}

// The persistent decode-step kernel's error word is cleared before a run of steps; a
// nonzero value after it means a bounded wait in the kernel gave up.  (Its per-CTA launch
// counters are never reset: the LL tags they generate must not repeat.)
static int reset_step_sync(itts_kv *kv) {
    CUDA_TRY(cudaMemsetAsync(kv->db.err, 0, sizeof(int) * 4, kv->gpt->stream));
    return ITTS_OK;
}

static int check_step_sync(itts_kv *kv) {
    int errw[2] = {0, 0};
    CUDA_TRY(cudaMemcpy(errw, kv->db.err, sizeof(errw), cudaMemcpyDeviceToHost));
    const int err = errw[0] ? errw[0] : errw[1];  // [0]: a bounded wait gave up; [1]: range
    if (err == MK_ERR_RANGE)
        return set_err(ITTS_E_CUDA, "device error: a c_proj or mlp partial of the decode step is finite but "
                                    "outside the fixed-point accumulator's range (|y| >= 2^17)");
    if (err != 0)
        return set_err(ITTS_E_TIMEOUT, "device wait timed out in the decode-step kernel (code " +
                                           std::to_string(err) + ")");
    return ITTS_OK;
}

// ------------------------------------------------------------------------------
// step (gpt.rs:706-754), batched over distinct slots
// ------------------------------------------------------------------------------
extern "C" int itts_gpt_step(itts_gpt *g, itts_kv *kv, int32_t n, const int32_t *slots,
                             const int32_t *toks, const int32_t *pos, float *logits_out) {
    NvtxRange nvtx("itts step");
    if (!g || !kv || kv->gpt != g) return validation("gpt", "null pointer or cache of another model");
    if (n <= 0 || n > kv->max_batch || !slots || !toks || !pos) return validation("n", "batch size out of range");
    const ModelView &m = g->m;
    std::vector<char> seen_slot(kv->max_batch, 0);
    for (int i = 0; i < n; ++i) {
        if (slots[i] < 0 || slots[i] >= kv->max_batch || seen_slot[slots[i]]) return validation("slots", "slots must be distinct and in range");
        TRY(check_not_live(kv, slots[i]));
        seen_slot[slots[i]] = 1;
        if (toks[i] < 0 || toks[i] >= m.mel_vocab)
            return validation("mel_token_id", "mel_token_id " + std::to_string(toks[i]) + " out of range 0.." + std::to_string(m.mel_vocab));
        if (pos[i] < 0 || pos[i] >= m.mel_pos_len)
            return validation("pos_idx", "pos_idx " + std::to_string(pos[i]) + " out of range 0.." + std::to_string(m.mel_pos_len));
        if (kv->h_state[slots[i]].valid_len + 1 > kv->max_seq)
            return validation("kv_cache", "sequence length " + std::to_string(kv->h_state[slots[i]].valid_len + 1) +
                                              " exceeds KV cache capacity " + std::to_string(kv->max_seq));
    }
    CUDA_TRY(cudaSetDevice(g->device));
    for (int i = 0; i < n; ++i) {
        SlotState &s = kv->h_state[slots[i]];
        s.tok = toks[i];
        s.pos = pos[i];
        s.active = 1;
        s.max_seq = kv->max_seq;
    }
    TRY(push_slots(kv, slots, n));
    TRY(set_batch_slots(kv, slots, n));
    TRY(reset_step_sync(kv));
    if (decode_uses_f16_weights(m, kv->db, n)) ensure_weights_f16(g);  // steps above 64 columns
    DecodeView dv = decode_view(kv, n);
    CUDA_TRY(decode_forward(m, dv, kv->db, g->stream));
    CUDA_TRY(cudaStreamSynchronize(g->stream));
    TRY(check_step_sync(kv));
    for (int i = 0; i < n; ++i) kv->h_state[slots[i]].valid_len += 1;
    TRY(push_slots(kv, slots, n));
    if (logits_out)
        CUDA_TRY(cudaMemcpyAsync(logits_out, kv->db.logits, sizeof(float) * n * m.mel_vocab,
                                 cudaMemcpyDeviceToHost, g->stream));
    CUDA_TRY(cudaStreamSynchronize(g->stream));
    return ITTS_OK;
}

// ------------------------------------------------------------------------------
// sampler (sampler.rs:191-284)
// ------------------------------------------------------------------------------
static void fill_params(SlotState &s, const itts_sampling_params *p) {
    s.greedy = p->greedy ? 1 : 0;
    s.top_k = p->top_k;
    s.top_p = p->top_p;
    s.temperature = p->temperature;
    s.rep_penalty = p->repetition_penalty;
}

extern "C" int itts_sample_next_token(itts_gpt *g, float *logits, int32_t n,
                                      const uint64_t *seen, const itts_sampling_params *params,
                                      uint64_t *rng_state, int32_t *token_out) {
    if (!g || !logits || !seen || !rng_state || !token_out) return validation("logits", "null pointer");
    if (n <= 0) return validation("logits", "logits slice must not be empty");
    if (n > ITTS_MAX_SAMPLE_LOGITS) return validation("logits", "at most 16384 logits");
    TRY(itts_sampling_params_validate(params));
    CUDA_TRY(cudaSetDevice(g->device));
    cudaStream_t st = g->stream;
    SlotState &s = *g->h_sstate;
    s = blank_slot(0x7FFFFFFF);
    fill_params(s, params);
    s.active = 1;
    s.max_steps = 0x7FFFFFFF;
    s.rng = *rng_state;
    std::memcpy(s.seen, seen, sizeof(s.seen));
    int *hidx = reinterpret_cast<int *>(reinterpret_cast<char *>(g->h_sstate) + sizeof(SlotState));
    hidx[0] = 0;
    CUDA_TRY(cudaMemcpyAsync(g->d_sstate, &s, sizeof(SlotState), cudaMemcpyHostToDevice, st));
    CUDA_TRY(cudaMemcpyAsync(g->d_sidx, hidx, sizeof(int), cudaMemcpyHostToDevice, st));
    CUDA_TRY(cudaMemcpyAsync(g->d_slogits, logits, sizeof(float) * n, cudaMemcpyHostToDevice, st));
    SampleArgs a{};
    a.slots = g->d_sstate;
    a.batch_slot = g->d_sidx;
    a.nb = 1;
    a.logits = g->d_slogits;
    a.ld_logits = n;
    a.n_logits = n;
    a.after_forward = 0;
    a.write_back = 1;
    a.codes = nullptr;
    a.token_out = g->d_sidx + 1;
    a.small_k = sample_small_ok(*params, n);
    launch_sample(a, st);
    CUDA_TRY(cudaGetLastError());
    CUDA_TRY(cudaMemcpyAsync(logits, g->d_slogits, sizeof(float) * n, cudaMemcpyDeviceToHost, st));
    CUDA_TRY(cudaMemcpyAsync(&s, g->d_sstate, sizeof(SlotState), cudaMemcpyDeviceToHost, st));
    CUDA_TRY(cudaMemcpyAsync(hidx + 1, g->d_sidx + 1, sizeof(int), cudaMemcpyDeviceToHost, st));
    CUDA_TRY(cudaStreamSynchronize(st));
    *rng_state = s.rng;
    *token_out = hidx[1];
    return ITTS_OK;
}

// ------------------------------------------------------------------------------
// decode loop (sampler.rs:340-392): prefill every request, sample, then replay the
// captured decode step until every request stopped.
// ------------------------------------------------------------------------------
static SampleArgs step_sample_args(itts_kv *kv, int nb, int small_k) {
    itts_gpt *g = kv->gpt;
    SampleArgs a{};
    a.slots = kv->d_slots;
    a.batch_slot = kv->d_batch_slot;
    a.nb = nb;
    a.logits = kv->db.logits;
    a.ld_logits = g->m.mel_vocab;
    a.n_logits = g->m.mel_vocab;
    a.after_forward = 1;
    a.write_back = 0;
    a.codes = kv->d_codes;
    a.codes_stride = kv->codes_stride;
    a.small_k = small_k;
    return a;
}

// One decode step: the forward, then the sampler.  (A version that ran the small-k sampler
// inside the batch-1 cluster kernel's last CTA measured slower: one 11-warp CTA after a
// counter hand-off takes longer than the sampler kernel of 32 warps and its launch.)
static cudaError_t launch_step(itts_kv *kv, int nb, int small_k, cudaStream_t st) {
    itts_gpt *g = kv->gpt;
    DecodeView dv = decode_view(kv, nb);
    const cudaError_t e = decode_forward(g->m, dv, kv->db, st);
    if (e != cudaSuccess) return e;
    launch_sample(step_sample_args(kv, nb, small_k), st);
    return cudaGetLastError();
}


// One decode step (forward + sampler) captured as a CUDA graph per batch size and sampler
// variant (small_k: the top-k <= 64 kernel), cached at index 2 nb + small_k.
static int get_graph(itts_kv *kv, int nb, int small_k, cudaGraphExec_t *out) {
    const int gi = 2 * nb + small_k;
    if (kv->graphs[gi]) { *out = kv->graphs[gi]; return ITTS_OK; }
    itts_gpt *g = kv->gpt;
    cudaStream_t st = g->stream;
    cudaGraph_t graph = nullptr;
    CUDA_TRY(cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal));
    const cudaError_t fe = launch_step(kv, nb, small_k, st);
    const cudaError_t ce = cudaStreamEndCapture(st, &graph);
    if (fe != cudaSuccess || ce != cudaSuccess) {
        if (graph) cudaGraphDestroy(graph);
        cudaGetLastError();
        return set_err(ITTS_E_CUDA, std::string("decode-step graph capture failed: ") +
                                        cudaGetErrorString(fe != cudaSuccess ? fe : ce));
    }
    cudaGraphExec_t exec = nullptr;
    CUDA_TRY(cudaGraphInstantiate(&exec, graph, 0));
    kv->graph_defs[gi] = graph;
    kv->graphs[gi] = exec;
    *out = exec;
    return ITTS_OK;
}

static int generate_impl(itts_gpt *g, itts_kv *kv, int n, const int *slots,
                         const itts_code_prompt *prompts, const itts_sampling_params *params,
                         int params_stride, uint64_t *rngs, int32_t *codes_out, int stride,
                         int32_t *n_out) {
    NvtxRange nvtx("itts generate");
    const ModelView &m = g->m;
    if (n <= 0 || n > kv->max_batch) return validation("n_req", "batch size out of range");
    std::vector<int> max_steps(n), Ts(n);
    int max_replays = 0;
    for (int r = 0; r < n; ++r) TRY(check_not_live(kv, slots[r]));
    for (int r = 0; r < n; ++r) {
        const itts_sampling_params *p = params + (size_t)r * params_stride;
        TRY(itts_sampling_params_validate(p));
        const itts_code_prompt &pr = prompts[r];
        const int cap = std::max(0, m.mel_pos_len - 3 - pr.n_prior);
        max_steps[r] = std::min((int)p->max_mel_tokens, cap);  // sampler.rs:348-349
        if (max_steps[r] == 0)
            return validation("max_mel_tokens", "no Mel positions left to generate (max_mel_tokens is 0 or the prior codes fill the capacity)");
        if (stride < max_steps[r]) return validation("codes_out", "buffer smaller than the step limit");
        TRY(validate_prompt(m, pr.text_tokens, pr.n_text, pr.conds, pr.n_conds, pr.lang_id,
                            pr.prior_codes, pr.n_prior, kv->max_seq, &Ts[r]));
        max_replays = std::max(max_replays, max_steps[r] - 1);
    }
    CUDA_TRY(cudaSetDevice(g->device));
    cudaStream_t st = g->stream;
    CUDA_TRY(cudaEventRecord(g->ev[0], st));
    for (int r = 0; r < n; ++r) kv->h_state[slots[r]].valid_len = 0;
    if (n > 1) {  // one packed prefill of all requests
        TRY(prefill_batch_impl(g, kv, n, slots, prompts, Ts.data(), kv->db.logits));
    } else {
        const itts_code_prompt &pr = prompts[0];
        TRY(prefill_impl(g, kv, slots[0], pr.text_tokens, pr.n_text, pr.conds, pr.n_conds,
                         pr.lang_id, pr.prior_codes, pr.n_prior, kv->db.logits));
    }
    CUDA_TRY(cudaEventRecord(g->ev[1], st));
    for (int r = 0; r < n; ++r) {
        SlotState s = blank_slot(kv->max_seq);
        fill_params(s, params + (size_t)r * params_stride);
        s.valid_len = Ts[r];
        s.active = 1;
        s.max_steps = max_steps[r];
        s.min_codes = prompts[r].min_codes;
        s.n_prior = prompts[r].n_prior;
        s.rng = rngs[r];
        itts_seen_initial(s.seen);  // sampler.rs:368: prior codes are not penalised
        kv->h_state[slots[r]] = s;
    }
    TRY(push_slots(kv, slots, n));
    TRY(set_batch_slots(kv, slots, n));
    TRY(reset_step_sync(kv));
    if (decode_uses_f16_weights(m, kv->db, n)) ensure_weights_f16(g);  // made before the capture
    int small_k = 1;  // every request greedy or with top_k <= 64: the small-k sampler
    for (int r = 0; r < n; ++r) small_k &= sample_small_ok(params[(size_t)r * params_stride], m.mel_vocab) ? 1 : 0;
    cudaGraphExec_t graph = nullptr;
    if (!kv->graph_failed[2 * n + small_k] && get_graph(kv, n, small_k, &graph) != ITTS_OK) {
        kv->graph_failed[2 * n + small_k] = 1;  // e.g. a cooperative launch the driver cannot capture
        graph = nullptr;
    }
    SampleArgs a{};
    a.slots = kv->d_slots;
    a.batch_slot = kv->d_batch_slot;
    a.nb = n;
    a.logits = kv->db.logits;
    a.ld_logits = m.mel_vocab;
    a.n_logits = m.mel_vocab;
    a.after_forward = 0;
    a.write_back = 0;
    a.codes = kv->d_codes;
    a.codes_stride = kv->codes_stride;
    a.small_k = small_k;
    launch_sample(a, st);
    CUDA_TRY(cudaGetLastError());
    int launched = 0, chunk = 8;
    for (;;) {
        TRY(pull_slots(kv, slots, n));
        bool any = false;
        for (int r = 0; r < n; ++r) any |= kv->h_state[slots[r]].active != 0;
        if (!any || launched >= max_replays) break;
        const int todo = std::min(chunk, max_replays - launched);
        NvtxRange nvtx_chunk("itts decode chunk");
        for (int i = 0; i < todo; ++i) {
            if (graph) {
                CUDA_TRY(cudaGraphLaunch(graph, st));
            } else {
                CUDA_TRY(launch_step(kv, n, small_k, st));
            }
        }
        launched += todo;
        chunk = std::min(chunk * 2, 64);
    }
    CUDA_TRY(cudaEventRecord(g->ev[2], st));
    int err_slot = -1;
    for (int r = 0; r < n; ++r) {
        SlotState &s = kv->h_state[slots[r]];
        if (s.error && err_slot < 0) err_slot = r;
        rngs[r] = s.rng;
        n_out[r] = s.n_codes;
        s.active = 0;
        if (s.n_codes > 0)
            CUDA_TRY(cudaMemcpyAsync(codes_out + (size_t)r * stride,
                                     kv->d_codes + (size_t)slots[r] * kv->codes_stride,
                                     sizeof(int32_t) * s.n_codes, cudaMemcpyDeviceToHost, st));
    }
    CUDA_TRY(cudaStreamSynchronize(st));
    TRY(check_step_sync(kv));
    CUDA_TRY(cudaEventElapsedTime(&g->last_prefill_ms, g->ev[0], g->ev[1]));
    CUDA_TRY(cudaEventElapsedTime(&g->last_decode_ms, g->ev[1], g->ev[2]));
    g->last_launches = launched;
    if (err_slot >= 0) {
        const SlotState &s = kv->h_state[slots[err_slot]];
        return validation("kv_cache", "sequence length " + std::to_string(s.valid_len + 1) +
                                          " exceeds KV cache capacity " + std::to_string(kv->max_seq));
    }
    return ITTS_OK;
}

extern "C" int itts_generate_codes_after(itts_gpt *g, itts_kv *kv, int32_t slot,
                                         const itts_code_prompt *prompt,
                                         const itts_sampling_params *params, uint64_t *rng_state,
                                         int32_t *codes_out, int32_t max_codes,
                                         int32_t *n_codes_out) {
    if (!g || !kv || kv->gpt != g || !prompt || !params || !rng_state || !codes_out || !n_codes_out)
        return validation("gpt", "null pointer or cache of another model");
    if (slot < 0 || slot >= kv->max_batch) return validation("slot", "out of range");
    int s = slot;
    return generate_impl(g, kv, 1, &s, prompt, params, 0, rng_state, codes_out, max_codes, n_codes_out);
}

extern "C" int itts_generate_batch(itts_gpt *g, itts_kv *kv, int32_t n_req,
                                   const itts_code_prompt *prompts,
                                   const itts_sampling_params *params, uint64_t *rng_states,
                                   int32_t *codes_out, int32_t codes_stride, int32_t *n_codes_out) {
    if (!g || !kv || kv->gpt != g || !prompts || !params || !rng_states || !codes_out || !n_codes_out)
        return validation("gpt", "null pointer or cache of another model");
    if (n_req <= 0 || n_req > kv->max_batch) return validation("n_req", "batch size out of range");
    std::vector<int> slots(n_req);
    for (int i = 0; i < n_req; ++i) slots[i] = i;
    return generate_impl(g, kv, n_req, slots.data(), prompts, params, 1, rng_states, codes_out,
                         codes_stride, n_codes_out);
}

// ------------------------------------------------------------------------------
// continuous batching: requests enter free slots between decode chunks and leave at
// their own STOP, so a worker keeps up to max_batch requests in every decode step
// (replaces the engine actor's one-request-at-a-time loop, actor.rs:1227-1277, around
// generate_codes_after, sampler.rs:340-392)
// ------------------------------------------------------------------------------
static bool slot_small_k(const SlotState &s, int n_logits) {
    itts_sampling_params p{};
    p.greedy = s.greedy;
    p.top_k = s.top_k;
    p.top_p = s.top_p;
    p.temperature = s.temperature;
    p.repetition_penalty = s.rep_penalty;
    p.max_mel_tokens = 1;
    return sample_small_ok(p, n_logits);
}

extern "C" int itts_batch_admit(itts_gpt *g, itts_kv *kv, int32_t n, const int32_t *slots,
                                const itts_code_prompt *prompts, const itts_sampling_params *params,
                                const uint64_t *rng_states) {
    NvtxRange nvtx("itts batch admit");
    if (!g || !kv || kv->gpt != g || !slots || !prompts || !params || !rng_states)
        return validation("gpt", "null pointer or cache of another model");
    if (n <= 0 || n > kv->max_batch) return validation("n", "number of requests out of range");
    const ModelView &m = g->m;
    std::vector<char> seen_slot(kv->max_batch, 0);
    std::vector<int> Ts(n), max_steps(n), sl(slots, slots + n);
    for (int r = 0; r < n; ++r) {
        const int s = slots[r];
        if (s < 0 || s >= kv->max_batch || seen_slot[s]) return validation("slots", "slots must be distinct and in range");
        seen_slot[s] = 1;
        if (kv->live[s]) return validation("slots", "slot " + std::to_string(s) + " holds a request that was not collected");
        TRY(itts_sampling_params_validate(params + r));
        const itts_code_prompt &pr = prompts[r];
        const int cap = std::max(0, m.mel_pos_len - 3 - pr.n_prior);
        max_steps[r] = std::min((int)params[r].max_mel_tokens, cap);  // sampler.rs:348-349
        if (max_steps[r] == 0)
            return validation("max_mel_tokens", "no Mel positions left to generate (max_mel_tokens is 0 or the prior codes fill the capacity)");
        TRY(validate_prompt(m, pr.text_tokens, pr.n_text, pr.conds, pr.n_conds, pr.lang_id, pr.prior_codes,
                            pr.n_prior, kv->max_seq, &Ts[r]));
    }
    CUDA_TRY(cudaSetDevice(g->device));
    cudaStream_t st = g->stream;
    for (int r = 0; r < n; ++r) kv->h_state[slots[r]].valid_len = 0;
    TRY(prefill_batch_impl(g, kv, n, sl.data(), prompts, Ts.data(), kv->db.logits));
    for (int r = 0; r < n; ++r) {
        SlotState s = blank_slot(kv->max_seq);
        fill_params(s, params + r);
        s.valid_len = Ts[r];
        s.active = 1;
        s.max_steps = max_steps[r];
        s.min_codes = prompts[r].min_codes;
        s.n_prior = prompts[r].n_prior;
        s.rng = rng_states[r];
        itts_seen_initial(s.seen);  // sampler.rs:368: prior codes are not penalised
        kv->h_state[slots[r]] = s;
    }
    TRY(push_slots(kv, sl.data(), n));
    {
        int32_t *h = kv->h_i32;  // staging is free: push_slots synchronized the stream
        for (int r = 0; r < n; ++r) h[r] = slots[r];
        CUDA_TRY(cudaMemcpyAsync(kv->d_admit, h, sizeof(int) * n, cudaMemcpyHostToDevice, st));
    }
    int small_k = 1;
    for (int r = 0; r < n; ++r) small_k &= sample_small_ok(params[r], m.mel_vocab) ? 1 : 0;
    SampleArgs a{};  // the first sample of each new request, from its prefill logits (row r)
    a.slots = kv->d_slots;
    a.batch_slot = kv->d_admit;
    a.nb = n;
    a.logits = kv->db.logits;
    a.ld_logits = m.mel_vocab;
    a.n_logits = m.mel_vocab;
    a.after_forward = 0;
    a.write_back = 0;
    a.codes = kv->d_codes;
    a.codes_stride = kv->codes_stride;
    a.small_k = small_k;
    launch_sample(a, st);
    CUDA_TRY(cudaGetLastError());
    CUDA_TRY(cudaStreamSynchronize(st));  // the staging buffer is reused by the next call
    for (int r = 0; r < n; ++r) {
        kv->live[slots[r]] = 1;
        kv->finished[slots[r]] = 0;
    }
    return ITTS_OK;
}

extern "C" int itts_batch_decode(itts_gpt *g, itts_kv *kv, int32_t max_steps, int32_t chunk,
                                 int32_t *finished_out, int32_t *n_finished, int32_t *n_live) {
    NvtxRange nvtx("itts batch decode");
    if (!g || !kv || kv->gpt != g || !finished_out || !n_finished || !n_live)
        return validation("gpt", "null pointer or cache of another model");
    if (max_steps < 0 || chunk <= 0) return validation("max_steps", "max_steps >= 0 and chunk >= 1 required");
    const ModelView &m = g->m;
    const int nb = kv->max_batch;
    *n_finished = 0;
    *n_live = 0;
    std::vector<int> all(nb), live_slots;
    for (int i = 0; i < nb; ++i) {
        all[i] = i;
        if (kv->live[i] && !kv->finished[i]) live_slots.push_back(i);
    }
    if (live_slots.empty()) return ITTS_OK;
    CUDA_TRY(cudaSetDevice(g->device));
    cudaStream_t st = g->stream;
    {  // the step runs every column: slots without a live request must not generate
        std::vector<int> idle;
        for (int i = 0; i < nb; ++i)
            if (!kv->live[i] && kv->h_state[i].active) {
                kv->h_state[i].active = 0;
                idle.push_back(i);
            }
        if (!idle.empty()) TRY(push_slots(kv, idle.data(), (int)idle.size()));
    }
    int small_k = 1;
    for (int s : live_slots) small_k &= slot_small_k(kv->h_state[s], m.mel_vocab) ? 1 : 0;
    TRY(set_batch_slots(kv, all.data(), nb));  // column i = slot i: one graph for any mix
    TRY(reset_step_sync(kv));
    if (decode_uses_f16_weights(m, kv->db, nb)) ensure_weights_f16(g);  // before the capture
    cudaGraphExec_t graph = nullptr;
    if (!kv->graph_failed[2 * nb + small_k] && get_graph(kv, nb, small_k, &graph) != ITTS_OK) {
        kv->graph_failed[2 * nb + small_k] = 1;
        graph = nullptr;
    }
    DecodeView dv = decode_view(kv, nb);
    int steps = 0;
    for (;;) {
        TRY(pull_slots(kv, live_slots.data(), (int)live_slots.size()));
        int nf = 0, nl = 0;
        for (int s : live_slots) {
            if (kv->h_state[s].active) {
                ++nl;
            } else {
                kv->finished[s] = 1;
                finished_out[nf++] = s;
            }
        }
        *n_finished = nf;
        *n_live = nl;
        if (nf > 0 || nl == 0 || steps >= max_steps) break;
        const int todo = std::min(chunk, max_steps - steps);
        NvtxRange nvtx_chunk("itts decode chunk");
        for (int i = 0; i < todo; ++i) {
            if (graph) {
                CUDA_TRY(cudaGraphLaunch(graph, st));
            } else {
                CUDA_TRY(launch_step(kv, nb, small_k, st));
            }
        }
        steps += todo;
    }
    TRY(check_step_sync(kv));
    g->last_launches = steps;
    return ITTS_OK;
}

extern "C" int itts_batch_collect(itts_kv *kv, int32_t slot, int32_t *codes_out, int32_t max_codes,
                                  int32_t *n_codes_out, uint64_t *rng_state_out, int32_t *status_out) {
    if (!kv || !n_codes_out || !rng_state_out || !status_out) return validation("kv", "null pointer");
    if (slot < 0 || slot >= kv->max_batch) return validation("slot", "out of range");
    if (!kv->live[slot] || !kv->finished[slot])
        return validation("slot", "slot " + std::to_string(slot) + " holds no finished request");
    const SlotState &s = kv->h_state[slot];
    if (s.n_codes > 0 && (!codes_out || max_codes < s.n_codes))
        return validation("codes_out", "buffer smaller than the request's " + std::to_string(s.n_codes) + " codes");
    CUDA_TRY(cudaSetDevice(kv->gpt->device));
    if (s.n_codes > 0)
        CUDA_TRY(cudaMemcpy(codes_out, kv->d_codes + (size_t)slot * kv->codes_stride, sizeof(int32_t) * s.n_codes,
                            cudaMemcpyDeviceToHost));
    *n_codes_out = s.n_codes;
    *rng_state_out = s.rng;
    *status_out = s.error ? ITTS_E_VALIDATION : ITTS_OK;
    kv->live[slot] = 0;
    kv->finished[slot] = 0;
    return ITTS_OK;
}

extern "C" int itts_gpt_last_timing(const itts_gpt *g, float *prefill_ms, float *decode_ms,
                                    int32_t *launches) {
    if (!g) return validation("gpt", "null pointer");
    if (prefill_ms) *prefill_ms = g->last_prefill_ms;
    if (decode_ms) *decode_ms = g->last_decode_ms;
    if (launches) *launches = g->last_launches;
    return ITTS_OK;
}

// ------------------------------------------------------------------------------
// measurement: the decode-step forward alone, replayed on fixed inputs
// ------------------------------------------------------------------------------
extern "C" int itts_bench_decode_forward(itts_gpt *g, itts_kv *kv, int32_t nb, int32_t kv_len,
                                         int32_t iters, float *ms, int32_t *launches) {
    if (!g || !kv || kv->gpt != g || !ms) return validation("gpt", "null pointer");
    if (nb <= 0 || nb > kv->max_batch || iters <= 0) return validation("nb", "out of range");
    if (kv_len < 1 || kv_len + 1 > kv->max_seq) return validation("kv_len", "out of range");
    CUDA_TRY(cudaSetDevice(g->device));
    cudaStream_t st = g->stream;
    std::vector<int> slots(nb);
    std::vector<SlotState> saved(nb);
    for (int i = 0; i < nb; ++i) TRY(check_not_live(kv, i));
    for (int i = 0; i < nb; ++i) {
        slots[i] = i;
        saved[i] = kv->h_state[i];
        SlotState &s = kv->h_state[i];
        s.active = 1;
        s.valid_len = kv_len;  // the forward appends position kv_len and reads 0..kv_len
        s.tok = 5 + i;
        s.pos = 2;
        s.max_seq = kv->max_seq;
    }
    TRY(push_slots(kv, slots.data(), nb));
    TRY(set_batch_slots(kv, slots.data(), nb));
    TRY(reset_step_sync(kv));
    if (decode_uses_f16_weights(g->m, kv->db, nb)) ensure_weights_f16(g);
    DecodeView dv = decode_view(kv, nb);
    for (int i = 0; i < 3; ++i) CUDA_TRY(decode_forward(g->m, dv, kv->db, st));
    CUDA_TRY(cudaEventRecord(g->ev[0], st));
    for (int i = 0; i < iters; ++i) CUDA_TRY(decode_forward(g->m, dv, kv->db, st));
    CUDA_TRY(cudaEventRecord(g->ev[1], st));
    CUDA_TRY(cudaStreamSynchronize(st));
    TRY(check_step_sync(kv));
    float t = 0.f;
    CUDA_TRY(cudaEventElapsedTime(&t, g->ev[0], g->ev[1]));
    for (int i = 0; i < nb; ++i) kv->h_state[i] = saved[i];
    TRY(push_slots(kv, slots.data(), nb));
    CUDA_TRY(cudaStreamSynchronize(st));
    *ms = t / (float)iters;
    if (launches) *launches = decode_forward_launches(g->m, kv->db, nb);
    return ITTS_OK;
}

// Runs one decode-step forward like itts_bench_decode_forward with per-CTA stage
// timestamps (globaltimer, ns) recorded by the persistent kernel; out receives
// [grid][events_per_cta] values (0 where a CTA recorded nothing).
extern "C" int itts_bench_trace(itts_gpt *g, itts_kv *kv, int32_t nb, int32_t kv_len,
                                unsigned long long *out, int32_t out_len, int32_t *grid,
                                int32_t *events_per_cta) {
    if (!g || !kv || kv->gpt != g || !out || !grid || !events_per_cta) return validation("gpt", "null pointer");
    if (kv->db.mk_grid <= 0 || nb > MK_MAX_NB) return validation("nb", "the persistent kernel is not used for this batch");
    const size_t n = (size_t)kv->db.mk_grid * MK_TRACE_EVENTS;
    if ((size_t)out_len < n) return validation("out_len", "too small");
    CUDA_TRY(cudaSetDevice(g->device));
    unsigned long long *d = nullptr;
    CUDA_TRY(cudaMalloc(&d, n * sizeof(unsigned long long)));
    cudaMemset(d, 0, n * sizeof(unsigned long long));
    kv->db.trace = d;
    float ms = 0.f;
    int32_t launches = 0;
    const int rc = itts_bench_decode_forward(g, kv, nb, kv_len, 1, &ms, &launches);
    kv->db.trace = nullptr;
    if (rc == ITTS_OK) cudaMemcpy(out, d, n * sizeof(unsigned long long), cudaMemcpyDeviceToHost);
    cudaFree(d);
    *grid = kv->db.mk_grid;
    *events_per_cta = MK_TRACE_EVENTS;
    return rc;
}

// Test hook: batch-1 steps on the cluster kernel first poll a device word that nothing sets,
// `polls` times about 1 us apart, then give up and report ITTS_E_TIMEOUT.  The step's cached
// CUDA graphs are dropped so that generate captures the new value.
extern "C" int itts_test_stall(itts_gpt *g, itts_kv *kv, int32_t polls) {
    if (!g || !kv || kv->gpt != g) return validation("gpt", "null pointer or cache of another model");
    if (polls < 0 || polls > (1 << 20)) return validation("polls", "out of range 0..2^20");
    if (kv->db.xk.grid <= 0) return validation("polls", "this cache does not run the cluster kernel");
    CUDA_TRY(cudaSetDevice(g->device));
    CUDA_TRY(cudaStreamSynchronize(g->stream));
    for (size_t i = 0; i < kv->graphs.size(); ++i) {
        if (kv->graphs[i]) cudaGraphExecDestroy(kv->graphs[i]);
        if (kv->graph_defs[i]) cudaGraphDestroy(kv->graph_defs[i]);
        kv->graphs[i] = nullptr;
        kv->graph_defs[i] = nullptr;
    }
    kv->db.stall = polls;
    return ITTS_OK;
}


// ------------------------------------------------------------------------------
// SemanticCodec decode (crates/core/src/models/codec.rs:104-239): the step after the
// decoder turns its mel codes into the features the length regulator takes
// (crates/core/src/engine/actor.rs:597-615).
// ------------------------------------------------------------------------------
struct itts_codec {
    int device = 0;
    CodecView v{};
    std::vector<CodecBlock> blocks;
    void *arena = nullptr;
    cudaStream_t stream = nullptr;
    cudaEvent_t ev[2] = {nullptr, nullptr};
    CodecBufs bufs{};
    int32_t *d_codes = nullptr;
    float *d_out = nullptr;
    int cap = 0;
    float last_ms = 0.f;
};

static void codec_free_bufs(itts_codec *c) {
    void *p[] = {c->bufs.x, c->bufs.t, c->bufs.h, c->bufs.u, c->d_codes, c->d_out};
    for (void *q : p) cudaFree(q);
    c->bufs = CodecBufs{};
    c->d_codes = nullptr;
    c->d_out = nullptr;
    c->cap = 0;
}

extern "C" void itts_codec_free(itts_codec *c) {
    if (!c) return;
    cudaSetDevice(c->device);
    if (c->stream) cudaStreamSynchronize(c->stream);
    codec_free_bufs(c);
    cudaFree(c->arena);
    for (cudaEvent_t e : c->ev)
        if (e) cudaEventDestroy(e);
    if (c->stream) cudaStreamDestroy(c->stream);
    delete c;
}

extern "C" int itts_codec_from_tensors(const itts_tensor *tensors, int32_t n_tensors, int device, itts_codec **out) {
    if (!out) return validation("out", "null pointer");
    *out = nullptr;
    if (!tensors || n_tensors <= 0) return validation("tensors", "no tensors");
    const char *art = "semantic_codec.safetensors";
    TensorTable tt;
    for (int i = 0; i < n_tensors; ++i)
        if (tensors[i].name) tt.by_name[tensors[i].name] = &tensors[i];
    // geometry from the tensors (codec.rs:27-42: hidden 1024, dim 384, 2048, codebook 8192 x 8)
    const itts_tensor *cb = tt.get("quantizer.quantizers.0.codebook.weight");
    const itts_tensor *pw1 = tt.get("decoder.0.convnext.0.pwconv1.weight");
    const itts_tensor *emb = tt.get("decoder.0.embed.weight");
    if (!cb || cb->ndim != 2) return weight_load(art, "missing tensor `quantizer.quantizers.0.codebook.weight`");
    if (!pw1 || pw1->ndim != 2) return weight_load(art, "missing tensor `decoder.0.convnext.0.pwconv1.weight`");
    if (!emb || emb->ndim != 3) return weight_load(art, "missing tensor `decoder.0.embed.weight`");
    const int64_t ncode = cb->shape[0], cdim = cb->shape[1], inter = pw1->shape[0], dim = pw1->shape[1];
    const int64_t embed_k = emb->shape[1], hidden = emb->shape[2];
    int n_layers = 0;
    while (tt.get("decoder.0.convnext." + std::to_string(n_layers) + ".gamma")) ++n_layers;
    const itts_tensor *upw = tt.get("up.weight");
    const int64_t up_k = upw && upw->ndim == 3 ? upw->shape[1] : 3;
    const itts_tensor *dw0 = tt.get("decoder.0.convnext.0.dwconv.weight");
    const int64_t dw_k = dw0 && dw0->ndim == 3 ? dw0->shape[1] : 7;
    struct Up { const itts_tensor *t; size_t off; };
    std::vector<Up> ups;
    auto f32 = [&](const std::string &name, std::vector<int64_t> shape, int *idx) -> int {
        const itts_tensor *t = nullptr;
        TRY(expect(tt, name, shape, &t, art));
        if (t->dtype != ITTS_DTYPE_F32) return weight_load(name, "expected F32");
        *idx = (int)ups.size();
        ups.push_back({t, 0});
        return ITTS_OK;
    };
    int i_cb, i_ow, i_ob, i_ew, i_eb, i_nw, i_nb, i_fw, i_fb, i_pw, i_pb, i_uw, i_ub;
    TRY(f32("quantizer.quantizers.0.codebook.weight", {ncode, cdim}, &i_cb));
    TRY(f32("quantizer.quantizers.0.out_project.weight", {hidden, 1, cdim}, &i_ow));
    TRY(f32("quantizer.quantizers.0.out_project.bias", {hidden}, &i_ob));
    TRY(f32("decoder.0.embed.weight", {dim, embed_k, hidden}, &i_ew));
    TRY(f32("decoder.0.embed.bias", {dim}, &i_eb));
    TRY(f32("decoder.0.norm.weight", {dim}, &i_nw));
    TRY(f32("decoder.0.norm.bias", {dim}, &i_nb));
    TRY(f32("decoder.0.final_layer_norm.weight", {dim}, &i_fw));
    TRY(f32("decoder.0.final_layer_norm.bias", {dim}, &i_fb));
    TRY(f32("decoder.1.weight", {hidden, dim}, &i_pw));
    TRY(f32("decoder.1.bias", {hidden}, &i_pb));
    TRY(f32("up.weight", {hidden, up_k, hidden}, &i_uw));
    TRY(f32("up.bias", {hidden}, &i_ub));
    std::vector<std::array<int, 9>> bi(n_layers);
    for (int l = 0; l < n_layers; ++l) {
        const std::string pre = "decoder.0.convnext." + std::to_string(l) + ".";
        TRY(f32(pre + "dwconv.weight", {dim, dw_k, 1}, &bi[l][0]));
        TRY(f32(pre + "dwconv.bias", {dim}, &bi[l][1]));
        TRY(f32(pre + "norm.weight", {dim}, &bi[l][2]));
        TRY(f32(pre + "norm.bias", {dim}, &bi[l][3]));
        TRY(f32(pre + "pwconv1.weight", {inter, dim}, &bi[l][4]));
        TRY(f32(pre + "pwconv1.bias", {inter}, &bi[l][5]));
        TRY(f32(pre + "pwconv2.weight", {dim, inter}, &bi[l][6]));
        TRY(f32(pre + "pwconv2.bias", {dim}, &bi[l][7]));
        TRY(f32(pre + "gamma", {dim}, &bi[l][8]));
    }
    if (n_layers < 1 || dim % 32 || embed_k % 2 == 0 || up_k % 2 == 0 || dw_k % 2 == 0)
        return weight_load(art, "unsupported codec geometry");
    CUDA_TRY(cudaSetDevice(device));
    itts_codec *c = new itts_codec();
    c->device = device;
    size_t total = 0;
    for (auto &u : ups) {
        u.off = total;
        size_t n = 1;
        for (int k = 0; k < u.t->ndim; ++k) n *= (size_t)u.t->shape[k];
        total = align256(total + n * 4);
    }
    cudaError_t e = cudaMalloc(&c->arena, total);
    for (size_t k = 0; k < ups.size() && e == cudaSuccess; ++k) {
        size_t n = 1;
        for (int j = 0; j < ups[k].t->ndim; ++j) n *= (size_t)ups[k].t->shape[j];
        e = cudaMemcpy((char *)c->arena + ups[k].off, ups[k].t->data, n * 4, cudaMemcpyHostToDevice);
    }
    if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking);
    if (e == cudaSuccess) e = cudaEventCreate(&c->ev[0]);
    if (e == cudaSuccess) e = cudaEventCreate(&c->ev[1]);
    if (e != cudaSuccess) {
        const std::string msg = std::string("device error: codec upload: ") + cudaGetErrorString(e);
        itts_codec_free(c);
        return set_err(ITTS_E_CUDA, msg);
    }
    auto F = [&](int i) { return (const float *)((const char *)c->arena + ups[i].off); };
    CodecView &v = c->v;
    v.n_layers = n_layers; v.hidden = (int)hidden; v.dim = (int)dim; v.inter = (int)inter; v.cdim = (int)cdim;
    v.n_codes = (int)ncode; v.embed_k = (int)embed_k; v.dw_k = (int)dw_k; v.up_k = (int)up_k;
    v.eps = 1e-6f;  // CODEC_NORM_EPS (codec.rs:39), convnext.rs:18
    v.codebook = F(i_cb); v.out_w = F(i_ow); v.out_b = F(i_ob); v.embed_w = F(i_ew); v.embed_b = F(i_eb);
    v.norm_w = F(i_nw); v.norm_b = F(i_nb); v.fnorm_w = F(i_fw); v.fnorm_b = F(i_fb);
    v.proj_w = F(i_pw); v.proj_b = F(i_pb); v.up_w = F(i_uw); v.up_b = F(i_ub);
    c->blocks.resize(n_layers);
    for (int l = 0; l < n_layers; ++l) {
        CodecBlock &b = c->blocks[l];
        b.dw_w = F(bi[l][0]); b.dw_b = F(bi[l][1]); b.norm_w = F(bi[l][2]); b.norm_b = F(bi[l][3]);
        b.pw1_w = F(bi[l][4]); b.pw1_b = F(bi[l][5]); b.pw2_w = F(bi[l][6]); b.pw2_b = F(bi[l][7]);
        b.gamma = F(bi[l][8]);
    }
    v.blocks = c->blocks.data();
    *out = c;
    return ITTS_OK;
}

extern "C" int itts_codec_load(const char *path, int device, itts_codec **out) {
    if (!out) return validation("out", "null pointer");
    *out = nullptr;
    return read_safetensors(path, [&](const itts_tensor *t, int32_t n) {
        return itts_codec_from_tensors(t, n, device, out);
    });
}

extern "C" int32_t itts_codec_num_layers(const itts_codec *c) { return c ? c->v.n_layers : 0; }

extern "C" int itts_codec_dims(const itts_codec *c, int32_t dims[5]) {
    if (!c || !dims) return validation("codec", "null pointer");
    dims[0] = c->v.n_layers;
    dims[1] = c->v.hidden;
    dims[2] = c->v.dim;
    dims[3] = c->v.inter;
    dims[4] = c->v.n_codes;
    return ITTS_OK;
}

extern "C" int itts_codec_decode(itts_codec *c, const int32_t *codes, int32_t n_codes, float *out, float *device_ms) {
    if (!c || !out) return validation("codec", "null pointer");
    if (!codes || n_codes <= 0) return validation("codes", "token sequence length T must be >= 1");
    for (int i = 0; i < n_codes; ++i)
        if (codes[i] < 0 || codes[i] >= c->v.n_codes)
            return validation("codes", "code " + std::to_string(codes[i]) + " out of range 0.." +
                                           std::to_string(c->v.n_codes));
    NvtxRange nvtx("itts codec decode");
    CUDA_TRY(cudaSetDevice(c->device));
    cudaStream_t st = c->stream;
    if (n_codes > c->cap) {  // work buffers grow with the longest sequence seen
        CUDA_TRY(cudaStreamSynchronize(st));
        codec_free_bufs(c);
        const size_t T = (size_t)n_codes;
        const CodecView &v = c->v;
        cudaError_t e = cudaSuccess;
        auto A = [&](void **p, size_t bytes) { if (e == cudaSuccess) e = cudaMalloc(p, bytes); };
        A((void **)&c->bufs.x, T * v.hidden * 4);
        A((void **)&c->bufs.t, T * v.dim * 4);
        A((void **)&c->bufs.h, T * v.dim * 4);
        A((void **)&c->bufs.u, T * v.inter * 4);
        A((void **)&c->d_codes, T * 4);
        A((void **)&c->d_out, 2 * T * v.hidden * 4);
        if (e != cudaSuccess) {
            codec_free_bufs(c);
            return set_err(ITTS_E_CUDA, std::string("device error: codec buffers: ") + cudaGetErrorString(e));
        }
        c->cap = n_codes;
    }
    CUDA_TRY(cudaMemcpyAsync(c->d_codes, codes, sizeof(int32_t) * n_codes, cudaMemcpyHostToDevice, st));
    CUDA_TRY(cudaEventRecord(c->ev[0], st));
    CUDA_TRY(codec_decode_forward(c->v, c->d_codes, n_codes, c->bufs, c->d_out, st));
    CUDA_TRY(cudaEventRecord(c->ev[1], st));
    CUDA_TRY(cudaMemcpyAsync(out, c->d_out, sizeof(float) * 2 * (size_t)n_codes * c->v.hidden,
                             cudaMemcpyDeviceToHost, st));
    CUDA_TRY(cudaStreamSynchronize(st));
    CUDA_TRY(cudaEventElapsedTime(&c->last_ms, c->ev[0], c->ev[1]));
    if (device_ms) *device_ms = c->last_ms;
    return ITTS_OK;
}

// ------------------------------------------------------------------------------
// Sampling without allocation.
//
// Some callers of the sampler cannot allocate device memory: a process whose GPU memory
// belongs to another runtime (a serving framework's caching allocator, or a fixed memory
// budget that must never grow), and a real-time audio thread, where cudaMalloc and
// cudaFree synchronize the whole device and would stall playback.  Such a caller cannot
// create an itts_gpt either, since loading allocates.  itts_sample_next_token_static runs
// the same on-device sampler as itts_sample_next_token, with the device-side working set
// of that kernel (its state block, the batch index, the token word and the logits it
// penalizes in place) in the file-scope array below instead of buffers of a handle.
// Every GPU that loads this library holds the array (67,072 bytes) until the process
// exits.
// ------------------------------------------------------------------------------
namespace {
constexpr size_t kStaticIdxOff = (sizeof(SlotState) + 255) / 256 * 256;  // state block at 0
constexpr size_t kStaticLogitsOff = kStaticIdxOff + 256;
constexpr size_t kStaticBytes = kStaticLogitsOff + sizeof(float) * ITTS_STATIC_SAMPLE_MAX_LOGITS;
constexpr int kStaticMaxDevices = 64;
std::mutex g_static_mu;
unsigned char *g_static_base[kStaticMaxDevices];  // device address of the array, per device
}  // namespace

// Host code never uses this name as an address: in host code it only stands for the
// symbol, whose device address per device comes from cudaGetSymbolAddress below.
static __device__ __align__(256) unsigned char g_static_sample_scratch[kStaticBytes];

// Set-up, once per device, with that device current: the array's device address and the
// sampler kernel's shared-memory attribute.
static int static_sample_setup(int dev, unsigned char **base) {
    if (dev < 0 || dev >= kStaticMaxDevices) return validation("device", "ordinal out of range");
    std::lock_guard<std::mutex> lock(g_static_mu);
    if (!g_static_base[dev]) {
        unsigned char *ptr = nullptr;
        const cudaError_t e = cudaGetSymbolAddress((void **)&ptr, g_static_sample_scratch);
        if (e != cudaSuccess)
            return set_err(ITTS_E_CUDA, std::string("device error: cudaGetSymbolAddress: ") + cudaGetErrorString(e));
        kernels_init_sample();
        CUDA_TRY(cudaGetLastError());
        g_static_base[dev] = ptr;
    }
    *base = g_static_base[dev];
    return ITTS_OK;
}

extern "C" int itts_sample_next_token_static(float *logits, int32_t n, const uint64_t *seen,
                                             const itts_sampling_params *params,
                                             uint64_t *rng_state, int32_t *token_out,
                                             void *stream) {
    if (!logits || !seen || !rng_state || !token_out) return validation("logits", "null pointer");
    if (n <= 0) return validation("logits", "logits slice must not be empty");
    if (n > ITTS_STATIC_SAMPLE_MAX_LOGITS)
        return validation("logits", "at most " + std::to_string(ITTS_STATIC_SAMPLE_MAX_LOGITS) +
                                        " logits fit the static scratch of itts_sample_next_token_static (got " +
                                        std::to_string(n) + ")");
    TRY(itts_sampling_params_validate(params));
    int dev = 0;
    CUDA_TRY(cudaGetDevice(&dev));
    unsigned char *base = nullptr;
    TRY(static_sample_setup(dev, &base));
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    // Every field the kernel reads is rewritten here, so nothing of an earlier call is
    // read: the whole state block, batch column 0 -> state 0, and the token word cleared.
    SlotState s = blank_slot(0x7FFFFFFF);
    fill_params(s, params);
    s.active = 1;
    s.max_steps = 0x7FFFFFFF;
    s.rng = *rng_state;
    std::memcpy(s.seen, seen, sizeof(s.seen));
    int32_t idx[2] = {0, -1};
    SlotState *d_state = reinterpret_cast<SlotState *>(base);
    int32_t *d_idx = reinterpret_cast<int32_t *>(base + kStaticIdxOff);
    float *d_logits = reinterpret_cast<float *>(base + kStaticLogitsOff);
    CUDA_TRY(cudaMemcpyAsync(d_state, &s, sizeof(SlotState), cudaMemcpyHostToDevice, st));
    CUDA_TRY(cudaMemcpyAsync(d_idx, idx, sizeof(idx), cudaMemcpyHostToDevice, st));
    CUDA_TRY(cudaMemcpyAsync(d_logits, logits, sizeof(float) * n, cudaMemcpyHostToDevice, st));
    SampleArgs a{};
    a.slots = d_state;
    a.batch_slot = d_idx;
    a.nb = 1;
    a.logits = d_logits;
    a.ld_logits = n;
    a.n_logits = n;
    a.after_forward = 0;
    a.write_back = 1;
    a.codes = nullptr;
    a.token_out = d_idx + 1;
    a.small_k = sample_small_ok(*params, n);
    launch_sample(a, st);
    CUDA_TRY(cudaGetLastError());
    CUDA_TRY(cudaMemcpyAsync(logits, d_logits, sizeof(float) * n, cudaMemcpyDeviceToHost, st));
    CUDA_TRY(cudaMemcpyAsync(&s, d_state, sizeof(SlotState), cudaMemcpyDeviceToHost, st));
    CUDA_TRY(cudaMemcpyAsync(idx + 1, d_idx + 1, sizeof(int32_t), cudaMemcpyDeviceToHost, st));
    CUDA_TRY(cudaStreamSynchronize(st));
    *rng_state = s.rng;
    *token_out = idx[1];
    return ITTS_OK;
}
