// mk.h -- device layout of the tiled weights and the parameters of the persistent
// decode-step kernel (mk_decode.cu).
//
// Tiled linear [out, in] (built once at load time from the reference's u32 [out, in/4]
// bytes and [out, in/64] scales / offsets):
//   tile (rb, kci) = rows [16 rb, 16 rb + 16) x inputs [kci KC, kci KC + KC), KC <= 1280:
//     q   16 rows x KC bytes; within row m, quantization group j (64 inputs) is stored at
//         group slot (j ^ (m & 1)) and its bytes in fragment order (frag_pos), so a
//         thread's mma.sync A operand for the group's four k16 blocks is one 16-byte load
//         and rows m, m+1 hit different shared-memory banks;
//     sb  16 rows x KC/64 (scale, offset) pairs (fp16x2 or f32x2), original group order;
//     bias 16 f32 (the rows' linear bias, repeated in every K chunk of the row block).
//   tiles are stored rb-major, then kci; rows past `out` are zero.
#pragma once
#include "common.cuh"

namespace itts {

constexpr int MK_SLOT_BYTES = 24576;
constexpr int MK_MAX_NB = 4;
constexpr int MK_MAX_KC = 1280;

struct MkLin {
    const uint8_t *tiles;
    const float *bias;
    int out, in, n_rb, n_kc, kc, tile_bytes, sbb;
    const __half *w16;  // optional fp16 copy [out][in] for long prefills (null until made)
};

struct MkLayer {
    const float *ln1_w, *ln1_b, *ln2_w, *ln2_b;
    MkLin qkv, proj, fc, mlp;
    // c_proj re-tiled by attention head (null when not made): for head h and row block rb
    // the chunk (h * n_rb + rb) of 16 rows x the head's 64 inputs (int8 bytes in fragment
    // order, row m at 64 m, no swizzle) followed by the 16 rows' (scale, offset) pairs of
    // that group; the batch-1 cluster decode step reads c_proj from here
    const uint8_t *proj_h;
    // mlp projection re-tiled by input slice (null when not made): for the S = ff / H inputs
    // [S c, S c + S) of cluster c and row block rb, a sub-tile of 16 rows x S bytes (row m's
    // group j of the slice at slot j ^ (m & 1), fragment order, as in the tiles) followed by
    // the 16 rows' (scale, offset) pairs of the slice's S / 64 groups; the sub-tiles of cluster
    // c that rank k of its cluster applies (row blocks k, k + 6, ...) are contiguous; the
    // batch-1 cluster decode step reads the mlp projection only from here
    const uint8_t *mlp_k;
};
__host__ __device__ inline int mk_projh_chunk_bytes(int sbb) { return 16 * 64 + 16 * sbb; }
__host__ __device__ inline int mk_mlpk_sub_bytes(int S, int sbb) { return 16 * S + 16 * (S / 64) * sbb; }
// byte offset of (cluster c, rank k)'s first sub-tile in a layer's sliced mlp copy (6 ranks)
__host__ __device__ inline size_t mk_mlpk_rank_offset(int n_rb, int S, int sbb, int c, int k) {
    size_t before = 0;  // sub-tiles of ranks 0..k-1 of the cluster
    for (int r = 0; r < k; ++r) before += r < n_rb ? (size_t)((n_rb - 1 - r) / 6 + 1) : 0;
    return ((size_t)c * n_rb + before) * (size_t)mk_mlpk_sub_bytes(S, sbb);
}

constexpr int MK_MAX_D = 2048;      // model dim limit of the persistent kernel
constexpr int MK_MAX_UNITS = 8;     // attention units per (column, head)
constexpr int MK_PART_WORDS = 68;   // LL words per attention partial: m, l, 0, 0, acc[64]

// Cross-CTA activations of one decode step travel as 64-bit LL words
// (low 32 bits: the fp32 value, high 32 bits: the tag of the producing stage) in
// buffers indexed by layer, so every buffer is written once per step and a reader
// simply polls the words it needs until their tags match.
struct MkParams {
    int n_layers, d, H, ff, mel_vocab, mel_pos_len;
    int nb, grid, nslot, xsk, sbb;
    const MkLayer *layers;  // device array [n_layers]
    MkLin head;
    const float *lnf_w, *lnf_b, *fin_w, *fin_b;
    const float *mel_emb, *mel_pos;
    SlotState *slots;
    const int *batch_slot;
    int n_slots, max_seq;
    __half *kc, *vc;
    uint64_t *qkv_ll;   // [L][MK_MAX_NB][3d]
    uint64_t *attn_ll;  // [L][MK_MAX_NB][H][MK_MAX_UNITS][MK_PART_WORDS] partials
    uint64_t *ao_ll;    // [L][MK_MAX_NB][d]     attention output (merged over units)
    uint64_t *h_ll;     // [L][MK_MAX_NB][d]     after attention + residual
    uint64_t *u_ll;     // [L][MK_MAX_NB][ff]    GELU(c_fc)
    uint64_t *x_ll;     // [L+1][MK_MAX_NB][d]   layer outputs (index l+1 from layer l)
    float *logits;
    uint32_t *epoch;    // [grid] launches completed, one counter per CTA
    int *err;
    unsigned long long *trace;  // optional [grid][MK_TRACE_EVENTS] stage stamps (globaltimer ns in
                                // the grid-wide kernel, SM clock cycles in the cluster kernel)
    int stall;  // test hook (0: off): the cluster kernel first polls err[3], which nothing sets,
                // this many times and then reports a timeout (MK_ERR_STALL)
};
constexpr int MK_TRACE_EVENTS = 512;
// Error word value of a decode step whose fixed-point c_proj sum would overflow (any other
// nonzero value names a bounded wait that gave up).
constexpr int MK_ERR_RANGE = 1000;
// Error word value of the test hook's wait (MkParams::stall) that gave up.
constexpr int MK_ERR_STALL = 97;

__host__ __device__ inline int frag_pos_host(int k) {
    const int b = k >> 4, kk = k & 15, c = (kk & 7) >> 1, hi = kk >> 3, lo = kk & 1;
    return c * 16 + b * 4 + hi * 2 + lo;
}

__host__ __device__ inline int mk_tile_bytes(int kc, int sbb) { return 16 * kc + 16 * (kc / 64) * sbb + 64; }
__host__ __device__ inline int mk_tile_bias_offset(int kc, int sbb) { return 16 * kc + 16 * (kc / 64) * sbb; }

// Byte offset of weight (o, k) inside a tiled linear (used by the prefill GEMM).
__host__ __device__ inline size_t mk_q_offset(const MkLin &L, int o, int k) {
    const int rb = o >> 4, m = o & 15, kci = k / L.kc, kk = k - kci * L.kc;
    const int j = kk >> 6;
    const size_t tile = (size_t)rb * L.n_kc + kci;
    return tile * L.tile_bytes + (size_t)m * L.kc + (size_t)((j ^ (m & 1)) * 64) +
           frag_pos_host(kk & 63);
}
__host__ __device__ inline size_t mk_sb_offset(const MkLin &L, int o, int k) {
    const int rb = o >> 4, m = o & 15, kci = k / L.kc, j = (k - kci * L.kc) >> 6;
    const size_t tile = (size_t)rb * L.n_kc + kci;
    return tile * L.tile_bytes + (size_t)16 * L.kc + (size_t)(m * (L.kc / 64) + j) * L.sbb;
}

cudaError_t mk_launch(const MkParams &p, cudaStream_t st);
int mk_config(int nb, int xsk, int d, int n_layers, int *nslot);

}  // namespace itts
