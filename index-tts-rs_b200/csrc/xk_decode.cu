// xk_decode.cu -- the decode step of one request (batch column) on one 6-CTA thread-block
// cluster per attention head (120 CTAs for the 20 heads of IndexTTS-2.5;
// crates/core/src/models/gpt.rs:706-754): step embedding, n_layers x [LN1 -> QKV -> KV append
// -> attention -> c_proj + residual -> LN2 -> c_fc + GELU -> mlp c_proj + residual], ln_f ->
// final_norm -> mel_head.
//
// Cluster c owns head c: its ranks compute the 12 QKV row blocks of the head (q, k, v rows
// 64c .. 64c + 63), append K/V to the cache and push the 192 values into every CTA of the
// cluster with st.async; each rank then attends over its range of the head's 84-position
// K/V tiles and pushes one (m, l, acc[64]) record into every CTA of the cluster, and each CTA
// merges the six records into the head's 64 outputs (fp16).  The cluster then applies the
// head's 64 columns of c_proj (a head-major copy of its weights made at load) to them and
// adds each row's partial into a per-step accumulator word with a 64-bit integer add.  The
// word is a counted fixed-point sum: bits 0..51 the sum of the partials in 2^-28 units
// (signed), bits 52..57 how many partials have been added, bits 58..63 how many were not
// representable (not finite, or |y| >= 2^17).  Integer adds do not depend on their order, and
// the count makes each word self-validating: the reader polls the words it needs until
// every count is complete, with no fence or separate counter between writer and reader.  So
// q/k/v, the attention partials and the attention output never cross clusters.
//
// The MLP runs by slices of its S = ff / H hidden units (256 for IndexTTS-2.5): cluster c
// computes the c_fc rows [S c, S c + S), pushes GELU of them (fp16) into every CTA of the
// cluster, and applies the matching S inputs of the mlp projection (a copy of its weights
// re-tiled by input slice, made at load) for all d outputs, adding the partials into the
// next x's accumulator words.  So the only vectors that cross clusters are h and x, each
// through its accumulator: rank k of every cluster polls the k-th sixth of the words until
// all H partials of each are in, adds the residual and the bias, and pushes the result into
// all 6 CTAs with st.async; each CTA's mbarrier counts the bytes.  The head tiles are dealt
// round-robin over the grid (tile t on CTA t % grid).
//
// Per CTA: 11 consumer warps + 1 producer warp.  The producer lane streams the CTA's weight
// tiles (cp.async.bulk) and K/V tiles (TMA tensor loads, 128-byte swizzle) into an 8-slot
// ring (no multicast) ahead of the stages; consumers dequantize in registers and run
// mma.sync m16n8k16 with the activation (the same arithmetic as the other decode kernels),
// and run the attention on mma.sync too.
//
// Buffer reuse: the landing buffers (x/h, u, the head's q/k/v, the head's attention records)
// are rewritten once per layer without double buffering.  Each is rewritten by a peer only
// after every CTA of the cluster has consumed its previous contents: a peer's next push into
// it needs this CTA's own contribution to a later hand-off (its q/k/v rows, its attention
// record, its c_fc rows or its accumulator partials), which this CTA makes only after it has
// read the buffer.
//
// Every wait and poll is bounded; on a timeout the kernel records an error code in p.err
// (read by the host as ITTS_E_TIMEOUT), skips the remaining waits and exits cleanly.
#include <algorithm>
#include <cstdio>
#include <cstdlib>

#include "kernels.h"
#include "mk.h"

namespace itts {
namespace {

constexpr int CS = 6;              // CTAs per cluster: one cluster per attention head
constexpr int CW = 11;             // consumer warps (20 quantization groups of a tile: at most 2 each)
constexpr int CT = CW * 32;        // consumer threads
constexpr int NT = CT + 32;        // + the producer warp
constexpr int NSLOT = 8;           // ring slots (power of two)
constexpr int SLOT = 22528;        // bytes per slot (a multiple of 1,024): a 16 x 1280 tile with its
                                   // scale pairs, or one K/V tile
constexpr int KVPOS = 84;          // positions per K/V tile: K rows at the slot's start, V at KV_VOFF
constexpr int KV_VOFF = 11264;     // (both 1,024-aligned: the 128-byte swizzle repeats every 1,024 B)
static_assert(SLOT % 1024 == 0 && KVPOS * 128 <= KV_VOFF && KV_VOFF + KVPOS * 128 <= SLOT, "K/V tile layout");
constexpr int REC = 68;            // floats per attention record: m, l, 0, 0, acc[64]
constexpr int QT = 12;             // QKV row blocks of one head (q, k, v x 64 rows / 16)
constexpr uint32_t SPIN = 1u << 22;
constexpr int TABW = 8;                          // layer-table words per thread loaded up front
constexpr int EMBW = (MK_MAX_KC + CT - 1) / CT;  // embedding values per consumer thread (d <= MK_MAX_KC)
constexpr int kXkRangeCode = MK_ERR_RANGE;  // error word: a partial outside the fixed-point range
// counted fixed-point accumulator words (see the top of the file)
// (2^-28 resolution: coarser units change the fp16 rounding of some activations downstream)
constexpr float kFxScale = 268435456.0f;                // 2^28 units
constexpr float kFxLimit = 131072.0f;                   // |partial| < 2^17: 62 of them stay below 2^51
constexpr unsigned long long kFxOne = 1ull << 52;       // one partial added
constexpr unsigned long long kFxBad = 1ull << 58;       // one partial not representable
constexpr int kFxMaxHeads = 31;                         // partials per word: H (h) or 2H (next x)
constexpr float kLog2e = 1.4426950408889634f;

// landing barriers: x/h (fp32), u (fp16), the head's q/k/v (fp32), the head's attention records
enum { B0 = 0, BU, BQ, BR, NSTB };
enum { TM_RR = 0, TM_QKV = 1, TM_FC = 2 };  // tile assignment of a stage (tile_of)

// ---------------------------------------------------------------------------
// PTX helpers
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t su32(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }
__device__ __forceinline__ void mb_init(uint64_t *b, uint32_t n) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(su32(b)), "r"(n));
}
__device__ __forceinline__ void mb_expect(uint64_t *b, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(su32(b)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mb_arrive(uint64_t *b) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(su32(b)) : "memory");
}
template <bool CLUSTER>
__device__ __forceinline__ bool mb_try(uint32_t a, uint32_t par) {
    uint32_t done;
    if (CLUSTER)
        asm volatile(
            "{\n .reg .pred p;\n mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n"
            " selp.u32 %0, 1, 0, p;\n}\n"
            : "=r"(done)
            : "r"(a), "r"(par)
            : "memory");
    else
        asm volatile(
            "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
            : "=r"(done)
            : "r"(a), "r"(par)
            : "memory");
    return done != 0;
}
// non-blocking test of a CTA-local barrier's phase (the common case: the copy landed long ago)
__device__ __forceinline__ bool mb_test(uint32_t a, uint32_t par) {
    uint32_t done;
    asm volatile("{\n .reg .pred p;\n mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
                 : "=r"(done)
                 : "r"(a), "r"(par)
                 : "memory");
    return done != 0;
}
template <bool CLUSTER>
__device__ __forceinline__ bool mb_wait(uint64_t *b, uint32_t par, const int *err) {
    const uint32_t a = su32(b);
    for (uint32_t it = 0; it < SPIN; ++it) {
        if (mb_try<CLUSTER>(a, par)) return true;
        if (err && (it & 4095u) == 4095u && *(volatile const int *)err) return false;
    }
    return false;
}
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void *src, uint32_t bytes, uint32_t bar, uint64_t pol) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(dst),
        "l"(src), "r"(bytes), "r"(bar), "l"(pol)
        : "memory");
}
// 84 positions x 64 values of a K or V cache (tensor map {64, max_seq, heads, slots, layers},
// 128-byte swizzle) into shared memory at dst, completing on bar (no multicast)
__device__ __forceinline__ void tma_kv(uint32_t dst, const CUtensorMap *map, int pos0, int head, int slot, int layer,
                                       uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.5d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, %5, "
        "%6}], [%7];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(0), "r"(pos0), "r"(head), "r"(slot), "r"(layer), "r"(bar)
        : "memory");
}
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t &a0, uint32_t &a1, uint32_t &a2, uint32_t &a3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(a0), "=r"(a1), "=r"(a2), "=r"(a3)
                 : "r"(addr)
                 : "memory");
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t &a0, uint32_t &a1, uint32_t &a2, uint32_t &a3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(a0), "=r"(a1), "=r"(a2), "=r"(a3)
                 : "r"(addr)
                 : "memory");
}
// shared address of 16-byte chunk `chunk` of the 128-byte row at `row` (128-byte swizzle: the
// chunk index is XORed with address bits 7..9)
__device__ __forceinline__ uint32_t swz(uint32_t row, int chunk) { return row + ((chunk ^ ((row >> 7) & 7)) << 4); }
__device__ __forceinline__ uint32_t mapa(uint32_t a, int rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(rank));
    return r;
}
__device__ __forceinline__ void st_async_v4(uint32_t raddr, uint4 v, uint32_t rbar) {
    asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.v4.b32 [%0], {%1, %2, %3, %4}, [%5];" ::"r"(raddr),
                 "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w), "r"(rbar)
                 : "memory");
}
__device__ __forceinline__ void st_async_b32(uint32_t raddr, uint32_t v, uint32_t rbar) {
    asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.b32 [%0], %1, [%2];" ::"r"(raddr), "r"(v),
                 "r"(rbar)
                 : "memory");
}
// the same 16 bytes into every CTA of the cluster
__device__ __forceinline__ void bcast_v4(uint32_t laddr, uint4 v, uint32_t lbar) {
#pragma unroll
    for (int r = 0; r < CS; ++r) st_async_v4(mapa(laddr, r), v, mapa(lbar, r));
}
__device__ __forceinline__ void cluster_sync_all() {
    asm volatile("barrier.cluster.arrive.release.aligned;\nbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ void csync() { asm volatile("bar.sync 1, %0;" ::"n"(CT) : "memory"); }
__device__ __forceinline__ bool csync_and(bool v) {
    uint32_t r;
    asm volatile(
        "{\n .reg .pred p, q;\n setp.ne.u32 p, %1, 0;\n bar.red.and.pred q, 1, %2, p;\n selp.u32 %0, 1, 0, q;\n}\n"
        : "=r"(r)
        : "r"((uint32_t)v), "n"(CT)
        : "memory");
    return r != 0;
}
__device__ __forceinline__ void mma16816(float *d, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                         uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t lo_h(uint32_t w) { return __byte_perm(w, 0x64646464u, 0x4140u); }
__device__ __forceinline__ uint32_t hi_h(uint32_t w) { return __byte_perm(w, 0x64646464u, 0x4342u); }
__device__ __forceinline__ uint32_t pack_h2(float a, float b) {
    const __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<const uint32_t *>(&h);
}
// ---------------------------------------------------------------------------
// shared-memory carve-up (identical on host and device)
// ---------------------------------------------------------------------------
struct XkSmem {
    uint32_t land, xln, xh, xu, sxln, sxu, red, qkvh, recs, stat, tab, lay, bar, total;
};
__host__ __device__ inline uint32_t xk_red_bytes(int rt, int d, int ff) {
    uint32_t m = (uint32_t)rt * CW * 16 * 4;                                   // tile partial sums
    m = max(m, (uint32_t)(CW + 1) * REC * 4);                                  // attention warp states
    return m;
}
struct XkTab {
    int active, lold, kvt, slot, tok, pos, head, t_lo, t_hi, pad[7];
};
__host__ __device__ inline XkSmem xk_layout(int d, int ff, int rt, int n_layers) {
    XkSmem L;
    uint32_t o = NSLOT * SLOT;
    auto take = [&](uint32_t bytes) {
        const uint32_t at = o;
        o = (o + bytes + 127u) & ~127u;
        return at;
    };
    L.land = take(d * 4);
    L.xln = take(d * 2);
    L.xh = take(64 * 2);  // the head's attention output (fp16, fragment order)
    const int S = ff / (d / 64);  // the cluster's slice of the MLP hidden units
    L.xu = take(S * 2);
    L.sxln = take(d / 64 * 4);
    L.sxu = take(S / 64 * 4);
    L.red = take(xk_red_bytes(rt, d, ff));
    L.qkvh = take(3 * 64 * 4);
    L.recs = take(CS * REC * 4);
    L.stat = take(64 * 4);
    L.tab = take(sizeof(XkTab));
    L.lay = take(n_layers * sizeof(MkLayer));  // the layer table (pointers, shapes) in shared memory
    L.bar = take((2 * NSLOT + NSTB) * 8);
    L.total = o;
    return L;
}

struct XkParams {
    CUtensorMap kmap, vmap;    // the K and V caches (tiled loads of KVPOS x 64 values)
    MkParams p;          // model, slots, KV cache, logits, err, trace
    unsigned long long *hacc;  // [2][L][d] counted fixed-point sums of the heads' c_proj partials,
                               // by step parity (this step's buffer p = epoch & 1; 1 - p zeroed)
    unsigned long long *xacc;  // [2][L][d] the same for the clusters' mlp partials (next x)
    uint32_t *epoch;     // [grid] launches completed per CTA
    int rt, dry;
};

// rows of [0, n) gathered by cluster rank k
__device__ __forceinline__ int slice_lo(int k, int n) { return k * n / CS; }

// QKV row block i (0 <= i < QT) of head h: q, k, v rows h*64 .. h*64 + 63
__device__ __forceinline__ int qkv_rb(int i, int h, int d) { return (i >> 2) * (d / 16) + 4 * h + (i & 3); }

// ---------------------------------------------------------------------------
// producer (one lane)
// ---------------------------------------------------------------------------
struct XkProducer {
    uint32_t ring, full;
    uint64_t *fullp, *emptyp;
    const int *err;
    uint64_t pol;
    uint32_t seq;
    int R, NR;
    bool ok;

    // the next ring slot, once its consumers have released it (false: a wait gave up); seq
    // counts the copies actually issued, so the drain below waits for exactly those
    __device__ __forceinline__ bool acquire(uint32_t &slot) {
        if (!ok) return false;
        slot = seq & (NSLOT - 1);
        if (seq >= (uint32_t)NSLOT) {
            ok = mb_wait<false>(emptyp + slot, ((seq / NSLOT) & 1u) ^ 1u, err);
            if (!ok) {
                atomicExch(const_cast<int *>(err), 1);
                return false;
            }
        }
        ++seq;
        return true;
    }
    __device__ __forceinline__ void issue(const void *s0, uint32_t b0, const void *s1, uint32_t b1) {
        uint32_t slot;
        if (!acquire(slot)) return;
        const uint32_t bar = full + slot * 8;
        mb_expect(fullp + slot, b0 + b1);
        const uint32_t dst = ring + slot * SLOT;
        bulk_g2s(dst, s0, b0, bar, pol);
        if (b1) bulk_g2s(dst + b0, s1, b1, bar, pol);
    }
    // K/V tile t of (layer, cache slot, head): the full box of KVPOS rows each (rows past the
    // cache's positions read as zero; rows past the valid length are never used)
    __device__ __forceinline__ void issue_kv(const CUtensorMap *km, const CUtensorMap *vm, int t, int head,
                                             int cslot, int layer) {
        uint32_t slot;
        if (!acquire(slot)) return;
        const uint32_t bar = full + slot * 8;
        mb_expect(fullp + slot, 2 * KVPOS * 128);
        const uint32_t dst = ring + slot * SLOT;
        tma_kv(dst, km, t * KVPOS, head, cslot, layer, bar);
        tma_kv(dst + KV_VOFF, vm, t * KVPOS, head, cslot, layer, bar);
    }
    // tiles t = R, R + NR, ... of a linear (tile index = rb * n_kc + kc)
    __device__ __forceinline__ void lin(const uint8_t *tiles, int n_tiles, uint32_t tb) {
        const uint8_t *t = tiles + (size_t)R * tb;
        const size_t step = (size_t)NR * tb;
        for (int i = R; i < n_tiles; i += NR, t += step) issue(t, tb, nullptr, 0);
    }
    __device__ __forceinline__ void lin(const MkLin *L) { lin(L->tiles, L->n_rb * L->n_kc, (uint32_t)L->tile_bytes); }
    __device__ __forceinline__ void run(const XkParams &xp, const XkTab &T, const MkLayer *lay, int rank) {
        const MkParams &p = xp.p;
        const int head = T.head, t_lo = T.t_lo, t_hi = T.t_hi, lold = T.lold, slot = T.slot;
        const int q0 = rank * QT / CS, q1 = (rank + 1) * QT / CS;
        for (int l = 0; l < p.n_layers && ok; ++l) {
            const MkLayer *Ly = lay + l;
            {  // this rank's QKV row blocks of the cluster's head
                const uint8_t *tiles = Ly->qkv.tiles;
                const uint32_t tb = (uint32_t)Ly->qkv.tile_bytes;
                for (int i = q0; i < q1; ++i) issue(tiles + (size_t)qkv_rb(i, head, p.d) * tb, tb, nullptr, 0);
            }
            // this rank's K/V tiles of the head
            for (int t = t_lo; t < t_hi; ++t)
                if (lold - t * KVPOS > 0) issue_kv(&xp.kmap, &xp.vmap, t, head, slot, l);
            {  // this rank's head-major c_proj chunks of the head (one copy)
                const int nrb = Ly->proj.n_rb, r0 = rank * nrb / CS, nc = (rank + 1) * nrb / CS - r0;
                const uint32_t cb = (uint32_t)mk_projh_chunk_bytes(Ly->proj.sbb);
                if (nc > 0) issue(Ly->proj_h + ((size_t)head * nrb + r0) * cb, (uint32_t)nc * cb, nullptr, 0);
            }
            {  // the cluster's slice of c_fc rows: row blocks S/16 head + rank + CS i
                const int nrb = p.ff / p.H / 16;
                const uint32_t tb = (uint32_t)Ly->fc.tile_bytes;
                for (int rb = rank; rb < nrb; rb += CS) issue(Ly->fc.tiles + (size_t)(head * nrb + rb) * tb, tb, nullptr, 0);
            }
            {  // this rank's sub-tiles of the cluster's K-slice of the mlp projection, contiguous
               // in the sliced copy, as many per ring slot as fit
                const int S = p.ff / p.H, nrb = Ly->mlp.n_rb, mine = rank < nrb ? (nrb - 1 - rank) / CS + 1 : 0;
                const uint32_t sub = (uint32_t)mk_mlpk_sub_bytes(S, p.sbb), per = SLOT / sub;
                const uint8_t *src = Ly->mlp_k + mk_mlpk_rank_offset(nrb, S, p.sbb, head, rank);
                for (int s0 = 0; s0 < mine; s0 += (int)per) {
                    const int ns = min((int)per, mine - s0);
                    issue(src + (size_t)s0 * sub, (uint32_t)ns * sub, nullptr, 0);
                }
            }
        }
        if (ok) lin(&p.head);
        // every issued copy lands before exit (the last one of each slot; the earlier ones
        // were consumed before the slot was reused).  Copies always complete, so this wait
        // ignores the error word and is bounded by SPIN only.
        for (uint32_t s = 0; s < NSLOT && s < seq; ++s) {
            const uint32_t last = ((seq - 1 - s) / NSLOT) * NSLOT + s;
            mb_wait<false>(fullp + s, (last / NSLOT) & 1u, nullptr);
        }
    }
};

// ---------------------------------------------------------------------------
// consumers (8 warps)
// ---------------------------------------------------------------------------
struct XkConsumer {
    const XkParams *xp;
    const MkParams *pp;
    XkTab *T;
    const MkLayer *lay;  // shared-memory copy of the layer table
    uint8_t *smem;
    float *land, *sxln, *sxu, *red, *qkvh, *recs, *stat;
    __half *xln, *xh, *xu;  // xh: the head's attention output (fp16, fragment order)
    uint32_t par;           // this step's accumulator buffer
    uint64_t *fullp, *emptyp, *stb;
    int tid, warp, lane, g, c, rank, R, NR, d, ff, H, rt, head;
    uint32_t seq;
    uint32_t ph[NSTB];
    uint32_t exp_bytes[NSTB];
    bool ok;
    int ev;

    __device__ __forceinline__ void trace() {
        if (pp->trace && tid == 0 && ev < MK_TRACE_EVENTS) {  // (SM clock cycles)
            unsigned long long t;
            asm volatile("mov.u64 %0, %%clock64;" : "=l"(t));
            pp->trace[(size_t)R * MK_TRACE_EVENTS + ev] = t;
        }
        ++ev;
    }
    __device__ __forceinline__ void fail(int code) {
        if (ok) atomicExch(pp->err, code);
        ok = false;
    }
    // every consumer thread learns whether any of them failed
    __device__ __forceinline__ void agree(bool good, int code) {
        good = csync_and(good);
        if (!good) fail(code);
    }
    __device__ __forceinline__ void wait_land(int b, int code) {
        bool good = !ok || mb_wait<true>(stb + b, ph[b] & 1u, pp->err);
        ++ph[b];
        agree(good, code);
        if (tid == 0) mb_expect(stb + b, exp_bytes[b]);
        trace();
    }
    static constexpr int LNC = (MK_MAX_D / 4 + CT - 1) / CT;
    struct LnRegs {
        float4 w[LNC], b[LNC];
    };
    __device__ __forceinline__ LnRegs ln_prefetch(const float *w, const float *b) const {
        LnRegs r;
#pragma unroll
        for (int j = 0; j < LNC; ++j) {
            const int k4 = tid + j * CT;
            if (k4 * 4 < d) {
                r.w[j] = __ldg(reinterpret_cast<const float4 *>(w) + k4);
                r.b[j] = __ldg(reinterpret_cast<const float4 *>(b) + k4);
            } else {
                r.w[j] = r.b[j] = make_float4(0.f, 0.f, 0.f, 0.f);
            }
        }
        return r;
    }
    // LayerNorm(land) * w + b into xln (fp16, fragment order, with its group sums) or back
    // into land (inplace).  Statistics in one pass over x - x[0] (the shift keeps
    // E[y^2] - E[y]^2 well conditioned); a group's 64 inputs are the float4 chunks of 16
    // consecutive lanes, so its fp16 sum takes 4 shuffles.
    __device__ __forceinline__ void layernorm(const LnRegs &P, bool inplace) {
        float4 x[LNC];
        const float sh = land[0];
        float s1 = 0.f, s2 = 0.f;
#pragma unroll
        for (int j = 0; j < LNC; ++j) {
            const int k4 = tid + j * CT;
            x[j] = k4 * 4 < d ? *reinterpret_cast<const float4 *>(land + k4 * 4) : make_float4(sh, sh, sh, sh);
            const float a = x[j].x - sh, b = x[j].y - sh, cc = x[j].z - sh, e = x[j].w - sh;
            s1 += (a + b) + (cc + e);
            s2 += (a * a + b * b) + (cc * cc + e * e);
        }
        s1 = warp_sum(s1);
        s2 = warp_sum(s2);
        if (lane == 0) { stat[2 * warp] = s1; stat[2 * warp + 1] = s2; }
        csync();
        float t1 = 0.f, t2 = 0.f;
#pragma unroll
        for (int w = 0; w < CW; ++w) { t1 += stat[2 * w]; t2 += stat[2 * w + 1]; }
        const float inv_d = 1.0f / (float)d;  // (a constant of the launch: hoisted by the compiler)
        const float m1 = t1 * inv_d;
        const float mean = sh + m1;
        const float rstd = rsqrtf(fmaxf(t2 * inv_d - m1 * m1, 0.f) + kNormEps);
#pragma unroll
        for (int j = 0; j < LNC; ++j) {
            if (j * CT >= d / 4) break;  // (uniform: no thread has inputs in this pass)
            const int k4 = tid + j * CT;
            const bool in = k4 * 4 < d;
            float4 y;
            y.x = (x[j].x - mean) * rstd * P.w[j].x + P.b[j].x;
            y.y = (x[j].y - mean) * rstd * P.w[j].y + P.b[j].y;
            y.z = (x[j].z - mean) * rstd * P.w[j].z + P.b[j].z;
            y.w = (x[j].w - mean) * rstd * P.w[j].w + P.b[j].w;
            if (inplace) {
                if (in) *reinterpret_cast<float4 *>(land + k4 * 4) = y;
            } else {
                const __half hx = __float2half_rn(y.x), hy = __float2half_rn(y.y), hz = __float2half_rn(y.z),
                             hw = __float2half_rn(y.w);
                float gs = in ? (__half2float(hx) + __half2float(hy)) + (__half2float(hz) + __half2float(hw)) : 0.f;
                gs += __shfl_xor_sync(0xffffffffu, gs, 1);
                gs += __shfl_xor_sync(0xffffffffu, gs, 2);
                gs += __shfl_xor_sync(0xffffffffu, gs, 4);
                gs += __shfl_xor_sync(0xffffffffu, gs, 8);
                if (in) {
                    const int k = k4 * 4, base = k & ~63;
                    xln[base + frag_pos_host(k & 63)] = hx;
                    xln[base + frag_pos_host((k + 1) & 63)] = hy;
                    xln[base + frag_pos_host((k + 2) & 63)] = hz;
                    xln[base + frag_pos_host((k + 3) & 63)] = hw;
                    if ((k4 & 15) == 0) sxln[k4 >> 4] = gs;
                }
            }
        }
        csync();
        trace();
    }

    // ---- GEMV tiles ----
    // one quantization group j (64 inputs) of a 16-row tile (row pitch KC bytes, G64 groups
    // per row) against the activation fragment (x0, x1) and its group sum: per-row partials
    // into a0 (row g) and a1 (row g + 8), int8 -> fp16 by byte permutation, y = s acc + (b -
    // 1024 s) sum(x)
    __device__ __forceinline__ void group_x(const uint8_t *tq, const uint8_t *tsb, int KC, int G64, int j, uint4 x0,
                                            uint4 x1, float sxg, bool half_sb, float &a0, float &a1) {
        const int jj = j ^ (g & 1);
        const uint4 wa = *reinterpret_cast<const uint4 *>(tq + g * KC + jj * 64 + c * 16);
        const uint4 wb = *reinterpret_cast<const uint4 *>(tq + (g + 8) * KC + jj * 64 + c * 16);
        float d0[4] = {0.f, 0.f, 0.f, 0.f}, d1[4] = {0.f, 0.f, 0.f, 0.f};
        mma16816(d0, lo_h(wa.x), lo_h(wb.x), hi_h(wa.x), hi_h(wb.x), x0.x, x0.y);
        mma16816(d1, lo_h(wa.y), lo_h(wb.y), hi_h(wa.y), hi_h(wb.y), x0.z, x0.w);
        mma16816(d0, lo_h(wa.z), lo_h(wb.z), hi_h(wa.z), hi_h(wb.z), x1.x, x1.y);
        mma16816(d1, lo_h(wa.w), lo_h(wb.w), hi_h(wa.w), hi_h(wb.w), x1.z, x1.w);
        float s0, z0, s1, z1;
        if (half_sb) {
            const float2 f0 = __half22float2(*reinterpret_cast<const __half2 *>(tsb + (g * G64 + j) * 4));
            const float2 f1 = __half22float2(*reinterpret_cast<const __half2 *>(tsb + ((g + 8) * G64 + j) * 4));
            s0 = f0.x; z0 = f0.y; s1 = f1.x; z1 = f1.y;
        } else {
            const float2 f0 = *reinterpret_cast<const float2 *>(tsb + (g * G64 + j) * 8);
            const float2 f1 = *reinterpret_cast<const float2 *>(tsb + ((g + 8) * G64 + j) * 8);
            s0 = f0.x; z0 = f0.y; s1 = f1.x; z1 = f1.y;
        }
        a0 += fmaf(s0, d0[0] + d1[0], fmaf(-1024.0f, s0, z0) * sxg);
        a1 += fmaf(s1, d0[2] + d1[2], fmaf(-1024.0f, s1, z1) * sxg);
    }
    __device__ __forceinline__ void wait_slot(uint32_t slot, int code) { wait_seq(seq, code); }
    // the copy of ring sequence number sq (slot sq % NSLOT, use sq / NSLOT) has landed
    __device__ __forceinline__ void wait_seq(uint32_t sq, int code) {
        uint64_t *b = fullp + (sq & (NSLOT - 1));
        const uint32_t par = (sq / NSLOT) & 1u;
        if (mb_test(su32(b), par)) return;  // (one warp instruction: the same answer in every lane)
        bool good = !ok || mb_wait<false>(b, par, pp->err);
        good = __all_sync(0xffffffffu, good);
        if (!good) fail(code);
    }
    __device__ __forceinline__ const uint8_t *ring_at(uint32_t sq) const { return smem + (sq & (NSLOT - 1)) * SLOT; }
    // releases the next n ring entries (after the warp is done with them)
    __device__ __forceinline__ void release(int n) {
        __syncwarp();
        if (lane == 0)
            for (int i = 0; i < n; ++i) mb_arrive(emptyp + ((seq + i) & (NSLOT - 1)));
        seq += n;
    }
    // This CTA's tiles t = R + NR i of linear L, i in [i0, i1), from the ring: per-warp
    // partial sums to red[i - i0] (group j of a tile goes to warp (tile * G64 + j) % 8).
    // global tile index of this CTA's i-th tile of L: round robin over the grid (TM_RR), the
    // rank's share of the QKV row blocks of the cluster's head (TM_QKV), or of the c_fc row
    // blocks of the cluster's slice of the MLP (TM_FC: rows [S head, S head + S), S = ff / H)
    __device__ __forceinline__ int tile_of(const MkLin &L, int i, int mode) const {
        if (mode == TM_QKV) return qkv_rb(rank * QT / CS + i, head, d);
        if (mode == TM_FC) return head * (ff / pp->H / 16) + rank + CS * i;
        return R + i * NR;
    }
    __device__ __forceinline__ int own_tiles(const MkLin &L, int mode) const {
        if (mode == TM_QKV) return (rank + 1) * QT / CS - rank * QT / CS;
        if (mode == TM_FC) {
            const int nrb = ff / pp->H / 16;
            return rank < nrb ? (nrb - 1 - rank) / CS + 1 : 0;
        }
        const int n = L.n_rb * L.n_kc;
        return R < n ? (n - 1 - R) / NR + 1 : 0;
    }
    // This CTA's tiles i in [i0, i1) of a linear with one K chunk (tile_of gives their
    // index), from the ring: per-warp partial sums to red[i - i0].  Warp w takes groups w and
    // w + CW of every tile (CW >= 10: at most 2 of the <= 20 groups), its two activation
    // fragments in registers for the whole stage.  Each tile is computed as soon as it has
    // landed (the later ones are often still in flight).
    __device__ __forceinline__ void tiles(const MkLin &L, const __half *xs, const float *sx, int i0, int i1) {
        static_assert(2 * CW >= MK_MAX_KC / 64, "two groups per warp cover a tile");
        const int KC = L.kc, G64 = KC / 64, n = i1 - i0;
        const bool half_sb = pp->sbb == 4;
        const int j0 = warp, j1 = warp + CW;
        const bool h0 = j0 < G64, h1 = j1 < G64;
        uint4 xa0 = make_uint4(0, 0, 0, 0), xa1 = xa0, xb0 = xa0, xb1 = xa0;
        float sa = 0.f, sb = 0.f;
        if (h0) {
            xa0 = *reinterpret_cast<const uint4 *>(xs + j0 * 64 + c * 16);
            xa1 = *reinterpret_cast<const uint4 *>(xs + j0 * 64 + c * 16 + 8);
            sa = sx[j0];
        }
        if (h1) {
            xb0 = *reinterpret_cast<const uint4 *>(xs + j1 * 64 + c * 16);
            xb1 = *reinterpret_cast<const uint4 *>(xs + j1 * 64 + c * 16 + 8);
            sb = sx[j1];
        }
        for (int i = 0; i < n; ++i) {
            wait_seq(seq, 2);
            const uint8_t *tq = ring_at(seq);
            float a0 = 0.f, a1 = 0.f;
            if (h0) group_x(tq, tq + 16 * KC, KC, G64, j0, xa0, xa1, sa, half_sb, a0, a1);
            if (h1) group_x(tq, tq + 16 * KC, KC, G64, j1, xb0, xb1, sb, half_sb, a0, a1);
            release(1);
            if (c == 0) {
                float *r = red + (i * CW + warp) * 16;
                r[g] = a0;
                r[g + 8] = a1;
            }
        }
        csync();
    }
    // rows [4q, 4q+4) of local tile i: the 8 warps' partial sums in a fixed order
    __device__ __forceinline__ float4 rows4(int i, int q) const {
        float v[4] = {0.f, 0.f, 0.f, 0.f};
        const float *r = red + (i * CW) * 16 + q * 4;
#pragma unroll
        for (int w = 0; w < CW; ++w) {
            const float4 x = *reinterpret_cast<const float4 *>(r + w * 16);
            v[0] += x.x; v[1] += x.y; v[2] += x.z; v[3] += x.w;
        }
        return make_float4(v[0], v[1], v[2], v[3]);
    }
    // bias of output rows [o, o + 4) (rows past L.out read as 0)
    __device__ __forceinline__ float4 bias4(const MkLin &L, int o) const {
        if (o + 4 <= L.out) return __ldg(reinterpret_cast<const float4 *>(L.bias + o));
        float b[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) b[e] = o + e < L.out ? __ldg(L.bias + o + e) : 0.f;
        return make_float4(b[0], b[1], b[2], b[3]);
    }
    // This thread's epilogue chunk of the first round of run_lin<P>: its bias, loaded before
    // the stage's input wait so that the L2 latency is off the critical path.
    template <int P>
    __device__ __forceinline__ float4 bias_pre(const MkLin &L, int mode) const {
        const int n = min(own_tiles(L, mode), rt), ch = tid / P;
        if (ch >= n * 4) return make_float4(0.f, 0.f, 0.f, 0.f);
        const int t = tile_of(L, ch >> 2, mode), o = t * 16 + (ch & 3) * 4;
        return o < L.out ? bias4(L, o) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    // Tiles of one linear (one K chunk), then per 4-row chunk and part p < P
    // epi(o, v, bias, p) (o: first output row; P threads per chunk, each sending one part of
    // its results).  Rows past L.out are skipped.
    template <int P, class Epi>
    __device__ __forceinline__ void run_lin(const MkLin &L, const __half *xs, const float *sx, float4 bpre, int mode,
                                            Epi epi) {
        const int n = own_tiles(L, mode);
        for (int i0 = 0; i0 < n; i0 += rt) {
            const int i1 = min(n, i0 + rt);
            tiles(L, xs, sx, i0, i1);
            for (int q = tid; q < (i1 - i0) * 4 * P; q += CT) {
                const int ch = q / P, part = q - ch * P, il = ch >> 2, t = tile_of(L, i0 + il, mode);
                const int o = t * 16 + (ch & 3) * 4;
                if (o < L.out) epi(o, rows4(il, ch & 3), i0 == 0 ? bpre : bias4(L, o), part);
            }
            csync();
        }
        trace();
    }

    // ---- exchanges (cluster rank k gathers its slice of the vector and pushes it to the
    // cluster) ----
    // one partial into a counted fixed-point accumulator word; a partial that is not finite or
    // too large adds only to the count and the "not representable" field (the reader then
    // yields NaN for the row, as the reference's fp32 sum would give NaN or a value the next
    // LayerNorm spreads to every output); the finite case is also reported in the error word
    __device__ __forceinline__ void add_part(unsigned long long *a, float y) const {
        unsigned long long v = kFxOne;
        if (fabsf(y) < kFxLimit) {
            v += (unsigned long long)__float2ll_rn(y * kFxScale);
        } else {
            v += kFxBad;
            if (isfinite(y)) atomicExch(pp->err + 1, kXkRangeCode);
        }
        asm volatile("red.relaxed.gpu.global.add.u64 [%0], %1;" ::"l"(a), "l"(v) : "memory");
    }
    // land += bias + the accumulated partials -> land of every CTA of the cluster.  Each of the
    // slice's threads polls its 4 words until all H partials of each are in, then pushes.  For
    // h: land holds x and the partials are the heads' c_proj rows; for the next x: land holds
    // h and the partials are the clusters' mlp slices.
    __device__ __forceinline__ void exchange_acc(const unsigned long long *acc, float4 bpre, const float *bias,
                                                 int want, int code) {
        const int c0 = slice_lo(rank, d / 4), nch = slice_lo(rank + 1, d / 4) - c0, o0 = c0 * 4;
        const uint32_t land_a = su32(land), bar_a = su32(stb + B0);
        for (int i = tid; i < nch && ok; i += CT) {
            const int o = o0 + i * 4;
            long long q[4];
            bool done = false;
            for (uint32_t it = 0; it < SPIN; ++it) {
                asm volatile("ld.relaxed.gpu.global.v2.b64 {%0,%1}, [%2];" : "=l"(q[0]), "=l"(q[1]) : "l"(acc + o) : "memory");
                asm volatile("ld.relaxed.gpu.global.v2.b64 {%0,%1}, [%2];" : "=l"(q[2]), "=l"(q[3]) : "l"(acc + o + 2) : "memory");
                // count field (bits 52..57) of each word, with the signed sum below it biased
                // to [0, 2^52) so that it does not borrow from the count
                done = true;
#pragma unroll
                for (int e = 0; e < 4; ++e) done &= (int)(((unsigned long long)q[e] + (1ull << 51)) >> 52 & 63) == want;
                if (done) break;
                if ((it & 255u) == 255u && *(volatile const int *)pp->err) break;
                if (it >= 4) __nanosleep(it < 64 ? 20u : 100u);
            }
            if (!done) {
                fail(code);
                break;
            }
            const float4 x = *reinterpret_cast<const float4 *>(land + o);
            const float4 bb = i == tid ? bpre : __ldg(reinterpret_cast<const float4 *>(bias + o));
            float v[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const unsigned long long u = (unsigned long long)q[e] + (1ull << 51);
                const long long sum = (long long)(u & ((1ull << 52) - 1)) - (1ll << 51);
                v[e] = (u >> 58) ? __int_as_float(0x7fc00000) : (float)sum * (1.0f / kFxScale);
            }
            bcast_v4(land_a + o * 4, make_uint4(__float_as_uint(x.x + bb.x + v[0]), __float_as_uint(x.y + bb.y + v[1]),
                                                __float_as_uint(x.z + bb.z + v[2]), __float_as_uint(x.w + bb.w + v[3])),
                     bar_a);
        }
        trace();
        wait_land(B0, code + 1);
    }
    __device__ __forceinline__ void exchange_h(int l, float4 bpre, int code) {
        const size_t li = (size_t)par * pp->n_layers + l;
        exchange_acc(xp->hacc + li * d, bpre, lay[l].proj.bias, pp->H, code);
    }
    // x of layer lprev + 1 = h + mlp bias + the clusters' mlp partials
    __device__ __forceinline__ void exchange_x(int lprev, int code) {
        const size_t li = (size_t)par * pp->n_layers + lprev;
        const int c0 = slice_lo(rank, d / 4), nch = slice_lo(rank + 1, d / 4) - c0;
        const float *mb = lay[lprev].mlp.bias;
        const float4 bpre = tid < nch ? __ldg(reinterpret_cast<const float4 *>(mb + c0 * 4 + tid * 4))
                                      : make_float4(0.f, 0.f, 0.f, 0.f);
        exchange_acc(xp->xacc + li * d, bpre, mb, 2 * pp->H, code);  // (two halves per cluster)
    }

    // ---- stages ----
    __device__ __forceinline__ void stage_qkv(int l) {
        const MkParams &p = *pp;
        const MkLayer &Ly = lay[l];
        const LnRegs ln1 = ln_prefetch(Ly.ln1_w, Ly.ln1_b);
        const float4 bpre = bias_pre<CS>(Ly.qkv, TM_QKV);
        if (l == 0) {
            trace();  // (the embedding went into land before the set-up barrier)
        } else {
            exchange_x(l - 1, 20);
        }
        layernorm(ln1, false);
        // this rank's share of the head's q/k/v rows: K/V appended to the cache, all 192
        // values pushed into the qkvh of every CTA of the cluster
        const MkLin &L = Ly.qkv;
        const int active = T->active, slot = T->slot, lold = T->lold, hd = head;
        const uint32_t q_a = su32(qkvh), bar_a = su32(stb + BQ);
        run_lin<CS>(L, xln, sxln, bpre, TM_QKV, [&](int o, float4 v, float4 bb, int r) {
            v.x += bb.x; v.y += bb.y; v.z += bb.z; v.w += bb.w;
            const int which = o / d, oo = o - which * d;
            if (r == 0 && which > 0 && active) {
                __half *cache = which == 1 ? p.kc : p.vc;
                uint2 hv;
                hv.x = pack_h2(v.x, v.y);
                hv.y = pack_h2(v.z, v.w);
                *reinterpret_cast<uint2 *>(cache + kv_index(l, slot, hd, lold, p.n_slots, p.H, p.max_seq) + (oo & 63)) = hv;
            }
            st_async_v4(mapa(q_a + (which * 64 + (oo & 63)) * 4, r),
                        make_uint4(__float_as_uint(v.x), __float_as_uint(v.y), __float_as_uint(v.z), __float_as_uint(v.w)),
                        mapa(bar_a, r));
        });
    }
    // attention of the cluster's head over this rank's K/V tiles: one record (m, l, acc[64])
    // per rank into every CTA of the cluster, each of which merges them into the head's 64
    // outputs.  Up to four tiles at a time, as one run of n <= 336 positions; warp w takes the
    // 16-position m-tiles w and w + CW of the run on the tensor cores: S = K q with mma.sync (K rows through
    // ldmatrix from the swizzled tile; q as the B operand, column 0 its fp16 value and column 1
    // the fp16 remainder, so the products carry about 22 bits of q), an online softmax per warp,
    // then O^T = V^T P (ldmatrix.trans; P split the same way into columns 0 and 1).  Rows past
    // the run read row 0 of the first tile (finite, with weight 0).
    __device__ __forceinline__ void stage_attn(int l) {
        wait_land(BQ, 30);
        float *ascr = red;  // [CW][REC] warp states, then [REC] this rank's record
        const float qscale = kAttnScale * kLog2e;
        uint32_t qb[4][2];  // B fragments of q: k16 step kk, dims 16 kk + 2c (+1) and + 8
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const int k0 = 16 * kk + 2 * c + 8 * h;
                const float q0 = qkvh[k0] * qscale, q1 = qkvh[k0 + 1] * qscale;
                const __half2 qh = __floats2half2_rn(q0, q1);
                const float2 qf = __half22float2(qh);
                const uint32_t hi = *reinterpret_cast<const uint32_t *>(&qh);
                const uint32_t lo = pack_h2(q0 - qf.x, q1 - qf.y);
                qb[kk][h] = g == 0 ? hi : g == 1 ? lo : 0u;
            }
        float m = -INFINITY, ls = 0.f;  // the warp's running max (uniform) and this lane's part of the sum
        float o[4][4];                  // O^T accumulators: dims 16 dt + g (+8), columns 2c, 2c + 1
#pragma unroll
        for (int dt = 0; dt < 4; ++dt) o[dt][0] = o[dt][1] = o[dt][2] = o[dt][3] = 0.f;
        const int kvt = T->kvt, lold = T->lold;
        const int mi = lane >> 3, r8 = lane & 7;  // ldmatrix: this lane addresses row r8 of matrix mi
        // up to KVG tiles at a time as one run of n positions (v -> tile v / KVPOS, row v % KVPOS:
        // only the last tile of the range can be short); warp w takes the 16-position m-tiles
        // w and w + CW of the run (one online-softmax update for both)
        constexpr int KVG = (2 * CW * 16) / KVPOS;  // 4
        static_assert(KVG >= 1 && KVG <= NSLOT / 2, "K/V tiles per update");
        for (int t = T->t_lo; t < T->t_hi;) {
            const int ng = min(KVG, T->t_hi - t);
            const int n = min(ng * KVPOS, lold - t * KVPOS);
            if (n <= 0) {  // (only with no cached positions: nothing was copied)
                ++t;
                continue;
            }
            for (int gi = 0; gi < ng; ++gi) wait_seq(seq + gi, 3);
            const int ma = warp * 16, mb = (warp + CW) * 16;  // first positions of the two m-tiles
            if (ma < n) {
                const uint32_t ring0 = su32(smem);
                // K row of position v (row 0 of the first tile past the run)
                auto row_of = [&](int v) -> uint32_t {
                    const int vv = v < n ? v : 0, tt = vv / KVPOS;
                    return ring0 + ((seq + tt) & (NSLOT - 1)) * SLOT + (vv - tt * KVPOS) * 128;
                };
                // S = K q for the m-tile at v0: A fragments rows v0 + r8 (+8 for matrices 1, 3), k
                // chunks 2 kk (+1 for 2, 3); lanes (g, 0) get the scores of v0 + g and v0 + g + 8
                auto scores = [&](int v0, float &sa, float &sb) {
                    const uint32_t rk = row_of(v0 + r8 + (mi & 1) * 8);
                    float s0[4] = {0.f, 0.f, 0.f, 0.f}, s1[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
                    for (int kk = 0; kk < 4; kk += 2) {
                        uint32_t a0, a1, a2, a3, b0, b1, b2, b3;
                        ldsm_x4(swz(rk, 2 * kk + (mi >> 1)), a0, a1, a2, a3);
                        ldsm_x4(swz(rk, 2 * kk + 2 + (mi >> 1)), b0, b1, b2, b3);
                        mma16816(s0, a0, a1, a2, a3, qb[kk][0], qb[kk][1]);
                        mma16816(s1, b0, b1, b2, b3, qb[kk + 1][0], qb[kk + 1][1]);
                    }
                    sa = c == 0 && v0 + g < n ? (s0[0] + s0[1]) + (s1[0] + s1[1]) : -INFINITY;
                    sb = c == 0 && v0 + g + 8 < n ? (s0[2] + s0[3]) + (s1[2] + s1[3]) : -INFINITY;
                };
                // O^T += V^T P for the m-tile at v0 with its weights pa (position v0 + g) and pb
                // (v0 + g + 8) on lanes (g, 0): P as B fragments (lane (g, c) takes positions 2c,
                // 2c + 1 and 2c + 8, 2c + 9 from lanes (2c, 0) and (2c + 1, 0); column 0 fp16
                // values, column 1 remainders), V^T through ldmatrix.trans (positions v0 + r8, +8
                // for matrices 2, 3; dim chunks 2 dt, +1 for matrices 1, 3)
                auto accumulate = [&](int v0, float pa, float pb) {
                    const float p0 = __shfl_sync(0xffffffffu, pa, 8 * c), p8 = __shfl_sync(0xffffffffu, pb, 8 * c);
                    const float p1 = __shfl_sync(0xffffffffu, pa, 8 * c + 4);
                    const float p9 = __shfl_sync(0xffffffffu, pb, 8 * c + 4);
                    const __half2 h01 = __floats2half2_rn(p0, p1), h89 = __floats2half2_rn(p8, p9);
                    uint32_t pb0 = 0u, pb1 = 0u;
                    if (g == 0) {
                        pb0 = *reinterpret_cast<const uint32_t *>(&h01);
                        pb1 = *reinterpret_cast<const uint32_t *>(&h89);
                    } else if (g == 1) {
                        const float2 f01 = __half22float2(h01), f89 = __half22float2(h89);
                        pb0 = pack_h2(p0 - f01.x, p1 - f01.y);
                        pb1 = pack_h2(p8 - f89.x, p9 - f89.y);
                    }
                    const uint32_t rv = row_of(v0 + r8 + (mi >> 1) * 8) + KV_VOFF;
#pragma unroll
                    for (int dt = 0; dt < 4; ++dt) {
                        uint32_t a0, a1, a2, a3;
                        ldsm_x4_t(swz(rv, 2 * dt + (mi & 1)), a0, a1, a2, a3);
                        mma16816(o[dt], a0, a1, a2, a3, pb0, pb1);
                    }
                };
                const bool two = mb < n;  // (uniform)
                float sa, sb, sc = -INFINITY, sd = -INFINITY;
                scores(ma, sa, sb);
                if (two) scores(mb, sc, sd);
                float mt = fmaxf(fmaxf(sa, sb), fmaxf(sc, sd));
                mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, 4));
                mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, 8));
                mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, 16));
                mt = fmaxf(m, __shfl_sync(0xffffffffu, mt, 0));
                if (mt != m) {  // (uniform)
                    const float corr = exp2f(m - mt);
                    ls *= corr;
#pragma unroll
                    for (int dt = 0; dt < 4; ++dt)
#pragma unroll
                        for (int e = 0; e < 4; ++e) o[dt][e] *= corr;
                    m = mt;
                }
                // (positions past the run weigh 0; a NaN score of a position in it stays NaN)
                const bool c0 = c == 0;
                const float pa = c0 && ma + g < n ? exp2f(sa - m) : 0.f, pb = c0 && ma + g + 8 < n ? exp2f(sb - m) : 0.f;
                const float pc = c0 && mb + g < n ? exp2f(sc - m) : 0.f, pd = c0 && mb + g + 8 < n ? exp2f(sd - m) : 0.f;
                ls += (pa + pb) + (pc + pd);
                accumulate(ma, pa, pb);
                if (two) accumulate(mb, pc, pd);
            }
            release(ng);
            t += ng;
        }
        if (T->active && T->t_hi == kvt && T->t_hi > T->t_lo && warp == CW - 1) {  // the new position
            const float *kn = qkvh + 64, *vn = qkvh + 128;
            float s = fmaf(qkvh[2 * lane] * qscale, kn[2 * lane], qkvh[2 * lane + 1] * qscale * kn[2 * lane + 1]);
            s = warp_sum(s);
            const float mn = fmaxf(m, s), corr = exp2f(m - mn), pj = exp2f(s - mn);
            ls *= corr;
            if (lane == 0) ls += pj;
#pragma unroll
            for (int dt = 0; dt < 4; ++dt) {
#pragma unroll
                for (int e = 0; e < 4; ++e) o[dt][e] *= corr;
                if (c == 0) {
                    o[dt][0] = fmaf(pj, vn[16 * dt + g], o[dt][0]);
                    o[dt][2] = fmaf(pj, vn[16 * dt + g + 8], o[dt][2]);
                }
            }
            m = mn;
        }
        {  // the warp's state: m, l, and O (columns 0 + 1 of lanes (g, 0))
            const float lw = warp_sum(ls);
            float *sw = ascr + warp * REC;
            if (lane == 0) { sw[0] = m; sw[1] = lw; }
            if (c == 0) {
#pragma unroll
                for (int dt = 0; dt < 4; ++dt) {
                    sw[4 + 16 * dt + g] = o[dt][0] + o[dt][1];
                    sw[4 + 16 * dt + g + 8] = o[dt][2] + o[dt][3];
                }
            }
        }
        csync();
        float *rec = ascr + CW * REC;
        if (tid < 64) {
            float M = -INFINITY;
#pragma unroll
            for (int w = 0; w < CW; ++w) M = fmaxf(M, ascr[w * REC]);
            float L2 = 0.f, A2 = 0.f;
#pragma unroll
            for (int w = 0; w < CW; ++w) {
                const float mw = ascr[w * REC];
                const float f = mw == -INFINITY ? 0.f : exp2f(mw - M);
                L2 += ascr[w * REC + 1] * f;
                A2 += ascr[w * REC + 4 + tid] * f;
            }
            rec[4 + tid] = A2;
            if (tid == 0) { rec[0] = M; rec[1] = L2; rec[2] = 0.f; rec[3] = 0.f; }
        }
        csync();
        {  // this rank's record into slot [rank] of every CTA of the cluster (one 16-byte push
           // per thread)
            const uint32_t dst = su32(recs + rank * REC), bar = su32(stb + BR);
            if (tid < CS * (REC / 4)) {
                const int r = tid / (REC / 4), q = tid - r * (REC / 4);
                st_async_v4(mapa(dst + q * 16, r), reinterpret_cast<const uint4 *>(rec)[q], mapa(bar, r));
            }
        }
        // every CTA merges the six records itself: the head's 64 outputs (fp16, fragment order)
        // into xh, their sum into stat[0] + stat[1]
        wait_land(BR, 31);
        if (tid < 64) {
            float M = -INFINITY;
            for (int r = 0; r < CS; ++r) M = fmaxf(M, recs[r * REC]);
            float L2 = 0.f, A = 0.f;
            for (int r = 0; r < CS; ++r) {
                const float mr = recs[r * REC];
                const float f = mr == -INFINITY ? 0.f : exp2f(mr - M);
                L2 += recs[r * REC + 1] * f;
                A += recs[r * REC + 4 + tid] * f;
            }
            const __half hv = __float2half_rn(L2 > 0.f ? A * __frcp_rn(L2) : 0.f);
            xh[frag_pos_host(tid)] = hv;
            const float hs = warp_sum(__half2float(hv));  // (warps 0 and 1, all lanes)
            if (lane == 0) stat[warp] = hs;
        }
        csync();
        trace();
    }
    // c_proj of the cluster's head: this rank's range of the head-major chunks (16 rows x the
    // head's 64 inputs, one chunk per warp at a time); each row's partial is added to the
    // step's fixed-point accumulator (64-bit integer adds: the sum does not depend on their
    // order), then the CTA counts itself in
    __device__ __forceinline__ void stage_proj(int l) {
        const MkLin &P = lay[l].proj;
        const int nrb = P.n_rb, r0 = rank * nrb / CS, nc = (rank + 1) * nrb / CS - r0;
        const bool half_sb = pp->sbb == 4;
        const int cb = mk_projh_chunk_bytes(pp->sbb);
        const float hsum = stat[0] + stat[1];  // (read before the next LayerNorm rewrites stat)
        unsigned long long *acc = xp->hacc + ((size_t)par * pp->n_layers + l) * d;
        if (nc > 0) {
            const uint32_t slot = seq & (NSLOT - 1);
            wait_slot(slot, 4);
            const uint8_t *base = smem + slot * SLOT;
            const uint4 x0 = *reinterpret_cast<const uint4 *>(xh + c * 16);
            const uint4 x1 = *reinterpret_cast<const uint4 *>(xh + c * 16 + 8);
            // chunk i: 16 rows x the head's 64 inputs (one quantization group)
            auto chunk = [&](int i, float &y0, float &y1) {
                const uint8_t *tq = base + i * cb, *tsb = tq + 16 * 64;
                const uint4 wa = *reinterpret_cast<const uint4 *>(tq + g * 64 + c * 16);
                const uint4 wb = *reinterpret_cast<const uint4 *>(tq + (g + 8) * 64 + c * 16);
                float d0[4] = {0.f, 0.f, 0.f, 0.f}, d1[4] = {0.f, 0.f, 0.f, 0.f};
                mma16816(d0, lo_h(wa.x), lo_h(wb.x), hi_h(wa.x), hi_h(wb.x), x0.x, x0.y);
                mma16816(d1, lo_h(wa.y), lo_h(wb.y), hi_h(wa.y), hi_h(wb.y), x0.z, x0.w);
                mma16816(d0, lo_h(wa.z), lo_h(wb.z), hi_h(wa.z), hi_h(wb.z), x1.x, x1.y);
                mma16816(d1, lo_h(wa.w), lo_h(wb.w), hi_h(wa.w), hi_h(wb.w), x1.z, x1.w);
                float s0, z0, s1, z1;
                if (half_sb) {
                    const float2 f0 = __half22float2(*reinterpret_cast<const __half2 *>(tsb + g * 4));
                    const float2 f1 = __half22float2(*reinterpret_cast<const __half2 *>(tsb + (g + 8) * 4));
                    s0 = f0.x; z0 = f0.y; s1 = f1.x; z1 = f1.y;
                } else {
                    const float2 f0 = *reinterpret_cast<const float2 *>(tsb + g * 8);
                    const float2 f1 = *reinterpret_cast<const float2 *>(tsb + (g + 8) * 8);
                    s0 = f0.x; z0 = f0.y; s1 = f1.x; z1 = f1.y;
                }
                y0 = fmaf(s0, d0[0] + d1[0], fmaf(-1024.0f, s0, z0) * hsum);
                y1 = fmaf(s1, d0[2] + d1[2], fmaf(-1024.0f, s1, z1) * hsum);
            };
            // this warp's chunks warp and warp + CW (nc <= 2 CW), computed together (the second
            // one twice when absent) so that their loads and mma chains overlap; the slot is
            // released before the adds, so that the release does not order them
            const int i = warp, i2 = i + CW < nc ? i + CW : i;
            float y0 = 0.f, y1 = 0.f, y2 = 0.f, y3 = 0.f;
            if (i < nc) {
                chunk(i, y0, y1);
                chunk(i2, y2, y3);
            }
            release(1);
            if (c == 0 && i < nc) {
                const int o = (r0 + i) * 16;
                add_part(acc + o + g, y0);
                add_part(acc + o + g + 8, y1);
                if (i2 != i) {
                    const int o2 = (r0 + i2) * 16;
                    add_part(acc + o2 + g, y2);
                    add_part(acc + o2 + g + 8, y3);
                }
            }
        }
        trace();
    }
    // The MLP by slices: cluster c owns the S = ff / H inputs [S c, S c + S) of the mlp
    // projection.  Its ranks compute those S c_fc rows (TM_FC) and push GELU of them as fp16
    // into the xu of every CTA of the cluster (fragment order, one mbarrier: S x 2 bytes); then
    // each rank applies the K-slice of the mlp projection to them for its share of the d
    // outputs and adds the partials into the next x's fixed-point accumulator.  No vector of
    // the MLP crosses clusters except the result.
    __device__ __forceinline__ void stage_fc(int l) {
        const MkLayer &Ly = lay[l];
        const LnRegs ln2 = ln_prefetch(Ly.ln2_w, Ly.ln2_b);
        const float4 bpre = bias_pre<CS>(Ly.fc, TM_FC);
        const int hc0 = slice_lo(rank, d / 4) * 4;
        const float4 hbias = tid < slice_lo(rank + 1, d / 4) - slice_lo(rank, d / 4)
                                 ? __ldg(reinterpret_cast<const float4 *>(Ly.proj.bias + hc0 + tid * 4))
                                 : make_float4(0.f, 0.f, 0.f, 0.f);
        exchange_h(l, hbias, 50);
        layernorm(ln2, false);
        const MkLin &L = Ly.fc;
        const int S = ff / pp->H, lo0 = head * S;
        const uint32_t xu_a = su32(xu), bar_a = su32(stb + BU);
        run_lin<CS>(L, xln, sxln, bpre, TM_FC, [&](int o, float4 v, float4 bb, int r) {
            // rows o..o+3 of the slice -> positions frag_pos(k), frag_pos(k) + 1 (k = o & 63)
            // and frag_pos(k + 2), + 1 of their group: two fp16 pairs, into cluster rank r
            const int lo = o - lo0, g = lo >> 6, k = lo & 63;
            const uint32_t p01 = pack_h2(gelu_tanh(v.x + bb.x), gelu_tanh(v.y + bb.y));
            const uint32_t p23 = pack_h2(gelu_tanh(v.z + bb.z), gelu_tanh(v.w + bb.w));
            const uint32_t a01 = xu_a + (g * 64 + frag_pos_host(k)) * 2, a23 = xu_a + (g * 64 + frag_pos_host(k + 2)) * 2;
            st_async_b32(mapa(a01, r), p01, mapa(bar_a, r));
            st_async_b32(mapa(a23, r), p23, mapa(bar_a, r));
        });
    }
    // The sub-tiles (16 rows x the slice's S <= 256 inputs) are applied in halves (S / 2
    // inputs each): slot by slot as they land, half h of this rank's run goes to warp h % CW,
    // which adds its rows' partials straight into the accumulator words (two partials per
    // row and cluster).  Every warp waits for each slot before releasing it, so that its
    // release counts towards the slot's current use.
    __device__ __forceinline__ void stage_mlp(int l) {
        wait_land(BU, 60);
        const int S = ff / pp->H, G = S / 64;  // G is 2 or 4 (xk_config)
        // the slice's group sums (the dequantization offset term), from the fp16 values
        if (warp < G) {
            const __half2 *u2 = reinterpret_cast<const __half2 *>(xu + warp * 64);
            const float2 f = __half22float2(u2[lane]);
            sxu[warp] = warp_sum(f.x + f.y);
        }
        csync();
        // group j of a sub-tile against the slice's activation fragment (from shared memory)
        auto grp_j = [&](const uint8_t *tq, const uint8_t *tsb, int j, bool half_sb, float &a0, float &a1) {
            const uint4 x0 = *reinterpret_cast<const uint4 *>(xu + j * 64 + c * 16);
            const uint4 x1 = *reinterpret_cast<const uint4 *>(xu + j * 64 + c * 16 + 8);
            group_x(tq, tsb, S, G, j, x0, x1, sxu[j], half_sb, a0, a1);
        };
        const MkLin &L = lay[l].mlp;
        const bool half_sb = pp->sbb == 4;
        const int sub = mk_mlpk_sub_bytes(S, pp->sbb), per_slot = SLOT / sub;
        const int nrb = L.n_rb, mine = rank < nrb ? (nrb - 1 - rank) / CS + 1 : 0;
        unsigned long long *acc = xp->xacc + ((size_t)par * pp->n_layers + l) * d;
        for (int s_lo = 0; s_lo < mine; s_lo += per_slot) {
            const int nh = 2 * (min(mine, s_lo + per_slot) - s_lo);
            wait_seq(seq, 4);
            // this warp's halves of the slot (at most 2: per_slot <= CW), computed before the
            // slot is released and added after, so that the release does not order the adds
            float r[2][2];
            int ro[2];
#pragma unroll
            for (int u = 0; u < 2; ++u) {
                const int h = (warp + CW - (2 * s_lo) % CW) % CW + u * CW;
                r[u][0] = r[u][1] = 0.f;
                ro[u] = -1;
                if (h < nh) {
                    const uint8_t *tq = ring_at(seq) + (h >> 1) * sub, *tsb = tq + 16 * S;
                    const int j0 = (h & 1) * (G / 2);  // this half's first group
                    grp_j(tq, tsb, j0, half_sb, r[u][0], r[u][1]);
                    if (G == 4) grp_j(tq, tsb, j0 + 1, half_sb, r[u][0], r[u][1]);
                    ro[u] = (rank + CS * (s_lo + (h >> 1))) * 16;
                }
            }
            release(1);  // (every consumer warp, once per slot)
            if (c == 0) {
#pragma unroll
                for (int u = 0; u < 2; ++u)
                    if (ro[u] >= 0) {
                        add_part(acc + ro[u] + g, r[u][0]);
                        add_part(acc + ro[u] + g + 8, r[u][1]);
                    }
            }
        }
        trace();
    }
    __device__ __forceinline__ void stage_head() {
        const MkParams &p = *pp;
        const LnRegs lnf = ln_prefetch(p.lnf_w, p.lnf_b);
        const LnRegs fin = ln_prefetch(p.fin_w, p.fin_b);
        const float4 bpre = bias_pre<1>(p.head, TM_RR);
        exchange_x(p.n_layers - 1, 70);
        layernorm(lnf, true);
        layernorm(fin, false);
        const MkLin &L = p.head;
        const int V = p.mel_vocab;
        run_lin<1>(L, xln, sxln, bpre, TM_RR, [&](int o, float4 v, float4 bb, int) {
            const float vv[4] = {v.x + bb.x, v.y + bb.y, v.z + bb.z, v.w + bb.w};
#pragma unroll
            for (int e = 0; e < 4; ++e)
                if (o + e < V) p.logits[o + e] = vv[e];
        });
    }
};

// ---------------------------------------------------------------------------
// kernel
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(NT, 1) xk_decode_kernel(const __grid_constant__ XkParams xp) {
    extern __shared__ __align__(1024) uint8_t smem[];
    if (xp.dry) {  // launch-configuration probe
        cluster_sync_all();
        return;
    }
    // the K/V tiles' 128-byte swizzle is laid out for 1,024-aligned ring slots (the same in
    // every CTA, so all of them leave here together)
    if (su32(smem) & 1023u) {
        if (threadIdx.x == 0) atomicExch(xp.p.err, 98);
        return;
    }
    const MkParams &p = xp.p;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    uint32_t rank_u;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(rank_u));
    const int rank = (int)rank_u, R = blockIdx.x, NR = gridDim.x;
    const XkSmem SL = xk_layout(p.d, p.ff, xp.rt, p.n_layers);
    XkTab *T = reinterpret_cast<XkTab *>(smem + SL.tab);
    uint64_t *fullp = reinterpret_cast<uint64_t *>(smem + SL.bar);
    uint64_t *emptyp = fullp + NSLOT;
    uint64_t *stb = emptyp + NSLOT;

    // Global loads issued ahead of the set-up, so that their latencies overlap: the layer
    // table, this CTA's launch counter, the slot state and then the embedding rows it names.
    const int words = (int)(p.n_layers * sizeof(MkLayer) / 4);
    const uint32_t *tsrc = reinterpret_cast<const uint32_t *>(p.layers);
    uint32_t tw[TABW];
#pragma unroll
    for (int j = 0; j < TABW; ++j) {
        const int i = tid + j * NT;
        tw[j] = i < words ? __ldg(tsrc + i) : 0u;
    }
    const uint32_t epoch = xp.epoch[R];
    // step shape: cluster c runs head c; rank k of it the k-th of CS ranges of the K/V tiles
    const int slot = p.batch_slot[0];
    const SlotState &st = p.slots[slot];
    const int active = st.active && st.valid_len < p.max_seq;
    const int lold = active ? st.valid_len : 0;
    const int kvt = active ? max(1, (lold + KVPOS - 1) / KVPOS) : 0;
    const int head = R / CS;
    const int tok = min(max(st.tok, 0), p.mel_vocab - 1), pos = min(max(st.pos, 0), p.mel_pos_len - 1);
    float emb[EMBW];  // layer 0's input x = mel_emb[tok] + mel_pos[pos] (gpt.rs:706-754)
    {
        const float *e = p.mel_emb + (size_t)tok * p.d, *ps = p.mel_pos + (size_t)pos * p.d;
#pragma unroll
        for (int j = 0; j < EMBW; ++j) {
            const int k = tid + j * CT;
            emb[j] = tid < CT && k < p.d ? __ldg(e + k) + __ldg(ps + k) : 0.f;
        }
    }
    // A step of a request that has stopped (sampler.rs:378) or failed does nothing: every
    // CTA reads the same slot state, so all of them leave here, before any barrier, copy or
    // write (the launch counter and the accumulators stay as the last real step left them).
    if (!active) return;
    // Test hook: a bounded wait on a word that nothing sets, made before any barrier, copy,
    // push or write of the step, so that every CTA leaves here the way a stopped request's
    // step does and the host reads the timeout from the error word.
    if (p.stall > 0) {
        if (tid == 0) {
            const volatile int *never = p.err + 3;
            int it = 0;
            while (it < p.stall && *never == 0) {
                __nanosleep(1000);
                ++it;
            }
            if (it == p.stall) atomicExch(p.err, MK_ERR_STALL);
        }
        return;
    }
    if (p.trace && tid == 0) {  // stamp 0: the CTA starts (SM clock cycles, as every stamp)
        unsigned long long t;
        asm volatile("mov.u64 %0, %%clock64;" : "=l"(t));
        p.trace[(size_t)R * MK_TRACE_EVENTS] = t;
    }
    {
        uint32_t *dst = reinterpret_cast<uint32_t *>(smem + SL.lay);
#pragma unroll
        for (int j = 0; j < TABW; ++j) {
            const int i = tid + j * NT;
            if (i < words) dst[i] = tw[j];
        }
        for (int i = tid + TABW * NT; i < words; i += NT) dst[i] = tsrc[i];
    }
    if (tid < CT) {  // (no peer pushes into land before this CTA's own layer-0 rows are out)
        float *land = reinterpret_cast<float *>(smem + SL.land);
#pragma unroll
        for (int j = 0; j < EMBW; ++j) {
            const int k = tid + j * CT;
            if (k < p.d) land[k] = emb[j];
        }
    }
    if (tid == 0) {
        for (int s = 0; s < NSLOT; ++s) {
            mb_init(fullp + s, 1);
            mb_init(emptyp + s, CW);
        }
        for (int b = 0; b < NSTB; ++b) mb_init(stb + b, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        mb_expect(stb + B0, (uint32_t)p.d * 4);
        mb_expect(stb + BU, (uint32_t)(p.ff / p.H) * 2);  // the cluster's slice of GELU(c_fc), fp16
        mb_expect(stb + BQ, 3 * 64 * 4);
        mb_expect(stb + BR, CS * REC * 4);  // (waited on by rank 0 only)
        T->active = active;
        T->lold = lold;
        T->kvt = kvt;
        T->slot = slot;
        T->head = head;
        // ranges rounded up, so the last rank (which also takes the new position) has the
        // smaller share
        T->t_lo = (rank * kvt + CS - 1) / CS;
        T->t_hi = ((rank + 1) * kvt + CS - 1) / CS;
        T->tok = tok;
        T->pos = pos;
    }
    __syncthreads();
    {  // the next step's accumulator words (this step's were zeroed by the last)
        const uint32_t q = (epoch & 1u) ^ 1u;
        const size_t n = (size_t)p.n_layers * p.d;
        unsigned long long *a = xp.hacc + q * n, *ax = xp.xacc + q * n;
        for (size_t i = (size_t)R * NT + tid; i < n; i += (size_t)NR * NT) {
            a[i] = 0ull;
            ax[i] = 0ull;
        }
    }
    // every CTA's barriers are armed before any CTA pushes into them
    cluster_sync_all();

    if (warp == CW) {
        if (lane == 0) {
            XkProducer P;
            P.ring = su32(smem);
            P.full = su32(fullp);
            P.fullp = fullp;
            P.emptyp = emptyp;
            P.err = p.err;
            asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(P.pol));
            P.seq = 0;
            P.R = R;
            P.NR = NR;
            P.ok = true;
            P.run(xp, *T, reinterpret_cast<const MkLayer *>(smem + SL.lay), rank);
        }
        __syncwarp();
    } else {
        XkConsumer C;
        C.xp = &xp;
        C.pp = &p;
        C.T = T;
        C.lay = reinterpret_cast<const MkLayer *>(smem + SL.lay);
        C.smem = smem;
        C.land = reinterpret_cast<float *>(smem + SL.land);
        C.xln = reinterpret_cast<__half *>(smem + SL.xln);
        C.xh = reinterpret_cast<__half *>(smem + SL.xh);
        C.par = epoch & 1u;
        C.xu = reinterpret_cast<__half *>(smem + SL.xu);
        C.sxln = reinterpret_cast<float *>(smem + SL.sxln);
        C.sxu = reinterpret_cast<float *>(smem + SL.sxu);
        C.red = reinterpret_cast<float *>(smem + SL.red);
        C.qkvh = reinterpret_cast<float *>(smem + SL.qkvh);
        C.recs = reinterpret_cast<float *>(smem + SL.recs);
        C.head = head;
        C.stat = reinterpret_cast<float *>(smem + SL.stat);
        C.fullp = fullp;
        C.emptyp = emptyp;
        C.stb = stb;
        C.tid = tid;
        C.warp = warp;
        C.lane = lane;
        C.g = lane >> 2;
        C.c = lane & 3;
        C.rank = rank;
        C.R = R;
        C.NR = NR;
        C.d = p.d;
        C.ff = p.ff;
        C.H = p.H;
        C.rt = xp.rt;
        C.seq = 0;
        C.ok = true;
        C.ev = 1;
        for (int b = 0; b < NSTB; ++b) C.ph[b] = 0;
        C.exp_bytes[B0] = (uint32_t)p.d * 4;
        C.exp_bytes[BU] = (uint32_t)(p.ff / p.H) * 2;
        C.exp_bytes[BQ] = 3 * 64 * 4;
        C.exp_bytes[BR] = CS * REC * 4;
        for (int l = 0; l < p.n_layers; ++l) {
            C.stage_qkv(l);
            C.stage_attn(l);
            C.stage_proj(l);
            C.stage_fc(l);
            C.stage_mlp(l);
        }
        C.stage_head();
    }
    __syncwarp();
    cluster_sync_all();  // no CTA leaves while a peer may still push into its shared memory
    if (tid == 0) xp.epoch[R] = epoch + 1;
    if (p.trace && tid == 0) {  // last stamp slot: the CTA ends
        unsigned long long t;
        asm volatile("mov.u64 %0, %%clock64;" : "=l"(t));
        p.trace[(size_t)R * MK_TRACE_EVENTS + MK_TRACE_EVENTS - 1] = t;
    }
}

cudaError_t xk_launch_cfg(const XkParams &xp, int grid, size_t smem, bool coop, cudaStream_t st) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(NT);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute at[2];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = CS;
    at[0].val.clusterDim.y = 1;
    at[0].val.clusterDim.z = 1;
    at[1].id = cudaLaunchAttributeCooperative;
    at[1].val.cooperative = 1;
    cfg.attrs = at;
    cfg.numAttrs = coop ? 2 : 1;
    return cudaLaunchKernelEx(&cfg, xk_decode_kernel, xp);
}

}  // namespace

static int xk_tiles_of(const MkLin &L, int nr) { return (L.n_rb * L.n_kc + nr - 1) / nr; }

int xk_config(const ModelView &m, XkConfig *out) {
    *out = XkConfig{};
    const char *off = getenv("ITTS_XK");
    if (off && off[0] == '0') return -1;
    if (m.n_layers < 1 || m.d > MK_MAX_KC || m.d % 64 || m.ff % 64 || m.n_heads * 64 != m.d || m.d / 4 < CS ||
        m.ff / 64 < CS || m.n_heads > kFxMaxHeads)
        return -1;
    int dev = 0, optin = 0, sms = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    for (int l = 0; l < m.n_layers; ++l) {
        const MkLayer &L = m.layers[l];
        for (const MkLin *x : {&L.qkv, &L.proj, &L.fc, &L.mlp})
            if (x->tile_bytes > SLOT || x->kc % 64) return -1;
        if (L.qkv.n_kc != 1 || L.proj.n_kc != 1 || L.fc.n_kc != 1) return -1;
        if (!L.proj_h || (L.proj.n_rb + CS - 1) / CS * mk_projh_chunk_bytes(L.proj.sbb) > SLOT ||
            (L.proj.n_rb + CS - 1) / CS > 2 * CW)
            return -1;
        if (L.qkv.out != 3 * m.d || L.proj.out != m.d || L.fc.out != m.ff || L.mlp.out != m.d) return -1;
        if (!L.mlp_k || !mlp_slice_ok(L.mlp, m.n_heads)) return -1;
    }
    if (m.mel_head.tile_bytes > SLOT || m.mel_head.n_kc != 1) return -1;
    // grid: one CS-CTA cluster per attention head, all resident at once
    const int rt_guess = 8;
    size_t smem = xk_layout(m.d, m.ff, rt_guess, m.n_layers).total;
    if ((int)smem > optin) return -1;
    if (cudaFuncSetAttribute(xk_decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess) {
        cudaGetLastError();
        return -1;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(CS);
    cfg.blockDim = dim3(NT);
    cfg.dynamicSmemBytes = smem;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = CS;
    at[0].val.clusterDim.y = 1;
    at[0].val.clusterDim.z = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    int ncl = 0;
    if (cudaOccupancyMaxActiveClusters(&ncl, xk_decode_kernel, &cfg) != cudaSuccess || ncl < 1) {
        cudaGetLastError();
        return -1;
    }
    if (ncl < m.n_heads || m.n_heads * CS > sms) {
        if (getenv("ITTS_DEBUG")) fprintf(stderr, "[itts] clustered decode kernel: %d heads, %d clusters fit\n", m.n_heads, ncl);
        return -1;
    }
    const int grid = m.n_heads * CS;
    int rt = 1;
    for (int l = 0; l < m.n_layers; ++l) {
        const MkLayer &L = m.layers[l];
        for (const MkLin *x : {&L.qkv, &L.proj, &L.fc}) rt = std::max(rt, xk_tiles_of(*x, grid));
    }
    rt = std::max(rt, (QT + CS - 1) / CS);  // this rank's share of the head's QKV row blocks
    rt = std::min(rt, rt_guess);
    smem = xk_layout(m.d, m.ff, rt, m.n_layers).total;
    cudaFuncSetAttribute(xk_decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    // probe the launch form: cooperative (co-residency guaranteed) with clusters, else plain
    XkParams probe{};
    probe.dry = 1;
    // ITTS_XK_COOP=0: plain cluster launch (co-residency then rests on the grid fitting the
    // device at once, which the cluster count above ensures; profilers replay it)
    const char *cp = getenv("ITTS_XK_COOP");
    bool coop = !(cp && cp[0] == '0');
    cudaError_t e = coop ? xk_launch_cfg(probe, grid, smem, true, 0) : cudaErrorNotSupported;
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e != cudaSuccess) {
        cudaGetLastError();
        coop = false;
        e = xk_launch_cfg(probe, grid, smem, false, 0);
        if (e == cudaSuccess) e = cudaDeviceSynchronize();
        if (e != cudaSuccess) {
            cudaGetLastError();
            return -1;
        }
    }
    out->grid = grid;
    out->rt = rt;
    out->coop = coop ? 1 : 0;
    if (getenv("ITTS_DEBUG"))
        fprintf(stderr, "[itts] clustered decode kernel: grid %d (%d-CTA clusters, %s), %zu B shared memory, rt %d\n",
                grid, CS, coop ? "cooperative" : "plain", smem, rt);
    return grid;
}

cudaError_t xk_make_kv_maps(const ModelView &m, __half *k_cache, __half *v_cache, int n_slots, int max_seq,
                            XkBufs &b) {
    EncodeTiledFn enc = encode_tiled();
    if (!enc || n_slots < 1 || max_seq < 1) return cudaErrorNotSupported;
    // kv_index order: ((layer * n_slots + slot) * heads + head) * max_seq + pos, 64 values each
    const cuuint64_t rowb = kHeadDim * sizeof(__half);
    const cuuint64_t dims[5] = {(cuuint64_t)kHeadDim, (cuuint64_t)max_seq, (cuuint64_t)m.n_heads, (cuuint64_t)n_slots,
                                (cuuint64_t)m.n_layers};
    const cuuint64_t strides[4] = {rowb, rowb * max_seq, rowb * max_seq * m.n_heads,
                                   rowb * max_seq * m.n_heads * n_slots};
    const cuuint32_t box[5] = {(cuuint32_t)kHeadDim, (cuuint32_t)KVPOS, 1, 1, 1};
    const cuuint32_t estr[5] = {1, 1, 1, 1, 1};
    for (int i = 0; i < 2; ++i)
        if (enc(i ? &b.vmap : &b.kmap, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 5, i ? v_cache : k_cache, dims, strides, box,
                estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return cudaErrorInvalidValue;
    return cudaSuccess;
}

cudaError_t xk_launch(const MkParams &p, const XkConfig &xc, const XkBufs &b, cudaStream_t st) {
    XkParams xp{};
    xp.p = p;
    xp.kmap = b.kmap;
    xp.vmap = b.vmap;
    xp.hacc = b.hacc;
    xp.xacc = b.xacc;
    xp.epoch = b.epoch;
    xp.rt = xc.rt;
    xp.dry = 0;
    return xk_launch_cfg(xp, xc.grid, xk_layout(p.d, p.ff, xc.rt, p.n_layers).total, xc.coop != 0, st);
}

// chunk (h, rb) of the head-major c_proj copy from tile rb (n_kc == 1): row m's bytes of group h
// (stored at group slot h ^ (m & 1) in the tile) to 64 m, then the 16 rows' (scale, offset)
// pairs of group h
__global__ void proj_by_head_kernel(const uint8_t *tiles, int tile_bytes, int kc, int sbb, uint8_t *dst) {
    const int rb = blockIdx.x, h = blockIdx.y, n_rb = gridDim.x, G64 = kc / 64;
    const uint8_t *t = tiles + (size_t)rb * tile_bytes;
    uint8_t *o = dst + ((size_t)h * n_rb + rb) * mk_projh_chunk_bytes(sbb);
    for (int i = threadIdx.x; i < 16 * 16; i += blockDim.x) {  // 16 rows x 16 words
        const int m = i >> 4, w = i & 15;
        reinterpret_cast<uint32_t *>(o + m * 64)[w] =
            reinterpret_cast<const uint32_t *>(t + (size_t)m * kc + (h ^ (m & 1)) * 64)[w];
    }
    for (int i = threadIdx.x; i < 16 * sbb / 4; i += blockDim.x) {
        const int m = i / (sbb / 4), w = i - m * (sbb / 4);
        reinterpret_cast<uint32_t *>(o + 16 * 64 + m * sbb)[w] =
            reinterpret_cast<const uint32_t *>(t + 16 * kc + (size_t)(m * G64 + h) * sbb)[w];
    }
}

// sub-tile (cluster c, row block rb) of the sliced mlp copy (MkLayer::mlp_k) from tile
// (rb, kc) with kc = S c / KC: each row's S bytes of the slice (its groups keep their slots:
// the row-parity swizzle stays inside the slice, whose group count is even), then the rows'
// (scale, offset) pairs of the slice's groups; placed in the copy so that each rank's
// sub-tiles (row blocks rank, rank + 6, ...) are contiguous
__global__ void mlp_by_slice_kernel(const uint8_t *tiles, int tile_bytes, int kc, int n_kc, int sbb, int S,
                                    uint8_t *dst) {
    const int rb = blockIdx.x, c = blockIdx.y, n_rb = gridDim.x, G = S / 64, G64 = kc / 64;
    const int kci = S * c / kc, q = (S * c - kci * kc) / 64;
    const uint8_t *t = tiles + ((size_t)rb * n_kc + kci) * tile_bytes;
    const int sub = mk_mlpk_sub_bytes(S, sbb);
    uint8_t *o = dst + mk_mlpk_rank_offset(n_rb, S, sbb, c, rb % 6) + (size_t)(rb / 6) * sub;
    const int wpr = S / 4;  // words per row
    for (int i = threadIdx.x; i < 16 * wpr; i += blockDim.x) {
        const int m = i / wpr, w = i - m * wpr;
        reinterpret_cast<uint32_t *>(o + m * S)[w] = reinterpret_cast<const uint32_t *>(t + (size_t)m * kc + q * 64)[w];
    }
    const int spw = sbb / 4;  // words per (scale, offset) pair
    for (int i = threadIdx.x; i < 16 * G * spw; i += blockDim.x) {
        const int m = i / (G * spw), r = i - m * G * spw, j = r / spw, w = r - j * spw;
        reinterpret_cast<uint32_t *>(o + 16 * S + (m * G + j) * sbb)[w] =
            reinterpret_cast<const uint32_t *>(t + 16 * kc + (size_t)(m * G64 + q + j) * sbb)[w];
    }
}

bool mlp_slice_ok(const MkLin &W, int n_heads) {
    const int S = W.in / n_heads;
    return n_heads > 0 && W.in % n_heads == 0 && S % 128 == 0 && S <= 256 && W.kc % S == 0 &&
           mk_mlpk_sub_bytes(S, W.sbb) <= SLOT && SLOT / mk_mlpk_sub_bytes(S, W.sbb) <= CW;
}

size_t mlp_slice_bytes(const MkLin &W, int n_heads) {
    return (size_t)n_heads * W.n_rb * mk_mlpk_sub_bytes(W.in / n_heads, W.sbb);
}

cudaError_t make_mlp_by_slice(const MkLin &W, int n_heads, uint8_t *dst, cudaStream_t st) {
    if (!mlp_slice_ok(W, n_heads)) return cudaErrorInvalidValue;
    mlp_by_slice_kernel<<<dim3(W.n_rb, n_heads), 128, 0, st>>>(W.tiles, W.tile_bytes, W.kc, W.n_kc, W.sbb,
                                                               W.in / n_heads, dst);
    return cudaGetLastError();
}

cudaError_t make_proj_by_head(const MkLin &W, int n_heads, uint8_t *dst, cudaStream_t st) {
    if (W.n_kc != 1 || W.kc != n_heads * 64) return cudaErrorInvalidValue;
    proj_by_head_kernel<<<dim3(W.n_rb, n_heads), 128, 0, st>>>(W.tiles, W.tile_bytes, W.kc, W.sbb, dst);
    return cudaGetLastError();
}

}  // namespace itts
