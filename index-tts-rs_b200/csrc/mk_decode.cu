// mk_decode.cu -- the persistent decode-step kernel for 1..4 batch columns: one
// cooperative launch runs the whole decoder step (crates/core/src/models/gpt.rs:706-754):
// step embedding, n_layers x [LN1 -> QKV -> KV append -> attention -> c_proj + residual ->
// LN2 -> c_fc + GELU -> mlp c_proj + residual], ln_f -> final_norm -> mel_head.
//
// Design (one CTA per SM, 8 consumer warps + 1 producer warp):
//  * Weights are pre-tiled (mk.h) into 16-row x KC-byte tiles carrying their (scale,
//    offset) pairs.  The tiles of a step and the cached K/V rows each attention unit reads
//    are dealt round-robin to the CTAs in a fixed order that every CTA computes.
//  * The producer warp streams its CTA's tiles with cp.async.bulk into a ring of
//    shared-memory slots (mbarrier complete_tx).  Weights and old K/V rows do not depend
//    on the step's activations, so the producer runs ahead across stage and layer
//    boundaries and HBM stays busy while consumers wait for activations.
//  * Consumers dequantize int8 -> fp16 in registers (the byte in the mantissa of 1024.0
//    gives 1024 + q exactly) and run mma.sync m16n8k16 with the activation as the 8-wide
//    B operand; per quantization group  y += s * D + (b - 1024 s) * sum(x).
//  * Activations cross CTAs as 64-bit LL words {fp32 value, stage tag} in per-layer
//    buffers (mk.h).  A stage polls exactly the words it consumes (all loads of a poll
//    round are issued before any check, so a round costs one L2 round trip) until the
//    tags match: no grid barrier, no flag, and no buffer is rewritten within a step.
//    Tags are per-CTA launch counters x stages + stage index, so a word from an
//    earlier step never matches.  Every spin is bounded and raises an error word.
#include <cstdio>
#include <cstdlib>

#include "kernels.h"
#include "mk.h"

namespace itts {

constexpr int MK_CWARPS = 8;
constexpr int MK_NTHR = MK_CWARPS * 32;
constexpr int MK_THREADS = MK_NTHR + 32;
constexpr int MK_KVPOS = 96;  // positions per KV tile: 96 * 128 B * 2 = 24 KB
constexpr uint32_t MK_SPIN_LIMIT = 1u << 22;
constexpr int MK_STAGES = 5;  // per layer: qkv, attention, h, u, x

// ------------------------------------------------------------------------------
// PTX helpers
// ------------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ void mbar_init(uint64_t *b, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(b)), "r"(count));
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t *b, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(b)),
                 "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t *b) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(b)) : "memory");
}
// Bounded wait for the phase with parity `par`; false on timeout or when another CTA
// raised the error word.
__device__ __forceinline__ bool mbar_wait(uint64_t *b, uint32_t par, const int *err) {
    const uint32_t a = smem_u32(b);
    for (uint32_t it = 0; it < MK_SPIN_LIMIT; ++it) {
        if ((it & 65535u) == 65535u && *(volatile const int *)err) return false;
        uint32_t done;
        asm volatile(
            "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
            " selp.u32 %0, 1, 0, p;\n}\n"
            : "=r"(done)
            : "r"(a), "r"(par)
            : "memory");
        if (done) return true;
    }
    return false;
}
// Bulk copy global -> shared completing on `bar`, marked evict-first in L2 so that the
// streamed weights and K/V rows do not push the small hot data (activations, LayerNorm
// parameters) out of L2.
// The producer's wait for a free slot: not latency critical, so it sleeps between polls
// instead of taking issue slots from the consumer warps.
__device__ __forceinline__ bool mbar_wait_sleep(uint64_t *b, uint32_t par, const int *err) {
    const uint32_t a = smem_u32(b);
    for (uint32_t it = 0; it < MK_SPIN_LIMIT; ++it) {
        uint32_t done;
        asm volatile(
            "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
            " selp.u32 %0, 1, 0, p;\n}\n"
            : "=r"(done)
            : "r"(a), "r"(par)
            : "memory");
        if (done) return true;
        if ((it & 1023u) == 1023u && *(volatile const int *)err) return false;
        __nanosleep(64);
    }
    return false;
}
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar,
                                         uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, "
        "[%3], %4;" ::"r"(smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}
__device__ __forceinline__ uint64_t evict_first_policy() {
    uint64_t pol;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
    return pol;
}
__device__ __forceinline__ void named_sync() {
    asm volatile("bar.sync 1, %0;" ::"n"(MK_NTHR) : "memory");
}
__device__ __forceinline__ void mma16816(float *d, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
        "{%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void ll_st(uint64_t *p, float v, uint32_t tag) {
    const uint64_t w = ((uint64_t)tag << 32) | (uint64_t)__float_as_uint(v);
    asm volatile("st.relaxed.gpu.global.b64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}
__device__ __forceinline__ void ll_ld2(const uint64_t *p, uint64_t &a, uint64_t &b) {
    asm volatile("ld.relaxed.gpu.global.v2.b64 {%0,%1}, [%2];" : "=l"(a), "=l"(b) : "l"(p) : "memory");
}
__device__ __forceinline__ float ll_val(uint64_t w) { return __uint_as_float((uint32_t)w); }
__device__ __forceinline__ bool ll_tag_ok(uint64_t w, uint32_t tag) { return (uint32_t)(w >> 32) == tag; }
__device__ __forceinline__ unsigned long long globaltimer() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Polls up to MAXC chunks of 4 LL words (32-byte aligned) until every tag equals `tag`.
// ptr(j) gives chunk j's address or nullptr; out(j, v) receives a ready chunk.  All loads
// of a round are issued before any check.  False on timeout / error word.
template <int MAXC, typename PtrF, typename OutF>
__device__ __forceinline__ bool ll_poll4(PtrF ptr, uint32_t tag, OutF out, const int *err) {
    uint32_t pending = 0;
#pragma unroll
    for (int j = 0; j < MAXC; ++j)
        if (ptr(j)) pending |= 1u << j;
    for (uint32_t it = 0; pending; ++it) {
        uint64_t w[MAXC][4];
#pragma unroll
        for (int j = 0; j < MAXC; ++j) {
            if ((pending >> j) & 1u) {
                const uint64_t *q = ptr(j);
                ll_ld2(q, w[j][0], w[j][1]);
                ll_ld2(q + 2, w[j][2], w[j][3]);
            }
        }
#pragma unroll
        for (int j = 0; j < MAXC; ++j) {
            if (((pending >> j) & 1u) && ll_tag_ok(w[j][0], tag) && ll_tag_ok(w[j][1], tag) &&
                ll_tag_ok(w[j][2], tag) && ll_tag_ok(w[j][3], tag)) {
                out(j, make_float4(ll_val(w[j][0]), ll_val(w[j][1]), ll_val(w[j][2]), ll_val(w[j][3])));
                pending &= ~(1u << j);
            }
        }
        if (pending) {
            if (it >= MK_SPIN_LIMIT || ((it & 255u) == 255u && *(volatile const int *)err)) return false;
            // back off so that spinning CTAs do not flood L2 with requests
            __nanosleep(it < 4 ? 32u : (it < 16 ? 128u : 256u));
        }
    }
    return true;
}

// Position of element k (0..63) of a quantization group in the fragment order: the
// bytes (or fp16 activations) a thread with threadID_in_group c needs for the four
// k16 blocks of the group are contiguous at [16c, 16c + 16).
__device__ __forceinline__ int frag_pos(int k) { return frag_pos_host(k); }

// Shared-memory carve-up (byte offsets), identical on host and device.
struct MkSmem {
    size_t xs, sx, rs, red, ared, cmb, lay, tbias, ctl, bar, total;
};
__host__ __device__ inline MkSmem mk_smem_layout(int nslot, int nb, int xsk, int d, int n_layers) {
    MkSmem L;
    size_t o = (size_t)nslot * MK_SLOT_BYTES;
    L.xs = o; o = (o + (size_t)nb * xsk * 2 + 15) & ~(size_t)15;
    L.sx = o; o = (o + (size_t)nb * (xsk / 64) * 4 + 15) & ~(size_t)15;
    L.rs = o; o = (o + (size_t)nb * d * 4 + 15) & ~(size_t)15;
    L.red = o; o = (o + (size_t)MK_CWARPS * 16 * nb * 4 + 15) & ~(size_t)15;
    L.ared = o; o = (o + (size_t)MK_CWARPS * MK_PART_WORDS * 4 + 64 + 15) & ~(size_t)15;
    L.cmb = o; o = (o + (size_t)MK_MAX_UNITS * MK_PART_WORDS * 4 + 15) & ~(size_t)15;
    L.lay = o; o = (o + (size_t)n_layers * sizeof(MkLayer) + 15) & ~(size_t)15;
    L.tbias = o; o = (o + 16 * 4 + 15) & ~(size_t)15;
    L.ctl = o; o = (o + 64 + 15) & ~(size_t)15;
    L.bar = o; o = (o + (size_t)2 * nslot * 8 + 16 + 15) & ~(size_t)15;
    L.total = o;
    return L;
}

struct StepShape {
    int lold[MK_MAX_NB];    // cached KV positions before this step (0 if inactive)
    int active[MK_MAX_NB];
    int kv_tiles[MK_MAX_NB];
    int units[MK_MAX_NB];   // attention units per head
    int slot[MK_MAX_NB];    // KV slot of each column
    int upt;                // KV tiles per attention unit
    int attn_units;         // total attention units of the step
};

__device__ __forceinline__ int lin_units(const MkLin &L) { return L.n_rb * L.n_kc; }
// Attention unit u (0 <= u < attn_units) of the step -> column n, head h, unit a of the
// head.  Units are numbered column-major over the active columns, then head, then unit.
__device__ __forceinline__ void attn_unit_of(const StepShape *S, int H, int u, int &n, int &h, int &a) {
    n = 0;
    for (int c = 0; c < MK_MAX_NB; ++c) {
        const int cnt = S->active[c] ? H * S->units[c] : 0;
        if (u < cnt) { n = c; break; }
        u -= cnt;
    }
    h = u / S->units[n];
    a = u - h * S->units[n];
}
__device__ __forceinline__ int first_owned(uint32_t ubase, int cta, int G) {
    return (int)((cta - (int)(ubase % (uint32_t)G) + G) % G);
}

// ------------------------------------------------------------------------------
// producer: streams the CTA's tiles (weights, then old K/V rows) in consumption order
// ------------------------------------------------------------------------------
struct MkProducer {
    const MkParams *pp;
    const StepShape *S;
    uint8_t *ring;
    uint64_t *full, *empty;
    const MkLayer *layers;  // shared-memory copy
    int nslot, cta, G;
    uint32_t seq, ubase;
    bool ok;
    uint64_t policy;
    uint32_t armed[16];  // seq + 1 of the last copy into each slot not known to have landed

    __device__ __forceinline__ void issue(const void *src0, uint32_t b0, const void *src1, uint32_t b1) {
        const uint32_t slot = seq % nslot, ph = (seq / nslot) & 1u;
        if (seq >= (uint32_t)nslot && ok) ok = mbar_wait_sleep(&empty[slot], ph ^ 1u, pp->err);
        if (!ok) { ++seq; return; }
        armed[slot] = seq + 1;  // the previous copy into this slot was consumed
        mbar_expect_tx(&full[slot], b0 + b1);
        uint8_t *dst = ring + (size_t)slot * MK_SLOT_BYTES;
        bulk_g2s(dst, src0, b0, &full[slot], policy);
        if (b1) bulk_g2s(dst + MK_SLOT_BYTES / 2, src1, b1, &full[slot], policy);
        ++seq;
    }
    __device__ __forceinline__ void stream_lin(const MkLin &L) {
        const int n = lin_units(L);
        for (int t = first_owned(ubase, cta, G); t < n; t += G)
            issue(L.tiles + (size_t)t * L.tile_bytes, (uint32_t)L.tile_bytes, nullptr, 0);
        ubase += n;
    }
    // dealt by row block: all K chunks of a block to one CTA
    __device__ __forceinline__ void stream_lin_rb(const MkLin &L) {
        for (int rb = first_owned(ubase, cta, G); rb < L.n_rb; rb += G)
            for (int kci = 0; kci < L.n_kc; ++kci)
                issue(L.tiles + ((size_t)rb * L.n_kc + kci) * L.tile_bytes, (uint32_t)L.tile_bytes, nullptr, 0);
        ubase += lin_units(L);
    }
    __device__ __forceinline__ void stream_attn(int l) {
        const MkParams &p = *pp;
        const int total = S->attn_units, upt = S->upt;
        for (int u = first_owned(ubase, cta, G); u < total; u += G) {
            int n, h, a;
            attn_unit_of(S, p.H, u, n, h, a);
            const int kvt = S->kv_tiles[n], lold = S->lold[n];
            const int t1 = min(kvt, (a + 1) * upt);
            for (int t = a * upt; t < t1; ++t) {
                const int p0 = t * MK_KVPOS, np = min(MK_KVPOS, lold - p0);
                const size_t off = kv_index(l, S->slot[n], h, p0, p.n_slots, p.H, p.max_seq);
                issue(p.kc + off, (uint32_t)np * 128u, p.vc + off, (uint32_t)np * 128u);
            }
        }
        ubase += total;
    }
    __device__ __forceinline__ void run() {
        const MkParams &p = *pp;
        for (int l = 0; l < p.n_layers && ok; ++l) {
            const MkLayer *Ly = layers + l;
            stream_lin(Ly->qkv);
            stream_attn(l);
            stream_lin(Ly->proj);
            stream_lin(Ly->fc);
            stream_lin_rb(Ly->mlp);
        }
        if (ok) stream_lin(p.head);
        // every copy issued must land before the CTA may exit
        for (int s = 0; s < nslot; ++s)
            if (armed[s]) mbar_wait(&full[s], ((armed[s] - 1) / nslot) & 1u, p.err);
    }
};

// ------------------------------------------------------------------------------
// One attention unit (column n, head h, unit a) on the 8 consumer warps: old positions
// from the ring, the new one from stage A's LL words; the last unit of a head merges its
// siblings' partials and writes the head's output.  Kept out of line so that its registers
// do not add to those live across the rest of the step.  Returns the ring sequence number
// after the unit's tiles; *ok is cleared on a wait timeout.
// ------------------------------------------------------------------------------
__device__ __forceinline__ uint32_t mk_attn_unit(const MkParams *pp, const StepShape *S, uint8_t *ring,
                                              uint64_t *full, uint64_t *empty, float *ared, float *cmb,
                                              int nslot, uint32_t seq, int *ok_io, int l, int n, int h,
                                              int a, uint32_t tag0, uint32_t tag1) {
    const MkParams &p = *pp;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, grp = lane >> 3, d8 = lane & 7;
    const int d = p.d;
    bool ok = *ok_io != 0;
    auto fail = [&](int code) {
        if (ok) atomicExch(p.err, code);
        ok = false;
    };
    const uint64_t *qrow = p.qkv_ll + ((size_t)l * MK_MAX_NB + n) * 3 * d + h * 64 + d8 * 8;
    const int units = S->units[n];
    const bool last = a == units - 1;
    const bool w0 = last && warp == 0;
    float qv[8];
    if (!ll_poll4<2>([&](int j) -> const uint64_t * { return qrow + j * 4; }, tag0,
                     [&](int j, float4 v) {
                         qv[4 * j] = v.x; qv[4 * j + 1] = v.y; qv[4 * j + 2] = v.z; qv[4 * j + 3] = v.w;
                     },
                     p.err))
        fail(12);
#pragma unroll
    for (int e = 0; e < 8; ++e) qv[e] *= kAttnScale;
    float m = -INFINITY, lsum = 0.f, acc[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) acc[e] = 0.f;
    const int upt = S->upt, t1 = min(S->kv_tiles[n], (a + 1) * upt), lold = S->lold[n];
    for (int t = a * upt; t < t1; ++t) {
        const uint32_t slot = seq % nslot, ph = (seq / nslot) & 1u;
        if (ok && !mbar_wait(&full[slot], ph, p.err)) fail(3);
        const __half *kt = reinterpret_cast<const __half *>(ring + (size_t)slot * MK_SLOT_BYTES);
        const __half *vt = reinterpret_cast<const __half *>(ring + (size_t)slot * MK_SLOT_BYTES + MK_SLOT_BYTES / 2);
        const int np = min(MK_KVPOS, lold - t * MK_KVPOS);
#pragma unroll
        for (int it = 0; it < MK_KVPOS / (4 * MK_CWARPS); ++it) {
            const int ppos = warp * (MK_KVPOS / MK_CWARPS) + it * 4 + grp;
            const bool in = ok && ppos < np;
            const int ppc = in ? ppos : 0;
            const uint4 kk = *reinterpret_cast<const uint4 *>(kt + (size_t)ppc * 64 + d8 * 8);
            const __half2 *k2 = reinterpret_cast<const __half2 *>(&kk);
            float s = 0.f;
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const float2 kf = __half22float2(k2[e]);
                s = fmaf(qv[2 * e], kf.x, s);
                s = fmaf(qv[2 * e + 1], kf.y, s);
            }
            s += __shfl_xor_sync(0xffffffffu, s, 1);
            s += __shfl_xor_sync(0xffffffffu, s, 2);
            s += __shfl_xor_sync(0xffffffffu, s, 4);
            if (in) {
                const uint4 vv = *reinterpret_cast<const uint4 *>(vt + (size_t)ppc * 64 + d8 * 8);
                const __half2 *v2 = reinterpret_cast<const __half2 *>(&vv);
                const float mn = fmaxf(m, s);
                const float corr = m == -INFINITY ? 0.f : expf(m - mn);
                const float pj = expf(s - mn);
                lsum = lsum * corr + pj;
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const float2 f = __half22float2(v2[e]);
                    acc[2 * e] = acc[2 * e] * corr + pj * f.x;
                    acc[2 * e + 1] = acc[2 * e + 1] * corr + pj * f.y;
                }
                m = mn;
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[slot]);
        ++seq;
    }
    if (w0) {  // the new position (fp32, from stage A)
        float kn[8], vn[8];
        if (!ll_poll4<4>([&](int j) -> const uint64_t * { return qrow + (j < 2 ? d : 2 * d) + (j & 1) * 4; },
                         tag0,
                         [&](int j, float4 v) {
                             float *dst = j < 2 ? kn : vn;
                             const int o = (j & 1) * 4;
                             dst[o] = v.x; dst[o + 1] = v.y; dst[o + 2] = v.z; dst[o + 3] = v.w;
                         },
                         p.err))
            fail(12);
        float s = 0.f;
#pragma unroll
        for (int e = 0; e < 8; ++e) s = fmaf(qv[e], kn[e], s);
        s += __shfl_xor_sync(0xffffffffu, s, 1);
        s += __shfl_xor_sync(0xffffffffu, s, 2);
        s += __shfl_xor_sync(0xffffffffu, s, 4);
        if (grp == 0) {
            const float mn = fmaxf(m, s);
            const float corr = m == -INFINITY ? 0.f : expf(m - mn);
            const float pj = expf(s - mn);
            lsum = lsum * corr + pj;
#pragma unroll
            for (int e = 0; e < 8; ++e) acc[e] = acc[e] * corr + pj * vn[e];
            m = mn;
        }
    }
    // merge the 4 position groups of each warp
#pragma unroll
    for (int off = 8; off <= 16; off <<= 1) {
        const float m2 = __shfl_xor_sync(0xffffffffu, m, off);
        const float l2 = __shfl_xor_sync(0xffffffffu, lsum, off);
        const float M = fmaxf(m, m2);
        const float fa = m == -INFINITY ? 0.f : expf(m - M);
        const float fb = m2 == -INFINITY ? 0.f : expf(m2 - M);
#pragma unroll
        for (int e = 0; e < 8; ++e) {
            const float a2 = __shfl_xor_sync(0xffffffffu, acc[e], off);
            acc[e] = acc[e] * fa + a2 * fb;
        }
        lsum = lsum * fa + l2 * fb;
        m = M;
    }
    if (grp == 0) {
        if (d8 == 0) { ared[warp * MK_PART_WORDS] = m; ared[warp * MK_PART_WORDS + 1] = lsum; }
#pragma unroll
        for (int e = 0; e < 8; ++e) ared[warp * MK_PART_WORDS + 4 + d8 * 8 + e] = acc[e];
    }
    const int nsib = last ? a : 0;
    uint64_t *part_base = p.attn_ll + ((((size_t)l * MK_MAX_NB + n) * p.H + h) * MK_MAX_UNITS) * MK_PART_WORDS;
    if (nsib > 0) {
        const int chunks = nsib * (MK_PART_WORDS / 4);
        constexpr int MAXC = (MK_MAX_UNITS * MK_PART_WORDS / 4 + MK_NTHR - 1) / MK_NTHR;
        if (!ll_poll4<MAXC>(
                [&](int j) -> const uint64_t * {
                    const int i = tid + j * MK_NTHR;
                    return i < chunks ? part_base + (size_t)i * 4 : nullptr;
                },
                tag1,
                [&](int j, float4 v) { *reinterpret_cast<float4 *>(cmb + (size_t)(tid + j * MK_NTHR) * 4) = v; },
                p.err))
            fail(13);
    }
    named_sync();
    if (tid < 64) {
        const int e = tid;
        float M = -INFINITY;
        for (int w = 0; w < MK_CWARPS; ++w) M = fmaxf(M, ared[w * MK_PART_WORDS]);
        for (int s2 = 0; s2 < nsib; ++s2) M = fmaxf(M, cmb[s2 * MK_PART_WORDS]);
        float L2 = 0.f, A2 = 0.f;
        for (int w = 0; w < MK_CWARPS; ++w) {
            const float mw = ared[w * MK_PART_WORDS];
            const float f = mw == -INFINITY ? 0.f : expf(mw - M);
            L2 += ared[w * MK_PART_WORDS + 1] * f;
            A2 += ared[w * MK_PART_WORDS + 4 + e] * f;
        }
        for (int s2 = 0; s2 < nsib; ++s2) {
            const float ms = cmb[s2 * MK_PART_WORDS];
            const float f = ms == -INFINITY ? 0.f : expf(ms - M);
            L2 += cmb[s2 * MK_PART_WORDS + 1] * f;
            A2 += cmb[s2 * MK_PART_WORDS + 4 + e] * f;
        }
        if (last) {
            ll_st(p.ao_ll + ((size_t)l * MK_MAX_NB + n) * d + h * 64 + e, A2 / L2, tag1);
        } else {
            uint64_t *dst = part_base + (size_t)a * MK_PART_WORDS;
            ll_st(dst + 4 + e, A2, tag1);
            if (e < 4) ll_st(dst + e, e == 0 ? M : (e == 1 ? L2 : 0.f), tag1);
        }
    }
    named_sync();
    *ok_io = ok ? 1 : 0;
    return seq;
}

// ------------------------------------------------------------------------------
// consumers: 8 warps
// ------------------------------------------------------------------------------
template <int NB>
struct MkConsumer {
    const MkParams *pp;
    const StepShape *S;
    uint8_t *ring;
    __half *xs;    // [NB][xsk] fp16, fragment order
    float *sx;     // [NB][xsk/64] group sums
    float *rs;     // [NB][d] residual / LN source
    float *red;    // [8 warps][16 rows][NB]
    float *ared;   // [8 warps][68] + stats
    float *cmb;    // [MK_MAX_UNITS][68]
    float *tbias;  // [16] bias of the rows of the tile being finished
    const MkLayer *layers;  // shared-memory copy
    uint64_t *full, *empty;
    int nslot, cta, G, tid, warp, lane, g, c, nb, d, xsk;
    uint32_t seq, ubase, tbase;
    bool ok;
    int ev;

    __device__ __forceinline__ uint32_t tag(int l, int st) const {
        return tbase + (uint32_t)(l * MK_STAGES + st) + 1u;
    }
    __device__ __forceinline__ void fail(int code) {
        if (ok) atomicExch(pp->err, code);
        ok = false;
    }
    __device__ __forceinline__ void trace() {
        if (pp->trace && tid == 0 && ev < MK_TRACE_EVENTS) pp->trace[(size_t)cta * MK_TRACE_EVENTS + ev] = globaltimer();
        ++ev;
    }
    __device__ __forceinline__ float *stat() const { return ared + MK_CWARPS * MK_PART_WORDS; }

    // rs[n][k] = LL vector base[n][k] (n < nb, k < d) once every word carries `tg`
    __device__ __forceinline__ void poll_rs(const uint64_t *base, uint32_t tg) {
        const int per = d / 4, total = nb * per;
        constexpr int MAXC = 2;
        const int t = tid, dd = d;
        float *r = rs;
        for (int r0 = 0; r0 < total; r0 += MAXC * MK_NTHR) {
            const bool okp = ll_poll4<MAXC>(
                [&](int j) -> const uint64_t * {
                    const int i = r0 + t + j * MK_NTHR;
                    if (i >= total) return nullptr;
                    const int n = i / per, k4 = i - n * per;
                    return base + (size_t)n * dd + k4 * 4;
                },
                tg,
                [&](int j, float4 v) {
                    const int i = r0 + t + j * MK_NTHR, n = i / per, k4 = i - n * per;
                    *reinterpret_cast<float4 *>(r + (size_t)n * dd + k4 * 4) = v;
                },
                pp->err);
            if (!okp) fail(10);
        }
        named_sync();
    }
    // Block-wide sum over the 256 consumer threads of one value per thread and column
    // (NB columns at once); every thread gets the totals.
    __device__ __forceinline__ void block_sum(float (&v)[NB]) {
        float *scratch = red;  // [8 warps][NB]
#pragma unroll
        for (int n = 0; n < NB; ++n) v[n] = warp_sum(v[n]);
        if (lane == 0)
#pragma unroll
            for (int n = 0; n < NB; ++n) scratch[warp * NB + n] = v[n];
        named_sync();
#pragma unroll
        for (int n = 0; n < NB; ++n) {
            float t = 0.f;
#pragma unroll
            for (int w = 0; w < MK_CWARPS; ++w) t += scratch[w * NB + n];
            v[n] = t;
        }
        named_sync();
    }
    // LayerNorm statistics of the rs columns (two passes, all consumer threads)
    __device__ __forceinline__ void ln_stats() {
        float *st = stat();
        const int d4 = d / 4;
        float sum[NB], var[NB];
#pragma unroll
        for (int n = 0; n < NB; ++n) {
            sum[n] = 0.f;
            if (n < nb)
                for (int k4 = tid; k4 < d4; k4 += MK_NTHR) {
                    const float4 x = *reinterpret_cast<const float4 *>(rs + (size_t)n * d + k4 * 4);
                    sum[n] += (x.x + x.y) + (x.z + x.w);
                }
        }
        block_sum(sum);
#pragma unroll
        for (int n = 0; n < NB; ++n) {
            var[n] = 0.f;
            const float mean = sum[n] / (float)d;
            if (n < nb)
                for (int k4 = tid; k4 < d4; k4 += MK_NTHR) {
                    const float4 x = *reinterpret_cast<const float4 *>(rs + (size_t)n * d + k4 * 4);
                    const float a = x.x - mean, b = x.y - mean, cc = x.z - mean, e = x.w - mean;
                    var[n] += (a * a + b * b) + (cc * cc + e * e);
                }
        }
        block_sum(var);
        if (tid < NB) {
            st[2 * tid] = sum[tid] / (float)d;
            st[2 * tid + 1] = 1.0f / sqrtf(var[tid] / (float)d + kNormEps);
        }
        named_sync();
    }
    // per-group sums of the fp16 activations just written to xs (K inputs): 8 threads per
    // group of 64, 16 bytes each, combined with shuffles
    __device__ __forceinline__ void group_sums(int K) {
        named_sync();
        const int G64 = K / 64, total = NB * G64 * 8;
        for (int i0 = 0; i0 < total; i0 += MK_NTHR) {
            const int i = i0 + tid;
            float s = 0.f;
            if (i < total) {
                const int grp = i >> 3, part = i & 7, n = grp / G64, j = grp - n * G64;
                const uint4 v = *reinterpret_cast<const uint4 *>(xs + (size_t)n * xsk + j * 64 + part * 8);
                const __half2 *h2 = reinterpret_cast<const __half2 *>(&v);
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const float2 f = __half22float2(h2[e]);
                    s += f.x + f.y;
                }
            }
            s += __shfl_xor_sync(0xffffffffu, s, 1);
            s += __shfl_xor_sync(0xffffffffu, s, 2);
            s += __shfl_xor_sync(0xffffffffu, s, 4);
            if (i < total && (i & 7) == 0) {
                const int grp = i >> 3, n = grp / G64, j = grp - n * G64;
                sx[n * (xsk / 64) + j] = s;
            }
        }
        named_sync();
    }
    __device__ __forceinline__ void put_x(int n, int k, float v) {
        xs[(size_t)n * xsk + (k & ~63) + frag_pos(k & 63)] = __float2half_rn(v);
    }
    // LayerNorm parameters of this thread's 4-wide chunks k4 = tid + j * 256 (d <= 2048),
    // loaded before the activations are polled so that the loads overlap the wait.
    static constexpr int LNC = (MK_MAX_D / 4 + MK_NTHR - 1) / MK_NTHR;
    struct LnRegs {
        float4 w[LNC], b[LNC];
    };
    __device__ __forceinline__ LnRegs ln_prefetch(const float *w, const float *b) const {
        LnRegs r;
#pragma unroll
        for (int j = 0; j < LNC; ++j) {
            const int k4 = tid + j * MK_NTHR;
            if (k4 * 4 < d) {
                r.w[j] = __ldg(reinterpret_cast<const float4 *>(w) + k4);
                r.b[j] = __ldg(reinterpret_cast<const float4 *>(b) + k4);
            } else {
                r.w[j] = r.b[j] = make_float4(0.f, 0.f, 0.f, 0.f);
            }
        }
        return r;
    }
    // xs = LayerNorm(rs) * w + b with the prefetched parameters
    __device__ __forceinline__ void xs_from_rs_ln(const LnRegs &P) {
        const float *st = stat();
#pragma unroll
        for (int j = 0; j < LNC; ++j) {
            const int k4 = tid + j * MK_NTHR;
            if (k4 * 4 >= d) continue;
            for (int n = 0; n < nb; ++n) {
                const float4 x = *reinterpret_cast<const float4 *>(rs + (size_t)n * d + k4 * 4);
                const float mean = st[2 * n], rstd = st[2 * n + 1];
                put_x(n, k4 * 4, (x.x - mean) * rstd * P.w[j].x + P.b[j].x);
                put_x(n, k4 * 4 + 1, (x.y - mean) * rstd * P.w[j].y + P.b[j].y);
                put_x(n, k4 * 4 + 2, (x.z - mean) * rstd * P.w[j].z + P.b[j].z);
                put_x(n, k4 * 4 + 3, (x.w - mean) * rstd * P.w[j].w + P.b[j].w);
            }
        }
        group_sums(d);
    }
    // rs = LayerNorm(rs) * w + b in place (prefetched parameters)
    __device__ __forceinline__ void rs_ln_inplace(const LnRegs &P) {
        const float *st = stat();
#pragma unroll
        for (int j = 0; j < LNC; ++j) {
            const int k4 = tid + j * MK_NTHR;
            if (k4 * 4 >= d) continue;
            for (int n = 0; n < nb; ++n) {
                float4 *xp = reinterpret_cast<float4 *>(rs + (size_t)n * d + k4 * 4);
                float4 x = *xp;
                const float mean = st[2 * n], rstd = st[2 * n + 1];
                x.x = (x.x - mean) * rstd * P.w[j].x + P.b[j].x;
                x.y = (x.y - mean) * rstd * P.w[j].y + P.b[j].y;
                x.z = (x.z - mean) * rstd * P.w[j].z + P.b[j].z;
                x.w = (x.w - mean) * rstd * P.w[j].w + P.b[j].w;
                *xp = x;
            }
        }
        named_sync();
    }
    // xs = LL vector base[n][k] (K inputs); with only_active, inactive columns (no
    // attention ran for them) get zeros instead
    __device__ __forceinline__ void xs_from_ll(const uint64_t *base, int K, uint32_t tg, bool only_active) {
        const int per = K / 4, total = nb * per;
        constexpr int MAXC = 3;
        if (only_active)
            for (int i = tid; i < nb * K; i += MK_NTHR) {
                const int n = i / K;
                if (!S->active[n]) put_x(n, i - n * K, 0.f);
            }
        for (int r0 = 0; r0 < total; r0 += MAXC * MK_NTHR) {
            const int t = tid;
            const bool okp = ll_poll4<MAXC>(
                [&](int j) -> const uint64_t * {
                    const int i = r0 + t + j * MK_NTHR;
                    if (i >= total) return nullptr;
                    const int n = i / per, k4 = i - n * per;
                    if (only_active && !S->active[n]) return nullptr;
                    return base + (size_t)n * K + k4 * 4;
                },
                tg,
                [&](int j, float4 v) {
                    const int i = r0 + t + j * MK_NTHR, n = i / per, k = (i - n * per) * 4;
                    put_x(n, k, v.x);
                    put_x(n, k + 1, v.y);
                    put_x(n, k + 2, v.z);
                    put_x(n, k + 3, v.w);
                },
                pp->err);
            if (!okp) fail(11);
        }
        group_sums(K);
    }

    // One GEMV tile (16 rows x KC) from the ring: the 8 warps split its groups and add
    // into acc (rows g, g+8 x columns 2c, 2c+1).
    __device__ __forceinline__ void group_mma(const uint8_t *tq, const uint8_t *tsb, int KC, int G64, int j,
                                              int gg, int n0, int n1, int xn, bool half_sb, float (&acc)[4]) {
        const int jj = j ^ (g & 1);
        const uint4 wa = *reinterpret_cast<const uint4 *>(tq + g * KC + jj * 64 + c * 16);
        const uint4 wb = *reinterpret_cast<const uint4 *>(tq + (g + 8) * KC + jj * 64 + c * 16);
        const __half *xg = xs + (size_t)xn * xsk + gg * 64 + c * 16;
        const uint4 x0 = *reinterpret_cast<const uint4 *>(xg);
        const uint4 x1 = *reinterpret_cast<const uint4 *>(xg + 8);
        float d0[4] = {0.f, 0.f, 0.f, 0.f}, d1[4] = {0.f, 0.f, 0.f, 0.f};
        // two independent accumulation chains (k16 blocks 0,2 and 1,3)
        mma16816(d0, __byte_perm(wa.x, 0x64646464u, 0x4140u), __byte_perm(wb.x, 0x64646464u, 0x4140u),
                 __byte_perm(wa.x, 0x64646464u, 0x4342u), __byte_perm(wb.x, 0x64646464u, 0x4342u), x0.x, x0.y);
        mma16816(d1, __byte_perm(wa.y, 0x64646464u, 0x4140u), __byte_perm(wb.y, 0x64646464u, 0x4140u),
                 __byte_perm(wa.y, 0x64646464u, 0x4342u), __byte_perm(wb.y, 0x64646464u, 0x4342u), x0.z, x0.w);
        mma16816(d0, __byte_perm(wa.z, 0x64646464u, 0x4140u), __byte_perm(wb.z, 0x64646464u, 0x4140u),
                 __byte_perm(wa.z, 0x64646464u, 0x4342u), __byte_perm(wb.z, 0x64646464u, 0x4342u), x1.x, x1.y);
        mma16816(d1, __byte_perm(wa.w, 0x64646464u, 0x4140u), __byte_perm(wb.w, 0x64646464u, 0x4140u),
                 __byte_perm(wa.w, 0x64646464u, 0x4342u), __byte_perm(wb.w, 0x64646464u, 0x4342u), x1.z, x1.w);
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
        const float sxa = sx[n0 * (xsk / 64) + gg], sxb = sx[n1 * (xsk / 64) + gg];
        const float o0 = fmaf(-1024.0f, s0, z0), o1 = fmaf(-1024.0f, s1, z1);
        acc[0] += fmaf(s0, d0[0] + d1[0], o0 * sxa);
        acc[1] += fmaf(s0, d0[1] + d1[1], o0 * sxb);
        acc[2] += fmaf(s1, d0[2] + d1[2], o1 * sxa);
        acc[3] += fmaf(s1, d0[3] + d1[3], o1 * sxb);
    }
    // One GEMV tile (16 rows x KC) from the ring: the 8 warps split its groups and add
    // into acc (rows g, g+8 x columns 2c, 2c+1); the rows' bias goes to tbias.
    __device__ __forceinline__ void tile_mma(const MkLin &L, int kci, float (&acc)[4]) {
        const uint32_t slot = seq % nslot, ph = (seq / nslot) & 1u;
        if (ok && !mbar_wait(&full[slot], ph, pp->err)) fail(2);
        const uint8_t *tq = ring + (size_t)slot * MK_SLOT_BYTES;
        const int KC = L.kc, G64 = KC / 64;
        const uint8_t *tsb = tq + 16 * KC;
        const int n0 = (2 * c) < NB ? 2 * c : 0, n1 = (2 * c + 1) < NB ? 2 * c + 1 : 0;
        const int xn = g < NB ? g : 0;
        const bool half_sb = pp->sbb == 4;
        if (ok) {
            int j = warp;
            for (; j + MK_CWARPS < G64; j += 2 * MK_CWARPS) {
                group_mma(tq, tsb, KC, G64, j, kci * G64 + j, n0, n1, xn, half_sb, acc);
                group_mma(tq, tsb, KC, G64, j + MK_CWARPS, kci * G64 + j + MK_CWARPS, n0, n1, xn, half_sb, acc);
            }
            if (j < G64) group_mma(tq, tsb, KC, G64, j, kci * G64 + j, n0, n1, xn, half_sb, acc);
            if (warp == 0 && lane < 16)
                tbias[lane] = *reinterpret_cast<const float *>(tq + mk_tile_bias_offset(KC, pp->sbb) + lane * 4);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[slot]);
        ++seq;
    }
    // Sums the 8 warp partials and runs epi(m, n, v) for rows m < 16, columns n < NB:
    // thread (m, n, w) reads warp w's value, 3 shuffles combine the 8 warps.
    template <class Epi>
    __device__ __forceinline__ void reduce_tile(const float (&acc)[4], Epi epi) {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int m = g + (i >> 1) * 8, n = 2 * c + (i & 1);
            if (n < NB) red[((m * NB) + n) * MK_CWARPS + warp] = acc[i];
        }
        named_sync();
        for (int i0 = 0; i0 < 16 * NB * MK_CWARPS; i0 += MK_NTHR) {
            const int i = i0 + tid;
            float v = i < 16 * NB * MK_CWARPS ? red[i] : 0.f;
            v += __shfl_xor_sync(0xffffffffu, v, 1);
            v += __shfl_xor_sync(0xffffffffu, v, 2);
            v += __shfl_xor_sync(0xffffffffu, v, 4);
            if (i < 16 * NB * MK_CWARPS && (i & 7) == 0) {
                const int mn = i >> 3, m = mn / NB, n = mn - m * NB;
                epi(m, n, v);
            }
        }
        named_sync();
    }
    // Units of linear L owned by this CTA, one tile each.
    template <class Epi>
    __device__ __forceinline__ void run_lin(const MkLin &L, Epi epi) {
        const int nu = lin_units(L);
        for (int t = first_owned(ubase, cta, G); t < nu; t += G) {
            const int rb = t / L.n_kc, kci = t - rb * L.n_kc;
            float acc[4] = {0.f, 0.f, 0.f, 0.f};
            tile_mma(L, kci, acc);
            const int out = L.out, nbl = nb;
            reduce_tile(acc, [&](int m, int n, float v) {
                const int o = rb * 16 + m;
                if (o < out && n < nbl) epi(o, n, v);
            });
        }
        ubase += nu;
    }
    // Row blocks of linear L owned by this CTA, all K chunks accumulated in registers.
    template <class Epi>
    __device__ __forceinline__ void run_lin_rb(const MkLin &L, Epi epi) {
        for (int rb = first_owned(ubase, cta, G); rb < L.n_rb; rb += G) {
            float acc[4] = {0.f, 0.f, 0.f, 0.f};
            for (int kci = 0; kci < L.n_kc; ++kci) tile_mma(L, kci, acc);
            const int out = L.out, nbl = nb;
            reduce_tile(acc, [&](int m, int n, float v) {
                const int o = rb * 16 + m;
                if (o < out && n < nbl) epi(o, n, v);
            });
        }
        ubase += lin_units(L);
    }

    // ---- per-CTA control block in shared memory (uniform state between stages) ----
    struct Ctl {
        uint32_t seq, ubase, tbase;
        int ok, ev;
    };
    __device__ __forceinline__ void init(const MkParams *p_, const StepShape *S_, uint8_t *smem, Ctl *ctl) {
        pp = p_;
        S = S_;
        const MkParams &p = *p_;
        nslot = p.nslot;
        const MkSmem SL = mk_smem_layout(nslot, NB, p.xsk, p.d, p.n_layers);
        ring = smem;
        xs = reinterpret_cast<__half *>(smem + SL.xs);
        sx = reinterpret_cast<float *>(smem + SL.sx);
        rs = reinterpret_cast<float *>(smem + SL.rs);
        red = reinterpret_cast<float *>(smem + SL.red);
        ared = reinterpret_cast<float *>(smem + SL.ared);
        cmb = reinterpret_cast<float *>(smem + SL.cmb);
        tbias = reinterpret_cast<float *>(smem + SL.tbias);
        layers = reinterpret_cast<const MkLayer *>(smem + SL.lay);
        full = reinterpret_cast<uint64_t *>(smem + SL.bar);
        empty = full + nslot;
        cta = blockIdx.x;
        G = gridDim.x;
        tid = threadIdx.x;
        warp = tid >> 5;
        lane = tid & 31;
        g = lane >> 2;
        c = lane & 3;
        nb = p.nb;
        d = p.d;
        xsk = p.xsk;
        seq = ctl->seq;
        ubase = ctl->ubase;
        tbase = ctl->tbase;
        ok = ctl->ok != 0;
        ev = ctl->ev;
    }
    __device__ __forceinline__ void save(Ctl *ctl) {
        named_sync();
        if (tid == 0) {
            ctl->seq = seq;
            ctl->ubase = ubase;
            ctl->ok = ok ? 1 : 0;
            ctl->ev = ev;
        }
        named_sync();
    }

    // ---- stage A: r_l -> LN1 -> QKV; K/V appended to the cache ----
    __device__ __forceinline__ void stage_a(int l) {
        const MkParams &p = *pp;
        const MkLayer *Ly = layers + l;
        const LnRegs ln1 = ln_prefetch(Ly->ln1_w, Ly->ln1_b);
        if (l == 0) {
            for (int i = tid; i < nb * d; i += MK_NTHR) {
                const int n = i / d, k = i - n * d;
                const SlotState &st = p.slots[S->slot[n]];
                const int tok = min(max(st.tok, 0), p.mel_vocab - 1);
                const int pos = min(max(st.pos, 0), p.mel_pos_len - 1);
                rs[i] = p.mel_emb[(size_t)tok * d + k] + p.mel_pos[(size_t)pos * d + k];
            }
            named_sync();
        } else {
            poll_rs(p.x_ll + (size_t)l * MK_MAX_NB * d, tag(l - 1, 4));
        }
        trace();
        ln_stats();
        xs_from_rs_ln(ln1);
        uint64_t *qkv_l = p.qkv_ll + (size_t)l * MK_MAX_NB * 3 * d;
        const MkLin Lq = Ly->qkv;
        const uint32_t tg = tag(l, 0);
        const int dd = d;
        run_lin(Lq, [&](int o, int n, float v) {
            v += tbias[o & 15];
            ll_st(qkv_l + (size_t)n * 3 * dd + o, v, tg);
            if (o >= dd && S->active[n]) {
                const int rr = o - dd, which = rr / dd, oo = rr - which * dd;
                __half *cache = which == 0 ? p.kc : p.vc;
                cache[kv_index(l, S->slot[n], oo >> 6, S->lold[n], p.n_slots, p.H, p.max_seq) + (oo & 63)] =
                    __float2half_rn(v);
            }
        });
        trace();
    }
    // ---- stage B: attention units of this CTA ----
    __device__ __forceinline__ void stage_b(int l) {
        const MkParams &p = *pp;
        const uint32_t t0 = tag(l, 0), t1 = tag(l, 1);
        const int total = S->attn_units;
        for (int u = first_owned(ubase, cta, G); u < total; u += G) {
            int n, h, a;
            attn_unit_of(S, p.H, u, n, h, a);
            int okf = ok ? 1 : 0;
            seq = mk_attn_unit(pp, S, ring, full, empty, ared, cmb, nslot, seq, &okf, l, n, h, a, t0, t1);
            ok = okf != 0;
        }
        ubase += total;
        trace();
    }
    // ---- stage C: attention output -> c_proj + residual -> h ----
    __device__ __forceinline__ void stage_c(int l) {
        const MkParams &p = *pp;
        xs_from_ll(p.ao_ll + (size_t)l * MK_MAX_NB * d, d, tag(l, 1), true);
        uint64_t *h_l = p.h_ll + (size_t)l * MK_MAX_NB * d;
        const MkLin Lp = layers[l].proj;
        const uint32_t tg = tag(l, 2);
        const int dd = d;
        run_lin(Lp, [&](int o, int n, float v) {
            ll_st(h_l + (size_t)n * dd + o, rs[(size_t)n * dd + o] + v + tbias[o & 15], tg);
        });
        trace();
    }
    // ---- stage D: LN2 + c_fc + GELU -> u ----
    __device__ __forceinline__ void stage_d(int l) {
        const MkParams &p = *pp;
        const MkLayer *Ly = layers + l;
        const LnRegs ln2 = ln_prefetch(Ly->ln2_w, Ly->ln2_b);
        poll_rs(p.h_ll + (size_t)l * MK_MAX_NB * d, tag(l, 2));
        ln_stats();
        xs_from_rs_ln(ln2);
        uint64_t *u_l = p.u_ll + (size_t)l * MK_MAX_NB * p.ff;
        const MkLin Lf = Ly->fc;
        const uint32_t tg = tag(l, 3);
        const int ff = p.ff;
        run_lin(Lf, [&](int o, int n, float v) {
            ll_st(u_l + (size_t)n * ff + o, gelu_tanh(v + tbias[o & 15]), tg);
        });
        trace();
    }
    // ---- stage E: mlp c_proj + residual -> x_{l+1} (rs still holds h) ----
    __device__ __forceinline__ void stage_e(int l) {
        const MkParams &p = *pp;
        xs_from_ll(p.u_ll + (size_t)l * MK_MAX_NB * p.ff, p.ff, tag(l, 3), false);
        uint64_t *x_next = p.x_ll + (size_t)(l + 1) * MK_MAX_NB * d;
        const MkLin Lm = layers[l].mlp;
        const uint32_t tg = tag(l, 4);
        const int dd = d;
        run_lin_rb(Lm, [&](int o, int n, float v) {
            ll_st(x_next + (size_t)n * dd + o, rs[(size_t)n * dd + o] + v + tbias[o & 15], tg);
        });
        trace();
    }
    // ---- head: ln_f -> final_norm -> mel_head ----
    __device__ __forceinline__ void stage_head() {
        const MkParams &p = *pp;
        const int L = p.n_layers;
        const LnRegs lnf = ln_prefetch(p.lnf_w, p.lnf_b);
        const LnRegs fin = ln_prefetch(p.fin_w, p.fin_b);
        poll_rs(p.x_ll + (size_t)L * MK_MAX_NB * d, tag(L - 1, 4));
        ln_stats();
        rs_ln_inplace(lnf);
        ln_stats();
        xs_from_rs_ln(fin);
        const MkLin Lh = p.head;
        float *logits = p.logits;
        const int V = p.mel_vocab;
        run_lin(Lh, [&](int o, int n, float v) { logits[(size_t)n * V + o] = v + tbias[o & 15]; });
        trace();
    }
};

// Each consumer stage is compiled as its own function: its registers are not shared with
// state that lives across the rest of the step (which is kept in the shared-memory Ctl).
template <int NB, int STAGE>
__device__ __forceinline__ void mk_stage(const MkParams *pp, const StepShape *S, uint8_t *smem, int l) {
    using Ctl = typename MkConsumer<NB>::Ctl;
    const MkSmem SL = mk_smem_layout(pp->nslot, NB, pp->xsk, pp->d, pp->n_layers);
    Ctl *ctl = reinterpret_cast<Ctl *>(smem + SL.ctl);
    MkConsumer<NB> C;
    C.init(pp, S, smem, ctl);
    if (STAGE == 0) C.stage_a(l);
    else if (STAGE == 1) C.stage_b(l);
    else if (STAGE == 2) C.stage_c(l);
    else if (STAGE == 3) C.stage_d(l);
    else if (STAGE == 4) C.stage_e(l);
    else C.stage_head();
    C.save(ctl);
}

// ------------------------------------------------------------------------------
// kernel
// ------------------------------------------------------------------------------
template <int NB>
__global__ void __launch_bounds__(MK_THREADS, 1) mk_decode_kernel(const __grid_constant__ MkParams p) {
    extern __shared__ __align__(1024) uint8_t smem[];
    __shared__ StepShape S;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int G = gridDim.x, cta = blockIdx.x;
    const int nslot = p.nslot;
    const MkSmem SL = mk_smem_layout(nslot, NB, p.xsk, p.d, p.n_layers);
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + SL.bar);
    uint64_t *empty = full + nslot;
    const uint32_t epoch = p.epoch[cta];

    MkLayer *lay = reinterpret_cast<MkLayer *>(smem + SL.lay);
    {
        const int words = (int)(p.n_layers * sizeof(MkLayer) / 4);
        const uint32_t *src = reinterpret_cast<const uint32_t *>(p.layers);
        uint32_t *dst = reinterpret_cast<uint32_t *>(lay);
        for (int i = tid; i < words; i += MK_THREADS) dst[i] = src[i];
    }
    if (tid == 0) {
        // step shape (identical in every CTA)
        int total = 0, max_tiles = 0;
        for (int n = 0; n < MK_MAX_NB; ++n) {
            S.active[n] = 0; S.lold[n] = 0; S.kv_tiles[n] = 0; S.units[n] = 0; S.slot[n] = 0;
            if (n < p.nb) {
                S.slot[n] = p.batch_slot[n];
                const SlotState &st = p.slots[S.slot[n]];
                S.active[n] = st.active && st.valid_len < p.max_seq;
                S.lold[n] = S.active[n] ? st.valid_len : 0;
                S.kv_tiles[n] = (S.lold[n] + MK_KVPOS - 1) / MK_KVPOS;
                if (S.active[n]) total += p.H * S.kv_tiles[n];
                max_tiles = max(max_tiles, S.kv_tiles[n]);
            }
        }
        S.upt = max(max(1, (total + G - 1) / G), (max_tiles + MK_MAX_UNITS - 1) / MK_MAX_UNITS);
        S.attn_units = 0;
        for (int n = 0; n < MK_MAX_NB; ++n)
            if (S.active[n]) {
                S.units[n] = max(1, (S.kv_tiles[n] + S.upt - 1) / S.upt);
                S.attn_units += p.H * S.units[n];
            }
        for (int s = 0; s < nslot; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], MK_CWARPS);
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        if (p.trace) p.trace[(size_t)cta * MK_TRACE_EVENTS] = globaltimer();
    }
    __syncthreads();
    // No column left generating (each stopped, sampler.rs:378, or failed): the step does
    // nothing.  S is the same in every CTA, so the whole grid leaves before any copy,
    // exchange or write; the launch counter stays, so no LL tag repeats.
    {
        int any = 0;
        for (int n = 0; n < MK_MAX_NB; ++n) any |= S.active[n];
        if (!any) return;
    }

    if (warp == MK_CWARPS) {
        if (lane != 0) return;
        MkProducer P;
        P.pp = &p; P.S = &S; P.ring = smem; P.full = full; P.empty = empty; P.layers = lay;
        P.policy = evict_first_policy();
        P.nslot = nslot; P.cta = cta; P.G = G; P.seq = 0; P.ubase = 0; P.ok = true;
#pragma unroll
        for (int s = 0; s < 16; ++s) P.armed[s] = 0;
        P.run();
        return;
    }
    {
        using Ctl = typename MkConsumer<NB>::Ctl;
        Ctl *ctl = reinterpret_cast<Ctl *>(smem + SL.ctl);
        if (tid == 0) {
            ctl->seq = 0;
            ctl->ubase = 0;
            ctl->tbase = epoch * (uint32_t)(MK_STAGES * p.n_layers);
            ctl->ok = 1;
            ctl->ev = 1;
        }
        named_sync();
    }
    for (int l = 0; l < p.n_layers; ++l) {
        mk_stage<NB, 0>(&p, &S, smem, l);
        mk_stage<NB, 1>(&p, &S, smem, l);
        mk_stage<NB, 2>(&p, &S, smem, l);
        mk_stage<NB, 3>(&p, &S, smem, l);
        mk_stage<NB, 4>(&p, &S, smem, l);
    }
    mk_stage<NB, 5>(&p, &S, smem, 0);
    named_sync();
    if (tid == 0) p.epoch[cta] = epoch + 1;
}

// ------------------------------------------------------------------------------
// host side
// ------------------------------------------------------------------------------
template <int NB>
static cudaError_t mk_launch_t(const MkParams &p, cudaStream_t st) {
    const size_t smem = mk_smem_layout(p.nslot, NB, p.xsk, p.d, p.n_layers).total;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(p.grid);
    cfg.blockDim = dim3(MK_THREADS);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, mk_decode_kernel<NB>, p);
}

cudaError_t mk_launch(const MkParams &p, cudaStream_t st) {
    if (p.nb <= 1) return mk_launch_t<1>(p, st);
    if (p.nb <= 2) return mk_launch_t<2>(p, st);
    return mk_launch_t<4>(p, st);
}

static void mk_debug(const char *what, int nb, long v) {
    if (getenv("ITTS_DEBUG")) fprintf(stderr, "[itts] persistent kernel nb=%d: %s (%ld)\n", nb, what, v);
}

template <int NB>
static int mk_config_t(int xsk, int d, int n_layers, int *nslot_out) {
    int dev = 0, optin = 0, sms = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (d > MK_MAX_D) { mk_debug("model dim too large", NB, d); return -1; }
    cudaFuncAttributes fa;
    cudaError_t e = cudaFuncGetAttributes(&fa, mk_decode_kernel<NB>);
    if (e != cudaSuccess) { mk_debug(cudaGetErrorString(e), NB, 0); cudaGetLastError(); return -1; }
    const size_t budget = (size_t)optin - fa.sharedSizeBytes;  // static shared memory counts too
    int nslot = 16;
    while (nslot >= 2 && mk_smem_layout(nslot, NB, xsk, d, n_layers).total > budget) --nslot;
    if (nslot < 2) { mk_debug("shared memory", NB, (long)budget); return -1; }
    const size_t smem = mk_smem_layout(nslot, NB, xsk, d, n_layers).total;
    e = cudaFuncSetAttribute(mk_decode_kernel<NB>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) { mk_debug(cudaGetErrorString(e), NB, (long)smem); cudaGetLastError(); return -1; }
    int occ = 0;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, mk_decode_kernel<NB>, MK_THREADS, smem);
    if (e != cudaSuccess || occ < 1) {
        mk_debug(e != cudaSuccess ? cudaGetErrorString(e) : "occupancy 0", NB, fa.numRegs);
        if (getenv("ITTS_DEBUG")) {
            fprintf(stderr, "[itts]   static smem %zu, local %zu, max threads %d, dyn smem %zu, optin %d\n",
                    fa.sharedSizeBytes, fa.localSizeBytes, fa.maxThreadsPerBlock, smem, optin);
            for (int t : {32, 64, 128, 256, 288}) {
                int o = -1;
                cudaOccupancyMaxActiveBlocksPerMultiprocessor(&o, mk_decode_kernel<NB>, t, smem);
                int o2 = -1;
                cudaOccupancyMaxActiveBlocksPerMultiprocessor(&o2, mk_decode_kernel<NB>, t, 1024);
                fprintf(stderr, "[itts]   threads %d: occupancy %d (with 1 KB dyn smem: %d)\n", t, o, o2);
            }
        }
        cudaGetLastError();
        return -1;
    }
    *nslot_out = nslot;
    return sms;
}

// Returns the grid size (SM count) and the ring depth for nb columns, or -1.
int mk_config(int nb, int xsk, int d, int n_layers, int *nslot) {
    if (nb <= 1) return mk_config_t<1>(xsk, d, n_layers, nslot);
    if (nb <= 2) return mk_config_t<2>(xsk, d, n_layers, nslot);
    return mk_config_t<4>(xsk, d, n_layers, nslot);
}

}  // namespace itts
