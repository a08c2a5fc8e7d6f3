// ck_decode.cu -- the decode step of one request (batch column) on ONE 16-CTA
// thread-block cluster (crates/core/src/models/gpt.rs:706-754): step embedding,
// n_layers x [LN1 -> QKV -> KV append -> attention -> c_proj + residual -> LN2 -> c_fc +
// GELU -> mlp c_proj + residual], ln_f -> final_norm -> mel_head.
//
// Why a cluster: a batch-1 step is a chain of ~5 dependent stages per layer.  Across the
// whole GPU every stage boundary costs a cross-SM round trip through L2 (0.5-1 us, plus the
// polling and the spread of 148 CTAs); inside a cluster the stage outputs are pushed into
// every CTA's shared memory with st.async, and the receiver's mbarrier counts the bytes,
// so a stage boundary costs one distributed-shared-memory write and an mbarrier wait.
// Sixteen SMs stream the weights at ~160 GB/s each when their copy loop is lean.
//
// Per CTA: 8 consumer warps + 1 producer warp.
//  * The producer lane streams this CTA's share of the step's weight tiles (the tiled
//    int8 layout of mk.h: 16 rows x KC inputs with their (scale, offset) pairs) and old
//    K/V rows into an 8-slot shared-memory ring with cp.async.bulk (no multicast).  Row
//    block rb of every linear belongs to CTA rb % 16, with all its K chunks; the K/V tiles
//    (head, 84 positions) are split into 16 contiguous ranges in head-major order.
//  * Consumers take every tile cooperatively: quantization group j of tile t goes to warp
//    (t * G64 + j) % 8, which dequantizes it in registers (the byte in the mantissa of
//    1024.0 gives 1024 + q exactly; y += s * D + (b - 1024 s) * sum(x)) and runs mma.sync
//    m16n8k16 against the activation.  Per-warp partial sums wait in shared memory until
//    the stage's last tile, so no tile holds its ring slot for a cross-warp reduction.
//  * Stage outputs are pushed with st.async to the CTAs that read them (QKV rows only to
//    the CTAs whose attention range covers the head; everything else to all 16).  Every
//    stage input has its own mbarrier with the byte count the CTA expects per layer.
//    Buffers are reused every layer without double buffering: each CTA starts a layer
//    only after it received the previous layer's output rows from ALL CTAs, which those
//    sent after they had finished reading every buffer of the previous layer.
//  * Every wait is bounded; on a timeout the kernel records an error code in p.err (read
//    by the host as ITTS_E_TIMEOUT), skips the remaining waits and exits cleanly.
#include <algorithm>
#include <cstdio>
#include <cstdlib>

#include "kernels.h"
#include "mk.h"

namespace itts {
namespace {

constexpr int CS = 16;             // CTAs per cluster
constexpr int CW = 8;              // consumer warps
constexpr int CT = CW * 32;        // consumer threads
constexpr int NT = CT + 32;        // + the producer warp
constexpr int NSLOT = 8;           // ring slots (power of two)
constexpr int SLOT = 21888;        // bytes per slot: a 16 x 1280 tile with fp16 pairs, or 84 K/V rows
constexpr int KVPOS = 84;          // positions per K/V tile: 2 x 84 x 128 B = 21,504 B
constexpr int MAXHC = 4;           // heads one CTA's attention range may touch (H <= 32)
constexpr int REC = 68;            // floats per attention record: m, l, 0, 0, acc[64]
constexpr uint32_t SPIN = 1u << 22;
constexpr float kLog2e = 1.4426950408889634f;

enum { BX = 0, BQKV, BP, BH, BU, NSTB };

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
__device__ __forceinline__ bool mb_try(uint32_t a, uint32_t par) {
    uint32_t done;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(done)
        : "r"(a), "r"(par)
        : "memory");
    return done != 0;
}
// acquire at cluster scope: the bytes were written by other CTAs' st.async
__device__ __forceinline__ bool mb_try_cluster(uint32_t a, uint32_t par) {
    uint32_t done;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n"
        " selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(done)
        : "r"(a), "r"(par)
        : "memory");
    return done != 0;
}
template <bool CLUSTER>
__device__ __forceinline__ bool mb_wait(uint64_t *b, uint32_t par, const int *err) {
    const uint32_t a = su32(b);
    for (uint32_t it = 0; it < SPIN; ++it) {
        if (CLUSTER ? mb_try_cluster(a, par) : mb_try(a, par)) return true;
        if ((it & 4095u) == 4095u && *(volatile const int *)err) return false;
    }
    return false;
}
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void *src, uint32_t bytes, uint32_t bar, uint64_t pol) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(dst),
        "l"(src), "r"(bytes), "r"(bar), "l"(pol)
        : "memory");
}
__device__ __forceinline__ uint32_t mapa(uint32_t a, int rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(rank));
    return r;
}
__device__ __forceinline__ void st_async_v4(uint32_t raddr, float4 v, uint32_t rbar) {
    asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.v4.f32 [%0], {%1, %2, %3, %4}, [%5];" ::"r"(raddr),
                 "f"(v.x), "f"(v.y), "f"(v.z), "f"(v.w), "r"(rbar)
                 : "memory");
}
__device__ __forceinline__ void st_async_v2(uint32_t raddr, uint2 v, uint32_t rbar) {
    asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.v2.b32 [%0], {%1, %2}, [%3];" ::"r"(raddr),
                 "r"(v.x), "r"(v.y), "r"(rbar)
                 : "memory");
}
__device__ __forceinline__ void cluster_sync_all() {
    asm volatile("barrier.cluster.arrive.release.aligned;\nbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ void csync() { asm volatile("bar.sync 1, %0;" ::"n"(CT) : "memory"); }
// consumer-wide barrier that also ANDs one predicate over the consumer threads
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
struct CkSmem {
    uint32_t res, qkv, part, xsa, xsu, sx, red, ostg, stat, tab, bar, total;
};
__host__ __device__ inline uint32_t ck_red_bytes(int rt) {
    const uint32_t lin = (uint32_t)rt * CW * 16 * 4;
    const uint32_t att = (uint32_t)(MAXHC * CW * REC + MAXHC * REC) * 4;
    return lin > att ? lin : att;
}
__host__ __device__ inline CkSmem ck_layout(int d, int ff, int H, int rt) {
    CkSmem L;
    uint32_t o = NSLOT * SLOT;
    auto take = [&](uint32_t bytes) {
        const uint32_t at = o;
        o = (o + bytes + 127u) & ~127u;
        return at;
    };
    L.res = take(d * 4);
    L.qkv = take(MAXHC * 3 * 64 * 4);
    L.part = take((H + CS - 1) * REC * 4);
    L.xsa = take(d * 2);
    L.xsu = take(ff * 2);
    L.sx = take((ff > d ? ff : d) / 64 * 4);
    L.red = take(ck_red_bytes(rt));
    L.ostg = take(rt * 16 * 4);
    L.stat = take(64 * 4);
    L.tab = take(4 * (4 * CS + 3 * 33 + 16));
    L.bar = take((2 * NSLOT + NSTB) * 8);
    L.total = o;
    return L;
}

// Step shape, identical in every CTA of the cluster (computed by each CTA's thread 0).
struct CkTab {
    int hlo[CS], nh[CS], seg0[CS], u0[CS];  // attention range of every CTA: heads, segments
    int hs0[33];                            // first segment of head h (hs0[H] = total)
    int rlo[33], rhi[33];                   // CTAs whose range covers head h
    int active, lold, kvt, units, nseg, slot, tok, pos, u_lo, u_hi, pad[6];
};

static_assert(sizeof(CkTab) == 4 * (4 * CS + 3 * 33 + 16), "step table layout");

struct CkParams {
    MkParams p;
    int rt;  // tiles of the largest linear stage per CTA (partial-sum buffer size)
};

// ---------------------------------------------------------------------------
// producer (one lane): the CTA's tiles in consumption order
// ---------------------------------------------------------------------------
struct CkProducer {
    uint8_t *smem;
    uint32_t ring, full, empty;  // shared addresses
    uint64_t *fullp, *emptyp;
    const int *err;
    uint64_t pol;
    uint32_t seq;
    int rank;
    bool ok;

    __device__ __forceinline__ void issue(const void *s0, uint32_t b0, const void *s1, uint32_t b1) {
        const uint32_t slot = seq & (NSLOT - 1);
        if (seq >= (uint32_t)NSLOT && ok) {
            ok = mb_wait<false>(emptyp + slot, ((seq / NSLOT) & 1u) ^ 1u, err);
            if (!ok) atomicExch(const_cast<int *>(err), 1);
        }
        ++seq;
        if (!ok) return;
        const uint32_t bar = full + slot * 8;
        mb_expect(fullp + slot, b0 + b1);
        const uint32_t dst = ring + slot * SLOT;
        bulk_g2s(dst, s0, b0, bar, pol);
        if (b1) bulk_g2s(dst + b0, s1, b1, bar, pol);
    }
    // (arguments by value: the loops must not reload them around the asm statements)
    __device__ __forceinline__ void lin(const uint8_t *tiles, int n_rb, int n_kc, uint32_t tb) {
        const size_t row_bytes = (size_t)n_kc * tb;
        const uint8_t *row = tiles + (size_t)rank * row_bytes;
        for (int rb = rank; rb < n_rb; rb += CS, row += CS * row_bytes)
            for (int k = 0; k < n_kc; ++k) issue(row + (size_t)k * tb, tb, nullptr, 0);
    }
    __device__ __forceinline__ void lin(const MkLin *L) {
        lin(L->tiles, L->n_rb, L->n_kc, (uint32_t)L->tile_bytes);
    }
    __device__ __forceinline__ void attn(const __half *kc, const __half *vc, size_t base, size_t head_stride, int u_lo,
                                         int u_hi, int kvt, int lold) {
        int h = u_lo / kvt, t = u_lo - h * kvt;
        base += (size_t)h * head_stride;
        for (int u = u_lo; u < u_hi; ++u) {
            const int np = min(KVPOS, lold - t * KVPOS);
            if (np > 0) {
                const size_t off = base + (size_t)t * KVPOS * kHeadDim;
                issue(kc + off, (uint32_t)np * 128u, vc + off, (uint32_t)np * 128u);
            }
            if (++t == kvt) { t = 0; base += head_stride; }
        }
    }
    __device__ __forceinline__ void run(const MkParams &p, const CkTab &T) {
        const int u_lo = T.u_lo, u_hi = T.u_hi, kvt = T.kvt, lold = T.lold, slot = T.slot;
        const size_t head_stride = (size_t)p.max_seq * kHeadDim;
        for (int l = 0; l < p.n_layers && ok; ++l) {
            const MkLayer *Ly = p.layers + l;
            lin(&Ly->qkv);
            if (u_hi > u_lo)
                attn(p.kc, p.vc, kv_index(l, slot, 0, 0, p.n_slots, p.H, p.max_seq), head_stride, u_lo, u_hi, kvt, lold);
            lin(&Ly->proj);
            lin(&Ly->fc);
            lin(&Ly->mlp);
        }
        if (ok) lin(&p.head);
        // every copy issued must land before the CTA may exit
        for (uint32_t s = 0; s < NSLOT && s < seq; ++s) {
            const uint32_t last = ((seq - 1 - s) / NSLOT) * NSLOT + s;  // last sequence number in slot s
            mb_wait<false>(fullp + s, (last / NSLOT) & 1u, err);
        }
    }
};

// ---------------------------------------------------------------------------
// consumers (8 warps)
// ---------------------------------------------------------------------------
struct CkConsumer {
    const MkParams *pp;
    CkTab *T;
    uint8_t *smem;
    float *res, *qkv, *part, *sx, *red, *ostg, *stat;
    __half *xsa, *xsu;
    uint64_t *fullp, *emptyp, *stb;
    uint32_t ring_a;
    int tid, warp, lane, g, c, rank, d, ff, H, rt;
    uint32_t seq;
    uint32_t ph[NSTB];  // phases waited so far per stage barrier
    uint32_t exp_bytes[NSTB];
    bool ok;
    int ev;  // next trace event (stage timestamps, only when p.trace is set)

    __device__ __forceinline__ void trace() {
        if (pp->trace && tid == 0 && ev < MK_TRACE_EVENTS) {
            unsigned long long t;
            asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
            pp->trace[(size_t)rank * MK_TRACE_EVENTS + ev] = t;
        }
        ++ev;
    }

    __device__ __forceinline__ void fail(int code) {
        if (ok) atomicExch(pp->err, code);
        ok = false;
    }
    // wait for this layer's bytes on stage barrier b, then re-arm it for the next layer
    __device__ __forceinline__ void wait_stage(int b, int code) {
        bool good = !ok || mb_wait<true>(stb + b, ph[b] & 1u, pp->err);
        ++ph[b];
        good = csync_and(good);  // the same verdict in every consumer thread
        if (!good) fail(code);
        if (tid == 0) mb_expect(stb + b, exp_bytes[b]);
        trace();
    }
    // wait for ring slot `seq`; the verdict is made warp-uniform so that the warp-wide
    // mma.sync and shuffles that follow always run converged
    __device__ __forceinline__ void wait_slot(uint32_t slot, int code) {
        bool good = !ok || mb_wait<false>(fullp + slot, (seq / NSLOT) & 1u, pp->err);
        good = __all_sync(0xffffffffu, good);
        if (!good) fail(code);
    }
    __device__ __forceinline__ void put_x(__half *xs, int k, float v) {
        xs[(k & ~63) + frag_pos_host(k & 63)] = __float2half_rn(v);
    }
    __device__ __forceinline__ float block_sum(float v) {
        v = warp_sum(v);
        if (lane == 0) stat[warp] = v;
        csync();
        float t = 0.f;
#pragma unroll
        for (int w = 0; w < CW; ++w) t += stat[w];
        csync();
        return t;
    }
    // sx[j] = sum of the fp16 inputs of group j (K inputs), 8 threads per group
    __device__ __forceinline__ void group_sums(const __half *xs, int K) {
        csync();
        const int total = K / 64 * 8;
        for (int i0 = 0; i0 < total; i0 += CT) {
            const int i = i0 + tid;
            float s = 0.f;
            if (i < total) {
                const uint4 v = *reinterpret_cast<const uint4 *>(xs + (i >> 3) * 64 + (i & 7) * 8);
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
            if (i < total && (i & 7) == 0) sx[i >> 3] = s;
        }
        csync();
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
    // y = LayerNorm(res) * w + b, two-pass statistics; to xsa (fp16, fragment order) or
    // back into res (inplace)
    __device__ __forceinline__ void layernorm(const LnRegs &P, bool inplace) {
        float4 x[LNC];
        float s = 0.f;
#pragma unroll
        for (int j = 0; j < LNC; ++j) {
            const int k4 = tid + j * CT;
            x[j] = k4 * 4 < d ? *reinterpret_cast<const float4 *>(res + k4 * 4) : make_float4(0.f, 0.f, 0.f, 0.f);
            s += (x[j].x + x[j].y) + (x[j].z + x[j].w);
        }
        const float mean = block_sum(s) / (float)d;
        float v = 0.f;
#pragma unroll
        for (int j = 0; j < LNC; ++j) {
            const int k4 = tid + j * CT;
            if (k4 * 4 < d) {
                const float a = x[j].x - mean, b = x[j].y - mean, cc = x[j].z - mean, e = x[j].w - mean;
                v += (a * a + b * b) + (cc * cc + e * e);
            }
        }
        const float rstd = 1.0f / sqrtf(block_sum(v) / (float)d + kNormEps);
#pragma unroll
        for (int j = 0; j < LNC; ++j) {
            const int k4 = tid + j * CT;
            if (k4 * 4 >= d) continue;
            float4 y;
            y.x = (x[j].x - mean) * rstd * P.w[j].x + P.b[j].x;
            y.y = (x[j].y - mean) * rstd * P.w[j].y + P.b[j].y;
            y.z = (x[j].z - mean) * rstd * P.w[j].z + P.b[j].z;
            y.w = (x[j].w - mean) * rstd * P.w[j].w + P.b[j].w;
            if (inplace) {
                *reinterpret_cast<float4 *>(res + k4 * 4) = y;
            } else {
                put_x(xsa, k4 * 4, y.x);
                put_x(xsa, k4 * 4 + 1, y.y);
                put_x(xsa, k4 * 4 + 2, y.z);
                put_x(xsa, k4 * 4 + 3, y.w);
            }
        }
        if (inplace) csync();
        else group_sums(xsa, d);
    }

    // one quantization group of a tile: rows g, g + 8 of the tile, input column 0
    __device__ __forceinline__ void group(const uint8_t *tq, const uint8_t *tsb, int KC, int G64, int j, int gg,
                                          const __half *xs, bool half_sb, float &a0, float &a1) {
        const int jj = j ^ (g & 1);
        const uint4 wa = *reinterpret_cast<const uint4 *>(tq + g * KC + jj * 64 + c * 16);
        const uint4 wb = *reinterpret_cast<const uint4 *>(tq + (g + 8) * KC + jj * 64 + c * 16);
        const uint4 x0 = *reinterpret_cast<const uint4 *>(xs + gg * 64 + c * 16);
        const uint4 x1 = *reinterpret_cast<const uint4 *>(xs + gg * 64 + c * 16 + 8);
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
        const float sxg = sx[gg];
        a0 += fmaf(s0, d0[0] + d1[0], fmaf(-1024.0f, s0, z0) * sxg);
        a1 += fmaf(s1, d0[2] + d1[2], fmaf(-1024.0f, s1, z1) * sxg);
    }
    // Tiles [t0, t1) of this CTA's share of linear L (row block i = t / n_kc, K chunk
    // t % n_kc) from the ring; partial sums of every warp to red[t - t0].
    __device__ __forceinline__ void tiles(const MkLin &L, const __half *xs, int t0, int t1) {
        const int KC = L.kc, G64 = KC / 64, nkc = L.n_kc;
        const bool half_sb = pp->sbb == 4;
        int w0 = 0;  // warp that takes group 0 of the tile
        int kci = t0 % nkc;
        for (int t = t0; t < t1; ++t) {
            const uint32_t slot = seq & (NSLOT - 1);
            wait_slot(slot, 2);
            const uint8_t *tq = smem + slot * SLOT;
            const uint8_t *tsb = tq + 16 * KC;
            float a0 = 0.f, a1 = 0.f;
            {
                // (after a failed wait this reads stale, in-bounds shared memory)
                int j = (warp - w0) & (CW - 1);
                for (; j + CW < G64; j += 2 * CW) {
                    group(tq, tsb, KC, G64, j, kci * G64 + j, xs, half_sb, a0, a1);
                    group(tq, tsb, KC, G64, j + CW, kci * G64 + j + CW, xs, half_sb, a0, a1);
                }
                if (j < G64) group(tq, tsb, KC, G64, j, kci * G64 + j, xs, half_sb, a0, a1);
            }
            __syncwarp();
            if (lane == 0) mb_arrive(emptyp + slot);
            ++seq;
            if (c == 0) {
                float *r = red + ((t - t0) * CW + warp) * 16;
                r[g] = a0;
                r[g + 8] = a1;
            }
            w0 = (w0 + G64) & (CW - 1);
            if (++kci == nkc) kci = 0;
        }
        csync();
        trace();
    }
    // rows [4 q, 4 q + 4) of local row block i (tiles (i - i0) * n_kc ..): sum over warps
    // and K chunks in a fixed order, plus the bias
    __device__ __forceinline__ float4 rows4(const MkLin &L, int i_rel, int q) const {
        float v[4] = {0.f, 0.f, 0.f, 0.f};
        for (int k = 0; k < L.n_kc; ++k) {
            const float *r = red + ((i_rel * L.n_kc + k) * CW) * 16 + q * 4;
#pragma unroll
            for (int w = 0; w < CW; ++w) {
                const float4 x = *reinterpret_cast<const float4 *>(r + w * 16);
                v[0] += x.x; v[1] += x.y; v[2] += x.z; v[3] += x.w;
            }
        }
        return make_float4(v[0], v[1], v[2], v[3]);
    }
    __device__ __forceinline__ int own_rb(const MkLin &L) const {
        return rank < L.n_rb ? (L.n_rb - 1 - rank) / CS + 1 : 0;
    }
    // h or x_{l+1} = res + y + bias for this CTA's rows, pushed to all CTAs' res
    __device__ __forceinline__ void epi_resid(const MkLin &L, int bar) {
        const int nrb = own_rb(L), nch = nrb * 4;
        for (int i = tid; i < nch; i += CT) {
            const int ir = i >> 2, q = i & 3, o = (rank + ir * CS) * 16 + q * 4;
            float4 v = rows4(L, ir, q);
            const float4 bb = __ldg(reinterpret_cast<const float4 *>(L.bias + o));
            const float4 r = *reinterpret_cast<const float4 *>(res + o);
            v.x += r.x + bb.x; v.y += r.y + bb.y; v.z += r.z + bb.z; v.w += r.w + bb.w;
            reinterpret_cast<float4 *>(ostg)[i] = v;
        }
        csync();
        const uint32_t res_a = su32(res), bar_a = su32(stb + bar);
        for (int i = tid; i < nch * CS; i += CT) {
            const int dst = i & (CS - 1), ch = i >> 4;
            const int o = (rank + (ch >> 2) * CS) * 16 + (ch & 3) * 4;
            st_async_v4(mapa(res_a + o * 4, dst), reinterpret_cast<const float4 *>(ostg)[ch], mapa(bar_a, dst));
        }
    }

    // ---- stage A: x_l -> LN1 -> QKV; K/V appended; rows pushed to the attention CTAs ----
    __device__ __forceinline__ void stage_a(int l) {
        const MkParams &p = *pp;
        const MkLayer &Ly = p.layers[l];
        const LnRegs ln1 = ln_prefetch(Ly.ln1_w, Ly.ln1_b);
        if (l == 0) {
            const float *e = p.mel_emb + (size_t)T->tok * d, *ps = p.mel_pos + (size_t)T->pos * d;
            for (int k = tid; k < d; k += CT) res[k] = e[k] + ps[k];
            csync();
            trace();
        } else {
            wait_stage(BX, 20);
        }
        layernorm(ln1, false);
        const MkLin &L = Ly.qkv;
        tiles(L, xsa, 0, own_rb(L) * L.n_kc);
        const int nrb = own_rb(L), nch = nrb * 4;
        for (int i = tid; i < nch; i += CT) {
            const int ir = i >> 2, q = i & 3, o = (rank + ir * CS) * 16 + q * 4;
            float4 v = rows4(L, ir, q);
            const float4 bb = __ldg(reinterpret_cast<const float4 *>(L.bias + o));
            v.x += bb.x; v.y += bb.y; v.z += bb.z; v.w += bb.w;
            reinterpret_cast<float4 *>(ostg)[i] = v;
            const int which = o / d, oo = o - which * d;
            if (which > 0 && T->active) {
                __half *cache = which == 1 ? p.kc : p.vc;
                uint2 hv;
                hv.x = pack_h2(v.x, v.y);
                hv.y = pack_h2(v.z, v.w);
                *reinterpret_cast<uint2 *>(cache + kv_index(l, T->slot, oo >> 6, T->lold, p.n_slots, p.H, p.max_seq) +
                                           (oo & 63)) = hv;
            }
        }
        csync();
        const uint32_t qkv_a = su32(qkv), bar_a = su32(stb + BQKV);
        if (T->active)
            for (int i = tid; i < nch; i += CT) {
                const int o = (rank + (i >> 2) * CS) * 16 + (i & 3) * 4;
                const int which = o / d, oo = o - which * d, h = oo >> 6, e = oo & 63;
                const float4 v = reinterpret_cast<const float4 *>(ostg)[i];
                for (int r = T->rlo[h]; r <= T->rhi[h]; ++r) {
                    if (T->nh[r] == 0) continue;  // (a CTA between two of the head's CTAs with no units)
                    const int idx = ((h - T->hlo[r]) * 3 + which) * 64 + e;
                    st_async_v4(mapa(qkv_a + idx * 4, r), v, mapa(bar_a, r));
                }
            }
    }
    // ---- stage B: attention over this CTA's (head, K/V tile) range ----
    __device__ __forceinline__ void stage_b(int l) {
        wait_stage(BQKV, 21);
        const int grp = lane >> 3, d8 = lane & 7;
        float *ascr = red;                            // [MAXHC][CW][REC] warp states
        float *recs = red + MAXHC * CW * REC;         // [MAXHC][REC] segment records
        const float qscale = kAttnScale * kLog2e;
        int k = -1, hcur = -1;
        float qv[8], m = -INFINITY, ls = 0.f, acc[8];
        auto close = [&]() {
#pragma unroll
            for (int off = 8; off <= 16; off <<= 1) {
                const float m2 = __shfl_xor_sync(0xffffffffu, m, off);
                const float l2 = __shfl_xor_sync(0xffffffffu, ls, off);
                const float M = fmaxf(m, m2);
                const float fa = m == -INFINITY ? 0.f : exp2f(m - M);
                const float fb = m2 == -INFINITY ? 0.f : exp2f(m2 - M);
#pragma unroll
                for (int e = 0; e < 8; ++e) {
                    const float a2 = __shfl_xor_sync(0xffffffffu, acc[e], off);
                    acc[e] = acc[e] * fa + a2 * fb;
                }
                ls = ls * fa + l2 * fb;
                m = M;
            }
            if (grp == 0) {
                float *s = ascr + (k * CW + warp) * REC;
                if (d8 == 0) { s[0] = m; s[1] = ls; }
#pragma unroll
                for (int e = 0; e < 8; ++e) s[4 + d8 * 8 + e] = acc[e];
            }
        };
        if (T->u_hi > T->u_lo) {
            int h = T->u_lo / T->kvt, t = T->u_lo - h * T->kvt;
            for (int u = T->u_lo; u < T->u_hi; ++u) {
                if (h != hcur) {
                    if (k >= 0) close();
                    ++k;
                    hcur = h;
                    const float *qh = qkv + ((h - T->hlo[rank]) * 3) * 64 + d8 * 8;
#pragma unroll
                    for (int e = 0; e < 8; ++e) { qv[e] = qh[e] * qscale; acc[e] = 0.f; }
                    m = -INFINITY;
                    ls = 0.f;
                }
                const int np = min(KVPOS, T->lold - t * KVPOS);
                if (np > 0) {
                    const uint32_t slot = seq & (NSLOT - 1);
                    wait_slot(slot, 3);
                    const __half *kt = reinterpret_cast<const __half *>(smem + slot * SLOT);
                    const __half *vt = kt + np * 64;
                    // this warp's position groups gi = warp + 8 q (4 positions each, 8 lanes
                    // per position): scores first, then one rescale per tile
                    constexpr int QG = (KVPOS / 4 + CW - 1) / CW;
                    float sc[QG];
                    uint4 vv[QG];
#pragma unroll
                    for (int q = 0; q < QG; ++q) {
                        const int pos = (warp + q * CW) * 4 + grp;
                        const int pc = pos < np ? pos : 0;
                        const uint4 kk = *reinterpret_cast<const uint4 *>(kt + pc * 64 + d8 * 8);
                        vv[q] = *reinterpret_cast<const uint4 *>(vt + pc * 64 + d8 * 8);
                        const __half2 *k2 = reinterpret_cast<const __half2 *>(&kk);
                        float s0 = 0.f, s1 = 0.f;
#pragma unroll
                        for (int e = 0; e < 4; e += 2) {
                            const float2 ka = __half22float2(k2[e]), kb = __half22float2(k2[e + 1]);
                            s0 = fmaf(qv[2 * e], ka.x, s0);
                            s1 = fmaf(qv[2 * e + 1], ka.y, s1);
                            s0 = fmaf(qv[2 * e + 2], kb.x, s0);
                            s1 = fmaf(qv[2 * e + 3], kb.y, s1);
                        }
                        sc[q] = s0 + s1;
                    }
#pragma unroll
                    for (int q = 0; q < QG; ++q) sc[q] += __shfl_xor_sync(0xffffffffu, sc[q], 1);
#pragma unroll
                    for (int q = 0; q < QG; ++q) sc[q] += __shfl_xor_sync(0xffffffffu, sc[q], 2);
#pragma unroll
                    for (int q = 0; q < QG; ++q) sc[q] += __shfl_xor_sync(0xffffffffu, sc[q], 4);
                    float mt = m;
#pragma unroll
                    for (int q = 0; q < QG; ++q)
                        if ((warp + q * CW) * 4 + grp < np) mt = fmaxf(mt, sc[q]);
                    if (mt != m) {  // a new maximum (m = -inf gives corr 0)
                        const float corr = exp2f(m - mt);
                        ls *= corr;
#pragma unroll
                        for (int e = 0; e < 8; ++e) acc[e] *= corr;
                        m = mt;
                    }
#pragma unroll
                    for (int q = 0; q < QG; ++q) {
                        if ((warp + q * CW) * 4 + grp < np) {
                            const float pj = exp2f(sc[q] - m);
                            ls += pj;
                            const __half2 *v2 = reinterpret_cast<const __half2 *>(&vv[q]);
#pragma unroll
                            for (int e = 0; e < 4; ++e) {
                                const float2 f = __half22float2(v2[e]);
                                acc[2 * e] = fmaf(pj, f.x, acc[2 * e]);
                                acc[2 * e + 1] = fmaf(pj, f.y, acc[2 * e + 1]);
                            }
                        }
                    }
                    __syncwarp();
                    if (lane == 0) mb_arrive(emptyp + slot);
                    ++seq;
                }
                if (t == T->kvt - 1 && warp == CW - 1) {  // the new position (fp32, from stage A)
                    const float *kn = qkv + ((h - T->hlo[rank]) * 3 + 1) * 64 + d8 * 8;
                    const float *vn = kn + 64;
                    float s = 0.f;
#pragma unroll
                    for (int e = 0; e < 8; ++e) s = fmaf(qv[e], kn[e], s);
                    s += __shfl_xor_sync(0xffffffffu, s, 1);
                    s += __shfl_xor_sync(0xffffffffu, s, 2);
                    s += __shfl_xor_sync(0xffffffffu, s, 4);
                    if (grp == 0) {
                        const float mn = fmaxf(m, s);
                        const float corr = exp2f(m - mn);
                        const float pj = exp2f(s - mn);
                        ls = ls * corr + pj;
#pragma unroll
                        for (int e = 0; e < 8; ++e) acc[e] = acc[e] * corr + pj * vn[e];
                        m = mn;
                    }
                }
                if (++t == T->kvt) { t = 0; ++h; }
            }
            close();
        }
        csync();
        trace();
        const int nh = T->nh[rank];
        for (int i = tid; i < nh * 64; i += CT) {
            const int kk = i >> 6, e = i & 63;
            const float *s = ascr + kk * CW * REC;
            float M = -INFINITY;
#pragma unroll
            for (int w = 0; w < CW; ++w) M = fmaxf(M, s[w * REC]);
            float L2 = 0.f, A2 = 0.f;
#pragma unroll
            for (int w = 0; w < CW; ++w) {
                const float f = exp2f(s[w * REC] - M);
                L2 += s[w * REC + 1] * f;
                A2 += s[w * REC + 4 + e] * f;
            }
            float *rec = recs + kk * REC;
            rec[4 + e] = A2;
            if (e == 0) { rec[0] = M; rec[1] = L2; rec[2] = 0.f; rec[3] = 0.f; }
        }
        csync();
        const uint32_t part_a = su32(part), bar_a = su32(stb + BP);
        const int seg0 = T->seg0[rank];
        for (int i = tid; i < nh * (REC / 4) * CS; i += CT) {
            const int dst = i & (CS - 1), ch = i >> 4, kk = ch / (REC / 4), q = ch - kk * (REC / 4);
            const float4 v = *reinterpret_cast<const float4 *>(recs + kk * REC + q * 4);
            st_async_v4(mapa(part_a + ((seg0 + kk) * REC + q * 4) * 4, dst), v, mapa(bar_a, dst));
        }
    }
    // ---- stage C: merge the heads' partials -> c_proj + residual -> h (all CTAs) ----
    __device__ __forceinline__ void stage_c(int l) {
        wait_stage(BP, 22);
        for (int i = tid; i < d; i += CT) {
            float o = 0.f;
            if (T->active) {
                const int h = i >> 6, e = i & 63, s0 = T->hs0[h], s1 = T->hs0[h + 1];
                float M = -INFINITY;
                for (int s = s0; s < s1; ++s) M = fmaxf(M, part[s * REC]);
                float L2 = 0.f, A2 = 0.f;
                for (int s = s0; s < s1; ++s) {
                    const float f = exp2f(part[s * REC] - M);
                    L2 += part[s * REC + 1] * f;
                    A2 += part[s * REC + 4 + e] * f;
                }
                o = A2 / L2;
            }
            put_x(xsa, i, o);
        }
        group_sums(xsa, d);
        const MkLin &L = pp->layers[l].proj;
        tiles(L, xsa, 0, own_rb(L) * L.n_kc);
        epi_resid(L, BH);
    }
    // ---- stage D: LN2 -> c_fc + GELU -> u (fp16, fragment order, all CTAs) ----
    __device__ __forceinline__ void stage_d(int l) {
        const MkLayer &Ly = pp->layers[l];
        const LnRegs ln2 = ln_prefetch(Ly.ln2_w, Ly.ln2_b);
        wait_stage(BH, 23);
        layernorm(ln2, false);
        const MkLin &L = Ly.fc;
        tiles(L, xsa, 0, own_rb(L) * L.n_kc);
        // chunk (row block i, c): rows 2c, 2c+1, 2c+8, 2c+9 = 4 consecutive fp16 slots
        const int nrb = own_rb(L), nch = nrb * 4;
        for (int i = tid; i < nch; i += CT) {
            const int ir = i >> 2, cc = i & 3, rb = rank + ir * CS;
            float v[4];
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const int m = 2 * cc + (q & 1) + (q >> 1) * 8;
                float s = 0.f;
                for (int k = 0; k < L.n_kc; ++k) {
                    const float *r = red + ((ir * L.n_kc + k) * CW) * 16 + m;
#pragma unroll
                    for (int w = 0; w < CW; ++w) s += r[w * 16];
                }
                v[q] = gelu_tanh(s + __ldg(L.bias + rb * 16 + m));
            }
            uint2 hv;
            hv.x = pack_h2(v[0], v[1]);
            hv.y = pack_h2(v[2], v[3]);
            reinterpret_cast<uint2 *>(ostg)[i] = hv;
        }
        csync();
        const uint32_t xsu_a = su32(xsu), bar_a = su32(stb + BU);
        for (int i = tid; i < nch * CS; i += CT) {
            const int dst = i & (CS - 1), ch = i >> 4, rb = rank + (ch >> 2) * CS, cc = ch & 3;
            const int k0 = rb * 16;  // first input of the row block in the next linear
            const int idx = (k0 & ~63) + cc * 16 + ((k0 & 63) >> 4) * 4;
            st_async_v2(mapa(xsu_a + idx * 2, dst), reinterpret_cast<const uint2 *>(ostg)[ch], mapa(bar_a, dst));
        }
    }
    // ---- stage E: mlp c_proj + residual -> x_{l+1} (all CTAs) ----
    __device__ __forceinline__ void stage_e(int l) {
        wait_stage(BU, 24);
        group_sums(xsu, ff);
        const MkLin &L = pp->layers[l].mlp;
        tiles(L, xsu, 0, own_rb(L) * L.n_kc);
        epi_resid(L, BX);
    }
    // ---- head: ln_f -> final_norm -> mel_head (this CTA's row blocks) ----
    __device__ __forceinline__ void stage_head() {
        const MkParams &p = *pp;
        const LnRegs lnf = ln_prefetch(p.lnf_w, p.lnf_b);
        const LnRegs fin = ln_prefetch(p.fin_w, p.fin_b);
        if (p.n_layers > 0) wait_stage(BX, 25);
        layernorm(lnf, true);
        layernorm(fin, false);
        const MkLin &L = p.head;
        const int nrb = own_rb(L), V = p.mel_vocab;
        for (int i0 = 0; i0 < nrb; i0 += rt) {
            const int i1 = min(nrb, i0 + rt);
            tiles(L, xsa, i0 * L.n_kc, i1 * L.n_kc);
            for (int i = tid; i < (i1 - i0) * 4; i += CT) {
                const int ir = i >> 2, q = i & 3, o = (rank + (i0 + ir) * CS) * 16 + q * 4;
                const float4 v = rows4(L, ir, q);
                const float vv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                for (int e = 0; e < 4; ++e)
                    if (o + e < V) p.logits[o + e] = vv[e] + __ldg(L.bias + o + e);
            }
            csync();
        }
    }
};

// ---------------------------------------------------------------------------
// kernel
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(NT, 1) ck_decode_kernel(const __grid_constant__ CkParams cp) {
    extern __shared__ __align__(1024) uint8_t smem[];
    const MkParams &p = cp.p;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    uint32_t rank_u;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(rank_u));
    const int rank = (int)rank_u;
    const CkSmem SL = ck_layout(p.d, p.ff, p.H, cp.rt);
    CkTab *T = reinterpret_cast<CkTab *>(smem + SL.tab);
    uint64_t *fullp = reinterpret_cast<uint64_t *>(smem + SL.bar);
    uint64_t *emptyp = fullp + NSLOT;
    uint64_t *stb = emptyp + NSLOT;
    uint32_t expb[NSTB];

    // step shape (every CTA computes the same tables)
    const int slot = p.batch_slot[0];
    const SlotState &st = p.slots[slot];
    const int active = st.active && st.valid_len < p.max_seq;
    const int lold = active ? st.valid_len : 0;
    const int kvt = active ? max(1, (lold + KVPOS - 1) / KVPOS) : 0;
    const int units = p.H * kvt;
    if (tid == 0) {
        T->active = active;
        T->lold = lold;
        T->kvt = kvt;
        T->units = units;
        T->slot = slot;
        T->tok = min(max(st.tok, 0), p.mel_vocab - 1);
        T->pos = min(max(st.pos, 0), p.mel_pos_len - 1);
        int nseg = 0;
        for (int h = 0; h <= p.H; ++h) { T->hs0[h] = 0; T->rlo[h] = CS; T->rhi[h] = -1; }
        for (int r = 0; r < CS; ++r) {
            const int a = (int)((long long)r * units / CS), b = (int)((long long)(r + 1) * units / CS);
            T->u0[r] = a;
            T->seg0[r] = nseg;
            if (b > a) {
                const int hl = a / kvt, hh = (b - 1) / kvt;
                T->hlo[r] = hl;
                T->nh[r] = hh - hl + 1;
                for (int h = hl; h <= hh; ++h) {
                    if (T->rlo[h] == CS) { T->rlo[h] = r; T->hs0[h] = nseg + (h - hl); }
                    T->rhi[h] = r;
                }
                nseg += hh - hl + 1;
            } else {
                T->hlo[r] = 0;
                T->nh[r] = 0;
            }
            if (r == rank) { T->u_lo = a; T->u_hi = b; }
        }
        T->hs0[p.H] = nseg;
        T->nseg = nseg;
        for (int s = 0; s < NSLOT; ++s) {
            mb_init(fullp + s, 1);
            mb_init(emptyp + s, CW);
        }
        for (int b = 0; b < NSTB; ++b) mb_init(stb + b, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();
    expb[BX] = (uint32_t)p.d * 4;
    expb[BQKV] = (uint32_t)T->nh[rank] * 3 * 64 * 4;
    expb[BP] = (uint32_t)T->nseg * REC * 4;
    expb[BH] = (uint32_t)p.d * 4;
    expb[BU] = (uint32_t)p.ff * 2;
    if (tid == 0)
        for (int b = 0; b < NSTB; ++b) mb_expect(stb + b, expb[b]);
    // every CTA's barriers are armed before any CTA pushes into them
    cluster_sync_all();

    if (warp == CW) {
        if (lane == 0) {
            CkProducer P;
            P.smem = smem;
            P.ring = su32(smem);
            P.fullp = fullp;
            P.emptyp = emptyp;
            P.full = su32(fullp);
            P.empty = su32(emptyp);
            P.err = p.err;
            asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(P.pol));
            P.seq = 0;
            P.rank = rank;
            P.ok = true;
            P.run(p, *T);
        }
        __syncwarp();
    } else {
        CkConsumer C;
        C.pp = &p;
        C.T = T;
        C.smem = smem;
        C.res = reinterpret_cast<float *>(smem + SL.res);
        C.qkv = reinterpret_cast<float *>(smem + SL.qkv);
        C.part = reinterpret_cast<float *>(smem + SL.part);
        C.xsa = reinterpret_cast<__half *>(smem + SL.xsa);
        C.xsu = reinterpret_cast<__half *>(smem + SL.xsu);
        C.sx = reinterpret_cast<float *>(smem + SL.sx);
        C.red = reinterpret_cast<float *>(smem + SL.red);
        C.ostg = reinterpret_cast<float *>(smem + SL.ostg);
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
        C.d = p.d;
        C.ff = p.ff;
        C.H = p.H;
        C.rt = cp.rt;
        C.seq = 0;
        C.ok = true;
        C.ev = 0;
        for (int b = 0; b < NSTB; ++b) { C.ph[b] = 0; C.exp_bytes[b] = expb[b]; }
        for (int l = 0; l < p.n_layers; ++l) {
            C.stage_a(l);
            C.stage_b(l);
            C.stage_c(l);
            C.stage_d(l);
            C.stage_e(l);
        }
        C.stage_head();
    }
    // no CTA leaves while another may still push into its shared memory
    __syncwarp();
    cluster_sync_all();
}

}  // namespace

// Tiles of the largest per-CTA linear stage of the decoder layers; -1 when the cluster
// kernel does not fit this model (then the persistent grid kernel runs batch 1 too).
static int ck_rt_of(const MkLin &L) { return (L.n_rb + CS - 1) / CS * L.n_kc; }

int ck_config(const ModelView &m) {
    // opt-in: on B200 this kernel is slower than the grid-wide one (16 SMs do not issue the
    // dequantization instructions of a step fast enough), so it runs only on request
    const char *on = getenv("ITTS_CLUSTER");
    if (!on || on[0] != '1') return -1;
    if (m.n_layers < 1 || m.d > MK_MAX_D || m.d % 64 || m.ff % 64 || m.n_heads * 64 != m.d ||
        m.n_heads > MAXHC * CS / 2)
        return -1;
    int rt = 0;
    for (int l = 0; l < m.n_layers; ++l) {
        const MkLayer &L = m.layers[l];
        for (const MkLin *x : {&L.qkv, &L.proj, &L.fc, &L.mlp}) {
            if (x->tile_bytes > SLOT || x->kc % 64) return -1;
            rt = std::max(rt, ck_rt_of(*x));
        }
        if (L.qkv.out != 3 * m.d || L.proj.out != m.d || L.fc.out != m.ff || L.mlp.out != m.d) return -1;
    }
    if (m.mel_head.tile_bytes > SLOT) return -1;
    const CkSmem SL = ck_layout(m.d, m.ff, m.n_heads, rt);
    int dev = 0, optin = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    if ((int)SL.total > optin) return -1;
    if (cudaFuncSetAttribute(ck_decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)SL.total) !=
            cudaSuccess ||
        cudaFuncSetAttribute(ck_decode_kernel, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) != cudaSuccess) {
        cudaGetLastError();
        return -1;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(CS);
    cfg.blockDim = dim3(NT);
    cfg.dynamicSmemBytes = SL.total;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = CS;
    at[0].val.clusterDim.y = 1;
    at[0].val.clusterDim.z = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    int nclusters = 0;
    if (cudaOccupancyMaxActiveClusters(&nclusters, ck_decode_kernel, &cfg) != cudaSuccess || nclusters < 1) {
        cudaGetLastError();
        if (getenv("ITTS_DEBUG")) fprintf(stderr, "[itts] cluster decode kernel: no 16-CTA cluster fits\n");
        return -1;
    }
    if (getenv("ITTS_DEBUG"))
        fprintf(stderr, "[itts] cluster decode kernel: %u B shared memory, %d partial tiles, %d clusters fit\n",
                SL.total, rt, nclusters);
    return rt;
}

cudaError_t ck_launch(const MkParams &p, int rt, cudaStream_t st) {
    CkParams cp;
    cp.p = p;
    cp.rt = rt;
    const CkSmem SL = ck_layout(p.d, p.ff, p.H, rt);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(CS);
    cfg.blockDim = dim3(NT);
    cfg.dynamicSmemBytes = SL.total;
    cfg.stream = st;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = CS;
    at[0].val.clusterDim.y = 1;
    at[0].val.clusterDim.z = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, ck_decode_kernel, cp);
}

}  // namespace itts
