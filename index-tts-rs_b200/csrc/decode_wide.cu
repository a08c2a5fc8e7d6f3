// decode_wide.cu -- decode steps of 5 to 64 batch columns on the int8 weights.
//
// Reference semantics: QuantizedLinear::forward (crates/core/src/models/gpt.rs:252-264, MLX
// quantized_matmul with group 64, 8 bits, affine W = s q + b) inside Gpt2Block::forward
// (gpt.rs:325-384) for a step of several requests.  A step of nb columns is a skinny GEMM
// per linear: nb <= 64 activation rows against 16-row weight tiles.  The work is bound by
// reading the weights (int8 tiles, the only copy read) and by latency, not by the tensor
// pipe, so the product runs on mma.sync m16n8k16 with the weights dequantized in registers;
// the 64-column batch is far below a tcgen05 tile.
//
// Activations between the stages are fp16 in the tiles' fragment order: within each group
// of 64 inputs, element k sits at frag_pos(k), so that one 16-byte load gives a thread its
// B operand for two k16 blocks (the same permutation as the weight bytes, mk.h).
//
// Persistent CTAs, one per SM: CTA b takes K chunk b % n_kc and every G-th row block from
// b / n_kc (G = CTAs per chunk).  It stages its K chunk of the nb columns' activations once
// by bulk copies, then streams its 16-row weight tiles through two shared-memory buffers
// (the next tile lands while the current one is multiplied).  Warp w takes n-tile (8
// columns) w % NT and every KS-th quantization group (NT * KS <= 8 warps); per group
// y += s (W_q . x) + (b - 1024 s) (sum of x), with W_q . x from the fp16 byte trick
// (1024 + q) of the other decode kernels.  The K parts are summed in a fixed order in shared
// memory; for linears with several K chunks (the mlp projection) each CTA writes its chunk's
// partials and the last CTA of the row block adds them in chunk order.  No atomics on
// values: results are deterministic.
#include <algorithm>
#include <cstdio>

#include "gemm.cuh"
#include "kernels.h"

namespace itts {
namespace {

// 16 warps per CTA when the K-part reduction buffer of 16 warps fits in shared memory, else 8
// (one CTA per SM either way: the activation block takes most of the shared memory)
constexpr int SK_THREADS = 512;
constexpr int SK_WARPS_LO = 8;
constexpr uint32_t SK_SPIN = 1u << 24;
// Dynamic shared memory of the skinny kernel: at most this (the kernel's static shared
// memory and the per-block reserve stay below the 227 KB opt-in limit of sm_100).
constexpr int SK_MAX_SMEM = 226 * 1024;
constexpr int SK_RPITCH = 17;  // floats per column of the K-part reduction buffer (16 rows + pad)
constexpr int SK_NTW = 2;      // n-tiles (8 columns each) per warp: its weight fragments serve both

// Warp roles for nb columns and `warps` warps: NT n-tiles in ng groups of ntw (a warp's weight
// fragments serve its ntw n-tiles), ks = warps / ng K parts (warp w: group w % ng, part w / ng);
// nc = ng*ntw*8.
struct SkShape {
    int ntw, ng, ks, nc;
};
__host__ __device__ inline SkShape sk_shape(int nb, int warps) {
    const int NT = (nb + 7) / 8;
    SkShape s;
    s.ntw = NT < SK_NTW ? NT : SK_NTW;
    s.ng = (NT + s.ntw - 1) / s.ntw;
    s.ks = warps / s.ng;
    s.nc = s.ng * s.ntw * 8;
    return s;
}

__device__ __forceinline__ uint32_t su32(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mma16816(float *d, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                         uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
// bytes 0,1 (2,3) of w as the fp16 values 1024 + q
__device__ __forceinline__ uint32_t lo_h(uint32_t w) { return __byte_perm(w, 0x64646464u, 0x4140u); }
__device__ __forceinline__ uint32_t hi_h(uint32_t w) { return __byte_perm(w, 0x64646464u, 0x4342u); }

__device__ __forceinline__ float hsum8(uint4 v) {
    const __half2 *h = reinterpret_cast<const __half2 *>(&v);
    float s = 0.f;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
        const float2 f = __half22float2(h[e]);
        s += f.x + f.y;
    }
    return s;
}

__device__ __forceinline__ int frag_pos(int k) {  // position of input k within its group of 64
    const int b = k >> 4, kk = k & 15, c = (kk & 7) >> 1, hi = kk >> 3, lo = kk & 1;
    return c * 16 + b * 4 + hi * 2 + lo;
}

}  // namespace

struct SkinnyParams {
    MkLin W;
    const __half *x;  // [n_kc][nb][KC] fp16 (K chunk-major; [nb][K] for one chunk), fragment order
    int nb;
    GemmParams gp;    // epilogue (QKV: q + K/V append; RESID: += ; PLAIN)
    __half *y16;      // EPI_GELU: fp16 in the next GEMM's input layout [out / y_kc][nb][y_kc]
    int y_kc;         // K chunk of the GEMM that reads y16
    float *ws;        // [n_kc][nb][out] partial sums when n_kc > 1
    int *counters;    // [n_rb], zero between launches (row blocks whose K chunks are combined)
};

// Per-column K/V destination of the QKV epilogue (Gpt2Block cache update, gpt.rs:340-360):
// the slot's valid_len, unless the slot is inactive or full.
struct SkKvDest {
    int slot[SK_MAX_NB], pos[SK_MAX_NB];
    unsigned char write[SK_MAX_NB];
};

// Outputs (o, n) for n = n0, n0 + ec, ... (< nb) of one row o: v[u] holds column n0 + ec u
// (ec = threads / 16: 16 or 32).  Every load of a thread is issued before its stores (the
// residual's x, nothing else).
template <int EPI>
__device__ __forceinline__ void skinny_epilogue(const SkinnyParams &p, const SkKvDest &kd, int o, int n0, int ec,
                                                const float *v) {
    const int OUT = p.W.out, nb = p.nb;
    float *y = p.gp.y;
    if constexpr (EPI == EPI_RESID) {
        float xv[SK_MAX_NB / 16];
#pragma unroll
        for (int u = 0; u < SK_MAX_NB / 16; ++u) {
            const int n = n0 + ec * u;
            xv[u] = n < nb ? y[(size_t)n * OUT + o] : 0.f;
        }
#pragma unroll
        for (int u = 0; u < SK_MAX_NB / 16; ++u) {
            const int n = n0 + ec * u;
            if (n < nb) y[(size_t)n * OUT + o] = xv[u] + v[u];
        }
    } else {
#pragma unroll
        for (int u = 0; u < SK_MAX_NB / 16; ++u) {
            const int n = n0 + ec * u;
            if (n >= nb) break;
            if (EPI == EPI_GELU) {
                const int kc = o / p.y_kc, w = o - kc * p.y_kc;
                p.y16[((size_t)kc * nb + n) * p.y_kc + (w & ~63) + frag_pos(w & 63)] = __float2half_rn(gelu_tanh(v[u]));
            } else {
                y[(size_t)n * OUT + o] = v[u];
                if (EPI == EPI_QKV && o >= p.gp.d && kd.write[n]) {
                    const int rr = o - p.gp.d, which = rr / p.gp.d, oo = rr - which * p.gp.d;
                    __half *cache = which == 0 ? p.gp.k_cache : p.gp.v_cache;
                    cache[kv_index(p.gp.layer, kd.slot[n], oo >> 6, kd.pos[n], p.gp.n_slots, p.gp.n_heads, p.gp.max_seq) +
                          (oo & 63)] = __float2half_rn(v[u]);
                }
            }
        }
    }
}

template <int EPI>
__global__ void __launch_bounds__(SK_THREADS, 1) skinny_q8_kernel(const __grid_constant__ SkinnyParams p) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ __align__(8) uint64_t bars[3];  // activations, weight buffers 0 and 1
    __shared__ int s_last;
    __shared__ SkKvDest kd;
    const MkLin &W = p.W;
    const int KC = W.kc, G64 = KC / 64, tb = W.tile_bytes, nb = p.nb, nkc = W.n_kc;
    const int groups = gridDim.x / nkc, kc = blockIdx.x % nkc, gi = blockIdx.x / nkc;
    const int nmine = gi < W.n_rb ? (W.n_rb - gi + groups - 1) / groups : 0;  // row blocks gi + i groups
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, c = lane & 3;
    const SkShape sh = sk_shape(nb, (int)(blockDim.x >> 5));
    const int nthr = (int)blockDim.x, ec = nthr >> 4;
    uint8_t *wbuf = smem;                                                    // [2][tile]
    __half *xs = reinterpret_cast<__half *>(smem + 2 * (size_t)tb);          // [nb][KC]
    float *sxs = reinterpret_cast<float *>(smem + 2 * (size_t)tb + (size_t)nb * KC * 2);  // [nb][G64] group sums
    float *red = sxs + (size_t)nb * G64;                                     // [KS][NC][pitch]
    if (nmine == 0) return;
    const uint32_t bx = su32(&bars[0]), bw0 = su32(&bars[1]);
    auto tile_src = [&](int i) { return W.tiles + ((size_t)(gi + i * groups) * nkc + kc) * tb; };
    auto copy = [&](uint32_t dst, const void *src, uint32_t bytes, uint32_t bar) {
        asm volatile(
            "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
            "l"(src), "r"(bytes), "r"(bar)
            : "memory");
    };
    auto expect = [&](uint32_t bar, uint32_t bytes) {
        asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
    };
    auto wait = [&](uint32_t bar, uint32_t parity) {  // copies always complete; bounded anyway
        uint32_t done = 0;
        for (uint32_t it = 0; it < SK_SPIN && !done; ++it)
            asm volatile("{\n .reg .pred q;\n mbarrier.try_wait.parity.shared::cta.b64 q, [%1], %2, 1000000;\n selp.u32 %0, 1, 0, q;\n}\n"
                         : "=r"(done)
                         : "r"(bar), "r"(parity)
                         : "memory");
    };
    if (tid == 0) {
        for (int b = 0; b < 3; ++b) asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(bx + 8 * b) : "memory");
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        expect(bx, (uint32_t)(nb * KC * 2));
        expect(bw0, (uint32_t)tb);
        if (nmine > 1) expect(bw0 + 8, (uint32_t)tb);
    }
    __syncthreads();
    if (tid == 0) {  // this K chunk of every column's activations (contiguous), once for all row blocks
        copy(su32(xs), p.x + (size_t)kc * nb * KC, (uint32_t)(nb * KC * 2), bx);
    } else if (tid <= 2 && tid - 1 < nmine) {  // the first two weight tiles
        const int i = tid - 1;
        copy(su32(wbuf + (size_t)i * tb), tile_src(i), (uint32_t)tb, bw0 + 8 * i);
    }
    if (EPI == EPI_QKV && tid < nb) {  // the columns' K/V destinations, while the copies land
        const QkvDest q = qkv_dest(p.gp, tid);
        kd.slot[tid] = q.slot;
        kd.pos[tid] = q.pos;
        kd.write[tid] = q.write ? 1 : 0;
    }
    const int KS = sh.ks, NTW = sh.ntw, NC = sh.nc;
    const int ng = warp % sh.ng, kp = warp / sh.ng;  // n-tiles ng * NTW .. + NTW - 1, K part kp
    const bool half_sb = W.sbb == 4;
    const int erow = tid & 15, en0 = tid >> 4;  // epilogue: row erow, columns en0 + ec u
    wait(bx, 0);
    // every column's group sums (the dequantization offset term), once for all row blocks
    for (int q = tid; q < nb * G64; q += nthr) {
        const uint4 *src = reinterpret_cast<const uint4 *>(xs + (size_t)(q / G64) * KC + (q % G64) * 64);
        float a = 0.f;
#pragma unroll
        for (int e = 0; e < 8; ++e) a += hsum8(src[e]);
        sxs[q] = a;
    }
    __syncthreads();
    for (int i = 0; i < nmine; ++i) {
        const int rb = gi + i * groups, buf = i & 1;
        const int eo = rb * 16 + erow;
        const bool erow_ok = eo < W.out;
        const float ebias = erow_ok ? __ldg(W.bias + eo) : 0.f;
        wait(bw0 + 8 * buf, (uint32_t)(i >> 1) & 1u);
        if (kp < KS) {
            const uint8_t *tq = wbuf + (size_t)buf * tb, *tsb = tq + 16 * KC;
            float y[SK_NTW][4];
#pragma unroll
            for (int t = 0; t < SK_NTW; ++t) y[t][0] = y[t][1] = y[t][2] = y[t][3] = 0.f;
            for (int j = kp; j < G64; j += KS) {
                // this group's weight fragments and (scale, offset) pairs, shared by the n-tiles
                const int jj = j ^ (g & 1);
                const uint4 wa = *reinterpret_cast<const uint4 *>(tq + g * KC + jj * 64 + c * 16);
                const uint4 wb = *reinterpret_cast<const uint4 *>(tq + (g + 8) * KC + jj * 64 + c * 16);
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
                const float c0 = fmaf(-1024.0f, s0, z0), c1 = fmaf(-1024.0f, s1, z1);
                const uint32_t a00 = lo_h(wa.x), a01 = lo_h(wb.x), a02 = hi_h(wa.x), a03 = hi_h(wb.x);
                const uint32_t a10 = lo_h(wa.y), a11 = lo_h(wb.y), a12 = hi_h(wa.y), a13 = hi_h(wb.y);
                const uint32_t a20 = lo_h(wa.z), a21 = lo_h(wb.z), a22 = hi_h(wa.z), a23 = hi_h(wb.z);
                const uint32_t a30 = lo_h(wa.w), a31 = lo_h(wb.w), a32 = hi_h(wa.w), a33 = hi_h(wb.w);
#pragma unroll
                for (int t = 0; t < SK_NTW; ++t) {
                    const int nt = ng * NTW + t, col = nt * 8 + g;
                    if (t >= NTW || nt * 8 >= nb) break;  // (warp-uniform)
                    uint4 x0 = make_uint4(0, 0, 0, 0), x1 = x0;
                    if (col < nb) {
                        const __half *xc = xs + (size_t)col * KC + j * 64 + c * 16;
                        x0 = *reinterpret_cast<const uint4 *>(xc);
                        x1 = *reinterpret_cast<const uint4 *>(xc + 8);
                    }
                    const int ca = nt * 8 + 2 * c;  // the D fragment's columns ca, ca + 1
                    const float sxa = ca < nb ? sxs[(size_t)ca * G64 + j] : 0.f;
                    const float sxb = ca + 1 < nb ? sxs[(size_t)(ca + 1) * G64 + j] : 0.f;
                    float d0[4] = {0.f, 0.f, 0.f, 0.f}, d1[4] = {0.f, 0.f, 0.f, 0.f};
                    mma16816(d0, a00, a01, a02, a03, x0.x, x0.y);
                    mma16816(d1, a10, a11, a12, a13, x0.z, x0.w);
                    mma16816(d0, a20, a21, a22, a23, x1.x, x1.y);
                    mma16816(d1, a30, a31, a32, a33, x1.z, x1.w);
                    y[t][0] += fmaf(s0, d0[0] + d1[0], c0 * sxa);  // row g,     column ca
                    y[t][1] += fmaf(s0, d0[1] + d1[1], c0 * sxb);  // row g,     column ca + 1
                    y[t][2] += fmaf(s1, d0[2] + d1[2], c1 * sxa);  // row g + 8, column ca
                    y[t][3] += fmaf(s1, d0[3] + d1[3], c1 * sxb);  // row g + 8, column ca + 1
                }
            }
            // red[kp][column][row 0..15] (padded pitch: no bank conflicts on either side)
            float *rk = red + (size_t)kp * NC * SK_RPITCH;
#pragma unroll
            for (int t = 0; t < SK_NTW; ++t) {
                const int nt = ng * NTW + t;
                if (t >= NTW || nt * 8 >= NC) break;
                const int cc = nt * 8 + 2 * c;
                rk[cc * SK_RPITCH + g] = y[t][0];
                rk[(cc + 1) * SK_RPITCH + g] = y[t][1];
                rk[cc * SK_RPITCH + g + 8] = y[t][2];
                rk[(cc + 1) * SK_RPITCH + g + 8] = y[t][3];
            }
        }
        __syncthreads();  // red complete; weight buffer `buf` no longer read
        if (tid == 0 && i + 2 < nmine) {
            expect(bw0 + 8 * buf, (uint32_t)tb);
            copy(su32(wbuf + (size_t)buf * tb), tile_src(i + 2), (uint32_t)tb, bw0 + 8 * buf);
        }
        // this thread's outputs: row erow, columns en0 + 16 u, summed over the K parts in order
        float v[SK_MAX_NB / 16];
#pragma unroll
        for (int u = 0; u < SK_MAX_NB / 16; ++u) {
            const int n = en0 + ec * u;
            float a = 0.f;
            if (n < nb)
                for (int k = 0; k < KS; ++k) a += red[((size_t)k * NC + n) * SK_RPITCH + erow];
            v[u] = a;
        }
        if (nkc == 1) {
            if (erow_ok) {
#pragma unroll
                for (int u = 0; u < SK_MAX_NB / 16; ++u) v[u] += ebias;
                skinny_epilogue<EPI>(p, kd, eo, en0, ec, v);
            }
        } else {  // several K chunks: partials, then the last of the row block's CTAs sums them
            if (erow_ok) {
                float *wsk = p.ws + (size_t)kc * nb * W.out;
#pragma unroll
                for (int u = 0; u < SK_MAX_NB / 16; ++u) {
                    const int n = en0 + ec * u;
                    if (n < nb) wsk[(size_t)n * W.out + eo] = v[u];
                }
            }
            __threadfence();
            __syncthreads();
            if (tid == 0) s_last = atomicAdd(p.counters + rb, 1) == nkc - 1;
            __syncthreads();
            if (s_last) {
                __threadfence();
                if (erow_ok) {
                    float t[SK_MAX_NB / 16];
#pragma unroll
                    for (int u = 0; u < SK_MAX_NB / 16; ++u) t[u] = ebias;
                    float part[SK_MAX_NB / 16];
#pragma unroll
                    for (int u = 0; u < SK_MAX_NB / 16; ++u) part[u] = 0.f;
                    for (int k = 0; k < nkc; ++k) {  // chunk order
                        const float *wk = p.ws + (size_t)k * nb * W.out;
#pragma unroll
                        for (int u = 0; u < SK_MAX_NB / 16; ++u) {
                            const int n = en0 + ec * u;
                            if (n < nb) part[u] += __ldcg(wk + (size_t)n * W.out + eo);
                        }
                    }
#pragma unroll
                    for (int u = 0; u < SK_MAX_NB / 16; ++u) t[u] += part[u];
                    skinny_epilogue<EPI>(p, kd, eo, en0, ec, t);
                }
                if (tid == 0) p.counters[rb] = 0;
            }
        }
        __syncthreads();  // red is rewritten by the next row block
    }
}

size_t skinny_smem_bytes(const MkLin &W, int nb, int warps) {
    const SkShape sh = sk_shape(nb, warps);
    return 2 * (size_t)W.tile_bytes + (size_t)nb * W.kc * 2 + (size_t)nb * (W.kc / 64) * 4 +
           (size_t)sh.ks * sh.nc * SK_RPITCH * 4;
}

// Warps per CTA for this GEMM and column count: 16 when every K part still gets at least 4 of
// the tile's quantization groups and the larger reduction buffer fits, else 8.  (At 64 columns
// 16 warps took the step from 3.42 to 3.33 ms; at 32 columns, 8 K parts of 2-3 groups each were
// slower than 4 parts of 5.)
static int skinny_warps(const MkLin &W, int nb) {
    const int hi = SK_THREADS / 32;
    const bool enough_groups = sk_shape(nb, hi).ks * 4 <= W.kc / 64;
    return enough_groups && skinny_smem_bytes(W, nb, hi) <= (size_t)SK_MAX_SMEM ? hi : SK_WARPS_LO;
}

bool skinny_ok(const MkLin &W, int nb) {
    return nb >= 1 && nb <= SK_MAX_NB && W.kc % 64 == 0 && W.tile_bytes % 16 == 0 && (W.kc * 2) % 16 == 0 &&
           W.n_rb <= 4096 && skinny_smem_bytes(W, nb, SK_WARPS_LO) <= (size_t)SK_MAX_SMEM;
}

constexpr int LNF_CH = MK_MAX_D / 128;
template <int NCH>
__global__ void ln_frag_kernel(const float *x, const float *w, const float *b, int rows, int d, __half *y);

void kernels_init_wide() {  // once per device, at model load
    cudaFuncSetAttribute(skinny_q8_kernel<EPI_PLAIN>, cudaFuncAttributeMaxDynamicSharedMemorySize, SK_MAX_SMEM);
    cudaFuncSetAttribute(skinny_q8_kernel<EPI_GELU>, cudaFuncAttributeMaxDynamicSharedMemorySize, SK_MAX_SMEM);
    cudaFuncSetAttribute(skinny_q8_kernel<EPI_RESID>, cudaFuncAttributeMaxDynamicSharedMemorySize, SK_MAX_SMEM);
    cudaFuncSetAttribute(skinny_q8_kernel<EPI_QKV>, cudaFuncAttributeMaxDynamicSharedMemorySize, SK_MAX_SMEM);
    cudaFuncSetAttribute(ln_frag_kernel<2>, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
    cudaFuncSetAttribute(ln_frag_kernel<6>, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
    cudaFuncSetAttribute(ln_frag_kernel<10>, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
    cudaFuncSetAttribute(ln_frag_kernel<LNF_CH>, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
    cudaGetLastError();  // a refusal shows up as skinny_ok() launches failing, never as a stale error
}

template <int EPI>
static cudaError_t skinny_launch_t(const SkinnyParams &p, cudaStream_t st) {
    const int warps = skinny_warps(p.W, p.nb);
    const size_t smem = skinny_smem_bytes(p.W, p.nb, warps);
    static int sms[64] = {0};  // SMs per device (one CTA per SM: the kernel takes most of the shared memory)
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && sms[dev] == 0) cudaDeviceGetAttribute(&sms[dev], cudaDevAttrMultiProcessorCount, dev);
    const int n_sm = dev >= 0 && dev < 64 && sms[dev] > 0 ? sms[dev] : 148;
    const int groups = std::max(1, std::min(p.W.n_rb, n_sm / p.W.n_kc));
    dim3 grid(groups * p.W.n_kc);
    skinny_q8_kernel<EPI><<<grid, warps * 32, smem, st>>>(p);
    return cudaGetLastError();
}

cudaError_t launch_skinny(int epi, const MkLin &W, const __half *x, int nb, void *y, const DecodeView *dv,
                          int layer, int d, float *ws, int *counters, cudaStream_t st, int y_kc) {
    SkinnyParams p{};
    p.y_kc = y_kc > 0 ? y_kc : W.out;
    p.W = W;
    p.x = x;
    p.nb = nb;
    p.ws = ws;
    p.counters = counters;
    GemmParams &g = p.gp;
    g.W = W;
    g.T = nb;
    g.y = reinterpret_cast<float *>(y);
    g.layer = layer;
    g.d = d;
    if (dv) {
        g.k_cache = dv->k_cache;
        g.v_cache = dv->v_cache;
        g.slots = dv->slots;
        g.batch_slot = dv->batch_slot;
        g.n_slots = dv->n_slots;
        g.n_heads = dv->n_heads;
        g.max_seq = dv->max_seq;
    }
    if (epi == EPI_GELU) p.y16 = reinterpret_cast<__half *>(y);
    switch (epi) {
        case EPI_PLAIN: return skinny_launch_t<EPI_PLAIN>(p, st);
        case EPI_GELU: return skinny_launch_t<EPI_GELU>(p, st);
        case EPI_RESID: return skinny_launch_t<EPI_RESID>(p, st);
        default: return skinny_launch_t<EPI_QKV>(p, st);
    }
}

// ---------------------------------------------------------------------------
// LayerNorm of nb rows into fp16 fragment order (the skinny GEMM's activation layout):
// one warp per row and two rows per CTA (so a 64-row step spreads over 32 SMs), two-pass
// statistics over the row held in registers; the row, its weights and its biases are all
// loaded before the first reduction.  NCH (>= d / 128) sizes the register arrays.
// ---------------------------------------------------------------------------
template <int NCH>
__global__ void __launch_bounds__(64) ln_frag_kernel(const float *x, const float *w, const float *b, int rows,
                                                     int d, __half *y) {
    const int t = blockIdx.x * 2 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (t >= rows) return;
    const int nch = d / 128;
    const float4 *row = reinterpret_cast<const float4 *>(x + (size_t)t * d);
    float4 v[NCH], ww[NCH], bb[NCH];
#pragma unroll
    for (int c = 0; c < NCH; ++c) {  // every load issued before the first use (no early exit)
        const bool in = c < nch;
        v[c] = in ? row[c * 32 + lane] : make_float4(0.f, 0.f, 0.f, 0.f);
        ww[c] = in ? __ldg(reinterpret_cast<const float4 *>(w) + c * 32 + lane) : v[c];
        bb[c] = in ? __ldg(reinterpret_cast<const float4 *>(b) + c * 32 + lane) : v[c];
    }
    float s = 0.f;
#pragma unroll
    for (int c = 0; c < NCH; ++c) s += (v[c].x + v[c].y) + (v[c].z + v[c].w);
    const float mean = warp_sum(s) / (float)d;
    float q = 0.f;
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
        if (c < nch) {
            const float a0 = v[c].x - mean, a1 = v[c].y - mean, a2 = v[c].z - mean, a3 = v[c].w - mean;
            q += (a0 * a0 + a1 * a1) + (a2 * a2 + a3 * a3);
        }
    }
    const float rstd = 1.0f / sqrtf(warp_sum(q) / (float)d + kNormEps);
    __half *yr = y + (size_t)t * d;
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
        if (c >= nch) break;
        const int k0 = (c * 32 + lane) * 4;
        const float o0 = (v[c].x - mean) * rstd * ww[c].x + bb[c].x, o1 = (v[c].y - mean) * rstd * ww[c].y + bb[c].y;
        const float o2 = (v[c].z - mean) * rstd * ww[c].z + bb[c].z, o3 = (v[c].w - mean) * rstd * ww[c].w + bb[c].w;
        // inputs k, k + 1 (k even) sit next to each other in fragment order
        __half *g = yr + (k0 & ~63);
        *reinterpret_cast<__half2 *>(g + frag_pos(k0 & 63)) = __floats2half2_rn(o0, o1);
        *reinterpret_cast<__half2 *>(g + frag_pos((k0 + 2) & 63)) = __floats2half2_rn(o2, o3);
    }
}

void launch_ln_frag(const float *x, const float *w, const float *b, int rows, int d, __half *y, cudaStream_t st) {
    const int nch = d / 128, grid = (rows + 1) / 2;
    if (nch <= 2) ln_frag_kernel<2><<<grid, 64, 0, st>>>(x, w, b, rows, d, y);
    else if (nch <= 6) ln_frag_kernel<6><<<grid, 64, 0, st>>>(x, w, b, rows, d, y);
    else if (nch <= 10) ln_frag_kernel<10><<<grid, 64, 0, st>>>(x, w, b, rows, d, y);
    else ln_frag_kernel<LNF_CH><<<grid, 64, 0, st>>>(x, w, b, rows, d, y);
}

}  // namespace itts
