// gemm_tc.cu -- the int8-weight GEMM on the 5th-generation tensor cores (tcgen05), used by
// prefill and by decode steps with more columns than the persistent kernel takes:
// y[t, o] = x[t, :] . W[o, :] + bias[o] with the plain / GELU / residual / QKV epilogues
// (crates/core/src/models/gpt.rs:252-264 QuantizedLinear::forward inside Gpt2Block).
//
// One CTA computes a 128-row (positions) x 128-column (weight rows) tile with an fp32
// accumulator in tensor memory.  The K loop runs over the 64-input quantization groups:
//  * the fp16 activation tile of a group (128 rows x 128 bytes) arrives by one TMA tensor
//    copy straight into one of four A stages, already in the 128-byte-swizzled K-major
//    layout the MMA reads;
//  * the group's int8 weight bytes and (scale, offset) pairs arrive by cp.async into one of
//    three raw stages, and the 8 warps dequantize them (s * q + b in fp32, then fp16) into
//    one of two B stages in the same swizzled layout;
//  * one thread issues the group's 4 tcgen05.mma (K = 16 each) and commits them to the B
//    stage's mbarrier.
// Copies run two groups ahead, so copies, dequantization and tensor-core work overlap.
// Every wait is bounded; on expiry the kernel records an error, skips the rest, lets its
// copies land, frees its tensor memory and returns.
#include <cuda.h>

#include <algorithm>
#include <mutex>

#include "gemm.cuh"

namespace itts {

constexpr int TC_BM = 128, TC_BN = 128, TC_BK = 64, TC_THREADS = 256;
constexpr int TC_TILE_BYTES = TC_BM * TC_BK * 2;  // one operand stage: 16 KB
constexpr int TC_A_STAGES = 4, TC_B_STAGES = 2, TC_RAW_STAGES = 3;
// raw weight stage: weight bytes (128 rows x 64) and (scale, offset) pairs (8 B per row)
constexpr int TC_RAW_B = TC_BN * TC_BK, TC_RAW_S = TC_BN * 8, TC_RAW_STAGE = TC_RAW_B + TC_RAW_S;
constexpr int TC_OFF_B = TC_A_STAGES * TC_TILE_BYTES;
constexpr int TC_OFF_RAW = TC_OFF_B + TC_B_STAGES * TC_TILE_BYTES;
constexpr int TC_SMEM = TC_OFF_RAW + TC_RAW_STAGES * TC_RAW_STAGE + 1024;
// epilogue staging of the fp32 accumulator tile over the A and B stages (row stride in
// floats, padded by 4)
constexpr int TC_STG_LD = TC_BN + 4;
static_assert(TC_BM * TC_STG_LD * 4 <= TC_OFF_RAW, "epilogue staging exceeds the operand stages");
constexpr uint32_t TC_TMEM_COLS = 128;
constexpr long TC_SPIN = 1L << 24;
// instruction descriptor (kind::f16): D f32, A and B f16, both K-major, N = 128, M = 128
constexpr uint32_t TC_IDESC = (1u << 4) | ((uint32_t)(TC_BN >> 3) << 17) | ((uint32_t)(TC_BM >> 4) << 24);

__device__ int g_gemm_tc_error;  // nonzero once a bounded wait gave up

__device__ __forceinline__ uint32_t tc_su32(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }

// Byte offset of element (r, k), k < 64, in a K-major tile of 64 fp16 per row with the
// 128-byte swizzle (the layout TMA writes with CU_TENSOR_MAP_SWIZZLE_128B): 8-row groups of
// 1024 B; in row r the 16-byte chunk k/8 sits at chunk position (k/8) ^ (r % 8).
__device__ __forceinline__ uint32_t tc_swz(int r, int k) {
    return (uint32_t)((r >> 3) * 1024 + (r & 7) * 128 + (((k >> 3) ^ (r & 7)) << 4) + (k & 7) * 2);
}
// Shared-memory matrix descriptor of such a tile (start address, stride between 8-row
// groups 1024 B, descriptor version 1, 128-byte swizzle).
__device__ __forceinline__ uint64_t tc_desc(uint32_t saddr) {
    return (uint64_t)((saddr >> 4) & 0x3FFF) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
           ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}
__device__ __forceinline__ bool tc_wait(uint64_t *bar, uint32_t parity) {
    for (long it = 0; it < TC_SPIN; ++it) {
        uint32_t done;
        asm volatile(
            "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
            " selp.u32 %0, 1, 0, p;\n}\n"
            : "=r"(done)
            : "r"(tc_su32(bar)), "r"(parity)
            : "memory");
        if (done) return true;
    }
    atomicExch(&g_gemm_tc_error, 1);
    return false;
}
__device__ __forceinline__ uint32_t pack_half2(float a, float b) {
    const __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<const uint32_t *>(&h);
}
// 16-byte (or 4 / 8-byte) asynchronous global -> shared copies, zero-filled past src_bytes.
__device__ __forceinline__ void cp_async16(void *dst, const void *src, uint32_t src_bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(tc_su32(dst)), "l"(src), "r"(src_bytes)
                 : "memory");
}
__device__ __forceinline__ void cp_async4(void *dst, const void *src, uint32_t src_bytes) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(tc_su32(dst)), "l"(src), "r"(src_bytes)
                 : "memory");
}
__device__ __forceinline__ void cp_async8(void *dst, const void *src, uint32_t src_bytes) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 8, %2;" ::"r"(tc_su32(dst)), "l"(src), "r"(src_bytes)
                 : "memory");
}
// The fp16 activation tile of group kb (x = kb * 64, rows m0.. ; rows past T read as zero)
// into an A stage, completing on `bar` (no multicast).
__device__ __forceinline__ void tc_load_a(const CUtensorMap *tmap, void *dst, int kb, int m0, uint64_t *bar) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(tc_su32(bar)), "r"(TC_TILE_BYTES)
                 : "memory");
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
        "[%4];" ::"r"(tc_su32(dst)),
        "l"(reinterpret_cast<uint64_t>(tmap)), "r"(kb * TC_BK), "r"(m0), "r"(tc_su32(bar))
        : "memory");
}
// The weight bytes (128 rows x 64 in fragment order) and (scale, offset) pairs of group kb
// into a raw stage; rows past the weight's rows are zero-filled.
__device__ __forceinline__ void tc_issue_raw_b(const GemmParams &p, uint8_t *raw, int kb, int o0, int rows_alloc) {
    const int tid = threadIdx.x, OUT = p.W.out;
#pragma unroll
    for (int i = 0; i < 2; ++i) {
        const int c = tid + i * TC_THREADS, r = c >> 2, fc = c & 3, o = o0 + r;
        const bool in = o < OUT && o < rows_alloc;
        cp_async16(raw + r * 64 + fc * 16,
                   in ? (const void *)(p.W.tiles + mk_q_offset(p.W, o, kb * TC_BK) + fc * 16) : (const void *)p.W.tiles,
                   in ? 16u : 0u);
    }
    if (tid < TC_BN) {
        const int o = o0 + tid;
        const bool in = o < OUT && o < rows_alloc;
        const void *src = in ? (const void *)(p.W.tiles + mk_sb_offset(p.W, o, kb * TC_BK)) : (const void *)p.W.tiles;
        if (p.W.sbb == 4) cp_async4(raw + TC_RAW_B + tid * 8, src, in ? 4u : 0u);
        else cp_async8(raw + TC_RAW_B + tid * 8, src, in ? 8u : 0u);
    }
}

template <int EPI>
__global__ void __launch_bounds__(TC_THREADS, 1) gemm_q8_tc_kernel(GemmParams p, const __grid_constant__ CUtensorMap tmap_a) {
    extern __shared__ uint8_t tc_smem_raw[];
    __shared__ uint64_t mma_bar[TC_B_STAGES], a_bar[TC_A_STAGES];
    __shared__ uint32_t tmem_base;
    __shared__ float bias_s[TC_BN];  // the tile's output-row biases, read once
    uint8_t *smem = tc_smem_raw + ((1024u - (tc_su32(tc_smem_raw) & 1023u)) & 1023u);
    uint8_t *sA = smem, *sB = smem + TC_OFF_B, *sR = smem + TC_OFF_RAW;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int K = p.W.in, OUT = p.W.out, T = p.T, rows_alloc = p.W.n_rb * 16;
    const int m0 = blockIdx.y * TC_BM, o0 = blockIdx.x * TC_BN;
    const int nkb = K / TC_BK;
    if (tid == 0) {
        for (int s = 0; s < TC_B_STAGES; ++s) asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(tc_su32(&mma_bar[s])));
        for (int s = 0; s < TC_A_STAGES; ++s) asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(tc_su32(&a_bar[s])));
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(tc_su32(&tmem_base)),
                     "r"(TC_TMEM_COLS));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    if (tid < TC_BN) bias_s[tid] = o0 + tid < OUT ? p.W.bias[o0 + tid] : 0.f;
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = tmem_base;
    // prologue: the copies of the first two groups
    int a_issued = 0, a_waited = 0;  // A tiles issued / waited for (meaningful in thread 0)
#pragma unroll 1
    for (int s = 0; s < 2; ++s) {
        if (s < nkb) {
            if (tid == 0) { tc_load_a(&tmap_a, sA + s * TC_TILE_BYTES, s, m0, &a_bar[s]); ++a_issued; }
            tc_issue_raw_b(p, sR + s * TC_RAW_STAGE, s, o0, rows_alloc);
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
    }
    const bool half_sb = p.W.sbb == 4;

    bool ok = true;
    int last = -1;  // last group whose MMAs were committed
    for (int kb = 0; kb < nkb; ++kb) {
        const int bs = kb & 1, as = kb % TC_A_STAGES;
        uint8_t *bt = sB + bs * TC_TILE_BYTES;
        const uint8_t *raw = sR + (kb % TC_RAW_STAGES) * TC_RAW_STAGE;
        // this thread's weight copies of group kb have landed (group kb + 1 may be pending)
        asm volatile("cp.async.wait_group 1;" ::: "memory");
        // the MMAs of group kb - 2 are done: B stage bs and A stage (kb + 2) % 4 are free
        const bool okw = kb < 2 || tc_wait(&mma_bar[bs], (uint32_t)((kb - 2) >> 1) & 1u);
        // every thread's copies of group kb are visible and every thread is done with the raw
        // stage of group kb - 1, which now receives group kb + 2
        __syncthreads();
        if (kb + 2 < nkb) {
            if (tid == 0 && okw) {
                tc_load_a(&tmap_a, sA + ((kb + 2) % TC_A_STAGES) * TC_TILE_BYTES, kb + 2, m0,
                          &a_bar[(kb + 2) % TC_A_STAGES]);
                ++a_issued;
            }
            tc_issue_raw_b(p, sR + ((kb + 2) % TC_RAW_STAGES) * TC_RAW_STAGE, kb + 2, o0, rows_alloc);
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
        if (okw) {
            // weights: a row's group is 4 chunks of 16 bytes in fragment order (chunk c holds
            // inputs 16b + 8hi + 2c + lo), dequantized as s * q + b in fp32, then fp16
#pragma unroll
            for (int i = 0; i < 2; ++i) {
                const int c = tid + i * TC_THREADS, r = c >> 2, fc = c & 3;
                const uint4 w = *reinterpret_cast<const uint4 *>(raw + r * 64 + fc * 16);
                const uint8_t *sbp = raw + TC_RAW_B + r * 8;
                float sc, zo;
                if (half_sb) {
                    const float2 f = __half22float2(*reinterpret_cast<const __half2 *>(sbp));
                    sc = f.x; zo = f.y;
                } else {
                    const float2 f = *reinterpret_cast<const float2 *>(sbp);
                    sc = f.x; zo = f.y;
                }
                const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
                for (int b = 0; b < 4; ++b) {
                    const int k0 = b * 16 + 2 * fc;  // bytes 0, 1 of word b; bytes 2, 3 are k0 + 8, + 9
                    *reinterpret_cast<uint32_t *>(bt + tc_swz(r, k0)) =
                        pack_half2(fmaf(sc, byte_to_float(ww[b], 0), zo), fmaf(sc, byte_to_float(ww[b], 1), zo));
                    *reinterpret_cast<uint32_t *>(bt + tc_swz(r, k0 + 8)) =
                        pack_half2(fmaf(sc, byte_to_float(ww[b], 2), zo), fmaf(sc, byte_to_float(ww[b], 3), zo));
                }
            }
        }
        // make the dequantized weights visible to the tensor core, agree on success, then
        // issue the group's MMAs once its activation tile has landed
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
        ok = __syncthreads_and(okw ? 1 : 0) != 0;
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        if (!ok) break;
        last = kb;
        if (tid == 0) {
            const bool oka = tc_wait(&a_bar[as], (uint32_t)(kb / TC_A_STAGES) & 1u);
            ++a_waited;
            if (oka) {
                const uint32_t at = tc_su32(sA + as * TC_TILE_BYTES), btu = tc_su32(bt);
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    const uint32_t accumulate = (kb > 0 || k > 0) ? 1u : 0u;
                    asm volatile(
                        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
                        " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(tmem),
                        "l"(tc_desc(at + k * 32)), "l"(tc_desc(btu + k * 32)), "r"(TC_IDESC), "r"(accumulate));
                }
                asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                                 tc_su32(&mma_bar[bs]))
                             : "memory");
            }
        }
    }
    // the last committed group's commit covers every MMA issued for the tile (also after a
    // failed wait, so that no MMA still writes the tensor memory when it is freed)
    const bool okl = last < 0 || tc_wait(&mma_bar[last & 1], (uint32_t)(last >> 1) & 1u);
    ok = __syncthreads_and((ok && okl) ? 1 : 0) != 0;
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    if (ok && last == nkb - 1 && nkb > 0) {
        // 1) accumulators TMEM -> shared memory, fp32 [128 rows][TC_STG_LD] over the operand
        //    stages (free now): warp w reads TMEM lanes 32 (w % 4) .. (its 32 rows), columns
        //    64 (w / 4) ..; the 4-float row padding keeps a quarter-warp's 16-byte stores on
        //    distinct banks
        float *stg = reinterpret_cast<float *>(smem);
        {
            const int q = warp & 3, half = warp >> 2, r = q * 32 + lane;
#pragma unroll 1
            for (int cc = 0; cc < 64; cc += 16) {
                uint32_t v[16];
                const uint32_t ta = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(half * 64 + cc);
                asm volatile(
                    "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, "
                    "[%16];"
                    : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
                      "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]),
                      "=r"(v[15])
                    : "r"(ta));
                asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
                float4 *dst = reinterpret_cast<float4 *>(stg + r * TC_STG_LD + half * 64 + cc);
#pragma unroll
                for (int j = 0; j < 4; ++j)
                    dst[j] = make_float4(__uint_as_float(v[4 * j]), __uint_as_float(v[4 * j + 1]),
                                         __uint_as_float(v[4 * j + 2]), __uint_as_float(v[4 * j + 3]));
            }
        }
        __syncthreads();
        // 2) row-wise write-out: warp w finishes rows w, w + 8, ...; lane j columns 4j .. 4j+3,
        //    so a warp's stores (and residual loads) cover whole rows
        const int c0 = 4 * lane, o = o0 + c0;
        const float4 bias4 = make_float4(bias_s[c0], bias_s[c0 + 1], bias_s[c0 + 2], bias_s[c0 + 3]);
        const bool vec = o + 3 < OUT && (OUT & 3) == 0;
#pragma unroll 1
        for (int r = warp; r < TC_BM; r += TC_THREADS / 32) {
            const int t = m0 + r;
            if (t >= T || o >= OUT) continue;
            const float4 a = *reinterpret_cast<const float4 *>(stg + r * TC_STG_LD + c0);
            float v4[4] = {a.x + bias4.x, a.y + bias4.y, a.z + bias4.z, a.w + bias4.w};
            float *yp = p.y + (size_t)t * OUT + o;
            if (EPI == EPI_RESID) {
                if (vec) {
                    const float4 old = *reinterpret_cast<const float4 *>(yp);
                    *reinterpret_cast<float4 *>(yp) = make_float4(old.x + v4[0], old.y + v4[1], old.z + v4[2], old.w + v4[3]);
                } else {
                    for (int j = 0; j < 4 && o + j < OUT; ++j) yp[j] += v4[j];
                }
            } else if (EPI == EPI_GELU) {
                __half *hp = reinterpret_cast<__half *>(p.y) + (size_t)t * OUT + o;
                if (vec) {
                    uint2 hv;
                    hv.x = pack_half2(gelu_tanh(v4[0]), gelu_tanh(v4[1]));
                    hv.y = pack_half2(gelu_tanh(v4[2]), gelu_tanh(v4[3]));
                    *reinterpret_cast<uint2 *>(hp) = hv;
                } else {
                    for (int j = 0; j < 4 && o + j < OUT; ++j) hp[j] = __float2half_rn(gelu_tanh(v4[j]));
                }
            } else {
                if (vec) *reinterpret_cast<float4 *>(yp) = make_float4(v4[0], v4[1], v4[2], v4[3]);
                else
                    for (int j = 0; j < 4 && o + j < OUT; ++j) yp[j] = v4[j];
                if (EPI == EPI_QKV && o >= p.d) {
                    // 4 consecutive dims of one head: 8 contiguous bytes of the cache row
                    const QkvDest qd = qkv_dest(p, t);
                    if (qd.write) {
                        const int rr = o - p.d, which = rr / p.d, oo = rr - which * p.d;
                        __half *cache = which == 0 ? p.k_cache : p.v_cache;
                        uint2 hv;
                        hv.x = pack_half2(v4[0], v4[1]);
                        hv.y = pack_half2(v4[2], v4[3]);
                        *reinterpret_cast<uint2 *>(
                            cache + kv_index(p.layer, qd.slot, oo >> 6, qd.pos, p.n_slots, p.n_heads, p.max_seq) +
                            (oo & 63)) = hv;
                    }
                }
            }
        }
    }
    // teardown: this thread's weight copies have landed, and every activation tile that was
    // issued but not waited for (a loop that stopped early) has landed too
    asm volatile("cp.async.wait_all;" ::: "memory");
    if (tid == 0) {
        for (int i = a_waited; i < a_issued; ++i) tc_wait(&a_bar[i % TC_A_STAGES], (uint32_t)(i / TC_A_STAGES) & 1u);
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    if (warp == 0) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TC_TMEM_COLS));
}

EncodeTiledFn encode_tiled() {
    static std::once_flag once;
    static EncodeTiledFn fn = nullptr;
    std::call_once(once, [] {
        void *f = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(f);
        else
            cudaGetLastError();
    });
    return fn;
}

bool launch_gemm_tc(int epi, const GemmParams &p, cudaStream_t st) {
    const int K = p.W.in;
    // the activation rows must be 16-byte aligned for the tensor map; K a multiple of 64
    if (K % TC_BK != 0 || (reinterpret_cast<uintptr_t>(p.x) & 15) != 0 || p.T <= 0) return false;
    EncodeTiledFn enc = encode_tiled();
    if (!enc) return false;
    CUtensorMap map;
    const cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)p.T};
    const cuuint64_t strides[1] = {(cuuint64_t)K * 2};
    const cuuint32_t box[2] = {(cuuint32_t)TC_BK, (cuuint32_t)TC_BM};
    const cuuint32_t estr[2] = {1, 1};
    if (enc(&map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<__half *>(p.x), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
        return false;
    const dim3 grid((p.W.out + TC_BN - 1) / TC_BN, (p.T + TC_BM - 1) / TC_BM);
    switch (epi) {
    case EPI_PLAIN: gemm_q8_tc_kernel<EPI_PLAIN><<<grid, TC_THREADS, TC_SMEM, st>>>(p, map); break;
    case EPI_GELU: gemm_q8_tc_kernel<EPI_GELU><<<grid, TC_THREADS, TC_SMEM, st>>>(p, map); break;
    case EPI_RESID: gemm_q8_tc_kernel<EPI_RESID><<<grid, TC_THREADS, TC_SMEM, st>>>(p, map); break;
    default: gemm_q8_tc_kernel<EPI_QKV><<<grid, TC_THREADS, TC_SMEM, st>>>(p, map); break;
    }
    return true;
}

// ------------------------------------------------------------------------------
// fp16 weight copies and the fp16 x fp16 GEMM for long prompts (prefill with many rows).
//
// With many rows per weight tile, dequantizing the int8 weights inside every CTA costs
// more than the MMAs (each 128-row tile of the prompt would dequantize the whole weight
// again).  So the weights of a model are dequantized once, exactly as the int8 kernel does
// (s * q + b in fp32, rounded to fp16), into a row-major fp16 copy [out][in], and the
// GEMM streams both operands with TMA:
//  * persistent CTAs (one per SM) walk 128 x 256 output tiles, row tiles fastest, so the
//    CTAs of a wave share one 256-row weight slab in L2;
//  * warp 0 (one thread) issues the TMA copies of A (128 x 64) and B (256 x 64) into a
//    4-stage ring (128-byte swizzle, no multicast); warp 1 (one thread) issues 4
//    tcgen05.mma (K = 16) per stage into one of two 256-column TMEM accumulators and
//    commits each stage back to the ring; warps 2-5 read a finished accumulator with
//    tcgen05.ld (warp w reads TMEM lanes 32 (w % 4) ..) and run the epilogue while the
//    MMAs of the next tile proceed in the other accumulator.
// Every wait is bounded; on expiry the kernel records an error and the roles stop.
// ------------------------------------------------------------------------------
constexpr int HB_BM = 128, HB_BN = 256, HB_BK = 64, HB_STAGES = 4, HB_THREADS = 192;
constexpr int HB_A_BYTES = HB_BM * HB_BK * 2, HB_B_BYTES = HB_BN * HB_BK * 2;
constexpr int HB_STAGE = HB_A_BYTES + HB_B_BYTES;
constexpr int HB_SMEM = HB_STAGES * HB_STAGE + 1024;
constexpr uint32_t HB_TMEM_COLS = 512;  // two accumulators of 256 fp32 columns
// instruction descriptor (kind::f16): D f32, A and B f16, both K-major, N = 256, M = 128
constexpr uint32_t HB_IDESC = (1u << 4) | ((uint32_t)(HB_BN >> 3) << 17) | ((uint32_t)(HB_BM >> 4) << 24);

__device__ __forceinline__ void hb_arrive_expect(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(tc_su32(bar)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void hb_tma(const CUtensorMap *map, void *dst, int x, int y, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
        "[%4];" ::"r"(tc_su32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(tc_su32(bar))
        : "memory");
}
__device__ __forceinline__ void hb_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(tc_su32(bar))
                 : "memory");
}

template <int EPI>
__global__ void __launch_bounds__(HB_THREADS, 1)
    gemm_f16_tc_kernel(GemmParams p, const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b) {
    extern __shared__ uint8_t hb_smem_raw[];
    __shared__ uint64_t full[HB_STAGES], empty[HB_STAGES], acc_full[2], acc_empty[2], mma_done;
    __shared__ uint32_t tmem_base;
    __shared__ int stop;
    uint8_t *smem = hb_smem_raw + ((1024u - (tc_su32(hb_smem_raw) & 1023u)) & 1023u);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int K = p.W.in, OUT = p.W.out, T = p.T;
    const int ks = p.ksplit > 1 ? p.ksplit : 1;  // K splits (tile index / (mt * ntile))
    const int mt = (T + HB_BM - 1) / HB_BM, ntile = (OUT + HB_BN - 1) / HB_BN, tiles = mt * ntile * ks, nk = K / HB_BK;
    // tile -> row tile m (fastest), column tile n, K split ksp covering k blocks [kb0, kb1)
    auto tile_of = [&](int tile, int &m0, int &n0, int &kb0, int &kb1, int &ksp) {
        const int mn = tile % (mt * ntile);
        ksp = tile / (mt * ntile);
        m0 = (mn % mt) * HB_BM;
        n0 = (mn / mt) * HB_BN;
        kb0 = ksp * nk / ks;
        kb1 = (ksp + 1) * nk / ks;
    };
    if (tid == 0) {
        for (int s = 0; s < HB_STAGES; ++s) {
            asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(tc_su32(&full[s])));
            asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(tc_su32(&empty[s])));
        }
        for (int b = 0; b < 2; ++b) {
            asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(tc_su32(&acc_full[b])));
            asm volatile("mbarrier.init.shared::cta.b64 [%0], 128;" ::"r"(tc_su32(&acc_empty[b])));
        }
        asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(tc_su32(&mma_done)));
        stop = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(tc_su32(&tmem_base)),
                     "r"(HB_TMEM_COLS));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = tmem_base;
    volatile int *vstop = &stop;

    if (warp == 0) {
        if (lane == 0) {  // ---- TMA producer ----
            int stage = 0, it = 0;
            uint32_t phase = 0;
            for (int tile = blockIdx.x; tile < tiles && !*vstop; tile += gridDim.x) {
                int m0, n0, kb0, kb1, ksp;
                tile_of(tile, m0, n0, kb0, kb1, ksp);
                for (int kb = kb0; kb < kb1; ++kb) {
                    if (it >= HB_STAGES && !tc_wait(&empty[stage], phase ^ 1u)) { *vstop = 1; break; }
                    uint8_t *st = smem + stage * HB_STAGE;
                    hb_arrive_expect(&full[stage], HB_STAGE);
                    hb_tma(&tmap_a, st, kb * HB_BK, m0, &full[stage]);
                    hb_tma(&tmap_b, st + HB_A_BYTES, kb * HB_BK, n0, &full[stage]);
                    ++it;
                    if (++stage == HB_STAGES) { stage = 0; phase ^= 1u; }
                }
            }
            // the copies in flight land before the CTA may exit: the last HB_STAGES stages
            for (int i = 0; i < HB_STAGES && i < it; ++i) {
                const int k = it - 1 - i, s2 = k % HB_STAGES;
                tc_wait(&full[s2], (uint32_t)(k / HB_STAGES) & 1u);
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {  // ---- MMA issuer ----
            int stage = 0, tl = 0;
            uint32_t phase = 0;
            for (int tile = blockIdx.x; tile < tiles && !*vstop; tile += gridDim.x, ++tl) {
                const int ab = tl & 1;
                if (tl >= 2 && !tc_wait(&acc_empty[ab], (uint32_t)((tl >> 1) - 1) & 1u)) { *vstop = 1; break; }
                asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                const uint32_t acc = tmem + (uint32_t)(ab * HB_BN);
                int m0, n0, kb0, kb1, ksp;
                tile_of(tile, m0, n0, kb0, kb1, ksp);
                bool okt = true;
                for (int kb = kb0; kb < kb1; ++kb) {
                    if (!tc_wait(&full[stage], phase)) { okt = false; break; }
                    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                    const uint32_t at = tc_su32(smem + stage * HB_STAGE), bt = at + HB_A_BYTES;
#pragma unroll
                    for (int k = 0; k < 4; ++k) {
                        const uint32_t accumulate = (kb > kb0 || k > 0) ? 1u : 0u;
                        asm volatile(
                            "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
                            " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(acc),
                            "l"(tc_desc(at + k * 32)), "l"(tc_desc(bt + k * 32)), "r"(HB_IDESC), "r"(accumulate));
                    }
                    hb_commit(&empty[stage]);  // the stage is free once these MMAs are done
                    if (++stage == HB_STAGES) { stage = 0; phase ^= 1u; }
                }
                hb_commit(&acc_full[ab]);  // the accumulator is final once every MMA is done
                if (!okt) { *vstop = 1; break; }
            }
            // no MMA may still write the tensor memory when it is freed
            hb_commit(&mma_done);
            tc_wait(&mma_done, 0);
        }
    } else {  // ---- epilogue: warps 2..5 ----
        const int q = warp & 3, r = q * 32 + lane;
        int tl = 0;
        for (int tile = blockIdx.x; tile < tiles && !*vstop; tile += gridDim.x, ++tl) {
            const int ab = tl & 1;
            const bool okw = tc_wait(&acc_full[ab], (uint32_t)(tl >> 1) & 1u);
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            if (!okw || *vstop) { *vstop = 1; break; }
            int m0, n0, kb0, kb1, ksp;
            tile_of(tile, m0, n0, kb0, kb1, ksp);
            const int t = m0 + r;
            const QkvDest qd = EPI == EPI_QKV && t < T && ks == 1 ? qkv_dest(p, t) : QkvDest{0, 0, false};
#pragma unroll 1
            for (int cc = 0; cc < HB_BN; cc += 16) {
                uint32_t v[16];
                const uint32_t ta = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(ab * HB_BN + cc);
                asm volatile(
                    "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, "
                    "[%16];"
                    : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
                      "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]),
                      "=r"(v[15])
                    : "r"(ta));
                asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
                const int o = n0 + cc;
                if (t >= T || o >= OUT) continue;
                if (ks > 1) {  // split K: this split's partial sums (no bias), finished by gemm_splitk_epilogue
                    float *wp = p.ws + ((size_t)ksp * T + t) * OUT + o;
                    if (o + 16 <= OUT && (OUT & 3) == 0) {
#pragma unroll
                        for (int j = 0; j < 16; j += 4)
                            *reinterpret_cast<float4 *>(wp + j) =
                                make_float4(__uint_as_float(v[j]), __uint_as_float(v[j + 1]), __uint_as_float(v[j + 2]),
                                            __uint_as_float(v[j + 3]));
                    } else {
                        for (int j = 0; j < 16 && o + j < OUT; ++j) wp[j] = __uint_as_float(v[j]);
                    }
                    continue;
                }
                float f[16];
#pragma unroll
                for (int j = 0; j < 16; ++j) f[j] = __uint_as_float(v[j]) + (o + j < OUT ? __ldg(p.W.bias + o + j) : 0.f);
                const bool full16 = o + 16 <= OUT && (OUT & 3) == 0;
                float *yp = p.y + (size_t)t * OUT + o;
                if (EPI == EPI_GELU) {
                    __half *hp = reinterpret_cast<__half *>(p.y) + (size_t)t * OUT + o;
                    if (full16 && (OUT & 7) == 0) {
#pragma unroll
                        for (int j = 0; j < 16; j += 8) {
                            uint4 hv;
                            hv.x = pack_half2(gelu_tanh(f[j]), gelu_tanh(f[j + 1]));
                            hv.y = pack_half2(gelu_tanh(f[j + 2]), gelu_tanh(f[j + 3]));
                            hv.z = pack_half2(gelu_tanh(f[j + 4]), gelu_tanh(f[j + 5]));
                            hv.w = pack_half2(gelu_tanh(f[j + 6]), gelu_tanh(f[j + 7]));
                            *reinterpret_cast<uint4 *>(hp + j) = hv;
                        }
                    } else {
                        for (int j = 0; j < 16 && o + j < OUT; ++j) hp[j] = __float2half_rn(gelu_tanh(f[j]));
                    }
                } else if (EPI == EPI_RESID) {
                    if (full16) {
#pragma unroll
                        for (int j = 0; j < 16; j += 4) {
                            const float4 old = *reinterpret_cast<const float4 *>(yp + j);
                            *reinterpret_cast<float4 *>(yp + j) =
                                make_float4(old.x + f[j], old.y + f[j + 1], old.z + f[j + 2], old.w + f[j + 3]);
                        }
                    } else {
                        for (int j = 0; j < 16 && o + j < OUT; ++j) yp[j] += f[j];
                    }
                } else {
                    if (full16) {
#pragma unroll
                        for (int j = 0; j < 16; j += 4)
                            *reinterpret_cast<float4 *>(yp + j) = make_float4(f[j], f[j + 1], f[j + 2], f[j + 3]);
                    } else {
                        for (int j = 0; j < 16 && o + j < OUT; ++j) yp[j] = f[j];
                    }
                    if (EPI == EPI_QKV && o >= p.d && qd.write) {
                        // 16 consecutive dims of one head: 32 contiguous bytes of the cache row
                        const int rr = o - p.d, which = rr / p.d, oo = rr - which * p.d;
                        __half *cache = (which == 0 ? p.k_cache : p.v_cache) +
                                        kv_index(p.layer, qd.slot, oo >> 6, qd.pos, p.n_slots, p.n_heads, p.max_seq) +
                                        (oo & 63);
#pragma unroll
                        for (int j = 0; j < 16; j += 8) {
                            uint4 hv;
                            hv.x = pack_half2(f[j], f[j + 1]);
                            hv.y = pack_half2(f[j + 2], f[j + 3]);
                            hv.z = pack_half2(f[j + 4], f[j + 5]);
                            hv.w = pack_half2(f[j + 6], f[j + 7]);
                            *reinterpret_cast<uint4 *>(cache + j) = hv;
                        }
                    }
                }
            }
            asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
            asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(tc_su32(&acc_empty[ab])) : "memory");
        }
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    if (warp == 1) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(HB_TMEM_COLS));
}

// The epilogue of a split-K fp16 GEMM: y[t, o] = sum of the splits' partials (in split
// order) + bias[o], stored per epilogue (gemm_store); one thread per output.
template <int EPI>
__global__ void gemm_splitk_epilogue(GemmParams p) {
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    const int OUT = p.W.out;
    if (i >= (size_t)p.T * OUT) return;
    const int t = (int)(i / OUT), o = (int)(i - (size_t)t * OUT);
    float v = 0.f;
    for (int s = 0; s < p.ksplit; ++s) v += p.ws[(size_t)s * p.T * OUT + i];
    v += p.W.bias[o];
    const QkvDest qd = EPI == EPI_QKV ? qkv_dest(p, t) : QkvDest{0, 0, false};
    gemm_store<EPI>(p, t, o, v, qd);
}

// fp16 copy of a tiled int8 linear: w16[o][k] = fp16(s * q + b), the value the int8
// GEMMs compute in registers or shared memory (rows past `out` are not written).
__global__ void dequant_f16_kernel(MkLin W, __half *w16) {
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;  // one thread per 8 inputs
    const int per = W.in / 8;
    if (i >= (size_t)W.out * per) return;
    const int o = (int)(i / per), k0 = (int)(i - (size_t)o * per) * 8;
    const uint8_t *sb = W.tiles + mk_sb_offset(W, o, k0);
    float sc, zo;
    if (W.sbb == 4) {
        const float2 f = __half22float2(*reinterpret_cast<const __half2 *>(sb));
        sc = f.x; zo = f.y;
    } else {
        const float2 f = *reinterpret_cast<const float2 *>(sb);
        sc = f.x; zo = f.y;
    }
    uint32_t hv[4];
#pragma unroll
    for (int j = 0; j < 8; j += 2) {
        const float a = fmaf(sc, (float)W.tiles[mk_q_offset(W, o, k0 + j)], zo);
        const float b = fmaf(sc, (float)W.tiles[mk_q_offset(W, o, k0 + j + 1)], zo);
        hv[j / 2] = pack_half2(a, b);
    }
    *reinterpret_cast<uint4 *>(w16 + (size_t)o * W.in + k0) = make_uint4(hv[0], hv[1], hv[2], hv[3]);
}

cudaError_t make_weights_f16(const MkLin &W, __half *w16, cudaStream_t st) {
    const size_t n = (size_t)W.out * (W.in / 8);
    dequant_f16_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(W, w16);
    return cudaGetLastError();
}

bool launch_gemm_f16(int epi, const GemmParams &p, const __half *w16, cudaStream_t st) {
    const int K = p.W.in;
    if (!w16 || K % HB_BK != 0 || (reinterpret_cast<uintptr_t>(p.x) & 15) != 0 ||
        (reinterpret_cast<uintptr_t>(w16) & 15) != 0 || p.T <= 0)
        return false;
    EncodeTiledFn enc = encode_tiled();
    if (!enc) return false;
    CUtensorMap ma, mb;
    const cuuint32_t estr[2] = {1, 1};
    {
        const cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)p.T};
        const cuuint64_t strides[1] = {(cuuint64_t)K * 2};
        const cuuint32_t box[2] = {(cuuint32_t)HB_BK, (cuuint32_t)HB_BM};
        if (enc(&ma, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<__half *>(p.x), dims, strides, box, estr,
                CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return false;
    }
    {
        const cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)p.W.out};
        const cuuint64_t strides[1] = {(cuuint64_t)K * 2};
        const cuuint32_t box[2] = {(cuuint32_t)HB_BK, (cuuint32_t)HB_BN};
        if (enc(&mb, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<__half *>(w16), dims, strides, box, estr,
                CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return false;
    }
    int dev = 0, sms = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    GemmParams q = p;
    const int tiles = ((p.T + HB_BM - 1) / HB_BM) * ((p.W.out + HB_BN - 1) / HB_BN);
    // few output tiles (a decode step of many columns): split K so that every SM streams
    // part of the weights; the partial sums meet in the workspace
    q.ksplit = 1;
    if (tiles < sms && p.ws && p.ws_splits > 1)
        q.ksplit = std::min({(sms + tiles - 1) / tiles, K / HB_BK, p.ws_splits});
    const dim3 grid((unsigned)std::min(tiles * q.ksplit, sms));
    switch (epi) {
    case EPI_PLAIN: gemm_f16_tc_kernel<EPI_PLAIN><<<grid, HB_THREADS, HB_SMEM, st>>>(q, ma, mb); break;
    case EPI_GELU: gemm_f16_tc_kernel<EPI_GELU><<<grid, HB_THREADS, HB_SMEM, st>>>(q, ma, mb); break;
    case EPI_RESID: gemm_f16_tc_kernel<EPI_RESID><<<grid, HB_THREADS, HB_SMEM, st>>>(q, ma, mb); break;
    default: gemm_f16_tc_kernel<EPI_QKV><<<grid, HB_THREADS, HB_SMEM, st>>>(q, ma, mb); break;
    }
    if (q.ksplit > 1) {
        const unsigned blocks = (unsigned)(((size_t)p.T * p.W.out + 255) / 256);
        switch (epi) {
        case EPI_PLAIN: gemm_splitk_epilogue<EPI_PLAIN><<<blocks, 256, 0, st>>>(q); break;
        case EPI_GELU: gemm_splitk_epilogue<EPI_GELU><<<blocks, 256, 0, st>>>(q); break;
        case EPI_RESID: gemm_splitk_epilogue<EPI_RESID><<<blocks, 256, 0, st>>>(q); break;
        default: gemm_splitk_epilogue<EPI_QKV><<<blocks, 256, 0, st>>>(q); break;
        }
    }
    return true;
}

void kernels_init_gemm_tc() {
    cudaFuncSetAttribute(gemm_f16_tc_kernel<EPI_PLAIN>, cudaFuncAttributeMaxDynamicSharedMemorySize, HB_SMEM);
    cudaFuncSetAttribute(gemm_f16_tc_kernel<EPI_GELU>, cudaFuncAttributeMaxDynamicSharedMemorySize, HB_SMEM);
    cudaFuncSetAttribute(gemm_f16_tc_kernel<EPI_RESID>, cudaFuncAttributeMaxDynamicSharedMemorySize, HB_SMEM);
    cudaFuncSetAttribute(gemm_f16_tc_kernel<EPI_QKV>, cudaFuncAttributeMaxDynamicSharedMemorySize, HB_SMEM);
    cudaFuncSetAttribute(gemm_q8_tc_kernel<EPI_PLAIN>, cudaFuncAttributeMaxDynamicSharedMemorySize, TC_SMEM);
    cudaFuncSetAttribute(gemm_q8_tc_kernel<EPI_GELU>, cudaFuncAttributeMaxDynamicSharedMemorySize, TC_SMEM);
    cudaFuncSetAttribute(gemm_q8_tc_kernel<EPI_RESID>, cudaFuncAttributeMaxDynamicSharedMemorySize, TC_SMEM);
    cudaFuncSetAttribute(gemm_q8_tc_kernel<EPI_QKV>, cudaFuncAttributeMaxDynamicSharedMemorySize, TC_SMEM);
    encode_tiled();
}

}  // namespace itts
