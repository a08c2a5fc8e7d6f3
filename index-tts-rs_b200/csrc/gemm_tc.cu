// gemm_tc.cu -- the int8-weight GEMM on the 5th-generation tensor cores (tcgen05), used by
// prefill and by decode steps with more columns than the persistent kernel takes:
// y[t, o] = x[t, :] . W[o, :] + bias[o] with the plain / GELU / residual / QKV epilogues
// (crates/core/src/models/gpt.rs:252-264 QuantizedLinear::forward inside Gpt2Block).
//
// One CTA computes a 128-row (positions) x 128-column (weight rows) tile with an fp32
// accumulator in tensor memory.  The K loop runs over the 64-input quantization groups:
// the 8 warps stage the group's activations (fp32 -> fp16) and its weights (int8 ->
// s * q + b in fp32 -> fp16) into shared memory in the 128-byte-swizzled K-major layout
// the MMA reads, and one thread issues the 4 tcgen05.mma (K = 16 each) of the group and
// commits them to the stage's mbarrier.  Two stages: the next group is staged while the
// tensor core runs the current one.  Every wait is bounded; on expiry the kernel records
// an error, skips the rest, frees its tensor memory and returns.
#include "gemm.cuh"

namespace itts {

constexpr int TC_BM = 128, TC_BN = 128, TC_BK = 64, TC_THREADS = 256;
constexpr int TC_TILE_BYTES = TC_BM * TC_BK * 2;  // one operand of one stage: 16 KB
constexpr int TC_SMEM = 2 * 2 * TC_TILE_BYTES + 1024;
constexpr uint32_t TC_TMEM_COLS = 128;
constexpr long TC_SPIN = 1L << 24;
// instruction descriptor (kind::f16): D f32, A and B f16, both K-major, N = 128, M = 128
constexpr uint32_t TC_IDESC = (1u << 4) | ((uint32_t)(TC_BN >> 3) << 17) | ((uint32_t)(TC_BM >> 4) << 24);

__device__ int g_gemm_tc_error;  // nonzero once a bounded wait gave up

__device__ __forceinline__ uint32_t tc_su32(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }

// Byte offset of element (r, k), k < 64, in a K-major tile of 64 fp16 per row with the
// 128-byte swizzle: 8-row groups of 1024 B; in row r the 16-byte chunk k/8 sits at chunk
// position (k/8) ^ (r % 8).
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

template <int EPI>
__global__ void __launch_bounds__(TC_THREADS, 1) gemm_q8_tc_kernel(GemmParams p) {
    extern __shared__ uint8_t tc_smem_raw[];
    __shared__ uint64_t bar[2];
    __shared__ uint32_t tmem_base;
    uint8_t *smem = tc_smem_raw + ((1024u - (tc_su32(tc_smem_raw) & 1023u)) & 1023u);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int K = p.W.in, OUT = p.W.out, T = p.T, rows_alloc = p.W.n_rb * 16;
    const int m0 = blockIdx.y * TC_BM, o0 = blockIdx.x * TC_BN;
    const int nkb = K / TC_BK;
    if (tid == 0) {
        asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(tc_su32(&bar[0])));
        asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(tc_su32(&bar[1])));
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(tc_su32(&tmem_base)),
                     "r"(TC_TMEM_COLS));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = tmem_base;
    const bool half_sb = p.W.sbb == 4;

    bool ok = true;
    int last = -1;  // last group whose MMAs were committed
    for (int kb = 0; kb < nkb; ++kb) {
        const int s = kb & 1;
        uint8_t *sa = smem + s * 2 * TC_TILE_BYTES, *sb = sa + TC_TILE_BYTES;
        // the MMAs of group kb - 2 read this stage: wait for them before overwriting it
        const bool okw = kb < 2 || tc_wait(&bar[s], (uint32_t)((kb - 2) >> 1) & 1u);
        if (okw) {
            // activations: 128 positions x 64 inputs, 8 per 16-byte chunk
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const int c = tid + i * TC_THREADS, r = c >> 3, ch = c & 7, t = m0 + r;
                uint4 h = make_uint4(0u, 0u, 0u, 0u);
                if (t < T) {
                    const float *src = p.x + (size_t)t * K + kb * TC_BK + ch * 8;
                    const float4 a = *reinterpret_cast<const float4 *>(src);
                    const float4 b = *reinterpret_cast<const float4 *>(src + 4);
                    h = make_uint4(pack_half2(a.x, a.y), pack_half2(a.z, a.w), pack_half2(b.x, b.y), pack_half2(b.z, b.w));
                }
                *reinterpret_cast<uint4 *>(sa + tc_swz(r, ch * 8)) = h;
            }
            // weights: 128 rows x 64 inputs; a row's group is 4 chunks of 16 bytes in fragment
            // order (chunk c holds inputs 16b + 8hi + 2c + lo), dequantized as s * q + b
#pragma unroll
            for (int i = 0; i < 2; ++i) {
                const int c = tid + i * TC_THREADS, r = c >> 2, fc = c & 3, o = o0 + r;
                uint32_t hv[8];
                if (o < OUT && o < rows_alloc) {
                    const uint4 w = ld_stream(p.W.tiles + mk_q_offset(p.W, o, kb * TC_BK) + fc * 16);
                    const uint8_t *sbp = p.W.tiles + mk_sb_offset(p.W, o, kb * TC_BK);
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
                        hv[2 * b] = pack_half2(fmaf(sc, byte_to_float(ww[b], 0), zo), fmaf(sc, byte_to_float(ww[b], 1), zo));
                        hv[2 * b + 1] =
                            pack_half2(fmaf(sc, byte_to_float(ww[b], 2), zo), fmaf(sc, byte_to_float(ww[b], 3), zo));
                    }
                } else {
#pragma unroll
                    for (int e = 0; e < 8; ++e) hv[e] = 0u;
                }
#pragma unroll
                for (int b = 0; b < 4; ++b) {
                    const int k0 = b * 16 + 2 * fc;  // bytes 0, 1 of word b
                    *reinterpret_cast<uint32_t *>(sb + tc_swz(r, k0)) = hv[2 * b];
                    *reinterpret_cast<uint32_t *>(sb + tc_swz(r, k0 + 8)) = hv[2 * b + 1];  // bytes 2, 3
                }
            }
        }
        // make the staged tiles visible to the tensor core, agree on success, then issue
        // the group's MMAs
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
        ok = __syncthreads_and(okw ? 1 : 0) != 0;
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        if (!ok) break;
        last = kb;
        if (tid == 0) {
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const uint64_t da = tc_desc(tc_su32(sa) + k * 32), db = tc_desc(tc_su32(sb) + k * 32);
                const uint32_t accumulate = (kb > 0 || k > 0) ? 1u : 0u;
                asm volatile(
                    "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
                    " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(tmem),
                    "l"(da), "l"(db), "r"(TC_IDESC), "r"(accumulate));
            }
            asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                             tc_su32(&bar[s]))
                         : "memory");
        }
    }
    // the last committed group's commit covers every MMA issued for the tile (also after a
    // failed wait, so that no MMA still writes the tensor memory when it is freed)
    const bool okl = last < 0 || tc_wait(&bar[last & 1], (uint32_t)(last >> 1) & 1u);
    ok = __syncthreads_and((ok && okl) ? 1 : 0) != 0;
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    if (ok && last == nkb - 1 && nkb > 0) {
        // warp w reads TMEM lanes 32 (w % 4) .. (its 32 positions), columns 64 (w / 4) ..
        const int q = warp & 3, half = warp >> 2, t = m0 + q * 32 + lane;
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
            if (t < T) {
#pragma unroll
                for (int j = 0; j < 16; ++j) {
                    const int o = o0 + half * 64 + cc + j;
                    if (o < OUT) gemm_store<EPI>(p, t, o, __uint_as_float(v[j]) + p.W.bias[o]);
                }
            }
        }
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    if (warp == 0) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TC_TMEM_COLS));
}

void launch_gemm_tc(int epi, const GemmParams &p, cudaStream_t st) {
    const dim3 grid((p.W.out + TC_BN - 1) / TC_BN, (p.T + TC_BM - 1) / TC_BM);
    switch (epi) {
    case EPI_PLAIN: gemm_q8_tc_kernel<EPI_PLAIN><<<grid, TC_THREADS, TC_SMEM, st>>>(p); break;
    case EPI_GELU: gemm_q8_tc_kernel<EPI_GELU><<<grid, TC_THREADS, TC_SMEM, st>>>(p); break;
    case EPI_RESID: gemm_q8_tc_kernel<EPI_RESID><<<grid, TC_THREADS, TC_SMEM, st>>>(p); break;
    default: gemm_q8_tc_kernel<EPI_QKV><<<grid, TC_THREADS, TC_SMEM, st>>>(p); break;
    }
}

void kernels_init_gemm_tc() {
    cudaFuncSetAttribute(gemm_q8_tc_kernel<EPI_PLAIN>, cudaFuncAttributeMaxDynamicSharedMemorySize, TC_SMEM);
    cudaFuncSetAttribute(gemm_q8_tc_kernel<EPI_GELU>, cudaFuncAttributeMaxDynamicSharedMemorySize, TC_SMEM);
    cudaFuncSetAttribute(gemm_q8_tc_kernel<EPI_RESID>, cudaFuncAttributeMaxDynamicSharedMemorySize, TC_SMEM);
    cudaFuncSetAttribute(gemm_q8_tc_kernel<EPI_QKV>, cudaFuncAttributeMaxDynamicSharedMemorySize, TC_SMEM);
}

}  // namespace itts
