// prefill_batch.cu -- prefill of several requests at once (the batched prompt path of
// generate_codes_after, crates/core/src/models/sampler.rs:340-392, for each request of a
// batch; Gpt::prefill_after, crates/core/src/models/gpt.rs:655-696).
//
// The requests' positions are packed into one row range: LayerNorm and the four linears
// of every layer run once over all rows (the int8 tcgen05 GEMM, M = total positions), the
// QKV epilogue writes each row's K/V into its own request's cache slot, and a causal
// flash attention on the tensor cores (mma.sync m16n8k16, fp16 operands, fp32 softmax and
// accumulation) attends within each request over its cache slot.  The head runs on each
// request's last row.
#include "gemm.cuh"

namespace itts {

// ---------------------------------------------------------------------------
// Causal attention of one 64-query tile of one request and one head (4 warps, 16 query
// rows each) over the request's cached keys 0..q: Q from the QKV output (fp32 -> fp16,
// pre-scaled by 0.125 * log2 e), K/V tiles of 64 positions from the fp16 cache into
// padded shared memory (144-byte rows: ldmatrix rows fall on distinct banks), online
// softmax in fp32 with exp2.
// ---------------------------------------------------------------------------
constexpr int FA_ROW = 72;  // halves per shared-memory row (64 + 8 padding)

__device__ __forceinline__ void fa_mma(float *d, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                       uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void fa_ldm4(uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3, const __half *p) {
    const uint32_t a = (uint32_t)__cvta_generic_to_shared(p);
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(a));
}
__device__ __forceinline__ void fa_ldm4t(uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3, const __half *p) {
    const uint32_t a = (uint32_t)__cvta_generic_to_shared(p);
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(a));
}
__device__ __forceinline__ uint32_t fa_pack(float lo, float hi) {
    const __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<const uint32_t *>(&h);
}
__device__ __forceinline__ void fa_cp16(__half *dst, const __half *src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"((uint32_t)__cvta_generic_to_shared(dst)),
                 "l"(src)
                 : "memory");
}

// tiles == null: one request of T1 positions in slot1 at row 0, tile blockIdx.x
__global__ void __launch_bounds__(128) attn_prefill_fa_kernel(const float *qkv, const AttnTile *tiles, int T1,
                                                              int slot1, const __half *kc, const __half *vc,
                                                              int layer, int n_slots, int H, int max_seq, int d,
                                                              __half *out) {
    __shared__ __align__(16) __half Ks[64 * FA_ROW];
    __shared__ __align__(16) __half Vs[64 * FA_ROW];
    const AttnTile tl = tiles ? tiles[blockIdx.x] : AttnTile{0, (int)blockIdx.x * 64, T1, slot1};
    const int h = blockIdx.y, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, c = lane & 3;
    const int T = tl.T, q0 = tl.q0;
    const int qa_row = q0 + warp * 16 + g, qb_row = qa_row + 8;  // this thread's two query rows
    const float qscale = 0.125f * 1.4426950408889634f;            // attention scale x log2(e)
    // Q fragments (A operand) of the 4 k16 steps over the head's 64 dims
    uint32_t qa[4][4];
    {
        const float *ra = qkv + (size_t)(tl.row0 + min(qa_row, T - 1)) * 3 * d + h * 64;
        const float *rb = qkv + (size_t)(tl.row0 + min(qb_row, T - 1)) * 3 * d + h * 64;
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
            const int e = kk * 16 + 2 * c;
            const float2 a0 = *reinterpret_cast<const float2 *>(ra + e), a1 = *reinterpret_cast<const float2 *>(rb + e);
            const float2 a2 = *reinterpret_cast<const float2 *>(ra + e + 8), a3 = *reinterpret_cast<const float2 *>(rb + e + 8);
            qa[kk][0] = fa_pack(a0.x * qscale, a0.y * qscale);
            qa[kk][1] = fa_pack(a1.x * qscale, a1.y * qscale);
            qa[kk][2] = fa_pack(a2.x * qscale, a2.y * qscale);
            qa[kk][3] = fa_pack(a3.x * qscale, a3.y * qscale);
        }
    }
    float o[8][4];
#pragma unroll
    for (int i = 0; i < 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
    float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
    const int last = min(T - 1, q0 + 63);
    const size_t head_base = kv_index(layer, tl.slot, h, 0, n_slots, H, max_seq);
    for (int k0 = 0; k0 <= last; k0 += 64) {
        __syncthreads();  // the previous tile is consumed
        // 64 positions x 8 chunks of 16 B for K and for V; positions past T are clamped
        // (in bounds of the slot, masked below)
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int ch = tid + i * 128, r = ch >> 3, cc = ch & 7;
            const size_t src = head_base + (size_t)min(k0 + r, T - 1) * 64 + cc * 8;
            fa_cp16(Ks + r * FA_ROW + cc * 8, kc + src);
            fa_cp16(Vs + r * FA_ROW + cc * 8, vc + src);
        }
        asm volatile("cp.async.commit_group;\ncp.async.wait_group 0;" ::: "memory");
        __syncthreads();
        // S = Q K^T for 64 keys (8 n8 tiles)
        float s[8][4];
#pragma unroll
        for (int i = 0; i < 8; ++i) s[i][0] = s[i][1] = s[i][2] = s[i][3] = 0.f;
        const int mi = lane >> 3, ri = lane & 7;
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
#pragma unroll
            for (int nt = 0; nt < 8; nt += 2) {
                uint32_t b0, b1, b2, b3;
                fa_ldm4(b0, b1, b2, b3, Ks + ((nt + (mi >> 1)) * 8 + ri) * FA_ROW + kk * 16 + (mi & 1) * 8);
                fa_mma(s[nt], qa[kk][0], qa[kk][1], qa[kk][2], qa[kk][3], b0, b1);
                fa_mma(s[nt + 1], qa[kk][0], qa[kk][1], qa[kk][2], qa[kk][3], b2, b3);
            }
        // causal mask (key > query), then the online softmax of rows qa_row and qb_row
        if (k0 + 63 > q0 + warp * 16) {
#pragma unroll
            for (int nt = 0; nt < 8; ++nt)
#pragma unroll
                for (int e = 0; e < 2; ++e) {
                    const int key = k0 + nt * 8 + 2 * c + e;
                    if (key > qa_row) s[nt][e] = -INFINITY;
                    if (key > qb_row) s[nt][2 + e] = -INFINITY;
                }
        }
        float mx0 = m0, mx1 = m1;
#pragma unroll
        for (int nt = 0; nt < 8; ++nt) {
            mx0 = fmaxf(mx0, fmaxf(s[nt][0], s[nt][1]));
            mx1 = fmaxf(mx1, fmaxf(s[nt][2], s[nt][3]));
        }
#pragma unroll
        for (int off = 1; off < 4; off <<= 1) {
            mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, off));
            mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, off));
        }
        // key 0 <= query always, so the running maxima are finite from the first tile on
        const float c0 = exp2f(m0 - mx0), c1 = exp2f(m1 - mx1);
        m0 = mx0;
        m1 = mx1;
        l0 *= c0;
        l1 *= c1;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            o[i][0] *= c0; o[i][1] *= c0; o[i][2] *= c1; o[i][3] *= c1;
        }
        uint32_t pa[4][4];  // P as the A operand of the 4 k16 steps over the 64 keys
#pragma unroll
        for (int nt = 0; nt < 8; ++nt) {
            const float p0 = exp2f(s[nt][0] - m0), p1 = exp2f(s[nt][1] - m0);
            const float p2 = exp2f(s[nt][2] - m1), p3 = exp2f(s[nt][3] - m1);
            l0 += p0 + p1;
            l1 += p2 + p3;
            pa[nt >> 1][(nt & 1) * 2] = fa_pack(p0, p1);
            pa[nt >> 1][(nt & 1) * 2 + 1] = fa_pack(p2, p3);
        }
        // O += P V: V tiles read transposed by ldmatrix
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
#pragma unroll
            for (int dt = 0; dt < 8; dt += 2) {
                uint32_t b0, b1, b2, b3;
                fa_ldm4t(b0, b1, b2, b3, Vs + (kk * 16 + (mi & 1) * 8 + ri) * FA_ROW + (dt + (mi >> 1)) * 8);
                fa_mma(o[dt], pa[kk][0], pa[kk][1], pa[kk][2], pa[kk][3], b0, b1);
                fa_mma(o[dt + 1], pa[kk][0], pa[kk][1], pa[kk][2], pa[kk][3], b2, b3);
            }
    }
#pragma unroll
    for (int off = 1; off < 4; off <<= 1) {
        l0 += __shfl_xor_sync(0xffffffffu, l0, off);
        l1 += __shfl_xor_sync(0xffffffffu, l1, off);
    }
    const float i0 = 1.0f / l0, i1 = 1.0f / l1;
#pragma unroll
    for (int dt = 0; dt < 8; ++dt) {
        const int e = h * 64 + dt * 8 + 2 * c;
        if (qa_row < T)
            *reinterpret_cast<__half2 *>(out + (size_t)(tl.row0 + qa_row) * d + e) = __floats2half2_rn(o[dt][0] * i0, o[dt][1] * i0);
        if (qb_row < T)
            *reinterpret_cast<__half2 *>(out + (size_t)(tl.row0 + qb_row) * d + e) = __floats2half2_rn(o[dt][2] * i1, o[dt][3] * i1);
    }
}

void launch_attn_prefill_fa(const float *qkv, int T, int slot, const DecodeView &dv, int layer, int d,
                            __half *out, cudaStream_t st) {
    attn_prefill_fa_kernel<<<dim3((T + 63) / 64, dv.n_heads), 128, 0, st>>>(
        qkv, nullptr, T, slot, dv.k_cache, dv.v_cache, layer, dv.n_slots, dv.n_heads, dv.max_seq, d, out);
}

// rows[r] = x[last row of request r]
__global__ void gather_rows_kernel(const float *x, const int *row_idx, int d, float *rows) {
    const int r = blockIdx.x;
    const float *src = x + (size_t)row_idx[r] * d;
    for (int i = threadIdx.x; i < d; i += blockDim.x) rows[(size_t)r * d + i] = src[i];
}

void prefill_batch_forward(const ModelView &m, const DecodeView &dv, const PrefillBatch &pb, int n_req,
                           int total, float *logits, cudaStream_t st) {
    const int d = m.d;
    __half *n16 = reinterpret_cast<__half *>(pb.n), *attn16 = reinterpret_cast<__half *>(pb.attn),
           *u16 = reinterpret_cast<__half *>(pb.u);
    for (int l = 0; l < m.n_layers; ++l) {
        const MkLayer &L = m.layers[l];
        launch_layernorm_rows_h(pb.x, L.ln1_w, L.ln1_b, total, d, n16, st);
        launch_gemm_rows(EPI_QKV, L.qkv, n16, pb.qkv, total, pb.row_slot, pb.row_pos, dv.k_cache, dv.v_cache,
                         dv.n_slots, dv.n_heads, dv.max_seq, l, d, st);
        attn_prefill_fa_kernel<<<dim3(pb.n_tiles, m.n_heads), 128, 0, st>>>(
            pb.qkv, pb.tiles, 0, 0, dv.k_cache, dv.v_cache, l, dv.n_slots, dv.n_heads, dv.max_seq, d, attn16);
        launch_gemm(EPI_RESID, L.proj, attn16, pb.x, total, nullptr, nullptr, nullptr, -1, 0, 0, 0, l, d, st);
        launch_layernorm_rows_h(pb.x, L.ln2_w, L.ln2_b, total, d, n16, st);
        launch_gemm(EPI_GELU, L.fc, n16, pb.u, total, nullptr, nullptr, nullptr, -1, 0, 0, 0, l, d, st);
        launch_gemm(EPI_RESID, L.mlp, u16, pb.x, total, nullptr, nullptr, nullptr, -1, 0, 0, 0, l, d, st);
    }
    // ln_f then final_norm on each request's last row, then mel_head (gpt.rs:673-692)
    gather_rows_kernel<<<n_req, 256, 0, st>>>(pb.x, pb.last_row, d, pb.qkv);
    launch_layernorm_rows(pb.qkv, m.ln_f_w, m.ln_f_b, n_req, d, pb.n, st);
    __half *fin16 = reinterpret_cast<__half *>(pb.attn);
    launch_layernorm_rows_h(pb.n, m.final_w, m.final_b, n_req, d, fin16, st);
    launch_gemm(EPI_PLAIN, m.mel_head, fin16, logits, n_req, nullptr, nullptr, nullptr, -1, 0, 0, 0, 0, d, st);
}

}  // namespace itts
