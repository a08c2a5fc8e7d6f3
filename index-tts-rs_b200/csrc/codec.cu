// codec.cu -- SemanticCodec decode (the step after the mel-code decoder): codes [T] ->
// features [2T, 1024].
//
// Reference: crates/core/src/models/codec.rs:202-239 (SemanticCodec::decode), the Vocos
// backbone codec.rs:83-102 and the ConvNeXt block crates/core/src/models/convnext.rs:66-73,
// all fp32 on MLX:
//   z_q   = codebook[codes]                          [T, 8]
//   x     = out_project(z_q)   (Conv1d k=1)          [T, 1024]
//   h     = LN(embed(x))       (Conv1d 1024->384, k=7, pad 3; LN eps 1e-6)
//   12 x  h = h + gamma * pw2(GELU(pw1(LN(dwconv(h)))))   (depthwise k=7 pad 3; 384->2048->384)
//   h     = LN(h) ; h = h W1^T + b1                  [T, 1024]
//   out   = up(repeat(h, 2))   (nearest x2 along time, Conv1d 1024->1024, k=3, pad 1)
// MLX conv weights are channels-last [C_out, K, C_in]; a convolution is then a GEMM with an
// implicit im2col row (x[t + k - pad, :] for k = 0..K-1, zero outside the sequence), which
// is how every dense layer here runs: one fp32 tiled GEMM kernel with fused epilogues
// (bias, exact GELU, layer-scaled residual).  The 2x upsample is folded into the last
// convolution's row index (source row r of the upsampled sequence is h[r / 2]).
#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>

#include "kernels.h"

namespace itts {

constexpr int CG_BM = 64, CG_BN = 64, CG_BK = 16, CG_THREADS = 256;

enum CodecEpi : int { CEPI_BIAS = 0, CEPI_GELU = 1, CEPI_RESID_GAMMA = 2 };

struct CodecGemm {
    const float *x;   // source rows [src_rows][cin]
    int src_rows, cin, ksize, pad, upsample;  // upsample 2: conv over the x2 nearest-repeated rows
    const float *w;   // [n][ksize * cin]
    const float *bias, *gamma;
    float *y;         // [m][n]
    int m, n;
};

// element (row, kk) of the implicit im2col matrix: x[row + k - pad, i], kk = k * cin + i
__device__ __forceinline__ float im2col(const CodecGemm &p, int row, int kk) {
    const int k = kk / p.cin, i = kk - k * p.cin;
    const int r = row + k - p.pad;                 // row of the (upsampled) sequence
    const int rows = p.src_rows * p.upsample;
    if (r < 0 || r >= rows) return 0.f;
    return p.x[(size_t)(r / p.upsample) * p.cin + i];
}

__device__ __forceinline__ float gelu_erf(float v) {  // nn::gelu (exact): x * Phi(x)
    return 0.5f * v * (1.0f + erff(v * 0.70710678118654752f));
}

// C[m, n] = sum_kk A[m, kk] W[n, kk] + bias[n], then the epilogue; 64 x 64 tiles, each thread
// a 4 x 4 block, K in steps of 16 through shared memory.
template <int EPI>
__global__ void __launch_bounds__(CG_THREADS) codec_gemm_kernel(CodecGemm p) {
    __shared__ float As[CG_BK][CG_BM + 4];
    __shared__ float Ws[CG_BK][CG_BN + 4];
    const int K = p.ksize * p.cin;
    const int m0 = blockIdx.y * CG_BM, n0 = blockIdx.x * CG_BN;
    const int tid = threadIdx.x, ty = tid >> 4, tx = tid & 15;
    float acc[4][4] = {};
    for (int k0 = 0; k0 < K; k0 += CG_BK) {
        for (int e = tid; e < CG_BM * CG_BK; e += CG_THREADS) {  // A tile (k-major in smem)
            const int r = e / CG_BK, kk = e % CG_BK;
            const int row = m0 + r, kg = k0 + kk;
            As[kk][r] = (row < p.m && kg < K) ? im2col(p, row, kg) : 0.f;
        }
        for (int e = tid; e < CG_BN * CG_BK; e += CG_THREADS) {  // W tile
            const int c = e / CG_BK, kk = e % CG_BK;
            const int col = n0 + c, kg = k0 + kk;
            Ws[kk][c] = (col < p.n && kg < K) ? p.w[(size_t)col * K + kg] : 0.f;
        }
        __syncthreads();
#pragma unroll
        for (int kk = 0; kk < CG_BK; ++kk) {
            float a[4], b[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) a[i] = As[kk][ty * 4 + i];
#pragma unroll
            for (int j = 0; j < 4; ++j) b[j] = Ws[kk][tx * 4 + j];
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int row = m0 + ty * 4 + i;
        if (row >= p.m) continue;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int col = n0 + tx * 4 + j;
            if (col >= p.n) continue;
            float v = acc[i][j] + p.bias[col];
            float *yp = p.y + (size_t)row * p.n + col;
            if (EPI == CEPI_GELU) v = gelu_erf(v);
            if (EPI == CEPI_RESID_GAMMA) v = *yp + p.gamma[col] * v;
            *yp = v;
        }
    }
}

// z = codebook[code] ([8]) then the k=1 out_project: x[t, o] = b[o] + sum_j z[j] w[o, j]
__global__ void codec_vq_kernel(const int32_t *codes, int T, const float *codebook, int cdim, const float *w,
                                const float *b, int hidden, float *x) {
    const int t = blockIdx.x;
    if (t >= T) return;
    const float *z = codebook + (size_t)codes[t] * cdim;
    for (int o = threadIdx.x; o < hidden; o += blockDim.x) {
        float v = 0.f;
        for (int j = 0; j < cdim; ++j) v = fmaf(z[j], w[(size_t)o * cdim + j], v);
        x[(size_t)t * hidden + o] = v + b[o];
    }
}

// depthwise Conv1d (groups = channels, k taps, pad (k-1)/2): y[t, c] = b[c] + sum_k x[t+k-pad, c] w[c, k]
__global__ void codec_dwconv_kernel(const float *x, int T, int C, const float *w, int K, const float *b, float *y) {
    const int t = blockIdx.x, pad = (K - 1) / 2;
    for (int c = threadIdx.x; c < C; c += blockDim.x) {
        float v = 0.f;
        for (int k = 0; k < K; ++k) {
            const int r = t + k - pad;
            if (r >= 0 && r < T) v = fmaf(x[(size_t)r * C + c], w[(size_t)c * K + k], v);
        }
        y[(size_t)t * C + c] = v + b[c];
    }
}

// LayerNorm of each row (fast::layer_norm, eps given): one warp per row, two-pass statistics
__global__ void codec_ln_kernel(const float *x, int rows, int C, const float *w, const float *b, float eps,
                                float *y) {
    const int r = blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (r >= rows) return;
    const float *xr = x + (size_t)r * C;
    float s = 0.f;
    for (int c = lane; c < C; c += 32) s += xr[c];
    const float mean = warp_sum(s) / (float)C;
    float q = 0.f;
    for (int c = lane; c < C; c += 32) {
        const float d = xr[c] - mean;
        q += d * d;
    }
    const float rstd = 1.0f / sqrtf(warp_sum(q) / (float)C + eps);
    float *yr = y + (size_t)r * C;
    for (int c = lane; c < C; c += 32) yr[c] = (xr[c] - mean) * rstd * w[c] + b[c];
}

static void gemm(int epi, const CodecGemm &p, cudaStream_t st) {
    dim3 grid((p.n + CG_BN - 1) / CG_BN, (p.m + CG_BM - 1) / CG_BM);
    if (epi == CEPI_GELU) codec_gemm_kernel<CEPI_GELU><<<grid, CG_THREADS, 0, st>>>(p);
    else if (epi == CEPI_RESID_GAMMA) codec_gemm_kernel<CEPI_RESID_GAMMA><<<grid, CG_THREADS, 0, st>>>(p);
    else codec_gemm_kernel<CEPI_BIAS><<<grid, CG_THREADS, 0, st>>>(p);
}

static CodecGemm linear(const float *x, int rows, int cin, const float *w, const float *b, float *y, int n) {
    CodecGemm p{};
    p.x = x; p.src_rows = rows; p.cin = cin; p.ksize = 1; p.pad = 0; p.upsample = 1;
    p.w = w; p.bias = b; p.y = y; p.m = rows; p.n = n;
    return p;
}

cudaError_t codec_decode_forward(const CodecView &c, const int32_t *d_codes, int T, const CodecBufs &bb,
                                 float *d_out, cudaStream_t st) {
    const int H = c.hidden, D = c.dim, FF = c.inter;
    codec_vq_kernel<<<T, 256, 0, st>>>(d_codes, T, c.codebook, c.cdim, c.out_w, c.out_b, H, bb.x);
    {  // embed: Conv1d(H -> D, k, pad (k-1)/2), then LN
        CodecGemm p{};
        p.x = bb.x; p.src_rows = T; p.cin = H; p.ksize = c.embed_k; p.pad = (c.embed_k - 1) / 2; p.upsample = 1;
        p.w = c.embed_w; p.bias = c.embed_b; p.y = bb.t; p.m = T; p.n = D;
        gemm(CEPI_BIAS, p, st);
    }
    const int ln_grid = (T + 7) / 8;
    codec_ln_kernel<<<ln_grid, 256, 0, st>>>(bb.t, T, D, c.norm_w, c.norm_b, c.eps, bb.h);
    for (int l = 0; l < c.n_layers; ++l) {
        const CodecBlock &k = c.blocks[l];
        codec_dwconv_kernel<<<T, 128, 0, st>>>(bb.h, T, D, k.dw_w, c.dw_k, k.dw_b, bb.t);
        codec_ln_kernel<<<ln_grid, 256, 0, st>>>(bb.t, T, D, k.norm_w, k.norm_b, c.eps, bb.t);
        gemm(CEPI_GELU, linear(bb.t, T, D, k.pw1_w, k.pw1_b, bb.u, FF), st);
        CodecGemm p2 = linear(bb.u, T, FF, k.pw2_w, k.pw2_b, bb.h, D);
        p2.gamma = k.gamma;
        gemm(CEPI_RESID_GAMMA, p2, st);
    }
    codec_ln_kernel<<<ln_grid, 256, 0, st>>>(bb.h, T, D, c.fnorm_w, c.fnorm_b, c.eps, bb.t);
    gemm(CEPI_BIAS, linear(bb.t, T, D, c.proj_w, c.proj_b, bb.x, H), st);
    {  // up: Conv1d(H -> H, k, pad (k-1)/2) over the x2 nearest-repeated rows
        CodecGemm p{};
        p.x = bb.x; p.src_rows = T; p.cin = H; p.ksize = c.up_k; p.pad = (c.up_k - 1) / 2; p.upsample = 2;
        p.w = c.up_w; p.bias = c.up_b; p.y = d_out; p.m = 2 * T; p.n = H;
        gemm(CEPI_BIAS, p, st);
    }
    return cudaGetLastError();
}

}  // namespace itts
