// gemm.cuh -- parameters and epilogue of the int8-weight GEMMs (prefill, and decode with
// more columns than the persistent kernel takes): y[t, o] = x[t, :] . W[o, :] + bias[o].
#pragma once
#include "kernels.h"

namespace itts {

struct GemmParams {
    MkLin W;
    const __half *x;  // [T, K] fp16 activations
    float *y;         // [T, OUT] (fp16 [T, OUT] for EPI_GELU, whose output feeds the next GEMM)
    int T;
    // EPI_QKV: prefill writes row t's K/V at position t of kv_slot; decode (slots != null)
    // writes them at the valid_len of slot batch_slot[t]
    __half *k_cache, *v_cache;
    const SlotState *slots;
    const int *batch_slot;
    // packed prefill of several requests: row t's K/V go to (row_slot[t], row_pos[t])
    const int *row_slot, *row_pos;
    // split-K of the fp16 GEMM (few rows): partial sums [ksplit][T][OUT] in ws, which holds
    // ws_splits of them; the epilogue then runs on their sum
    float *ws;
    int ksplit, ws_splits;
    int kv_slot, n_slots, n_heads, max_seq, layer, d;
};

// Where row t's new K/V go (EPI_QKV): position t of kv_slot in prefill; (row_slot[t],
// row_pos[t]) in a packed prefill of several requests; the valid_len of slot
// batch_slot[t] in decode, unless that slot is inactive or full.
struct QkvDest {
    int slot, pos;
    bool write;
};
__device__ __forceinline__ QkvDest qkv_dest(const GemmParams &p, int t) {
    QkvDest q{p.kv_slot, t, t < p.max_seq};
    if (p.row_slot) {
        q.slot = p.row_slot[t];
        q.pos = p.row_pos[t];
        q.write = q.pos < p.max_seq;
    } else if (p.slots) {
        q.slot = p.batch_slot[t];
        const SlotState &st = p.slots[q.slot];
        q.pos = st.valid_len;
        q.write = st.active && q.pos < p.max_seq;
    }
    return q;
}

// Output (t, o) with value v = accumulator + bias[o], per epilogue (qd: row t's K/V
// destination, used by EPI_QKV).
template <int EPI>
__device__ __forceinline__ void gemm_store(const GemmParams &p, int t, int o, float v, const QkvDest &qd) {
    const int OUT = p.W.out;
    float *yp = p.y + (size_t)t * OUT + o;
    if (EPI == EPI_PLAIN) {
        *yp = v;
    } else if (EPI == EPI_GELU) {
        reinterpret_cast<__half *>(p.y)[(size_t)t * OUT + o] = __float2half_rn(gelu_tanh(v));
    } else if (EPI == EPI_RESID) {
        *yp += v;
    } else {
        *yp = v;
        if (o >= p.d && qd.write) {
            const int rr = o - p.d, which = rr / p.d, oo = rr - which * p.d;
            __half *cache = which == 0 ? p.k_cache : p.v_cache;
            cache[kv_index(p.layer, qd.slot, oo >> 6, qd.pos, p.n_slots, p.n_heads, p.max_seq) + (oo & 63)] =
                __float2half_rn(v);
        }
    }
}

// Tensor-core version (gemm_tc.cu): tcgen05 MMA on 128 x 128 tiles, TMEM accumulators.
// False when the activation tensor map could not be built (the caller then uses the
// CUDA-core kernel).
bool launch_gemm_tc(int epi, const GemmParams &p, cudaStream_t st);
// fp16 x fp16 tensor-core GEMM over an fp16 copy of the weights (long prefills); false
// when it cannot run (no copy, misaligned operands, no tensor-map encoder).
bool launch_gemm_f16(int epi, const GemmParams &p, const __half *w16, cudaStream_t st);
void kernels_init_gemm_tc();

}  // namespace itts
