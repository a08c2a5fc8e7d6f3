// gemm.cuh -- parameters and epilogue of the int8-weight GEMMs (prefill, and decode with
// more columns than the persistent kernel takes): y[t, o] = x[t, :] . W[o, :] + bias[o].
#pragma once
#include "kernels.h"

namespace itts {

struct GemmParams {
    MkLin W;
    const float *x;  // [T, K]
    float *y;        // [T, OUT]
    int T;
    // EPI_QKV: prefill writes row t's K/V at position t of kv_slot; decode (slots != null)
    // writes them at the valid_len of slot batch_slot[t]
    __half *k_cache, *v_cache;
    const SlotState *slots;
    const int *batch_slot;
    int kv_slot, n_slots, n_heads, max_seq, layer, d;
};

// Output (t, o) with value v = accumulator + bias[o], per epilogue.
template <int EPI>
__device__ __forceinline__ void gemm_store(const GemmParams &p, int t, int o, float v) {
    const int OUT = p.W.out;
    float *yp = p.y + (size_t)t * OUT + o;
    if (EPI == EPI_PLAIN) {
        *yp = v;
    } else if (EPI == EPI_GELU) {
        *yp = gelu_tanh(v);
    } else if (EPI == EPI_RESID) {
        *yp += v;
    } else {
        *yp = v;
        if (o >= p.d) {
            const int rr = o - p.d, which = rr / p.d, oo = rr - which * p.d;
            __half *cache = which == 0 ? p.k_cache : p.v_cache;
            int slot = p.kv_slot, pos = t;
            bool write = t < p.max_seq;
            if (p.slots) {
                slot = p.batch_slot[t];
                const SlotState &st = p.slots[slot];
                pos = st.valid_len;
                write = st.active && pos < p.max_seq;
            }
            if (write)
                cache[kv_index(p.layer, slot, oo >> 6, pos, p.n_slots, p.n_heads, p.max_seq) + (oo & 63)] =
                    __float2half_rn(v);
        }
    }
}

// Tensor-core version (gemm_tc.cu): tcgen05 MMA on 128 x 128 tiles, TMEM accumulators.
void launch_gemm_tc(int epi, const GemmParams &p, cudaStream_t st);
void kernels_init_gemm_tc();

}  // namespace itts
