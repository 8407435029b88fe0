// Fused epilogue arithmetic shared by the tensor-core GEMMs and the GEMV.
//
// The reference applies these after its quantised matmul, each as a separate
// array operation rounded to the activation dtype: the bias add of
// Weights::project (native/backends/mlx.cpp:687-688), SiLU(gate) * up of the
// SwiGLU FFN (native/models/qwen21/transformer.cpp:971-976) and the AdaLN
// gated residual hidden + gate * projected (transformer.cpp:950, :980).  Here
// they run in fp32 on the accumulator, with one rounding to the output dtype.
//
// SwiGLU weights (tc_cuda_weight_upload_glu) hold 8 gate rows and then the
// same 8 up rows in every group of 16 weight rows, so weight row n is a gate
// row when (n & 8) == 0, its partner (the up row of the same output column)
// is row n + 8, and its output column is (n >> 4) * 8 + (n & 7).
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cstdint>

#include "../../include/turbocider_cuda.h"
#include "tc_internal.h"

namespace tc {

__device__ __forceinline__ uint32_t glu_column(uint32_t n) { return (n >> 4) * 8 + (n & 7); }

// t * logistic(z) = t / (1 + e^-z), with the fast exponential and division:
// relative error ~1e-6 (the exponent's rounding, scaled by |z| <~ 20 where it
// matters), far below every output dtype's rounding.  For very negative z the
// denominator overflows to +inf and the quotient is 0, the limit.
__device__ __forceinline__ float times_logistic(float t, float z) { return __fdividef(t, 1.f + __expf(-z)); }
// tanh-form GELU, 0.5 t (1 + tanh(u)) with u = sqrt(2/pi) (t + 0.044715 t^3),
// written as t * logistic(2u) (1 + tanh(u) = 2 logistic(2u)).
__device__ __forceinline__ float gelu_tanh(float t) {
    const float u = 0.7978845608028654f * (t + 0.044715f * t * t * t);   // sqrt(2/pi)
    return times_logistic(t, 2.f * u);
}
__device__ __forceinline__ float gelu_erf(float t) { return 0.5f * t * (1.f + erff(t * 0.7071067811865476f)); }
__device__ __forceinline__ float silu(float t) { return times_logistic(t, t); }

// Per output row (weight row n of the tile) state of the fused epilogue.
struct EpiRow {
    float bias;    // bias of weight row n (gate or up part for SwiGLU)
    float gate;    // gate vector value of this output column
    uint32_t col;  // output column
    bool writer;   // this row produces an output (SwiGLU: gate rows only)
};

// n: weight row (< rows, the weight's row count).  gate_row: the segment's
// gate vector.
__device__ __forceinline__ EpiRow epi_row(const EpiView &e, uint32_t n, uint32_t gate_row) {
    EpiRow r;
    const bool glu = e.flags & TC_EPI_SWIGLU;
    r.col = glu ? glu_column(n) : n;
    r.writer = !glu || (n & 8) == 0;
    r.bias = 0.f;
    if (e.flags & TC_EPI_BIAS) r.bias = __ldg(e.bias + (glu && (n & 8) ? e.bias_up + r.col : r.col));
    r.gate = 0.f;
    if (e.flags & TC_EPI_GATE_RESIDUAL) r.gate = __ldg(e.gate + (uint64_t)gate_row * e.ld_gate + r.col);
    return r;
}

// Value before the gated residual: bias and activation.  For SwiGLU `up` is
// the partner row's biased accumulator (already through epi_pre's bias).
__device__ __forceinline__ float epi_act(uint32_t flags, float t) {
    if (flags & TC_EPI_GELU_TANH) return gelu_tanh(t);
    if (flags & TC_EPI_GELU_ERF) return gelu_erf(t);
    return t;
}

__device__ __forceinline__ float load_out(const void *p, uint64_t off, bool f32, bool f16) {
    if (f32) return static_cast<const float *>(p)[off];
    if (f16) return __half2float(static_cast<const __half *>(p)[off]);
    return __bfloat162float(static_cast<const __nv_bfloat16 *>(p)[off]);
}
__device__ __forceinline__ void store_out(void *p, uint64_t off, float v, bool f32, bool f16) {
    if (f32) static_cast<float *>(p)[off] = v;
    else if (f16) static_cast<__half *>(p)[off] = __float2half_rn(v);
    else static_cast<__nv_bfloat16 *>(p)[off] = __float2bfloat16_rn(v);
}
// Store to Y and to every peer replica of it (N-column sharding: the peers'
// Y buffers over NVLink).
__device__ __forceinline__ void store_out_all(const EpiView &e, void *y, uint64_t off, float v, bool f32, bool f16) {
    if (!tc_in_bounds(!e.y_limit || off < e.y_limit, e.status)) return;
    store_out(y, off, v, f32, f16);
    for (uint32_t i = 0; i < e.n_peer; ++i) store_out(e.peer[i], off, v, f32, f16);
}

// One 32-token piece of a TMEM accumulator through the fused epilogue:
// thread = weight row n (all 32 lanes of the warp call this together, the
// SwiGLU pairing shuffles between lanes L and L + 8), v[c] = accumulator of
// token m0 + c.  Rows past the weight (row_ok false) and tokens past m_end
// store nothing.
template <bool OUT_F32>
__device__ __forceinline__ void epi_piece(const EpiView &e, const EpiRow &r, const uint32_t (&v)[32], bool row_ok,
                                          uint32_t m0, uint32_t m_end, void *y, uint64_t ldy) {
    const bool glu = e.flags & TC_EPI_SWIGLU, gres = e.flags & TC_EPI_GATE_RESIDUAL, f16 = e.out_f16;
#pragma unroll
    for (uint32_t c = 0; c < 32; ++c) {
        float t = __uint_as_float(v[c]) + r.bias;
        if (glu) {
            const float up = __shfl_down_sync(0xffffffffu, t, 8);
            t = silu(t) * up;
        } else {
            t = epi_act(e.flags, t);
        }
        const uint32_t m = m0 + c;
        if (row_ok && r.writer && m < m_end) {
            if (gres) t = load_out(e.res, (uint64_t)m * e.ld_res + r.col, OUT_F32, f16) + r.gate * t;
            store_out_all(e, y, (uint64_t)m * ldy + r.col, t, OUT_F32, f16);
        }
    }
}

}  // namespace tc
