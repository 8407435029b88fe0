// Split-K reduction of the 2-CTA tensor-core GEMM (kq_gemm_pair_sm100.cu).
//
// When a call has too few 256-weight-row x 256-token tiles to occupy the
// GPU's SM pairs (256 tokens x 3072 rows = 12 tiles for
// 74 pairs), each tile is computed as ksplit units over equal shares of the
// K super-blocks.  Every unit stores its fp32 partial product
// part[s][m][row] (s = the unit's share, row = weight row); this kernel adds
// the shares in order s = 0, 1, ... (so the result does not depend on which
// unit finished first) and applies the call's fused epilogue, the one
// rounding to the output dtype and the peer-replica stores, exactly as the
// GEMM epilogue does for an unsplit tile.
//
// HBM/L2-bound byte work: one thread per output element, consecutive threads
// on consecutive output columns, so the partial reads and the Y stores are
// coalesced.  The partials were written just before and usually still sit in
// the 126 MB L2.
#include <type_traits>

#include "kq_epilogue.cuh"
#include "tc_internal.h"

namespace tc {
namespace {

constexpr uint32_t kMaxShares = 16;   // pair_ksplit never splits further

// V consecutive output columns per thread (V = 4 when every row offset is a
// multiple of 4 floats, so the loads are 16-byte vectors); S = the number of
// shares, a template parameter so that the share loads unroll exactly (few
// registers, full occupancy: enough loads in flight to cover the memory
// latency).  All shares are loaded before they are added; the sum runs in
// share order.
template <int V, int S>
__global__ void __launch_bounds__(256) split_reduce_kernel(const float *__restrict__ part, uint64_t stride,
                                                           uint32_t n_w, uint32_t n_out, uint32_t m_begin,
                                                           uint32_t rows, EpiView e, uint32_t gate_row, void *y,
                                                           uint64_t ldy, int dt) {
    using Vec = typename std::conditional<V == 4, float4, float>::type;
    const uint64_t idx = ((uint64_t)blockIdx.x * blockDim.x + threadIdx.x) * V;
    if (idx >= (uint64_t)rows * n_out) return;
    const uint32_t c0 = (uint32_t)(idx % n_out);
    const uint64_t m = (uint64_t)m_begin + idx / n_out;
    const bool glu = e.flags & TC_EPI_SWIGLU;
    // SwiGLU weights interleave 8 gate rows and the same 8 up rows; V = 4
    // columns starting at a multiple of 4 stay inside one group of 8.
    const uint32_t row0 = glu ? (c0 >> 3) * 16 + (c0 & 7) : c0;
    if (!tc_in_bounds(m * n_w + row0 + (glu ? 8 : 0) + V <= stride, e.status)) return;
    const float *src = part + m * n_w + row0;
    Vec pa[S], pu[S];
#pragma unroll
    for (int s = 0; s < S; ++s) {
        pa[s] = __ldcg(reinterpret_cast<const Vec *>(src + s * stride));
        if (glu) pu[s] = __ldcg(reinterpret_cast<const Vec *>(src + s * stride + 8));
    }
    float a[V] = {}, u[V] = {};
#pragma unroll
    for (int s = 0; s < S; ++s) {
        const float *va = reinterpret_cast<const float *>(&pa[s]), *vu = reinterpret_cast<const float *>(&pu[s]);
#pragma unroll
        for (int i = 0; i < V; ++i) {
            a[i] += va[i];
            if (glu) u[i] += vu[i];
        }
    }
#pragma unroll
    for (int i = 0; i < V; ++i) {
        const uint32_t row = row0 + i;
        const EpiRow er = epi_row(e, row, gate_row);
        float t = a[i] + er.bias;
        if (glu) t = silu(t) * (u[i] + epi_row(e, row + 8, gate_row).bias);
        else t = epi_act(e.flags, t);
        if (e.flags & TC_EPI_GATE_RESIDUAL)
            t = load_out(e.res, m * e.ld_res + er.col, dt == 0, dt == 1) + er.gate * t;
        store_out_all(e, y, m * ldy + er.col, t, dt == 0, dt == 1);
    }
}

template <int V, int S>
cudaError_t launch_shares(uint32_t ksplit, const float *part, uint64_t stride, uint32_t n_w, uint32_t n_out,
                          uint32_t m_begin, uint32_t rows, const EpiView &e, uint32_t gate_row, void *y, uint64_t ldy,
                          int dt, cudaStream_t s) {
    if constexpr (S < (int)kMaxShares) {
        if ((uint32_t)S != ksplit)
            return launch_shares<V, S + 1>(ksplit, part, stride, n_w, n_out, m_begin, rows, e, gate_row, y, ldy, dt, s);
    }
    const uint64_t threads = (uint64_t)rows * n_out / V;
    split_reduce_kernel<V, S><<<(unsigned)((threads + 255) / 256), 256, 0, s>>>(part, stride, n_w, n_out, m_begin,
                                                                              rows, e, gate_row, y, ldy, dt);
    return cudaGetLastError();
}

}  // namespace

cudaError_t launch_split_reduce(const float *part, uint32_t ksplit, uint64_t stride, uint32_t n_w, uint32_t m_begin,
                                uint32_t rows, const EpiView &e, uint32_t gate_row, void *y, uint64_t ldy,
                                int out_dtype, cudaStream_t s) {
    const uint32_t n_out = (e.flags & TC_EPI_SWIGLU) ? n_w / 2 : n_w;
    const uint64_t total = (uint64_t)rows * n_out;
    if (!total) return cudaSuccess;
    if (!part || !ksplit || ksplit > kMaxShares) return cudaErrorInvalidValue;
    const bool vec = n_out % 4 == 0 && n_w % 4 == 0 && (reinterpret_cast<uintptr_t>(part) & 15u) == 0;
    if (ksplit < 2) return cudaErrorInvalidValue;
    return vec ? launch_shares<4, 2>(ksplit, part, stride, n_w, n_out, m_begin, rows, e, gate_row, y, ldy, out_dtype, s)
               : launch_shares<1, 2>(ksplit, part, stride, n_w, n_out, m_begin, rows, e, gate_row, y, ldy, out_dtype, s);
}

}  // namespace tc
