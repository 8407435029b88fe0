// Small-M quantised GEMV: Y[m, n] = sum_k X[m, k] * W[n, k] for M <= 16
// (timestep / AdaLN-modulation linears).  HBM-bound on the packed weight.
//
// One warp owns one weight row n (= one output column) at a time and walks
// its super-blocks; the 32 lanes split each 256-weight block 8 weights each,
// reading the block's packed fields straight from the panel layout with
// coalesced 32-bit loads (a warp reads whole 32-byte sectors of each field).
// Weights are dequantised in fp32 with the reference's exact arithmetic, so
// the result equals the fp32 decode + fp32 matmul up to summation order.
#include "kq_format.cuh"
#include "tc_internal.h"

namespace tc {
namespace {

__device__ __forceinline__ float bf16_lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }

template <int MT>
__device__ __forceinline__ void fma4(float (&acc)[MT], int m, const float wv[4], uint2 xv) {
    acc[m] = fmaf(wv[0], bf16_lo(xv.x), acc[m]);
    acc[m] = fmaf(wv[1], bf16_hi(xv.x), acc[m]);
    acc[m] = fmaf(wv[2], bf16_lo(xv.y), acc[m]);
    acc[m] = fmaf(wv[3], bf16_hi(xv.y), acc[m]);
}

template <int TYPE, int MT, int DT>
__global__ void __launch_bounds__(256) gemv_kernel(WeightView w, const uint16_t *__restrict__ x,
                                                   uint32_t m_begin, uint32_t m_count, uint64_t k,
                                                   void *__restrict__ y, uint64_t ldy) {
    const uint32_t lane = threadIdx.x & 31;
    const uint32_t warps = gridDim.x * (blockDim.x / 32);
    constexpr uint32_t chunk = TYPE == 12 ? kQ4KChunk : kQ6KChunk;
    for (uint32_t row = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32; row < w.n; row += warps) {
        const uint32_t r = row % kPanelRows, slot = row_slot(r);
        const uint8_t *panel = w.chunks + (uint64_t)(row / kPanelRows) * w.kb * chunk;
        float acc[MT];
#pragma unroll
        for (int m = 0; m < MT; ++m) acc[m] = 0.f;
        for (uint32_t kb = 0; kb < w.kb; ++kb) {
            const uint8_t *c = panel + (uint64_t)kb * chunk;
            if (TYPE == 12) {
                const uint32_t s = lane / 8, t = lane % 8;
                const uint32_t q = __ldg(reinterpret_cast<const uint32_t *>(c + kQ4Qs + s * 4096 + slot * 32 + t * 4));
                const uint32_t *scw = reinterpret_cast<const uint32_t *>(c + kQ4Sc + r * 12);
                uint32_t sw[3] = {__ldg(scw), __ldg(scw + 1), __ldg(scw + 2)};
                const uint8_t *sc = reinterpret_cast<const uint8_t *>(sw);
                const uint32_t dm = __ldg(reinterpret_cast<const uint32_t *>(c + kQ4Dm + r * 4));
                const float d = half_bits_to_float((uint16_t)(dm & 0xffffu));
                const float dmin = half_bits_to_float((uint16_t)(dm >> 16));
                uint32_t sc0, mn0, sc1, mn1;
                q4k_scale_min(2 * s, sc, sc0, mn0);
                q4k_scale_min(2 * s + 1, sc, sc1, mn1);
                const float d0 = d * (float)sc0, m0 = dmin * (float)mn0;
                const float d1 = d * (float)sc1, m1 = dmin * (float)mn1;
                float lo[4], hi[4];
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    lo[i] = q4k_value(d0, m0, (q >> (8 * i)) & 15u);
                    hi[i] = q4k_value(d1, m1, (q >> (8 * i + 4)) & 15u);
                }
                const uint64_t k0 = (uint64_t)kb * 256 + 64 * s + 4 * t;
#pragma unroll
                for (int m = 0; m < MT; ++m) {
                    if (m < (int)m_count) {
                        const uint16_t *xr = x + (uint64_t)(m_begin + m) * k;
                        fma4<MT>(acc, m, lo, __ldg(reinterpret_cast<const uint2 *>(xr + k0)));
                        fma4<MT>(acc, m, hi, __ldg(reinterpret_cast<const uint2 *>(xr + k0 + 32)));
                    }
                }
            } else {
                const uint32_t h = lane / 16, part = (lane / 8) % 2, t = lane % 8;
                const uint32_t ql = __ldg(reinterpret_cast<const uint32_t *>(
                    c + kQ6Ql + ((h * 2 + part) * kPanelRows + slot) * 32 + t * 4));
                const uint32_t qh = __ldg(reinterpret_cast<const uint32_t *>(
                    c + kQ6Qh + (h * kPanelRows + slot) * 32 + t * 4));
                const float d = half_bits_to_float(__ldg(reinterpret_cast<const uint16_t *>(c + kQ6D + r * 2)));
                const int8_t *sc = reinterpret_cast<const int8_t *>(c + kQ6Sc + r * 16);
                const uint32_t ga = part, gb = 2 + part;     // low / high nibble groups
                const float da = d * (float)__ldg(sc + 8 * h + t / 4 + 2 * ga);
                const float db = d * (float)__ldg(sc + 8 * h + t / 4 + 2 * gb);
                float va[4], vb[4];
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const uint32_t lb = (ql >> (8 * i)) & 0xffu, hb = (qh >> (8 * i)) & 0xffu;
                    const int ca = (int)((lb & 15u) | (((hb >> (2 * ga)) & 3u) << 4)) - 32;
                    const int cb = (int)((lb >> 4) | (((hb >> (2 * gb)) & 3u) << 4)) - 32;
                    va[i] = da * (float)ca;
                    vb[i] = db * (float)cb;
                }
                const uint64_t ka = (uint64_t)kb * 256 + 128 * h + 32 * ga + 4 * t;
                const uint64_t kb2 = (uint64_t)kb * 256 + 128 * h + 32 * gb + 4 * t;
#pragma unroll
                for (int m = 0; m < MT; ++m) {
                    if (m < (int)m_count) {
                        const uint16_t *xr = x + (uint64_t)(m_begin + m) * k;
                        fma4<MT>(acc, m, va, __ldg(reinterpret_cast<const uint2 *>(xr + ka)));
                        fma4<MT>(acc, m, vb, __ldg(reinterpret_cast<const uint2 *>(xr + kb2)));
                    }
                }
            }
        }
#pragma unroll
        for (int m = 0; m < MT; ++m)
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) acc[m] += __shfl_xor_sync(0xffffffffu, acc[m], o);
#pragma unroll
        for (int m = 0; m < MT; ++m) {
            if (lane == (uint32_t)m && m < (int)m_count) {
                const uint64_t off = (uint64_t)(m_begin + m) * ldy + row;
                if (DT == 0) static_cast<float *>(y)[off] = acc[m];
                else static_cast<__nv_bfloat16 *>(y)[off] = __float2bfloat16_rn(acc[m]);
            }
        }
    }
}

template <int TYPE, int MT>
cudaError_t launch_typed(const SegmentView &seg, const uint16_t *x, uint64_t k, void *y, uint64_t ldy,
                         int out_dtype, cudaStream_t s) {
    const unsigned blocks = (seg.w.n + 7) / 8;
    const uint32_t mc = seg.m_end - seg.m_begin;
    if (out_dtype == 0) gemv_kernel<TYPE, MT, 0><<<blocks, 256, 0, s>>>(seg.w, x, seg.m_begin, mc, k, y, ldy);
    else gemv_kernel<TYPE, MT, 2><<<blocks, 256, 0, s>>>(seg.w, x, seg.m_begin, mc, k, y, ldy);
    return cudaGetLastError();
}

template <int TYPE>
cudaError_t launch_m(const SegmentView &seg, const uint16_t *x, uint64_t k, void *y, uint64_t ldy,
                     int out_dtype, cudaStream_t s) {
    const uint32_t m = seg.m_end - seg.m_begin;
    if (m <= 1) return launch_typed<TYPE, 1>(seg, x, k, y, ldy, out_dtype, s);
    if (m <= 2) return launch_typed<TYPE, 2>(seg, x, k, y, ldy, out_dtype, s);
    if (m <= 4) return launch_typed<TYPE, 4>(seg, x, k, y, ldy, out_dtype, s);
    if (m <= 8) return launch_typed<TYPE, 8>(seg, x, k, y, ldy, out_dtype, s);
    return launch_typed<TYPE, 16>(seg, x, k, y, ldy, out_dtype, s);
}

}  // namespace

cudaError_t launch_gemv(const SegmentView &seg, const uint16_t *x, uint64_t k, void *y, uint64_t ldy,
                        int out_dtype, uint32_t *status, cudaStream_t s) {
    (void)status;
    if (seg.m_end <= seg.m_begin) return cudaSuccess;
    if (seg.m_end - seg.m_begin > 16) return cudaErrorInvalidValue;
    return seg.w.type == 12 ? launch_m<12>(seg, x, k, y, ldy, out_dtype, s)
                            : launch_m<14>(seg, x, k, y, ldy, out_dtype, s);
}

}  // namespace tc
