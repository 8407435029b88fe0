// Small-M quantised GEMV (M <= 16 rows of X: timestep / AdaLN-modulation
// linears): Y[m, n] = sum_k X[m, k] * W[n, k].  HBM-bound on the packed
// weight: at 6.5 TB/s an SM must retire ~28 weights per clock, which leaves
// no room for an fp32 dequantise-and-FMA per weight per token.  So the
// weights stay in code space:
//
//   * each K16 step of mma.sync.m16n8k16 (bf16 in, fp32 accumulate) takes the
//     raw 4-/6-bit codes of 16 weight rows as bf16 -- exact: a prmt places
//     each code byte under the exponent of 128 (0x43cc = 128 + c) and one
//     bf16x2 subtract removes the 128 (and Q6_K's bias 32);
//   * the K16 step never crosses a scale group (Q6_K: 16 weights, Q4_K: 32
//     weights = two chained steps), so the fp32 fragment holds
//     sum_k x_k * q_k of one group, scaled afterwards by d*sc in fp32;
//   * Q4_K's min term -dmin*m_g * sum_k x_k takes sum_k x_k from one more MMA
//     with an all-ones A fragment (no extra loads: same B fragment);
//   * within each K16 step the thread <-> k assignment is permuted so that a
//     thread's four codes are four consecutive packed bytes (one 32-bit
//     load), and its four activations are four consecutive bf16 (one 64-bit
//     load): logical k {2t, 2t+1, 2t+8, 2t+9} <-> physical {4t .. 4t+3}.
// Result: fp32 accumulation of exactly-represented products; equal to the
// fp32-decode + fp32 matmul oracle up to summation order.
//
// Work split: CTA (x, y) = (16 weight rows, one K slice of 4*u super-blocks),
// 4 warps each taking u super-blocks, so that thousands of short CTAs keep
// every SM's loads in flight (the CTA count is independent of the SM count).
// Each warp issues all loads of its super-block before computing.  A CTA
// sums its warps through shared memory; with several K slices it stores the
// 16 x M partial in the context workspace, and the last CTA of the row tile to
// finish (per-tile arrival counter) adds the slices in slice order -- a fixed
// order, so results are deterministic -- writes Y and resets the counter.
// The N8 side of the MMA carries the tokens: NT = 1 or 2 tiles of 8.
#include "kq_format.cuh"
#include "tc_internal.h"

namespace tc {
namespace {

constexpr int kWarps = 4;

__device__ __forceinline__ uint32_t ldg32(const uint8_t *p) { return __ldg(reinterpret_cast<const uint32_t *>(p)); }

// Two code bytes (selector 0x4140: bytes 0,1; 0x4342: bytes 2,3) as the bf16
// pair (128 + c0, 128 + c1).
__device__ __forceinline__ uint32_t code_pair(uint32_t codes, uint32_t sel) {
    uint32_t r;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(codes), "r"(0x43434343u), "r"(sel));
    return r;
}
__device__ __forceinline__ uint32_t bf16x2_sub(uint32_t a, uint32_t b) {
    uint32_t r;
    asm("sub.rn.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
    return r;
}
__device__ __forceinline__ void mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1, const float (&c)[4]) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%10, %11, %12, %13};"
        : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "f"(c[0]), "f"(c[1]), "f"(c[2]), "f"(c[3]));
}

// A fragment from the code words of rows g (cg) and g+8 (cg8), minus `bias`
// (a bf16x2 constant: 128 for Q4_K, 160 for Q6_K).
struct AFrag { uint32_t r0, r1, r2, r3; };
__device__ __forceinline__ AFrag a_frag(uint32_t cg, uint32_t cg8, uint32_t bias) {
    return {bf16x2_sub(code_pair(cg, 0x4140u), bias), bf16x2_sub(code_pair(cg8, 0x4140u), bias),
            bf16x2_sub(code_pair(cg, 0x4342u), bias), bf16x2_sub(code_pair(cg8, 0x4342u), bias)};
}

template <int NT>
__device__ __forceinline__ void x_frag(const uint16_t *const (&xr)[NT], uint64_t kpos, uint32_t (&b)[NT][2]) {
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
        if (xr[nt]) {
            const uint2 v = __ldg(reinterpret_cast<const uint2 *>(xr[nt] + kpos));
            b[nt][0] = v.x;
            b[nt][1] = v.y;
        } else {
            b[nt][0] = b[nt][1] = 0u;
        }
    }
}

template <int TYPE, int NT, int DT>
__global__ void __launch_bounds__(kWarps * 32) gemv_kernel(WeightView w, const uint16_t *__restrict__ x,
                                                           uint32_t m_begin, uint32_t m_count, uint64_t k,
                                                           void *__restrict__ y, uint64_t ldy,
                                                           uint32_t kb_per_slice, float *__restrict__ partials,
                                                           uint32_t *__restrict__ counters) {
    constexpr uint32_t chunk = TYPE == 12 ? kQ4KChunk : kQ6KChunk;
    __shared__ float red[kWarps][32][4 * NT];
    __shared__ __align__(16) float tab[kWarps][16 * 16];
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
    const uint32_t row0 = blockIdx.x * 16, panel = row0 / kPanelRows, r0 = row0 % kPanelRows;
    const uint32_t n_slices = gridDim.y, kb_begin = blockIdx.y * kb_per_slice;
    const uint32_t kb_end = min(w.kb, kb_begin + kb_per_slice);
    const uint32_t sg = row_slot(r0 + g), sg8 = row_slot(r0 + g + 8);
    const uint8_t *pbase = w.chunks + (uint64_t)panel * w.kb * chunk;
    const uint16_t *xr[NT];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
        xr[nt] = (8 * nt + g < m_count) ? x + (uint64_t)(m_begin + 8 * nt + g) * k : nullptr;
    float acc[NT][4];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int i = 0; i < 4; ++i) acc[nt][i] = 0.f;
    float *wt = tab[warp];

    for (uint32_t kb = kb_begin + warp; kb < kb_end; kb += kWarps) {
        const uint8_t *c = pbase + (uint64_t)kb * chunk;
        const uint64_t kbase = (uint64_t)kb * 256;
        __syncwarp();
        if (TYPE == 12) {
            // scale table: rows r0..r0+15 x 8 sub-blocks of (d*sc, dmin*m)
            {
                const uint32_t rr = r0 + (lane >> 1), half = lane & 1;
                const uint32_t dm = __ldg(reinterpret_cast<const uint32_t *>(c + kQ4Dm + rr * 4));
                const float d = half_bits_to_float((uint16_t)(dm & 0xffffu));
                const float dmin = half_bits_to_float((uint16_t)(dm >> 16));
                uint32_t sw[3];
                const uint32_t *sp = reinterpret_cast<const uint32_t *>(c + kQ4Sc + rr * 12);
                sw[0] = __ldg(sp); sw[1] = __ldg(sp + 1); sw[2] = __ldg(sp + 2);
                const uint8_t *sc = reinterpret_cast<const uint8_t *>(sw);
                float2 *o = reinterpret_cast<float2 *>(wt) + (lane >> 1) * 8 + half * 4;
#pragma unroll
                for (uint32_t i = 0; i < 4; ++i) {
                    uint32_t s, m;
                    q4k_scale_min(half * 4 + i, sc, s, m);
                    o[i] = make_float2(d * (float)s, dmin * (float)m);
                }
            }
            __syncwarp();
            const uint32_t bias = 0x43004300u;     // bf16x2 (128, 128)
            const uint32_t ones = 0x3F803F80u;     // bf16x2 (1, 1)
#pragma unroll
            for (uint32_t s = 0; s < 4; ++s) {
                uint32_t wg[2], wg8[2];
#pragma unroll
                for (uint32_t jj = 0; jj < 2; ++jj) {
                    wg[jj] = ldg32(c + kQ4Qs + s * 4096 + sg * 32 + 16 * jj + 4 * t);
                    wg8[jj] = ldg32(c + kQ4Qs + s * 4096 + sg8 * 32 + 16 * jj + 4 * t);
                }
#pragma unroll
                for (uint32_t nib = 0; nib < 2; ++nib) {
                    const uint32_t G = 2 * s + nib;
                    float cq[NT][4], c1[NT][4];
#pragma unroll
                    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                        for (int i = 0; i < 4; ++i) cq[nt][i] = c1[nt][i] = 0.f;
#pragma unroll
                    for (uint32_t jj = 0; jj < 2; ++jj) {
                        const AFrag a = a_frag((wg[jj] >> (4 * nib)) & 0x0F0F0F0Fu,
                                               (wg8[jj] >> (4 * nib)) & 0x0F0F0F0Fu, bias);
                        uint32_t b[NT][2];
                        x_frag<NT>(xr, kbase + 32 * G + 16 * jj + 4 * t, b);
#pragma unroll
                        for (int nt = 0; nt < NT; ++nt) {
                            mma16816(cq[nt], a.r0, a.r1, a.r2, a.r3, b[nt][0], b[nt][1], cq[nt]);
                            mma16816(c1[nt], ones, ones, ones, ones, b[nt][0], b[nt][1], c1[nt]);
                        }
                    }
                    const float2 sgv = reinterpret_cast<const float2 *>(wt)[g * 8 + G];
                    const float2 sg8v = reinterpret_cast<const float2 *>(wt)[(g + 8) * 8 + G];
#pragma unroll
                    for (int nt = 0; nt < NT; ++nt) {
                        acc[nt][0] = fmaf(sgv.x, cq[nt][0], fmaf(-sgv.y, c1[nt][0], acc[nt][0]));
                        acc[nt][1] = fmaf(sgv.x, cq[nt][1], fmaf(-sgv.y, c1[nt][1], acc[nt][1]));
                        acc[nt][2] = fmaf(sg8v.x, cq[nt][2], fmaf(-sg8v.y, c1[nt][2], acc[nt][2]));
                        acc[nt][3] = fmaf(sg8v.x, cq[nt][3], fmaf(-sg8v.y, c1[nt][3], acc[nt][3]));
                    }
                }
            }
        } else {
            // scale table: rows r0..r0+15 x 16 sub-blocks of d*sc
            {
                const uint32_t rr = r0 + (lane >> 1), half = lane & 1;
                const float d = half_bits_to_float(__ldg(reinterpret_cast<const uint16_t *>(c + kQ6D + rr * 2)));
                const uint2 sw = __ldg(reinterpret_cast<const uint2 *>(c + kQ6Sc + rr * 16 + 8 * half));
                const uint32_t words[2] = {sw.x, sw.y};
                float *o = wt + (lane >> 1) * 16 + half * 8;
#pragma unroll
                for (uint32_t i = 0; i < 8; ++i)
                    o[i] = d * (float)(int8_t)((words[i >> 2] >> (8 * (i & 3))) & 0xffu);
            }
            __syncwarp();
            const uint32_t bias = 0x43204320u;     // bf16x2 (160, 160) = 128 + 32
#pragma unroll
            for (uint32_t h = 0; h < 2; ++h) {
                uint32_t hg[2], hg8[2];
#pragma unroll
                for (uint32_t jj = 0; jj < 2; ++jj) {
                    hg[jj] = ldg32(c + kQ6Qh + (h * kPanelRows + sg) * 32 + 16 * jj + 4 * t);
                    hg8[jj] = ldg32(c + kQ6Qh + (h * kPanelRows + sg8) * 32 + 16 * jj + 4 * t);
                }
#pragma unroll
                for (uint32_t part = 0; part < 2; ++part) {
                    uint32_t lg[2], lg8[2];
#pragma unroll
                    for (uint32_t jj = 0; jj < 2; ++jj) {
                        lg[jj] = ldg32(c + kQ6Ql + ((h * 2 + part) * kPanelRows + sg) * 32 + 16 * jj + 4 * t);
                        lg8[jj] = ldg32(c + kQ6Ql + ((h * 2 + part) * kPanelRows + sg8) * 32 + 16 * jj + 4 * t);
                    }
#pragma unroll
                    for (uint32_t nib = 0; nib < 2; ++nib) {
                        const uint32_t grp = part + 2 * nib;
#pragma unroll
                        for (uint32_t jj = 0; jj < 2; ++jj) {
                            const uint32_t cg = ((lg[jj] >> (4 * nib)) & 0x0F0F0F0Fu) |
                                                (((hg[jj] >> (2 * grp)) & 0x03030303u) << 4);
                            const uint32_t cg8 = ((lg8[jj] >> (4 * nib)) & 0x0F0F0F0Fu) |
                                                 (((hg8[jj] >> (2 * grp)) & 0x03030303u) << 4);
                            const AFrag a = a_frag(cg, cg8, bias);
                            uint32_t b[NT][2];
                            x_frag<NT>(xr, kbase + 128 * h + 32 * grp + 16 * jj + 4 * t, b);
                            const uint32_t sb = 8 * h + 2 * grp + jj;
                            const float dg = wt[g * 16 + sb], dg8 = wt[(g + 8) * 16 + sb];
#pragma unroll
                            for (int nt = 0; nt < NT; ++nt) {
                                float cq[4] = {0.f, 0.f, 0.f, 0.f};
                                mma16816(cq, a.r0, a.r1, a.r2, a.r3, b[nt][0], b[nt][1], cq);
                                acc[nt][0] = fmaf(dg, cq[0], acc[nt][0]);
                                acc[nt][1] = fmaf(dg, cq[1], acc[nt][1]);
                                acc[nt][2] = fmaf(dg8, cq[2], acc[nt][2]);
                                acc[nt][3] = fmaf(dg8, cq[3], acc[nt][3]);
                            }
                        }
                    }
                }
            }
        }
    }

    // Reduce the warps' partial fragments; then either store Y directly (one
    // K slice) or publish the partial and let the tile's last CTA finish.
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int i = 0; i < 4; ++i) red[warp][lane][4 * nt + i] = acc[nt][i];
    __syncthreads();
    __shared__ uint32_t last;
    float v[4 * NT];
    if (warp == 0) {
#pragma unroll
        for (int j = 0; j < 4 * NT; ++j) {
            float s = 0.f;
#pragma unroll
            for (int ww = 0; ww < kWarps; ++ww) s += red[ww][lane][j];
            v[j] = s;
        }
        if (n_slices > 1) {
            // partials[slice][tile][lane][4*NT]
            float *dst = partials + (((uint64_t)blockIdx.y * gridDim.x + blockIdx.x) * 32 + lane) * (4 * NT);
#pragma unroll
            for (int j = 0; j < 4 * NT; ++j) __stcg(dst + j, v[j]);
            __threadfence();
            __syncwarp();
            if (lane == 0) last = (atomicAdd(counters + blockIdx.x, 1u) + 1 == n_slices) ? 1u : 0u;
            __syncwarp();
            if (last) {
                __threadfence();
#pragma unroll
                for (int j = 0; j < 4 * NT; ++j) v[j] = 0.f;
                for (uint32_t sl = 0; sl < n_slices; ++sl) {
                    const float *src = partials + (((uint64_t)sl * gridDim.x + blockIdx.x) * 32 + lane) * (4 * NT);
#pragma unroll
                    for (int j = 0; j < 4 * NT; ++j) v[j] += __ldcg(src + j);
                }
                if (lane == 0) counters[blockIdx.x] = 0u;
            }
        }
        if (n_slices == 1 || last) {
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const uint32_t tok = 8 * nt + 2 * t + (i & 1);
                    const uint32_t row = row0 + g + 8 * (i >> 1);
                    if (tok < m_count && row < w.n) {
                        const uint64_t off = (uint64_t)(m_begin + tok) * ldy + row;
                        if (DT == 0) static_cast<float *>(y)[off] = v[4 * nt + i];
                        else static_cast<__nv_bfloat16 *>(y)[off] = __float2bfloat16_rn(v[4 * nt + i]);
                    }
                }
            }
        }
    }
}

template <int TYPE, int NT>
cudaError_t launch_typed(const SegmentView &seg, const uint16_t *x, uint64_t k, void *y, uint64_t ldy,
                         int out_dtype, const GemvSplit &sp, cudaStream_t s) {
    const dim3 grid((seg.w.n + 15) / 16, sp.n_slices);
    const uint32_t mc = seg.m_end - seg.m_begin;
    if (out_dtype == 0)
        gemv_kernel<TYPE, NT, 0><<<grid, kWarps * 32, 0, s>>>(seg.w, x, seg.m_begin, mc, k, y, ldy, sp.kb_per_slice,
                                                               sp.partials, sp.counters);
    else
        gemv_kernel<TYPE, NT, 2><<<grid, kWarps * 32, 0, s>>>(seg.w, x, seg.m_begin, mc, k, y, ldy, sp.kb_per_slice,
                                                               sp.partials, sp.counters);
    return cudaGetLastError();
}

}  // namespace

GemvSplit gemv_split(const WeightView &w) {
    // Aim for >= 8 CTAs per SM of work, one super-block per warp (K slices of
    // 4 super-blocks); two per warp when the grid is large anyway.
    const uint32_t tiles = (w.n + 15) / 16;
    uint32_t per = 4;
    if ((uint64_t)tiles * ((w.kb + 7) / 8) >= 148u * 8u) per = 8;
    GemvSplit sp;
    sp.kb_per_slice = per;
    sp.n_slices = (w.kb + per - 1) / per;
    return sp;
}

size_t gemv_workspace_floats(const WeightView &w) {
    const GemvSplit sp = gemv_split(w);
    return sp.n_slices > 1 ? (size_t)sp.n_slices * ((w.n + 15) / 16) * 32 * 8 : 0;
}

cudaError_t launch_gemv(const SegmentView &seg, const uint16_t *x, uint64_t k, void *y, uint64_t ldy,
                        int out_dtype, const GemvSplit &sp, cudaStream_t s) {
    if (seg.m_end <= seg.m_begin) return cudaSuccess;
    const uint32_t m = seg.m_end - seg.m_begin;
    if (m > 16) return cudaErrorInvalidValue;
    if (sp.n_slices > 1 && (!sp.partials || !sp.counters)) return cudaErrorInvalidValue;
    if (seg.w.type == 12)
        return m <= 8 ? launch_typed<12, 1>(seg, x, k, y, ldy, out_dtype, sp, s)
                      : launch_typed<12, 2>(seg, x, k, y, ldy, out_dtype, sp, s);
    return m <= 8 ? launch_typed<14, 1>(seg, x, k, y, ldy, out_dtype, sp, s)
                  : launch_typed<14, 2>(seg, x, k, y, ldy, out_dtype, sp, s);
}

}  // namespace tc
