// Weight re-layout (raw GGUF rows -> panel chunks), the bit-exact dequantise
// kernels (panel layout and raw GGUF layout) and the bf16 -> fp16 activation
// conversion used by fp16 staging.  All of these are HBM-bound byte work: one
// thread per 32-weight group, coalesced along the fastest-varying index.
#include "../../include/turbocider_cuda.h"
#include "kq_format.cuh"
#include "tc_internal.h"

#include <cstdio>

namespace tc {
namespace {

enum : uint32_t { kNonfinite = 1u << 0, kF16Overflow = 1u << 1, kBf16Overflow = 1u << 4 };

__device__ __forceinline__ uint16_t ld16(const uint8_t *p) { return (uint16_t)(p[0] | (p[1] << 8)); }

// ---------------------------------------------------------------- re-layout
// One thread per (panel row, super-block column).  Threads are ordered with
// the row fastest so that every field store of a chunk is contiguous across a
// warp.  Rows past N are written as zero blocks.
__global__ void relayout_kernel(uint32_t type, const uint8_t *__restrict__ raw, uint64_t n,
                                uint32_t kb, uint8_t *__restrict__ chunks, uint32_t panels,
                                uint32_t *status, uint64_t glu_c) {
    const uint64_t idx = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const uint64_t total = (uint64_t)panels * kb * kPanelRows;
    if (idx >= total) return;
    const uint32_t r = (uint32_t)(idx % kPanelRows);
    const uint64_t pk = idx / kPanelRows;           // panel * kb + column
    const uint32_t col = (uint32_t)(pk % kb);
    const uint64_t panel = pk / kb;
    const uint64_t row = panel * kPanelRows + r;
    uint8_t *chunk = chunks + pk * chunk_bytes(type);
    const uint32_t bb = block_bytes(type);
    // SwiGLU weights: panel row 16 g + i holds gate row 8 g + i (i < 8) or up
    // row 8 g + i - 8, the up rows following the glu_c gate rows in `raw`.
    const uint64_t src = glu_c ? (row >> 4) * 8 + (row & 7) + ((row & 8) ? glu_c : 0) : row;
    const uint8_t *blk = row < n ? raw + (src * kb + col) * bb : nullptr;
    if (type == 12) {
        // qs quarters: 4 x 32 bytes
        for (uint32_t s = 0; s < 4; ++s) {
            uint8_t *dst = chunk + kQ4Qs + s * 4096 + row_slot(r) * 32;
            for (uint32_t i = 0; i < 32; i += 4) {
                uint32_t v = 0;
                if (blk) v = blk[16 + 32 * s + i] | (blk[17 + 32 * s + i] << 8) |
                             (blk[18 + 32 * s + i] << 16) | ((uint32_t)blk[19 + 32 * s + i] << 24);
                *reinterpret_cast<uint32_t *>(dst + i) = v;
            }
        }
        uint8_t *sc = chunk + kQ4Sc + r * 12;
        for (uint32_t i = 0; i < 12; ++i) sc[i] = blk ? blk[4 + i] : 0;
        uint16_t d = blk ? ld16(blk) : 0, dmin = blk ? ld16(blk + 2) : 0;
        *reinterpret_cast<uint32_t *>(chunk + kQ4Dm + r * 4) = (uint32_t)d | ((uint32_t)dmin << 16);
        if (!half_bits_finite(d) || !half_bits_finite(dmin)) atomicOr(status, kNonfinite);
    } else if (type == 13) {
        // qs quarters (block bytes 48..175), the qh plane (16..47), scales, d/dmin
        for (uint32_t s = 0; s < 4; ++s) {
            uint8_t *dst = chunk + kQ5Qs + s * 4096 + row_slot(r) * 32;
            for (uint32_t i = 0; i < 32; ++i) dst[i] = blk ? blk[48 + 32 * s + i] : 0;
        }
        uint8_t *qh = chunk + kQ5Qh + row_slot(r) * 32;
        for (uint32_t i = 0; i < 32; ++i) qh[i] = blk ? blk[16 + i] : 0;
        uint8_t *sc = chunk + kQ5Sc + r * 12;
        for (uint32_t i = 0; i < 12; ++i) sc[i] = blk ? blk[4 + i] : 0;
        uint16_t d = blk ? ld16(blk) : 0, dmin = blk ? ld16(blk + 2) : 0;
        *reinterpret_cast<uint32_t *>(chunk + kQ5Dm + r * 4) = (uint32_t)d | ((uint32_t)dmin << 16);
        if (!half_bits_finite(d) || !half_bits_finite(dmin)) atomicOr(status, kNonfinite);
    } else {
        // ql: [h][part][row][32]
        for (uint32_t h = 0; h < 2; ++h)
            for (uint32_t part = 0; part < 2; ++part) {
                uint8_t *dst = chunk + kQ6Ql + ((h * 2 + part) * kPanelRows + row_slot(r)) * 32;
                for (uint32_t i = 0; i < 32; ++i) dst[i] = blk ? blk[64 * h + 32 * part + i] : 0;
            }
        for (uint32_t h = 0; h < 2; ++h) {
            uint8_t *dst = chunk + kQ6Qh + (h * kPanelRows + row_slot(r)) * 32;
            for (uint32_t i = 0; i < 32; ++i) dst[i] = blk ? blk[128 + 32 * h + i] : 0;
        }
        uint8_t *sc = chunk + kQ6Sc + r * 16;
        for (uint32_t i = 0; i < 16; ++i) sc[i] = blk ? blk[192 + i] : 0;
        const uint16_t d = blk ? ld16(blk + 208) : 0;
        *reinterpret_cast<uint16_t *>(chunk + kQ6D + r * 2) = d;
        if (!half_bits_finite(d)) atomicOr(status, kNonfinite);
    }
}

// ------------------------------------------------------------ value writer
template <int DT>
__device__ __forceinline__ void store_value(uint8_t *p, float v, bool &ovf) {
    if (DT == 0) *reinterpret_cast<float *>(p) = v;
    else if (DT == 1) *reinterpret_cast<uint16_t *>(p) = to_f16_bits(v, ovf);
    else *reinterpret_cast<uint16_t *>(p) = to_bf16_bits(v);
}
// Store with fp16 / bf16 overflow detection.  Strided targets of the raw
// decode need not be aligned to the item size: an unaligned target is
// written with byte stores, an aligned one with one store of the item's width.
template <int DT>
__device__ __forceinline__ void store_value_bytes(uint8_t *p, float v, bool &f16_ovf, bool &bf16_ovf) {
    if (DT == 0) {
        const uint32_t bits = __float_as_uint(v);
        if ((reinterpret_cast<uintptr_t>(p) & 3u) == 0) {
            *reinterpret_cast<uint32_t *>(p) = bits;
        } else {
            volatile uint8_t *q = p;
            q[0] = (uint8_t)bits;
            q[1] = (uint8_t)(bits >> 8);
            q[2] = (uint8_t)(bits >> 16);
            q[3] = (uint8_t)(bits >> 24);
        }
        return;
    }
    const uint16_t h = DT == 1 ? to_f16_bits(v, f16_ovf) : to_bf16_bits(v, bf16_ovf);
    if ((reinterpret_cast<uintptr_t>(p) & 1u) == 0) {
        *reinterpret_cast<uint16_t *>(p) = h;
    } else {
        // Widen the 16-bit result with an explicit move before taking its
        // bytes: byte stores taken straight from the conversion's 16-bit
        // value lost the low byte on this toolchain.
        uint32_t w;
        asm("cvt.u32.u16 %0, %1;" : "=r"(w) : "h"(h));
        volatile uint8_t *q = p;
        q[0] = (uint8_t)(w & 0xffu);
        q[1] = (uint8_t)((w >> 8) & 0xffu);
    }
}
__device__ __forceinline__ uint32_t ld32b(const uint8_t *p) {
    return (uint32_t)p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16) | ((uint32_t)p[3] << 24);
}

// The 32 weights of one Q4_0 / Q4_1 / Q5_0 / Q5_1 / Q8_0 block
// (gguf_decode.cpp:59-76): d (and the affine types' minimum) fp16, codes of
// 4, 5 (fifth bits in a 32-bit word) or 8 bits.  The affine types round the
// product and the sum separately, as the reference does.
__device__ __forceinline__ void legacy_block(uint32_t type, const uint8_t *p, float v[32], bool &bad) {
    const uint16_t dh = ld16(p);
    const float d = half_bits_to_float(dh);
    bad |= !half_bits_finite(dh);
    if (type == 8) {
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] = __fmul_rn((float)(int8_t)p[2 + i], d);
        return;
    }
    const bool affine = type == 3 || type == 7, five = type == 6 || type == 7;
    float mn = 0.f;
    if (affine) {
        const uint16_t mh = ld16(p + 2);
        mn = half_bits_to_float(mh);
        bad |= !half_bits_finite(mh);
    }
    const uint32_t off = affine ? 4 : 2;
    const uint32_t high = five ? ld32b(p + off) : 0u;
    const uint8_t *low = p + off + (five ? 4 : 0);
    const int bias = affine ? 0 : five ? 16 : 8;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
        const int a = (int)((low[i] & 15u) | (((high >> i) & 1u) << 4)) - bias;
        const int b = (int)((low[i] >> 4) | (((high >> (i + 16)) & 1u) << 4)) - bias;
        v[i] = affine ? __fadd_rn(__fmul_rn((float)a, d), mn) : __fmul_rn((float)a, d);
        v[i + 16] = affine ? __fadd_rn(__fmul_rn((float)b, d), mn) : __fmul_rn((float)b, d);
    }
}

// Decode the 32 weights of group G (0..7) of one super-block whose fields are
// reached through the accessor.  Q4_K group G = sub-block G; Q6_K group
// G = 4h + g covers weights 128h + 32g + j.
struct Q4Fields { const uint8_t *qs32; const uint8_t *sc12; uint16_t d, dmin; const uint8_t *qh32 = nullptr; };
struct Q6Fields { const uint8_t *ql32; const uint8_t *qh32; const uint8_t *sc16; uint16_t d; };

__device__ __forceinline__ void q4k_group(const Q4Fields &f, uint32_t g, float out[32], bool &bad) {
    const float d = half_bits_to_float(f.d), dmin = half_bits_to_float(f.dmin);
    bad |= !half_bits_finite(f.d) || !half_bits_finite(f.dmin);
    uint32_t sc, mn;
    q4k_scale_min(g, f.sc12, sc, mn);
    const float dg = d * (float)sc, mg = dmin * (float)mn;
    const uint32_t shift = (g & 1) * 4;
    if (f.qh32) {  // Q5_K: fifth bit of weight j of sub-block g is bit g of qh[j] (gguf_decode.cpp:87)
#pragma unroll
        for (int j = 0; j < 32; ++j)
            out[j] = q4k_value(dg, mg, ((f.qs32[j] >> shift) & 15u) | (((f.qh32[j] >> g) & 1u) << 4));
        return;
    }
#pragma unroll
    for (int j = 0; j < 32; ++j) out[j] = q4k_value(dg, mg, (f.qs32[j] >> shift) & 15u);
}

__device__ __forceinline__ void q6k_group(const Q6Fields &f, uint32_t h, uint32_t g, float out[32],
                                          bool &bad) {
    const float d = half_bits_to_float(f.d);
    bad |= !half_bits_finite(f.d);
    const uint32_t shift = g < 2 ? 0 : 4;
#pragma unroll
    for (int j = 0; j < 32; ++j) {
        const int code = (int)(((f.ql32[j] >> shift) & 15u) | (((f.qh32[j] >> (2 * g)) & 3u) << 4)) - 32;
        const float ds = d * (float)(int8_t)f.sc16[8 * h + j / 16 + 2 * g];
        out[j] = ds * (float)code;
    }
}

// -------------------------------------------------------- panel dequantise
// One thread per (row, super-block column, group).  dst is row-major [n, k].
template <int DT>
__global__ void dequant_panel_kernel(WeightView w, uint8_t *__restrict__ dst, uint64_t ld,
                                     uint32_t *status) {
    const uint64_t idx = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const uint64_t total = (uint64_t)w.n * w.kb * 8;
    if (idx >= total) return;
    const uint32_t G = (uint32_t)(idx % 8);
    const uint32_t col = (uint32_t)((idx / 8) % w.kb);
    const uint64_t row = idx / 8 / w.kb;
    const uint32_t r = (uint32_t)(row % kPanelRows);
    const uint8_t *chunk = w.chunks + ((row / kPanelRows) * w.kb + col) * chunk_bytes(w.type);
    float v[32];
    bool bad = false, ovf = false;
    if (w.type == 12) {
        const uint32_t dm = *reinterpret_cast<const uint32_t *>(chunk + kQ4Dm + r * 4);
        Q4Fields f{chunk + kQ4Qs + (G / 2) * 4096 + row_slot(r) * 32, chunk + kQ4Sc + r * 12,
                   (uint16_t)(dm & 0xffffu), (uint16_t)(dm >> 16)};
        q4k_group(f, G, v, bad);
    } else if (w.type == 13) {
        const uint32_t dm = *reinterpret_cast<const uint32_t *>(chunk + kQ5Dm + r * 4);
        Q4Fields f{chunk + kQ5Qs + (G / 2) * 4096 + row_slot(r) * 32, chunk + kQ5Sc + r * 12,
                   (uint16_t)(dm & 0xffffu), (uint16_t)(dm >> 16), chunk + kQ5Qh + row_slot(r) * 32};
        q4k_group(f, G, v, bad);
    } else {
        const uint32_t h = G / 4, g = G % 4;
        Q6Fields f{chunk + kQ6Ql + ((h * 2 + (g & 1)) * kPanelRows + row_slot(r)) * 32,
                   chunk + kQ6Qh + (h * kPanelRows + row_slot(r)) * 32, chunk + kQ6Sc + r * 16,
                   *reinterpret_cast<const uint16_t *>(chunk + kQ6D + r * 2)};
        q6k_group(f, h, g, v, bad);
    }
    constexpr uint32_t item = DT == 0 ? 4 : 2;
    uint8_t *out = dst + (row * ld + (uint64_t)col * 256 + G * 32) * item;
#pragma unroll
    for (int j = 0; j < 32; ++j) store_value<DT>(out + j * item, v[j], ovf);
    if (bad) atomicOr(status, kNonfinite);
    if (ovf) atomicOr(status, kF16Overflow);
}

// ------------------------------------------------------------ raw decode
// Device mirror of decode_cpu_into over raw GGUF rows: one thread per
// (slice row, touched group).  Writes only the columns inside the slice.
template <int DT>
__global__ void decode_raw_kernel(uint32_t type, const uint8_t *__restrict__ src, uint64_t row_bytes,
                                  uint64_t row_begin, uint64_t rows, uint64_t column_begin,
                                  uint64_t columns, uint8_t *__restrict__ dst, uint64_t row_stride,
                                  uint64_t column_stride, uint64_t first_group, uint64_t groups,
                                  uint32_t *status, const uint64_t *__restrict__ gather, uint64_t source_rows,
                                  uint64_t dst_bytes) {
    const uint64_t idx = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= rows * groups) return;
    const uint64_t r = idx / groups;
    const uint64_t gid = first_group + idx % groups;   // global 32-group index in the row
    // Gather (decode_cpu_gather, gguf_decode.cpp:446-465): target row r takes
    // source row gather[r]; an index past the matrix is reported, never read.
    uint64_t src_row = row_begin + r;
    if (gather) {
        src_row = __ldg(gather + r);
        if (src_row >= source_rows) {
            atomicOr(status, (uint32_t)TC_STATUS_GEOMETRY);
            return;
        }
    }
    const uint8_t *row = src + src_row * row_bytes;
    float v[32];
    bool bad = false, ovf = false, bovf = false;
    const uint64_t c0 = gid * 32;
    if (type_elements(type) == 1) {
        // F32 / F16 / BF16 (gguf_decode.cpp:56-58): every element is its own
        // block; only the elements inside the slice are read and checked.
        for (int j = 0; j < 32; ++j) {
            const uint64_t c = c0 + j;
            if (c < column_begin || c >= column_begin + columns) continue;
            float x;
            bool fin;
            if (type == 0) {
                const uint32_t b = ld32b(row + c * 4);
                x = __uint_as_float(b);
                fin = (b & 0x7f800000u) != 0x7f800000u;
            } else {
                const uint16_t h = ld16(row + c * 2);
                x = type == 1 ? half_bits_to_float(h) : __uint_as_float((uint32_t)h << 16);
                fin = type == 1 ? half_bits_finite(h) : (h & 0x7f80u) != 0x7f80u;
            }
            if (!fin) { bad = true; continue; }
            store_value_bytes<DT>(dst + r * row_stride + (c - column_begin) * column_stride, x, ovf, bovf);
        }
        if (bad) atomicOr(status, kNonfinite);
        if (ovf) atomicOr(status, kF16Overflow);
        if (bovf) atomicOr(status, kBf16Overflow);
        return;
    }
    if (type_elements(type) == 32) {
        legacy_block(type, row + gid * type_bytes(type), v, bad);
    } else {
    const uint64_t block = gid / 8;
    const uint32_t G = (uint32_t)(gid % 8);
    const uint8_t *p = row + block * block_bytes(type);
    if (type == 12) {
        Q4Fields f{p + 16 + (G / 2) * 32, p + 4, ld16(p), ld16(p + 2)};
        q4k_group(f, G, v, bad);
    } else if (type == 13) {
        Q4Fields f{p + 48 + (G / 2) * 32, p + 4, ld16(p), ld16(p + 2), p + 16};
        q4k_group(f, G, v, bad);
    } else {
        const uint32_t h = G / 4, g = G % 4;
        Q6Fields f{p + 64 * h + 32 * (g & 1), p + 128 + 32 * h, p + 192, ld16(p + 208)};
        q6k_group(f, h, g, v, bad);
    }
    }
#pragma unroll 4
    for (int j = 0; j < 32; ++j) {
        const uint64_t c = c0 + j;
        if (c < column_begin || c >= column_begin + columns) continue;
        const uint64_t at = r * row_stride + (c - column_begin) * column_stride;
        if (!tc_in_bounds(!dst_bytes || at + (DT == 0 ? 4 : 2) <= dst_bytes, status)) continue;
        store_value_bytes<DT>(dst + at, v[j], ovf, bovf);
    }
    if (bad) atomicOr(status, kNonfinite);
    if (ovf) atomicOr(status, kF16Overflow);
    if (bovf) atomicOr(status, kBf16Overflow);
}

// ---------------------------------------------------- bf16 -> fp16 (staging)
__global__ void x_to_f16_kernel(const uint16_t *__restrict__ x, uint16_t *__restrict__ y,
                                uint64_t count, uint32_t *status) {
    const uint64_t i = ((uint64_t)blockIdx.x * blockDim.x + threadIdx.x) * 8;
    bool ovf = false;
    if (i + 8 <= count) {
        const uint4 in = *reinterpret_cast<const uint4 *>(x + i);
        const uint32_t w[4] = {in.x, in.y, in.z, in.w};
        uint32_t o[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const float lo = __uint_as_float(w[q] << 16), hi = __uint_as_float(w[q] & 0xffff0000u);
            o[q] = (uint32_t)to_f16_bits(lo, ovf) | ((uint32_t)to_f16_bits(hi, ovf) << 16);
        }
        *reinterpret_cast<uint4 *>(y + i) = make_uint4(o[0], o[1], o[2], o[3]);
    } else {
        for (uint64_t j = i; j < count; ++j) y[j] = to_f16_bits(__uint_as_float((uint32_t)x[j] << 16), ovf);
    }
    if (ovf) atomicOr(status, kF16Overflow);
}

inline unsigned blocks_for(uint64_t threads, unsigned per) { return (unsigned)((threads + per - 1) / per); }

}  // namespace

cudaError_t launch_relayout(uint32_t type, const uint8_t *raw, uint64_t n, uint32_t kb,
                            uint8_t *chunks, uint32_t panels, uint32_t *status, cudaStream_t s, uint64_t glu_c) {
    const uint64_t total = (uint64_t)panels * kb * kPanelRows;
    if (!total) return cudaSuccess;
    relayout_kernel<<<blocks_for(total, 256), 256, 0, s>>>(type, raw, n, kb, chunks, panels, status, glu_c);
    return cudaGetLastError();
}

cudaError_t launch_dequant_panel(const WeightView &w, int dtype, void *dst, uint64_t ld,
                                 uint32_t *status, cudaStream_t s) {
    const uint64_t total = (uint64_t)w.n * w.kb * 8;
    if (!total) return cudaSuccess;
    const unsigned g = blocks_for(total, 256);
    auto *d = static_cast<uint8_t *>(dst);
    if (dtype == 0) dequant_panel_kernel<0><<<g, 256, 0, s>>>(w, d, ld, status);
    else if (dtype == 1) dequant_panel_kernel<1><<<g, 256, 0, s>>>(w, d, ld, status);
    else dequant_panel_kernel<2><<<g, 256, 0, s>>>(w, d, ld, status);
    return cudaGetLastError();
}

cudaError_t launch_decode_raw(uint32_t type, const uint8_t *src, uint64_t row_bytes,
                              uint64_t row_begin, uint64_t rows, uint64_t column_begin,
                              uint64_t columns, int dtype, uint8_t *dst, uint64_t row_stride,
                              uint64_t column_stride, uint32_t *status, cudaStream_t s, const uint64_t *gather,
                              uint64_t source_rows, uint64_t dst_bytes) {
    // Every block touched by the column range is decoded (and checked), as in
    // the reference's row_into (gguf_decode.cpp:340-364); threads work on
    // 32-weight groups (an eighth of a K-quant super-block, one legacy block,
    // or 32 floating-point elements).
    const uint64_t el = type_elements(type) == 256 ? 256 : 32;
    const uint64_t first_block = column_begin / el, last_block = (column_begin + columns - 1) / el;
    const uint64_t first_group = first_block * (el / 32), groups = (last_block - first_block + 1) * (el / 32);
    const uint64_t total = rows * groups;
    const unsigned g = blocks_for(total, 128);
    if (dtype == 0)
        decode_raw_kernel<0><<<g, 128, 0, s>>>(type, src, row_bytes, row_begin, rows, column_begin, columns,
                                               dst, row_stride, column_stride, first_group, groups, status, gather,
                                               source_rows, dst_bytes);
    else if (dtype == 1)
        decode_raw_kernel<1><<<g, 128, 0, s>>>(type, src, row_bytes, row_begin, rows, column_begin, columns,
                                               dst, row_stride, column_stride, first_group, groups, status, gather,
                                               source_rows, dst_bytes);
    else
        decode_raw_kernel<2><<<g, 128, 0, s>>>(type, src, row_bytes, row_begin, rows, column_begin, columns,
                                               dst, row_stride, column_stride, first_group, groups, status, gather,
                                               source_rows, dst_bytes);
    return cudaGetLastError();
}

cudaError_t launch_x_to_f16(const uint16_t *x, uint16_t *x16, uint64_t count, uint32_t *status,
                            cudaStream_t s) {
    if (!count) return cudaSuccess;
    x_to_f16_kernel<<<blocks_for((count + 7) / 8, 256), 256, 0, s>>>(x, x16, count, status);
    return cudaGetLastError();
}

}  // namespace tc
