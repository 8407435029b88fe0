// GGUF K-quant block formats, the HBM panel layout used by the kernels, and
// the bit-exact decode arithmetic shared by every kernel.
//
// Block formats (reference native/core/gguf_decode.cpp:77-105):
//   Q4_K, 144 B / 256 weights: d fp16 @0, dmin fp16 @2, 12 packed 6-bit
//     (scale, min) pairs @4, 128 bytes of nibbles @16.  Sub-block g (32
//     weights) uses byte 16 + (g/2)*32 + j, low nibble if g even, high if odd;
//     w = (d*sc_g)*q - dmin*m_g.
//   Q6_K, 210 B / 256 weights: ql[128] @0, qh[64] @128, int8 scales[16] @192,
//     d fp16 @208.  Weight 128h + 32g + j: q = nibble of ql[64h + j + 32(g&1)]
//     (low if g < 2) | ((qh[32h + j] >> 2g) & 3) << 4, minus 32;
//     w = (d*sc[8h + j/16 + 2g])*q.
//
// Exactness (why one FMA / one multiply reproduces the reference's separate
// roundings bit for bit): d and dmin carry at most 11 significant bits, a
// 6-bit scale adds 6 and a 4-bit code 4, so d*sc*q (<= 21 bits) and dmin*m
// (<= 17 bits) are exact in fp32; the only rounding in the reference's
// `d*code - m` is the final subtraction, which fmaf(d_g, q, -m_g) performs
// identically.  For Q6_K, |d*sc*q| needs at most 11+7+5 = 23 bits, so the
// product is exact whatever the association.
//
// Panel layout in HBM: rows are grouped in panels of 128 (the tensor-core
// tile height); for each panel p and super-block column kb the 128 blocks
// form one contiguous "chunk" at ((p * KB) + kb) * chunk_bytes, with each
// block's bytes split by field so that one 64-weight K slice of all 128 rows
// is contiguous (conflict-free shared-memory reads, one bulk copy per chunk):
//   Q4_K chunk (18432 B = 128 * 144):
//     qs  [4 quarters][128 rows][32 B] @0      quarter s = qs bytes 32s..32s+31
//     sc  [128 rows][12 B]             @16384
//     dm  [128 rows][d, dmin fp16]     @17920
//   Q6_K chunk (26880 B = 128 * 210):
//     ql  [2 halves][2 parts][128 rows][32 B] @0   = ql bytes 64h + 32part ..
//     qh  [2 halves][128 rows][32 B]          @16384 = qh bytes 32h ..
//     sc  [128 rows][16 B]                    @24576
//     d   [128 rows] fp16                     @26624
// Rows past N in the last panel are zero blocks (d = 0: every weight is 0).
// The per-row 32-byte pieces of qs / ql / qh are stored at row_slot(r), a
// permutation inside each aligned group of four rows chosen so that the four
// rows read by a half-warp of dequantisers fall in four different 32-byte
// shared-memory bank windows; sc / dm / d stay in natural row order.
#pragma once
#include <cstdint>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

namespace tc {

constexpr uint32_t kBlockWeights = 256;
constexpr uint32_t kPanelRows = 128;
constexpr uint32_t kQ4KBytes = 144, kQ5KBytes = 176, kQ6KBytes = 210;
constexpr uint32_t kQ4KChunk = kPanelRows * kQ4KBytes;  // 18432
constexpr uint32_t kQ5KChunk = kPanelRows * kQ5KBytes;  // 22528
constexpr uint32_t kQ6KChunk = kPanelRows * kQ6KBytes;  // 26880

// Q4_K chunk field offsets
constexpr uint32_t kQ4Qs = 0, kQ4Sc = 16384, kQ4Dm = 17920;
// Q5_K chunk field offsets: Q4_K's fields plus the fifth-bit plane qh (32
// bytes per row, bit g of qh[j] belongs to weight j of sub-block g)
constexpr uint32_t kQ5Qs = 0, kQ5Qh = 16384, kQ5Sc = 20480, kQ5Dm = 22016;
// Q6_K chunk field offsets
constexpr uint32_t kQ6Ql = 0, kQ6Qh = 16384, kQ6Sc = 24576, kQ6D = 26624;

__host__ __device__ constexpr uint32_t row_slot(uint32_t r) {
    return (r & ~3u) | ((r + 2u * ((r >> 2) & 1u)) & 3u);
}

// Block geometry of every GGML type the reference registers
// (native/core/gguf_directory.hpp:21-26): weights per block, bytes per block.
__host__ __device__ constexpr uint32_t type_elements(uint32_t t) {
    return (t == 0 || t == 1 || t == 30) ? 1u
           : (t == 2 || t == 3 || t == 6 || t == 7 || t == 8) ? 32u
           : (t == 12 || t == 13 || t == 14) ? 256u : 0u;
}
__host__ __device__ constexpr uint32_t type_bytes(uint32_t t) {
    return t == 0 ? 4u : (t == 1 || t == 30) ? 2u : t == 2 ? 18u : t == 3 ? 20u : t == 6 ? 22u : t == 7 ? 24u
           : t == 8 ? 34u : t == 12 ? 144u : t == 13 ? 176u : t == 14 ? 210u : 0u;
}

__host__ __device__ constexpr uint32_t block_bytes(uint32_t type) {
    return type == 12 ? kQ4KBytes : type == 14 ? kQ6KBytes : type == 13 ? kQ5KBytes : 0u;
}
__host__ __device__ constexpr uint32_t chunk_bytes(uint32_t type) {
    return type == 12 ? kQ4KChunk : type == 14 ? kQ6KChunk : type == 13 ? kQ5KChunk : 0u;
}

// fp16 bits -> fp32, exact (hardware conversion; equals the reference's
// bit-level fp16_to_float, gguf_decode.cpp:377-388, for every finite input).
__device__ __forceinline__ float half_bits_to_float(uint16_t h) {
    return __half2float(__ushort_as_half(h));
}
__device__ __forceinline__ bool half_bits_finite(uint16_t h) { return (h & 0x7c00u) != 0x7c00u; }

// The 6-bit (scale, min) pair of Q4_K sub-block g (gguf_decode.cpp:48-54).
__device__ __forceinline__ void q4k_scale_min(uint32_t g, const uint8_t *s, uint32_t &sc, uint32_t &mn) {
    if (g < 4) { sc = s[g] & 63u; mn = s[g + 4] & 63u; }
    else {
        sc = (s[g + 4] & 15u) | ((uint32_t)(s[g - 4] >> 6) << 4);
        mn = (uint32_t)(s[g + 4] >> 4) | ((uint32_t)(s[g] >> 6) << 4);
    }
}

// Same, from the 12 scale bytes held in three little-endian 32-bit words
// (register-resident: no byte-addressed local array).
__device__ __forceinline__ void q4k_scale_min_w(uint32_t g, uint32_t w0, uint32_t w1, uint32_t w2,
                                                uint32_t &sc, uint32_t &mn) {
    auto byte = [&](uint32_t i) -> uint32_t {
        const uint32_t w = i < 4 ? w0 : i < 8 ? w1 : w2;
        return (w >> (8 * (i & 3))) & 0xffu;
    };
    if (g < 4) { sc = byte(g) & 63u; mn = byte(g + 4) & 63u; }
    else {
        sc = (byte(g + 4) & 15u) | ((byte(g - 4) >> 6) << 4);
        mn = (byte(g + 4) >> 4) | ((byte(g) >> 6) << 4);
    }
}

// Q4_K weight value: exactly the reference's (d*sc)*q - dmin*m (see header).
__device__ __forceinline__ float q4k_value(float dg, float mg, uint32_t q) {
    return fmaf(dg, (float)q, -mg);
}

// Round-to-nearest-even conversions of finite values.  fp16 overflow is
// reported by the caller (the reference rejects |v| that rounds past 65504).
__device__ __forceinline__ uint16_t to_bf16_bits(float v) {
    return __bfloat16_as_ushort(__float2bfloat16_rn(v));
}
// bf16 conversion with the reference's overflow rejection (a finite value
// that rounds to infinity: float_to_bf16_rne, gguf_decode.cpp:389-394).
__device__ __forceinline__ uint16_t to_bf16_bits(float v, bool &overflow) {
    const uint16_t h = __bfloat16_as_ushort(__float2bfloat16_rn(v));
    overflow |= (h & 0x7f80u) == 0x7f80u;
    return h;
}
__device__ __forceinline__ uint16_t to_f16_bits(float v, bool &overflow) {
    const uint16_t h = __half_as_ushort(__float2half_rn(v));
    overflow |= (h & 0x7c00u) == 0x7c00u;
    return h;
}

}  // namespace tc
