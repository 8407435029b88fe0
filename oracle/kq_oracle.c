/*
 * TEST INFRASTRUCTURE ONLY -- the CPU oracle for the K-quant decode path.
 *
 * Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / reference
 * legs may load this library, and only as the checker or the timed CPU
 * baseline.  The product (turbocider_b200) never links or calls it.
 *
 * It is a plain-C restatement of the reference decoder
 * (magicKD/TurboCider native/core/gguf_decode.cpp), which itself follows the
 * ggml block formats pinned at llama.cpp 64e9bceb.  Each function cites the
 * reference line it restates.  Parity is pinned by tests/test_oracle.py
 * against golden digests produced by the reference decoder itself
 * (oracle/_ref, built from the reference sources by oracle/Makefile) and
 * cross-checked against gguf-py 0.19.0 quants.dequantize.
 *
 * Build with -ffp-contract=off: the reference computes d*code and the
 * subtraction of the minimum as separate roundings (gguf_decode.cpp:5-7).
 */
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <string.h>

#if defined(__FP_FAST_FMAF) && !defined(KQ_ALLOW_CONTRACT)
/* nothing: contraction is controlled by the build flag */
#endif

enum { KQ_F32 = 0, KQ_F16 = 1, KQ_BF16 = 2 };

static __thread char kq_error[160];

static int fail(const char *reason) {
    snprintf(kq_error, sizeof kq_error, "%s", reason);
    return 1;
}

const char *kq_last_error(void) { return kq_error; }

/* Registry of block geometry: gguf_directory.hpp:21-26. */
int kq_type_geometry(uint32_t type, uint32_t *elements, uint32_t *bytes) {
    static const uint32_t table[][3] = {
        {0, 1, 4}, {1, 1, 2}, {2, 32, 18}, {3, 32, 20}, {6, 32, 22}, {7, 32, 24},
        {8, 32, 34}, {12, 256, 144}, {13, 256, 176}, {14, 256, 210}, {30, 1, 2}};
    for (unsigned i = 0; i < sizeof table / sizeof table[0]; ++i)
        if (table[i][0] == type) { *elements = table[i][1]; *bytes = table[i][2]; return 0; }
    return 1;
}

static uint16_t rd16(const uint8_t *p) { return (uint16_t)(p[0] | (p[1] << 8)); }

static float bits_f32(uint32_t b) { float f; memcpy(&f, &b, 4); return f; }
static uint32_t f32_bits(float f) { uint32_t b; memcpy(&b, &f, 4); return b; }

/* fp16 -> fp32, exact incl. subnormals: gguf_decode.cpp:377-388. */
float kq_half_to_float(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t exponent = (h >> 10) & 31u, mantissa = h & 1023u, bits;
    if (exponent == 0 && mantissa != 0) {
        /* normalise the subnormal: value = mantissa * 2^-24 */
        int shift = 0;
        while (!(mantissa & 1024u)) { mantissa <<= 1; ++shift; }
        bits = sign | ((uint32_t)(113 - shift) << 23) | ((mantissa & 1023u) << 13);
    } else if (exponent == 0) {
        bits = sign;
    } else if (exponent == 31) {
        bits = sign | 0x7f800000u | (mantissa << 13);
    } else {
        bits = sign | ((exponent + 112u) << 23) | (mantissa << 13);
    }
    return bits_f32(bits);
}

/* fp32 -> bf16 round-to-nearest-even, rejecting nonfinite input and overflow:
 * gguf_decode.cpp:389-394. */
int kq_float_to_bf16(float value, uint16_t *out) {
    if (!isfinite(value)) return fail("nonfinite weight/scale or conversion overflow");
    uint32_t b = f32_bits(value);
    uint16_t r = (uint16_t)((b + 0x7fffu + ((b >> 16) & 1u)) >> 16);
    if ((r & 0x7f80u) == 0x7f80u) return fail("BF16 conversion overflow");
    *out = r;
    return 0;
}

/* Integer round-right with ties to even, used by the fp16 narrowing. */
static uint32_t shift_right_even(uint32_t value, uint32_t shift) {
    uint32_t q = value >> shift, rem = value & ((1u << shift) - 1u), half = 1u << (shift - 1u);
    return q + (rem > half || (rem == half && (q & 1u)));
}

/* fp32 -> fp16 round-to-nearest-even, rejecting overflow: gguf_decode.cpp:395-405. */
int kq_float_to_half(float value, uint16_t *out) {
    if (!isfinite(value)) return fail("nonfinite weight/scale or conversion overflow");
    uint32_t b = f32_bits(value), frac = b & 0x7fffffu;
    uint16_t sign = (uint16_t)((b >> 16) & 0x8000u);
    int e = (int)((b >> 23) & 255u) - 127;
    if (e < -25) { *out = sign; return 0; }
    if (e > 15) return fail("FP16 conversion overflow");
    if (e < -14) { *out = (uint16_t)(sign | shift_right_even(0x800000u | frac, (uint32_t)(-e - 1))); return 0; }
    uint32_t r = (uint32_t)(e + 15) * 1024u + shift_right_even(frac, 13);
    if (r >= 0x7c00u) return fail("FP16 conversion overflow");
    *out = (uint16_t)(sign | r);
    return 0;
}

/* 6-bit (scale, min) pair of sub-block g from the 12 packed bytes:
 * gguf_decode.cpp:48-54. */
static void q4k_scale_min(unsigned g, const uint8_t *s, unsigned *sc, unsigned *mn) {
    if (g < 4) { *sc = s[g] & 63u; *mn = s[g + 4] & 63u; }
    else {
        *sc = (s[g + 4] & 15u) | ((unsigned)(s[g - 4] >> 6) << 4);
        *mn = (unsigned)(s[g + 4] >> 4) | ((unsigned)(s[g] >> 6) << 4);
    }
}

static uint32_t rd32(const uint8_t *p) {
    return (uint32_t)p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16) | ((uint32_t)p[3] << 24);
}

/* One block to fp32 values.  F32 / F16 / BF16 single elements:
 * gguf_decode.cpp:56-58; Q4_0 / Q4_1 / Q5_0 / Q5_1 / Q8_0 (32 weights):
 * :59-76; Q4_K / Q5_K super-blocks: :77-90; Q6_K: :91-105.  Every value must
 * be finite (:110).  Returns nonzero (with the reference's message) otherwise. */
int kq_decode_block(uint32_t type, const uint8_t *p, float *out) {
    static const char *nonfinite = "nonfinite weight/scale or conversion overflow";
    if (type == 0 || type == 1 || type == 30) {
        out[0] = type == 0 ? bits_f32(rd32(p)) : type == 1 ? kq_half_to_float(rd16(p))
                                                            : bits_f32((uint32_t)rd16(p) << 16);
        return isfinite(out[0]) ? 0 : fail(nonfinite);
    }
    if (type == 2 || type == 3 || type == 6 || type == 7 || type == 8) {
        const float d = kq_half_to_float(rd16(p));
        if (!isfinite(d)) return fail(nonfinite);
        if (type == 8) {
            for (unsigned i = 0; i < 32; ++i) out[i] = (float)(int8_t)p[2 + i] * d;
            return 0;
        }
        const int affine = type == 3 || type == 7, five = type == 6 || type == 7;
        const float mn = affine ? kq_half_to_float(rd16(p + 2)) : 0.f;
        if (!isfinite(mn)) return fail(nonfinite);
        const unsigned off = affine ? 4 : 2;
        const uint32_t high = five ? rd32(p + off) : 0;
        const uint8_t *low = p + off + (five ? 4 : 0);
        const int bias = affine ? 0 : five ? 16 : 8;
        for (unsigned i = 0; i < 16; ++i) {
            const int a = (int)((low[i] & 15u) | (((high >> i) & 1u) << 4)) - bias;
            const int b = (int)((low[i] >> 4) | (((high >> (i + 16)) & 1u) << 4)) - bias;
            const float pa = (float)a * d, pb = (float)b * d; /* separate rounding */
            out[i] = affine ? pa + mn : pa;
            out[i + 16] = affine ? pb + mn : pb;
        }
        return 0;
    }
    if (type == 12 || type == 13) {
        const float d = kq_half_to_float(rd16(p)), dmin = kq_half_to_float(rd16(p + 2));
        if (!isfinite(d) || !isfinite(dmin)) return fail("nonfinite weight/scale or conversion overflow");
        const uint8_t *scales = p + 4, *high = p + 16, *low = p + (type == 13 ? 48 : 16);
        for (unsigned g = 0; g < 8; ++g) {
            unsigned sc, mn;
            q4k_scale_min(g, scales, &sc, &mn);
            const float dg = d * (float)sc, mg = dmin * (float)mn;
            for (unsigned j = 0; j < 32; ++j) {
                const uint8_t byte = low[(g / 2) * 32 + j];
                int code = (g & 1) ? byte >> 4 : byte & 15;
                if (type == 13 && (high[j] & (1u << g))) code += 16;
                const float product = dg * (float)code; /* separate rounding */
                out[g * 32 + j] = product - mg;
            }
        }
        return 0;
    }
    if (type == 14) {
        const float d = kq_half_to_float(rd16(p + 208));
        if (!isfinite(d)) return fail("nonfinite weight/scale or conversion overflow");
        for (unsigned h = 0; h < 2; ++h) {
            const uint8_t *ql = p + 64 * h, *qh = p + 128 + 32 * h;
            const int8_t *sc = (const int8_t *)(p + 192 + 8 * h);
            for (unsigned j = 0; j < 32; ++j)
                for (unsigned g = 0; g < 4; ++g) {
                    const uint8_t byte = ql[j + (g & 1) * 32];
                    const int code = (int)((g < 2 ? (byte & 15) : (byte >> 4)) |
                                           (((qh[j] >> (2 * g)) & 3) << 4)) - 32;
                    const float ds = d * (float)sc[j / 16 + 2 * g];
                    out[128 * h + 32 * g + j] = ds * (float)code;
                }
        }
        return 0;
    }
    return fail("gguf_decode: unsupported tensor type");
}

static int write_value(uint8_t *dst, uint32_t dtype, float v) {
    uint16_t h;
    if (dtype == KQ_F32) { memcpy(dst, &v, 4); return 0; }
    if (dtype == KQ_BF16) { if (kq_float_to_bf16(v, &h)) return 1; }
    else if (kq_float_to_half(v, &h)) return 1;
    memcpy(dst, &h, 2);
    return 0;
}

/* Slice decode into a strided target with the reference's geometry checks:
 * decode_cpu_into gguf_decode.cpp:433-445, validate :160-183, row_into :320-367.
 * Every registered type is restated; returns 0 or 1. */
int kq_decode(uint32_t type, const void *source, uint64_t source_bytes, uint64_t rows,
              uint64_t columns, uint64_t row_begin, uint64_t nrows, uint64_t column_begin,
              uint64_t ncolumns, uint32_t dtype, void *target, uint64_t target_bytes,
              uint64_t row_stride, uint64_t column_stride) {
    uint32_t elements, block_bytes;
    if (kq_type_geometry(type, &elements, &block_bytes))
        return fail("gguf_decode: unsupported tensor type");
    if (!source || !target) return fail("null source/target storage");
    if (row_begin > rows || nrows > rows - row_begin) return fail("row slice out of bounds");
    if (!rows || !columns || columns % elements) return fail("invalid source geometry");
    if (!nrows || !ncolumns || column_begin > columns || ncolumns > columns - column_begin)
        return fail("invalid decode slice");
    const uint64_t row_bytes = columns / elements * block_bytes;
    if (rows * row_bytes > source_bytes) return fail("packed source too short");
    if (dtype > KQ_BF16) return fail("gguf_decode: invalid target dtype");
    const uint32_t item = dtype == KQ_F32 ? 4 : 2;
    if (column_stride < item) return fail("invalid/overlapping column stride");
    const uint64_t row_extent = (ncolumns - 1) * column_stride + item;
    if (row_stride < row_extent) return fail("invalid/overlapping row stride");
    if ((nrows - 1) * row_stride + row_extent > target_bytes) return fail("decode target too short");
    const uint8_t *src = (const uint8_t *)source;
    uint8_t *dst = (uint8_t *)target;
    float scratch[256];
    /* Same floating type as the target, written contiguously: a checked byte
     * copy (row_into's copy_finite branch, gguf_decode.cpp:325-330, :136-158). */
    const int identical = (type == 0 && dtype == KQ_F32) || (type == 1 && dtype == KQ_F16) ||
                          (type == 30 && dtype == KQ_BF16);
    if (identical && column_stride == block_bytes) {
        const uint32_t mask = type == 0 ? 0x7f800000u : type == 1 ? 0x7c00u : 0x7f80u;
        for (uint64_t r = 0; r < nrows; ++r)
            for (uint64_t c = 0; c < ncolumns; ++c) {
                const uint8_t *p = src + (row_begin + r) * row_bytes + (column_begin + c) * block_bytes;
                const uint32_t bits = block_bytes == 4 ? rd32(p) : rd16(p);
                if ((bits & mask) == mask) return fail("nonfinite source float");
                memcpy(dst + r * row_stride + c * block_bytes, p, block_bytes);
            }
        kq_error[0] = 0;
        return 0;
    }
    for (uint64_t r = 0; r < nrows; ++r) {
        const uint64_t first = column_begin / elements, last = (column_begin + ncolumns - 1) / elements;
        for (uint64_t b = first; b <= last; ++b) {
            if (kq_decode_block(type, src + (row_begin + r) * row_bytes + b * block_bytes, scratch)) return 1;
            const uint64_t lo = b * elements > column_begin ? b * elements : column_begin;
            const uint64_t hi = (b + 1) * elements < column_begin + ncolumns ? (b + 1) * elements : column_begin + ncolumns;
            for (uint64_t c = lo; c < hi; ++c)
                if (write_value(dst + r * row_stride + (c - column_begin) * column_stride, dtype,
                                scratch[c - b * elements])) return 1;
        }
    }
    kq_error[0] = 0;
    return 0;
}
