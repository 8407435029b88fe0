// Host-side GGUF K-quant quantiser (Q4_K, Q6_K) used to build synthetic
// weights.  The reference ships no encoder, so this is an independent design
// written from the block formats alone:
//
//   Q4_K  each 32-weight sub-block g is fitted by the affine range
//         [-b_g, 15 a_g - b_g] with b_g = max(0, -min w) and
//         a_g = (max w + b_g) / 15; the super-block scales are
//         d = max a_g / 63 and dmin = max b_g / 63 (rounded to fp16), the
//         6-bit sc_g / m_g are the nearest integers to a_g / d and b_g / dmin,
//         and each code is the nearest integer to (w + dmin m_g) / (d sc_g),
//         clamped to [0, 15].
//   Q6_K  each 16-weight sub-block s gets the symmetric scale
//         c_s = max|w| / 31; d = max c_s / 127 (fp16), sc_s = nearest integer
//         to c_s / d, and each code is nearest(w / (d sc_s)) clamped to
//         [-32, 31], stored with the +32 bias.
//
// Rounding is ties-to-even throughout, so the output is a deterministic
// function of the input.  Quality is a data-generation concern only: every
// parity check decodes the same blocks on both sides.
#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <string>
#include <thread>
#include <vector>

#include "../../include/turbocider_cuda.h"

namespace {

uint16_t f32_to_f16_bits(float v) {
    // Round-to-nearest-even fp32 -> fp16 for finite non-negative or negative
    // values of moderate size (scales here are far from the fp16 limits).
    uint32_t b;
    std::memcpy(&b, &v, 4);
    const uint32_t sign = (b >> 16) & 0x8000u;
    const int e = (int)((b >> 23) & 255u) - 127;
    uint32_t mant = b & 0x7fffffu;
    if (e > 15) return (uint16_t)(sign | 0x7bffu);  // saturate (never reached by the fits below)
    if (e < -25) return (uint16_t)sign;
    uint32_t full, shift;
    if (e < -14) { full = mant | 0x800000u; shift = (uint32_t)(-e - 1); }
    else { full = mant; shift = 13; }
    uint32_t q = full >> shift, rem = full & ((1u << shift) - 1u), half = 1u << (shift - 1);
    q += (rem > half || (rem == half && (q & 1u)));
    if (e < -14) return (uint16_t)(sign | q);
    return (uint16_t)(sign | (((uint32_t)(e + 15) << 10) + q));
}

float f16_bits_to_f32(uint16_t h) {
    const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t e = (h >> 10) & 31u, m = h & 1023u, bits;
    if (e == 0) {
        float f = std::ldexp((float)m, -24);
        return sign ? -f : f;
    }
    bits = sign | ((e + 112u) << 23) | (m << 13);
    float f;
    std::memcpy(&f, &bits, 4);
    return f;
}

inline int nearest(float x) { return (int)std::nearbyint(x); }

void quantize_q4k_block(const float *w, uint8_t *p) {
    float a[8], b[8];
    for (int g = 0; g < 8; ++g) {
        float lo = w[32 * g], hi = w[32 * g];
        for (int j = 1; j < 32; ++j) { lo = std::min(lo, w[32 * g + j]); hi = std::max(hi, w[32 * g + j]); }
        b[g] = std::max(0.f, -lo);
        a[g] = std::max(0.f, (hi + b[g]) / 15.f);
    }
    const float amax = *std::max_element(a, a + 8), bmax = *std::max_element(b, b + 8);
    const uint16_t dh = f32_to_f16_bits(amax / 63.f), mh = f32_to_f16_bits(bmax / 63.f);
    const float d = f16_bits_to_f32(dh), dmin = f16_bits_to_f32(mh);
    uint32_t sc[8], mn[8];
    for (int g = 0; g < 8; ++g) {
        sc[g] = d > 0 ? (uint32_t)std::clamp(nearest(a[g] / d), 0, 63) : 0u;
        mn[g] = dmin > 0 ? (uint32_t)std::clamp(nearest(b[g] / dmin), 0, 63) : 0u;
    }
    std::memset(p, 0, 144);
    p[0] = (uint8_t)(dh & 0xff); p[1] = (uint8_t)(dh >> 8);
    p[2] = (uint8_t)(mh & 0xff); p[3] = (uint8_t)(mh >> 8);
    uint8_t *s = p + 4;
    for (int g = 0; g < 4; ++g) {
        s[g] = (uint8_t)(sc[g] | ((sc[g + 4] >> 4) << 6));
        s[g + 4] = (uint8_t)(mn[g] | ((mn[g + 4] >> 4) << 6));
        s[g + 8] = (uint8_t)((sc[g + 4] & 15u) | ((mn[g + 4] & 15u) << 4));
    }
    uint8_t *qs = p + 16;
    for (int g = 0; g < 8; ++g) {
        const float A = d * (float)sc[g], B = dmin * (float)mn[g];
        for (int j = 0; j < 32; ++j) {
            const int q = A > 0 ? std::clamp(nearest((w[32 * g + j] + B) / A), 0, 15) : 0;
            qs[(g / 2) * 32 + j] |= (uint8_t)(q << ((g & 1) * 4));
        }
    }
}

// Q5_K: the Q4_K fit with 31 code levels; the fifth bit of weight j of
// sub-block g goes to bit g of qh[j] (block bytes 16..47), the low nibbles to
// qs (bytes 48..175) as in Q4_K.
void quantize_q5k_block(const float *w, uint8_t *p) {
    float a[8], b[8];
    for (int g = 0; g < 8; ++g) {
        float lo = w[32 * g], hi = w[32 * g];
        for (int j = 1; j < 32; ++j) { lo = std::min(lo, w[32 * g + j]); hi = std::max(hi, w[32 * g + j]); }
        b[g] = std::max(0.f, -lo);
        a[g] = std::max(0.f, (hi + b[g]) / 31.f);
    }
    const float amax = *std::max_element(a, a + 8), bmax = *std::max_element(b, b + 8);
    const uint16_t dh = f32_to_f16_bits(amax / 63.f), mh = f32_to_f16_bits(bmax / 63.f);
    const float d = f16_bits_to_f32(dh), dmin = f16_bits_to_f32(mh);
    uint32_t sc[8], mn[8];
    for (int g = 0; g < 8; ++g) {
        sc[g] = d > 0 ? (uint32_t)std::clamp(nearest(a[g] / d), 0, 63) : 0u;
        mn[g] = dmin > 0 ? (uint32_t)std::clamp(nearest(b[g] / dmin), 0, 63) : 0u;
    }
    std::memset(p, 0, 176);
    p[0] = (uint8_t)(dh & 0xff); p[1] = (uint8_t)(dh >> 8);
    p[2] = (uint8_t)(mh & 0xff); p[3] = (uint8_t)(mh >> 8);
    uint8_t *s = p + 4;
    for (int g = 0; g < 4; ++g) {
        s[g] = (uint8_t)(sc[g] | ((sc[g + 4] >> 4) << 6));
        s[g + 4] = (uint8_t)(mn[g] | ((mn[g + 4] >> 4) << 6));
        s[g + 8] = (uint8_t)((sc[g + 4] & 15u) | ((mn[g + 4] & 15u) << 4));
    }
    uint8_t *qh = p + 16, *qs = p + 48;
    for (int g = 0; g < 8; ++g) {
        const float A = d * (float)sc[g], B = dmin * (float)mn[g];
        for (int j = 0; j < 32; ++j) {
            const int q = A > 0 ? std::clamp(nearest((w[32 * g + j] + B) / A), 0, 31) : 0;
            qs[(g / 2) * 32 + j] |= (uint8_t)((q & 15) << ((g & 1) * 4));
            qh[j] |= (uint8_t)((q >> 4) << g);
        }
    }
}

void quantize_q6k_block(const float *w, uint8_t *p) {
    float c[16];
    for (int s = 0; s < 16; ++s) {
        float m = 0.f;
        for (int j = 0; j < 16; ++j) m = std::max(m, std::fabs(w[16 * s + j]));
        c[s] = m / 31.f;
    }
    const float cmax = *std::max_element(c, c + 16);
    const uint16_t dh = f32_to_f16_bits(cmax / 127.f);
    const float d = f16_bits_to_f32(dh);
    int sc[16];
    for (int s = 0; s < 16; ++s) sc[s] = d > 0 ? std::clamp(nearest(c[s] / d), -128, 127) : 0;
    std::memset(p, 0, 210);
    uint8_t *ql = p, *qh = p + 128;
    for (int e = 0; e < 256; ++e) {
        const float S = d * (float)sc[e / 16];
        const int q = (S > 0 ? std::clamp(nearest(w[e] / S), -32, 31) : 0) + 32;
        const int h = e / 128, g = (e % 128) / 32, j = e % 32;
        ql[64 * h + j + 32 * (g & 1)] |= (uint8_t)((q & 15) << (g >= 2 ? 4 : 0));
        qh[32 * h + j] |= (uint8_t)((q >> 4) << (2 * g));
    }
    for (int s = 0; s < 16; ++s) p[192 + s] = (uint8_t)(int8_t)sc[s];
    p[208] = (uint8_t)(dh & 0xff);
    p[209] = (uint8_t)(dh >> 8);
}

}  // namespace

extern "C" int tc_quantize(uint32_t type, const float *w, uint64_t rows, uint64_t cols, void *blocks,
                           uint64_t blocks_bytes, int threads) {
    if (!w || !blocks) return TC_CUDA_FAIL;
    if (type != TC_GGML_Q4_K && type != TC_GGML_Q5_K && type != TC_GGML_Q6_K) return TC_CUDA_FAIL;
    if (!rows || !cols || cols % 256) return TC_CUDA_FAIL;
    const uint64_t bb = type == TC_GGML_Q4_K ? 144 : type == TC_GGML_Q5_K ? 176 : 210, per_row = cols / 256;
    if (blocks_bytes / bb / per_row < rows) return TC_CUDA_FAIL;
    const int nt = std::max(1, std::min<int>(threads, 256));
    auto *out = static_cast<uint8_t *>(blocks);
    std::vector<uint8_t> bad(256, 0);
    auto work = [&](uint64_t r0, uint64_t r1, int slot) {
        for (uint64_t i = r0 * cols; i < r1 * cols; ++i)
            if (!std::isfinite(w[i])) { bad[slot] = 1; return; }
        for (uint64_t r = r0; r < r1; ++r)
            for (uint64_t b = 0; b < per_row; ++b) {
                const float *src = w + r * cols + b * 256;
                uint8_t *dst = out + (r * per_row + b) * bb;
                if (type == TC_GGML_Q4_K) quantize_q4k_block(src, dst);
                else if (type == TC_GGML_Q5_K) quantize_q5k_block(src, dst);
                else quantize_q6k_block(src, dst);
            }
    };
    if (nt == 1 || rows < 2) {
        work(0, rows, 0);
    } else {
        std::vector<std::thread> pool;
        const uint64_t step = (rows + nt - 1) / nt;
        for (int t = 0; t < nt; ++t) {
            const uint64_t r0 = std::min<uint64_t>(rows, t * step), r1 = std::min<uint64_t>(rows, r0 + step);
            if (r0 < r1) pool.emplace_back(work, r0, r1, t);
        }
        for (auto &th : pool) th.join();
    }
    for (uint8_t b : bad)
        if (b) return TC_CUDA_FAIL;
    return TC_CUDA_OK;
}
