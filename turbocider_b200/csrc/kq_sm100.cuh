// Shared sm_100a building blocks of the quantised GEMM kernels: mbarrier,
// TMA / bulk-copy, tcgen05 (MMA, commit, TMEM load) wrappers in inline PTX,
// and the in-shared-memory K-quant unpack into the 128-byte-swizzled bf16 /
// fp16 operand tile (bit-exact to the reference decoder,
// native/core/gguf_decode.cpp:77-105).
#pragma once
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "kq_format.cuh"

namespace tc {
namespace {

constexpr uint64_t kTimeoutNs = 1000000000ull;
constexpr uint32_t kStatusTimeout = 1u << 2, kStatusF16 = 1u << 1;

// ------------------------------------------------------------ PTX helpers
__device__ __forceinline__ uint32_t su32(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }
__device__ __forceinline__ uint64_t gtimer() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
__device__ __forceinline__ void bar_init(uint32_t b, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(b), "r"(count));
}
__device__ __forceinline__ void bar_expect_tx(uint32_t b, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(b), "r"(bytes) : "memory");
}
__device__ __forceinline__ void bar_arrive(uint32_t b) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(b) : "memory");
}
__device__ __forceinline__ bool bar_try(uint32_t b, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok) : "r"(b), "r"(parity) : "memory");
    return ok != 0;
}
// Waits up to `hint_ns` with the thread suspended (it resumes as soon as the
// phase completes), so waiting warps do not take issue slots from the
// dequantisers.
__device__ __forceinline__ bool bar_try_sleep(uint32_t b, uint32_t parity, uint32_t hint_ns) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok) : "r"(b), "r"(parity), "r"(hint_ns) : "memory");
    return ok != 0;
}
// Bounded wait.  Returns false if the CTA is aborting or the wait timed out
// (which starts the abort).  `honor_abort` = false is used by the drains.
__device__ __noinline__ bool bar_wait_slow(uint32_t b, uint32_t parity, volatile uint32_t *abort_flag,
                                           uint32_t *status, bool honor_abort) {
    const uint64_t t0 = gtimer();
    for (;;) {
        if (bar_try_sleep(b, parity, 20000u)) return true;
        if (honor_abort && *abort_flag) return false;
        if (gtimer() - t0 > kTimeoutNs) {
            atomicOr(status, kStatusTimeout);
            *abort_flag = 1u;
            return false;
        }
    }
}
__device__ __forceinline__ bool bar_wait(uint32_t b, uint32_t parity, volatile uint32_t *abort_flag,
                                         uint32_t *status, bool honor_abort = true) {
    if (bar_try(b, parity)) return true;
    return bar_wait_slow(b, parity, abort_flag, status, honor_abort);
}
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap *map, uint32_t b, int x, int y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
        ::"r"(dst), "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(b) : "memory");
}
__device__ __forceinline__ void bulk_load(uint32_t dst, const void *src, uint32_t bytes, uint32_t b) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                 ::"r"(dst), "l"(src), "r"(bytes), "r"(b) : "memory");
}
__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Shared-memory matrix descriptor (tcgen05): K-major, 128-byte swizzle,
// 8-row core groups 1024 bytes apart (SBO), version 1, layout type 2.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
    return (uint64_t)((saddr & 0x3FFFFu) >> 4) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
           ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}
// Instruction descriptor, kind::f16: D fp32, A/B bf16 (or fp16), both K-major.
template <int BN, bool F16>
__device__ __forceinline__ constexpr uint32_t mma_idesc() {
    return (1u << 4) | ((F16 ? 0u : 1u) << 7) | ((F16 ? 0u : 1u) << 10) | ((uint32_t)(BN >> 3) << 17) |
           ((uint32_t)(128 >> 4) << 24);
}
__device__ __forceinline__ void mma_f16(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n"
        ::"r"(d_tmem), "l"(a), "l"(b), "r"(idesc), "r"(acc));
}
__device__ __forceinline__ void mma_commit(uint32_t b) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(b) : "memory");
}
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&v)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, "
        "%14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
          "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]),
          "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]),
          "=r"(v[24]), "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}


// ------------------------------------------------------------ dequant
// Packed fp32x2 arithmetic (sm_100a): two lanes of fp32 per 64-bit register.
__device__ __forceinline__ uint64_t f2pack(uint32_t lo, uint32_t hi) {
    uint64_t r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "r"(lo), "r"(hi));
    return r;
}
__device__ __forceinline__ void f2unpack(uint64_t v, float &lo, float &hi) {
    asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ uint64_t f2add(uint64_t a, uint64_t b) {
    uint64_t r;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}
__device__ __forceinline__ uint64_t f2mul(uint64_t a, uint64_t b) {
    uint64_t r;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}
__device__ __forceinline__ uint64_t f2fma(uint64_t a, uint64_t b, uint64_t c) {
    uint64_t r;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
    return r;
}
__device__ __forceinline__ uint64_t f2splat(float v) { return f2pack(__float_as_uint(v), __float_as_uint(v)); }
// fp16 staging's compensated min (see four_values_h): m * fp16(s) / s, formed
// as m + (m / s) (fp16(s) - s), while fp16(s) is a normal fp16 number.
__device__ __forceinline__ float min_compensated(float s, float m) {
    const float sh = __half2float(__float2half_rn(s));
    if (!(sh >= 6.103515625e-05f)) return m;   // fp16(s) subnormal or zero: plain min
    float r;
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(s));
    return fmaf(m * r, sh - s, m);
}

// Byte i of w as the float 2^23 + byte (exact): the byte goes into the low
// mantissa bits under the exponent of 2^23.
__device__ __forceinline__ uint32_t magic_byte(uint32_t w, uint32_t i) {
    uint32_t r;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(w), "r"(0x4B000000u), "r"(0x7440u | i));
    return r;
}

// Scale table of one chunk (shared memory, 128 rows x 80 bytes):
//   Q4_K row r: {d*sc_g, dmin*m_g} for g = 0..7, with d*sc_g pre-divided by 16
//               for odd g (their codes are read in place from the high nibble,
//               i.e. multiplied by 16; the power of two keeps every product exact);
//   Q6_K row r: d*sc_i for the 16 sub-blocks.
// Thread dt writes 16 bytes of row dt % 128 (conflict-free with the odd
// 80-byte stride, as are the reads of the dequant tasks).
// Q4_K and Q5_K share the per-sub-block (scale, min) form d*sc*q - dmin*m
// (gguf_decode.cpp:77-90); Q6_K is scale-only.
__device__ __forceinline__ constexpr bool affine_type(int type) { return type == 12 || type == 13; }

// With fp16 staging the range check is done here, once per sub-block: the
// decode is affine in the code, so the largest magnitude a sub-block can
// produce sits at an end code (Q4_K: q = 0 or 15; Q5_K: 0 or 31; Q6_K:
// q - 32 = -32); `ovf` is raised when that value would round to inf in fp16.
// Q5_K's odd sub-blocks are not pre-divided: their 5-bit codes are shifted
// down to the low bits instead of being read in place.
template <int TYPE, bool F16>
__device__ __forceinline__ void build_table(const uint8_t *wc, float *tab, uint32_t dt, bool &ovf) {
    constexpr float kF16Inf = 65520.0f;   // smallest magnitude that rounds to inf
    const uint32_t r = dt & 127, j = dt >> 7;
    float4 v;
    if (affine_type(TYPE)) {
        constexpr uint32_t kDm = TYPE == 12 ? kQ4Dm : kQ5Dm, kSc = TYPE == 12 ? kQ4Sc : kQ5Sc;
        constexpr float kQMax = TYPE == 12 ? 15.0f : 31.0f, kOddScale = TYPE == 12 ? 0.0625f : 1.0f;
        const uint32_t dm = *reinterpret_cast<const uint32_t *>(wc + kDm + r * 4);
        const float d = half_bits_to_float((uint16_t)(dm & 0xffffu)), dmin = half_bits_to_float((uint16_t)(dm >> 16));
        const uint8_t *sc = wc + kSc + r * 12;
        uint32_t s0, m0, s1, m1;
        q4k_scale_min(2 * j, sc, s0, m0);
        q4k_scale_min(2 * j + 1, sc, s1, m1);
        v = make_float4(d * (float)s0, dmin * (float)m0, d * (float)s1 * kOddScale, dmin * (float)m1);
        if (F16) {
            const float a1 = d * (float)s1;
            ovf |= fmaxf(fabsf(v.y), fabsf(fmaf(v.x, kQMax, -v.y))) >= kF16Inf ||
                   fmaxf(fabsf(v.w), fabsf(fmaf(a1, kQMax, -v.w))) >= kF16Inf;
            v.y = min_compensated(v.x, v.y);   // fp16 staging: see four_values_h
            v.w = min_compensated(v.z, v.w);
        }
    } else {
        const float d = half_bits_to_float(*reinterpret_cast<const uint16_t *>(wc + kQ6D + r * 2));
        const int8_t *sc = reinterpret_cast<const int8_t *>(wc + kQ6Sc + r * 16 + 4 * j);
        v = make_float4(d * (float)sc[0], d * (float)sc[1], d * (float)sc[2], d * (float)sc[3]);
        if (F16) ovf |= 32.0f * fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))) >= kF16Inf;
    }
    *reinterpret_cast<float4 *>(reinterpret_cast<uint8_t *>(tab) + r * 80 + 16 * j) = v;
}

template <bool F16>
__device__ __forceinline__ uint32_t pack_pair(uint64_t v) {
    float lo, hi;
    f2unpack(v, lo, hi);
    if (F16) {
        const __half2 h = __floats2half2_rn(lo, hi);
        return *reinterpret_cast<const uint32_t *>(&h);
    } else {
        const __nv_bfloat162 b = __floats2bfloat162_rn(lo, hi);
        return *reinterpret_cast<const uint32_t *>(&b);
    }
}

// Four weights from the four bytes of `codes` (each 2^23 + byte exactly),
// as v = scale * (byte - bias) [Q6_K, bias = 2^23 + 32] or
// v = scale * (byte - 2^23) - min [Q4_K]: one magic subtract and one
// multiply / FMA per pair, both exact except the Q4_K FMA's single rounding,
// which is the reference's own rounding of d*q - m.
template <int TYPE, bool F16>
__device__ __forceinline__ uint2 four_values(uint32_t codes, uint64_t scale2, uint64_t off2, uint64_t min2) {
    const uint64_t p0 = f2add(f2pack(magic_byte(codes, 0), magic_byte(codes, 1)), off2);
    const uint64_t p1 = f2add(f2pack(magic_byte(codes, 2), magic_byte(codes, 3)), off2);
    uint64_t v0, v1;
    if (affine_type(TYPE)) { v0 = f2fma(scale2, p0, min2); v1 = f2fma(scale2, p1, min2); }
    else { v0 = f2mul(scale2, p0); v1 = f2mul(scale2, p1); }
    return make_uint2(pack_pair<F16>(v0), pack_pair<F16>(v1));
}

// ---- fp16 staging (TC_STAGE_F16 / TC_STAGE_F16_X16): packed f16x2 arithmetic.
// The GEMM's output bar is rel-L2 <= 1e-3 against dequant + fp32 matmul, not
// bit-exact staging (the dequantise hooks, tc_cuda_dequant / tc_cuda_decode,
// stay bit-exact), so fp16 staging computes each weight as
//     Q4_K / Q5_K: fp16(code * fp16(d sc) - fp16(dmin m))   one fma.rn.f16x2
//     Q6_K:        fp16((code - 32) * fp16(d sc))           one mul.rn.f16x2
// with the per-sub-block scale rounded to fp16 once (Q4_K high nibbles, read
// in place as 16 code, use fp16(d sc / 16)) and the min compensated for that
// rounding: m' = m * fp16(s) / s (min_compensated), so the sub-block's zero
// point m / s is kept and the scale's rounding error scales with the weight
// rather than with the code; only the min's own fp16 rounding remains.
// Compensation applies while fp16(s) is a normal fp16 number (>= 2^-14).
// Per 4 weights: 2
// prmt (each code byte under the fp16 exponent of 1024: 0x64cc = 1024 + code),
// 2 exact f16x2 subtracts, 2 f16x2 FMAs -- against 4 prmt, 2 f32x2 adds, 2
// f32x2 FMAs and 2 conversions for the exact form.
__device__ __forceinline__ uint32_t h2splat(float v) {
    const __half2 h = __floats2half2_rn(v, v);
    return *reinterpret_cast<const uint32_t *>(&h);
}
__device__ __forceinline__ uint32_t h2_code(uint32_t codes, uint32_t sel) {
    uint32_t r;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(codes), "r"(0x64646464u), "r"(sel));
    return r;
}
__device__ __forceinline__ uint32_t h2_sub(uint32_t a, uint32_t b) {
    uint32_t r;
    asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
    return r;
}
__device__ __forceinline__ uint32_t h2_fma(uint32_t a, uint32_t b, uint32_t c) {
    uint32_t r;
    asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(c));
    return r;
}
__device__ __forceinline__ uint32_t h2_mul(uint32_t a, uint32_t b) {
    uint32_t r;
    asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
    return r;
}
// Four weights from the four code bytes (Q4_K / Q5_K: 0..255 as read, Q6_K:
// 0..63 with the +32 bias), scale / min as fp16 pairs (min negated).
template <int TYPE>
__device__ __forceinline__ uint2 four_values_h(uint32_t codes, uint32_t scale_h2, uint32_t min_h2) {
    constexpr uint32_t kOff = TYPE == 14 ? 0x64206420u : 0x64006400u;   // 1024 + 32 / 1024
    const uint32_t p0 = h2_sub(h2_code(codes, 0x4140u), kOff), p1 = h2_sub(h2_code(codes, 0x4342u), kOff);
    if (affine_type(TYPE)) return make_uint2(h2_fma(p0, scale_h2, min_h2), h2_fma(p1, scale_h2, min_h2));
    return make_uint2(h2_mul(p0, scale_h2), h2_mul(p1, scale_h2));
}
// The task's four-weight groups: the exact form for bf16 staging, the f16x2
// form for fp16 staging (scale / min given in fp32, converted here).
template <int TYPE, bool F16>
__device__ __forceinline__ uint2 four_any(uint32_t codes, float scale, float min_neg) {
    if constexpr (F16) return four_values_h<TYPE>(codes, h2splat(scale), h2splat(min_neg));
    return four_values<TYPE, F16>(codes, f2splat(scale), f2splat(TYPE == 14 ? -8388640.0f : -8388608.0f),
                                  f2splat(min_neg));
}

// One task: weight row r, bytes 8t..8t+7 of the 64-weight slice q.  Writes
// two 16-byte chunks (slice K 8t..8t+7 and 32+8t..32+8t+7) of the swizzled
// A tile.  Q4_K: low nibbles = sub-block 2q, high nibbles = sub-block 2q+1.
// Q6_K: half h = q/2, groups g0 = 2(q&1) (ql part 0) and g0+1 (part 1).
template <int TYPE, bool F16>
__device__ __forceinline__ void dequant_task(const uint8_t *wc, const float *tab, uint32_t q, uint32_t r,
                                             uint32_t t, uint8_t *a) {
    const uint32_t slot = row_slot(r);
    const uint8_t *trow = reinterpret_cast<const uint8_t *>(tab) + r * 80;
    uint2 lo0, lo1, hi0, hi1;
    if (TYPE == 12) {
        const uint2 b = *reinterpret_cast<const uint2 *>(wc + kQ4Qs + q * 4096 + slot * 32 + t * 8);
        const float4 s = *reinterpret_cast<const float4 *>(trow + 16 * q);
        lo0 = four_any<12, F16>(b.x & 0x0F0F0F0Fu, s.x, -s.y);
        lo1 = four_any<12, F16>(b.y & 0x0F0F0F0Fu, s.x, -s.y);
        hi0 = four_any<12, F16>(b.x & 0xF0F0F0F0u, s.z, -s.w);
        hi1 = four_any<12, F16>(b.y & 0xF0F0F0F0u, s.z, -s.w);
    } else if (TYPE == 13) {
        // Q5_K: low nibble | fifth bit (bit 2q of qh) for sub-block 2q, high
        // nibble shifted down | bit 2q+1 for sub-block 2q+1 (codes 0..31).
        const uint2 b = *reinterpret_cast<const uint2 *>(wc + kQ5Qs + q * 4096 + slot * 32 + t * 8);
        const uint2 hb = *reinterpret_cast<const uint2 *>(wc + kQ5Qh + slot * 32 + t * 8);
        const float4 s = *reinterpret_cast<const float4 *>(trow + 16 * q);
        const uint32_t bl = 2 * q, bh = 2 * q + 1;
        lo0 = four_any<13, F16>((b.x & 0x0F0F0F0Fu) | (((hb.x >> bl) & 0x01010101u) << 4), s.x, -s.y);
        lo1 = four_any<13, F16>((b.y & 0x0F0F0F0Fu) | (((hb.y >> bl) & 0x01010101u) << 4), s.x, -s.y);
        hi0 = four_any<13, F16>(((b.x >> 4) & 0x0F0F0F0Fu) | (((hb.x >> bh) & 0x01010101u) << 4), s.z, -s.w);
        hi1 = four_any<13, F16>(((b.y >> 4) & 0x0F0F0F0Fu) | (((hb.y >> bh) & 0x01010101u) << 4), s.z, -s.w);
    } else {
        const uint32_t h = q >> 1, shift = (q & 1) * 4, g0 = 2 * (q & 1);
        const uint2 la = *reinterpret_cast<const uint2 *>(wc + kQ6Ql + ((h * 2 + 0) * kPanelRows + slot) * 32 + t * 8);
        const uint2 lb = *reinterpret_cast<const uint2 *>(wc + kQ6Ql + ((h * 2 + 1) * kPanelRows + slot) * 32 + t * 8);
        const uint2 qh = *reinterpret_cast<const uint2 *>(wc + kQ6Qh + (h * kPanelRows + slot) * 32 + t * 8);
        const float *tf = reinterpret_cast<const float *>(trow);
        const float da = tf[8 * h + (t >> 1) + 2 * g0], db = tf[8 * h + (t >> 1) + 2 * g0 + 2];
        const uint32_t ca0 = ((la.x >> shift) & 0x0F0F0F0Fu) | (((qh.x >> (2 * g0)) & 0x03030303u) << 4);
        const uint32_t ca1 = ((la.y >> shift) & 0x0F0F0F0Fu) | (((qh.y >> (2 * g0)) & 0x03030303u) << 4);
        const uint32_t cb0 = ((lb.x >> shift) & 0x0F0F0F0Fu) | (((qh.x >> (2 * g0 + 2)) & 0x03030303u) << 4);
        const uint32_t cb1 = ((lb.y >> shift) & 0x0F0F0F0Fu) | (((qh.y >> (2 * g0 + 2)) & 0x03030303u) << 4);
        lo0 = four_any<14, F16>(ca0, da, 0.f);
        lo1 = four_any<14, F16>(ca1, da, 0.f);
        hi0 = four_any<14, F16>(cb0, db, 0.f);
        hi1 = four_any<14, F16>(cb1, db, 0.f);
    }
    uint8_t *row = a + (r >> 3) * 1024 + (r & 7) * 128;
    *reinterpret_cast<uint4 *>(row + ((t ^ (r & 7)) << 4)) = make_uint4(lo0.x, lo0.y, lo1.x, lo1.y);
    *reinterpret_cast<uint4 *>(row + (((4 + t) ^ (r & 7)) << 4)) = make_uint4(hi0.x, hi0.y, hi1.x, hi1.y);
}

}  // namespace
}  // namespace tc
