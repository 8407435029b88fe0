// Quantised GEMM on the 5th-generation tensor cores (sm_100a):
//     Y[m, n] = sum_k X[m, k] * W[n, k],  W in GGUF Q4_K / Q6_K, X bf16.
//
// The tensor-core operands are A = the dequantised weight tile (128 weight
// rows n, MMA M = 128) and B = the activation tile (BN tokens, MMA N = BN),
// both K-major with the 128-byte swizzle, so D = W_tile * X_tile^T lands in
// TMEM as [128 lanes = n] x [BN columns = tokens] fp32.  Each weight element
// is dequantised once per BN tokens.
//
// One persistent CTA per SM, 22 warps, warp-specialised:
//   warp 0     TMA producer: one bulk copy per packed weight chunk (128 rows x
//              256 K, 18/26 KB) and one 2-D tensor copy per activation stage
//              (BN x 64 bf16, SWIZZLE_128B);
//   warp 1     TMEM allocator and the single MMA-issuing thread
//              (tcgen05.mma kind::f16, 4 x K16 per stage, commit to mbarriers);
//   warps 2-5  epilogue: tcgen05.ld 32 columns at a time and store Y;
//   warps 6-21 dequantisers: unpack the packed chunk in shared memory into the
//              swizzled bf16 (or fp16) A tile, bit-exact to the reference
//              decoder, then fence.proxy.async and arrive.
// TMEM holds two BN-column accumulators so the epilogue of tile i overlaps
// the main loop of tile i+1.  Every mbarrier wait is bounded (globaltimer);
// on timeout the kernel sets TC_STATUS_TIMEOUT, drains its own copies and
// MMAs, frees TMEM and returns -- it never traps.
// No TMA multicast is used anywhere (every CTA loads its own tiles).
// Launched with programmatic dependent launch: the prologue (barriers, TMEM)
// of this GEMM overlaps the tail of the previous kernel; the producer waits
// (griddepcontrol.wait) before its first activation load.
#include <cuda.h>
#include <cudaTypedefs.h>

#include "kq_format.cuh"
#include "tc_internal.h"

namespace tc {
namespace {

constexpr int kThreads = 704;   // 22 warps
constexpr int kEpiWarp0 = 2, kEpiThreads = 128, kDequantWarp0 = 6, kDequantThreads = 512;
constexpr int kStages = 3;      // activation / A-tile pipeline depth (64 K each)
constexpr int kWStages = 2;     // packed chunk pipeline depth (256 K each)
constexpr int kMaxSeg = 32;
constexpr uint64_t kTimeoutNs = 1000000000ull;
constexpr uint32_t kStatusTimeout = 1u << 2, kStatusF16 = 1u << 1;

struct GemmSeg {
    uint32_t m_begin, m_end, tile_begin, pad;
    const uint8_t *w;
};
struct GemmParams {
    GemmSeg seg[kMaxSeg];
    uint32_t n_seg, n_tiles, kb, panels, n;
    void *y;
    uint64_t ldy;
    uint32_t *status;
};

template <int TYPE, int BN>
struct Layout {
    static constexpr uint32_t x_stage = BN * 128;
    static constexpr uint32_t a_stage = 128 * 128;
    static constexpr uint32_t w_stage = chunk_bytes(TYPE);
    static constexpr uint32_t x_off = 0;
    static constexpr uint32_t a_off = x_off + kStages * x_stage;
    static constexpr uint32_t w_off = a_off + kStages * a_stage;
    static constexpr uint32_t t_off = (w_off + kWStages * w_stage + 127) / 128 * 128;
    static constexpr uint32_t table_bytes = 128 * 80;  // 80-byte row stride (conflict-free)
    static constexpr uint32_t bar_off = t_off + 2 * table_bytes;
    // x_full[S] a_full[S] st_empty[S] w_full[W] w_empty[W] t_ready[2] acc_full[2] acc_empty[2] fin
    static constexpr uint32_t n_bars = 3 * kStages + 2 * kWStages + 7;
    static constexpr uint32_t misc_off = bar_off + n_bars * 8;
    static constexpr uint32_t bytes = misc_off + 16 + 1024;  // + alignment slack
    static constexpr uint32_t tmem_cols = BN * 2 <= 32 ? 32 : BN * 2;
};

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

// ------------------------------------------------------------ tiles
struct Tile {
    uint32_t m0, m_end, panel;
    const uint8_t *w;
};
template <int BN>
__device__ __forceinline__ Tile tile_of(const GemmParams &p, uint32_t t) {
    uint32_t s = 0;
    while (s + 1 < p.n_seg && t >= p.seg[s + 1].tile_begin) ++s;
    const uint32_t local = t - p.seg[s].tile_begin;
    return {p.seg[s].m_begin + (local / p.panels) * BN, p.seg[s].m_end, local % p.panels, p.seg[s].w};
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
template <int TYPE>
__device__ __forceinline__ void build_table(const uint8_t *wc, float *tab, uint32_t dt) {
    const uint32_t r = dt & 127, j = dt >> 7;
    float4 v;
    if (TYPE == 12) {
        const uint32_t dm = *reinterpret_cast<const uint32_t *>(wc + kQ4Dm + r * 4);
        const float d = half_bits_to_float((uint16_t)(dm & 0xffffu)), dmin = half_bits_to_float((uint16_t)(dm >> 16));
        const uint8_t *sc = wc + kQ4Sc + r * 12;
        uint32_t s0, m0, s1, m1;
        q4k_scale_min(2 * j, sc, s0, m0);
        q4k_scale_min(2 * j + 1, sc, s1, m1);
        v = make_float4(d * (float)s0, dmin * (float)m0, d * (float)s1 * 0.0625f, dmin * (float)m1);
    } else {
        const float d = half_bits_to_float(*reinterpret_cast<const uint16_t *>(wc + kQ6D + r * 2));
        const int8_t *sc = reinterpret_cast<const int8_t *>(wc + kQ6Sc + r * 16 + 4 * j);
        v = make_float4(d * (float)sc[0], d * (float)sc[1], d * (float)sc[2], d * (float)sc[3]);
    }
    *reinterpret_cast<float4 *>(reinterpret_cast<uint8_t *>(tab) + r * 80 + 16 * j) = v;
}

template <bool F16>
__device__ __forceinline__ uint32_t pack_pair(uint64_t v, bool &ovf) {
    float lo, hi;
    f2unpack(v, lo, hi);
    if (F16) {
        const __half2 h = __floats2half2_rn(lo, hi);
        const uint32_t u = *reinterpret_cast<const uint32_t *>(&h);
        ovf |= ((u & 0x7c00u) == 0x7c00u) || ((u & 0x7c000000u) == 0x7c000000u);
        return u;
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
__device__ __forceinline__ uint2 four_values(uint32_t codes, uint64_t scale2, uint64_t off2, uint64_t min2, bool &ovf) {
    const uint64_t p0 = f2add(f2pack(magic_byte(codes, 0), magic_byte(codes, 1)), off2);
    const uint64_t p1 = f2add(f2pack(magic_byte(codes, 2), magic_byte(codes, 3)), off2);
    uint64_t v0, v1;
    if (TYPE == 12) { v0 = f2fma(scale2, p0, min2); v1 = f2fma(scale2, p1, min2); }
    else { v0 = f2mul(scale2, p0); v1 = f2mul(scale2, p1); }
    return make_uint2(pack_pair<F16>(v0, ovf), pack_pair<F16>(v1, ovf));
}

// One task: weight row r, bytes 8t..8t+7 of the 64-weight slice q.  Writes
// two 16-byte chunks (slice K 8t..8t+7 and 32+8t..32+8t+7) of the swizzled
// A tile.  Q4_K: low nibbles = sub-block 2q, high nibbles = sub-block 2q+1.
// Q6_K: half h = q/2, groups g0 = 2(q&1) (ql part 0) and g0+1 (part 1).
template <int TYPE, bool F16>
__device__ __forceinline__ void dequant_task(const uint8_t *wc, const float *tab, uint32_t q, uint32_t r,
                                             uint32_t t, uint8_t *a, bool &ovf) {
    const uint32_t slot = row_slot(r);
    const uint8_t *trow = reinterpret_cast<const uint8_t *>(tab) + r * 80;
    uint2 lo0, lo1, hi0, hi1;
    if (TYPE == 12) {
        const uint2 b = *reinterpret_cast<const uint2 *>(wc + kQ4Qs + q * 4096 + slot * 32 + t * 8);
        const float4 s = *reinterpret_cast<const float4 *>(trow + 16 * q);
        const uint64_t off2 = f2splat(-8388608.0f);
        const uint64_t dl = f2splat(s.x), ml = f2splat(-s.y), dh = f2splat(s.z), mh = f2splat(-s.w);
        lo0 = four_values<12, F16>(b.x & 0x0F0F0F0Fu, dl, off2, ml, ovf);
        lo1 = four_values<12, F16>(b.y & 0x0F0F0F0Fu, dl, off2, ml, ovf);
        hi0 = four_values<12, F16>(b.x & 0xF0F0F0F0u, dh, off2, mh, ovf);
        hi1 = four_values<12, F16>(b.y & 0xF0F0F0F0u, dh, off2, mh, ovf);
    } else {
        const uint32_t h = q >> 1, shift = (q & 1) * 4, g0 = 2 * (q & 1);
        const uint2 la = *reinterpret_cast<const uint2 *>(wc + kQ6Ql + ((h * 2 + 0) * kPanelRows + slot) * 32 + t * 8);
        const uint2 lb = *reinterpret_cast<const uint2 *>(wc + kQ6Ql + ((h * 2 + 1) * kPanelRows + slot) * 32 + t * 8);
        const uint2 qh = *reinterpret_cast<const uint2 *>(wc + kQ6Qh + (h * kPanelRows + slot) * 32 + t * 8);
        const float *tf = reinterpret_cast<const float *>(trow);
        const uint64_t da = f2splat(tf[8 * h + (t >> 1) + 2 * g0]);
        const uint64_t db = f2splat(tf[8 * h + (t >> 1) + 2 * g0 + 2]);
        const uint64_t off2 = f2splat(-8388640.0f);  // -(2^23 + 32)
        const uint32_t ca0 = ((la.x >> shift) & 0x0F0F0F0Fu) | (((qh.x >> (2 * g0)) & 0x03030303u) << 4);
        const uint32_t ca1 = ((la.y >> shift) & 0x0F0F0F0Fu) | (((qh.y >> (2 * g0)) & 0x03030303u) << 4);
        const uint32_t cb0 = ((lb.x >> shift) & 0x0F0F0F0Fu) | (((qh.x >> (2 * g0 + 2)) & 0x03030303u) << 4);
        const uint32_t cb1 = ((lb.y >> shift) & 0x0F0F0F0Fu) | (((qh.y >> (2 * g0 + 2)) & 0x03030303u) << 4);
        lo0 = four_values<14, F16>(ca0, da, off2, 0, ovf);
        lo1 = four_values<14, F16>(ca1, da, off2, 0, ovf);
        hi0 = four_values<14, F16>(cb0, db, off2, 0, ovf);
        hi1 = four_values<14, F16>(cb1, db, off2, 0, ovf);
    }
    uint8_t *row = a + (r >> 3) * 1024 + (r & 7) * 128;
    *reinterpret_cast<uint4 *>(row + ((t ^ (r & 7)) << 4)) = make_uint4(lo0.x, lo0.y, lo1.x, lo1.y);
    *reinterpret_cast<uint4 *>(row + (((4 + t) ^ (r & 7)) << 4)) = make_uint4(hi0.x, hi0.y, hi1.x, hi1.y);
}

// ------------------------------------------------------------ the kernel
template <int TYPE, int BN, bool F16, bool OUT_F32>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap xmap, const __grid_constant__ GemmParams p) {
    using L = Layout<TYPE, BN>;
    constexpr uint32_t kChunk = chunk_bytes(TYPE);
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const uint32_t warp = threadIdx.x / 32, lane = threadIdx.x % 32;

    const uint32_t bars = su32(smem + L::bar_off);
    auto x_full = [&](uint32_t i) { return bars + 8 * i; };
    auto a_full = [&](uint32_t i) { return bars + 8 * (kStages + i); };
    auto st_empty = [&](uint32_t i) { return bars + 8 * (2 * kStages + i); };
    auto w_full = [&](uint32_t i) { return bars + 8 * (3 * kStages + i); };
    auto w_empty = [&](uint32_t i) { return bars + 8 * (3 * kStages + kWStages + i); };
    auto t_ready = [&](uint32_t i) { return bars + 8 * (3 * kStages + 2 * kWStages + i); };
    auto acc_full = [&](uint32_t i) { return bars + 8 * (3 * kStages + 2 * kWStages + 2 + i); };
    auto acc_empty = [&](uint32_t i) { return bars + 8 * (3 * kStages + 2 * kWStages + 4 + i); };
    const uint32_t fin = bars + 8 * (3 * kStages + 2 * kWStages + 6);
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + L::misc_off);
    volatile uint32_t *abort_flag = tmem_slot + 1;

    if (threadIdx.x == 0) {
        for (int i = 0; i < kStages; ++i) {
            bar_init(x_full(i), 1);
            bar_init(a_full(i), kDequantThreads);
            bar_init(st_empty(i), 1);
        }
        for (int i = 0; i < kWStages; ++i) {
            bar_init(w_full(i), 1);
            bar_init(w_empty(i), kDequantThreads);
        }
        for (int i = 0; i < 2; ++i) {
            bar_init(t_ready(i), kDequantThreads);
            bar_init(acc_full(i), 1);
            bar_init(acc_empty(i), kEpiThreads);
        }
        bar_init(fin, 1);
        *abort_flag = 0u;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                     ::"r"(su32(tmem_slot)), "r"(L::tmem_cols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (threadIdx.x == 0) asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    if (warp == 0) {
        // ---------------------------------------------------- producer
        if (lane == 0) {
            // X (and the Y the epilogue writes) may belong to the previous
            // kernel in the stream: wait for it before the first activation load.
            asm volatile("griddepcontrol.wait;" ::: "memory");
            uint32_t st = 0, ph = 0, ws = 0, wph = 0;
            uint32_t x_last[kStages], w_last[kWStages];
            bool x_used[kStages] = {}, w_used[kWStages] = {};
            bool ok = true;
            for (uint32_t t = blockIdx.x; ok && t < p.n_tiles; t += gridDim.x) {
                const Tile T = tile_of<BN>(p, t);
                const uint8_t *panel = T.w + (uint64_t)T.panel * p.kb * kChunk;
                for (uint32_t kb = 0; ok && kb < p.kb; ++kb) {
                    if (!(ok = bar_wait(w_empty(ws), wph ^ 1, abort_flag, p.status))) break;
                    bar_expect_tx(w_full(ws), kChunk);
                    bulk_load(su32(smem + L::w_off + ws * L::w_stage), panel + (uint64_t)kb * kChunk, kChunk, w_full(ws));
                    w_last[ws] = wph; w_used[ws] = true;
                    if (++ws == kWStages) { ws = 0; wph ^= 1; }
                    for (uint32_t q = 0; q < 4; ++q) {
                        if (!(ok = bar_wait(st_empty(st), ph ^ 1, abort_flag, p.status))) break;
                        bar_expect_tx(x_full(st), L::x_stage);
                        tma_load_2d(su32(smem + L::x_off + st * L::x_stage), &xmap, x_full(st),
                                    (int)(kb * 256 + q * 64), (int)T.m0);
                        x_last[st] = ph; x_used[st] = true;
                        if (++st == kStages) { st = 0; ph ^= 1; }
                    }
                }
            }
            // Drain: every copy this thread issued has landed before exit.
            for (int i = 0; i < kStages; ++i)
                if (x_used[i]) bar_wait(x_full(i), x_last[i], abort_flag, p.status, false);
            for (int i = 0; i < kWStages; ++i)
                if (w_used[i]) bar_wait(w_full(i), w_last[i], abort_flag, p.status, false);
        }
        __syncwarp();
    } else if (warp == 1) {
        // ---------------------------------------------------- MMA issuer
        if (lane == 0) {
            constexpr uint32_t idesc = mma_idesc<BN, F16>();
            uint32_t st = 0, ph = 0, acc = 0, aph = 0;
            bool ok = true;
            for (uint32_t t = blockIdx.x; ok && t < p.n_tiles; t += gridDim.x) {
                if (!(ok = bar_wait(acc_empty(acc), aph ^ 1, abort_flag, p.status))) break;
                tc_fence_after();
                const uint32_t d_tmem = tmem + acc * BN;
                for (uint32_t kb = 0; ok && kb < p.kb; ++kb) {
                    for (uint32_t q = 0; q < 4; ++q) {
                        if (!(ok = bar_wait(x_full(st), ph, abort_flag, p.status))) break;
                        if (!(ok = bar_wait(a_full(st), ph, abort_flag, p.status))) break;
                        tc_fence_after();
                        const uint32_t a_addr = su32(smem + L::a_off + st * L::a_stage);
                        const uint32_t b_addr = su32(smem + L::x_off + st * L::x_stage);
#pragma unroll
                        for (uint32_t kk = 0; kk < 4; ++kk)
                            mma_f16(d_tmem, sw128_desc(a_addr + kk * 32), sw128_desc(b_addr + kk * 32), idesc,
                                    (kb | q | kk) ? 1u : 0u);
                        mma_commit(st_empty(st));
                        if (++st == kStages) { st = 0; ph ^= 1; }
                    }
                }
                if (!ok) break;
                mma_commit(acc_full(acc));
                acc ^= 1;
                if (acc == 0) aph ^= 1;
            }
            // Every MMA issued by this thread has completed before TMEM is freed.
            mma_commit(fin);
            bar_wait(fin, 0, abort_flag, p.status, false);
        }
        __syncwarp();
    } else if (warp >= (uint32_t)kDequantWarp0) {
        // ---------------------------------------------------- dequantisers
        const uint32_t dt = threadIdx.x - kDequantWarp0 * 32, dw = dt / 32;
        uint32_t st = 0, ph = 0, ws = 0, wph = 0, tb = 0, tph = 0;
        bool ok = true, ovf = false;
        for (uint32_t t = blockIdx.x; ok && t < p.n_tiles; t += gridDim.x) {
            for (uint32_t kb = 0; ok && kb < p.kb; ++kb) {
                if (!(ok = bar_wait(w_full(ws), wph, abort_flag, p.status))) break;
                const uint8_t *wc = smem + L::w_off + ws * L::w_stage;
                float *tab = reinterpret_cast<float *>(smem + L::t_off + tb * L::table_bytes);
                build_table<TYPE>(wc, tab, dt);
                bar_arrive(t_ready(tb));
                if (!(ok = bar_wait(t_ready(tb), tph, abort_flag, p.status))) break;
                for (uint32_t q = 0; q < 4; ++q) {
                    if (!(ok = bar_wait(st_empty(st), ph ^ 1, abort_flag, p.status))) break;
                    uint8_t *a = smem + L::a_off + st * L::a_stage;
                    {
                        const uint32_t r = 8 * dw + (lane >> 3) + 4 * ((lane >> 2) & 1);
                        dequant_task<TYPE, F16>(wc, tab, q, r, lane & 3, a, ovf);
                    }
                    fence_proxy_async();
                    bar_arrive(a_full(st));
                    if (++st == kStages) { st = 0; ph ^= 1; }
                }
                if (!ok) break;
                bar_arrive(w_empty(ws));
                if (++ws == kWStages) { ws = 0; wph ^= 1; }
                if (++tb == 2) { tb = 0; tph ^= 1; }
            }
        }
        if (F16 && ovf) atomicOr(p.status, kStatusF16);
    } else {
        // ---------------------------------------------------- epilogue
        const uint32_t quad = warp & 3;
        uint32_t acc = 0, aph = 0;
        for (uint32_t t = blockIdx.x; t < p.n_tiles; t += gridDim.x) {
            const Tile T = tile_of<BN>(p, t);
            if (!bar_wait(acc_full(acc), aph, abort_flag, p.status)) break;
            tc_fence_after();
            const uint32_t n = T.panel * 128 + quad * 32 + lane;
            const uint32_t taddr = tmem + ((quad * 32) << 16) + acc * BN;
#pragma unroll 1
            for (uint32_t c0 = 0; c0 < (uint32_t)BN; c0 += 32) {
                uint32_t v[32];
                tmem_ld32(taddr + c0, v);
                if (n < p.n) {
#pragma unroll
                    for (uint32_t c = 0; c < 32; ++c) {
                        const uint32_t m = T.m0 + c0 + c;
                        if (m < T.m_end) {
                            const uint64_t off = (uint64_t)m * p.ldy + n;
                            if (OUT_F32) static_cast<float *>(p.y)[off] = __uint_as_float(v[c]);
                            else static_cast<__nv_bfloat16 *>(p.y)[off] = __float2bfloat16_rn(__uint_as_float(v[c]));
                        }
                    }
                }
            }
            tc_fence_before();
            bar_arrive(acc_empty(acc));
            acc ^= 1;
            if (acc == 0) aph ^= 1;
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(L::tmem_cols));
    }
}

// ------------------------------------------------------------ host side
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    if (!fn) {
        void *ptr = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
    }
    return fn;
}

template <int TYPE, int BN, bool F16, bool OUT_F32>
cudaError_t launch_inst(const CUtensorMap &map, const GemmParams &p, int sm_count, cudaStream_t s) {
    using L = Layout<TYPE, BN>;
    auto kernel = gemm_kernel<TYPE, BN, F16, OUT_F32>;
    static bool configured = false;
    if (!configured) {
        cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)L::bytes);
        if (e != cudaSuccess) return e;
        configured = true;
    }
    const unsigned grid = p.n_tiles < (uint32_t)sm_count ? p.n_tiles : (unsigned)sm_count;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = L::bytes;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, map, p);
}

template <int TYPE, int BN>
cudaError_t launch_bn(const CUtensorMap &map, const GemmParams &p, int f16, int out_f32, int sm, cudaStream_t s) {
    if (f16) return out_f32 ? launch_inst<TYPE, BN, true, true>(map, p, sm, s) : launch_inst<TYPE, BN, true, false>(map, p, sm, s);
    return out_f32 ? launch_inst<TYPE, BN, false, true>(map, p, sm, s) : launch_inst<TYPE, BN, false, false>(map, p, sm, s);
}

}  // namespace

cudaError_t launch_gemm(const SegmentView *segs, uint32_t n_seg, const uint16_t *x, uint64_t m_total, uint64_t k,
                        void *y, uint64_t ldy, int out_dtype, int stage_f16, int sm_count, uint32_t *status,
                        cudaStream_t s) {
    if (n_seg == 0) return cudaSuccess;
    if (n_seg > (uint32_t)kMaxSeg) return cudaErrorInvalidValue;
    uint32_t max_rows = 0;
    for (uint32_t i = 0; i < n_seg; ++i) max_rows = max(max_rows, segs[i].m_end - segs[i].m_begin);
    const int bn = max_rows <= 64 ? 64 : max_rows <= 128 ? 128 : 256;
    GemmParams p{};
    p.n_seg = n_seg;
    p.kb = segs[0].w.kb;
    p.panels = segs[0].w.panels;
    p.n = segs[0].w.n;
    p.y = y;
    p.ldy = ldy;
    p.status = status;
    uint32_t tiles = 0;
    for (uint32_t i = 0; i < n_seg; ++i) {
        p.seg[i] = {segs[i].m_begin, segs[i].m_end, tiles, 0u, segs[i].w.chunks};
        tiles += (segs[i].m_end - segs[i].m_begin + bn - 1) / bn * p.panels;
    }
    p.n_tiles = tiles;
    if (!tiles) return cudaSuccess;

    auto enc = encode_fn();
    if (!enc) return cudaErrorNotSupported;
    CUtensorMap map;
    const cuuint64_t dims[2] = {k, m_total};
    const cuuint64_t strides[1] = {k * 2};
    const cuuint32_t box[2] = {64u, (cuuint32_t)bn};
    const cuuint32_t estr[2] = {1u, 1u};
    const CUresult r = enc(&map, stage_f16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2,
                           const_cast<uint16_t *>(x), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                           CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return cudaErrorInvalidValue;
    const int out_f32 = out_dtype == 0;
    const uint32_t type = segs[0].w.type;
    if (type == 12) {
        if (bn == 64) return launch_bn<12, 64>(map, p, stage_f16, out_f32, sm_count, s);
        if (bn == 128) return launch_bn<12, 128>(map, p, stage_f16, out_f32, sm_count, s);
        return launch_bn<12, 256>(map, p, stage_f16, out_f32, sm_count, s);
    }
    if (bn == 64) return launch_bn<14, 64>(map, p, stage_f16, out_f32, sm_count, s);
    if (bn == 128) return launch_bn<14, 128>(map, p, stage_f16, out_f32, sm_count, s);
    return launch_bn<14, 256>(map, p, stage_f16, out_f32, sm_count, s);
}

}  // namespace tc
