// Quantised GEMM on CTA pairs with the weight operand in tensor memory
// (tcgen05 cta_group::2, sm_100a):
//     Y[m, n] = sum_k X[m, k] * W[n, k],  W in GGUF Q4_K / Q6_K, X bf16 (or fp16).
//
// A cluster of two CTAs computes one 256-weight-row x 256-token tile with
// MMAs of shape M = 256 (weight rows) x N = 256 (tokens) x K = 16, issued by
// one thread of CTA 0 (the leader) for both SMs:
//   A = dequantised weights, in TMEM: each CTA holds its own 128-row weight
//       panel as 128 lanes x 32 columns (64 K of bf16 / fp16 pairs) per stage,
//       written by the dequant warps with tcgen05.st straight from registers;
//   B = activations, in shared memory: each CTA loads its own 128 tokens x 64 K
//       per stage by TMA (K-major, 128-byte swizzle); the MMA reads both halves.
// Unpacked weights never touch shared memory.  Per 64-K stage an SM's shared
// memory serves only the activation copy and its MMA read (16 KB each), the
// packed bytes (about 4.5 KB) and the dequant warps' code reads; with the
// weight tile staged in shared memory instead, its stores and MMA reads made
// the shared-memory pipe, not the tensor core, the limit.
//
// TMEM (512 columns per CTA): columns 0-255 hold the accumulator D as
// [128 lanes = this CTA's weight rows] x [256 columns = the tile's tokens];
// columns 256 onwards hold the ring of A stages (32 columns each).  There is
// room for one accumulator only: the epilogue copies it to a shared-memory
// staging area (tcgen05.ld, then 2-byte stores that are conflict-free because
// a warp's 32 lanes hold 32 consecutive outputs of one token), releases it to
// the MMA right away, and writes Y from the staging area with TMA stores while
// the next tile accumulates.  (Splitting each k-step into two N = 128 MMAs to
// double-buffer halves of D measured slower than this single short stall.)
//
// Dequant mapping: one thread per weight row.  The 16 dequant warps form four
// groups of four (one warp per TMEM lane quarter); group q unpacks the q-th
// 64-K quarter of every packed chunk (128 rows x 256 K), 64 weights per thread,
// reading its sub-block scales directly from the packed bytes -- bit-exact to
// the reference decoder (native/core/gguf_decode.cpp:77-105).
//
// Warp roles (23 warps, both CTAs):
//   warp 0     activation producer (TMA);
//   warp 1     TMEM allocator (cta_group::2); in the leader, the MMA-issuing
//              thread; in the peer, a relay that forwards "this CTA's stage is
//              complete" to the leader's `full` barrier (one remote arrival per
//              stage, kept off the dequant warps);
//   warps 2-5  epilogue: tcgen05.ld of 32 tokens per thread-row, stores of Y;
//   warps 6-21 dequantisers;
//   warp 22    packed-chunk producer: one bulk copy per chunk as soon as its
//              slot frees (never queued behind activation copies that wait on
//              the MMA), plus an L2 prefetch of the chunk two ahead.
// The leader's MMA completion is committed to both CTAs' barriers
// (tcgen05.commit with a CTA mask).  No TMA load uses cluster multicast:
// every copy lands in the CTA that issued it and signals that CTA's own
// barrier.  Every wait is bounded; on timeout both CTAs raise their abort
// flags, set TC_STATUS_TIMEOUT, drain their own copies and MMAs, free TMEM and
// return.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <cstring>

#include "kq_epilogue.cuh"
#include "kq_sm100.cuh"
#include "tc_internal.h"

namespace tc {
namespace {

constexpr int kThreads = 736;
constexpr int kWProdWarp = 22;   // packed-chunk producer
constexpr int kDequantWarp0 = 6, kDequantWarps = 16;
constexpr int kEpiWarps = 4;
// Stage ring (activations in shared memory + A in TMEM, 64 K per stage):
// as deep as shared memory allows next to the packed-chunk ring and the
// 64 KB epilogue staging area -- 7 stages for Q4_K, 6 for Q6_K.
constexpr int stages_for(int type) { return type == 12 ? 7 : 6; }
constexpr int kWStages = 2;      // packed chunk ring (256 K per chunk)
constexpr int kMaxSeg = 32;
constexpr uint32_t kTileRows = 256, kTileTokens = 256, kHalf = 128;
constexpr uint32_t kACol0 = 256, kAStageCols = 32;

struct PairSeg {
    uint32_t m_begin, m_end, tile_begin, gate_row;
    const uint8_t *w;
};
// Tensor maps of the bf16 / fp16 Y tiles: this rank's Y, then its peer replicas.
struct YMaps {
    CUtensorMap m[kMaxPeers];
};
struct PairParams {
    PairSeg seg[kMaxSeg];
    uint32_t n_seg, n_tiles, kb, panels, pair_panels, n;
    // Work units: unit u is tile u / ksplit over super-block columns
    // [(u % ksplit) * kbu, +kbu).  ksplit > 1 (few tiles, split-K): each unit
    // stores its fp32 partial product at y + (u % ksplit) * split_stride and a
    // reduce kernel adds the splits in order; ksplit = 1: kbu = kb.
    uint32_t ksplit, kbu, n_units;
    uint64_t split_stride;
    void *y;
    uint64_t ldy;
    uint32_t *status;
    uint32_t y_tma;   // 16-bit Y written by TMA stores (16-byte aligned base and row pitch)
    EpiView epi;      // fused epilogue (flags 0: plain store); out_f16: fp16 rather than bf16
};

template <int TYPE>
struct PairLayout {
    static constexpr uint32_t x_stage = kHalf * 128;   // 128 tokens x 64 K x 2 B
    static constexpr uint32_t w_stage = chunk_bytes(TYPE);
    static constexpr uint32_t x_off = 0;
    static constexpr int kS = stages_for(TYPE);
    static constexpr uint32_t w_off = x_off + kS * x_stage;
    // Epilogue staging per warp: eight 32-token x 32-output bf16 boxes (16 KB).
    static constexpr uint32_t e_box = 32 * 64, e_warp = 8 * e_box;
    static constexpr uint32_t e_off = (w_off + kWStages * w_stage + 1023) / 1024 * 1024;
    static constexpr uint32_t bar_off = e_off + kEpiWarps * e_warp;
    // x_full[S] a_full[S] full[S] st_empty[S] w_full[W] w_empty[W] acc_full acc_empty fin
    static constexpr uint32_t n_bars = 4 * kS + 2 * kWStages + 3;
    static constexpr uint32_t misc_off = bar_off + n_bars * 8;
    static constexpr uint32_t bytes = misc_off + 16 + 1024;  // + alignment slack
    static constexpr uint32_t tmem_cols = 512;
    static_assert(bytes <= 232448, "shared memory per CTA exceeds the sm_100 limit");
    static_assert(kACol0 + kS * kAStageCols <= tmem_cols, "TMEM budget");
};

// ------------------------------------------------------------ cluster PTX
__device__ __forceinline__ uint32_t cta_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
// Address of the same shared-memory offset in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t cluster_addr(uint32_t saddr, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
    return r;
}
// Arrive on a barrier of either CTA of the pair (default .release.cta
// semantics).  What the arrival publishes lives in the arriving CTA (its
// activation stage and TMEM A stage, or TMEM already read back), completed
// before the arrival is sent; a cluster-scope release would add a full memory
// barrier to every stage.
__device__ __forceinline__ void bar_arrive_cluster(uint32_t caddr) {
    asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(caddr) : "memory");
}
__device__ __forceinline__ void cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// Abort state of one CTA: its own flag and the peer's flag (cluster address).
struct Abort {
    volatile uint32_t *flag;
    uint32_t peer_flag;
    uint32_t *status;
};
__device__ __noinline__ bool pwait_slow(uint32_t b, uint32_t parity, volatile uint32_t *flag, uint32_t peer_flag,
                                        uint32_t *status, bool honor_abort) {
    const uint64_t t0 = gtimer();
    for (;;) {
        if (bar_try_sleep(b, parity, 20000u)) return true;
        if (honor_abort && *flag) return false;
        if (gtimer() - t0 > kTimeoutNs) {
            atomicOr(status, kStatusTimeout);
            *flag = 1u;
            asm volatile("st.shared::cluster.u32 [%0], %1;" ::"r"(peer_flag), "r"(1u) : "memory");
            return false;
        }
    }
}
__device__ __forceinline__ bool pwait(uint32_t b, uint32_t parity, const Abort &a, bool honor_abort = true) {
    if (bar_try(b, parity)) return true;
    return pwait_slow(b, parity, a.flag, a.peer_flag, a.status, honor_abort);
}

// Instruction descriptor, kind::f16, cta_group::2: D fp32, A/B bf16 (or fp16),
// A from TMEM, B K-major, M = 256, N = 256.
template <bool F16>
__device__ __forceinline__ constexpr uint32_t pair_idesc() {
    return (1u << 4) | ((F16 ? 0u : 1u) << 7) | ((F16 ? 0u : 1u) << 10) | ((kTileTokens >> 3) << 17) |
           ((kTileRows >> 4) << 24);
}
__device__ __forceinline__ void mma_pair_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b, uint32_t idesc,
                                            uint32_t acc) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::2.kind::f16 [%0], [%1], %2, %3, p;\n}\n"
        ::"r"(d_tmem), "r"(a_tmem), "l"(b), "r"(idesc), "r"(acc));
}
// Arrive (once the leader's MMAs issued so far complete) on the barrier at
// offset `b` in both CTAs of the pair.
__device__ __forceinline__ void commit_both(uint32_t b) {
    asm volatile(
        "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;"
        ::"r"(b), "h"((uint16_t)3) : "memory");
}
// 16 consecutive 32-bit TMEM columns of this thread's lane.
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&v)[16]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, "
        "%14, %15, %16};"
        ::"r"(taddr), "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]),
          "r"(v[8]), "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
        : "memory");
}
// Hint: bring `bytes` at `src` into L2 (no completion tracking).
__device__ __forceinline__ void l2_prefetch(const void *src, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}
__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tma_store_2d(const CUtensorMap *map, uint32_t src, int x, int y) {
    asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];"
                 ::"l"(reinterpret_cast<uint64_t>(map)), "r"(src), "r"(x), "r"(y) : "memory");
}
// fp32 box (x = output columns, y = tokens, z = split-K share) of a 3-D map.
__device__ __forceinline__ void tma_store_3d(const CUtensorMap *map, uint32_t src, int x, int y, int z) {
    asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%2, %3, %4}], [%1];"
                 ::"l"(reinterpret_cast<uint64_t>(map)), "r"(src), "r"(x), "r"(y), "r"(z) : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_read0() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
__device__ __forceinline__ uint32_t lds32(const uint8_t *p) { return *reinterpret_cast<const uint32_t *>(p); }
__device__ __forceinline__ uint4 lds128(const uint8_t *p) { return *reinterpret_cast<const uint4 *>(p); }

// The 32-byte code slice of one row, as 8 words in K order.  The two 16-byte
// halves are read in an order set by bit 2 of the row slot, so the eight rows
// served by one shared-memory wavefront fall in eight different bank groups.
__device__ __forceinline__ void load_row32(const uint8_t *p, uint32_t slot, uint32_t (&w)[8]) {
    const uint32_t h = (slot >> 2) & 1u;
    const uint4 a = lds128(p + 16 * h), b = lds128(p + 16 * (h ^ 1u));
    const uint4 lo = h ? b : a, hi = h ? a : b;
    w[0] = lo.x; w[1] = lo.y; w[2] = lo.z; w[3] = lo.w;
    w[4] = hi.x; w[5] = hi.y; w[6] = hi.z; w[7] = hi.w;
}

// One thread's share of a stage: weight row r, the q-th 64-K quarter of the
// packed chunk `wc`, written to the TMEM A stage at `ta` (this thread's lane)
// as 32 columns of packed pairs (column j = weights 2j, 2j+1 of the quarter).
// Q4_K: byte j of the row's quarter holds weight j (low nibble, sub-block 2q)
// and weight 32 + j (high nibble, sub-block 2q + 1).  Q5_K: the same, plus
// bits 2q and 2q + 1 of qh[j] as each code's fifth bit.  Q6_K: half h = q / 2,
// parts of ql and the 2-bit planes of qh give weights j and 32 + j.
template <int TYPE, bool F16>
__device__ __forceinline__ void unpack_row(const uint8_t *wc, uint32_t q, uint32_t r, uint32_t ta, bool &ovf) {
    constexpr float kF16Inf = 65520.0f;   // smallest magnitude that rounds to inf
    const uint32_t slot = row_slot(r);
    uint32_t out[16];
    if (affine_type(TYPE)) {
        constexpr bool kQ5 = TYPE == 13;
        constexpr uint32_t kDm = kQ5 ? kQ5Dm : kQ4Dm, kSc = kQ5 ? kQ5Sc : kQ4Sc, kQs = kQ5 ? kQ5Qs : kQ4Qs;
        constexpr float kQMax = kQ5 ? 31.0f : 15.0f;
        const uint32_t dm = lds32(wc + kDm + r * 4);
        const float d = half_bits_to_float((uint16_t)(dm & 0xffffu)), dmin = half_bits_to_float((uint16_t)(dm >> 16));
        const uint8_t *scp = wc + kSc + r * 12;
        uint32_t s0, m0, s1, m1;
        const uint32_t sw0 = lds32(scp), sw1 = lds32(scp + 4), sw2 = lds32(scp + 8);
        q4k_scale_min_w(2 * q, sw0, sw1, sw2, s0, m0);
        q4k_scale_min_w(2 * q + 1, sw0, sw1, sw2, s1, m1);
        const float a0 = d * (float)s0, b0 = dmin * (float)m0, a1 = d * (float)s1, b1 = dmin * (float)m1;
        if (F16)
            ovf |= fmaxf(fabsf(b0), fabsf(fmaf(a0, kQMax, -b0))) >= kF16Inf ||
                   fmaxf(fabsf(b1), fabsf(fmaf(a1, kQMax, -b1))) >= kF16Inf;
        uint32_t w[8], hb[8];
        load_row32(wc + kQs + q * 4096 + slot * 32, slot, w);
        if (kQ5) load_row32(wc + kQ5Qh + slot * 32, slot, hb);
        // Scales in the form the staging needs (f32x2 exact, or f16x2).
        const uint64_t off2 = f2splat(-8388608.0f);
        uint64_t sc2 = f2splat(a0), mn2 = f2splat(-b0);
        uint32_t sch = 0, mnh = 0;
        if (F16) { sch = h2splat(a0); mnh = h2splat(-min_compensated(a0, b0)); }
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const uint32_t c = kQ5 ? (w[i] & 0x0F0F0F0Fu) | (((hb[i] >> (2 * q)) & 0x01010101u) << 4)
                                   : w[i] & 0x0F0F0F0Fu;
            const uint2 v = F16 ? four_values_h<TYPE>(c, sch, mnh) : four_values<TYPE, F16>(c, sc2, off2, mn2);
            out[2 * i] = v.x;
            out[2 * i + 1] = v.y;
        }
        tmem_st16(ta, out);
        // Q4_K high nibbles are read in place (16 q) with the scale
        // pre-divided by 16, a power of two, so every product stays exact;
        // Q5_K's 5-bit codes are shifted down instead.
        const float a1s = kQ5 ? a1 : a1 * 0.0625f;
        sc2 = f2splat(a1s);
        mn2 = f2splat(-b1);
        if (F16) { sch = h2splat(a1s); mnh = h2splat(-min_compensated(a1s, b1)); }
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const uint32_t c = kQ5 ? ((w[i] >> 4) & 0x0F0F0F0Fu) | (((hb[i] >> (2 * q + 1)) & 0x01010101u) << 4)
                                   : w[i] & 0xF0F0F0F0u;
            const uint2 v = F16 ? four_values_h<TYPE>(c, sch, mnh) : four_values<TYPE, F16>(c, sc2, off2, mn2);
            out[2 * i] = v.x;
            out[2 * i + 1] = v.y;
        }
        tmem_st16(ta + 16, out);
    } else {
        const uint32_t h = q >> 1, shift = (q & 1) * 4, g0 = 2 * (q & 1);
        const float d = half_bits_to_float(*reinterpret_cast<const uint16_t *>(wc + kQ6D + r * 2));
        const uint32_t sc4 = lds32(wc + kQ6Sc + r * 16 + 8 * h + 2 * g0);   // 4 int8 scales
        const float sa0 = d * (float)(int8_t)(sc4 & 0xff), sa1 = d * (float)(int8_t)((sc4 >> 8) & 0xff);
        const float sb0 = d * (float)(int8_t)((sc4 >> 16) & 0xff), sb1 = d * (float)(int8_t)(sc4 >> 24);
        if (F16)
            ovf |= 32.0f * fmaxf(fmaxf(fabsf(sa0), fabsf(sa1)), fmaxf(fabsf(sb0), fabsf(sb1))) >= kF16Inf;
        const uint64_t off2 = f2splat(-8388640.0f);  // -(2^23 + 32)
        uint32_t qh[8], l[8];
        load_row32(wc + kQ6Qh + (h * kPanelRows + slot) * 32, slot, qh);
        load_row32(wc + kQ6Ql + ((h * 2 + 0) * kPanelRows + slot) * 32, slot, l);
        {
            const uint64_t s0 = f2splat(sa0), s1 = f2splat(sa1);
            const uint32_t h0 = F16 ? h2splat(sa0) : 0u, h1 = F16 ? h2splat(sa1) : 0u;
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const uint32_t c = ((l[i] >> shift) & 0x0F0F0F0Fu) | (((qh[i] >> (2 * g0)) & 0x03030303u) << 4);
                const uint2 v = F16 ? four_values_h<14>(c, i < 4 ? h0 : h1, 0u)
                                    : four_values<14, F16>(c, i < 4 ? s0 : s1, off2, 0);
                out[2 * i] = v.x;
                out[2 * i + 1] = v.y;
            }
            tmem_st16(ta, out);
        }
        load_row32(wc + kQ6Ql + ((h * 2 + 1) * kPanelRows + slot) * 32, slot, l);
        {
            const uint64_t s0 = f2splat(sb0), s1 = f2splat(sb1);
            const uint32_t h0 = F16 ? h2splat(sb0) : 0u, h1 = F16 ? h2splat(sb1) : 0u;
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const uint32_t c = ((l[i] >> shift) & 0x0F0F0F0Fu) | (((qh[i] >> (2 * g0 + 2)) & 0x03030303u) << 4);
                const uint2 v = F16 ? four_values_h<14>(c, i < 4 ? h0 : h1, 0u)
                                    : four_values<14, F16>(c, i < 4 ? s0 : s1, off2, 0);
                out[2 * i] = v.x;
                out[2 * i + 1] = v.y;
            }
            tmem_st16(ta + 16, out);
        }
    }
}

// ------------------------------------------------------------ tiles
struct PairTile {
    uint32_t m0, m_end, pp;   // first token, segment end, pair-panel (256 weight rows)
    const uint8_t *w;
    uint32_t gate_row;
};
__device__ __forceinline__ PairTile pair_tile(const PairParams &p, uint32_t t) {
    uint32_t s = 0;
    while (s + 1 < p.n_seg && t >= p.seg[s + 1].tile_begin) ++s;
    const uint32_t local = t - p.seg[s].tile_begin;
    return {p.seg[s].m_begin + (local / p.pair_panels) * kTileTokens, p.seg[s].m_end, local % p.pair_panels,
            p.seg[s].w, p.seg[s].gate_row};
}
__device__ __forceinline__ uint16_t to16(float v, bool f16) {
    return f16 ? __half_as_ushort(__float2half_rn(v)) : __bfloat16_as_ushort(__float2bfloat16_rn(v));
}

// ------------------------------------------------------------ the kernel
template <int TYPE, bool F16, bool OUT_F32>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    pair_gemm_kernel(const __grid_constant__ CUtensorMap xmap, const __grid_constant__ YMaps ymaps,
                     const __grid_constant__ PairParams p) {
    using L = PairLayout<TYPE>;
    constexpr uint32_t kChunk = chunk_bytes(TYPE);
    constexpr int kStages = L::kS;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const uint32_t warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    const uint32_t rank = cta_rank();          // 0: leader, issues the MMAs for both CTAs
    const uint32_t pair = blockIdx.x >> 1, n_pairs = gridDim.x >> 1;

    const uint32_t bars = su32(smem + L::bar_off);
    auto x_full = [&](uint32_t i) { return bars + 8 * i; };
    auto a_full = [&](uint32_t i) { return bars + 8 * (kStages + i); };
    auto full = [&](uint32_t i) { return bars + 8 * (2 * kStages + i); };
    auto st_empty = [&](uint32_t i) { return bars + 8 * (3 * kStages + i); };
    auto w_full = [&](uint32_t i) { return bars + 8 * (4 * kStages + i); };
    auto w_empty = [&](uint32_t i) { return bars + 8 * (4 * kStages + kWStages + i); };
    const uint32_t acc_full = bars + 8 * (4 * kStages + 2 * kWStages);
    const uint32_t acc_empty = acc_full + 8, fin = acc_full + 16;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + L::misc_off);
    volatile uint32_t *abort_flag = tmem_slot + 1;
    // Units of this pair: pair, pair + n_pairs, ...; 4 stages per packed chunk.
    const uint32_t my_units = p.n_units > pair ? (p.n_units - pair + n_pairs - 1) / n_pairs : 0;
    const uint32_t n_chunks = my_units * p.kbu;

    if (threadIdx.x == 0) {
        for (int i = 0; i < kStages; ++i) {
            bar_init(x_full(i), 1);
            bar_init(a_full(i), 4);        // the four warps of one dequant group
            bar_init(full(i), 1);          // leader's copy: the peer's relay
            bar_init(st_empty(i), 1);
        }
        for (int i = 0; i < kWStages; ++i) {
            bar_init(w_full(i), 1);
            bar_init(w_empty(i), kDequantWarps);
        }
        bar_init(acc_full, 1);
        bar_init(acc_empty, 2 * kEpiWarps);   // leader's copy is the one used
        bar_init(fin, 1);
        *abort_flag = 0u;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;"
                     ::"r"(su32(tmem_slot)), "r"(L::tmem_cols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;");
    }
    tc_fence_before();
    cluster_sync();   // both CTAs: barriers initialised, TMEM allocated
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const Abort ab{abort_flag, cluster_addr(su32(tmem_slot + 1), rank ^ 1u), p.status};

    if (threadIdx.x == 0) asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    if (warp == 0) {
        // ---------------------------------------------------- activation producer
        if (lane == 0) {
            // X (and the Y the epilogue writes) may belong to the previous
            // kernel in the stream: wait for it before the first load.
            asm volatile("griddepcontrol.wait;" ::: "memory");
            uint32_t x_last[kStages];
            bool x_used[kStages] = {};
            bool ok = true;
            uint32_t i = 0;   // stage counter
            for (uint32_t u = pair; ok && u < p.n_units; u += n_pairs) {
                const int my_m = (int)(pair_tile(p, u / p.ksplit).m0 + rank * kHalf);
                const uint32_t s0 = 4 * (u % p.ksplit) * p.kbu;   // first 64-K stage of the unit
                for (uint32_t s = 0; ok && s < 4 * p.kbu; ++s, ++i) {
                    const uint32_t st = i % kStages, ph = (i / kStages) & 1;
                    if (!(ok = pwait(st_empty(st), ph ^ 1, ab))) break;
                    bar_expect_tx(x_full(st), L::x_stage);
                    tma_load_2d(su32(smem + L::x_off + st * L::x_stage), &xmap, x_full(st), (int)((s0 + s) * 64),
                                my_m);
                    x_last[st] = ph; x_used[st] = true;
                }
            }
            // Drain: every copy this thread issued has landed before exit.
            for (int k = 0; k < kStages; ++k)
                if (x_used[k]) pwait(x_full(k), x_last[k], ab, false);
        }
        __syncwarp();
    } else if (warp == (uint32_t)kWProdWarp) {
        // ---------------------------------------------------- packed-chunk producer
        if (lane == 0) {
            asm volatile("griddepcontrol.wait;" ::: "memory");
            uint32_t w_last[kWStages];
            bool w_used[kWStages] = {};
            bool ok = true;
            // Chunk c of this pair's sequence: unit c / kbu, K block
            // (unit % ksplit) * kbu + c % kbu.  A missing second panel (odd
            // panel count) re-reads the last panel; its outputs fall past N
            // and are never stored.
            auto chunk_src = [&](uint32_t c) -> const uint8_t * {
                const uint32_t u = pair + (c / p.kbu) * n_pairs;
                const PairTile T = pair_tile(p, u / p.ksplit);
                uint32_t panel = 2 * T.pp + rank;
                if (panel >= p.panels) panel = p.panels - 1;
                uint64_t at = (uint64_t)panel * p.kb + (u % p.ksplit) * p.kbu + c % p.kbu;
                if (!tc_in_bounds(at < (uint64_t)p.panels * p.kb, p.status)) at = 0;
                return T.w + at * kChunk;
            };
            for (uint32_t c = 0; c < kWStages && c < n_chunks; ++c) l2_prefetch(chunk_src(c), kChunk);
            for (uint32_t c = 0; ok && c < n_chunks; ++c) {
                const uint32_t ws = c % kWStages, wph = (c / kWStages) & 1;
                if (c + kWStages < n_chunks) l2_prefetch(chunk_src(c + kWStages), kChunk);
                if (!(ok = pwait(w_empty(ws), wph ^ 1, ab))) break;
                bar_expect_tx(w_full(ws), kChunk);
                bulk_load(su32(smem + L::w_off + ws * L::w_stage), chunk_src(c), kChunk, w_full(ws));
                w_last[ws] = wph; w_used[ws] = true;
            }
            for (int k = 0; k < kWStages; ++k)
                if (w_used[k]) pwait(w_full(k), w_last[k], ab, false);
        }
        __syncwarp();
    } else if (warp == 1) {
        if (lane == 0 && rank == 0) {
            // ---------------------------------------------------- MMA issuer (leader)
            constexpr uint32_t idesc = pair_idesc<F16>();
            bool ok = true;
            uint32_t i = 0;   // stage counter
            for (uint32_t tt = 0; ok && tt < my_units; ++tt) {
                if (!(ok = pwait(acc_empty, (tt & 1) ^ 1, ab))) break;
                tc_fence_after();
                for (uint32_t s = 0; ok && s < 4 * p.kbu; ++s, ++i) {
                    const uint32_t st = i % kStages, ph = (i / kStages) & 1;
                    if (!(ok = pwait(x_full(st), ph, ab))) break;
                    if (!(ok = pwait(a_full(st), ph, ab))) break;
                    if (!(ok = pwait(full(st), ph, ab))) break;   // the peer's stage
                    tc_fence_after();
                    const uint32_t a_col = tmem + kACol0 + st * kAStageCols;
                    const uint32_t b_addr = su32(smem + L::x_off + st * L::x_stage);
#pragma unroll
                    for (uint32_t kk = 0; kk < 4; ++kk)
                        mma_pair_ts(tmem, a_col + 8 * kk, sw128_desc(b_addr + kk * 32), idesc, (s | kk) ? 1u : 0u);
                    commit_both(st_empty(st));
                }
                if (!ok) break;
                commit_both(acc_full);
            }
            // Every MMA issued by this thread has completed (in both CTAs)
            // before either CTA frees its TMEM.
            commit_both(fin);
        } else if (lane == 0) {
            // ---------------------------------------------------- relay (peer)
            for (uint32_t i = 0; i < 4 * n_chunks; ++i) {
                const uint32_t st = i % kStages, ph = (i / kStages) & 1;
                if (!pwait(x_full(st), ph, ab)) break;
                if (!pwait(a_full(st), ph, ab)) break;
                bar_arrive_cluster(cluster_addr(full(st), 0));
            }
        }
        if (lane == 0) pwait(fin, 0, ab, false);
        __syncwarp();
    } else if (warp >= (uint32_t)kDequantWarp0 && warp < (uint32_t)kWProdWarp) {
        // ---------------------------------------------------- dequantisers
        // Group q = (warp - 6) / 4 unpacks quarter q of every chunk: stage
        // 4c + q.  Waits are warp-uniform (__all_sync) because tcgen05.st is
        // a warp-collective; on abort the whole warp leaves.
        const uint32_t q = (warp - kDequantWarp0) / 4, quarter = warp & 3;
        const uint32_t r = 32 * quarter + lane;            // weight row = TMEM lane
        const uint32_t t_lane = tmem + ((32 * quarter) << 16) + kACol0;
        bool ovf = false;
        for (uint32_t c = 0; c < n_chunks; ++c) {
            const uint32_t ws = c % kWStages, i = 4 * c + q, st = i % kStages, ph = (i / kStages) & 1;
            if (!__all_sync(0xffffffffu, pwait(w_full(ws), (c / kWStages) & 1, ab))) break;
            if (!__all_sync(0xffffffffu, pwait(st_empty(st), ph ^ 1, ab))) break;
            tc_fence_after();
            unpack_row<TYPE, F16>(smem + L::w_off + ws * L::w_stage, q, r, t_lane + st * kAStageCols, ovf);
            tmem_st_wait();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) {
                bar_arrive(w_empty(ws));
                bar_arrive(a_full(st));
            }
        }
        if (F16 && ovf) atomicOr(p.status, kStatusF16);
    } else {
        // ---------------------------------------------------- epilogue
        // Thread = weight row n of this CTA's panel; D column c = token m0 + c
        // (columns 0-127: CTA 0's activation rows, 128-255: CTA 1's).  The
        // accumulator is read out in eight 32-token pieces; a piece that lies
        // inside the segment goes to this warp's staging box (bf16, [token]
        // [32 outputs]) for a TMA store, a piece at a ragged segment end (and
        // f32 output) is stored directly, the warp's 32 lanes writing 32
        // consecutive outputs of one token.  TMEM is released before the TMA
        // stores are issued.
        const uint32_t quad = warp & 3;   // TMEM lanes 32*quad .. +31
        uint8_t *stage = smem + L::e_off + quad * L::e_warp;
        for (uint32_t tt = 0; tt < my_units; ++tt) {
            const uint32_t u = pair + tt * n_pairs;
            const PairTile T = pair_tile(p, u / p.ksplit);
            const uint64_t yoff = (uint64_t)(u % p.ksplit) * p.split_stride;   // split-K partial slice
            const uint32_t n0 = (2 * T.pp + rank) * 128 + quad * 32, n = n0 + lane;
            if (!__all_sync(0xffffffffu, pwait(acc_full, tt & 1, ab))) break;
            tc_fence_after();
            if (p.y_tma) {
                if (lane == 0) bulk_wait_read0();   // the last tile's stores have read the staging area
                __syncwarp();
            }
            const uint32_t taddr = tmem + ((quad * 32) << 16);
            if (OUT_F32 && p.y_tma) {
                // Plain fp32 tile (also every split-K partial): 32-token x
                // 32-output fp32 boxes (4 KB) staged in shared memory and
                // written by TMA stores -- per-element stores from the four
                // epilogue warps measured several times slower.  The warp's
                // 16 KB staging area holds four boxes, so the eight pieces go
                // out in two rounds; TMEM is released after the second
                // round's loads.  Ragged pieces are stored directly.
                const uint32_t split = u % p.ksplit;
#pragma unroll 1
                for (uint32_t half = 0; half < 2; ++half) {
                    if (half) {
                        if (lane == 0) bulk_wait_read0();   // round 0 has left the staging area
                        __syncwarp();
                    }
                    uint32_t boxes = 0;
#pragma unroll 1
                    for (uint32_t jj = 0; jj < 4; ++jj) {
                        const uint32_t j = 4 * half + jj, t0 = T.m0 + 32 * j;
                        if (t0 >= T.m_end || n0 >= p.n) break;
                        uint32_t v[32];
                        tmem_ld32(taddr + 32 * j, v);
                        if (t0 + 32 <= T.m_end && n0 + 32 <= p.n) {
                            float *sb = reinterpret_cast<float *>(stage + jj * 4096) + lane;
#pragma unroll
                            for (uint32_t c = 0; c < 32; ++c) sb[c * 32] = __uint_as_float(v[c]);
                            boxes |= 1u << jj;
                        } else if (n < p.n) {
#pragma unroll
                            for (uint32_t c = 0; c < 32; ++c)
                                if (t0 + c < T.m_end)
                                    store_out_all(p.epi, p.y, yoff + (uint64_t)(t0 + c) * p.ldy + n,
                                                  __uint_as_float(v[c]), true, false);
                        }
                    }
                    if (half) {   // every TMEM load of the tile is done: hand D back
                        tc_fence_before();
                        __syncwarp();
                        if (lane == 0) bar_arrive_cluster(cluster_addr(acc_empty, 0));
                    }
                    if (boxes) {
                        fence_proxy_async();
                        __syncwarp();
                        if (lane == 0) {
                            for (uint32_t jj = 0; jj < 4; ++jj)
                                if (boxes & (1u << jj))
                                    tma_store_3d(&ymaps.m[0], su32(stage + jj * 4096), (int)n0,
                                                 (int)(T.m0 + 32 * (4 * half + jj)), (int)split);
                            bulk_commit();
                        }
                    }
                }
                continue;
            }
            uint32_t tma_pieces = 0;   // bit j: piece j goes out by TMA
            const bool f16 = p.epi.out_f16;
            // Fused epilogue (p.epi.flags): bias / GELU / SwiGLU are applied on
            // the way into the staging box, so the accumulator is held no
            // longer than for a plain store; a SwiGLU box is 32 tokens x the
            // warp's 16 outputs (its gate rows).  Pieces that cannot go out by
            // TMA (ragged ends, f32 output, gated residual: the host leaves
            // y_tma 0) take the direct per-element path.
            const uint32_t fl = p.epi.flags;
            const bool glu = fl & TC_EPI_SWIGLU;
            const EpiRow er = fl ? epi_row(p.epi, min(n, p.n - 1), T.gate_row) : EpiRow{0.f, 0.f, n, true};
#pragma unroll 1
            for (uint32_t j = 0; j < kTileTokens / 32; ++j) {
                const uint32_t t0 = T.m0 + 32 * j;
                if (t0 >= T.m_end || n0 >= p.n) break;   // past the segment / a missing second panel
                uint32_t v[32];
                tmem_ld32(taddr + 32 * j, v);
                // TMA only for boxes wholly inside Y: past a ragged N the store
                // would write up to the next 16-byte boundary of the row.
                if (!OUT_F32 && p.y_tma && t0 + 32 <= T.m_end && n0 + 32 <= p.n) {
                    tma_pieces |= 1u << j;
                    if (!fl) {
                        uint16_t *sb = reinterpret_cast<uint16_t *>(stage + j * L::e_box) + lane;
#pragma unroll
                        for (uint32_t c = 0; c < 32; ++c) sb[c * 32] = to16(__uint_as_float(v[c]), f16);
                    } else if (glu) {
                        // Gate lane L (L & 8 == 0) and up lane L + 8 share
                        // output column (L >> 4) * 8 + (L & 7): the gate lane
                        // produces tokens 0-15 of the piece, the up lane 16-31,
                        // each fetching the partner's value with one shuffle.
                        // No divergent branch in the loop.
                        const bool gate_lane = er.writer;
                        uint16_t *sb = reinterpret_cast<uint16_t *>(stage + j * L::e_box) + (lane >> 4) * 8 + (lane & 7) +
                                       (gate_lane ? 0 : 16 * 16);
#pragma unroll
                        for (uint32_t c = 0; c < 16; ++c) {
                            const float lo = __uint_as_float(v[c]) + er.bias;        // token c
                            const float hi = __uint_as_float(v[c + 16]) + er.bias;   // token c + 16
                            const float up_lo = __shfl_down_sync(0xffffffffu, lo, 8);    // to the gate lane
                            const float gate_hi = __shfl_up_sync(0xffffffffu, hi, 8);    // to the up lane
                            const float g = gate_lane ? lo : gate_hi, u = gate_lane ? up_lo : hi;
                            sb[c * 16] = to16(silu(g) * u, f16);
                        }
                    } else {
                        uint16_t *sb = reinterpret_cast<uint16_t *>(stage + j * L::e_box) + lane;
                        if (fl & TC_EPI_GELU_TANH) {
#pragma unroll
                            for (uint32_t c = 0; c < 32; ++c)
                                sb[c * 32] = to16(gelu_tanh(__uint_as_float(v[c]) + er.bias), f16);
                        } else if (fl & TC_EPI_GELU_ERF) {
#pragma unroll
                            for (uint32_t c = 0; c < 32; ++c)
                                sb[c * 32] = to16(gelu_erf(__uint_as_float(v[c]) + er.bias), f16);
                        } else {
#pragma unroll
                            for (uint32_t c = 0; c < 32; ++c) sb[c * 32] = to16(__uint_as_float(v[c]) + er.bias, f16);
                        }
                    }
                } else if (fl) {
                    // all lanes: the SwiGLU pairing shuffles
                    epi_piece<OUT_F32>(p.epi, er, v, n < p.n, t0, T.m_end, p.y, p.ldy);
                } else if (n < p.n) {
#pragma unroll
                    for (uint32_t c = 0; c < 32; ++c) {
                        const uint32_t m = t0 + c;
                        if (m < T.m_end)
                            store_out_all(p.epi, p.y, yoff + (uint64_t)m * p.ldy + n, __uint_as_float(v[c]), OUT_F32,
                                          f16);
                    }
                }
            }
            // Every TMEM load has completed (tcgen05.ld waits): hand D back.
            tc_fence_before();
            __syncwarp();
            if (lane == 0) bar_arrive_cluster(cluster_addr(acc_empty, 0));
            if (tma_pieces) {
                fence_proxy_async();
                __syncwarp();
                if (lane == 0) {
                    // this rank's Y, then each peer replica (N-column sharding)
                    for (uint32_t d = 0; d <= p.epi.n_peer; ++d)
                        for (uint32_t j = 0; j < kTileTokens / 32; ++j)
                            if (tma_pieces & (1u << j))
                                tma_store_2d(&ymaps.m[d], su32(stage + j * L::e_box), (int)(glu ? n0 / 2 : n0),
                                             (int)(T.m0 + 32 * j));
                    bulk_commit();
                }
            }
        }
        if (lane == 0) bulk_wait_all();
        __syncwarp();
        // Peer replicas: make this thread's stores (and, after the bulk wait,
        // its TMA stores) visible system-wide before the kernel ends, so that
        // a flag raised after it publishes them (tc_cuda_peer_barrier).
        if (p.epi.n_peer) __threadfence_system();
    }

    tc_fence_before();
    cluster_sync();   // no CTA leaves while its peer may still signal it
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(L::tmem_cols));
    }
}

// ------------------------------------------------------------ host side
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    // The driver entry point is process-wide; a function-local static is
    // initialised once, thread-safely.
    static const PFN_cuTensorMapEncodeTiled_v12000 fn = [] {
        void *ptr = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
        return static_cast<PFN_cuTensorMapEncodeTiled_v12000>(nullptr);
    }();
    return fn;
}

template <int TYPE, bool F16, bool OUT_F32>
cudaError_t launch_pair_inst(const CUtensorMap &xm, const YMaps &ym, const PairParams &p, int sm_count,
                             cudaStream_t s) {
    using L = PairLayout<TYPE>;
    auto kernel = pair_gemm_kernel<TYPE, F16, OUT_F32>;
    // Shared-memory opt-in and co-resident 2-CTA clusters, per device.
    static DeviceCache cache;
    int max_clusters = 0;
    cudaError_t e = per_device(cache, max_clusters, [&](int &v) {
        cudaError_t r = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)L::bytes);
        if (r != cudaSuccess) return r;
        cudaLaunchConfig_t q = {};
        q.gridDim = dim3(2);
        q.blockDim = dim3(kThreads);
        q.dynamicSmemBytes = L::bytes;
        if ((r = cudaOccupancyMaxActiveClusters(&v, kernel, &q)) != cudaSuccess) return r;
        return v < 1 ? cudaErrorInvalidConfiguration : cudaSuccess;
    });
    if (e != cudaSuccess) return e;
    uint32_t pairs = p.n_units < (uint32_t)max_clusters ? p.n_units : (uint32_t)max_clusters;
    if (sm_count >= 2 && pairs > (uint32_t)sm_count / 2) pairs = (uint32_t)sm_count / 2;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * pairs);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = L::bytes;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, xm, ym, p);
}

// fp32 Y (or split-K partials) as a 3-D tensor map: x = output columns (n),
// y = tokens (m_total, row pitch ld), z = split-K share (pitch `plane`
// elements); 32 x 32 x 1 boxes.  Base and pitches must be 16-byte aligned.
bool encode_f32_map(PFN_cuTensorMapEncodeTiled_v12000 enc, CUtensorMap *map, void *base, uint32_t n,
                    uint64_t m_total, uint64_t ld, uint32_t planes, uint64_t plane) {
    if ((reinterpret_cast<uintptr_t>(base) & 15u) || (ld * 4) % 16 || (plane * 4) % 16) return false;
    const cuuint64_t dims[3] = {n, m_total, planes};
    const cuuint64_t strides[2] = {ld * 4, plane * 4};
    const cuuint32_t box[3] = {32u, 32u, 1u};
    const cuuint32_t estr[3] = {1u, 1u, 1u};
    return enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, base, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
               CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_NONE,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

uint32_t pair_tiles(const SegmentView *segs, uint32_t n_seg) {
    const uint32_t pair_panels = (segs[0].w.panels + 1) / 2;
    uint32_t tiles = 0;
    for (uint32_t i = 0; i < n_seg; ++i)
        tiles += (segs[i].m_end - segs[i].m_begin + kTileTokens - 1) / kTileTokens * pair_panels;
    return tiles;
}

}  // namespace

uint32_t pair_ksplit(const SegmentView *segs, uint32_t n_seg, int sm_count) {
    if (!n_seg) return 1;
    const uint32_t tiles = pair_tiles(segs, n_seg), clusters = (uint32_t)max(sm_count, 2) / 2, kb = segs[0].w.kb;
    if (!tiles || 2 * tiles >= clusters) return 1;   // at least half the pairs busy without a split
    // The divisor of kb (at most 16 shares, the reduce kernel's limit) that
    // fills the most pairs in one wave.
    uint32_t best = 1;
    for (uint32_t d = 2; d <= kb && d <= 16 && d * tiles <= clusters; ++d)
        if (kb % d == 0) best = d;
    return best;
}

cudaError_t launch_split_reduce(const float *part, uint32_t ksplit, uint64_t stride, uint32_t n_w, uint32_t m_begin,
                                uint32_t rows, const EpiView &e, uint32_t gate_row, void *y, uint64_t ldy,
                                int out_dtype, cudaStream_t s);

namespace {

cudaError_t launch_pair_split(const CUtensorMap &xm, const YMaps &ym, PairParams p, const SegmentView *segs,
                              uint32_t n_seg, const SplitK &sk, void *y, uint64_t ldy, int out_dtype, int stage_f16,
                              uint64_t m_total, int sm_count, cudaStream_t s);

}  // namespace

cudaError_t launch_gemm_pair(const SegmentView *segs, uint32_t n_seg, const uint16_t *x, uint64_t m_total,
                             uint64_t k, void *y, uint64_t ldy, int out_dtype, int stage_f16, int sm_count,
                             uint32_t *status, cudaStream_t s, const EpiView *epi, const SplitK *split) {
    if (n_seg == 0) return cudaSuccess;
    if (n_seg > (uint32_t)kMaxSeg) return cudaErrorInvalidValue;
    PairParams p{};
    p.n_seg = n_seg;
    p.kb = segs[0].w.kb;
    p.panels = segs[0].w.panels;
    p.pair_panels = (p.panels + 1) / 2;
    p.n = segs[0].w.n;
    p.y = y;
    p.ldy = ldy;
    p.status = status;
    if (epi) p.epi = *epi;
    p.epi.out_f16 = out_dtype == 1;
    uint32_t tiles = 0;
    for (uint32_t i = 0; i < n_seg; ++i) {
        p.seg[i] = {segs[i].m_begin, segs[i].m_end, tiles, segs[i].gate_row, segs[i].w.chunks};
        tiles += (segs[i].m_end - segs[i].m_begin + kTileTokens - 1) / kTileTokens * p.pair_panels;
    }
    p.n_tiles = tiles;
    if (!tiles) return cudaSuccess;
    p.ksplit = 1;
    p.kbu = p.kb;
    p.n_units = tiles;
    p.split_stride = 0;

    auto enc = encode_fn();
    if (!enc) return cudaErrorNotSupported;
    CUtensorMap xm;
    const cuuint64_t dims[2] = {k, m_total};
    const cuuint64_t strides[1] = {k * 2};
    const cuuint32_t box[2] = {64u, kHalf};
    const cuuint32_t estr[2] = {1u, 1u};
    const CUresult r = enc(&xm, stage_f16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2,
                           const_cast<uint16_t *>(x), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                           CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return cudaErrorInvalidValue;
    const int out_f32 = out_dtype == 0;
    YMaps ym;
    memset(&ym, 0, sizeof(ym));
    bool aligned = (reinterpret_cast<uintptr_t>(y) & 15u) == 0 && (ldy * 2) % 16 == 0;
    for (uint32_t d = 0; d < p.epi.n_peer; ++d) aligned &= (reinterpret_cast<uintptr_t>(p.epi.peer[d]) & 15u) == 0;
    if (!out_f32 && !(p.epi.flags & TC_EPI_GATE_RESIDUAL) && aligned) {
        // SwiGLU: Y has one column per gate / up row pair, and a warp's box is
        // its 16 outputs wide
        const bool glu = p.epi.flags & TC_EPI_SWIGLU;
        const cuuint64_t ydims[2] = {glu ? p.n / 2 : p.n, m_total};
        const cuuint64_t ystrides[1] = {ldy * 2};
        const cuuint32_t ybox[2] = {glu ? 16u : 32u, 32u};
        bool ok = true;
        for (uint32_t d = 0; d <= p.epi.n_peer && ok; ++d) {
            void *base = d == 0 ? y : p.epi.peer[d - 1];
            ok = enc(&ym.m[d], out_dtype == 1 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2,
                     base, ydims, ystrides, ybox, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                     CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
        }
        p.y_tma = ok ? 1u : 0u;
    } else if (out_f32 && !p.epi.flags && !p.epi.n_peer && (reinterpret_cast<uintptr_t>(y) & 15u) == 0 &&
               (ldy * 4) % 16 == 0) {
        p.y_tma = encode_f32_map(enc, &ym.m[0], y, p.n, m_total, ldy, 1, m_total * ldy) ? 1u : 0u;
    }
    if (split && split->ksplit > 1) {
        if (!split->ws || p.kb % split->ksplit) return cudaErrorInvalidValue;
        return launch_pair_split(xm, ym, p, segs, n_seg, *split, y, ldy, out_dtype, stage_f16, m_total, sm_count, s);
    }
    const uint32_t type = segs[0].w.type;
    if (type == 12) {
        if (stage_f16) return out_f32 ? launch_pair_inst<12, true, true>(xm, ym, p, sm_count, s) : launch_pair_inst<12, true, false>(xm, ym, p, sm_count, s);
        return out_f32 ? launch_pair_inst<12, false, true>(xm, ym, p, sm_count, s) : launch_pair_inst<12, false, false>(xm, ym, p, sm_count, s);
    }
    if (type == 13) {
        if (stage_f16) return out_f32 ? launch_pair_inst<13, true, true>(xm, ym, p, sm_count, s) : launch_pair_inst<13, true, false>(xm, ym, p, sm_count, s);
        return out_f32 ? launch_pair_inst<13, false, true>(xm, ym, p, sm_count, s) : launch_pair_inst<13, false, false>(xm, ym, p, sm_count, s);
    }
    if (stage_f16) return out_f32 ? launch_pair_inst<14, true, true>(xm, ym, p, sm_count, s) : launch_pair_inst<14, true, false>(xm, ym, p, sm_count, s);
    return out_f32 ? launch_pair_inst<14, false, true>(xm, ym, p, sm_count, s) : launch_pair_inst<14, false, false>(xm, ym, p, sm_count, s);
}

namespace {
// Split-K launch: the units store fp32 partials (plain stores, no epilogue,
// no peers) into sk.ws; one reduce per segment adds them in split order and
// writes Y (with the call's epilogue and peer replicas).
cudaError_t launch_pair_split(const CUtensorMap &xm, const YMaps &ym, PairParams p, const SegmentView *segs,
                              uint32_t n_seg, const SplitK &sk, void *y, uint64_t ldy, int out_dtype, int stage_f16,
                              uint64_t m_total, int sm_count, cudaStream_t s) {
    const EpiView epi = p.epi;
    p.ksplit = sk.ksplit;
    p.kbu = p.kb / sk.ksplit;
    p.n_units = p.n_tiles * sk.ksplit;
    p.split_stride = m_total * p.n;
    p.y = sk.ws;
    p.ldy = p.n;
    p.epi = EpiView{};
    p.epi.y_limit = (uint64_t)sk.ksplit * p.split_stride;
    p.epi.status = p.status;
    YMaps pm;
    memset(&pm, 0, sizeof(pm));
    p.y_tma = encode_f32_map(encode_fn(), &pm.m[0], sk.ws, p.n, m_total, p.n, sk.ksplit, p.split_stride) ? 1u : 0u;
    cudaError_t e;
    const uint32_t type = segs[0].w.type;
    if (type == 12) e = stage_f16 ? launch_pair_inst<12, true, true>(xm, pm, p, sm_count, s)
                                  : launch_pair_inst<12, false, true>(xm, pm, p, sm_count, s);
    else if (type == 13) e = stage_f16 ? launch_pair_inst<13, true, true>(xm, pm, p, sm_count, s)
                                       : launch_pair_inst<13, false, true>(xm, pm, p, sm_count, s);
    else e = stage_f16 ? launch_pair_inst<14, true, true>(xm, pm, p, sm_count, s)
                       : launch_pair_inst<14, false, true>(xm, pm, p, sm_count, s);
    for (uint32_t i = 0; i < n_seg && e == cudaSuccess; ++i)
        e = launch_split_reduce(sk.ws, sk.ksplit, p.split_stride, p.n, segs[i].m_begin, segs[i].m_end - segs[i].m_begin,
                                epi, segs[i].gate_row, y, ldy, out_dtype, s);
    return e;
}
}  // namespace

}  // namespace tc
