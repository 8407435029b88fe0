// Small-M quantised GEMV (M <= 16 rows of X: timestep / AdaLN-modulation
// linears): Y[m, n] = sum_k X[m, k] * W[n, k].  HBM-bound on the packed
// weight: at 6.5 TB/s an SM must retire ~28 weights per clock, which leaves
// no room for an fp32 dequantise-and-FMA per weight per token.  So the
// weights stay in code space:
//
//   * each K16 step of mma.sync.m16n8k16 (bf16 in, fp32 accumulate) takes the
//     raw 4-/6-bit codes of 16 weight rows as bf16 -- exact: a prmt places
//     each code byte under the exponent of 128 (0x43cc = 128 + c); the 128
//     leaves through sum_k x_k of the group (one more MMA with an all-ones A
//     on the same B fragment), or, for Q6_K, a bf16x2 subtract makes A =
//     q - 32 exactly (the per-shape choice is q6_centred below);
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
// Work split: CTA (x, y) = (one row tile, one K slice), 4 warps, stages
// filled by per-lane cp.async copies; two tile shapes (gemv_row_warps):
//   * several tokens: 64 weight rows, warp w owning rows 16 w .. 16 w + 15.
//     The four warps walk the same super-blocks of the slice in step through
//     one ring of stages (3; 2 with 8 tokens per tile): a stage holds the
//     four warps' packed fields and the super-block's 256 columns of X for
//     every token, copied once per CTA and read by the MMA steps from shared
//     memory; one __syncthreads per super-block publishes the stage and frees
//     the slot computed before it.  (With 16 rows per CTA and X fragments
//     loaded from global memory, X -- 16 tokens x the K slice -- came from L2
//     for every 16 weight rows, 75 MB per config-2 call against 31 MB of
//     weights, and the kernel stalled on those loads.)
//   * one token: 16 weight rows; the warps take interleaved super-blocks of
//     the slice, each through its own ring (W piece + the token's 512 B of
//     X), and their sums meet in shared memory.
// Hundreds of short CTAs keep every SM's loads in flight (the K split sizes
// the grid, not the SM count).  With several K slices each row warp stores
// its 16 x M partial in the workspace, and the last CTA of the tile to
// finish (per-tile arrival counter) adds the slices in slice order -- a fixed
// order, so results are deterministic -- writes Y and resets the counter.
// The N8 side of the MMA carries the tokens: NT = 1 or 2 tiles of 8.
// Launches use programmatic dependent launch: weight prefetch overlaps the
// tail of the previous kernel in the stream; X, the workspace and Y are
// touched only after griddepcontrol.wait.
#include "kq_epilogue.cuh"
#include "kq_format.cuh"
#include "tc_internal.h"

namespace tc {
namespace {

constexpr int kWarps = 4;
// Row pitch (floats) of a warp's scale table [16 rows][16]: 20, so that the
// eight row pairs a warp reads at once (rows g, g + 8) fall in distinct banks
// (with 16 every second row shares a bank: four-way conflicts).
constexpr uint32_t kTabPitch = 20;
// Q6_K codes as q - 32 (an exact bf16 subtract per pair) or as 128 + q with
// the offset removed per group through an extra all-ones MMA per step.
// Measured on config 2 (us per call, M = 1 / 8 / 16): centred 9.33 / 12.46 /
// 13.95, offset 9.68 / 11.02 / 15.12 -- the offset form only for one tile of
// 8 tokens.
template <int TP, int NT> constexpr bool q6_centred() { return !(TP == 8 && NT == 1); }

// Two code bytes (selector 0x4140: bytes 0,1; 0x4342: bytes 2,3) as the bf16
// pair (128 + c0, 128 + c1): each byte lands under the exponent of 128.
__device__ __forceinline__ uint32_t code_pair(uint32_t codes, uint32_t sel) {
    uint32_t r;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(codes), "r"(0x43434343u), "r"(sel));
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

// ---------------------------------------------------------------- staging
// A warp's piece of a stage: the packed fields of its 16 weight rows for one
// super-block (contiguous pieces of the panel chunk).
//   Q4_K: qs [4][16 rows][32] | sc [16][12] | dm [16][4]              = 2304 B
//   Q6_K: ql [4 = h*2+part][16][32] | qh [2][16][32] | sc [16][16] | d [16][2] = 3360 B
// Row r of a piece is at row_slot(r0 + r) - r0.
template <int TYPE> struct StageGeo;
template <> struct StageGeo<12> {
    static constexpr uint32_t w_bytes = 2304, qs = 0, sc = 2048, dm = 2240;
};
//   Q5_K: qs [4][16][32] | qh [16][32] | sc [16][12] | dm [16][4]     = 2816 B
template <> struct StageGeo<13> {
    static constexpr uint32_t w_bytes = 2816, qs = 0, qh = 2048, sc = 2560, dm = 2752;
};
template <> struct StageGeo<14> {
    static constexpr uint32_t w_bytes = 3360, ql = 0, qh = 2048, sc = 3072, d = 3328;
};

__device__ __forceinline__ uint32_t s_u32(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }
// Per-lane asynchronous copies (cp.async, 16 bytes per lane per copy, L2
// only): the 32 lanes of a warp move a 512-byte piece with one instruction
// each.  A stage is one commit group; cp.async.wait_group + __syncwarp make
// it visible to the whole warp.  Unlike bulk copies these do not queue on
// the SM's single TMA unit, which at the start of a short launch holds
// hundreds of small requests (every warp's ring of stages) and delays the
// first arrivals.
__device__ __forceinline__ void cpa16(uint32_t dst, const void *src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cpa_piece(uint32_t dst, const uint8_t *src, uint32_t bytes, uint32_t lane) {
    for (uint32_t o = lane * 16; o < bytes; o += 512) cpa16(dst + o, src + o);
}
__device__ __forceinline__ void cpa_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cpa_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// All lanes of a warp: copy the packed fields of the warp's 16 rows of one
// super-block (panel chunk `chunk`, rows r0..r0+15) into stage buffer st.
template <int TYPE>
__device__ __forceinline__ void issue_w(uint8_t *st, const uint8_t *chunk, uint32_t r0, uint32_t lane) {
    using SG = StageGeo<TYPE>;
    const uint32_t d = s_u32(st);
    if constexpr (TYPE == 12) {
#pragma unroll
        for (uint32_t q = 0; q < 4; ++q) cpa_piece(d + SG::qs + q * 512, chunk + kQ4Qs + q * 4096 + r0 * 32, 512, lane);
        cpa_piece(d + SG::sc, chunk + kQ4Sc + r0 * 12, 192, lane);
        cpa_piece(d + SG::dm, chunk + kQ4Dm + r0 * 4, 64, lane);
    } else if constexpr (TYPE == 13) {
#pragma unroll
        for (uint32_t q = 0; q < 4; ++q) cpa_piece(d + SG::qs + q * 512, chunk + kQ5Qs + q * 4096 + r0 * 32, 512, lane);
        cpa_piece(d + SG::qh, chunk + kQ5Qh + r0 * 32, 512, lane);
        cpa_piece(d + SG::sc, chunk + kQ5Sc + r0 * 12, 192, lane);
        cpa_piece(d + SG::dm, chunk + kQ5Dm + r0 * 4, 64, lane);
    } else {
#pragma unroll
        for (uint32_t hp = 0; hp < 4; ++hp)
            cpa_piece(d + SG::ql + hp * 512, chunk + kQ6Ql + (hp * kPanelRows + r0) * 32, 512, lane);
#pragma unroll
        for (uint32_t h = 0; h < 2; ++h)
            cpa_piece(d + SG::qh + h * 512, chunk + kQ6Qh + (h * kPanelRows + r0) * 32, 512, lane);
        cpa_piece(d + SG::sc, chunk + kQ6Sc + r0 * 16, 256, lane);
        cpa_piece(d + SG::d, chunk + kQ6D + r0 * 2, 32, lane);
    }
}
// Programmatic dependent launch: let the next kernel in the stream start its
// prologue, and wait for the previous one before touching its outputs.
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// Tile arrival counter: atomic add with acquire-release semantics at GPU scope.
__device__ __forceinline__ uint32_t arrive_acq_rel(uint32_t *counter) {
    uint32_t old;
    asm volatile("atom.add.acq_rel.gpu.u32 %0, [%1], 1;" : "=r"(old) : "l"(counter) : "memory");
    return old;
}

__device__ __forceinline__ uint32_t lds32(const uint8_t *p) { return *reinterpret_cast<const uint32_t *>(p); }

// Four bytes of a word as exact small-integer floats (byte = 0..255):
// prmt under the exponent of 2^23, then subtract 2^23.
__device__ __forceinline__ void bytes_to_float4(uint32_t w, float (&f)[4]) {
#pragma unroll
    for (uint32_t i = 0; i < 4; ++i) {
        uint32_t r;
        asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(w), "r"(0x4B000000u), "r"(0x7440u | i));
        f[i] = __uint_as_float(r) - 8388608.0f;
    }
}

// Q6_K codes as exact signed bf16 pairs (q0 - 32, q1 - 32): the 128 + q of
// code_pair minus 160, one bf16x2 subtract whose result (-32..31) is exact.
__device__ __forceinline__ uint32_t centred_pair(uint32_t codes, uint32_t sel) {
    uint32_t r;
    asm("sub.rn.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(code_pair(codes, sel)), "r"(0x43204320u));
    return r;
}

// Columns of the MMA's N8 side: with TP tokens per tile (1, 2, 4 or 8),
// column n carries token n % TP of the n / TP-th scale group of the current
// chain, so a chain of S = 8 / TP scale groups accumulates unscaled in one
// fp32 fragment; the B fragment of a K16 step is non-zero only in the columns
// of that step's group.  The A operand is the bf16 value 128 + code (no
// subtract) for Q4_K: the chain also accumulates sum_k x_k per column with an
// all-ones A (C1), and the group's result is d*sc * (C - 128 C1) - dmin*m C1.
// Q6_K has no per-group min, so its A is the centred code q - 32 itself
// (centred_pair) and the group's result is d*sc * C: one MMA per step.
//
// Visit order of the scale groups (v = 0..GROUPS-1) follows the packed words:
//   Q4_K: v = sub-block (quarter v/2, nibble v&1), two K16 steps each;
//   Q6_K: v = 8h + 4jj + grp -> 16-weight group 8h + 2grp + jj, one step each.
template <int TYPE>
__device__ __forceinline__ constexpr uint32_t group_of_visit(uint32_t v) {
    return TYPE != 14 ? v : 8 * (v >> 3) + 2 * (v & 3) + ((v >> 2) & 1);
}

// B operand: in the K16 step of scale-group visit v the MMA column slot is
// j = v % S, and only the quad whose token column g / TP equals j supplies X
// (every other thread supplies zeros).  So a thread needs X on 2 TP of the 16
// steps of a super-block -- its "own" steps, visits v = g / TP + S c -- and
// keeps just those fragments; on every step it supplies own[c] * bmask[j]
// with bmask[j] = 1 for its own slot and 0 otherwise (an integer multiply:
// exact, and off the integer / logic pipe that unpacks the codes).
//   Q6_K:        own step c = visit my_j + S c (one K16 step per visit);
//   Q4_K / Q5_K: own step c = sub-block my_j + S (c / 2), K16 half c % 2.
// With one token the fragments come from the stage in shared memory; with
// several from global memory (L1 / L2), loaded one super-block ahead of their
// use (one token tile) so that the load latency overlaps the previous
// super-block's arithmetic.
template <int TYPE, int TP>
__device__ __forceinline__ uint32_t own_col(uint32_t c, uint32_t my_j, uint32_t t) {
    constexpr uint32_t S = 8 / TP;
    if constexpr (TYPE == 14) {
        const uint32_t v = my_j + S * c;
        return 128 * (v >> 3) + 32 * (v & 3) + 16 * ((v >> 2) & 1) + 4 * t;
    } else {
        return 32 * (my_j + S * (c >> 1)) + 8 * t + 4 * (c & 1);
    }
}
// X in the stage: TP * NT token rows of one super-block's 256 columns (one
// row for TP = 1), rows clamped to the last real token.  With several rows the
// row pitch is 544 bytes: the lanes of a quad group (g = 0..7) read rows
// 8 g apart in banks, so the 16 lanes of one 64-bit phase hit 32 distinct
// banks.
template <int TP, int NT> struct XGeo {
    static constexpr uint32_t rows = TP == 1 ? 1u : (uint32_t)(TP * NT);
    static constexpr uint32_t pitch = TP == 1 ? 512u : 544u;
    static constexpr uint32_t bytes = rows * pitch;
};
__device__ __forceinline__ uint2 lds64(const uint8_t *p) { return *reinterpret_cast<const uint2 *>(p); }
// One super-block of the warp's 16 rows (packed fields at st) against the
// stage's X rows (xs): the scale table first, then the K16 steps.
template <int TYPE, int TP, int NT>
__device__ __forceinline__ void compute_stage(const uint8_t *st, const uint8_t *xs, uint32_t g, uint32_t t,
                                              uint32_t lane, const uint32_t (&bmask)[8 / TP], float *wt,
                                              float (&acc)[NT][4]) {
    using SG = StageGeo<TYPE>;
    constexpr uint32_t S = 8 / TP;
    const uint32_t rg = row_slot(g), rg8 = row_slot(g + 8);   // slots inside the 16-row piece
    const uint32_t half = lane & 1, rr = lane >> 1;
    // Scale table, written by all lanes: row rr, half `half` of its groups.
    //   Q4_K: float2 (d*sc_g, dmin*m_g) [16][8];  Q6_K: float d*sc_i [16][16].
    {
    __syncwarp();
    if constexpr (TYPE != 14) {
        const uint32_t dm = lds32(st + SG::dm + rr * 4);
        const float d = half_bits_to_float((uint16_t)(dm & 0xffffu)), dmin = half_bits_to_float((uint16_t)(dm >> 16));
        const uint32_t w0 = lds32(st + SG::sc + rr * 12), w1 = lds32(st + SG::sc + rr * 12 + 4),
                       w2 = lds32(st + SG::sc + rr * 12 + 8);
        // byte lanes: sc0..3 = w0 & 63, m0..3 = w1 & 63,
        // sc4..7 = (w2 & 15) | (w0 >> 6) << 4, m4..7 = (w2 >> 4) | (w1 >> 6) << 4
        const uint32_t scw = half ? ((w2 & 0x0F0F0F0Fu) | ((w0 >> 2) & 0x30303030u)) : (w0 & 0x3F3F3F3Fu);
        const uint32_t mnw = half ? (((w2 >> 4) & 0x0F0F0F0Fu) | ((w1 >> 2) & 0x30303030u)) : (w1 & 0x3F3F3F3Fu);
        float scf[4], mnf[4];
        bytes_to_float4(scw, scf);
        bytes_to_float4(mnw, mnf);
        float4 *o = reinterpret_cast<float4 *>(wt + rr * kTabPitch + half * 8);
        o[0] = make_float4(d * scf[0], dmin * mnf[0], d * scf[1], dmin * mnf[1]);
        o[1] = make_float4(d * scf[2], dmin * mnf[2], d * scf[3], dmin * mnf[3]);
    } else {
        const float d = half_bits_to_float(*reinterpret_cast<const uint16_t *>(st + SG::d + rr * 2));
        const uint2 sw = *reinterpret_cast<const uint2 *>(st + SG::sc + rr * 16 + 8 * half);
        float a[4], b[4];
        bytes_to_float4(sw.x ^ 0x80808080u, a);   // int8 + 128 as unsigned bytes
        bytes_to_float4(sw.y ^ 0x80808080u, b);
        float4 *o = reinterpret_cast<float4 *>(wt + rr * kTabPitch + half * 8);
        o[0] = make_float4(d * (a[0] - 128.f), d * (a[1] - 128.f), d * (a[2] - 128.f), d * (a[3] - 128.f));
        o[1] = make_float4(d * (b[0] - 128.f), d * (b[1] - 128.f), d * (b[2] - 128.f), d * (b[3] - 128.f));
    }
    __syncwarp();
    }
    const uint32_t my_j = g / TP;
    // the X rows of this thread's tokens (8 nt + g % TP) in the stage
    const uint8_t *xrow[NT];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) xrow[nt] = xs + (8 * nt + g % TP) * XGeo<TP, NT>::pitch;
    const uint32_t ones = 0x3F803F80u;
    constexpr float off = 128.f;    // Q4_K: the code-space offset of code_pair
    constexpr float off6 = 160.f;   // Q6_K: that offset plus the code bias 32
    // A = 128 + code (one prmt per pair), the offset removed per group
    // through sum_k x_k from an all-ones MMA; or, for Q6_K where
    // q6_centred, A = code - 32 exactly (a bf16x2 subtract per pair, no
    // second MMA).
    constexpr bool kOffsetA = TYPE != 14 || !q6_centred<TP, NT>();
    float cq[NT][4], c1[NT][4];

    // One K16 step of scale group visit v: A from code words (rows g, g+8).
    // c = this step's own-step index (see own_col)
    auto step = [&](uint32_t v, uint32_t c, uint32_t cg, uint32_t cg8, bool chain_start) {
        const uint32_t j = v % S;
        if (chain_start) {
#pragma unroll
            for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                for (int i = 0; i < 4; ++i) cq[nt][i] = c1[nt][i] = 0.f;
        }
        uint32_t a0, a1, a2, a3;
        if constexpr (kOffsetA) {
            a0 = code_pair(cg, 0x4140u); a1 = code_pair(cg8, 0x4140u);
            a2 = code_pair(cg, 0x4342u); a3 = code_pair(cg8, 0x4342u);
        } else {
            a0 = centred_pair(cg, 0x4140u); a1 = centred_pair(cg8, 0x4140u);
            a2 = centred_pair(cg, 0x4342u); a3 = centred_pair(cg8, 0x4342u);
        }
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
            const uint2 xv = lds64(xrow[nt] + 2 * own_col<TYPE, TP>(c, my_j, t));
            const uint32_t b0 = xv.x * bmask[j], b1 = xv.y * bmask[j];
            mma16816(cq[nt], a0, a1, a2, a3, b0, b1, cq[nt]);
            if constexpr (kOffsetA) mma16816(c1[nt], ones, ones, ones, ones, b0, b1, c1[nt]);
        }
    };
    // Scale the finished chain `chain` into the accumulators.
    auto close_chain = [&](uint32_t chain) {
#pragma unroll
        for (uint32_t ci = 0; ci < 2; ++ci) {
            const uint32_t G = group_of_visit<TYPE>(chain * S + (2 * t + ci) / TP);
            if constexpr (TYPE != 14) {
                const float2 a = reinterpret_cast<const float2 *>(wt + g * kTabPitch)[G];
                const float2 b = reinterpret_cast<const float2 *>(wt + (g + 8) * kTabPitch)[G];
#pragma unroll
                for (int nt = 0; nt < NT; ++nt) {
                    acc[nt][ci] = fmaf(a.x, fmaf(-off, c1[nt][ci], cq[nt][ci]), fmaf(-a.y, c1[nt][ci], acc[nt][ci]));
                    acc[nt][2 + ci] = fmaf(b.x, fmaf(-off, c1[nt][2 + ci], cq[nt][2 + ci]),
                                           fmaf(-b.y, c1[nt][2 + ci], acc[nt][2 + ci]));
                }
            } else {
                const float a = wt[g * kTabPitch + G], b = wt[(g + 8) * kTabPitch + G];
#pragma unroll
                for (int nt = 0; nt < NT; ++nt) {
                    if constexpr (kOffsetA) {   // sum x (128 + q) - 160 sum x = sum x (q - 32)
                        acc[nt][ci] = fmaf(a, fmaf(-off6, c1[nt][ci], cq[nt][ci]), acc[nt][ci]);
                        acc[nt][2 + ci] = fmaf(b, fmaf(-off6, c1[nt][2 + ci], cq[nt][2 + ci]), acc[nt][2 + ci]);
                    } else {
                        acc[nt][ci] = fmaf(a, cq[nt][ci], acc[nt][ci]);
                        acc[nt][2 + ci] = fmaf(b, cq[nt][2 + ci], acc[nt][2 + ci]);
                    }
                }
            }
        }
    };

    if constexpr (TYPE != 14) {
        // Q5_K: the fifth bit of code j of sub-block v is bit v of qh[j]
        uint2 hq = make_uint2(0u, 0u), hq8 = make_uint2(0u, 0u);
        if constexpr (TYPE == 13) {
            hq = *reinterpret_cast<const uint2 *>(st + StageGeo<13>::qh + rg * 32 + 8 * t);
            hq8 = *reinterpret_cast<const uint2 *>(st + StageGeo<13>::qh + rg8 * 32 + 8 * t);
        }
#pragma unroll
        for (uint32_t q = 0; q < 4; ++q) {
            const uint2 wg = *reinterpret_cast<const uint2 *>(st + SG::qs + q * 512 + rg * 32 + 8 * t);
            const uint2 wg8 = *reinterpret_cast<const uint2 *>(st + SG::qs + q * 512 + rg8 * 32 + 8 * t);
#pragma unroll
            for (uint32_t nib = 0; nib < 2; ++nib) {
                const uint32_t v = 2 * q + nib;
#pragma unroll
                for (uint32_t sp = 0; sp < 2; ++sp) {
                    const uint32_t w = sp ? wg.y : wg.x, w8 = sp ? wg8.y : wg8.x;
                    uint32_t c = (w >> (4 * nib)) & 0x0F0F0F0Fu, c8 = (w8 >> (4 * nib)) & 0x0F0F0F0Fu;
                    if constexpr (TYPE == 13) {
                        c |= (((sp ? hq.y : hq.x) >> v) & 0x01010101u) << 4;
                        c8 |= (((sp ? hq8.y : hq8.x) >> v) & 0x01010101u) << 4;
                    }
                    step(v, 2 * (v / S) + sp, c, c8, sp == 0 && v % S == 0);
                }
                if (v % S == S - 1) close_chain(v / S);
            }
        }
    } else {
#pragma unroll
        for (uint32_t h = 0; h < 2; ++h) {
#pragma unroll
            for (uint32_t jj = 0; jj < 2; ++jj) {
                const uint32_t o0 = SG::ql + (h * 2) * 512 + 16 * jj + 4 * t;
                const uint32_t o1 = o0 + 512, oh = SG::qh + h * 512 + 16 * jj + 4 * t;
                const uint32_t l0 = lds32(st + o0 + rg * 32), l1 = lds32(st + o1 + rg * 32), hq = lds32(st + oh + rg * 32);
                const uint32_t l08 = lds32(st + o0 + rg8 * 32), l18 = lds32(st + o1 + rg8 * 32),
                               hq8 = lds32(st + oh + rg8 * 32);
                // high-bit planes for groups 0..3, already at bits 4..5 of each byte
                const uint32_t hb[4] = {(hq << 4) & 0x30303030u, (hq << 2) & 0x30303030u, hq & 0x30303030u,
                                        (hq >> 2) & 0x30303030u};
                const uint32_t hb8[4] = {(hq8 << 4) & 0x30303030u, (hq8 << 2) & 0x30303030u, hq8 & 0x30303030u,
                                         (hq8 >> 2) & 0x30303030u};
                const uint32_t lw[4] = {l0, l1, l0 >> 4, l1 >> 4}, lw8[4] = {l08, l18, l08 >> 4, l18 >> 4};
#pragma unroll
                for (uint32_t grp = 0; grp < 4; ++grp) {
                    const uint32_t v = 8 * h + 4 * jj + grp;
                    step(v, v / S, (lw[grp] & 0x0F0F0F0Fu) | hb[grp], (lw8[grp] & 0x0F0F0F0Fu) | hb8[grp],
                         v % S == 0);
                    if (v % S == S - 1) close_chain(v / S);
                }
            }
        }
    }
}

// Row warps of a CTA (RW; the other 4 / RW split K inside the CTA):
//   1 (one token): 16 rows; warp w takes super-blocks kb_begin + w + 4 i of
//     the slice through its own stage ring (its W piece and the token's 512
//     bytes of X), and the four sums meet in shared memory.  X is small next
//     to W, and independent warps hide each other's load latency; the K
//     split inside the CTA spares three quarters of the global fix-up.
//   4 (several tokens): 64 rows, warp w owning rows 16 w .. 16 w + 15; one
//     stage ring for the CTA holds the four W pieces and the super-block's X
//     for every token, copied once and read by all four warps.
template <int TP> constexpr uint32_t gemv_row_warps() { return TP == 1 ? 1u : 4u; }
// Depth of the stage rings: 3 stages, except with 8 tokens per tile (M > 4),
// where the stage's X (8 or 16 rows) leaves room for four resident CTAs only
// with 2 (measured at M = 8: 3 stages, three CTAs per SM, 15.3 us per call).
template <int TP>
constexpr uint32_t gemv_stages() { return TP == 8 ? 2u : 3u; }
// Bytes of one stage: per warp (RW = 1) or per CTA (RW = 4).
template <int TYPE, int TP, int NT>
constexpr uint32_t gemv_stage_bytes() {
    return (gemv_row_warps<TP>() * StageGeo<TYPE>::w_bytes + XGeo<TP, NT>::bytes + 127) / 128 * 128;
}
template <int TYPE, int TP, int NT>
constexpr uint32_t gemv_smem_bytes() {
    return gemv_stage_bytes<TYPE, TP, NT>() * gemv_stages<TP>() * (kWarps / gemv_row_warps<TP>());
}

// Weights of one launch: blockIdx.x runs over the 16 RW-row tiles of all of
// them (entry e owns tiles [tile_begin, next entry's tile_begin)), blockIdx.y
// over the K slices of kb_per_slice super-blocks; they share K, type and X,
// each has its own Y.
template <int TYPE, int TP, int NT, int DT>
__global__ void __launch_bounds__(kWarps * 32, 4) gemv_kernel(const __grid_constant__ GemvBatch b,
                                                           const uint16_t *__restrict__ x, uint32_t m_begin,
                                                           uint32_t m_count, uint64_t k, uint32_t kb_per_slice,
                                                           float *__restrict__ partials,
                                                           uint32_t *__restrict__ counters, uint32_t *status) {
    using SG = StageGeo<TYPE>;
    using XG = XGeo<TP, NT>;
    constexpr uint32_t chunk = chunk_bytes(TYPE);
    constexpr uint32_t RW = gemv_row_warps<TP>(), KW = kWarps / RW;
    constexpr uint32_t kStages = gemv_stages<TP>(), stage_bytes = gemv_stage_bytes<TYPE, TP, NT>();
    constexpr uint32_t w_all = RW * SG::w_bytes;   // X follows the stage's W pieces
    extern __shared__ __align__(128) uint8_t dyn[];
    __shared__ __align__(16) float tab[kWarps][16 * kTabPitch];
    __shared__ uint32_t last;
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
    const uint32_t rw = warp % RW, kw = warp / RW;
    const uint32_t kb = b.kb, tile = blockIdx.x, n_slices = gridDim.y;
    const uint32_t kb_begin = blockIdx.y * kb_per_slice, kb_end = min(kb, kb_begin + kb_per_slice);
    uint32_t ei = 0;
    while (ei + 1 < b.n_entries && tile >= b.e[ei + 1].tile_begin) ++ei;
    const GemvEntry &w = b.e[ei];
    const uint32_t row0 = (tile - w.tile_begin) * (16 * RW) + rw * 16;
    // rows past n up to the panel end are zero blocks (read, never stored)
    const uint32_t panel =
        tc_in_bounds(row0 / kPanelRows < (w.n + kPanelRows - 1) / kPanelRows, status) ? row0 / kPanelRows : 0;
    const uint8_t *pbase = w.chunks + (uint64_t)panel * kb * chunk;
    const uint32_t r0 = row0 % kPanelRows;
    float *wt = tab[warp];

    // This warp's super-blocks: kb_begin + kw + KW i (RW = 1: its own; RW = 4:
    // every warp the same).  Stage i of the warp's ring (RW = 1) or the CTA's
    // (RW = 4) is slot i % kStages: the W pieces, then the X rows.
    const uint32_t first = kb_begin + kw;
    const uint32_t count = first < kb_end ? (kb_end - first + KW - 1) / KW : 0;
    uint8_t *const ring = dyn + (size_t)kw * kStages * stage_bytes;
    auto slot = [&](uint32_t i) { return ring + (i % kStages) * stage_bytes; };
    auto issue_w_stage = [&](uint32_t i) {
        issue_w<TYPE>(slot(i) + rw * SG::w_bytes, pbase + (uint64_t)(first + KW * i) * chunk, r0, lane);
    };
    // X rows of stage i: by the warp itself (RW = 1) or shared by the CTA.
    auto issue_x = [&](uint32_t i) {
        const uint32_t d = s_u32(slot(i) + w_all), kbx = first + KW * i;
        const uint32_t me = RW == 1 ? lane : threadIdx.x, step = RW == 1 ? 32u : kWarps * 32u;
        for (uint32_t q = me; q < XG::rows * 32; q += step) {
            const uint32_t r = q / 32, c16 = q % 32;
            const uint64_t tok = m_begin + min(r, m_count - 1);
            cpa16(d + r * XG::pitch + c16 * 16, x + tok * k + (uint64_t)kbx * 256 + c16 * 8);
        }
    };
    // Each thread commits its copies of a stage as one group; the W of the
    // first kStages - 1 stages is issued before the wait on the previous
    // kernel (it does not depend on it), their X after it, as groups of their
    // own, so that before computing stage i at most kStages - 2 of this
    // thread's groups -- once stage i + kStages - 1 is committed, kStages - 1
    // -- may still be in flight.
#pragma unroll
    for (uint32_t i = 0; i < kStages - 1; ++i) {
        if (i < count) issue_w_stage(i);
        cpa_commit();
    }
    if (threadIdx.x == 0) pdl_launch_dependents();
    pdl_wait();
#pragma unroll
    for (uint32_t i = 0; i < kStages - 1; ++i) {
        if (i < count) issue_x(i);
        cpa_commit();
    }
    float acc[NT][4];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int i = 0; i < 4; ++i) acc[nt][i] = 0.f;
    uint32_t bmask[8 / TP];
#pragma unroll
    for (uint32_t j = 0; j < 8 / TP; ++j) bmask[j] = g / TP == j ? 1u : 0u;
    for (uint32_t i = 0; i < count; ++i) {
        if constexpr (RW == 1) {
            // The warp's own ring: refill the slot computed in the previous
            // iteration (every lane is past it: __syncwarp below), then wait
            // for stage i.
            if (i + kStages - 1 < count) {
                issue_w_stage(i + kStages - 1);
                issue_x(i + kStages - 1);
            }
            cpa_commit();
            cpa_wait<kStages - 1>();
            __syncwarp();
        } else {
            // The CTA's ring: stage i has landed for every thread, and every
            // warp is past stage i - 1, whose slot is refilled.
            cpa_wait<kStages - 2>();
            __syncthreads();
            if (i + kStages - 1 < count) {
                issue_w_stage(i + kStages - 1);
                issue_x(i + kStages - 1);
            }
            cpa_commit();
        }
        compute_stage<TYPE, TP, NT>(slot(i) + rw * SG::w_bytes, slot(i) + w_all, g, t, lane, bmask, wt, acc);
        if constexpr (RW == 1) __syncwarp();
    }

    // The warp's 16 x M result of the slice (rows g, g + 8 of its piece;
    // token 8 nt + column, written by the lanes whose column < TP).
    // Columns of one token are spread over the quad (TP < 8): sum them so
    // that every lane holds the full value of its (row, token) pairs.
    auto fold = [&](float (&v)[4 * NT]) {
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
            for (int i = 0; i < 4; ++i) v[4 * nt + i] = acc[nt][i];
        if constexpr (TP == 1) {   // all 8 columns are token 0: fold the thread's two columns
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
                v[4 * nt] += v[4 * nt + 1];
                v[4 * nt + 2] += v[4 * nt + 3];
            }
        }
        if constexpr (TP <= 2) {
#pragma unroll
            for (int j = 0; j < 4 * NT; ++j) {
                v[j] += __shfl_xor_sync(0xffffffffu, v[j], 1);
                v[j] += __shfl_xor_sync(0xffffffffu, v[j], 2);
            }
        } else if constexpr (TP == 4) {
#pragma unroll
            for (int j = 0; j < 4 * NT; ++j) v[j] += __shfl_xor_sync(0xffffffffu, v[j], 2);
        }
    };
    // Partial slot of (K slice, tile, row warp): 16 tokens x 16 rows of fp32.
    auto partial_slot = [&](uint32_t slice) {
        return partials + (((uint64_t)slice * gridDim.x + tile) * RW + rw) * 256;
    };
    auto publish = [&](const float (&v)[4 * NT]) {
        float *dst = partial_slot(blockIdx.y);
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const uint32_t col = 2 * t + (i & 1);
                if (col < TP) __stcg(dst + (8 * nt + col) * 16 + g + 8 * (i >> 1), v[4 * nt + i]);
            }
    };
    // Arrival of this CTA at its tile after publishing its partial; true in
    // the last CTA to arrive, with the tile's sum in v.  The barrier
    // orders every thread's partial before thread 0's release (acquire-release
    // arrival at GPU scope, cumulative over the barrier); in the CTA that
    // arrives last, the acquire and the second barrier order the other
    // participants' partials before its loads.
    auto arrive = [&](float (&v)[4 * NT]) -> bool {
        __syncthreads();
        if (threadIdx.x == 0) last = (arrive_acq_rel(counters + tile) + 1 == n_slices) ? 1u : 0u;
        __syncthreads();
        if (!last) return false;
#pragma unroll
        for (int j = 0; j < 4 * NT; ++j) v[j] = 0.f;
        // slices in order (deterministic), four slices' loads in flight
#pragma unroll 4
        for (uint32_t q = 0; q < (kw == 0 ? n_slices : 0u); ++q) {
            const float *src = partial_slot(q);
#pragma unroll
            for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const uint32_t col = 2 * t + (i & 1);
                    if (col < TP) v[4 * nt + i] += __ldcg(src + (8 * nt + col) * 16 + g + 8 * (i >> 1));
                }
        }
        if (threadIdx.x == 0) counters[tile] = 0u;
        return true;
    };
    // Y (with the fused epilogue) of the warp's rows of the finished tile.
    auto store_tile = [&](const float (&v)[4 * NT]) {
        void *const y = w.y;
        const uint64_t ldy = w.ldy;
        if (b.epi.flags) {
            // Fused epilogue.  A thread holds rows g and g + 8 of the piece
            // for the same token: for a SwiGLU weight the gate row and its up
            // row.
            const EpiView &e = b.epi;
            const bool glu = e.flags & TC_EPI_SWIGLU;
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const uint32_t col = 2 * t + (i & 1);
                    const uint32_t tok = 8 * nt + col % TP;
                    const uint32_t row = row0 + g + 8 * (i >> 1);
                    if (glu && i >= 2) continue;   // up rows are read with their gate row
                    if (col < TP && tok < m_count && row < w.n) {
                        const EpiRow er = epi_row(e, row, b.gate_row);
                        float val = v[4 * nt + i] + er.bias;
                        if (glu) val = silu(val) * (v[4 * nt + i + 2] + epi_row(e, row + 8, b.gate_row).bias);
                        else val = epi_act(e.flags, val);
                        const uint64_t m = m_begin + tok;
                        if (e.flags & TC_EPI_GATE_RESIDUAL)
                            val = load_out(e.res, m * e.ld_res + er.col, DT == 0, DT == 1) + er.gate * val;
                        store_out_all(e, y, m * ldy + er.col, val, DT == 0, DT == 1);
                    }
                }
            }
        } else {
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    // column 2t + (i & 1) carries token (column % TP); the lanes
                    // whose column < TP are the designated writers
                    const uint32_t col = 2 * t + (i & 1);
                    const uint32_t tok = 8 * nt + col % TP;
                    const uint32_t row = row0 + g + 8 * (i >> 1);
                    if (col < TP && tok < m_count && row < w.n) {
                        const uint64_t off = (uint64_t)(m_begin + tok) * ldy + row;
                        store_out_all(b.epi, y, off, v[4 * nt + i], DT == 0, DT == 1);
                    }
                }
            }
        }
    };

    float v[4 * NT];
    fold(v);
    if constexpr (KW > 1) {
        // the K-split warps of the same rows meet in shared memory; warp 0
        // adds them in warp order
        __shared__ float red[KW][32][4 * NT];
#pragma unroll
        for (int j = 0; j < 4 * NT; ++j) red[kw][lane][j] = v[j];
        __syncthreads();
        if (kw == 0) {
#pragma unroll
            for (int j = 0; j < 4 * NT; ++j) {
                float sum = red[0][lane][j];
#pragma unroll
                for (uint32_t q = 1; q < KW; ++q) sum += red[q][lane][j];
                v[j] = sum;
            }
        }
    }
    const bool owner = kw == 0;   // the warps that hold the rows' sums
    if (n_slices == 1) {
        if (owner) store_tile(v);
    } else {
        if (owner) publish(v);
        if (arrive(v) && owner) store_tile(v);
    }
    if (b.epi.n_peer) __threadfence_system();   // publish peer-replica stores
}

template <int TYPE, int TP, int NT>
cudaError_t launch_typed(const GemvBatch &bt_in, uint32_t m_begin, uint32_t mc, const uint16_t *x, uint64_t k,
                         int out_dtype, const GemvSplit &sp, cudaStream_t s) {
    constexpr uint32_t RW = gemv_row_warps<TP>();
    const size_t smem = gemv_smem_bytes<TYPE, TP, NT>();
    // tiles of 16 RW rows, numbered across the entries
    GemvBatch bt = bt_in;
    uint32_t tiles = 0;
    for (uint32_t i = 0; i < bt.n_entries; ++i) {
        bt.e[i].tile_begin = tiles;
        tiles += (bt.e[i].n + 16 * RW - 1) / (16 * RW);
    }
    if (!tiles) return cudaSuccess;
    auto kern = out_dtype == 0 ? gemv_kernel<TYPE, TP, NT, 0>
                : out_dtype == 1 ? gemv_kernel<TYPE, TP, NT, 1> : gemv_kernel<TYPE, TP, NT, 2>;
    // Opt in once per instantiation and device to its shared-memory size.
    static DeviceCache cache[3];
    int unused = 0;
    cudaError_t e = per_device(cache[out_dtype], unused, [&](int &) {
        return cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    });
    if (e != cudaSuccess) return e;
    const GemvSplit plan = gemv_split_tiles(tiles, bt.kb, RW);
    if (plan.n_slices > 1 && (!sp.partials || !sp.counters)) return cudaErrorInvalidValue;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(tiles, plan.n_slices);
    cfg.blockDim = dim3(kWarps * 32);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, bt, x, m_begin, mc, k, plan.kb_per_slice, sp.partials, sp.counters,
                              sp.status);
}

template <int TYPE>
cudaError_t launch_m(const GemvBatch &bt, uint32_t m_begin, uint32_t m, const uint16_t *x, uint64_t k,
                     int out_dtype, const GemvSplit &sp, cudaStream_t s) {
    if (m <= 1) return launch_typed<TYPE, 1, 1>(bt, m_begin, m, x, k, out_dtype, sp, s);
    if (m <= 2) return launch_typed<TYPE, 2, 1>(bt, m_begin, m, x, k, out_dtype, sp, s);
    if (m <= 4) return launch_typed<TYPE, 4, 1>(bt, m_begin, m, x, k, out_dtype, sp, s);
    if (m <= 8) return launch_typed<TYPE, 8, 1>(bt, m_begin, m, x, k, out_dtype, sp, s);
    return launch_typed<TYPE, 8, 2>(bt, m_begin, m, x, k, out_dtype, sp, s);
}

}  // namespace

GemvSplit gemv_split_tiles(uint32_t tiles, uint32_t kb, uint32_t row_warps) {
    // Enough CTAs to fill the resident slots of every SM -- three per SM
    // with the in-CTA K split of one token, four otherwise -- with as few K
    // slices as that allows (each slice costs a partial store and a share of
    // the fixup).  A slice keeps at least two super-blocks per warp, so that
    // the stage ring has something to overlap; with the in-CTA split its
    // super-blocks are a multiple of the four warps.  slices x tiles <
    // 2 kGemvMaxCtas, so the partials fit kGemvPartialFloats.
    const uint32_t kw = kWarps / row_warps;
    const uint32_t want = row_warps == 1 ? 148u * 3u : kGemvMaxCtas;
    uint32_t slices = tiles >= want ? 1u : (want + tiles - 1) / tiles;
    slices = std::max(1u, std::min(slices, kb / (2 * kw)));
    uint32_t per = (kb + slices - 1) / slices;
    per = (per + kw - 1) / kw * kw;
    GemvSplit sp;
    sp.kb_per_slice = per;
    sp.n_slices = (kb + per - 1) / per;
    return sp;
}

cudaError_t launch_gemv_batch(const GemvBatch &bt_in, uint32_t type, uint32_t m_begin, uint32_t m, const uint16_t *x,
                              uint64_t k, int out_dtype, const GemvSplit &sp, cudaStream_t s, const EpiView *epi,
                              uint32_t gate_row) {
    if (!m) return cudaSuccess;
    if (out_dtype < 0 || out_dtype > 2) return cudaErrorInvalidValue;
    GemvBatch bt = bt_in;
    bt.epi = epi ? *epi : EpiView{};
    bt.gate_row = gate_row;
    if (m > 16 || bt.n_entries == 0 || bt.n_entries > kMaxGemvBatch || !bt.kb) return cudaErrorInvalidValue;
    if (type == 12) return launch_m<12>(bt, m_begin, m, x, k, out_dtype, sp, s);
    if (type == 13) return launch_m<13>(bt, m_begin, m, x, k, out_dtype, sp, s);
    return launch_m<14>(bt, m_begin, m, x, k, out_dtype, sp, s);
}

cudaError_t launch_gemv(const SegmentView &seg, const uint16_t *x, uint64_t k, void *y, uint64_t ldy,
                        int out_dtype, const GemvSplit &sp, cudaStream_t s, const EpiView *epi) {
    if (seg.m_end <= seg.m_begin) return cudaSuccess;
    GemvBatch bt{};
    bt.n_entries = 1;
    bt.kb = seg.w.kb;
    bt.e[0] = {seg.w.chunks, y, ldy, seg.w.n, 0u};
    return launch_gemv_batch(bt, seg.w.type, seg.m_begin, seg.m_end - seg.m_begin, x, k, out_dtype, sp, s, epi,
                             seg.gate_row);
}

}  // namespace tc
