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
// Work split: CTA (x, y) = (16 weight rows, one K slice of 4 super-blocks),
// 4 warps each taking one super-block, so that thousands of short CTAs keep
// every SM's loads in flight (the CTA count is independent of the SM count).
// Each warp streams its super-blocks' packed fields through a ring of 3 (2
// with more than 8 tokens) stages of per-lane cp.async copies.  With one token (TP = 1) the stage also carries
// that token's 256 columns of X (512 B); with more tokens X is read straight
// from global memory instead (at most 16 rows x K, the same for every row
// tile, so it stays in L1 / L2), all of a super-block's X fragments at once:
// staging M rows per stage would shrink the number of resident CTAs as M
// grows (one CTA of 4 warps per SM at M = 16).  A CTA
// sums its warps through shared memory; with several K slices it stores the
// 16 x M partial in the context workspace, and the last CTA of the row tile to
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
// Per-warp stage in shared memory: the packed fields of 16 weight rows for one
// super-block (contiguous pieces of the panel chunk, one bulk copy each).
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
// All lanes: the single token's 256 columns of X for super-block kb (TP = 1).
template <int TYPE>
__device__ __forceinline__ void issue_x1(uint8_t *st, const uint16_t *x, uint64_t k, uint32_t m, uint32_t kb,
                                         uint32_t lane) {
    cpa_piece(s_u32(st) + StageGeo<TYPE>::w_bytes,
              reinterpret_cast<const uint8_t *>(x + (uint64_t)m * k + (uint64_t)kb * 256), 512, lane);
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
// N own steps' fragments (N = 2 TP: a whole super-block; 8: half of one).
template <int N, int NT> struct XFrags { uint2 v[N][NT]; };
template <int TYPE, int TP, int NT, int N>
__device__ __forceinline__ void load_x(XFrags<N, NT> &xs, const uint16_t *__restrict__ x, uint64_t k,
                                       uint32_t m_begin, uint32_t kb, uint32_t m_count, uint32_t g, uint32_t t,
                                       uint32_t c_begin) {
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
        const uint16_t *xr = x + (uint64_t)(m_begin + min(8 * nt + g % TP, m_count - 1)) * k + (uint64_t)kb * 256;
#pragma unroll
        for (uint32_t c = 0; c < (uint32_t)N; ++c)
            xs.v[c][nt] = __ldg(reinterpret_cast<const uint2 *>(xr + own_col<TYPE, TP>(c_begin + c, g / TP, t)));
    }
}

// Halves [H0, H1) of one super-block (weights 128 H0 .. 128 H1 - 1 of its
// rows); the scale table is built with half 0.  The own-step fragments in
// xs_global start at own step C0 (0, or 8 for a second-half call; halves are
// only computed separately with 8 tokens per tile, where every chain is
// within a half).
template <int TYPE, int TP, int NT, int N, uint32_t H0 = 0, uint32_t H1 = 2, uint32_t C0 = 0>
__device__ __forceinline__ void compute_stage(const uint8_t *st, const XFrags<N, NT> &xs_global, uint32_t g,
                                              uint32_t t, uint32_t lane, const uint32_t (&bmask)[8 / TP],
                                              float *wt, float (&acc)[NT][4]) {
    using SG = StageGeo<TYPE>;
    constexpr uint32_t S = 8 / TP;
    const uint32_t rg = row_slot(g), rg8 = row_slot(g + 8);   // slots inside the 16-row piece
    const uint32_t half = lane & 1, rr = lane >> 1;
    // Scale table, written by all lanes: row rr, half `half` of its groups.
    //   Q4_K: float2 (d*sc_g, dmin*m_g) [16][8];  Q6_K: float d*sc_i [16][16].
    if constexpr (H0 == 0) {
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
        float4 *o = reinterpret_cast<float4 *>(wt + rr * 16 + half * 8);
        o[0] = make_float4(d * scf[0], dmin * mnf[0], d * scf[1], dmin * mnf[1]);
        o[1] = make_float4(d * scf[2], dmin * mnf[2], d * scf[3], dmin * mnf[3]);
    } else {
        const float d = half_bits_to_float(*reinterpret_cast<const uint16_t *>(st + SG::d + rr * 2));
        const uint2 sw = *reinterpret_cast<const uint2 *>(st + SG::sc + rr * 16 + 8 * half);
        float a[4], b[4];
        bytes_to_float4(sw.x ^ 0x80808080u, a);   // int8 + 128 as unsigned bytes
        bytes_to_float4(sw.y ^ 0x80808080u, b);
        float4 *o = reinterpret_cast<float4 *>(wt + rr * 16 + half * 8);
        o[0] = make_float4(d * (a[0] - 128.f), d * (a[1] - 128.f), d * (a[2] - 128.f), d * (a[3] - 128.f));
        o[1] = make_float4(d * (b[0] - 128.f), d * (b[1] - 128.f), d * (b[2] - 128.f), d * (b[3] - 128.f));
    }
    __syncwarp();
    }
    const uint32_t my_j = g / TP;
    // one token: its 256 columns of X are part of the stage; read the own steps'
    XFrags<N, NT> xs_stage;
    if constexpr (TP == 1) {
        const uint16_t *x1 = reinterpret_cast<const uint16_t *>(st + SG::w_bytes);
#pragma unroll
        for (uint32_t c = 0; c < 2; ++c)
            xs_stage.v[c][0] = *reinterpret_cast<const uint2 *>(x1 + own_col<TYPE, TP>(c, my_j, t));
    }
    const XFrags<N, NT> &xs = TP == 1 ? xs_stage : xs_global;
    const uint32_t ones = 0x3F803F80u;
    constexpr float off = 128.f;   // Q4_K: the code-space offset of code_pair
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
        if constexpr (TYPE != 14) {
            a0 = code_pair(cg, 0x4140u); a1 = code_pair(cg8, 0x4140u);
            a2 = code_pair(cg, 0x4342u); a3 = code_pair(cg8, 0x4342u);
        } else {
            a0 = centred_pair(cg, 0x4140u); a1 = centred_pair(cg8, 0x4140u);
            a2 = centred_pair(cg, 0x4342u); a3 = centred_pair(cg8, 0x4342u);
        }
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
            const uint2 xv = xs.v[c - C0][nt];
            const uint32_t b0 = xv.x * bmask[j], b1 = xv.y * bmask[j];
            mma16816(cq[nt], a0, a1, a2, a3, b0, b1, cq[nt]);
            if constexpr (TYPE != 14) mma16816(c1[nt], ones, ones, ones, ones, b0, b1, c1[nt]);
        }
    };
    // Scale the finished chain `chain` into the accumulators.
    auto close_chain = [&](uint32_t chain) {
#pragma unroll
        for (uint32_t ci = 0; ci < 2; ++ci) {
            const uint32_t G = group_of_visit<TYPE>(chain * S + (2 * t + ci) / TP);
            if constexpr (TYPE != 14) {
                const float2 a = reinterpret_cast<const float2 *>(wt)[g * 8 + G];
                const float2 b = reinterpret_cast<const float2 *>(wt)[(g + 8) * 8 + G];
#pragma unroll
                for (int nt = 0; nt < NT; ++nt) {
                    acc[nt][ci] = fmaf(a.x, fmaf(-off, c1[nt][ci], cq[nt][ci]), fmaf(-a.y, c1[nt][ci], acc[nt][ci]));
                    acc[nt][2 + ci] = fmaf(b.x, fmaf(-off, c1[nt][2 + ci], cq[nt][2 + ci]),
                                           fmaf(-b.y, c1[nt][2 + ci], acc[nt][2 + ci]));
                }
            } else {
                const float a = wt[g * 16 + G], b = wt[(g + 8) * 16 + G];
#pragma unroll
                for (int nt = 0; nt < NT; ++nt) {
                    acc[nt][ci] = fmaf(a, cq[nt][ci], acc[nt][ci]);
                    acc[nt][2 + ci] = fmaf(b, cq[nt][2 + ci], acc[nt][2 + ci]);
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
        for (uint32_t q = 2 * H0; q < 2 * H1; ++q) {
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
        for (uint32_t h = H0; h < H1; ++h) {
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

// Depth of each warp's stage ring: 3 stages, except with two token tiles
// (M > 8), where 2 stages leave room for more resident CTAs (measured: per
// call at M = 16, 19.0 -> 18.0 us; at M = 1 a 2-stage ring is slower).
template <int NT>
constexpr uint32_t gemv_stages() { return NT == 2 ? 2u : 3u; }

// Weights of one launch: blockIdx.x runs over the 16-row tiles of all of
// them (entry e owns tiles [tile_begin, next entry's tile_begin)); they share
// K, type and X, each has its own Y.
template <int TYPE, int TP, int NT, int DT>
__global__ void __launch_bounds__(kWarps * 32, 4) gemv_kernel(const __grid_constant__ GemvBatch b,
                                                           const uint16_t *__restrict__ x, uint32_t m_begin,
                                                           uint32_t m_count, uint64_t k, uint32_t kb_per_slice,
                                                           float *__restrict__ partials,
                                                           uint32_t *__restrict__ counters, uint32_t *status) {
    using SG = StageGeo<TYPE>;
    constexpr uint32_t chunk = chunk_bytes(TYPE);
    extern __shared__ __align__(128) uint8_t dyn[];
    __shared__ float red[kWarps][32][4 * NT];
    __shared__ __align__(16) float tab[kWarps][16 * 16];
    uint32_t ei = 0;
    while (ei + 1 < b.n_entries && blockIdx.x >= b.e[ei + 1].tile_begin) ++ei;
    const GemvEntry &w = b.e[ei];
    void *const y = w.y;
    const uint64_t ldy = w.ldy;
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
    const uint32_t row0 = (blockIdx.x - w.tile_begin) * 16, panel = row0 / kPanelRows, r0 = row0 % kPanelRows;
    const uint32_t n_slices = gridDim.y, kb_begin = blockIdx.y * kb_per_slice;
    const uint32_t kb_end = min(b.kb, kb_begin + kb_per_slice);
    const uint8_t *pbase =
        w.chunks + (uint64_t)(tc_in_bounds(row0 < w.n && kb_end <= b.kb, status) ? panel : 0) * b.kb * chunk;
    constexpr bool kStageX = TP == 1;
    constexpr uint32_t stage_bytes = (SG::w_bytes + (kStageX ? 512u : 0u) + 127) / 128 * 128;
    constexpr uint32_t kGemvStages = gemv_stages<NT>();
    uint8_t *mine = dyn + (size_t)warp * kGemvStages * stage_bytes;
    float *wt = tab[warp];

    // This warp's super-blocks: kb_begin + warp + kWarps * i.  Stage i is
    // commit group i; the weights of the first S-1 stages are issued before
    // the wait on the previous kernel (they do not depend on it), their X
    // after it, each as a group of its own, so that before computing stage i
    // exactly the S-1 most recent groups may still be in flight.
    const uint32_t first = kb_begin + warp;
    const uint32_t count = first < kb_end ? (kb_end - first + kWarps - 1) / kWarps : 0;
#pragma unroll
    for (uint32_t i = 0; i < kGemvStages - 1; ++i) {
        if (i < count) issue_w<TYPE>(mine + i * stage_bytes, pbase + (uint64_t)(first + kWarps * i) * chunk, r0, lane);
        cpa_commit();
    }
    if (threadIdx.x == 0) pdl_launch_dependents();
    pdl_wait();
#pragma unroll
    for (uint32_t i = 0; i < kGemvStages - 1; ++i) {
        if (kStageX && i < count) issue_x1<TYPE>(mine + i * stage_bytes, x, k, m_begin, first + kWarps * i, lane);
        cpa_commit();
    }
    float acc[NT][4];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int i = 0; i < 4; ++i) acc[nt][i] = 0.f;
    // One super-block: refill the slot computed in the previous iteration
    // (every lane is past it: __syncwarp at the end of the iteration), wait
    // for this one's stage, load the next super-block's X fragments, compute.
    // With two token tiles (NT = 2) a second fragment set would halve the
    // resident CTAs (registers): there X is loaded at the start of its own
    // super-block instead.
    constexpr bool kAhead = NT == 1;
    uint32_t bmask[8 / TP];
#pragma unroll
    for (uint32_t j = 0; j < 8 / TP; ++j) bmask[j] = g / TP == j ? 1u : 0u;
    auto refill_and_wait = [&](uint32_t i) {
        if (i + kGemvStages - 1 < count) {
            const uint32_t j = i + kGemvStages - 1, kb = first + kWarps * j;
            uint8_t *sj = mine + (j % kGemvStages) * stage_bytes;
            issue_w<TYPE>(sj, pbase + (uint64_t)kb * chunk, r0, lane);
            if (kStageX) issue_x1<TYPE>(sj, x, k, m_begin, kb, lane);
        }
        cpa_commit();
        cpa_wait<kGemvStages - 1>();
        __syncwarp();
    };
    if constexpr (kAhead) {
        // One super-block per iteration: refill the slot computed in the
        // previous iteration (every lane is past it: __syncwarp at the end of
        // the iteration), wait for this one's stage, load the next
        // super-block's X fragments (several tokens), compute.
        using XF = XFrags<2 * TP, NT>;
        auto iteration = [&](uint32_t i, XF &xs_cur, XF &xs_next) {
            refill_and_wait(i);
            if constexpr (TP > 1)
                if (i + 1 < count)
                    load_x<TYPE, TP, NT>(xs_next, x, k, m_begin, first + kWarps * (i + 1), m_count, g, t, 0);
            compute_stage<TYPE, TP, NT>(mine + (i % kGemvStages) * stage_bytes, xs_cur, g, t, lane, bmask, wt, acc);
            __syncwarp();
        };
        XF xa, xb;
        if (TP > 1 && count) load_x<TYPE, TP, NT>(xa, x, k, m_begin, first, m_count, g, t, 0);
        for (uint32_t i = 0; i < count; i += 2) {
            iteration(i, xa, xb);
            if (i + 1 < count) iteration(i + 1, xb, xa);
        }
    } else {
        // Two token tiles (8 tokens each): a second whole-super-block fragment
        // set would cost resident CTAs (registers), so X runs half a
        // super-block ahead instead -- half 1's fragments load while half 0
        // computes, the next super-block's half 0 while half 1 computes.
        using XF = XFrags<8, NT>;
        XF xa, xb;
        if (count) load_x<TYPE, TP, NT>(xa, x, k, m_begin, first, m_count, g, t, 0);
        for (uint32_t i = 0; i < count; ++i) {
            refill_and_wait(i);
            const uint8_t *st = mine + (i % kGemvStages) * stage_bytes;
            const uint32_t kb = first + kWarps * i;
            load_x<TYPE, TP, NT>(xb, x, k, m_begin, kb, m_count, g, t, 8);
            compute_stage<TYPE, TP, NT, 8, 0, 1, 0>(st, xa, g, t, lane, bmask, wt, acc);
            if (i + 1 < count) load_x<TYPE, TP, NT>(xa, x, k, m_begin, kb + kWarps, m_count, g, t, 0);
            compute_stage<TYPE, TP, NT, 8, 1, 2, 8>(st, xb, g, t, lane, bmask, wt, acc);
            __syncwarp();
        }
    }
    // Columns of one token are spread over the quad (TP < 8): sum them so that
    // every lane holds the full value of its (row, token) pairs.
    if constexpr (TP == 1) {   // all 8 columns are token 0: fold the thread's two columns
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
            acc[nt][0] += acc[nt][1];
            acc[nt][2] += acc[nt][3];
            acc[nt][1] = acc[nt][0];
            acc[nt][3] = acc[nt][2];
        }
    }
    if constexpr (TP <= 2) {
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                acc[nt][i] += __shfl_xor_sync(0xffffffffu, acc[nt][i], 1);
                acc[nt][i] += __shfl_xor_sync(0xffffffffu, acc[nt][i], 2);
            }
    } else if constexpr (TP == 4) {
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
            for (int i = 0; i < 4; ++i) acc[nt][i] += __shfl_xor_sync(0xffffffffu, acc[nt][i], 2);
    }

    // Reduce the warps' fragments; then either store Y directly (one K slice)
    // or publish the partial and let the tile's last CTA finish.
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int i = 0; i < 4; ++i) red[warp][lane][4 * nt + i] = acc[nt][i];
    __syncthreads();
    __shared__ uint32_t last;
    if (warp == 0) {
        float v[4 * NT];
#pragma unroll
        for (int j = 0; j < 4 * NT; ++j) {
            float sum = 0.f;
#pragma unroll
            for (int ww2 = 0; ww2 < kWarps; ++ww2) sum += red[ww2][lane][j];
            v[j] = sum;
        }
        bool store = n_slices == 1;
        if (n_slices > 1) {
            // partials[slice][tile][lane][4*NT]
            float *dst = partials + (((uint64_t)blockIdx.y * gridDim.x + blockIdx.x) * 32 + lane) * (4 * NT);
#pragma unroll
            for (int j = 0; j < 4 * NT; ++j) __stcg(dst + j, v[j]);
            // The warp barrier orders every lane's partial stores before lane
            // 0's arrival; the arrival is one acquire-release atomic: release
            // publishes this slice's partial, acquire (for the last slice to
            // arrive) makes the other slices' partials visible -- one round
            // trip to L2 instead of fence + atomic + fence.
            __syncwarp();
            if (lane == 0) last = (arrive_acq_rel(counters + blockIdx.x) + 1 == n_slices) ? 1u : 0u;
            __syncwarp();
            if (last) {
#pragma unroll
                for (int j = 0; j < 4 * NT; ++j) v[j] = 0.f;
                for (uint32_t sl = 0; sl < n_slices; ++sl) {
                    const float *src = partials + (((uint64_t)sl * gridDim.x + blockIdx.x) * 32 + lane) * (4 * NT);
#pragma unroll
                    for (int j = 0; j < 4 * NT; ++j) v[j] += __ldcg(src + j);
                }
                if (lane == 0) counters[blockIdx.x] = 0u;
                store = true;
            }
        }
        if (store && b.epi.flags) {
            // Fused epilogue.  A thread holds rows g and g + 8 of the tile for
            // the same token: for a SwiGLU weight the gate row and its up row.
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
        } else if (store) {
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
        if (store && b.epi.n_peer) __threadfence_system();   // publish peer-replica stores
    }
}

template <int TYPE, int TP, int NT>
cudaError_t launch_typed(const GemvBatch &bt, uint32_t tiles, uint32_t m_begin, uint32_t mc, const uint16_t *x,
                         uint64_t k, int out_dtype, const GemvSplit &sp, cudaStream_t s) {
    const dim3 grid(tiles, sp.n_slices);
    const size_t stage = (StageGeo<TYPE>::w_bytes + (TP == 1 ? 512u : 0u) + 127) / 128 * 128;
    const size_t smem = stage * gemv_stages<NT>() * kWarps;
    auto kern = out_dtype == 0 ? gemv_kernel<TYPE, TP, NT, 0>
                : out_dtype == 1 ? gemv_kernel<TYPE, TP, NT, 1> : gemv_kernel<TYPE, TP, NT, 2>;
    // Opt in once per instantiation and device to its shared-memory size.
    static DeviceCache cache[3];
    int unused = 0;
    cudaError_t e = per_device(cache[out_dtype], unused, [&](int &) {
        return cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    });
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(kWarps * 32);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, bt, x, m_begin, mc, k, sp.kb_per_slice, sp.partials, sp.counters,
                              sp.status);
}

template <int TYPE>
cudaError_t launch_m(const GemvBatch &bt, uint32_t tiles, uint32_t m_begin, uint32_t m, const uint16_t *x,
                     uint64_t k, int out_dtype, const GemvSplit &sp, cudaStream_t s) {
    if (m <= 1) return launch_typed<TYPE, 1, 1>(bt, tiles, m_begin, m, x, k, out_dtype, sp, s);
    if (m <= 2) return launch_typed<TYPE, 2, 1>(bt, tiles, m_begin, m, x, k, out_dtype, sp, s);
    if (m <= 4) return launch_typed<TYPE, 4, 1>(bt, tiles, m_begin, m, x, k, out_dtype, sp, s);
    if (m <= 8) return launch_typed<TYPE, 8, 1>(bt, tiles, m_begin, m, x, k, out_dtype, sp, s);
    return launch_typed<TYPE, 8, 2>(bt, tiles, m_begin, m, x, k, out_dtype, sp, s);
}

}  // namespace

GemvSplit gemv_split_tiles(uint32_t tiles, uint32_t kb) {
    // Enough CTAs for about three per SM, with as few K slices as that allows
    // (each slice costs a partial store and a share of the fixup): a single
    // weight of a few hundred row tiles splits K three ways, a batch of
    // thousands of tiles runs whole rows per CTA.  Slices hold a multiple of
    // the 4 warps' super-blocks.
    const uint32_t want = 148u * 3u;
    uint32_t slices = tiles >= want ? 1u : (want + tiles - 1) / tiles;
    slices = max(1u, min(slices, (kb + kWarps - 1) / kWarps));
    uint32_t per = (kb + slices - 1) / slices;
    per = (per + kWarps - 1) / kWarps * kWarps;
    GemvSplit sp;
    sp.kb_per_slice = per;
    sp.n_slices = (kb + per - 1) / per;
    return sp;
}
GemvSplit gemv_split(const WeightView &w) { return gemv_split_tiles((w.n + 15) / 16, w.kb); }

size_t gemv_workspace_floats_tiles(uint32_t tiles, uint32_t kb) {
    const GemvSplit sp = gemv_split_tiles(tiles, kb);
    return sp.n_slices > 1 ? (size_t)sp.n_slices * tiles * 32 * 8 : 0;
}
size_t gemv_workspace_floats(const WeightView &w) { return gemv_workspace_floats_tiles((w.n + 15) / 16, w.kb); }

cudaError_t launch_gemv_batch(const GemvBatch &bt_in, uint32_t type, uint32_t tiles, uint32_t m_begin, uint32_t m,
                              const uint16_t *x, uint64_t k, int out_dtype, const GemvSplit &sp, cudaStream_t s,
                              const EpiView *epi, uint32_t gate_row) {
    if (!m || !tiles) return cudaSuccess;
    if (out_dtype < 0 || out_dtype > 2) return cudaErrorInvalidValue;
    GemvBatch bt = bt_in;
    bt.epi = epi ? *epi : EpiView{};
    bt.gate_row = gate_row;
    if (m > 16 || bt.n_entries == 0 || bt.n_entries > kMaxGemvBatch) return cudaErrorInvalidValue;
    if (sp.n_slices > 1 && (!sp.partials || !sp.counters)) return cudaErrorInvalidValue;
    if (type == 12) return launch_m<12>(bt, tiles, m_begin, m, x, k, out_dtype, sp, s);
    if (type == 13) return launch_m<13>(bt, tiles, m_begin, m, x, k, out_dtype, sp, s);
    return launch_m<14>(bt, tiles, m_begin, m, x, k, out_dtype, sp, s);
}

cudaError_t launch_gemv(const SegmentView &seg, const uint16_t *x, uint64_t k, void *y, uint64_t ldy,
                        int out_dtype, const GemvSplit &sp, cudaStream_t s, const EpiView *epi) {
    if (seg.m_end <= seg.m_begin) return cudaSuccess;
    GemvBatch bt{};
    bt.n_entries = 1;
    bt.kb = seg.w.kb;
    bt.e[0] = {seg.w.chunks, y, ldy, seg.w.n, 0u};
    return launch_gemv_batch(bt, seg.w.type, (seg.w.n + 15) / 16, seg.m_begin, seg.m_end - seg.m_begin, x, k,
                             out_dtype, sp, s, epi, seg.gate_row);
}

}  // namespace tc
