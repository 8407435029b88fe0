// Quantised GEMM on CTA pairs (tcgen05 cta_group::2, sm_100a):
//     Y[m, n] = sum_k X[m, k] * W[n, k],  W in GGUF Q4_K / Q6_K, X bf16 (or fp16).
//
// A cluster of two CTAs computes one 256-token x 256-weight-row tile with
// MMAs of shape M = 256 (tokens) x N = 256 (weight rows) x K = 16, issued by a
// single thread of CTA 0 (the leader) for both SMs:
//   A = activations, K-major, 128-byte swizzle: each CTA holds its own 128
//       tokens x 64 K per stage, loaded by TMA;
//   B = dequantised weights: each CTA unpacks its own 128-row weight panel
//       (one packed chunk = 128 rows x 256 K) into the swizzled bf16 tile, bit-
//       exact to the reference decoder; the MMA reads B's halves from both CTAs.
// Compared with a one-CTA 128 x 256 tile doing the same MMA work per SM, each
// CTA streams half the activation bytes from L2 per stage (16 KB instead of
// 32 KB), which leaves room for a 4-deep pipeline in shared memory.
// D lands in each CTA's TMEM as [128 lanes = its tokens] x [256 columns =
// weight rows], two accumulators of 256 columns each (all 512 TMEM columns),
// so the epilogue of tile i overlaps the main loop of tile i+1.  An epilogue
// thread owns one token and 32 consecutive outputs per TMEM load: it packs
// them into a 64-byte-swizzled staging tile and the warp writes whole lines
// with a TMA store (plain stores for f32 output and ragged edges).
//
// Warp roles (22 warps, both CTAs):
//   warp 0     producer: bulk copy of the packed chunk, TMA of the activations;
//   warp 1     TMEM allocator (cta_group::2, both CTAs); in the leader, the
//              MMA-issuing thread;
//   warps 2-5  epilogue;
//   warps 6-21 dequantisers.
// Per stage, each CTA's dequant warps arrive on a local `dq_done` barrier and
// its activation copy completes a local `x_full`; the leader's MMA thread
// waits on its own two barriers and on `full`, to which the peer CTA's warp 1
// relays one remote arrival per stage once the peer's two barriers complete
// (a remote arrival takes a DSMEM round trip; keeping it off the dequant
// warps keeps them unpacking).  The leader's MMA completion is committed to
// both CTAs' barriers (tcgen05.commit with a CTA mask).  No TMA load uses cluster multicast: every copy lands in the CTA
// that issued it and signals that CTA's own barrier.  Every wait is bounded;
// on timeout both CTAs raise their abort flags, set TC_STATUS_TIMEOUT, drain
// their own copies and MMAs, free TMEM and return.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <cstring>

#include "kq_sm100.cuh"
#include "tc_internal.h"

namespace tc {
namespace {

constexpr int kThreads = 704;
constexpr int kDequantWarp0 = 6, kDequantWarps = 16, kDequantThreads = 512;
constexpr int kEpiWarps = 4;
constexpr int kStages = 4;       // activation + B-tile pipeline depth (64 K each)
constexpr int kWStages = 2;      // packed chunk pipeline depth (256 K each)
constexpr int kMaxSeg = 32;
constexpr uint32_t kTileM = 256, kHalfM = 128, kTileN = 256;

struct PairSeg {
    uint32_t m_begin, m_end, tile_begin, pad;
    const uint8_t *w;
};
struct PairParams {
    PairSeg seg[kMaxSeg];
    uint32_t n_seg, n_tiles, kb, panels, pair_panels, n;
    void *y;
    uint64_t ldy;
    uint32_t *status;
    uint32_t y_tma;   // bf16 Y through TMA stores (16-byte aligned base and row pitch)
    uint32_t y_vec;   // 16-byte vector stores allowed on the plain-store path
};

template <int TYPE>
struct PairLayout {
    static constexpr uint32_t x_stage = kHalfM * 128;   // 128 tokens x 64 K x 2 B
    static constexpr uint32_t b_stage = 128 * 128;      // 128 weight rows x 64 K x 2 B
    static constexpr uint32_t e_piece = 32 * 64;        // 32 tokens x 32 outputs x 2 B
    static constexpr uint32_t e_bufs = TYPE == 12 ? 2 : 1;   // per epilogue warp (Q6_K: smem-bound)
    static constexpr uint32_t w_stage = chunk_bytes(TYPE);
    static constexpr uint32_t x_off = 0;
    static constexpr uint32_t b_off = x_off + kStages * x_stage;
    static constexpr uint32_t e_off = b_off + kStages * b_stage;
    static constexpr uint32_t w_off = e_off + kEpiWarps * e_bufs * e_piece;
    static constexpr uint32_t t_off = (w_off + kWStages * w_stage + 127) / 128 * 128;
    static constexpr uint32_t table_bytes = 128 * 80;
    static constexpr uint32_t n_tables = 3;
    static constexpr uint32_t bar_off = t_off + n_tables * table_bytes;
    // x_full[S] dq_done[S] full[S] st_empty[S] w_full[W] w_empty[W] t_ready[3]
    // acc_full[2] acc_empty[2] fin
    static constexpr uint32_t n_bars = 4 * kStages + 2 * kWStages + n_tables + 5;
    static constexpr uint32_t misc_off = bar_off + n_bars * 8;
    static constexpr uint32_t bytes = misc_off + 16 + 1024;  // + alignment slack
    static constexpr uint32_t tmem_cols = 512;
    static_assert(bytes <= 232448, "shared memory per CTA exceeds the sm_100 limit");
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
// semantics).  The data this arrival publishes is this CTA's own shared memory
// (dequantised B tile, or TMEM already read back), which the CTA-scope release
// has completed before the arrival is sent; a cluster-scope release would add
// a full memory barrier (hundreds of cycles) to every pipeline stage.
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
// both K-major, M = 256, N = 256.
template <bool F16>
__device__ __forceinline__ constexpr uint32_t pair_idesc() {
    return (1u << 4) | ((F16 ? 0u : 1u) << 7) | ((F16 ? 0u : 1u) << 10) | ((kTileN >> 3) << 17) |
           ((kTileM >> 4) << 24);
}
__device__ __forceinline__ void mma_pair(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n}\n"
        ::"r"(d_tmem), "l"(a), "l"(b), "r"(idesc), "r"(acc));
}
// Arrive (once the leader's MMAs issued so far complete) on the barrier at
// offset `b` in both CTAs of the pair.
__device__ __forceinline__ void commit_both(uint32_t b) {
    asm volatile(
        "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;"
        ::"r"(b), "h"((uint16_t)3) : "memory");
}
__device__ __forceinline__ void tma_store_2d(const CUtensorMap *map, uint32_t src, int x, int y) {
    asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];"
                 ::"l"(reinterpret_cast<uint64_t>(map)), "r"(src), "r"(x), "r"(y) : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_read1() { asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_read0() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
__device__ __forceinline__ uint32_t bf16x2(uint32_t lo, uint32_t hi) {
    uint32_t r;
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(__uint_as_float(hi)), "f"(__uint_as_float(lo)));
    return r;
}

// ------------------------------------------------------------ tiles
struct PairTile {
    uint32_t m0, m_end, pp;   // first token, segment end, pair-panel (256 weight rows)
    const uint8_t *w;
};
__device__ __forceinline__ PairTile pair_tile(const PairParams &p, uint32_t t) {
    uint32_t s = 0;
    while (s + 1 < p.n_seg && t >= p.seg[s + 1].tile_begin) ++s;
    const uint32_t local = t - p.seg[s].tile_begin;
    return {p.seg[s].m_begin + (local / p.pair_panels) * kTileM, p.seg[s].m_end, local % p.pair_panels, p.seg[s].w};
}

// Plain stores of one token's 32 outputs (ragged edges, f32 output, or Y
// without TMA-compatible alignment).
template <bool OUT_F32>
__device__ __forceinline__ void store_row(const PairParams &p, uint32_t m, uint32_t n0, const uint32_t (&v)[32]) {
    if (OUT_F32) {
        float *y = static_cast<float *>(p.y) + (uint64_t)m * p.ldy;
#pragma unroll
        for (uint32_t j = 0; j < 32; j += 4) {
            if (p.y_vec && n0 + j + 4 <= p.n) {
                *reinterpret_cast<uint4 *>(y + n0 + j) = make_uint4(v[j], v[j + 1], v[j + 2], v[j + 3]);
            } else {
#pragma unroll
                for (uint32_t c = 0; c < 4; ++c)
                    if (n0 + j + c < p.n) y[n0 + j + c] = __uint_as_float(v[j + c]);
            }
        }
    } else {
        __nv_bfloat16 *y = static_cast<__nv_bfloat16 *>(p.y) + (uint64_t)m * p.ldy;
#pragma unroll
        for (uint32_t j = 0; j < 32; j += 8) {
            if (p.y_vec && n0 + j + 8 <= p.n) {
                *reinterpret_cast<uint4 *>(y + n0 + j) =
                    make_uint4(bf16x2(v[j], v[j + 1]), bf16x2(v[j + 2], v[j + 3]), bf16x2(v[j + 4], v[j + 5]),
                               bf16x2(v[j + 6], v[j + 7]));
            } else {
#pragma unroll
                for (uint32_t c = 0; c < 8; ++c)
                    if (n0 + j + c < p.n) y[n0 + j + c] = __float2bfloat16_rn(__uint_as_float(v[j + c]));
            }
        }
    }
}

// ------------------------------------------------------------ the kernel
template <int TYPE, bool F16, bool OUT_F32>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    pair_gemm_kernel(const __grid_constant__ CUtensorMap xmap, const __grid_constant__ CUtensorMap ymap,
                     const __grid_constant__ PairParams p) {
    using L = PairLayout<TYPE>;
    constexpr uint32_t kChunk = chunk_bytes(TYPE);
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const uint32_t warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    const uint32_t rank = cta_rank();          // 0: leader, issues the MMAs for both CTAs
    const uint32_t pair = blockIdx.x >> 1, n_pairs = gridDim.x >> 1;

    const uint32_t bars = su32(smem + L::bar_off);
    constexpr uint32_t kT = L::n_tables;
    auto x_full = [&](uint32_t i) { return bars + 8 * i; };
    auto dq_done = [&](uint32_t i) { return bars + 8 * (kStages + i); };
    auto full = [&](uint32_t i) { return bars + 8 * (2 * kStages + i); };
    auto st_empty = [&](uint32_t i) { return bars + 8 * (3 * kStages + i); };
    auto w_full = [&](uint32_t i) { return bars + 8 * (4 * kStages + i); };
    auto w_empty = [&](uint32_t i) { return bars + 8 * (4 * kStages + kWStages + i); };
    auto t_ready = [&](uint32_t i) { return bars + 8 * (4 * kStages + 2 * kWStages + i); };
    auto acc_full = [&](uint32_t i) { return bars + 8 * (4 * kStages + 2 * kWStages + kT + i); };
    auto acc_empty = [&](uint32_t i) { return bars + 8 * (4 * kStages + 2 * kWStages + kT + 2 + i); };
    const uint32_t fin = bars + 8 * (4 * kStages + 2 * kWStages + kT + 4);
    auto table = [&](uint32_t i) { return reinterpret_cast<float *>(smem + L::t_off + i * L::table_bytes); };
    // Tiles of this pair: pair, pair + n_pairs, ...
    const uint32_t my_tiles = p.n_tiles > pair ? (p.n_tiles - pair + n_pairs - 1) / n_pairs : 0;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + L::misc_off);
    volatile uint32_t *abort_flag = tmem_slot + 1;

    if (threadIdx.x == 0) {
        for (int i = 0; i < kStages; ++i) {
            bar_init(x_full(i), 1);
            bar_init(dq_done(i), kDequantWarps);
            bar_init(full(i), 1);                   // leader's copy: the peer's relay
            bar_init(st_empty(i), 1);
        }
        for (int i = 0; i < kWStages; ++i) {
            bar_init(w_full(i), 1);
            bar_init(w_empty(i), kDequantWarps);
        }
        for (uint32_t i = 0; i < kT; ++i) bar_init(t_ready(i), kDequantThreads);
        for (int i = 0; i < 2; ++i) {
            bar_init(acc_full(i), 1);
            bar_init(acc_empty(i), 2 * kEpiWarps);  // leader's copy is the one used
        }
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
        // ---------------------------------------------------- producer
        if (lane == 0) {
            // X (and the Y the epilogue writes) may belong to the previous
            // kernel in the stream: wait for it before the first activation load.
            asm volatile("griddepcontrol.wait;" ::: "memory");
            uint32_t st = 0, ph = 0, ws = 0, wph = 0;
            uint32_t x_last[kStages], w_last[kWStages];
            bool x_used[kStages] = {}, w_used[kWStages] = {};
            bool ok = true;
            for (uint32_t t = pair; ok && t < p.n_tiles; t += n_pairs) {
                const PairTile T = pair_tile(p, t);
                // A missing second panel (odd panel count) re-reads the last
                // panel; its outputs fall past N and are never stored.
                uint32_t panel = 2 * T.pp + rank;
                if (panel >= p.panels) panel = p.panels - 1;
                const uint8_t *pw = T.w + (uint64_t)panel * p.kb * kChunk;
                const int my_m = (int)(T.m0 + rank * kHalfM);
                for (uint32_t kb = 0; ok && kb < p.kb; ++kb) {
                    if (!(ok = pwait(w_empty(ws), wph ^ 1, ab))) break;
                    bar_expect_tx(w_full(ws), kChunk);
                    bulk_load(su32(smem + L::w_off + ws * L::w_stage), pw + (uint64_t)kb * kChunk, kChunk, w_full(ws));
                    w_last[ws] = wph; w_used[ws] = true;
                    if (++ws == kWStages) { ws = 0; wph ^= 1; }
                    for (uint32_t q = 0; q < 4; ++q) {
                        if (!(ok = pwait(st_empty(st), ph ^ 1, ab))) break;
                        bar_expect_tx(x_full(st), L::x_stage);
                        tma_load_2d(su32(smem + L::x_off + st * L::x_stage), &xmap, x_full(st),
                                    (int)(kb * 256 + q * 64), my_m);
                        x_last[st] = ph; x_used[st] = true;
                        if (++st == kStages) { st = 0; ph ^= 1; }
                    }
                }
            }
            // Drain: every copy this thread issued has landed before exit.
            for (int i = 0; i < kStages; ++i)
                if (x_used[i]) pwait(x_full(i), x_last[i], ab, false);
            for (int i = 0; i < kWStages; ++i)
                if (w_used[i]) pwait(w_full(i), w_last[i], ab, false);
        }
        __syncwarp();
    } else if (warp == 1) {
        // ---------------------------------------------------- MMA issuer (leader)
        if (lane == 0 && rank == 0) {
            constexpr uint32_t idesc = pair_idesc<F16>();
            uint32_t st = 0, ph = 0, acc = 0, aph = 0;
            bool ok = true;
            for (uint32_t t = pair; ok && t < p.n_tiles; t += n_pairs) {
                if (!(ok = pwait(acc_empty(acc), aph ^ 1, ab))) break;
                tc_fence_after();
                const uint32_t d_tmem = tmem + acc * kTileN;
                for (uint32_t kb = 0; ok && kb < p.kb; ++kb) {
                    for (uint32_t q = 0; q < 4; ++q) {
                        if (!(ok = pwait(x_full(st), ph, ab))) break;
                        if (!(ok = pwait(dq_done(st), ph, ab))) break;
                        if (!(ok = pwait(full(st), ph, ab))) break;   // the peer's stage
                        tc_fence_after();
                        const uint32_t a_addr = su32(smem + L::x_off + st * L::x_stage);
                        const uint32_t b_addr = su32(smem + L::b_off + st * L::b_stage);
#pragma unroll
                        for (uint32_t kk = 0; kk < 4; ++kk)
                            mma_pair(d_tmem, sw128_desc(a_addr + kk * 32), sw128_desc(b_addr + kk * 32), idesc,
                                     (kb | q | kk) ? 1u : 0u);
                        commit_both(st_empty(st));
                        if (++st == kStages) { st = 0; ph ^= 1; }
                    }
                }
                if (!ok) break;
                commit_both(acc_full(acc));
                acc ^= 1;
                if (acc == 0) aph ^= 1;
            }
            // Every MMA issued by this thread has completed (in both CTAs)
            // before either CTA frees its TMEM.
            commit_both(fin);
        } else if (lane == 0) {
            // ---------------------------------------------------- relay (peer)
            // Forwards "this CTA's stage is complete" to the leader's `full`.
            uint32_t st = 0, ph = 0;
            const uint32_t n_stages = my_tiles * p.kb * 4;
            for (uint32_t i = 0; i < n_stages; ++i) {
                if (!pwait(x_full(st), ph, ab)) break;
                if (!pwait(dq_done(st), ph, ab)) break;
                bar_arrive_cluster(cluster_addr(full(st), 0));
                if (++st == kStages) { st = 0; ph ^= 1; }
            }
        }
        if (lane == 0) pwait(fin, 0, ab, false);
        __syncwarp();
    } else if (warp >= (uint32_t)kDequantWarp0) {
        // ---------------------------------------------------- dequantisers
        // Chunks (128 weight rows x 256 K) are unpacked in order.  The scale
        // table of chunk c + 1 is built during chunk c's last stage, into the
        // next of three table buffers (a buffer is rewritten only after every
        // thread has passed the chunk that read it), so a chunk never starts
        // with a CTA-wide wait on a table that was just built.  Waits are
        // warp-uniform (__all_sync): the warp synchronises after every stage
        // and leaves together on abort.
        const uint32_t dt = threadIdx.x - kDequantWarp0 * 32, dw = dt / 32;
        const uint32_t r = 8 * dw + (lane >> 3) + 4 * ((lane >> 2) & 1);
        const uint32_t n_chunks = my_tiles * p.kb;
        uint32_t st = 0, ph = 0;
        bool ok = true, ovf = false;
        auto build = [&](uint32_t c) -> bool {
            const uint32_t ws = c % kWStages;
            if (!__all_sync(0xffffffffu, pwait(w_full(ws), (c / kWStages) & 1, ab))) return false;
            build_table<TYPE, F16>(smem + L::w_off + ws * L::w_stage, table(c % kT), dt, ovf);
            bar_arrive(t_ready(c % kT));
            return true;
        };
        if (n_chunks) ok = build(0);
        for (uint32_t c = 0; ok && c < n_chunks; ++c) {
            const uint8_t *wc = smem + L::w_off + (c % kWStages) * L::w_stage;
            const float *tab = table(c % kT);
            if (!(ok = __all_sync(0xffffffffu, pwait(t_ready(c % kT), (c / kT) & 1, ab)))) break;
            for (uint32_t q = 0; q < 4; ++q) {
                if (q == 3 && c + 1 < n_chunks && !(ok = build(c + 1))) break;
                if (!(ok = __all_sync(0xffffffffu, pwait(st_empty(st), ph ^ 1, ab)))) break;
                dequant_task<TYPE, F16>(wc, tab, q, r, lane & 3, smem + L::b_off + st * L::b_stage);
                fence_proxy_async();
                __syncwarp();
                if (lane == 0) bar_arrive(dq_done(st));
                if (++st == kStages) { st = 0; ph ^= 1; }
            }
            if (!ok) break;
            __syncwarp();
            if (lane == 0) bar_arrive(w_empty(c % kWStages));
        }
        if (F16 && ovf) atomicOr(p.status, kStatusF16);
    } else {
        // ---------------------------------------------------- epilogue
        const uint32_t quad = warp & 3;   // TMEM lanes 32*quad .. +31
        uint32_t acc = 0, aph = 0, piece = 0;
        uint8_t *stage = smem + L::e_off + quad * L::e_bufs * L::e_piece;
        for (uint32_t t = pair; t < p.n_tiles; t += n_pairs) {
            const PairTile T = pair_tile(p, t);
            if (!__all_sync(0xffffffffu, pwait(acc_full(acc), aph, ab))) break;
            tc_fence_after();
            const uint32_t row0 = T.m0 + rank * kHalfM + quad * 32;   // this warp's first token
            const bool rows_all = row0 + 32 <= T.m_end, rows_any = row0 < T.m_end;
            const uint32_t taddr = tmem + ((quad * 32) << 16) + acc * kTileN;
#pragma unroll 1
            for (uint32_t c0 = 0; c0 < kTileN; c0 += 32) {
                const uint32_t n0 = T.pp * kTileN + c0;
                if (!rows_any || n0 >= p.n) continue;
                uint32_t v[32];
                tmem_ld32(taddr + c0, v);
                if (!OUT_F32 && p.y_tma && rows_all) {
                    uint8_t *buf = stage + (piece % L::e_bufs) * L::e_piece;
                    if (lane == 0) {   // the store that last used `buf` has read it
                        if (L::e_bufs == 2) bulk_wait_read1();
                        else bulk_wait_read0();
                    }
                    __syncwarp();
                    uint8_t *row = buf + lane * 64;
                    const uint32_t sw = (lane >> 1) & 3;   // 64-byte swizzle of the TMA box
#pragma unroll
                    for (uint32_t j = 0; j < 4; ++j)
                        *reinterpret_cast<uint4 *>(row + ((j ^ sw) << 4)) =
                            make_uint4(bf16x2(v[8 * j], v[8 * j + 1]), bf16x2(v[8 * j + 2], v[8 * j + 3]),
                                       bf16x2(v[8 * j + 4], v[8 * j + 5]), bf16x2(v[8 * j + 6], v[8 * j + 7]));
                    fence_proxy_async();
                    __syncwarp();
                    if (lane == 0) {
                        tma_store_2d(&ymap, su32(buf), (int)n0, (int)row0);
                        bulk_commit();
                    }
                    ++piece;
                } else if (row0 + lane < T.m_end) {
                    store_row<OUT_F32>(p, row0 + lane, n0, v);
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) bar_arrive_cluster(cluster_addr(acc_empty(acc), 0));
            acc ^= 1;
            if (acc == 0) aph ^= 1;
        }
        if (lane == 0) bulk_wait_all();
        __syncwarp();
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

template <int TYPE, bool F16, bool OUT_F32>
cudaError_t launch_pair_inst(const CUtensorMap &xm, const CUtensorMap &ym, const PairParams &p, cudaStream_t s) {
    using L = PairLayout<TYPE>;
    auto kernel = pair_gemm_kernel<TYPE, F16, OUT_F32>;
    static int max_clusters = 0;   // co-resident 2-CTA clusters on this GPU
    if (!max_clusters) {
        cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)L::bytes);
        if (e != cudaSuccess) return e;
        cudaLaunchConfig_t q = {};
        q.gridDim = dim3(2);
        q.blockDim = dim3(kThreads);
        q.dynamicSmemBytes = L::bytes;
        e = cudaOccupancyMaxActiveClusters(&max_clusters, kernel, &q);
        if (e != cudaSuccess) return e;
        if (max_clusters < 1) return cudaErrorInvalidConfiguration;
    }
    const uint32_t pairs = p.n_tiles < (uint32_t)max_clusters ? p.n_tiles : (uint32_t)max_clusters;
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

}  // namespace

bool gemm_pair_supported(uint32_t n_seg) { return n_seg <= (uint32_t)kMaxSeg; }

cudaError_t launch_gemm_pair(const SegmentView *segs, uint32_t n_seg, const uint16_t *x, uint64_t m_total,
                             uint64_t k, void *y, uint64_t ldy, int out_dtype, int stage_f16, uint32_t *status,
                             cudaStream_t s) {
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
    uint32_t tiles = 0;
    for (uint32_t i = 0; i < n_seg; ++i) {
        p.seg[i] = {segs[i].m_begin, segs[i].m_end, tiles, 0u, segs[i].w.chunks};
        tiles += (segs[i].m_end - segs[i].m_begin + kTileM - 1) / kTileM * p.pair_panels;
    }
    p.n_tiles = tiles;
    if (!tiles) return cudaSuccess;

    auto enc = encode_fn();
    if (!enc) return cudaErrorNotSupported;
    CUtensorMap xm, ym;
    {
        const cuuint64_t dims[2] = {k, m_total};
        const cuuint64_t strides[1] = {k * 2};
        const cuuint32_t box[2] = {64u, kHalfM};
        const cuuint32_t estr[2] = {1u, 1u};
        const CUresult r = enc(&xm, stage_f16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2,
                               const_cast<uint16_t *>(x), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                               CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        if (r != CUDA_SUCCESS) return cudaErrorInvalidValue;
    }
    const int out_f32 = out_dtype == 0;
    const uint64_t esize = out_f32 ? 4 : 2;
    p.y_vec = ((reinterpret_cast<uintptr_t>(y) & 15u) == 0 && (ldy * esize) % 16 == 0) ? 1u : 0u;
    memset(&ym, 0, sizeof(ym));
    if (!out_f32 && p.y_vec) {
        const cuuint64_t dims[2] = {p.n, m_total};
        const cuuint64_t strides[1] = {ldy * 2};
        const cuuint32_t box[2] = {32u, 32u};
        const cuuint32_t estr[2] = {1u, 1u};
        const CUresult r = enc(&ym, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, y, dims, strides, box, estr,
                               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B,
                               CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        p.y_tma = r == CUDA_SUCCESS ? 1u : 0u;
    }
    const uint32_t type = segs[0].w.type;
    if (type == 12) {
        if (stage_f16) return out_f32 ? launch_pair_inst<12, true, true>(xm, ym, p, s) : launch_pair_inst<12, true, false>(xm, ym, p, s);
        return out_f32 ? launch_pair_inst<12, false, true>(xm, ym, p, s) : launch_pair_inst<12, false, false>(xm, ym, p, s);
    }
    if (stage_f16) return out_f32 ? launch_pair_inst<14, true, true>(xm, ym, p, s) : launch_pair_inst<14, true, false>(xm, ym, p, s);
    return out_f32 ? launch_pair_inst<14, false, true>(xm, ym, p, s) : launch_pair_inst<14, false, false>(xm, ym, p, s);
}

}  // namespace tc
