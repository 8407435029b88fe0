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

#include "kq_epilogue.cuh"
#include "kq_sm100.cuh"
#include "tc_internal.h"

namespace tc {
namespace {

constexpr int kThreads = 704;   // 22 warps
constexpr int kEpiWarp0 = 2, kEpiThreads = 128, kDequantWarp0 = 6, kDequantThreads = 512;
constexpr int kStages = 3;      // activation / A-tile pipeline depth (64 K each)
constexpr int kWStages = 2;     // packed chunk pipeline depth (256 K each)
constexpr int kMaxSeg = 32;

struct GemmSeg {
    uint32_t m_begin, m_end, tile_begin, gate_row;
    const uint8_t *w;
};
struct GemmParams {
    GemmSeg seg[kMaxSeg];
    uint32_t n_seg, n_tiles, kb, panels, n;
    void *y;
    uint64_t ldy;
    uint32_t *status;
    EpiView epi;      // fused epilogue (flags 0: plain store); out_f16: fp16 rather than bf16
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

// ------------------------------------------------------------ tiles
struct Tile {
    uint32_t m0, m_end, panel;
    const uint8_t *w;
    uint32_t gate_row;
};
template <int BN>
__device__ __forceinline__ Tile tile_of(const GemmParams &p, uint32_t t) {
    uint32_t s = 0;
    while (s + 1 < p.n_seg && t >= p.seg[s + 1].tile_begin) ++s;
    const uint32_t local = t - p.seg[s].tile_begin;
    return {p.seg[s].m_begin + (local / p.panels) * BN, p.seg[s].m_end, local % p.panels, p.seg[s].w,
            p.seg[s].gate_row};
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
                const uint8_t *panel = T.w + (uint64_t)(tc_in_bounds(T.panel < p.panels, p.status) ? T.panel : 0) *
                                                 p.kb * kChunk;
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
                build_table<TYPE, F16>(wc, tab, dt, ovf);
                bar_arrive(t_ready(tb));
                if (!(ok = bar_wait(t_ready(tb), tph, abort_flag, p.status))) break;
                for (uint32_t q = 0; q < 4; ++q) {
                    if (!(ok = bar_wait(st_empty(st), ph ^ 1, abort_flag, p.status))) break;
                    uint8_t *a = smem + L::a_off + st * L::a_stage;
                    {
                        const uint32_t r = 8 * dw + (lane >> 3) + 4 * ((lane >> 2) & 1);
                        dequant_task<TYPE, F16>(wc, tab, q, r, lane & 3, a);
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
            const bool f16 = p.epi.out_f16;
            if (p.epi.flags) {
                const EpiRow er = epi_row(p.epi, min(n, p.n - 1), T.gate_row);
#pragma unroll 1
                for (uint32_t c0 = 0; c0 < (uint32_t)BN; c0 += 32) {
                    uint32_t v[32];
                    tmem_ld32(taddr + c0, v);
                    epi_piece<OUT_F32>(p.epi, er, v, n < p.n, T.m0 + c0, T.m_end, p.y, p.ldy);
                }
            } else {
#pragma unroll 1
            for (uint32_t c0 = 0; c0 < (uint32_t)BN; c0 += 32) {
                uint32_t v[32];
                tmem_ld32(taddr + c0, v);
                if (n < p.n) {
#pragma unroll
                    for (uint32_t c = 0; c < 32; ++c) {
                        const uint32_t m = T.m0 + c0 + c;
                        if (m < T.m_end)
                            store_out_all(p.epi, p.y, (uint64_t)m * p.ldy + n, __uint_as_float(v[c]), OUT_F32, f16);
                    }
                }
            }
            }
            tc_fence_before();
            bar_arrive(acc_empty(acc));
            acc ^= 1;
            if (acc == 0) aph ^= 1;
        }
        if (p.epi.n_peer) __threadfence_system();   // publish peer-replica stores (see the pair kernel)
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

template <int TYPE, int BN, bool F16, bool OUT_F32>
cudaError_t launch_inst(const CUtensorMap &map, const GemmParams &p, int sm_count, cudaStream_t s) {
    using L = Layout<TYPE, BN>;
    auto kernel = gemm_kernel<TYPE, BN, F16, OUT_F32>;
    static DeviceCache cache;   // shared-memory opt-in, per device
    int unused = 0;
    cudaError_t e = per_device(cache, unused, [&](int &) {
        return cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)L::bytes);
    });
    if (e != cudaSuccess) return e;
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
                        int allow_pair, cudaStream_t s, const EpiView *epi, const SplitK *split) {
    if (n_seg == 0) return cudaSuccess;
    if (n_seg > (uint32_t)kMaxSeg) return cudaErrorInvalidValue;
    uint32_t max_rows = 0;
    for (uint32_t i = 0; i < n_seg; ++i) max_rows = max(max_rows, segs[i].m_end - segs[i].m_begin);
    const int bn = max_rows <= 64 ? 64 : max_rows <= 128 ? 128 : 256;
    if (bn == 256 && allow_pair)
        return launch_gemm_pair(segs, n_seg, x, m_total, k, y, ldy, out_dtype, stage_f16, sm_count, status, s, epi,
                                split);
    GemmParams p{};
    p.n_seg = n_seg;
    p.kb = segs[0].w.kb;
    p.panels = segs[0].w.panels;
    p.n = segs[0].w.n;
    p.y = y;
    p.ldy = ldy;
    p.status = status;
    if (epi) p.epi = *epi;
    p.epi.out_f16 = out_dtype == 1;
    uint32_t tiles = 0;
    for (uint32_t i = 0; i < n_seg; ++i) {
        p.seg[i] = {segs[i].m_begin, segs[i].m_end, tiles, segs[i].gate_row, segs[i].w.chunks};
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
    if (type == 13) {
        if (bn == 64) return launch_bn<13, 64>(map, p, stage_f16, out_f32, sm_count, s);
        if (bn == 128) return launch_bn<13, 128>(map, p, stage_f16, out_f32, sm_count, s);
        return launch_bn<13, 256>(map, p, stage_f16, out_f32, sm_count, s);
    }
    if (bn == 64) return launch_bn<14, 64>(map, p, stage_f16, out_f32, sm_count, s);
    if (bn == 128) return launch_bn<14, 128>(map, p, stage_f16, out_f32, sm_count, s);
    return launch_bn<14, 256>(map, p, stage_f16, out_f32, sm_count, s);
}

}  // namespace tc
