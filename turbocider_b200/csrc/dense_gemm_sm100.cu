// Linear on dense ("passthrough") weights on the 5th-generation tensor cores
// (sm_100a): Y[m, n] = sum_k X[m, k] * W[n, k], W the bf16 or fp16 copy of an
// F32 / F16 / BF16 / Q4_0 / Q4_1 / Q5_0 / Q5_1 / Q8_0 tensor made once at
// upload by the bit-exact raw decoder (dense_linear.cu).
//
// The K-quant kernels unpack their A operand into shared memory; here A is
// already dense, so the producer loads it with TMA: a [128 rows x 64 K] box
// with the 128-byte swizzle lands in exactly the layout the dequantisers
// write (8-row groups of 1024 bytes, 16-byte chunks XOR-swizzled by row), and
// the same smem descriptors drive tcgen05.mma.  One CTA per SM, persistent
// over the 128-row x BN-token tiles of one request segment:
//   warp 0     TMA producer: per 64-K stage one A box and one X box, both
//              completing on the stage's barrier (expect_tx);
//   warp 1     TMEM allocator and the single MMA-issuing thread (4 x K16 per
//              stage, M = 128, N = BN, fp32 accumulate);
//   warps 2-5  epilogue: tcgen05.ld of 32 tokens per row, the fused epilogue
//              of kq_epilogue.cuh, stores of Y.
// Two accumulators in TMEM let the epilogue of tile i overlap the main loop
// of tile i + 1.  K need not be a multiple of 64: boxes past K (and rows
// past N or past X) are zero-filled by TMA and add nothing.  Every wait is
// bounded; on timeout the kernel sets TC_STATUS_TIMEOUT, drains its copies
// and MMAs, frees TMEM and returns.  No multicast.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <cstring>

#include "kq_epilogue.cuh"
#include "kq_sm100.cuh"
#include "tc_internal.h"

namespace tc {
namespace {

constexpr int kThreads = 192;   // 6 warps
constexpr int kStages = 4;

struct DenseParams {
    uint32_t m_begin, m_end, n, kblocks, panels, n_tiles, gate_row;
    void *y;
    uint64_t ldy;
    uint32_t *status;
    EpiView epi;
};

template <int BN>
struct DenseLayout {
    static constexpr uint32_t a_stage = 128 * 128;   // 128 rows x 64 K x 2 B
    static constexpr uint32_t x_stage = BN * 128;
    static constexpr uint32_t a_off = 0, x_off = kStages * a_stage;
    static constexpr uint32_t bar_off = x_off + kStages * x_stage;
    // full[S] empty[S] acc_full[2] acc_empty[2] fin
    static constexpr uint32_t misc_off = bar_off + (2 * kStages + 5) * 8;
    static constexpr uint32_t bytes = misc_off + 16 + 1024;
    static constexpr uint32_t tmem_cols = 2 * BN < 32 ? 32 : 2 * BN;
    static_assert(bytes <= 232448, "shared memory per CTA exceeds the sm_100 limit");
};

template <int BN, bool F16, bool OUT_F32>
__global__ void __launch_bounds__(kThreads, 1)
    dense_gemm_kernel(const __grid_constant__ CUtensorMap amap, const __grid_constant__ CUtensorMap xmap,
                      const __grid_constant__ DenseParams p) {
    using L = DenseLayout<BN>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const uint32_t warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    const uint32_t bars = su32(smem + L::bar_off);
    auto full = [&](uint32_t i) { return bars + 8 * i; };
    auto empty = [&](uint32_t i) { return bars + 8 * (kStages + i); };
    auto acc_full = [&](uint32_t i) { return bars + 8 * (2 * kStages + i); };
    auto acc_empty = [&](uint32_t i) { return bars + 8 * (2 * kStages + 2 + i); };
    const uint32_t fin = bars + 8 * (2 * kStages + 4);
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + L::misc_off);
    volatile uint32_t *abort_flag = tmem_slot + 1;

    if (threadIdx.x == 0) {
        for (int i = 0; i < kStages; ++i) {
            bar_init(full(i), 1);
            bar_init(empty(i), 1);
        }
        for (int i = 0; i < 2; ++i) {
            bar_init(acc_full(i), 1);
            bar_init(acc_empty(i), 128);
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
        // ---------------------------------------------------- TMA producer
        if (lane == 0) {
            asm volatile("griddepcontrol.wait;" ::: "memory");   // X may come from the previous kernel
            uint32_t st = 0, ph = 0, last[kStages];
            bool used[kStages] = {}, ok = true;
            for (uint32_t t = blockIdx.x; ok && t < p.n_tiles; t += gridDim.x) {
                const int row0 = (int)((t % p.panels) * 128), m0 = (int)(p.m_begin + (t / p.panels) * BN);
                for (uint32_t kb = 0; ok && kb < p.kblocks; ++kb) {
                    if (!(ok = bar_wait(empty(st), ph ^ 1, abort_flag, p.status))) break;
                    bar_expect_tx(full(st), L::a_stage + L::x_stage);
                    tma_load_2d(su32(smem + L::a_off + st * L::a_stage), &amap, full(st), (int)(kb * 64), row0);
                    tma_load_2d(su32(smem + L::x_off + st * L::x_stage), &xmap, full(st), (int)(kb * 64), m0);
                    last[st] = ph;
                    used[st] = true;
                    if (++st == kStages) { st = 0; ph ^= 1; }
                }
            }
            for (int i = 0; i < kStages; ++i)   // every copy issued has landed before exit
                if (used[i]) bar_wait(full(i), last[i], abort_flag, p.status, false);
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
                for (uint32_t kb = 0; ok && kb < p.kblocks; ++kb) {
                    if (!(ok = bar_wait(full(st), ph, abort_flag, p.status))) break;
                    tc_fence_after();
                    const uint32_t a_addr = su32(smem + L::a_off + st * L::a_stage);
                    const uint32_t b_addr = su32(smem + L::x_off + st * L::x_stage);
#pragma unroll
                    for (uint32_t kk = 0; kk < 4; ++kk)
                        mma_f16(d_tmem, sw128_desc(a_addr + kk * 32), sw128_desc(b_addr + kk * 32), idesc,
                                (kb | kk) ? 1u : 0u);
                    mma_commit(empty(st));
                    if (++st == kStages) { st = 0; ph ^= 1; }
                }
                if (!ok) break;
                mma_commit(acc_full(acc));
                acc ^= 1;
                if (acc == 0) aph ^= 1;
            }
            mma_commit(fin);   // every MMA issued has completed before TMEM is freed
            bar_wait(fin, 0, abort_flag, p.status, false);
        }
        __syncwarp();
    } else {
        // ---------------------------------------------------- epilogue
        const uint32_t quad = warp & 3;   // TMEM lanes 32 quad .. +31 (warps 2-5 cover all four)
        uint32_t acc = 0, aph = 0;
        for (uint32_t t = blockIdx.x; t < p.n_tiles; t += gridDim.x) {
            const uint32_t row0 = (t % p.panels) * 128, m0 = p.m_begin + (t / p.panels) * BN;
            if (!__all_sync(0xffffffffu, bar_wait(acc_full(acc), aph, abort_flag, p.status))) break;
            tc_fence_after();
            const uint32_t n = row0 + quad * 32 + lane;
            const uint32_t taddr = tmem + ((quad * 32) << 16) + acc * BN;
            const bool f16 = p.epi.out_f16;
            const EpiRow er = p.epi.flags ? epi_row(p.epi, min(n, p.n - 1), p.gate_row) : EpiRow{0.f, 0.f, n, true};
#pragma unroll 1
            for (uint32_t c0 = 0; c0 < (uint32_t)BN; c0 += 32) {
                if (m0 + c0 >= p.m_end) break;
                uint32_t v[32];
                tmem_ld32(taddr + c0, v);
                if (p.epi.flags) {
                    epi_piece<OUT_F32>(p.epi, er, v, n < p.n, m0 + c0, p.m_end, p.y, p.ldy);
                } else if (n < p.n) {
#pragma unroll
                    for (uint32_t c = 0; c < 32; ++c) {
                        const uint32_t m = m0 + c0 + c;
                        if (m < p.m_end)
                            store_out_all(p.epi, p.y, (uint64_t)m * p.ldy + n, __uint_as_float(v[c]), OUT_F32, f16);
                    }
                }
            }
            tc_fence_before();
            bar_arrive(acc_empty(acc));
            acc ^= 1;
            if (acc == 0) aph ^= 1;
        }
        if (p.epi.n_peer) __threadfence_system();   // publish peer-replica stores
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(L::tmem_cols));
    }
}

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

// A K-major [rows x cols] 16-bit matrix (row pitch `ld` elements) as a map of
// 64-column x `box_rows` boxes with the 128-byte swizzle.
bool encode_k_major(CUtensorMap *map, const void *base, uint64_t cols, uint64_t rows, uint64_t ld, uint32_t box_rows,
                    bool f16) {
    auto enc = encode_fn();
    if (!enc || (reinterpret_cast<uintptr_t>(base) & 15u) || (ld * 2) % 16) return false;
    const cuuint64_t dims[2] = {cols, rows};
    const cuuint64_t strides[1] = {ld * 2};
    const cuuint32_t box[2] = {64u, box_rows};
    const cuuint32_t estr[2] = {1u, 1u};
    return enc(map, f16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2,
               const_cast<void *>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
               CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int BN, bool F16, bool OUT_F32>
cudaError_t launch_inst(const CUtensorMap &amap, const CUtensorMap &xmap, const DenseParams &p, int sm_count,
                        cudaStream_t s) {
    using L = DenseLayout<BN>;
    auto kernel = dense_gemm_kernel<BN, F16, OUT_F32>;
    static DeviceCache cache;   // shared-memory opt-in, per device
    int unused = 0;
    cudaError_t e = per_device(cache, unused, [&](int &) {
        return cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)L::bytes);
    });
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(p.n_tiles < (uint32_t)sm_count ? p.n_tiles : (uint32_t)sm_count);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = L::bytes;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, amap, xmap, p);
}

template <int BN>
cudaError_t launch_bn(const CUtensorMap &amap, const CUtensorMap &xmap, const DenseParams &p, bool f16, bool out_f32,
                      int sm, cudaStream_t s) {
    if (f16) return out_f32 ? launch_inst<BN, true, true>(amap, xmap, p, sm, s) : launch_inst<BN, true, false>(amap, xmap, p, sm, s);
    return out_f32 ? launch_inst<BN, false, true>(amap, xmap, p, sm, s) : launch_inst<BN, false, false>(amap, xmap, p, sm, s);
}

}  // namespace

cudaError_t launch_dense_gemm(const uint16_t *w, uint64_t ldw, uint32_t n, const uint16_t *x, uint64_t ldx,
                              uint64_t m_total, uint64_t k, uint32_t m_begin, uint32_t m_end, uint32_t gate_row,
                              void *y, uint64_t ldy, int out_dtype, int f16, int sm_count, uint32_t *status,
                              const EpiView *epi, cudaStream_t s) {
    if (m_end <= m_begin || !n) return cudaSuccess;
    const uint32_t rows = m_end - m_begin;
    const int bn = rows <= 64 ? 64 : rows <= 128 ? 128 : 256;
    DenseParams p{};
    p.m_begin = m_begin;
    p.m_end = m_end;
    p.n = n;
    p.kblocks = (uint32_t)((k + 63) / 64);
    p.panels = (n + 127) / 128;
    p.n_tiles = (rows + bn - 1) / bn * p.panels;
    p.gate_row = gate_row;
    p.y = y;
    p.ldy = ldy;
    p.status = status;
    if (epi) p.epi = *epi;
    p.epi.out_f16 = out_dtype == 1;
    CUtensorMap amap, xmap;
    if (!encode_k_major(&amap, w, k, n, ldw, 128, f16) ||
        !encode_k_major(&xmap, x, k, m_total, ldx, (uint32_t)bn, f16))
        return cudaErrorInvalidValue;
    const bool out_f32 = out_dtype == 0;
    if (bn == 64) return launch_bn<64>(amap, xmap, p, f16, out_f32, sm_count, s);
    if (bn == 128) return launch_bn<128>(amap, xmap, p, f16, out_f32, sm_count, s);
    return launch_bn<256>(amap, xmap, p, f16, out_f32, sm_count, s);
}

}  // namespace tc
