// Internal host-side declarations shared by the C-ABI layer and the kernel
// launchers.  Nothing here crosses the public ABI.
#pragma once
#include <cstdint>
#include <mutex>
#include <string>
#include <cuda_runtime.h>

struct tc_cuda_ctx {
    int device = 0;
    int sm_count = 0;
    uint32_t *status = nullptr;      // device status word (TC_STATUS_* bits)
    void *workspace = nullptr;       // grows on demand: fp16 copy of X
    size_t workspace_bytes = 0;
    float *gemv_partials = nullptr;  // GEMV K-slice partials (grows on demand)
    size_t gemv_partials_floats = 0;
    uint32_t *gemv_counters = nullptr;  // per-16-row-tile arrival counters, kept at 0
    size_t gemv_counters_n = 0;
    int path = 0;                    // 0 auto, 1 GEMV, 2 GEMM, 3 GEMM with one-CTA tiles only
    int sm_limit = 0;                // SMs the tensor-core GEMM may occupy (0 = all)
    uint16_t *dense_x = nullptr;     // X with a 16-byte row pitch for the dense GEMM (grows on demand)
    size_t dense_x_bytes = 0;
    // Copy-engine all-gather (tc_cuda_peer_push): by default the copies to
    // the peers go back to back on the caller's stream; push_fanout = k >= 2
    // spreads them over k side streams (created on first use), forked from
    // and joined back into the caller's stream.  push_ctas > 0 runs the
    // pushes as one kernel of that many 128-thread blocks instead (the SMs
    // store to the peers over NVLink).
    int push_fanout = 0;
    int push_ctas = 0;
    cudaStream_t push_stream[8] = {};
    cudaEvent_t push_fork = nullptr, push_join[8] = {};
    float *split_ws = nullptr;       // split-K partial products of the tensor-core GEMM
    size_t split_ws_floats = 0;
    // Streaming GGUF loader (tc_cuda_weight_load_gguf): two pinned host and
    // two device staging slots (grow-only), its stream and per-slot events.
    void *load_host[2] = {}, *load_dev[2] = {};
    size_t load_slot_bytes = 0;
    cudaStream_t load_stream = nullptr;
    cudaEvent_t load_freed[2] = {};
};

struct tc_cuda_weight {
    int device = 0;
    uint32_t type = 0;               // 12 = Q4_K, 13 = Q5_K, 14 = Q6_K
    uint32_t glu = 0;                // rows are 8-row gate / up groups (tc_cuda_weight_upload_glu)
    uint64_t n = 0, k = 0;
    uint32_t kb = 0;                 // super-blocks per row, K / 256
    uint32_t panels = 0;             // ceil(N / 128)
    uint8_t *chunks = nullptr;       // panel layout, panels * kb chunks (K-quants)
    uint64_t bytes = 0;
    // Dense weights (F32 / F16 / BF16 / Q4_0 / Q4_1 / Q5_0 / Q5_1 / Q8_0): raw
    // GGUF rows plus row-major bf16 and fp16 copies (fp16 null when a value
    // does not fit fp16).
    uint8_t *raw = nullptr;
    uint64_t raw_row_bytes = 0;
    uint16_t *dense_bf16 = nullptr, *dense_f16 = nullptr;
    uint64_t dense_ld = 0;           // row pitch (elements) of the dense copies: K rounded up to 8
};

namespace tc {

// Sets the thread-local message returned by tc_cuda_last_error().
void set_last_error(const std::string &reason);

// Per-device launch set-up (a kernel's shared-memory opt-in, its occupancy):
// cudaFuncSetAttribute acts on the current device only, so the result is
// cached per device ordinal, and the cache is shared by concurrent callers.
// Each instantiation of a launch template owns one cache.
constexpr int kMaxDevices = 64;
struct DeviceCache {
    std::mutex mu;
    bool done[kMaxDevices] = {};
    int value[kMaxDevices] = {};
};
// Runs setup(int &value) once per device (the current one) and returns the
// cached value in `out`; a failed set-up is retried on the next call.
template <class F>
cudaError_t per_device(DeviceCache &c, int &out, F &&setup) {
    int dev = -1;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
    std::lock_guard<std::mutex> lock(c.mu);
    if (!c.done[dev]) {
        int v = 0;
        if ((e = setup(v)) != cudaSuccess) return e;
        c.value[dev] = v;
        c.done[dev] = true;
    }
    out = c.value[dev];
    return cudaSuccess;
}

// Geometry handed to the kernels for one weight.
struct WeightView {
    const uint8_t *chunks;
    uint32_t type, kb, panels;
    uint32_t n;
};

// One ragged request segment of a quantised linear.
struct SegmentView {
    uint32_t m_begin, m_end;         // rows of X / Y
    WeightView w;
    uint32_t gate_row = 0;           // row of the epilogue's gate vectors
};

constexpr uint32_t kMaxPeers = 8;    // ranks of one N-sharded linear, this one included

// Fused epilogue (device pointers), flags = TC_EPI_* bits; flags == 0 is a
// plain store.  out_f16 selects fp16 over bf16 for 16-bit outputs.
struct EpiView {
    uint32_t flags = 0, out_f16 = 0;
    const float *bias = nullptr;     // by weight row; SwiGLU: gate c at c, up c at bias_up + c
    uint64_t bias_up = 0;
    const float *gate = nullptr;     // [rows][ld_gate], over output columns
    uint64_t ld_gate = 0;
    const void *res = nullptr;       // [M][ld_res] in the output dtype
    uint64_t ld_res = 0;
    // Output replication (N-column sharding): every value stored to Y is also
    // stored at the same offset from each peer[i] (other ranks' Y buffers,
    // mapped into this process), so the all-gather happens in the epilogue.
    uint32_t n_peer = 0;
    void *peer[kMaxPeers - 1] = {};
    // Bounds-checked builds (TC_BOUNDS_CHECK): elements addressable from Y's
    // base (0: not checked) and the status word that records a violation.
    uint64_t y_limit = 0;
    uint32_t *status = nullptr;
};

// Bounds checks of the -DTC_BOUNDS_CHECK build (libturbocider_cuda_checked.so,
// the substitute for compute-sanitizer, which this GPU pool does not offer):
// tc_in_bounds(cond, status) records TC_STATUS_BOUNDS when cond is false and
// returns cond, so the caller skips (stores) or clamps (reads) the access
// instead of faulting; in the normal build it is `true` and costs nothing.
#ifdef TC_BOUNDS_CHECK
#ifdef __CUDACC__
__device__ __forceinline__ bool tc_in_bounds(bool cond, uint32_t *status) {
    if (!cond && status) atomicOr(status, 1u << 5);
    return cond;
}
#endif
#else
#define tc_in_bounds(cond, status) true
#endif

// glu_c > 0: the source holds glu_c gate rows then glu_c up rows, and panel
// row 16 g + i takes gate row 8 g + i (i < 8) or up row 8 g + i - 8.
cudaError_t launch_relayout(uint32_t type, const uint8_t *raw, uint64_t n, uint32_t kb,
                            uint8_t *chunks, uint32_t panels, uint32_t *status, cudaStream_t s,
                            uint64_t glu_c = 0);
cudaError_t launch_dequant_panel(const WeightView &w, int dtype, void *dst, uint64_t ld,
                                 uint32_t *status, cudaStream_t s);
// gather != nullptr: target row r decodes source row gather[r] (device array,
// checked against source_rows; TC_STATUS_GEOMETRY for an index past it).
// dst_bytes: the target's size (0: not checked by bounds-checked builds).
cudaError_t launch_decode_raw(uint32_t type, const uint8_t *src, uint64_t row_bytes,
                              uint64_t row_begin, uint64_t rows, uint64_t column_begin,
                              uint64_t columns, int dtype, uint8_t *dst, uint64_t row_stride,
                              uint64_t column_stride, uint32_t *status, cudaStream_t s,
                              const uint64_t *gather = nullptr, uint64_t source_rows = 0, uint64_t dst_bytes = 0);
// Small-M GEMV: a CTA covers a tile of 16 or 64 weight rows (one or four
// row warps) and one K slice; n_slices CTAs per tile.  With n_slices > 1 the
// kernel needs `partials` (at most kGemvPartialFloats floats) and one zeroed
// uint32 counter per tile (at most gemv_counters(n) per weight); both are
// left as found (counters back to 0).
constexpr uint32_t kGemvMaxCtas = 148u * 4u;   // a K split aims at four CTAs per SM
constexpr size_t kGemvPartialFloats = (size_t)kGemvMaxCtas * 2 * 4 * 256;   // slice x tile < 2 kGemvMaxCtas, 4 warps x 16 x 16
inline uint32_t gemv_counters(uint64_t n) { return (uint32_t)((n + 15) / 16); }
struct GemvSplit {
    uint32_t kb_per_slice = 0, n_slices = 1;
    float *partials = nullptr;
    uint32_t *counters = nullptr;
    uint32_t *status = nullptr;
};
GemvSplit gemv_split_tiles(uint32_t tiles, uint32_t kb, uint32_t row_warps);
// Several weights with the same K, type and X in one GEMV launch.
constexpr uint32_t kMaxGemvBatch = 64;
struct GemvEntry {
    const uint8_t *chunks;
    void *y;
    uint64_t ldy;
    uint32_t n, tile_begin;   // rows; first tile of this weight in the launch (set by the launcher)
};
struct GemvBatch {
    uint32_t n_entries, kb;
    GemvEntry e[kMaxGemvBatch];
    EpiView epi;          // fused epilogue of every entry (flags 0: plain store)
    uint32_t gate_row;    // gate vector row of the launch's segment
};
// out_dtype: TC_DTYPE_F32 / F16 / BF16.  epi (optional) applies to every
// entry, with gate row `gate_row`.
cudaError_t launch_gemv_batch(const GemvBatch &bt, uint32_t type, uint32_t m_begin, uint32_t m, const uint16_t *x,
                              uint64_t k, int out_dtype, const GemvSplit &sp, cudaStream_t s,
                              const EpiView *epi = nullptr, uint32_t gate_row = 0);
cudaError_t launch_gemv(const SegmentView &seg, const uint16_t *x, uint64_t k, void *y,
                        uint64_t ldy, int out_dtype, const GemvSplit &split, cudaStream_t s,
                        const EpiView *epi = nullptr);
cudaError_t launch_x_to_f16(const uint16_t *x, uint16_t *x16, uint64_t count, uint32_t *status,
                            cudaStream_t s);
// Split-K of the 2-CTA GEMM when a call has too few 256 x 256 tiles to fill
// the GPU (e.g. 256 tokens x 3072 rows: 12 tiles for 74 SM pairs): each tile
// becomes ksplit work units over equal shares of the super-block columns,
// each unit stores its fp32 partial product in `ws` ([ksplit][m_total][n]),
// and a reduce kernel adds the shares in split order (deterministic) and
// applies the fused epilogue.
struct SplitK {
    uint32_t ksplit = 1;
    float *ws = nullptr;
};
// ksplit for these segments on `sm_count` SMs (1: no split); the 2-CTA path
// only (a segment longer than 128 rows).
uint32_t pair_ksplit(const SegmentView *segs, uint32_t n_seg, int sm_count);
inline size_t pair_split_floats(uint32_t ksplit, uint64_t m_total, uint32_t n) {
    return ksplit > 1 ? (size_t)ksplit * m_total * n : 0;
}
// Tensor-core GEMM over a list of segments that share type, N and K.  Uses
// 2-CTA (cta_group::2) 256 x 256 tiles when a segment has more than 128 rows
// and allow_pair is set, one-CTA 128 x {64, 128, 256} tiles otherwise.
cudaError_t launch_gemm(const SegmentView *segs, uint32_t n_seg, const uint16_t *x,
                        uint64_t m_total, uint64_t k, void *y, uint64_t ldy, int out_dtype,
                        int stage_f16, int sm_count, uint32_t *status, int allow_pair, cudaStream_t s,
                        const EpiView *epi = nullptr, const SplitK *split = nullptr);
cudaError_t launch_gemm_pair(const SegmentView *segs, uint32_t n_seg, const uint16_t *x,
                             uint64_t m_total, uint64_t k, void *y, uint64_t ldy, int out_dtype,
                             int stage_f16, int sm_count, uint32_t *status, cudaStream_t s,
                             const EpiView *epi = nullptr, const SplitK *split = nullptr);
// Y rows [m_begin, +rows) = epilogue(sum over s < ksplit of part[s][m][.]) in
// split order; n_w = the weight's rows (SwiGLU: gate / up interleaved).
cudaError_t launch_split_reduce(const float *part, uint32_t ksplit, uint64_t stride, uint32_t n_w, uint32_t m_begin,
                                uint32_t rows, const EpiView &e, uint32_t gate_row, void *y, uint64_t ldy,
                                int out_dtype, cudaStream_t s);

// Dense (passthrough) weights, dense_linear.cu.
bool dense_type(uint32_t type);
// Y rows [m_begin, m_end) = X * W^T on the tensor cores (dense_gemm_sm100.cu):
// W [n, k] 16-bit, row pitch ldw; X [m_total, k] 16-bit, row pitch ldx (both
// pitches multiples of 8 elements, bases 16-byte aligned); f16: fp16
// operands, else bf16; fused epilogue and peer stores as the K-quant GEMMs.
cudaError_t launch_dense_gemm(const uint16_t *w, uint64_t ldw, uint32_t n, const uint16_t *x, uint64_t ldx,
                              uint64_t m_total, uint64_t k, uint32_t m_begin, uint32_t m_end, uint32_t gate_row,
                              void *y, uint64_t ldy, int out_dtype, int f16, int sm_count, uint32_t *status,
                              const EpiView *epi, cudaStream_t s);
// Copy X [m, k] (row pitch k) into out [m, ld] (ld >= k, zeros past k).
cudaError_t launch_pad_rows(const uint16_t *x, uint16_t *out, uint64_t m, uint64_t k, uint64_t ld, cudaStream_t s);

}  // namespace tc
