#ifndef TURBOCIDER_CUDA_H
#define TURBOCIDER_CUDA_H
/*
 * TurboCider CUDA backend for B200 (sm_100a): GGUF K-quant (Q4_K / Q5_K / Q6_K)
 * dequantise-and-matmul, exported as a plain C ABI.
 *
 * This backend sits beside the reference's native backends.  Its operator
 * replaces the quantised branch of Weights::project
 * (reference native/backends/mlx.cpp:626-690, reached from linear() at
 * native/backends/mlx.cpp:1624), and its dequantiser is bit-exact to the
 * reference CPU decoder decode_cpu_into (native/core/gguf_decode.cpp:433-445).
 *
 * Conventions (mirroring bindings/c/include/turbocider/turbocider.h:7-12 and
 * the op-level probe ABI tests/native/gguf_core_probe.cpp:31-65):
 *   - every int-returning call returns TC_CUDA_OK (0), TC_CUDA_FAIL (1) or
 *     TC_CUDA_CANCELLED (2); the reason for a failure is available from
 *     tc_cuda_last_error() on the calling thread;
 *   - no C++ exception crosses this boundary and no kernel traps: device-side
 *     faults (nonfinite scales, fp16 overflow, pipeline timeouts) set bits in
 *     the context's status word, read with tc_cuda_status();
 *   - device pointers are caller-owned unless returned by this API; `stream`
 *     is a cudaStream_t passed as void* (NULL = the legacy default stream);
 *     every launch is asynchronous on that stream;
 *   - calls on one context are serialised by the caller.
 *
 * Ratios: Q4_K = 256 weights / 144 bytes, Q5_K = 256 / 176, Q6_K = 256 / 210
 * (reference native/core/gguf_directory.hpp:21-26).
 */
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define TC_CUDA_ABI_VERSION 2u

enum { TC_CUDA_OK = 0, TC_CUDA_FAIL = 1, TC_CUDA_CANCELLED = 2 };

/* GGML on-disk type ids (reference native/core/gguf_directory.hpp:21-26).
 * The quantised linear takes the K-quants; tc_cuda_decode takes every
 * registered type. */
enum {
    TC_GGML_F32 = 0, TC_GGML_F16 = 1, TC_GGML_Q4_0 = 2, TC_GGML_Q4_1 = 3, TC_GGML_Q5_0 = 6, TC_GGML_Q5_1 = 7,
    TC_GGML_Q8_0 = 8, TC_GGML_Q4_K = 12, TC_GGML_Q5_K = 13, TC_GGML_Q6_K = 14, TC_GGML_BF16 = 30
};

/* Target / output dtypes; same numbering as tc::gguf::DecodeDType
 * (reference native/core/gguf_decode.hpp:18). */
enum { TC_DTYPE_F32 = 0, TC_DTYPE_F16 = 1, TC_DTYPE_BF16 = 2 };

/* Staging precision of the dequantised weight inside the tensor-core GEMM,
 * and the type of X:
 *   TC_STAGE_BF16     X bf16, W staged bf16 (rel-L2 ~1.7e-3 vs an fp32 decode);
 *   TC_STAGE_F16      X bf16, converted to fp16 into the context workspace,
 *                     W staged fp16 (rel-L2 ~2e-4);
 *   TC_STAGE_F16_X16  X already fp16 (the reference's GGUF execution runs fp16
 *                     activations), W staged fp16, no conversion pass; every
 *                     segment takes the tensor-core GEMM. */
enum { TC_STAGE_BF16 = 0, TC_STAGE_F16 = 1, TC_STAGE_F16_X16 = 2 };

/* Status-word bits (tc_cuda_status). */
enum {
    TC_STATUS_NONFINITE_SCALE = 1u << 0, /* a d/dmin master scale is inf/nan   */
    TC_STATUS_F16_OVERFLOW    = 1u << 1, /* a value does not fit fp16          */
    TC_STATUS_TIMEOUT         = 1u << 2, /* a bounded pipeline wait gave up    */
    TC_STATUS_GEOMETRY        = 1u << 3, /* a kernel saw an impossible tile    */
    TC_STATUS_BF16_OVERFLOW   = 1u << 4, /* a value rounds past the bf16 range */
    TC_STATUS_BOUNDS          = 1u << 5  /* bounds-checked build only: an index
                                            outside its buffer (access skipped) */
};

typedef struct tc_cuda_ctx tc_cuda_ctx;
typedef struct tc_cuda_weight tc_cuda_weight;

/* ABI version of this library (cf. tc_abi_version, turbocider.h:24). */
uint32_t tc_cuda_abi_version(void);

/* Reason for the last failure on this thread; "" after a success
 * (cf. tc_gguf_test_error, gguf_core_probe.cpp:31). */
const char *tc_cuda_last_error(void);

/* Create a context on `device`.  The context owns the device status word,
 * reusable workspaces (split-K partials, fp16 staging of X) and the side
 * streams of tc_cuda_peer_push; it never takes over the caller's streams. */
int tc_cuda_init(int device, tc_cuda_ctx **ctx);
void tc_cuda_free(tc_cuda_ctx *ctx);

/* Read (and, if clear != 0, reset) the device status word.  Synchronises the
 * device.  Replaces the reference's DecodeError throw sites
 * (gguf_decode.cpp:43, :393, :401-404) for work done on the GPU. */
int tc_cuda_status(tc_cuda_ctx *ctx, uint32_t *bits, int clear);

/* Upload a GGUF tensor [N rows, K columns] (ne[0] = K contiguous) of type
 * Q4_K, Q5_K or Q6_K from host memory and keep it resident in HBM in the
 * kernels' panel layout.  `raw_host` holds whole rows, row pitch K/256*block_bytes, as
 * in the GGUF payload.  Rows [n_begin, n_begin + n_count) are uploaded (an
 * N-column shard); n_count = 0 means all rows.  The blocks' bytes are moved,
 * never re-encoded; every d/dmin is checked finite (the reference rejects
 * such blocks at decode time, gguf_decode.cpp:78, :92).  Synchronous.
 * Replaces the MLX-affine import of GgufPackedBank::load_candidate
 * (reference native/runtime/streaming/gguf_packed_bank.cpp:374-517). */
int tc_cuda_weight_upload(tc_cuda_ctx *ctx, uint32_t ggml_type, uint64_t n, uint64_t k,
                          const void *raw_host, uint64_t raw_bytes, uint64_t n_begin,
                          uint64_t n_count, tc_cuda_weight **weight);

/* Upload the two halves of a SwiGLU projection as ONE weight for the fused
 * TC_EPI_SWIGLU epilogue of tc_cuda_qlinear_ex: `gate_raw` and `up_raw` are
 * raw GGUF matrices [f, k] of the same type (two tensors such as Z-Image's
 * w1 / w3, or the two halves of a gate_up tensor [2f, k], up_raw = gate_raw +
 * f rows, as in reference native/models/qwen21/transformer.cpp:971-976).
 * Output columns [col_begin, col_begin + col_count) (col_count = 0: to the
 * end; a multiple of 8 unless it reaches f) are taken from both halves and
 * interleaved in groups of 8 rows (8 gate rows, then the same 8 up rows), so
 * that one tile holds both factors of each output.  The weight has
 * 2 * col_count rows; tc_cuda_dequant shows them in that interleaved order.
 * Synchronous; checks every d/dmin finite. */
int tc_cuda_weight_upload_glu(tc_cuda_ctx *ctx, uint32_t ggml_type, uint64_t f, uint64_t k,
                              const void *gate_raw, const void *up_raw, uint64_t raw_bytes_each,
                              uint64_t col_begin, uint64_t col_count, tc_cuda_weight **weight);

/* As tc_cuda_weight_upload, but the raw rows are already in device memory
 * (e.g. a staging buffer the caller filled with cudaMemcpyAsync) and the re-layout is
 * enqueued on `stream` without synchronising.  `weight` must have been
 * created by tc_cuda_weight_create with the same type and shape. */
int tc_cuda_weight_create(tc_cuda_ctx *ctx, uint32_t ggml_type, uint64_t n, uint64_t k,
                          tc_cuda_weight **weight);
int tc_cuda_weight_fill_device(tc_cuda_ctx *ctx, tc_cuda_weight *weight, const void *raw_device,
                               uint64_t raw_bytes, void *stream);
void tc_cuda_weight_free(tc_cuda_weight *weight);

/* Streaming from pinned host memory (cf. the reference's streamed GGUF
 * weights: GgufPackedBank / GgufWeightPager, native/runtime/streaming/).
 * tc_relayout_host re-lays rows [n_begin, n_begin + n_count) (0 = to the end)
 * of a raw GGUF matrix [n, k] into the panel layout of an n_count-row weight,
 * on `threads` CPU threads, checking every d/dmin is finite; tc_panel_bytes
 * is the size of that layout.  `cancel` (NULL: not cancellable) is a
 * caller-owned flag polled once per panel chunk: nonzero stops the work and
 * the call returns TC_CUDA_CANCELLED ("generation cancelled"; the panels are
 * then incomplete), as the reference polls its cancel flag once per block
 * (gguf_decode.cpp:44-47, :344).  tc_cuda_weight_copy_panels then copies panel
 * bytes (pinned host or device memory, exactly weight_info's device_bytes)
 * into a weight made by tc_cuda_weight_create, asynchronously on `stream`,
 * with no kernel (so it overlaps a running GEMM). */
uint64_t tc_panel_bytes(uint32_t ggml_type, uint64_t n, uint64_t k);
int tc_relayout_host(uint32_t ggml_type, const void *raw, uint64_t raw_bytes, uint64_t n, uint64_t k,
                     uint64_t n_begin, uint64_t n_count, void *panels, uint64_t panel_bytes, int threads,
                     const volatile int32_t *cancel);
int tc_cuda_weight_copy_panels(tc_cuda_ctx *ctx, tc_cuda_weight *weight, const void *panels, uint64_t bytes,
                               void *stream);

/* Shape queries of an uploaded weight. */
int tc_cuda_weight_info(const tc_cuda_weight *weight, uint32_t *ggml_type, uint64_t *n,
                        uint64_t *k, uint64_t *device_bytes);

/* Dequantise an uploaded weight to a dense row-major [n, k] matrix with leading
 * dimension `ld` elements, dtype TC_DTYPE_*.  Bit-exact to decode_cpu_into
 * with the same target dtype (gguf_decode.cpp:433-445, write_value :112-116). */
int tc_cuda_dequant(tc_cuda_ctx *ctx, const tc_cuda_weight *weight, int dtype, void *dst,
                    uint64_t ld, void *stream);

/* Device mirror of decode_cpu_into (gguf_decode.cpp:433-445 and the probe ABI
 * tc_gguf_test_decode, gguf_core_probe.cpp:32-50): decode the slice
 * [row_begin, +rows) x [column_begin, +columns) of a raw GGUF matrix of any
 * registered type (F32, F16, BF16, Q4_0, Q4_1, Q5_0, Q5_1, Q8_0, Q4_K, Q5_K,
 * Q6_K) in device memory into a strided device target (byte strides, no
 * alignment needed).  Geometry is validated on the host with the reference's
 * rules and messages; value errors (nonfinite input or scale, fp16 / bf16
 * overflow) are reported in the status word. */
int tc_cuda_decode(tc_cuda_ctx *ctx, uint32_t ggml_type, const void *source, uint64_t source_bytes,
                   uint64_t source_rows, uint64_t source_columns, uint64_t row_begin,
                   uint64_t rows, uint64_t column_begin, uint64_t columns, int dtype,
                   void *target, uint64_t target_bytes, uint64_t row_stride,
                   uint64_t column_stride, void *stream);

/* Device mirror of decode_cpu_gather (gguf_decode.cpp:446-465, declared at
 * gguf_decode.hpp:60-62; the probe ABI's gather mode, gguf_core_probe.cpp:44):
 * bounded row gather for embedding-style lookups -- target row r is source row
 * row_indices[r] (device array of n_indices uint64, duplicates and order
 * kept), columns [column_begin, +columns), any registered type, strided
 * target as tc_cuda_decode.  Host checks: the reference's validate() rules
 * with one row per index, then "gather indices overlap target".  Each index
 * is checked on the device: one past source_rows sets TC_STATUS_GEOMETRY
 * (reported as "gather row out of bounds") and its target row is not
 * written. */
int tc_cuda_decode_gather(tc_cuda_ctx *ctx, uint32_t ggml_type, const void *source, uint64_t source_bytes,
                          uint64_t source_rows, uint64_t source_columns, const uint64_t *row_indices,
                          uint64_t n_indices, uint64_t column_begin, uint64_t columns, int dtype, void *target,
                          uint64_t target_bytes, uint64_t row_stride, uint64_t column_stride, void *stream);

/* Quantised linear Y[M, N] = X[M, K] * W^T (fp32 accumulate) -- the operator
 * behind Weights::project (reference native/backends/mlx.cpp:668-679).
 *   X        bf16 [M, K] row-major, device (fp16 with TC_STAGE_F16_X16);
 *            M = seg_offsets[n_seg].
 *   Y        [M, N] row-major, device, dtype out_dtype (TC_DTYPE_BF16,
 *            TC_DTYPE_F16 or TC_DTYPE_F32); row stride ldy elements (0 = N).
 *   weights  n_weights uploaded weights with identical N, K;
 *   seg_offsets  int32 [n_seg + 1] host array, 0 = seg_offsets[0] <= ... :
 *            rows of X that belong to request segment s (ragged packing of
 *            several requests along M);
 *   seg_weight   int32 [n_seg] host array: which weight segment s uses (e.g.
 *            image vs text stream);  NULL = weight 0 for every segment.
 * Dispatch: the warp GEMV for segments with at most 16 rows, the tcgen05
 * tensor-core GEMM otherwise (2-CTA 256 x 256 tiles once a segment has more
 * than 128 rows).  `stage` selects the GEMM's operand precision and X's type
 * (TC_STAGE_*). */
int tc_cuda_qlinear(tc_cuda_ctx *ctx, const tc_cuda_weight *const *weights, uint32_t n_weights,
                    const int32_t *seg_offsets, const int32_t *seg_weight, uint32_t n_seg,
                    const void *x, void *y, uint64_t ldy, int out_dtype, int stage, void *stream);

/* Fused epilogue of tc_cuda_qlinear_ex, applied in fp32 to each accumulator
 * value before the one rounding to out_dtype, in this order:
 *   TC_EPI_BIAS          t = acc + bias[row]             (mlx.cpp:687-688)
 *   TC_EPI_GELU_TANH     t = 0.5 t (1 + tanh(sqrt(2/pi) (t + 0.044715 t^3)))
 *   TC_EPI_GELU_ERF      t = 0.5 t (1 + erf(t / sqrt(2)))
 *   TC_EPI_SWIGLU        t = silu(t_gate) * t_up        (transformer.cpp:971-976;
 *                        the weight must come from tc_cuda_weight_upload_glu;
 *                        the output has col_count = rows / 2 columns)
 *   TC_EPI_GATE_RESIDUAL y = residual[m][c] + gate[g][c] * t, g the gate row
 *                        of m's segment (the AdaLN gated residual
 *                        hidden + gate * proj, transformer.cpp:950, :980;
 *                        the caller applies any tanh to the gate vector).
 * bias: f32 [rows] in the weight's row order; for a SwiGLU weight the gate
 *   bias of output column c is bias[c] and its up bias bias[bias_up_offset + c].
 * gate: f32 [n_gate_rows][ld_gate]; seg_gate: host int32 [n_seg] gate row of
 *   each segment (NULL: segment s uses row s).
 * residual: [M][ld_residual] in out_dtype; may be Y itself (in-place update:
 *   each element is read and then written by the same thread).
 * The reference rounds after the product and again after each following
 * operation; here every step is fp32 with one rounding at the end. */
enum {
    TC_EPI_BIAS = 1u << 0,
    TC_EPI_GELU_TANH = 1u << 1,
    TC_EPI_GELU_ERF = 1u << 2,
    TC_EPI_SWIGLU = 1u << 3,
    TC_EPI_GATE_RESIDUAL = 1u << 4
};
typedef struct tc_epilogue {
    uint32_t flags;
    uint32_t n_gate_rows;
    const float *bias;
    uint64_t bias_up_offset;
    const float *gate;
    uint64_t ld_gate;
    const int32_t *seg_gate;
    const void *residual;
    uint64_t ld_residual;
} tc_epilogue;

/* tc_cuda_qlinear with a fused epilogue (NULL = none, the same as
 * tc_cuda_qlinear) and any of the three output dtypes (TC_DTYPE_F16 is the
 * reference's output dtype for fp16 activations: mlx.cpp:668-679 returns
 * X's dtype).  For a SwiGLU weight Y has rows/2 columns and ldy counts those. */
int tc_cuda_qlinear_ex(tc_cuda_ctx *ctx, const tc_cuda_weight *const *weights, uint32_t n_weights,
                       const int32_t *seg_offsets, const int32_t *seg_weight, uint32_t n_seg,
                       const void *x, void *y, uint64_t ldy, int out_dtype, int stage,
                       const tc_epilogue *epilogue, void *stream);

/* ------------------------------------------------ multi-GPU: fused all-gather
 * N-column sharding over the GPUs of one box (one process per GPU): rank r
 * holds output columns [c_r, c_r + n_r) of every weight (tc_cuda_weight_upload
 * with n_begin / n_count) and every rank needs the full Y[M, N].  Instead of
 * a separate all-gather after each linear, tc_cuda_qlinear_gather writes each
 * output element into this rank's Y and into every peer's replica of Y over
 * NVLink, from the GEMM's epilogue, tile by tile:
 *   y       this rank's columns of its own Y: full_Y + c_r, row stride ldy = N;
 *   peer_y  the same columns of the other ranks' Y buffers, as mapped in this
 *           process (tc_cuda_peer_open), n_peer <= 7.
 * All destinations must have identical layout.  Afterwards
 * tc_cuda_peer_barrier(epoch) on every rank makes every rank wait (on its
 * stream) until all ranks have finished: then every Y is complete.
 *
 * Buffers reachable from peers come from tc_cuda_peer_alloc (device memory
 * plus a 64-byte CUDA IPC handle to send to the other ranks, e.g. through
 * torch.distributed) and tc_cuda_peer_open (map another rank's handle).
 * tc_cuda_peer_barrier: flags[r] = rank r's flag array (n_ranks uint32, zeroed,
 * from tc_cuda_peer_alloc; flags[rank] the local one); epoch = 1, 2, ... per
 * call; waits at most timeout_us (0: one second) and then sets
 * TC_STATUS_TIMEOUT instead of hanging. */
int tc_cuda_qlinear_gather(tc_cuda_ctx *ctx, const tc_cuda_weight *const *weights, uint32_t n_weights,
                           const int32_t *seg_offsets, const int32_t *seg_weight, uint32_t n_seg,
                           const void *x, void *y, uint64_t ldy, int out_dtype, int stage,
                           const tc_epilogue *epilogue, void *const *peer_y, uint32_t n_peer, void *stream);
int tc_cuda_peer_alloc(tc_cuda_ctx *ctx, uint64_t bytes, void **ptr, void *ipc_handle_64b);
int tc_cuda_peer_open(tc_cuda_ctx *ctx, const void *ipc_handle_64b, void **ptr);
int tc_cuda_peer_close(tc_cuda_ctx *ctx, void *ptr);
int tc_cuda_peer_free(tc_cuda_ctx *ctx, void *ptr);
int tc_cuda_peer_barrier(tc_cuda_ctx *ctx, uint32_t *const *flags, uint32_t n_ranks, uint32_t rank,
                         uint32_t epoch, uint32_t timeout_us, void *stream);

/* All-gather by a push after the GEMM instead of the GEMM epilogue: after a
 * plain tc_cuda_qlinear has written this rank's shard (e.g. its slot of a
 * shard-major Y[g][M][N/g], the layout of an NCCL all-gather), push the shard
 * into the same place of every peer's buffer, enqueued on `stream` (a side
 * stream, so the transfer overlaps the next linear).  rows x width_bytes
 * region, row pitches src_pitch / dst_pitch (ignored for rows == 1; equal to
 * the width: one linear copy per peer).  Completion on every rank:
 * tc_cuda_peer_barrier on the same stream.  Like the fused gather, this
 * replaces the ncclAllGather that follows each N-sharded linear; the
 * reference runs on one device and has no counterpart.  By default the copy
 * engines do it, back to back on `stream` (no SMs taken); see
 * tc_cuda_set_push_fanout and tc_cuda_set_push_kernel for the other forms. */
int tc_cuda_peer_push(tc_cuda_ctx *ctx, const void *src, void *const *dst, uint32_t n_dst, uint64_t width_bytes,
                      uint64_t rows, uint64_t src_pitch, uint64_t dst_pitch, void *stream);
/* streams >= 2: tc_cuda_peer_push spreads the destinations' copies over that
 * many side streams owned by the context (destination i on stream
 * i % streams; created on first use), forked from `stream` and joined back
 * into it -- to `stream` still one ordered step.  0 or 1 (the default): back
 * to back on `stream`.  Measured on 8 B200s with one stream per peer the
 * concurrent copies contend (369 GB/s received per GPU against 535 GB/s back
 * to back). */
int tc_cuda_set_push_fanout(tc_cuda_ctx *ctx, int streams);
/* ctas > 0: tc_cuda_peer_push moves the bytes with a kernel of `ctas`
 * 128-thread blocks on `stream` (each 16-byte vector read once, stored to
 * every destination by the SMs over NVLink; small blocks that fit beside a
 * resident GEMM CTA) whenever every address, the width and the pitches are
 * multiples of 16 bytes; otherwise, and with 0 (the default), by the copy
 * engines.  Measured on B200s beside the N-sharded GEMM stack: faster than
 * the copy engines at 8 GPUs (296 blocks: 632 against 535 GB/s received per
 * GPU), slower at 2 and 4, where its stores compete with the GEMM. */
int tc_cuda_set_push_kernel(tc_cuda_ctx *ctx, int ctas);

/* Batched small-M linear: Y_i[m, N_i] = X[m, K] * W_i^T for n_weights
 * (1..64) weights that share K and X (e.g. every block's AdaLN modulation
 * linear, which all take the timestep embedding), m = 1..16 rows of bf16 X.
 * One GEMV launch per weight type streams all of them, so a call moves the
 * sum of the weights' bytes instead of paying a launch per weight.  ys[i] is
 * the output of weight i (f32, f16 or bf16, row stride ldys[i], NULL / 0 =
 * N_i).  SwiGLU weights are not accepted here. */
int tc_cuda_qlinear_batched(tc_cuda_ctx *ctx, const tc_cuda_weight *const *weights, uint32_t n_weights,
                            const void *x, uint32_t m, void *const *ys, const uint64_t *ldys, int out_dtype,
                            void *stream);

/* Force one kernel family for a call (testing and benchmarking):
 *   0 automatic, 1 warp GEMV (any M), 2 tensor-core GEMM (any M),
 *   3 tensor-core GEMM with one-CTA tiles only (no 2-CTA pairs). */
int tc_cuda_set_path(tc_cuda_ctx *ctx, int path);

/* Which kernel family a one-segment call with m rows of X on `weight` takes
 * under the context's current settings, and for the 2-CTA GEMM into how many
 * K shares each tile is split (1: none; more when the call has too few tiles
 * to occupy the GPU's SM pairs: each share's fp32 partial product goes to the
 * context workspace and a reduce kernel adds them in order).  No launch; for
 * tests and for sizing work.  No counterpart in the reference. */
enum { TC_KERNEL_GEMV = 1, TC_KERNEL_GEMM_PAIR = 2, TC_KERNEL_GEMM_1CTA = 3, TC_KERNEL_DENSE = 4 };
int tc_cuda_qlinear_plan(tc_cuda_ctx *ctx, const tc_cuda_weight *weight, uint32_t m, int stage, uint32_t *kernel,
                         uint32_t *ksplit);

/* Cap the SMs the tensor-core GEMM's persistent grid may occupy (0 = all, the
 * default).  The GEMM holds one CTA per SM for its whole run; with N-column
 * sharding a communication kernel (the all-gather of the previous linear's
 * output) runs beside it, and it needs free SMs to make progress. */
int tc_cuda_set_sm_limit(tc_cuda_ctx *ctx, int sms);

/* Allocation-free small-M quantised linear.  No counterpart in the reference.
 * For callers that must not allocate device memory while they run a linear
 * (a pre-sized memory arena, code under an allocator callback, a loop that
 * cannot take cudaMalloc's implicit synchronisation): computes
 * Y[m, N] = X[m, K] * W^T for 1 <= m <= 16 with the split-K GEMV of
 * tc_cuda_qlinear, whose scratch (K-slice partials, per-tile counters, status
 * word) here lives in an 8 MiB file-scope device array instead of a cudaMalloc'd
 * context workspace.  No context argument; X bf16 [m, K] (16-byte aligned), Y
 * f32, f16 or bf16 with row stride ldy (0 = N), all device memory, enqueued on
 * `stream`.  The first call on a device looks up the array's address and
 * clears its status word, synchronously (make it before any stream capture);
 * a call needs 4.6 MiB of it plus 4 bytes per 16 weight rows, and a
 * size check rejects anything over 8 MiB; every call shares the array, so
 * calls that may overlap on the GPU must be serialised by the caller.
 * Device-side errors (TC_STATUS_* bits) accumulate in the array's status word
 * until read with tc_cuda_small_static_status.  Allocates nothing. */
int tc_cuda_qlinear_small_static(const tc_cuda_weight *weight, const void *x, uint32_t m, void *y, uint64_t ldy,
                                 int out_dtype, void *stream);
/* Status word of tc_cuda_qlinear_small_static on `device` (the counterpart of
 * tc_cuda_status for that entry point, which has no context): synchronises
 * the device, returns the accumulated TC_STATUS_* bits and, if clear != 0,
 * resets them.  No counterpart in the reference.  Allocates nothing. */
int tc_cuda_small_static_status(int device, uint32_t *bits, int clear);

/* ---------------------------------------------------------------- GGUF files
 * Directory parser and payload reader for GGUF v2/v3 containers, with the
 * reference's acceptance rules and error texts (read_directory,
 * native/core/gguf_directory.hpp:199-271): magic and version, metadata with
 * parse limits, tensor table (rank <= 4, block-aligned rows, known GGML type),
 * general.alignment, payload bounds and overlap.  Host only, no GPU work. */
typedef struct tc_gguf tc_gguf;

/* Open and parse `path`; `limit` is NULL (or a test hook shrinking one parse
 * limit: "retained", "directory", "string", "count", "array").  The file
 * stays open for tc_gguf_read until tc_gguf_close. */
int tc_gguf_open(const char *path, const char *limit, tc_gguf **file);
void tc_gguf_close(tc_gguf *file);
int tc_gguf_info(const tc_gguf *file, uint32_t *version, uint32_t *alignment, uint64_t *n_tensors,
                 uint64_t *data_offset, uint64_t *n_metadata);
/* Tensor `index`: NUL-terminated name (name_cap bytes available), GGML type,
 * rank, dims[4] (dims[0] = contiguous extent K; unused dims = 1), absolute
 * file offset and payload bytes (cf. TensorDescriptor, gguf_directory.hpp:63-71). */
int tc_gguf_tensor(const tc_gguf *file, uint64_t index, char *name, uint64_t name_cap, uint32_t *ggml_type,
                   uint32_t *rank, uint64_t *dims, uint64_t *file_offset, uint64_t *bytes);
int tc_gguf_find(const tc_gguf *file, const char *name, uint64_t *index);
/* Metadata entry `key`: GGUF value type, raw unsigned bits, sign-extended
 * value, float value, string text (type 8), element count (type 9 arrays). */
int tc_gguf_meta(const tc_gguf *file, const char *key, uint32_t *type, uint64_t *u, int64_t *i, double *f,
                 char *text, uint64_t text_cap, uint64_t *array_count);
/* Read rows [row_begin, row_begin + rows) of a tensor's payload (raw GGUF
 * blocks, row pitch dims[0] / block_elements * block_bytes) into host memory
 * (pinned memory lets the following upload run at full PCIe rate), in preads
 * of at most 8 MiB; `cancel` (NULL: not cancellable) is polled before each:
 * nonzero returns TC_CUDA_CANCELLED ("generation cancelled"). */
int tc_gguf_read(const tc_gguf *file, uint64_t index, uint64_t row_begin, uint64_t rows, void *dst,
                 uint64_t dst_bytes, const volatile int32_t *cancel);

/* Streaming load of a K-quant tensor (rows [n_begin, +n_count), 0 = to the
 * end: an N-column shard) from the file into a new weight in HBM, replacing
 * GgufPackedBank::load_candidate's read / decode / publish loop
 * (native/runtime/streaming/gguf_packed_bank.cpp:393-452) and its read-ahead
 * worker (native/runtime/streaming/read_ahead_worker.hpp:21-70).  Chunks of
 * whole 128-row panels, about chunk_bytes each (0: 8 MiB), flow through two
 * pinned host slots and two device slots: a worker thread preads chunk i + 1
 * while chunk i is copied to HBM and re-laid into the weight's panels on the
 * GPU.  `cancel` (NULL: not cancellable) is polled before every chunk and
 * between preads.  Synchronous; every d/dmin is checked finite.  On failure
 * or cancellation (TC_CUDA_CANCELLED) no weight is returned (the one being
 * filled is freed).  The staging slots are the context's, allocated by the
 * first load and reused.  stats (may be NULL): bytes loaded, chunks, wall
 * seconds, seconds spent in pread, seconds the loading thread waited for
 * reads. */
typedef struct tc_gguf_load_stats {
    uint64_t bytes, chunks;
    double seconds, read_seconds, wait_seconds;
} tc_gguf_load_stats;
int tc_cuda_weight_load_gguf(tc_cuda_ctx *ctx, const tc_gguf *file, uint64_t index, uint64_t n_begin,
                             uint64_t n_count, uint64_t chunk_bytes, const volatile int32_t *cancel,
                             tc_cuda_weight **weight, tc_gguf_load_stats *stats);
/* Validate a split set (validate_split_set, gguf_directory.hpp:273-304). */
int tc_gguf_validate_split(const tc_gguf *const *shards, uint32_t n);

/* Host-side GGUF K-quant quantiser (not in the reference, which ships no
 * encoder): quantise a row-major fp32 [rows, cols] matrix (cols % 256 == 0) to
 * raw GGUF blocks of `ggml_type` (Q4_K or Q6_K) using `threads` CPU threads.
 * Used to build synthetic weights; decode(quantise(W)) approximates W. */
int tc_quantize(uint32_t ggml_type, const float *w, uint64_t rows, uint64_t cols, void *blocks,
                uint64_t blocks_bytes, int threads);

#ifdef __cplusplus
}
#endif
#endif
