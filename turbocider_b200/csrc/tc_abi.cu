// C-ABI layer of the TurboCider CUDA backend (declared in
// include/turbocider_cuda.h).  Validates arguments with the reference's
// rules and messages, owns device buffers, and dispatches the kernels.
// No exception crosses the boundary; errors are returned as status codes
// with a thread-local message (as tests/native/gguf_core_probe.cpp:10-50 of
// the reference does for its op-level probe ABI).
#include <algorithm>
#include <cstdio>
#include <cstring>
#include <new>
#include <string>
#include <vector>

#include "../../include/turbocider_cuda.h"
#include "kq_format.cuh"
#include "tc_internal.h"

namespace {

thread_local std::string g_error;

int fail(const std::string &reason) {
    g_error = reason;
    return TC_CUDA_FAIL;
}
int ok() {
    g_error.clear();
    return TC_CUDA_OK;
}
int cuda_fail(const char *what, cudaError_t e) {
    return fail(std::string(what) + ": " + cudaGetErrorString(e));
}

// Runs a body with the context's device current, restoring the caller's.
struct DeviceGuard {
    int previous = -1;
    explicit DeviceGuard(int device) {
        if (cudaGetDevice(&previous) != cudaSuccess) previous = -1;
        if (previous != device) cudaSetDevice(device);
    }
    ~DeviceGuard() {
        int now = -1;
        if (previous >= 0 && cudaGetDevice(&now) == cudaSuccess && now != previous) cudaSetDevice(previous);
    }
};

bool supported_type(uint32_t type) {
    return type == TC_GGML_Q4_K || type == TC_GGML_Q5_K || type == TC_GGML_Q6_K;
}

tc::WeightView view_of(const tc_cuda_weight *w) {
    return {w->chunks, w->type, w->kb, w->panels, (uint32_t)w->n};
}

// Grows the context workspace (never shrinks; freed with the context).
int ensure_workspace(tc_cuda_ctx *ctx, size_t bytes) {
    if (ctx->workspace_bytes >= bytes) return TC_CUDA_OK;
    if (ctx->workspace) cudaFree(ctx->workspace);
    ctx->workspace = nullptr;
    ctx->workspace_bytes = 0;
    cudaError_t e = cudaMalloc(&ctx->workspace, bytes);
    if (e != cudaSuccess) return cuda_fail("workspace allocation", e);
    ctx->workspace_bytes = bytes;
    return TC_CUDA_OK;
}

// Grows the GEMV split-K workspace: partials and per-tile counters.  The
// counters are zeroed once here; every complete kernel leaves them at zero.
int ensure_gemv_workspace(tc_cuda_ctx *ctx, size_t floats, size_t counters) {
    if (floats > ctx->gemv_partials_floats) {
        if (ctx->gemv_partials) cudaFree(ctx->gemv_partials);
        ctx->gemv_partials = nullptr;
        ctx->gemv_partials_floats = 0;
        cudaError_t e = cudaMalloc(&ctx->gemv_partials, floats * sizeof(float));
        if (e != cudaSuccess) return cuda_fail("GEMV workspace allocation", e);
        ctx->gemv_partials_floats = floats;
    }
    if (counters > ctx->gemv_counters_n) {
        if (ctx->gemv_counters) cudaFree(ctx->gemv_counters);
        ctx->gemv_counters = nullptr;
        ctx->gemv_counters_n = 0;
        cudaError_t e = cudaMalloc(&ctx->gemv_counters, counters * sizeof(uint32_t));
        if (e == cudaSuccess) e = cudaMemset(ctx->gemv_counters, 0, counters * sizeof(uint32_t));
        if (e != cudaSuccess) return cuda_fail("GEMV counter allocation", e);
        ctx->gemv_counters_n = counters;
    }
    return TC_CUDA_OK;
}

}  // namespace

void tc::set_last_error(const std::string &reason) { g_error = reason; }

extern "C" {

uint32_t tc_cuda_abi_version(void) { return TC_CUDA_ABI_VERSION; }

const char *tc_cuda_last_error(void) { return g_error.c_str(); }

int tc_cuda_init(int device, tc_cuda_ctx **out) {
    if (!out) return fail("null context out-parameter");
    *out = nullptr;
    int count = 0;
    cudaError_t e = cudaGetDeviceCount(&count);
    if (e != cudaSuccess || count == 0) return fail("no CUDA device available (the TurboCider CUDA backend has no CPU fallback)");
    if (device < 0 || device >= count) return fail("invalid CUDA device ordinal");
    cudaDeviceProp prop{};
    if ((e = cudaGetDeviceProperties(&prop, device)) != cudaSuccess) return cuda_fail("device query", e);
    if (prop.major != 10) return fail("the TurboCider CUDA backend targets sm_100a (B200); found sm_" +
                                      std::to_string(prop.major) + std::to_string(prop.minor));
    DeviceGuard guard(device);
    auto *ctx = new (std::nothrow) tc_cuda_ctx;
    if (!ctx) return fail("out of host memory");
    ctx->device = device;
    ctx->sm_count = prop.multiProcessorCount;
    if ((e = cudaMalloc(&ctx->status, 4 * sizeof(uint32_t))) != cudaSuccess) {
        delete ctx;
        return cuda_fail("status word allocation", e);
    }
    if ((e = cudaMemset(ctx->status, 0, 4 * sizeof(uint32_t))) != cudaSuccess) {
        cudaFree(ctx->status);
        delete ctx;
        return cuda_fail("status word init", e);
    }
    *out = ctx;
    return ok();
}

void tc_cuda_free(tc_cuda_ctx *ctx) {
    if (!ctx) return;
    DeviceGuard guard(ctx->device);
    if (ctx->workspace) cudaFree(ctx->workspace);
    if (ctx->gemv_partials) cudaFree(ctx->gemv_partials);
    if (ctx->gemv_counters) cudaFree(ctx->gemv_counters);
    if (ctx->dense_x) cudaFree(ctx->dense_x);
    if (ctx->split_ws) cudaFree(ctx->split_ws);
    for (int i = 0; i < 8; ++i) {
        if (ctx->push_stream[i]) cudaStreamDestroy(ctx->push_stream[i]);
        if (ctx->push_join[i]) cudaEventDestroy(ctx->push_join[i]);
    }
    if (ctx->push_fork) cudaEventDestroy(ctx->push_fork);
    for (int i = 0; i < 2; ++i) {
        if (ctx->load_host[i]) cudaFreeHost(ctx->load_host[i]);
        if (ctx->load_dev[i]) cudaFree(ctx->load_dev[i]);
        if (ctx->load_freed[i]) cudaEventDestroy(ctx->load_freed[i]);
    }
    if (ctx->load_stream) cudaStreamDestroy(ctx->load_stream);
    if (ctx->status) cudaFree(ctx->status);
    delete ctx;
}

int tc_cuda_status(tc_cuda_ctx *ctx, uint32_t *bits, int clear) {
    if (!ctx || !bits) return fail("null context or out-parameter");
    DeviceGuard guard(ctx->device);
    cudaError_t e = cudaDeviceSynchronize();
    if (e != cudaSuccess) return cuda_fail("device synchronise", e);
    if ((e = cudaMemcpy(bits, ctx->status, sizeof(uint32_t), cudaMemcpyDeviceToHost)) != cudaSuccess)
        return cuda_fail("status read", e);
    if (clear && (e = cudaMemset(ctx->status, 0, sizeof(uint32_t))) != cudaSuccess) return cuda_fail("status clear", e);
    return ok();
}

int tc_cuda_weight_create(tc_cuda_ctx *ctx, uint32_t type, uint64_t n, uint64_t k, tc_cuda_weight **out) {
    if (!ctx || !out) return fail("null context or out-parameter");
    *out = nullptr;
    if (!supported_type(type)) return fail("gguf_decode: unsupported tensor type");
    if (!n || !k || k % tc::kBlockWeights) return fail("invalid source geometry");
    if (n > (1ull << 31) || k > (1ull << 31)) return fail("weight shape exceeds the 2^31 limit");
    DeviceGuard guard(ctx->device);
    auto *w = new (std::nothrow) tc_cuda_weight;
    if (!w) return fail("out of host memory");
    w->device = ctx->device;
    w->type = type;
    w->n = n;
    w->k = k;
    w->kb = (uint32_t)(k / tc::kBlockWeights);
    w->panels = (uint32_t)((n + tc::kPanelRows - 1) / tc::kPanelRows);
    w->bytes = (uint64_t)w->panels * w->kb * tc::chunk_bytes(type);
    cudaError_t e = cudaMalloc(&w->chunks, w->bytes);
    if (e != cudaSuccess) {
        delete w;
        return cuda_fail("weight allocation", e);
    }
    *out = w;
    return ok();
}

int tc_cuda_weight_fill_device(tc_cuda_ctx *ctx, tc_cuda_weight *w, const void *raw, uint64_t raw_bytes,
                               void *stream) {
    if (!ctx || !w || !raw) return fail("null context, weight or source");
    const uint64_t need = w->n * w->kb * tc::block_bytes(w->type);
    if (raw_bytes < need) return fail("packed source too short");
    DeviceGuard guard(ctx->device);
    cudaError_t e = tc::launch_relayout(w->type, static_cast<const uint8_t *>(raw), w->n, w->kb, w->chunks, w->panels,
                                        ctx->status, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail("re-layout launch", e);
    return ok();
}

}  // extern "C"

namespace {
// Copy `n_src` host row ranges of `bytes_each` into one device staging buffer,
// re-lay them into w's panels (glu_c > 0: gate then up rows, interleaved) and
// check every scale finite.  Frees w on failure; synchronous.
int upload_rows(tc_cuda_ctx *ctx, tc_cuda_weight *w, const uint8_t *const *src, int n_src, uint64_t bytes_each,
                uint64_t glu_c, tc_cuda_weight **out) {
    DeviceGuard guard(ctx->device);
    void *staging = nullptr;
    cudaError_t e = cudaMalloc(&staging, bytes_each * n_src);
    for (int i = 0; i < n_src && e == cudaSuccess; ++i)
        e = cudaMemcpy(static_cast<uint8_t *>(staging) + i * bytes_each, src[i], bytes_each, cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = cudaMemset(ctx->status + 1, 0, sizeof(uint32_t));
    if (e == cudaSuccess)
        e = tc::launch_relayout(w->type, static_cast<const uint8_t *>(staging), w->n, w->kb, w->chunks, w->panels,
                                ctx->status + 1, nullptr, glu_c);
    uint32_t bits = 0;
    if (e == cudaSuccess) e = cudaMemcpy(&bits, ctx->status + 1, sizeof(uint32_t), cudaMemcpyDeviceToHost);
    if (staging) cudaFree(staging);
    if (e != cudaSuccess) {
        tc_cuda_weight_free(w);
        return cuda_fail("weight upload", e);
    }
    if (bits & TC_STATUS_NONFINITE_SCALE) {
        tc_cuda_weight_free(w);
        return fail("nonfinite weight/scale or conversion overflow");
    }
    *out = w;
    return ok();
}
// Dense (passthrough) weight: raw rows [n_begin, +n_count) resident, plus bf16
// and (when every value fits) fp16 row-major copies decoded on the device.
int upload_dense(tc_cuda_ctx *ctx, uint32_t type, uint64_t n, uint64_t k, const void *raw_host, uint64_t raw_bytes,
                 uint64_t n_begin, uint64_t n_count, tc_cuda_weight **out) {
    const uint32_t el = tc::type_elements(type);
    if (!n || !k || k % el) return fail("invalid source geometry");
    if (n_count == 0) n_count = n - std::min(n_begin, n);
    if (n_begin >= n || n_count > n - n_begin) return fail("row slice out of bounds");
    if (n_count > (1ull << 31) || k > (1ull << 31)) return fail("weight shape exceeds the 2^31 limit");
    const uint64_t row_bytes = k / el * tc::type_bytes(type);
    if (raw_bytes / row_bytes < n) return fail("packed source too short");
    DeviceGuard guard(ctx->device);
    auto *w = new (std::nothrow) tc_cuda_weight;
    if (!w) return fail("out of host memory");
    w->device = ctx->device;
    w->type = type;
    w->n = n_count;
    w->k = k;
    w->raw_row_bytes = row_bytes;
    w->dense_ld = (k + 7) / 8 * 8;   // 16-byte row pitch for TMA
    const uint64_t elems = n_count * w->dense_ld;
    w->bytes = n_count * row_bytes + 4 * elems;
    cudaError_t e = cudaMalloc(&w->raw, n_count * row_bytes);
    if (e == cudaSuccess) e = cudaMalloc(&w->dense_bf16, elems * 2);
    if (e == cudaSuccess) e = cudaMalloc(&w->dense_f16, elems * 2);
    if (e == cudaSuccess) e = cudaMemset(w->dense_bf16, 0, elems * 2);   // pad columns stay zero
    if (e == cudaSuccess) e = cudaMemset(w->dense_f16, 0, elems * 2);
    if (e == cudaSuccess)
        e = cudaMemcpy(w->raw, static_cast<const uint8_t *>(raw_host) + n_begin * row_bytes, n_count * row_bytes,
                       cudaMemcpyHostToDevice);
    uint32_t bits[2] = {0, 0};
    for (int dt = 2; dt >= 1 && e == cudaSuccess; --dt) {   // bf16 first: its errors reject the weight
        uint16_t *dst = dt == 2 ? w->dense_bf16 : w->dense_f16;
        e = cudaMemset(ctx->status + 1, 0, sizeof(uint32_t));
        if (e == cudaSuccess)
            e = tc::launch_decode_raw(type, w->raw, row_bytes, 0, n_count, 0, k, dt, reinterpret_cast<uint8_t *>(dst),
                                      w->dense_ld * 2, 2, ctx->status + 1, nullptr);
        if (e == cudaSuccess) e = cudaMemcpy(&bits[dt - 1], ctx->status + 1, sizeof(uint32_t), cudaMemcpyDeviceToHost);
    }
    if (e != cudaSuccess) {
        tc_cuda_weight_free(w);
        return cuda_fail("weight upload", e);
    }
    if (bits[1] & TC_STATUS_NONFINITE_SCALE) {
        tc_cuda_weight_free(w);
        return fail("nonfinite weight/scale or conversion overflow");
    }
    if (bits[1] & TC_STATUS_BF16_OVERFLOW) {
        tc_cuda_weight_free(w);
        return fail("BF16 conversion overflow");
    }
    if (bits[0] & TC_STATUS_F16_OVERFLOW) {   // fp16 staging is refused for this weight
        cudaFree(w->dense_f16);
        w->dense_f16 = nullptr;
    }
    *out = w;
    return ok();
}

}  // namespace

extern "C" {

int tc_cuda_weight_upload(tc_cuda_ctx *ctx, uint32_t type, uint64_t n, uint64_t k, const void *raw_host,
                          uint64_t raw_bytes, uint64_t n_begin, uint64_t n_count, tc_cuda_weight **out) {
    if (!ctx || !out || !raw_host) return fail("null context, source or out-parameter");
    *out = nullptr;
    if (tc::dense_type(type)) return upload_dense(ctx, type, n, k, raw_host, raw_bytes, n_begin, n_count, out);
    if (!supported_type(type)) return fail("gguf_decode: unsupported tensor type");
    if (!n || !k || k % tc::kBlockWeights) return fail("invalid source geometry");
    if (n_count == 0) n_count = n - std::min(n_begin, n);
    if (n_begin >= n || n_count > n - n_begin) return fail("row slice out of bounds");
    const uint64_t row_bytes = k / tc::kBlockWeights * tc::block_bytes(type);
    if (raw_bytes / row_bytes < n) return fail("packed source too short");
    tc_cuda_weight *w = nullptr;
    int rc = tc_cuda_weight_create(ctx, type, n_count, k, &w);
    if (rc) return rc;
    const uint8_t *src = static_cast<const uint8_t *>(raw_host) + n_begin * row_bytes;
    return upload_rows(ctx, w, &src, 1, n_count * row_bytes, 0, out);
}

int tc_cuda_weight_upload_glu(tc_cuda_ctx *ctx, uint32_t type, uint64_t f, uint64_t k, const void *gate_raw,
                              const void *up_raw, uint64_t raw_bytes_each, uint64_t col_begin, uint64_t col_count,
                              tc_cuda_weight **out) {
    if (!ctx || !out || !gate_raw || !up_raw) return fail("null context, source or out-parameter");
    *out = nullptr;
    if (!supported_type(type)) return fail("SwiGLU weights take the K-quant types");
    if (!f || !k || k % tc::kBlockWeights) return fail("invalid source geometry");
    if (col_count == 0) col_count = f - std::min(col_begin, f);
    if (col_begin >= f || col_count > f - col_begin) return fail("row slice out of bounds");
    if (col_count % 8) return fail("SwiGLU column count must be a multiple of 8");
    const uint64_t row_bytes = k / tc::kBlockWeights * tc::block_bytes(type);
    if (raw_bytes_each / row_bytes < f) return fail("packed source too short");
    tc_cuda_weight *w = nullptr;
    int rc = tc_cuda_weight_create(ctx, type, 2 * col_count, k, &w);
    if (rc) return rc;
    w->glu = 1;
    const uint8_t *src[2] = {static_cast<const uint8_t *>(gate_raw) + col_begin * row_bytes,
                             static_cast<const uint8_t *>(up_raw) + col_begin * row_bytes};
    return upload_rows(ctx, w, src, 2, col_count * row_bytes, col_count, out);
}

void tc_cuda_weight_free(tc_cuda_weight *w) {
    if (!w) return;
    DeviceGuard guard(w->device);
    if (w->chunks) cudaFree(w->chunks);
    if (w->raw) cudaFree(w->raw);
    if (w->dense_bf16) cudaFree(w->dense_bf16);
    if (w->dense_f16) cudaFree(w->dense_f16);
    delete w;
}

int tc_cuda_weight_info(const tc_cuda_weight *w, uint32_t *type, uint64_t *n, uint64_t *k, uint64_t *bytes) {
    if (!w) return fail("null weight");
    if (type) *type = w->type;
    if (n) *n = w->n;
    if (k) *k = w->k;
    if (bytes) *bytes = w->bytes;
    return ok();
}

int tc_cuda_dequant(tc_cuda_ctx *ctx, const tc_cuda_weight *w, int dtype, void *dst, uint64_t ld, void *stream) {
    if (!ctx || !w || !dst) return fail("null context, weight or target");
    if (dtype < 0 || dtype > 2) return fail("gguf_decode: invalid target dtype");
    if (ld < w->k) return fail("invalid/overlapping row stride");
    DeviceGuard guard(ctx->device);
    if (w->raw) {
        const uint64_t item = dtype == TC_DTYPE_F32 ? 4 : 2;
        cudaError_t e = tc::launch_decode_raw(w->type, w->raw, w->raw_row_bytes, 0, w->n, 0, w->k, dtype,
                                              static_cast<uint8_t *>(dst), ld * item, item, ctx->status,
                                              static_cast<cudaStream_t>(stream));
        if (e != cudaSuccess) return cuda_fail("dequant launch", e);
        return ok();
    }
    cudaError_t e = tc::launch_dequant_panel(view_of(w), dtype, dst, ld, ctx->status, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail("dequant launch", e);
    return ok();
}

}  // extern "C"

namespace {
// The reference's validate() (native/core/gguf_decode.cpp:160-183): source and
// target geometry for `rows` decoded rows, same checks, order and messages.
// Returns 0 and the source row pitch / target extent, or fails.
int validate_decode(uint32_t type, const void *source, uint64_t source_bytes, uint64_t source_rows,
                    uint64_t source_columns, uint64_t rows, uint64_t column_begin, uint64_t columns, int dtype,
                    const void *target, uint64_t target_bytes, uint64_t row_stride, uint64_t column_stride,
                    uint64_t *row_bytes_out, uint64_t *extent_out) {
    const uint32_t elements = tc::type_elements(type);
    if (!elements) return fail("gguf_decode: unsupported tensor type");
    if (!source || !target) return fail("null source/target storage");
    if (!source_rows || !source_columns || source_columns % elements) return fail("invalid source geometry");
    if (!rows || !columns || column_begin > source_columns || columns > source_columns - column_begin)
        return fail("invalid decode slice");
    const uint64_t row_bytes = source_columns / elements * tc::type_bytes(type);
    if (source_rows > UINT64_MAX / row_bytes) return fail("gguf_decode: multiplication overflow");
    if (source_rows * row_bytes > source_bytes) return fail("packed source too short");
    if (dtype < 0 || dtype > 2) return fail("gguf_decode: invalid target dtype");
    const uint64_t item = dtype == TC_DTYPE_F32 ? 4 : 2;
    if (column_stride < item) return fail("invalid/overlapping column stride");
    if (columns - 1 > (UINT64_MAX - item) / column_stride) return fail("gguf_decode: multiplication overflow");
    const uint64_t row_extent = (columns - 1) * column_stride + item;
    if (row_stride < row_extent) return fail("invalid/overlapping row stride");
    if (rows - 1 > (UINT64_MAX - row_extent) / row_stride) return fail("gguf_decode: multiplication overflow");
    const uint64_t extent = (rows - 1) * row_stride + row_extent;
    if (extent > target_bytes) return fail("decode target too short");
    const uintptr_t s0 = reinterpret_cast<uintptr_t>(source), t0 = reinterpret_cast<uintptr_t>(target);
    const uint64_t source_extent = source_rows * row_bytes;
    if (!(s0 + source_extent <= t0 || t0 + extent <= s0)) return fail("packed source overlaps target");
    *row_bytes_out = row_bytes;
    *extent_out = extent;
    return TC_CUDA_OK;
}
}  // namespace

extern "C" {

// Geometry rules and messages of the reference's validate() and
// decode_cpu_into() (native/core/gguf_decode.cpp:160-183, :433-438).
int tc_cuda_decode(tc_cuda_ctx *ctx, uint32_t type, const void *source, uint64_t source_bytes, uint64_t source_rows,
                   uint64_t source_columns, uint64_t row_begin, uint64_t rows, uint64_t column_begin,
                   uint64_t columns, int dtype, void *target, uint64_t target_bytes, uint64_t row_stride,
                   uint64_t column_stride, void *stream) {
    if (!ctx) return fail("null context");
    if (row_begin > source_rows || rows > source_rows - row_begin) return fail("row slice out of bounds");
    uint64_t row_bytes = 0, extent = 0;
    int rc = validate_decode(type, source, source_bytes, source_rows, source_columns, rows, column_begin, columns,
                             dtype, target, target_bytes, row_stride, column_stride, &row_bytes, &extent);
    if (rc) return rc;
    DeviceGuard guard(ctx->device);
    cudaError_t e = tc::launch_decode_raw(type, static_cast<const uint8_t *>(source), row_bytes, row_begin, rows,
                                          column_begin, columns, dtype, static_cast<uint8_t *>(target), row_stride,
                                          column_stride, ctx->status, static_cast<cudaStream_t>(stream), nullptr, 0,
                                          target_bytes);
    if (e != cudaSuccess) return cuda_fail("decode launch", e);
    return ok();
}

// decode_cpu_gather (native/core/gguf_decode.cpp:446-465): validate() with
// one row per index, then the indices must not overlap the target; every
// index is checked on the device (an index past the matrix sets
// TC_STATUS_GEOMETRY and its row is not written -- the reference rejects the
// call before decoding; its contract already has callers discard a target
// that a failed call touched).
int tc_cuda_decode_gather(tc_cuda_ctx *ctx, uint32_t type, const void *source, uint64_t source_bytes,
                          uint64_t source_rows, uint64_t source_columns, const uint64_t *row_indices,
                          uint64_t n_indices, uint64_t column_begin, uint64_t columns, int dtype, void *target,
                          uint64_t target_bytes, uint64_t row_stride, uint64_t column_stride, void *stream) {
    if (!ctx) return fail("null context");
    uint64_t row_bytes = 0, extent = 0;
    int rc = validate_decode(type, source, source_bytes, source_rows, source_columns, n_indices, column_begin, columns,
                             dtype, target, target_bytes, row_stride, column_stride, &row_bytes, &extent);
    if (rc) return rc;
    if (!row_indices) return fail("null gather indices");
    const uintptr_t i0 = reinterpret_cast<uintptr_t>(row_indices), t0 = reinterpret_cast<uintptr_t>(target);
    if (n_indices > UINT64_MAX / sizeof(uint64_t)) return fail("gguf_decode: multiplication overflow");
    const uint64_t index_bytes = n_indices * sizeof(uint64_t);
    if (!(index_bytes <= UINTPTR_MAX - i0 && (i0 + index_bytes <= t0 || t0 + extent <= i0)))
        return fail("gather indices overlap target");
    DeviceGuard guard(ctx->device);
    cudaError_t e = tc::launch_decode_raw(type, static_cast<const uint8_t *>(source), row_bytes, 0, n_indices,
                                          column_begin, columns, dtype, static_cast<uint8_t *>(target), row_stride,
                                          column_stride, ctx->status, static_cast<cudaStream_t>(stream), row_indices,
                                          source_rows, target_bytes);
    if (e != cudaSuccess) return cuda_fail("gather launch", e);
    return ok();
}

int tc_cuda_set_path(tc_cuda_ctx *ctx, int path) {
    if (!ctx) return fail("null context");
    if (path < 0 || path > 3) return fail("invalid path selector");
    ctx->path = path;
    return ok();
}

int tc_cuda_qlinear_batched(tc_cuda_ctx *ctx, const tc_cuda_weight *const *weights, uint32_t n_weights,
                            const void *x, uint32_t m, void *const *ys, const uint64_t *ldys, int out_dtype,
                            void *stream) {
    if (!ctx || !weights || !x || !ys) return fail("null argument");
    if (!n_weights || n_weights > tc::kMaxGemvBatch) return fail("1..64 weights per batched call");
    if (m < 1 || m > 16) return fail("the batched GEMV takes 1..16 rows of X");
    if (out_dtype < TC_DTYPE_F32 || out_dtype > TC_DTYPE_BF16) return fail("invalid output dtype");
    if (reinterpret_cast<uintptr_t>(x) % 16) return fail("X must be 16-byte aligned");
    const uint64_t k = weights[0] ? weights[0]->k : 0;
    for (uint32_t i = 0; i < n_weights; ++i) {
        const tc_cuda_weight *w = weights[i];
        if (!w || !ys[i]) return fail("null weight or output");
        if (w->k != k) return fail("weights of one batched call must share K");
        if (w->device != ctx->device) return fail("weight lives on another device");
        if (w->glu) return fail("a SwiGLU weight needs TC_EPI_SWIGLU (tc_cuda_qlinear_ex)");
        if (w->raw) return fail("dense weights run through tc_cuda_qlinear");
        if (ldys && ldys[i] && ldys[i] < w->n) return fail("invalid/overlapping row stride");
    }
    DeviceGuard guard(ctx->device);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    // One launch per weight type (the kernel is specialised on it).
    for (const uint32_t type : {uint32_t(TC_GGML_Q4_K), uint32_t(TC_GGML_Q5_K), uint32_t(TC_GGML_Q6_K)}) {
        tc::GemvBatch bt{};
        uint32_t counters = 0;
        for (uint32_t i = 0; i < n_weights; ++i) {
            const tc_cuda_weight *w = weights[i];
            if (w->type != type) continue;
            bt.e[bt.n_entries++] = {w->chunks, ys[i], ldys && ldys[i] ? ldys[i] : w->n, (uint32_t)w->n, 0u};
            counters += tc::gemv_counters(w->n);
        }
        if (!bt.n_entries) continue;
        bt.kb = (uint32_t)(k / 256);
        tc::GemvSplit sp;
        sp.status = ctx->status;
        int rc = ensure_gemv_workspace(ctx, tc::kGemvPartialFloats, counters);
        if (rc) return rc;
        sp.partials = ctx->gemv_partials;
        sp.counters = ctx->gemv_counters;
        cudaError_t e = tc::launch_gemv_batch(bt, type, 0, m, static_cast<const uint16_t *>(x), k, out_dtype, sp, s);
        if (e != cudaSuccess) return cuda_fail("batched GEMV launch", e);
    }
    return ok();
}

int tc_cuda_qlinear_plan(tc_cuda_ctx *ctx, const tc_cuda_weight *w, uint32_t m, int stage, uint32_t *kernel,
                         uint32_t *ksplit) {
    if (!ctx || !w || !kernel || !ksplit) return fail("null argument");
    if (stage != TC_STAGE_BF16 && stage != TC_STAGE_F16 && stage != TC_STAGE_F16_X16)
        return fail("invalid staging precision");
    *ksplit = 1;
    if (w->raw) {
        *kernel = TC_KERNEL_DENSE;
        return ok();
    }
    const bool small = m <= 16 && stage != TC_STAGE_F16_X16;
    if ((small && ctx->path < 2) || ctx->path == 1) {
        *kernel = TC_KERNEL_GEMV;
        return ok();
    }
    if (m <= 128 || ctx->path == 3) {
        *kernel = TC_KERNEL_GEMM_1CTA;
        return ok();
    }
    *kernel = TC_KERNEL_GEMM_PAIR;
    const tc::SegmentView sv{0u, m, view_of(w)};
    const int sms = ctx->sm_limit > 0 ? std::min(ctx->sm_limit, ctx->sm_count) : ctx->sm_count;
    if (!(w->glu && w->n % 16)) *ksplit = tc::pair_ksplit(&sv, 1, sms);
    return ok();
}

int tc_cuda_set_sm_limit(tc_cuda_ctx *ctx, int sms) {
    if (!ctx) return fail("null context");
    if (sms < 0) return fail("negative SM limit");
    ctx->sm_limit = sms;
    return ok();
}

int tc_cuda_qlinear(tc_cuda_ctx *ctx, const tc_cuda_weight *const *weights, uint32_t n_weights,
                    const int32_t *seg_offsets, const int32_t *seg_weight, uint32_t n_seg, const void *x, void *y,
                    uint64_t ldy, int out_dtype, int stage, void *stream) {
    return tc_cuda_qlinear_ex(ctx, weights, n_weights, seg_offsets, seg_weight, n_seg, x, y, ldy, out_dtype, stage,
                              nullptr, stream);
}

int tc_cuda_qlinear_ex(tc_cuda_ctx *ctx, const tc_cuda_weight *const *weights, uint32_t n_weights,
                       const int32_t *seg_offsets, const int32_t *seg_weight, uint32_t n_seg, const void *x, void *y,
                       uint64_t ldy, int out_dtype, int stage, const tc_epilogue *epilogue, void *stream) {
    return tc_cuda_qlinear_gather(ctx, weights, n_weights, seg_offsets, seg_weight, n_seg, x, y, ldy, out_dtype,
                                  stage, epilogue, nullptr, 0, stream);
}

int tc_cuda_qlinear_gather(tc_cuda_ctx *ctx, const tc_cuda_weight *const *weights, uint32_t n_weights,
                           const int32_t *seg_offsets, const int32_t *seg_weight, uint32_t n_seg, const void *x,
                           void *y, uint64_t ldy, int out_dtype, int stage, const tc_epilogue *epilogue,
                           void *const *peer_y, uint32_t n_peer, void *stream) {
    if (!ctx || !weights || !n_weights || !x || !y || !seg_offsets) return fail("null argument");
    if (n_peer > tc::kMaxPeers - 1) return fail("at most 7 peer replicas");
    if (n_peer && !peer_y) return fail("null peer output list");
    for (uint32_t i = 0; i < n_peer; ++i)
        if (!peer_y[i]) return fail("null peer output");
    if (!n_seg) return fail("no segments");
    if (out_dtype < TC_DTYPE_F32 || out_dtype > TC_DTYPE_BF16) return fail("invalid output dtype");
    if (stage != TC_STAGE_BF16 && stage != TC_STAGE_F16 && stage != TC_STAGE_F16_X16)
        return fail("invalid staging precision");
    if (stage == TC_STAGE_F16_X16 && ctx->path == 1) return fail("the warp GEMV takes bf16 X");
    const tc_cuda_weight *w0 = weights[0];
    if (!w0) return fail("null weight");
    for (uint32_t i = 0; i < n_weights; ++i) {
        if (!weights[i]) return fail("null weight");
        if (weights[i]->n != w0->n || weights[i]->k != w0->k) return fail("weights of one call must share N and K");
        if (weights[i]->device != ctx->device) return fail("weight lives on another device");
        if (weights[i]->glu != w0->glu) return fail("SwiGLU and plain weights cannot share a call");
    }
    const uint32_t flags = epilogue ? epilogue->flags : 0u;
    const uint32_t known = TC_EPI_BIAS | TC_EPI_GELU_TANH | TC_EPI_GELU_ERF | TC_EPI_SWIGLU | TC_EPI_GATE_RESIDUAL;
    if (flags & ~known) return fail("unknown epilogue flag");
    if (__builtin_popcount(flags & (TC_EPI_GELU_TANH | TC_EPI_GELU_ERF | TC_EPI_SWIGLU)) > 1)
        return fail("at most one activation per epilogue");
    if (bool(flags & TC_EPI_SWIGLU) != bool(w0->glu))
        return fail(w0->glu ? "a SwiGLU weight needs TC_EPI_SWIGLU" : "TC_EPI_SWIGLU needs a weight from tc_cuda_weight_upload_glu");
    const uint64_t n_out = w0->glu ? w0->n / 2 : w0->n;
    if (ldy == 0) ldy = n_out;
    if (ldy < n_out) return fail("invalid/overlapping row stride");
    tc::EpiView epi;
    epi.flags = flags;
    epi.n_peer = n_peer;
    for (uint32_t i = 0; i < n_peer; ++i) epi.peer[i] = peer_y[i];
    if (flags & TC_EPI_BIAS) {
        if (!epilogue->bias) return fail("TC_EPI_BIAS needs a bias vector");
        epi.bias = epilogue->bias;
        epi.bias_up = epilogue->bias_up_offset;
        if (w0->glu && epi.bias_up < n_out) return fail("SwiGLU up-bias offset overlaps the gate biases");
    }
    if (flags & TC_EPI_GATE_RESIDUAL) {
        if (!epilogue->gate || !epilogue->residual) return fail("TC_EPI_GATE_RESIDUAL needs gate and residual");
        epi.gate = epilogue->gate;
        epi.ld_gate = epilogue->ld_gate ? epilogue->ld_gate : n_out;
        epi.res = epilogue->residual;
        epi.ld_res = epilogue->ld_residual ? epilogue->ld_residual : n_out;
        if (epi.ld_gate < n_out || epi.ld_res < n_out) return fail("invalid/overlapping row stride");
        for (uint32_t s = 0; s < n_seg; ++s) {
            const int64_t g = epilogue->seg_gate ? epilogue->seg_gate[s] : (int64_t)s;
            if (g < 0 || g >= (int64_t)epilogue->n_gate_rows) return fail("segment gate row out of range");
        }
    }
    if (seg_offsets[0] != 0) return fail("seg_offsets[0] must be 0");
    for (uint32_t s = 0; s < n_seg; ++s) {
        if (seg_offsets[s + 1] < seg_offsets[s]) return fail("seg_offsets must be non-decreasing");
        if (seg_weight && (seg_weight[s] < 0 || (uint32_t)seg_weight[s] >= n_weights))
            return fail("seg_weight out of range");
    }
    if (reinterpret_cast<uintptr_t>(x) % 16) return fail("X must be 16-byte aligned");
    const uint64_t m_total = (uint64_t)seg_offsets[n_seg];
    if (!m_total) return ok();
    epi.y_limit = (m_total - 1) * ldy + n_out;   // checked by bounds-checked builds
    epi.status = ctx->status;
    DeviceGuard guard(ctx->device);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const uint64_t k = w0->k;

    // Split segments: small ones to the GEMV, the rest to the tensor-core GEMM
    // (one launch per weight type).
    std::vector<tc::SegmentView> gemm[3];   // Q4_K, Q6_K, Q5_K
    std::vector<tc::SegmentView> gemv;
    struct DenseSeg { uint32_t b, e, gate_row; const tc_cuda_weight *w; };
    std::vector<DenseSeg> dense;             // F32 / F16 / BF16 / 32-weight block types
    for (uint32_t i = 0; i < n_seg; ++i) {
        const uint32_t b = (uint32_t)seg_offsets[i], e = (uint32_t)seg_offsets[i + 1];
        if (b == e) continue;
        const tc_cuda_weight *w = weights[seg_weight ? seg_weight[i] : 0];
        tc::SegmentView sv{b, e, view_of(w)};
        if (flags & TC_EPI_GATE_RESIDUAL) sv.gate_row = (uint32_t)(epilogue->seg_gate ? epilogue->seg_gate[i] : i);
        if (w->raw) {
            if (stage != TC_STAGE_BF16 && !w->dense_f16)
                return fail("weight values exceed the fp16 range; use TC_STAGE_BF16");
            dense.push_back({b, e, sv.gate_row, w});
            continue;
        }
        // fp16 X (TC_STAGE_F16_X16) always takes the tensor-core GEMM: the
        // warp GEMV works in bf16 code space.
        const bool small = (e - b) <= 16 && stage != TC_STAGE_F16_X16;
        if ((small && ctx->path < 2) || ctx->path == 1) {
            // The GEMV handles at most 16 rows per launch; longer forced
            // segments are cut into 16-row pieces.
            for (uint32_t m = b; m < e; m += 16) gemv.push_back({m, std::min(e, m + 16), sv.w, sv.gate_row});
        } else {
            gemm[w->type == TC_GGML_Q4_K ? 0 : w->type == TC_GGML_Q5_K ? 2 : 1].push_back(sv);
        }
    }
    const uint16_t *xg = static_cast<const uint16_t *>(x);
    if (stage == TC_STAGE_F16 && (!gemm[0].empty() || !gemm[1].empty() || !gemm[2].empty() || !dense.empty())) {
        int rc = ensure_workspace(ctx, m_total * k * 2);
        if (rc) return rc;
        cudaError_t e = tc::launch_x_to_f16(xg, static_cast<uint16_t *>(ctx->workspace), m_total * k, ctx->status, s);
        if (e != cudaSuccess) return cuda_fail("fp16 staging launch", e);
        xg = static_cast<const uint16_t *>(ctx->workspace);
    }
    const int gemm_sms = ctx->sm_limit > 0 ? std::min(ctx->sm_limit, ctx->sm_count) : ctx->sm_count;
    for (int t = 0; t < 3; ++t) {
        for (size_t i = 0; i < gemm[t].size(); i += 32) {
            const uint32_t cnt = (uint32_t)std::min<size_t>(32, gemm[t].size() - i);
            const tc::SegmentView *sv = gemm[t].data() + i;
            // Split-K for the 2-CTA path when its tiles cannot fill the SM
            // pairs (SwiGLU weights only with whole 16-row gate / up groups).
            tc::SplitK sk;
            uint32_t max_rows = 0;
            for (uint32_t j = 0; j < cnt; ++j) max_rows = std::max(max_rows, sv[j].m_end - sv[j].m_begin);
            if (ctx->path != 3 && max_rows > 128 && !(w0->glu && w0->n % 16)) {
                sk.ksplit = tc::pair_ksplit(sv, cnt, gemm_sms);
                if (sk.ksplit > 1) {
                    const size_t need = tc::pair_split_floats(sk.ksplit, m_total, (uint32_t)w0->n);
                    if (need > ctx->split_ws_floats) {
                        if (ctx->split_ws) cudaFree(ctx->split_ws);
                        ctx->split_ws = nullptr;
                        ctx->split_ws_floats = 0;
                        cudaError_t e = cudaMalloc(&ctx->split_ws, need * sizeof(float));
                        if (e != cudaSuccess) return cuda_fail("split-K workspace allocation", e);
                        ctx->split_ws_floats = need;
                    }
                    sk.ws = ctx->split_ws;
                }
            }
            cudaError_t e = tc::launch_gemm(sv, cnt, xg, m_total, k, y, ldy, out_dtype, stage != TC_STAGE_BF16,
                                            gemm_sms, ctx->status, ctx->path != 3, s, &epi, &sk);
            if (e != cudaSuccess) return cuda_fail("GEMM launch", e);
        }
    }
    for (const auto &sv : gemv) {
        tc::GemvSplit sp;
        sp.status = ctx->status;
        int rc = ensure_gemv_workspace(ctx, tc::kGemvPartialFloats, tc::gemv_counters(sv.w.n));
        if (rc) return rc;
        sp.partials = ctx->gemv_partials;
        sp.counters = ctx->gemv_counters;
        cudaError_t e = tc::launch_gemv(sv, static_cast<const uint16_t *>(x), k, y, ldy, out_dtype, sp, s, &epi);
        if (e != cudaSuccess) return cuda_fail("GEMV launch", e);
    }
    // Dense weights: the dense tensor-core GEMM on the bf16 or fp16 copy, with
    // the fused epilogue and peer stores in its epilogue.  X needs a 16-byte
    // row pitch: with K not a multiple of 8 it is copied (zero-padded) first.
    if (!dense.empty()) {
        const uint16_t *xd = xg;
        uint64_t ldx = k;
        if (k % 8) {
            ldx = (k + 7) / 8 * 8;
            const size_t need = m_total * ldx * 2;
            if (need > ctx->dense_x_bytes) {
                if (ctx->dense_x) cudaFree(ctx->dense_x);
                ctx->dense_x = nullptr;
                ctx->dense_x_bytes = 0;
                cudaError_t e = cudaMalloc(&ctx->dense_x, need);
                if (e != cudaSuccess) return cuda_fail("dense X workspace allocation", e);
                ctx->dense_x_bytes = need;
            }
            cudaError_t e = tc::launch_pad_rows(xg, ctx->dense_x, m_total, k, ldx, s);
            if (e != cudaSuccess) return cuda_fail("X pitch copy", e);
            xd = ctx->dense_x;
        }
        for (const auto &d : dense) {
            const bool f16 = stage != TC_STAGE_BF16;
            cudaError_t e = tc::launch_dense_gemm(f16 ? d.w->dense_f16 : d.w->dense_bf16, d.w->dense_ld,
                                                  (uint32_t)d.w->n, xd, ldx, m_total, k, d.b, d.e, d.gate_row, y, ldy,
                                                  out_dtype, f16, gemm_sms, ctx->status, &epi, s);
            if (e != cudaSuccess) return cuda_fail("dense GEMM launch", e);
        }
    }
    return ok();
}

}  // extern "C"
