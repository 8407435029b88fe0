// Streaming GGUF tensor loader: file -> pinned host memory -> HBM -> panel
// layout, with read-ahead and cancellation (tc_cuda_weight_load_gguf).
//
// The reference loads a GGUF tensor in bounded chunks: a read-ahead worker
// thread preads chunk i + 1 into the second of two buffers while the loading
// thread decodes chunk i, the cancel flag is polled once per chunk, and
// nothing is published until every chunk succeeded
// (native/runtime/streaming/read_ahead_worker.hpp:21-70 and
// GgufPackedBank::load_candidate, native/runtime/streaming/
// gguf_packed_bank.cpp:393-452).  Here the work that follows each read is a
// host -> HBM copy of the chunk's raw blocks and the device re-layout of its
// 128-row panels, so the pipeline has three stages in flight at once:
//   worker thread   pread chunk i + 1 into pinned slot (i + 1) % 2
//   copy engine     chunk i, pinned slot i % 2 -> device staging slot i % 2
//   SMs             re-layout of chunk i's panels into the weight
// A pinned slot is handed to the worker again only after the copy out of it
// completed (an event per slot).  Chunks are whole panels (multiples of 128
// rows), so each chunk's re-layout writes its own panels and nothing else.
// The cancel flag (caller-owned int32, nonzero = cancel) is read before every
// chunk and between the worker's preads; a cancelled or failed load drains
// the worker and the stream, frees the weight and returns
// TC_CUDA_CANCELLED / TC_CUDA_FAIL.  The staging slots belong to the context
// and are reused by the next load.
#include <chrono>
#include <condition_variable>
#include <cstring>
#include <mutex>
#include <string>
#include <thread>

#include "../../include/turbocider_cuda.h"
#include "kq_format.cuh"
#include "tc_internal.h"

namespace {

using Clock = std::chrono::steady_clock;
double seconds_since(Clock::time_point t0) { return std::chrono::duration<double>(Clock::now() - t0).count(); }

bool cancel_set(const volatile int32_t *cancel) { return cancel && *cancel != 0; }

// One pread job in flight on a worker thread (the read-ahead worker).
class ReadAhead {
  public:
    ReadAhead(const tc_gguf *file, uint64_t index, const volatile int32_t *cancel)
        : file_(file), index_(index), cancel_(cancel), th_([this] { run(); }) {}
    ~ReadAhead() {
        {
            std::lock_guard<std::mutex> lock(mu_);
            stop_ = true;
        }
        work_.notify_all();
        th_.join();   // an in-flight pread finishes first: its buffer outlives it
    }
    void submit(uint64_t row_begin, uint64_t rows, void *dst, uint64_t bytes) {
        {
            std::lock_guard<std::mutex> lock(mu_);
            job_ = {row_begin, rows, dst, bytes, true};
            ready_ = false;
        }
        work_.notify_all();
    }
    // Waits for the submitted job; returns its status (TC_CUDA_*) and message.
    int take(double *read_seconds, std::string *error) {
        std::unique_lock<std::mutex> lock(mu_);
        done_.wait(lock, [&] { return ready_; });
        ready_ = false;
        *read_seconds += seconds_;
        *error = error_;
        return rc_;
    }

  private:
    struct Job {
        uint64_t row_begin, rows;
        void *dst;
        uint64_t bytes;
        bool valid;
    };
    void run() {
        std::unique_lock<std::mutex> lock(mu_);
        for (;;) {
            work_.wait(lock, [&] { return stop_ || job_.valid; });
            if (stop_) return;
            const Job job = job_;
            job_.valid = false;
            lock.unlock();
            const auto t0 = Clock::now();
            const int rc = tc_gguf_read(file_, index_, job.row_begin, job.rows, job.dst, job.bytes, cancel_);
            const std::string error = rc ? tc_cuda_last_error() : "";
            lock.lock();
            rc_ = rc;
            error_ = error;
            seconds_ = seconds_since(t0);
            ready_ = true;
            done_.notify_all();
        }
    }
    const tc_gguf *file_;
    const uint64_t index_;
    const volatile int32_t *cancel_;
    std::mutex mu_;
    std::condition_variable work_, done_;
    Job job_{0, 0, nullptr, 0, false};
    bool stop_ = false, ready_ = false;
    int rc_ = 0;
    double seconds_ = 0;
    std::string error_;
    std::thread th_;   // last: starts after every other member exists
};

}  // namespace

extern "C" int tc_cuda_weight_load_gguf(tc_cuda_ctx *ctx, const tc_gguf *file, uint64_t index, uint64_t n_begin,
                                        uint64_t n_count, uint64_t chunk_bytes, const volatile int32_t *cancel,
                                        tc_cuda_weight **out, tc_gguf_load_stats *stats) {
    auto fail = [](const std::string &m) {
        tc::set_last_error(m);
        return TC_CUDA_FAIL;
    };
    if (!ctx || !file || !out) return fail("null argument");
    *out = nullptr;
    const auto t_start = Clock::now();
    if (cancel_set(cancel)) {
        tc::set_last_error("generation cancelled");
        return TC_CUDA_CANCELLED;
    }
    char name[4096];
    uint32_t type = 0, rank = 0;
    uint64_t dims[4] = {1, 1, 1, 1}, offset = 0, bytes = 0;
    if (tc_gguf_tensor(file, index, name, sizeof(name), &type, &rank, dims, &offset, &bytes)) return TC_CUDA_FAIL;
    if (type != TC_GGML_Q4_K && type != TC_GGML_Q5_K && type != TC_GGML_Q6_K)
        return fail("tc_cuda_weight_load_gguf takes K-quant tensors (Q4_K, Q5_K, Q6_K)");
    const uint64_t k = dims[0], rows_total = dims[1] * dims[2] * dims[3];
    if (n_count == 0) n_count = rows_total - std::min(n_begin, rows_total);
    if (n_begin >= rows_total || n_count > rows_total - n_begin) return fail("row slice out of bounds");
    const uint64_t row_bytes = k / tc::kBlockWeights * tc::block_bytes(type);
    // Chunks of whole panels (128 rows), about chunk_bytes each (default 8 MiB).
    if (chunk_bytes == 0) chunk_bytes = 8ull << 20;
    uint64_t chunk_rows = chunk_bytes / row_bytes / tc::kPanelRows * tc::kPanelRows;
    if (chunk_rows == 0) chunk_rows = tc::kPanelRows;
    const uint64_t slot_bytes = chunk_rows * row_bytes;
    const uint64_t n_chunks = (n_count + chunk_rows - 1) / chunk_rows;

    tc_cuda_weight *w = nullptr;
    int rc = tc_cuda_weight_create(ctx, type, n_count, k, &w);
    if (rc) return rc;
    int previous = -1;
    cudaGetDevice(&previous);
    if (previous != ctx->device) cudaSetDevice(ctx->device);

    // Staging slots, stream and events live in the context (grow-only), so a
    // model's many tensors pay the pinned allocation once.
    cudaError_t e = cudaSuccess;
    if (!ctx->load_stream) {
        e = cudaStreamCreateWithFlags(&ctx->load_stream, cudaStreamNonBlocking);
        for (int i = 0; i < 2 && e == cudaSuccess; ++i)
            e = cudaEventCreateWithFlags(&ctx->load_freed[i], cudaEventDisableTiming);
    }
    if (e == cudaSuccess && ctx->load_slot_bytes < slot_bytes) {
        for (int i = 0; i < 2; ++i) {
            if (ctx->load_host[i]) cudaFreeHost(ctx->load_host[i]);
            if (ctx->load_dev[i]) cudaFree(ctx->load_dev[i]);
            ctx->load_host[i] = ctx->load_dev[i] = nullptr;
        }
        ctx->load_slot_bytes = 0;
        for (int i = 0; i < 2 && e == cudaSuccess; ++i) {
            e = cudaHostAlloc(&ctx->load_host[i], slot_bytes, cudaHostAllocDefault);
            if (e == cudaSuccess) e = cudaMalloc(&ctx->load_dev[i], slot_bytes);
        }
        if (e == cudaSuccess) ctx->load_slot_bytes = slot_bytes;
    }
    void *const host[2] = {ctx->load_host[0], ctx->load_host[1]};
    void *const dev[2] = {ctx->load_dev[0], ctx->load_dev[1]};
    cudaEvent_t *const freed = ctx->load_freed;
    const cudaStream_t s = ctx->load_stream;
    // d / dmin finiteness of the re-laid blocks lands in status word 1
    if (e == cudaSuccess) e = cudaMemsetAsync(ctx->status + 1, 0, sizeof(uint32_t), s);

    double read_seconds = 0, wait_seconds = 0;
    std::string error;
    rc = e == cudaSuccess ? TC_CUDA_OK : TC_CUDA_FAIL;
    if (rc) error = std::string("loader set-up: ") + cudaGetErrorString(e);
    if (!rc) {
        ReadAhead reader(file, index, cancel);
        reader.submit(n_begin, std::min(chunk_rows, n_count), host[0], slot_bytes);
        for (uint64_t c = 0; c < n_chunks && !rc; ++c) {
            const uint32_t slot = (uint32_t)(c & 1);
            const uint64_t r0 = c * chunk_rows, rows = std::min(chunk_rows, n_count - r0);
            const auto t_wait = Clock::now();
            rc = reader.take(&read_seconds, &error);
            wait_seconds += seconds_since(t_wait);
            if (rc) break;
            if (cancel_set(cancel)) {
                rc = TC_CUDA_CANCELLED;
                error = "generation cancelled";
                break;
            }
            if (c + 1 < n_chunks) {
                // the other pinned slot is free once the copy out of it is done
                const uint32_t next = slot ^ 1u;
                if ((e = cudaEventSynchronize(freed[next])) != cudaSuccess) break;
                const uint64_t r1 = r0 + rows;
                reader.submit(n_begin + r1, std::min(chunk_rows, n_count - r1), host[next], slot_bytes);
            }
            e = cudaMemcpyAsync(dev[slot], host[slot], rows * row_bytes, cudaMemcpyHostToDevice, s);
            if (e == cudaSuccess) e = cudaEventRecord(freed[slot], s);
            if (e == cudaSuccess)
                e = tc::launch_relayout(type, static_cast<const uint8_t *>(dev[slot]), rows, w->kb,
                                        w->chunks + (r0 / tc::kPanelRows) * w->kb * tc::chunk_bytes(type),
                                        (uint32_t)((rows + tc::kPanelRows - 1) / tc::kPanelRows), ctx->status + 1, s);
            if (e != cudaSuccess) break;
        }
        // ~ReadAhead drains the worker before the slots can be freed
    }
    if (!rc && e != cudaSuccess) {
        rc = TC_CUDA_FAIL;
        error = std::string("loader: ") + cudaGetErrorString(e);
    }
    uint32_t bits = 0;
    cudaError_t e2 = s ? cudaStreamSynchronize(s) : cudaSuccess;
    if (e2 == cudaSuccess && !rc) e2 = cudaMemcpy(&bits, ctx->status + 1, sizeof(uint32_t), cudaMemcpyDeviceToHost);
    if (!rc && e2 != cudaSuccess) {
        rc = TC_CUDA_FAIL;
        error = std::string("loader: ") + cudaGetErrorString(e2);
    }
    if (!rc && (bits & TC_STATUS_NONFINITE_SCALE)) {
        rc = TC_CUDA_FAIL;
        error = "nonfinite weight/scale or conversion overflow";
    }
    if (previous != ctx->device && previous >= 0) cudaSetDevice(previous);
    if (stats) {
        stats->bytes = rc ? 0 : n_count * row_bytes;
        stats->chunks = n_chunks;
        stats->seconds = seconds_since(t_start);
        stats->read_seconds = read_seconds;
        stats->wait_seconds = wait_seconds;
    }
    if (rc) {
        tc_cuda_weight_free(w);
        tc::set_last_error(error);
        return rc;
    }
    *out = w;
    tc::set_last_error("");
    return TC_CUDA_OK;
}
