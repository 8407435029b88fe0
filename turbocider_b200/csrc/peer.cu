// N-column sharding with the all-gather fused into the GEMM epilogue: buffers
// shared between the ranks' processes (CUDA IPC) and the completion barrier.
//
// The reference partitions nothing (one Apple GPU).  The north star shards
// every quantised weight by output columns over the GPUs of one box and
// replicates the outputs with an all-gather; here each rank's GEMM writes its
// output tiles into every rank's Y directly (tc_cuda_qlinear_gather, NVLink
// peer stores from the epilogue), and tc_cuda_peer_barrier tells every rank
// when all of them have finished a linear.
//
// The barrier is one small kernel per rank: it raises this rank's flag in
// every rank's flag array (a system-scope release store, after a system fence
// that publishes the preceding GEMM's peer stores) and waits, with a time
// limit, until every rank's flag in its own array reached the epoch.  On
// timeout it sets TC_STATUS_TIMEOUT and returns; it never traps.  The ranks are
// separate processes on separate GPUs, so the waiting kernels run concurrently.
#include <algorithm>
#include <cstring>
#include <string>

#include "../../include/turbocider_cuda.h"
#include "tc_internal.h"

namespace tc {
namespace {

struct FlagPtrs {
    uint32_t *p[kMaxPeers];   // flag array of rank r, as mapped in this process
};

__global__ void peer_barrier_kernel(FlagPtrs f, uint32_t n, uint32_t rank, uint32_t epoch, uint64_t timeout_ns,
                                    uint32_t *status) {
    const uint32_t t = threadIdx.x;
    if (t >= n) return;
    __threadfence_system();
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(f.p[t] + rank), "r"(epoch) : "memory");
    const uint32_t *mine = f.p[rank] + t;
    uint64_t t0;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t0));
    for (;;) {
        uint32_t v;
        asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(mine) : "memory");
        if ((int32_t)(v - epoch) >= 0) break;
        uint64_t now;
        asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(now));
        if (now - t0 > timeout_ns) {
            atomicOr(status, (uint32_t)TC_STATUS_TIMEOUT);
            break;
        }
        __nanosleep(256);
    }
}

// Push by the SMs: every thread moves 16-byte vectors, each read once from
// this GPU and stored to every destination over NVLink (destination order
// rotated by block, so that all links carry stores at once).  128-thread
// blocks with few registers fit beside a resident GEMM CTA on an SM, so the
// push overlaps the next linear without taking SMs from it.
struct PushDst {
    uint4 *p[kMaxPeers];
};
constexpr int kPushUnroll = 4;
template <bool LINEAR>
__global__ void __launch_bounds__(128) push_kernel(const uint4 *__restrict__ src, PushDst dst, uint32_t n_dst,
                                                   uint64_t width16, uint64_t rows, uint64_t src_pitch16,
                                                   uint64_t dst_pitch16) {
    const uint64_t total = width16 * rows, per_iter = (uint64_t)blockDim.x * kPushUnroll;
    for (uint64_t base = (uint64_t)blockIdx.x * per_iter + threadIdx.x; base < total;
         base += (uint64_t)gridDim.x * per_iter) {
        uint4 v[kPushUnroll];
        uint64_t to[kPushUnroll];
#pragma unroll
        for (int u = 0; u < kPushUnroll; ++u) {
            const uint64_t i = base + (uint64_t)u * blockDim.x;
            to[u] = ~0ull;
            if (i < total) {
                uint64_t from = i;
                to[u] = i;
                if (!LINEAR) {
                    const uint64_t r = i / width16, c = i % width16;
                    from = r * src_pitch16 + c;
                    to[u] = r * dst_pitch16 + c;
                }
                v[u] = __ldg(src + from);
            }
        }
        for (uint32_t d = 0; d < n_dst; ++d) {
            uint4 *out = dst.p[(d + blockIdx.x) % n_dst];
#pragma unroll
            for (int u = 0; u < kPushUnroll; ++u)
                if (to[u] != ~0ull) out[to[u]] = v[u];
        }
    }
}

int fail(const std::string &reason) {
    set_last_error(reason);
    return TC_CUDA_FAIL;
}
int cuda_fail(const char *what, cudaError_t e) { return fail(std::string(what) + ": " + cudaGetErrorString(e)); }
int ok() {
    set_last_error("");
    return TC_CUDA_OK;
}

struct DeviceGuard {
    int previous = -1;
    explicit DeviceGuard(int device) {
        if (cudaGetDevice(&previous) == cudaSuccess && previous != device) cudaSetDevice(device);
    }
    ~DeviceGuard() {
        int now = -1;
        if (previous >= 0 && cudaGetDevice(&now) == cudaSuccess && now != previous) cudaSetDevice(previous);
    }
};

}  // namespace
}  // namespace tc

extern "C" {

int tc_cuda_peer_alloc(tc_cuda_ctx *ctx, uint64_t bytes, void **ptr, void *handle) {
    if (!ctx || !ptr || !handle || !bytes) return tc::fail("null argument or empty buffer");
    tc::DeviceGuard guard(ctx->device);
    *ptr = nullptr;
    cudaError_t e = cudaMalloc(ptr, bytes);
    if (e != cudaSuccess) return tc::cuda_fail("peer buffer allocation", e);
    if ((e = cudaMemset(*ptr, 0, bytes)) == cudaSuccess) {
        cudaIpcMemHandle_t h;
        if ((e = cudaIpcGetMemHandle(&h, *ptr)) == cudaSuccess) {
            std::memcpy(handle, &h, sizeof(h));
            return tc::ok();
        }
    }
    cudaFree(*ptr);
    *ptr = nullptr;
    return tc::cuda_fail("peer buffer export", e);
}

int tc_cuda_peer_open(tc_cuda_ctx *ctx, const void *handle, void **ptr) {
    if (!ctx || !ptr || !handle) return tc::fail("null argument");
    tc::DeviceGuard guard(ctx->device);
    cudaIpcMemHandle_t h;
    std::memcpy(&h, handle, sizeof(h));
    *ptr = nullptr;
    cudaError_t e = cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) return tc::cuda_fail("peer buffer import", e);
    return tc::ok();
}

int tc_cuda_peer_close(tc_cuda_ctx *ctx, void *ptr) {
    if (!ctx || !ptr) return tc::fail("null argument");
    tc::DeviceGuard guard(ctx->device);
    cudaError_t e = cudaIpcCloseMemHandle(ptr);
    if (e != cudaSuccess) return tc::cuda_fail("peer buffer close", e);
    return tc::ok();
}

int tc_cuda_peer_free(tc_cuda_ctx *ctx, void *ptr) {
    if (!ctx || !ptr) return tc::fail("null argument");
    tc::DeviceGuard guard(ctx->device);
    cudaError_t e = cudaFree(ptr);
    if (e != cudaSuccess) return tc::cuda_fail("peer buffer free", e);
    return tc::ok();
}

int tc_cuda_peer_push(tc_cuda_ctx *ctx, const void *src, void *const *dst, uint32_t n_dst, uint64_t width_bytes,
                      uint64_t rows, uint64_t src_pitch, uint64_t dst_pitch, void *stream) {
    if (!ctx || !src || (n_dst && !dst)) return tc::fail("null argument");
    if (n_dst > tc::kMaxPeers) return tc::fail("more destinations than ranks");
    if (!width_bytes || !rows) return tc::ok();
    if (rows > 1 && (src_pitch < width_bytes || dst_pitch < width_bytes))
        return tc::fail("row pitch smaller than the row width");
    for (uint32_t i = 0; i < n_dst; ++i)
        if (!dst[i]) return tc::fail("null destination");
    tc::DeviceGuard guard(ctx->device);
    const cudaStream_t s = static_cast<cudaStream_t>(stream);
    // Contiguous regions go as one linear copy (the copy engines' fastest form).
    const bool linear = rows == 1 || (src_pitch == width_bytes && dst_pitch == width_bytes);
    // The SMs' push kernel, when chosen and every address, width and pitch
    // is a multiple of 16 bytes.
    bool aligned16 = reinterpret_cast<uintptr_t>(src) % 16 == 0 && width_bytes % 16 == 0 &&
                     (linear || (src_pitch % 16 == 0 && dst_pitch % 16 == 0));
    for (uint32_t i = 0; i < n_dst; ++i) aligned16 = aligned16 && reinterpret_cast<uintptr_t>(dst[i]) % 16 == 0;
    if (ctx->push_ctas > 0 && aligned16 && n_dst) {
        tc::PushDst d{};
        for (uint32_t i = 0; i < n_dst; ++i) d.p[i] = static_cast<uint4 *>(dst[i]);
        const uint64_t w16 = linear ? width_bytes * rows / 16 : width_bytes / 16, r = linear ? 1 : rows;
        const unsigned ctas = (unsigned)ctx->push_ctas;
        if (linear)
            tc::push_kernel<true><<<ctas, 128, 0, s>>>(static_cast<const uint4 *>(src), d, n_dst, w16, r, w16, w16);
        else
            tc::push_kernel<false><<<ctas, 128, 0, s>>>(static_cast<const uint4 *>(src), d, n_dst, w16, r,
                                                        src_pitch / 16, dst_pitch / 16);
        cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess) return tc::cuda_fail("peer push kernel", e);
        return tc::ok();
    }
    auto copy = [&](uint32_t i, cudaStream_t on) {
        return linear ? cudaMemcpyAsync(dst[i], src, width_bytes * rows, cudaMemcpyDeviceToDevice, on)
                      : cudaMemcpy2DAsync(dst[i], dst_pitch, src, src_pitch, width_bytes, rows,
                                          cudaMemcpyDeviceToDevice, on);
    };
    const uint32_t lanes = std::min<uint32_t>((uint32_t)ctx->push_fanout, n_dst);
    if (lanes < 2) {
        for (uint32_t i = 0; i < n_dst; ++i) {
            cudaError_t e = copy(i, s);
            if (e != cudaSuccess) return tc::cuda_fail("peer push", e);
        }
        return tc::ok();
    }
    // Fan out over `lanes` side streams (destination i on stream i % lanes,
    // back to back within a stream), ordered after the work already on
    // `stream`; `stream` continues only after all of them.  (Measured on 8
    // B200s with one stream per peer: 369 GB/s received per GPU, against
    // 535 GB/s for the same copies back to back -- the copies contend.)
    cudaError_t e = cudaSuccess;
    if (!ctx->push_fork) {
        e = cudaEventCreateWithFlags(&ctx->push_fork, cudaEventDisableTiming);
        for (uint32_t i = 0; i < tc::kMaxPeers && e == cudaSuccess; ++i) {
            e = cudaStreamCreateWithFlags(&ctx->push_stream[i], cudaStreamNonBlocking);
            if (e == cudaSuccess) e = cudaEventCreateWithFlags(&ctx->push_join[i], cudaEventDisableTiming);
        }
        if (e != cudaSuccess) return tc::cuda_fail("push stream creation", e);
    }
    if ((e = cudaEventRecord(ctx->push_fork, s)) != cudaSuccess) return tc::cuda_fail("peer push", e);
    for (uint32_t l = 0; l < lanes; ++l)
        if ((e = cudaStreamWaitEvent(ctx->push_stream[l], ctx->push_fork, 0)) != cudaSuccess)
            return tc::cuda_fail("peer push", e);
    for (uint32_t i = 0; i < n_dst; ++i)
        if ((e = copy(i, ctx->push_stream[i % lanes])) != cudaSuccess) return tc::cuda_fail("peer push", e);
    for (uint32_t l = 0; l < lanes; ++l)
        if ((e = cudaEventRecord(ctx->push_join[l], ctx->push_stream[l])) != cudaSuccess ||
            (e = cudaStreamWaitEvent(s, ctx->push_join[l], 0)) != cudaSuccess)
            return tc::cuda_fail("peer push", e);
    return tc::ok();
}

int tc_cuda_set_push_kernel(tc_cuda_ctx *ctx, int ctas) {
    if (!ctx) return tc::fail("null context");
    if (ctas < 0 || ctas > 4096) return tc::fail("push kernel blocks out of range 0..4096");
    ctx->push_ctas = ctas;
    return tc::ok();
}

int tc_cuda_set_push_fanout(tc_cuda_ctx *ctx, int streams) {
    if (!ctx) return tc::fail("null context");
    if (streams < 0 || streams > (int)tc::kMaxPeers) return tc::fail("fan-out streams out of range 0..8");
    ctx->push_fanout = streams;
    return tc::ok();
}

int tc_cuda_peer_barrier(tc_cuda_ctx *ctx, uint32_t *const *flags, uint32_t n_ranks, uint32_t rank, uint32_t epoch,
                         uint32_t timeout_us, void *stream) {
    if (!ctx || !flags) return tc::fail("null argument");
    if (n_ranks < 1 || n_ranks > tc::kMaxPeers || rank >= n_ranks) return tc::fail("invalid rank / rank count");
    tc::FlagPtrs f{};
    for (uint32_t r = 0; r < n_ranks; ++r) {
        if (!flags[r]) return tc::fail("null flag array");
        f.p[r] = flags[r];
    }
    tc::DeviceGuard guard(ctx->device);
    const uint64_t limit = (uint64_t)(timeout_us ? timeout_us : 1000000u) * 1000u;
    tc::peer_barrier_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(f, n_ranks, rank, epoch, limit,
                                                                            ctx->status);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return tc::cuda_fail("peer barrier launch", e);
    return tc::ok();
}

}  // extern "C"
