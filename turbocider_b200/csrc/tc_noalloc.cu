// Allocation-free small-M quantised linear: tc_cuda_qlinear_small_static.
//
// Who needs it: callers that must not allocate device memory at the moment
// they run a linear.  Examples: an inference server whose device memory is
// one pre-sized arena carved up at start-up; code running under a custom
// allocator callback, where a nested cudaMalloc could re-enter the allocator;
// or a latency-critical decode loop that cannot afford the implicit device
// synchronisation of cudaMalloc / cudaFree.  tc_cuda_qlinear cannot serve them
// on its small-M path: the split-K GEMV keeps K-slice partial sums, per-tile
// arrival counters and a status word in a context workspace that grows with
// cudaMalloc the first time a shape needs more.  This entry point runs the
// same kernel with that scratch in a fixed file-scope device array.
//
// The array (kScratchBytes below) exists once per device that loads this
// library and stays allocated until the process exits.  Its host-side name is
// only a stand-in for the symbol, not a device address, so the address is
// fetched with cudaGetSymbolAddress once per device (with that device current)
// and passed to the kernel as an argument.
//
// Contract:
//   * the first call on a device fetches that address and clears the status
//     word (one-time set-up, synchronous); make that first call before
//     capturing any stream;
//   * every call shares the one array, which keeps the previous call's
//     contents: the per-tile counters are cleared on the call's stream before
//     the kernel runs, and the partials are fully written before they are
//     read;
//   * the status word (TC_STATUS_* bits: nonfinite scale, timeout) is sticky
//     across calls, like a context's: tc_cuda_small_static_status reads it
//     (and optionally clears it) after synchronising the device;
//   * calls whose kernels may overlap on the GPU (different streams, or
//     different host threads) race on the array -- serialise them;
//   * sizes whose scratch exceeds kScratchBytes are rejected with an error
//     (a guard: the GEMV needs 4.6 MiB of partials and 4 bytes per 16 weight
//     rows, so only weights of over 12 million rows are refused).
// Nothing here calls cudaMalloc, cudaFree or any allocating library routine.
#include <mutex>
#include <string>

#include "../../include/turbocider_cuda.h"
#include "kq_format.cuh"
#include "tc_internal.h"

namespace {

constexpr size_t kScratchBytes = size_t(8) << 20;   // 8 MiB per device
constexpr size_t kStatusBytes = 256;                // status word, padded

static __device__ __align__(256) unsigned char g_gemv_scratch[kScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_setup_mutex;
void *g_scratch_ptr[kMaxDevices] = {};

// Errors are reported through tc_cuda_last_error(), like every other call.
int fail(const std::string &reason) {
    tc::set_last_error(reason);
    return TC_CUDA_FAIL;
}

// Device address of this device's copy of the array (fetched once).
int scratch_address(int device, void **out) {
    if (device < 0 || device >= kMaxDevices) return fail("device ordinal out of range");
    std::lock_guard<std::mutex> lock(g_setup_mutex);
    if (!g_scratch_ptr[device]) {
        int previous = -1;
        if (cudaGetDevice(&previous) != cudaSuccess) return fail("cudaGetDevice failed");
        if (previous != device && cudaSetDevice(device) != cudaSuccess) return fail("cudaSetDevice failed");
        void *ptr = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&ptr, g_gemv_scratch);
        // the status word starts at zero (it is only cleared on request later)
        if (e == cudaSuccess) e = cudaMemset(ptr, 0, kStatusBytes);
        if (e == cudaSuccess) e = cudaDeviceSynchronize();
        if (previous != device) cudaSetDevice(previous);
        if (e != cudaSuccess)
            return fail(std::string("set-up of the static GEMV scratch failed: ") + cudaGetErrorString(e));
        g_scratch_ptr[device] = ptr;
    }
    *out = g_scratch_ptr[device];
    return TC_CUDA_OK;
}

}  // namespace

extern "C" int tc_cuda_qlinear_small_static(const tc_cuda_weight *weight, const void *x, uint32_t m, void *y,
                                            uint64_t ldy, int out_dtype, void *stream) {
    if (!weight || !x || !y) return fail("null weight, X or Y");
    if (m == 0 || m > 16) return fail("tc_cuda_qlinear_small_static handles 1..16 rows of X");
    if (out_dtype < TC_DTYPE_F32 || out_dtype > TC_DTYPE_BF16) return fail("invalid output dtype");
    if (reinterpret_cast<uintptr_t>(x) % 16) return fail("X must be 16-byte aligned");
    if (weight->glu) return fail("a SwiGLU weight needs TC_EPI_SWIGLU (tc_cuda_qlinear_ex)");
    if (weight->raw) return fail("dense weights run through tc_cuda_qlinear");
    if (ldy == 0) ldy = weight->n;
    if (ldy < weight->n) return fail("invalid/overlapping row stride");

    const tc::WeightView view{weight->chunks, weight->type, weight->kb, weight->panels, (uint32_t)weight->n};
    tc::GemvSplit sp;
    const size_t tiles = tc::gemv_counters(weight->n);
    const size_t counter_bytes = (tiles * sizeof(uint32_t) + 255) / 256 * 256;
    const size_t partial_bytes = tc::kGemvPartialFloats * sizeof(float);
    const size_t need = kStatusBytes + counter_bytes + partial_bytes;
    if (need > kScratchBytes)
        return fail("weight needs " + std::to_string(need) + " bytes of GEMV scratch; the static scratch holds " +
                    std::to_string(kScratchBytes) + " (N=" + std::to_string(weight->n) +
                    ", K=" + std::to_string(weight->k) + ")");

    int previous = -1;
    if (cudaGetDevice(&previous) != cudaSuccess) return fail("cudaGetDevice failed");
    void *base = nullptr;
    int rc = scratch_address(weight->device, &base);
    if (rc) return rc;
    if (previous != weight->device && cudaSetDevice(weight->device) != cudaSuccess)
        return fail("cudaSetDevice failed");
    auto *bytes = static_cast<unsigned char *>(base);
    sp.status = reinterpret_cast<uint32_t *>(bytes);
    sp.counters = reinterpret_cast<uint32_t *>(bytes + kStatusBytes);
    sp.partials = reinterpret_cast<float *>(bytes + kStatusBytes + counter_bytes);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    // the per-tile counters must start at zero; the status word is sticky
    cudaError_t e = cudaMemsetAsync(bytes + kStatusBytes, 0, counter_bytes, s);
    if (e == cudaSuccess) {
        const tc::SegmentView seg{0u, m, view};
        tc::EpiView plain;   // no epilogue; Y's extent for bounds-checked builds
        plain.y_limit = (uint64_t)(m - 1) * ldy + weight->n;
        plain.status = sp.status;
        e = tc::launch_gemv(seg, static_cast<const uint16_t *>(x), weight->k, y, ldy, out_dtype, sp, s, &plain);
    }
    if (previous != weight->device) cudaSetDevice(previous);
    if (e != cudaSuccess) return fail(std::string("static-scratch GEMV launch: ") + cudaGetErrorString(e));
    tc::set_last_error("");
    return TC_CUDA_OK;
}

extern "C" int tc_cuda_small_static_status(int device, uint32_t *bits, int clear) {
    if (!bits) return fail("null out-parameter");
    void *base = nullptr;
    int rc = scratch_address(device, &base);
    if (rc) return rc;
    int previous = -1;
    if (cudaGetDevice(&previous) != cudaSuccess) return fail("cudaGetDevice failed");
    if (previous != device && cudaSetDevice(device) != cudaSuccess) return fail("cudaSetDevice failed");
    cudaError_t e = cudaDeviceSynchronize();
    if (e == cudaSuccess) e = cudaMemcpy(bits, base, sizeof(uint32_t), cudaMemcpyDeviceToHost);
    if (e == cudaSuccess && clear) e = cudaMemset(base, 0, sizeof(uint32_t));
    if (previous != device) cudaSetDevice(previous);
    if (e != cudaSuccess) return fail(std::string("static GEMV status read: ") + cudaGetErrorString(e));
    tc::set_last_error("");
    return TC_CUDA_OK;
}
