// Host-side panel re-layout and panel copies: the loader path for weights that
// are streamed from pinned host memory.
//
// tc_relayout_host produces, on the CPU, exactly the bytes relayout_kernel
// (kq_dequant.cu) writes on the device: 128-row panels x 256-K chunks split
// by field, qs / ql / qh row pieces at row_slot(r), rows past N zero.  A
// loader does this once per weight while reading the GGUF file into pinned
// memory; each later transfer to HBM is then a plain asynchronous copy
// (tc_cuda_weight_copy_panels) that needs no SMs, so streaming the next
// layer's weights overlaps the current layer's GEMM, which occupies every SM.
// Like the upload path it rejects blocks whose d / dmin are not finite (the
// reference rejects them at decode time, native/core/gguf_decode.cpp:78, :92).
#include <algorithm>
#include <atomic>
#include <cstring>
#include <string>
#include <thread>
#include <vector>

#include "../../include/turbocider_cuda.h"
#include "kq_format.cuh"
#include "tc_internal.h"

namespace {

inline bool finite_half(uint16_t h) { return (h & 0x7c00u) != 0x7c00u; }
inline uint16_t rd16(const uint8_t *p) { return (uint16_t)(p[0] | (p[1] << 8)); }

// One chunk (panel p, super-block column c) of an n-row weight; `rows` points
// at the weight's first row (row pitch kb * block bytes).  Returns false on a
// nonfinite scale.
bool chunk_host(uint32_t type, const uint8_t *rows, uint64_t n, uint32_t kb, uint64_t p, uint32_t c, uint8_t *chunk) {
    using namespace tc;
    const uint32_t bb = block_bytes(type);
    bool ok = true;
    std::memset(chunk, 0, chunk_bytes(type));
    for (uint32_t r = 0; r < kPanelRows; ++r) {
        const uint64_t row = p * kPanelRows + r;
        if (row >= n) break;
        const uint8_t *blk = rows + (row * kb + c) * bb;
        const uint32_t slot = row_slot(r);
        if (type == 12) {
            for (uint32_t s = 0; s < 4; ++s) std::memcpy(chunk + kQ4Qs + s * 4096 + slot * 32, blk + 16 + 32 * s, 32);
            std::memcpy(chunk + kQ4Sc + r * 12, blk + 4, 12);
            std::memcpy(chunk + kQ4Dm + r * 4, blk, 4);   // d, dmin (little endian, as on the device)
            ok &= finite_half(rd16(blk)) && finite_half(rd16(blk + 2));
        } else if (type == 13) {
            for (uint32_t s = 0; s < 4; ++s) std::memcpy(chunk + kQ5Qs + s * 4096 + slot * 32, blk + 48 + 32 * s, 32);
            std::memcpy(chunk + kQ5Qh + slot * 32, blk + 16, 32);
            std::memcpy(chunk + kQ5Sc + r * 12, blk + 4, 12);
            std::memcpy(chunk + kQ5Dm + r * 4, blk, 4);
            ok &= finite_half(rd16(blk)) && finite_half(rd16(blk + 2));
        } else {
            for (uint32_t h = 0; h < 2; ++h)
                for (uint32_t part = 0; part < 2; ++part)
                    std::memcpy(chunk + kQ6Ql + ((h * 2 + part) * kPanelRows + slot) * 32, blk + 64 * h + 32 * part, 32);
            for (uint32_t h = 0; h < 2; ++h) std::memcpy(chunk + kQ6Qh + (h * kPanelRows + slot) * 32, blk + 128 + 32 * h, 32);
            std::memcpy(chunk + kQ6Sc + r * 16, blk + 192, 16);
            std::memcpy(chunk + kQ6D + r * 2, blk + 208, 2);
            ok &= finite_half(rd16(blk + 208));
        }
    }
    return ok;
}

}  // namespace

extern "C" {

uint64_t tc_panel_bytes(uint32_t ggml_type, uint64_t n, uint64_t k) {
    if ((ggml_type != TC_GGML_Q4_K && ggml_type != TC_GGML_Q5_K && ggml_type != TC_GGML_Q6_K) || !n || !k ||
        k % 256)
        return 0;
    return (n + tc::kPanelRows - 1) / tc::kPanelRows * (k / 256) * tc::chunk_bytes(ggml_type);
}

int tc_relayout_host(uint32_t ggml_type, const void *raw, uint64_t raw_bytes, uint64_t n, uint64_t k,
                     uint64_t n_begin, uint64_t n_count, void *panels, uint64_t panel_bytes, int threads,
                     const volatile int32_t *cancel) {
    if (!raw || !panels) {
        tc::set_last_error("null argument");
        return TC_CUDA_FAIL;
    }
    if (n_count == 0) n_count = n - std::min(n, n_begin);
    const uint64_t need = tc_panel_bytes(ggml_type, n_count, k);
    if (!need || n_begin > n || n_count > n - n_begin) {
        tc::set_last_error("unsupported type or invalid shape / row range");
        return TC_CUDA_FAIL;
    }
    const uint32_t kb = (uint32_t)(k / 256);
    const uint64_t row_bytes = (uint64_t)kb * tc::block_bytes(ggml_type);
    if (raw_bytes / row_bytes < n) {
        tc::set_last_error("packed source too short");
        return TC_CUDA_FAIL;
    }
    if (panel_bytes < need) {
        tc::set_last_error("panel buffer too small");
        return TC_CUDA_FAIL;
    }
    const uint8_t *rows = static_cast<const uint8_t *>(raw) + n_begin * row_bytes;
    auto *out = static_cast<uint8_t *>(panels);
    const uint64_t n_panels = (n_count + tc::kPanelRows - 1) / tc::kPanelRows;
    const uint64_t total = n_panels * kb;
    std::atomic<uint64_t> next{0};
    std::atomic<bool> finite{true}, stopped{false};
    auto work = [&]() {
        for (uint64_t pc; (pc = next.fetch_add(1)) < total;) {
            // the caller's cancel flag is polled once per chunk (128 rows x 256 K)
            if (cancel && *cancel) {
                stopped = true;
                return;
            }
            if (!chunk_host(ggml_type, rows, n_count, kb, pc / kb, (uint32_t)(pc % kb),
                            out + pc * tc::chunk_bytes(ggml_type)))
                finite = false;
        }
    };
    const int t = std::max(1, std::min(threads, 64));
    std::vector<std::thread> pool;
    for (int i = 1; i < t; ++i) pool.emplace_back(work);
    work();
    for (auto &th : pool) th.join();
    if (stopped) {
        tc::set_last_error("generation cancelled");
        return TC_CUDA_CANCELLED;
    }
    if (!finite) {
        tc::set_last_error("nonfinite d/dmin in a K-quant block");
        return TC_CUDA_FAIL;
    }
    tc::set_last_error("");
    return TC_CUDA_OK;
}

int tc_cuda_weight_copy_panels(tc_cuda_ctx *ctx, tc_cuda_weight *w, const void *panels, uint64_t bytes, void *stream) {
    if (!ctx || !w || !panels) {
        tc::set_last_error("null argument");
        return TC_CUDA_FAIL;
    }
    if (bytes != w->bytes) {
        tc::set_last_error("panel bytes do not match the weight (tc_panel_bytes)");
        return TC_CUDA_FAIL;
    }
    int cur = 0;
    cudaGetDevice(&cur);
    if (cur != w->device) cudaSetDevice(w->device);
    const cudaError_t e = cudaMemcpyAsync(w->chunks, panels, bytes, cudaMemcpyDefault, static_cast<cudaStream_t>(stream));
    if (cur != w->device) cudaSetDevice(cur);
    if (e != cudaSuccess) {
        tc::set_last_error(std::string("panel copy: ") + cudaGetErrorString(e));
        return TC_CUDA_FAIL;
    }
    tc::set_last_error("");
    return TC_CUDA_OK;
}

}  // extern "C"
