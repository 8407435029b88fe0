// Dense ("passthrough") weights: the non-K-quant tensors of a GGUF K-quant
// model file -- F32 / F16 / BF16 matrices and the 32-weight block types
// Q4_0 / Q4_1 / Q5_0 / Q5_1 / Q8_0 (reference native/core/gguf_directory.hpp:
// 21-26; e.g. the Q8_0 and BF16 tensors of a Q4_K_M DiT).  They are small, K
// need not be a multiple of 256, and the reference runs them either as MLX's
// native quantised types or as dense matmuls (native/backends/mlx.cpp:680-686,
// gguf_directory.hpp native_mlx_type).
//
// Layout: the raw GGUF rows stay resident (tc_cuda_dequant decodes them with
// the bit-exact raw decoder) next to two dense row-major copies, bf16 and
// fp16, decoded once at upload by the same decoder, with a row pitch of K
// rounded up to 8 elements (16 bytes, as TMA needs).  The fp16 copy is kept
// only when every value fits fp16.  A linear on such a weight is the
// tensor-core GEMM of dense_gemm_sm100.cu with the fused epilogue; X is copied
// to a 16-byte row pitch first when K is not a multiple of 8.
#include "kq_format.cuh"
#include "tc_internal.h"

namespace tc {
namespace {

__global__ void pad_rows_kernel(const uint16_t *__restrict__ x, uint16_t *__restrict__ out, uint64_t m, uint64_t k,
                                uint64_t ld) {
    const uint64_t idx = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= m * ld) return;
    const uint64_t r = idx / ld, c = idx % ld;
    out[idx] = c < k ? x[r * k + c] : (uint16_t)0;
}

}  // namespace

bool dense_type(uint32_t type) { return type_elements(type) == 1 || type_elements(type) == 32; }

cudaError_t launch_pad_rows(const uint16_t *x, uint16_t *out, uint64_t m, uint64_t k, uint64_t ld, cudaStream_t s) {
    const uint64_t total = m * ld;
    if (!total) return cudaSuccess;
    pad_rows_kernel<<<(unsigned)((total + 255) / 256), 256, 0, s>>>(x, out, m, k, ld);
    return cudaGetLastError();
}

}  // namespace tc
