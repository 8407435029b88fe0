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
// fp16, decoded once at upload by the same decoder.  The fp16 copy is kept
// only when every value fits fp16.  A linear on such a weight is a plain
// library GEMM (cuBLAS, fp32 accumulation) followed, when the call asks for a
// fused epilogue, by the epilogue kernel below.
#include <cublas_v2.h>

#include "kq_epilogue.cuh"
#include "kq_format.cuh"
#include "tc_internal.h"

namespace tc {
namespace {

// One thread per output element, the column fastest: coalesced reads of the
// fp32 product and writes of Y.
__global__ void epi_rows_kernel(const float *__restrict__ acc, uint32_t rows, uint32_t n, EpiView e,
                                uint32_t gate_row, uint32_t m_begin, void *y, uint64_t ldy, int dt) {
    const uint64_t idx = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= (uint64_t)rows * n) return;
    const uint32_t r = (uint32_t)(idx / n), c = (uint32_t)(idx % n);
    const EpiRow er = epi_row(e, c, gate_row);
    float t = epi_act(e.flags, acc[idx] + er.bias);
    const uint64_t m = (uint64_t)m_begin + r;
    if (e.flags & TC_EPI_GATE_RESIDUAL) t = load_out(e.res, m * e.ld_res + c, dt == 0, dt == 1) + er.gate * t;
    store_out(y, m * ldy + c, t, dt == 0, dt == 1);
}

cudaDataType_t cuda_type(int dtype) {
    return dtype == 0 ? CUDA_R_32F : dtype == 1 ? CUDA_R_16F : CUDA_R_16BF;
}

}  // namespace

bool dense_type(uint32_t type) { return type_elements(type) == 1 || type_elements(type) == 32; }

cudaError_t launch_epi_rows(const float *acc, uint32_t rows, uint32_t n, const EpiView &e, uint32_t gate_row,
                            uint32_t m_begin, void *y, uint64_t ldy, int out_dtype, cudaStream_t s) {
    const uint64_t total = (uint64_t)rows * n;
    if (!total) return cudaSuccess;
    epi_rows_kernel<<<(unsigned)((total + 255) / 256), 256, 0, s>>>(acc, rows, n, e, gate_row, m_begin, y, ldy,
                                                                  out_dtype);
    return cudaGetLastError();
}

// Y[rows, n] (+ ldy) = X[rows, k] * W^T on `s`: X and W both bf16 (x_f16 = 0)
// or both fp16; Y in out_dtype (TC_DTYPE_*), fp32 accumulation.
int dense_gemm(void *blas, const void *w, const void *x, int x_f16, uint32_t rows, uint32_t n, uint64_t k, void *y,
               uint64_t ldy, int out_dtype, cudaStream_t s) {
    auto h = static_cast<cublasHandle_t>(blas);
    if (cublasSetStream(h, s) != CUBLAS_STATUS_SUCCESS) return 1;
    const float one = 1.f, zero = 0.f;
    const cudaDataType_t in = x_f16 ? CUDA_R_16F : CUDA_R_16BF;
    // Column-major view: Y^T[n, rows] = W[n, k] (row-major = (k x n)^T) * X^T.
    const cublasStatus_t st = cublasGemmEx(h, CUBLAS_OP_T, CUBLAS_OP_N, (int)n, (int)rows, (int)k, &one, w, in,
                                           (int)k, x, in, (int)k, &zero, y, cuda_type(out_dtype), (int)ldy,
                                           CUBLAS_COMPUTE_32F, CUBLAS_GEMM_DEFAULT);
    return st == CUBLAS_STATUS_SUCCESS ? 0 : 1;
}

int dense_blas_create(void **blas) {
    cublasHandle_t h = nullptr;
    if (cublasCreate(&h) != CUBLAS_STATUS_SUCCESS) return 1;
    *blas = h;
    return 0;
}

void dense_blas_destroy(void *blas) {
    if (blas) cublasDestroy(static_cast<cublasHandle_t>(blas));
}

}  // namespace tc
