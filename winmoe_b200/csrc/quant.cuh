// Launchers of the GGUF quant kernels (quant.cu) and the tensor-core GEMM
// (gemm_tc.cu).  All are stream-ordered and return a gdn_status.
#pragma once
#include "gdn_common.cuh"

namespace gdn {

int launch_q8_0_repack(const void* blocks, int8_t* qs, uint16_t* d, int64_t rows, int64_t cols, cudaStream_t s);
int launch_q8_0_dequant(const int8_t* qs, const uint16_t* d, float* out, int64_t rows, int64_t cols,
                        cudaStream_t s);
// y[m][n] = x[m][:] . W[n][:] on CUDA cores, dequantising in registers.
int launch_q8_0_gemv(const int8_t* qs, const uint16_t* d, int64_t n, int64_t k, const void* x, int x_dtype,
                     int64_t m, float* y, cudaStream_t s);
int launch_q4_k_dequant(const void* blocks, float* out, int64_t rows, int64_t cols, cudaStream_t s);
int launch_q4_k_gemv(const void* blocks, int64_t n, int64_t k, const void* x, int x_dtype, int64_t m, float* y,
                     cudaStream_t s);

// Tensor-core (tcgen05) Q8_0 GEMM: y[m][n] = a[m][:] . W[n][:], a fp16
// [m][k] row-major (k % 64 == 0, 16-byte aligned rows), fp32 out.
int launch_q8_0_gemm_tc(const int8_t* qs, const uint16_t* d, int64_t n, int64_t k, const __half* a, int64_t m,
                        float* y, cudaStream_t s);
// fp32 / bf16 activations -> fp16 (for the tensor-core operand).
int launch_to_f16(const void* x, int x_dtype, __half* out, int64_t count, cudaStream_t s);

}  // namespace gdn
