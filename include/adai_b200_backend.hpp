// adai_b200_backend.hpp — the decode-path functions of the reference's GPU backend table with the
// reference's own C++ signatures (namespace adai::gpu, src/gpu/MatrixGPU.hpp:27-201), implemented
// by libadai_b200.so on the context bound with adai_b200_backend_bind(). Callers of the table
// keep their code: build against the reference's MatrixGPU.hpp (the declarations below are the
// same, so include one or the other) and link libadai_b200.so in place of MatrixGPU.cu for these
// seven functions.
//
// Semantics match the reference's (row-major device buffers, C = alpha op(A) op(B) with beta 0,
// and so on). Two differences: the products run as 3xTF32 on the tensor cores (fp32 accuracy,
// as the tests check against the CPU Matrix path), and the stream is the bound context's
// (adai_b200_ctx_stream) rather than GPUManager::get_stream(). The GEMMs wait for their result.
// The other functions are asynchronous on that stream. Failures throw std::invalid_argument,
// std::out_of_range or std::runtime_error, as CUDA_CHECK and the shape checks do
// (src/gpu/GPUUtils.hpp:54-70).
#ifndef ADAI_B200_BACKEND_HPP
#define ADAI_B200_BACKEND_HPP

#include "adai_b200.h"

namespace adai {
namespace gpu {

enum class ActivationType { RELU = 0, SIGMOID = 1, TANH = 2, GELU = 3 };

ADAI_B200_API void matrix_multiply_gpu(const float* a, const float* b, float* c, int m, int k, int n);
ADAI_B200_API void matrix_gemm_strided_gpu(bool trans_a, bool trans_b, int m, int n, int k,
                                           float alpha, const float* a, int lda, const float* b,
                                           int ldb, float* c, int ldc);
ADAI_B200_API void matrix_apply_activation_gpu(float* data, int size, ActivationType type);
ADAI_B200_API void matrix_softmax_rows_gpu(float* data, int rows, int cols);
ADAI_B200_API void matrix_layer_norm_fwd_gpu(const float* input, float* output, float* out_normed,
                                             const float* gamma, const float* beta, float* out_mean,
                                             float* out_rstd, int rows, int cols, float eps);
ADAI_B200_API void matrix_add_row_bias_gpu(const float* mat, const float* bias, float* out, int rows,
                                           int cols);
ADAI_B200_API void embedding_gather_add_pe_gpu(const float* table, const int* ids, const float* pe,
                                               int pe_rows, int pos_offset, float* out, int n, int d);

}  // namespace gpu
}  // namespace adai

#endif  // ADAI_B200_BACKEND_HPP
