// backend_shim.cu — adai::gpu::matrix_*_gpu with the reference's signatures
// (include/adai_b200_backend.hpp), forwarding to the C ABI on the bound context.
#include <atomic>
#include <stdexcept>
#include <string>

#include "../../include/adai_b200.h"
#include "../../include/adai_b200_backend.hpp"

namespace {

std::atomic<adai_b200_ctx*> g_bound{nullptr};

adai_b200_ctx* bound() {
    adai_b200_ctx* c = g_bound.load();
    if (!c) throw std::runtime_error("adai_b200: no context bound (adai_b200_backend_bind)");
    return c;
}

void check(int rc) {
    if (rc == ADAI_B200_OK) return;
    const std::string msg = adai_b200_last_error();
    if (rc == ADAI_B200_ERR_INVALID_ARGUMENT) throw std::invalid_argument(msg);
    if (rc == ADAI_B200_ERR_OUT_OF_RANGE) throw std::out_of_range(msg);
    throw std::runtime_error(msg);
}

}  // namespace

extern "C" ADAI_B200_API int adai_b200_backend_bind(adai_b200_ctx* ctx) {
    g_bound.store(ctx);
    return ADAI_B200_OK;
}

namespace adai {
namespace gpu {

void matrix_multiply_gpu(const float* a, const float* b, float* c, int m, int k, int n) {
    check(adai_b200_gemm_strided(bound(), 0, 0, m, n, k, 1.0f, a, k, b, n, c, n));
}

void matrix_gemm_strided_gpu(bool trans_a, bool trans_b, int m, int n, int k, float alpha,
                             const float* a, int lda, const float* b, int ldb, float* c, int ldc) {
    check(adai_b200_gemm_strided(bound(), trans_a ? 1 : 0, trans_b ? 1 : 0, m, n, k, alpha, a, lda,
                                 b, ldb, c, ldc));
}

void matrix_apply_activation_gpu(float* data, int size, ActivationType type) {
    check(adai_b200_activation(bound(), data, size, static_cast<int>(type)));
}

void matrix_softmax_rows_gpu(float* data, int rows, int cols) {
    check(adai_b200_softmax_rows(bound(), data, rows, cols));
}

void matrix_layer_norm_fwd_gpu(const float* input, float* output, float* out_normed,
                               const float* gamma, const float* beta, float* out_mean,
                               float* out_rstd, int rows, int cols, float eps) {
    check(adai_b200_layernorm_fwd(bound(), input, output, out_normed, gamma, beta, out_mean,
                                  out_rstd, rows, cols, eps));
}

void matrix_add_row_bias_gpu(const float* mat, const float* bias, float* out, int rows, int cols) {
    check(adai_b200_add_row_bias(bound(), mat, bias, out, rows, cols));
}

void embedding_gather_add_pe_gpu(const float* table, const int* ids, const float* pe, int pe_rows,
                                 int pos_offset, float* out, int n, int d) {
    check(adai_b200_embedding_gather_add_pe(bound(), table, ids, pe, pe_rows, pos_offset, out, n, d, 0));
}

}  // namespace gpu
}  // namespace adai
