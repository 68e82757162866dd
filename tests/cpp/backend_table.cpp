// Calls the decode-path functions of the reference backend table through their reference C++
// signatures (adai::gpu::matrix_*_gpu: the reference's src/gpu/MatrixGPU.hpp when built with
// ADAI_REFERENCE_HEADERS, else include/adai_b200_backend.hpp) on a bound context, and
// checks each against a host computation. Prints "all ok" and exits 0 when every check passes.
#include <cuda_runtime.h>

#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <stdexcept>
#include <vector>

#include "adai_b200.h"
#ifdef ADAI_REFERENCE_HEADERS
// The reference's own declarations (src/gpu/MatrixGPU.hpp, built with ADAI_ENABLE_GPU): the
// program then proves that untouched callers compile against them and link to libadai_b200.so.
#include "gpu/MatrixGPU.hpp"
#else
#include "adai_b200_backend.hpp"
#endif

static int failures = 0;
static void expect(bool ok, const char* what) {
    if (!ok) {
        std::printf("FAIL %s\n", what);
        ++failures;
    }
}
static float* up(const std::vector<float>& h) {
    float* d = nullptr;
    cudaMalloc(&d, h.size() * sizeof(float) + 16);
    cudaMemcpy(d, h.data(), h.size() * sizeof(float), cudaMemcpyHostToDevice);
    return d;
}
static std::vector<float> down(const float* d, size_t n) {
    std::vector<float> h(n);
    cudaMemcpy(h.data(), d, n * sizeof(float), cudaMemcpyDeviceToHost);
    return h;
}

int main() {
    adai_b200_ctx* ctx = nullptr;
    if (adai_b200_ctx_create(0, 0.f, &ctx) != ADAI_B200_OK) {
        std::printf("no device: %s\n", adai_b200_last_error());
        return 2;
    }
    adai_b200_backend_bind(ctx);
    std::srand(7);
    auto rnd = [] { return static_cast<float>(std::rand()) / RAND_MAX * 2.f - 1.f; };

    // C = A B, [5 x 33] [33 x 19]
    const int m = 5, k = 33, n = 19;
    std::vector<float> A(m * k), B(k * n);
    for (auto& v : A) v = rnd();
    for (auto& v : B) v = rnd();
    float *dA = up(A), *dB = up(B), *dC = up(std::vector<float>(m * n, 0.f));
    adai::gpu::matrix_multiply_gpu(dA, dB, dC, m, k, n);
    std::vector<float> C = down(dC, m * n);
    bool ok = true;
    for (int i = 0; i < m; ++i)
        for (int j = 0; j < n; ++j) {
            double s = 0, sa = 0;
            for (int t = 0; t < k; ++t) {
                s += static_cast<double>(A[i * k + t]) * B[t * n + j];
                sa += std::fabs(static_cast<double>(A[i * k + t]) * B[t * n + j]);
            }
            ok = ok && std::fabs(C[i * n + j] - s) <= 1e-5 + 1e-5 * sa;
        }
    expect(ok, "matrix_multiply_gpu");

    // C = 0.5 A^T B^T with A stored [k x m], B stored [n x k]
    std::vector<float> At(k * m), Bt(n * k);
    for (int i = 0; i < m; ++i)
        for (int t = 0; t < k; ++t) At[t * m + i] = A[i * k + t];
    for (int t = 0; t < k; ++t)
        for (int j = 0; j < n; ++j) Bt[j * k + t] = B[t * n + j];
    float *dAt = up(At), *dBt = up(Bt);
    adai::gpu::matrix_gemm_strided_gpu(true, true, m, n, k, 0.5f, dAt, m, dBt, k, dC, n);
    std::vector<float> C2 = down(dC, m * n);
    ok = true;
    for (int i = 0; i < m * n; ++i) ok = ok && std::fabs(C2[i] - 0.5f * C[i]) <= 1e-5f + 1e-6f * std::fabs(C[i]);
    expect(ok, "matrix_gemm_strided_gpu");

    // softmax rows, LayerNorm, bias, activation, embedding
    const int rows = 3, cols = 130;
    std::vector<float> X(rows * cols), g(cols), b(cols);
    for (auto& v : X) v = 3.f * rnd();
    for (int j = 0; j < cols; ++j) {
        g[j] = 1.f + 0.5f * rnd();
        b[j] = 0.2f * rnd();
    }
    float *dX = up(X), *dg = up(g), *db = up(b), *dY = up(X), *dN = up(X);
    float *dmean = up(std::vector<float>(rows)), *drstd = up(std::vector<float>(rows));
    adai::gpu::matrix_layer_norm_fwd_gpu(dX, dY, dN, dg, db, dmean, drstd, rows, cols, 1e-5f);
    cudaDeviceSynchronize();
    std::vector<float> Y = down(dY, rows * cols);
    ok = true;
    for (int r = 0; r < rows; ++r) {
        double mu = 0, var = 0;
        for (int j = 0; j < cols; ++j) mu += X[r * cols + j];
        mu /= cols;
        for (int j = 0; j < cols; ++j) var += (X[r * cols + j] - mu) * (X[r * cols + j] - mu);
        const double rs = 1.0 / std::sqrt(var / cols + 1e-5);
        for (int j = 0; j < cols; ++j) {
            const double want = (X[r * cols + j] - mu) * rs * g[j] + b[j];
            ok = ok && std::fabs(Y[r * cols + j] - want) <= 1e-5 + 1e-4 * std::fabs(want);
        }
    }
    expect(ok, "matrix_layer_norm_fwd_gpu");

    adai::gpu::matrix_softmax_rows_gpu(dX, rows, cols);
    cudaDeviceSynchronize();
    std::vector<float> S = down(dX, rows * cols);
    ok = true;
    for (int r = 0; r < rows; ++r) {
        double mx = -1e30, sum = 0;
        for (int j = 0; j < cols; ++j) mx = std::fmax(mx, X[r * cols + j]);
        for (int j = 0; j < cols; ++j) sum += std::exp(X[r * cols + j] - mx);
        for (int j = 0; j < cols; ++j) {
            const double want = std::exp(X[r * cols + j] - mx) / sum;
            ok = ok && std::fabs(S[r * cols + j] - want) <= 1e-5 + 1e-4 * want;
        }
    }
    expect(ok, "matrix_softmax_rows_gpu");

    float* dO = up(std::vector<float>(rows * cols));
    float* dY2 = up(Y);
    adai::gpu::matrix_add_row_bias_gpu(dY2, db, dO, rows, cols);
    adai::gpu::matrix_apply_activation_gpu(dO, rows * cols, adai::gpu::ActivationType::RELU);
    cudaDeviceSynchronize();
    std::vector<float> O = down(dO, rows * cols);
    ok = true;
    for (int i = 0; i < rows * cols; ++i) ok = ok && O[i] == std::fmax(0.f, Y[i] + b[i % cols]);
    expect(ok, "matrix_add_row_bias_gpu + matrix_apply_activation_gpu(RELU)");

    std::vector<float> table(10 * cols), pe(2 * cols);
    for (auto& v : table) v = rnd();
    for (auto& v : pe) v = rnd();
    std::vector<int> ids = {4, 9, 0};
    int* dids = nullptr;
    cudaMalloc(&dids, ids.size() * sizeof(int));
    cudaMemcpy(dids, ids.data(), ids.size() * sizeof(int), cudaMemcpyHostToDevice);
    float *dt = up(table), *dpe = up(pe), *dE = up(std::vector<float>(3 * cols));
    adai::gpu::embedding_gather_add_pe_gpu(dt, dids, dpe, 2, 1, dE, 3, cols);
    cudaDeviceSynchronize();
    std::vector<float> E = down(dE, 3 * cols);
    ok = true;
    for (int i = 0; i < 3; ++i)
        for (int j = 0; j < cols; ++j) {
            float want = table[ids[i] * cols + j];
            if (1 + i < 2) want += pe[(1 + i) * cols + j];
            ok = ok && E[i * cols + j] == want;
        }
    expect(ok, "embedding_gather_add_pe_gpu");

    // an unbound backend throws
    adai_b200_backend_bind(nullptr);
    bool threw = false;
    try {
        adai::gpu::matrix_softmax_rows_gpu(dX, rows, cols);
    } catch (const std::runtime_error&) {
        threw = true;
    }
    expect(threw, "unbound backend throws");
    adai_b200_ctx_destroy(ctx);
    if (failures == 0) std::printf("all ok\n");
    return failures == 0 ? 0 : 1;
}
