// backend_ops.cu — the row and elementwise operations of the reference's GPU backend table
// (adai::gpu::matrix_*_gpu, src/gpu/MatrixGPU.hpp:43-201) that sit on the decode path, for callers
// of that table outside the fused decode step: softmax over rows, LayerNorm forward with its
// statistics, row-bias add, the four activations, embedding gather + positional row. Each kernel
// is memory-bound: one pass over its data (two for the row reductions, which re-read the row from
// L2).
#include <algorithm>

#include "common.cuh"
#include "kernels.h"

namespace adai_b200 {
namespace {

constexpr int kRowThreads = 256;

__device__ __forceinline__ float block_reduce_sum(float v, float* scratch) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) scratch[warp] = v;
    __syncthreads();
    float t = (threadIdx.x < blockDim.x / 32) ? scratch[threadIdx.x] : 0.f;
    if (warp == 0) {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
        if (lane == 0) scratch[32] = t;
    }
    __syncthreads();
    const float r = scratch[32];
    __syncthreads();  // scratch is reused by the next reduction
    return r;
}

__device__ __forceinline__ float block_reduce_max(float v, float* scratch) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) scratch[warp] = v;
    __syncthreads();
    float t = (threadIdx.x < blockDim.x / 32) ? scratch[threadIdx.x] : -INFINITY;
    if (warp == 0) {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) t = fmaxf(t, __shfl_xor_sync(0xffffffffu, t, o));
        if (lane == 0) scratch[32] = t;
    }
    __syncthreads();
    const float r = scratch[32];
    __syncthreads();
    return r;
}

// Activation::softmax_row (src/Activation.cpp:12-31): subtract the row maximum, exponentiate,
// divide by the sum when the sum is positive (a row of -inf stays all zeros).
__global__ void __launch_bounds__(kRowThreads) softmax_rows_kernel(float* __restrict__ data, int cols) {
    __shared__ float scratch[33];
    float* row = data + static_cast<size_t>(blockIdx.x) * cols;
    float mx = -INFINITY;
    for (int j = threadIdx.x; j < cols; j += blockDim.x) mx = fmaxf(mx, row[j]);
    mx = block_reduce_max(mx, scratch);
    float sum = 0.f;
    for (int j = threadIdx.x; j < cols; j += blockDim.x) {
        const float e = expf(row[j] - mx);
        row[j] = e;
        sum += e;
    }
    sum = block_reduce_sum(sum, scratch);
    if (sum > 0.f)
        for (int j = threadIdx.x; j < cols; j += blockDim.x) row[j] = row[j] / sum;
}

// LayerNorm::forward (src/LayerNorm.cpp:56-109), any width: two-pass mean and biased variance,
// rstd = 1 / sqrt(var + eps); optional normalised copy and per-row statistics as
// matrix_layer_norm_fwd_gpu returns them.
__global__ void __launch_bounds__(kRowThreads) layernorm_rows_kernel(
    const float* __restrict__ x, float* __restrict__ y, float* __restrict__ xn,
    const float* __restrict__ g, const float* __restrict__ b, float* __restrict__ mean_out,
    float* __restrict__ rstd_out, int cols, float eps) {
    __shared__ float scratch[33];
    const size_t off = static_cast<size_t>(blockIdx.x) * cols;
    const float* xr = x + off;
    float s = 0.f;
    for (int j = threadIdx.x; j < cols; j += blockDim.x) s += xr[j];
    const float mean = block_reduce_sum(s, scratch) / static_cast<float>(cols);
    float v = 0.f;
    for (int j = threadIdx.x; j < cols; j += blockDim.x) {
        const float d = xr[j] - mean;
        v += d * d;
    }
    const float var = block_reduce_sum(v, scratch) / static_cast<float>(cols);
    const float rstd = 1.0f / sqrtf(var + eps);
    if (threadIdx.x == 0) {
        if (mean_out) mean_out[blockIdx.x] = mean;
        if (rstd_out) rstd_out[blockIdx.x] = rstd;
    }
    for (int j = threadIdx.x; j < cols; j += blockDim.x) {
        const float n = (xr[j] - mean) * rstd;
        if (xn) xn[off + j] = n;
        y[off + j] = n * g[j] + b[j];
    }
}

__global__ void add_row_bias_kernel(const float* __restrict__ m, const float* __restrict__ bias,
                                    float* __restrict__ out, size_t total, int cols) {
    for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<size_t>(gridDim.x) * blockDim.x)
        out[i] = m[i] + bias[i % cols];
}

__device__ __forceinline__ float activate(float x, int type) {
    switch (type) {
        case 0: return fmaxf(0.f, x);               // ReLU
        case 1: return 1.0f / (1.0f + expf(-x));    // sigmoid
        case 2: return tanhf(x);                    // tanh
        default: return gelu_tanh(x);               // GELU, tanh form (src/Activation.cpp:69-86)
    }
}

__global__ void activation_kernel(float* __restrict__ data, size_t n, int type) {
    for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<size_t>(gridDim.x) * blockDim.x)
        data[i] = activate(data[i], type);
}

// out[i, :] = table[ids[i], :] + pe[pos_offset + i, :] (no positional row past pe_rows or
// without a table: TokenEmbedding::forward + PositionalEncoding, src/TokenEmbedding.cpp:33-59).
__global__ void embed_pe_kernel(const float* __restrict__ table, const int* __restrict__ ids,
                                const float* __restrict__ pe, int pe_rows, int pos_offset,
                                float* __restrict__ out, int n, int d, int vocab, int* err) {
    const size_t total = static_cast<size_t>(n) * d;
    for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<size_t>(gridDim.x) * blockDim.x) {
        const int r = static_cast<int>(i / d), j = static_cast<int>(i % d);
        const int id = ids[r];
        if (id < 0 || id >= vocab) {  // TokenEmbedding throws std::out_of_range
            record_error(err, kDevBadShape);
            out[i] = 0.f;
            continue;
        }
        float v = table[static_cast<size_t>(id) * d + j];
        const int pos = pos_offset + r;
        if (pe && pos >= 0 && pos < pe_rows) v += pe[static_cast<size_t>(pos) * d + j];
        out[i] = v;
    }
}

int grid_for(size_t n) {
    return static_cast<int>(std::min<size_t>((n + 255) / 256, 148 * 32));
}

}  // namespace

void launch_softmax_rows(float* data, int rows, int cols, cudaStream_t st) {
    if (rows <= 0 || cols <= 0) return;
    softmax_rows_kernel<<<rows, kRowThreads, 0, st>>>(data, cols);
}

void launch_layernorm_rows(const float* x, float* y, float* xn, const float* g, const float* b,
                           float* mean, float* rstd, int rows, int cols, float eps, cudaStream_t st) {
    if (rows <= 0 || cols <= 0) return;
    layernorm_rows_kernel<<<rows, kRowThreads, 0, st>>>(x, y, xn, g, b, mean, rstd, cols, eps);
}

void launch_add_row_bias(const float* m, const float* bias, float* out, int rows, int cols,
                         cudaStream_t st) {
    const size_t total = static_cast<size_t>(rows) * cols;
    if (total == 0) return;
    add_row_bias_kernel<<<grid_for(total), 256, 0, st>>>(m, bias, out, total, cols);
}

void launch_activation(float* data, size_t n, int type, cudaStream_t st) {
    if (n == 0) return;
    activation_kernel<<<grid_for(n), 256, 0, st>>>(data, n, type);
}

void launch_embed_pe(const float* table, const int* ids, const float* pe, int pe_rows, int pos_offset,
                     float* out, int n, int d, int vocab, int* err, cudaStream_t st) {
    const size_t total = static_cast<size_t>(n) * d;
    if (total == 0) return;
    embed_pe_kernel<<<grid_for(total), 256, 0, st>>>(table, ids, pe, pe_rows, pos_offset, out, n, d,
                                                     vocab, err);
}

}  // namespace adai_b200
