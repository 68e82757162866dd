// kernels.cu — the bandwidth-bound kernels of the decode step (sm_100a, no tensor cores):
//   * single-query decode attention over the KV cache, self-attention append fused in
//     (reference: MultiHeadAttention::forward_with_cache, src/MultiHeadAttention.cpp:278-395;
//      CrossAttention::forward_with_cache, src/CrossAttention.cpp:343-486; KVCache::append,
//      src/KVCache.hpp:99-128; softmax_row, src/Activation.cpp:12-31)
//   * encoder prefill attention over ragged sequences (src/MultiHeadAttention.cpp:176-240)
//   * LayerNorm (src/LayerNorm.cpp:56-109), fused with the token embedding + positional row for
//     the first one (src/Decoder.cpp:224-243, src/TokenEmbedding.cpp:33-59)
//   * the tf32 operand split and the weight transpose-split used at upload.
#include <algorithm>

#include "common.cuh"
#include "kernels.h"

namespace adai_b200 {

namespace {

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// ---------------------------------------------------------------------------------------------
__global__ void split_kernel(const float* __restrict__ x, float* __restrict__ hi,
                             float* __restrict__ lo, size_t n) {
    for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<size_t>(gridDim.x) * blockDim.x) {
        float h, l;
        split_tf32(x[i], h, l);
        hi[i] = h;
        lo[i] = l;
    }
}

// w [K, N] row-major -> hi_t / lo_t [N, K] row-major (tf32 split), 32x32 tiles through smem.
__global__ void transpose_split_kernel(const float* __restrict__ w, int K, int N,
                                       float* __restrict__ hi_t, float* __restrict__ lo_t) {
    __shared__ float tile[32][33];
    const int n0 = blockIdx.x * 32, k0 = blockIdx.y * 32;
    for (int i = threadIdx.y; i < 32; i += blockDim.y) {
        const int k = k0 + i, n = n0 + threadIdx.x;
        tile[i][threadIdx.x] = (k < K && n < N) ? w[static_cast<size_t>(k) * N + n] : 0.f;
    }
    __syncthreads();
    for (int i = threadIdx.y; i < 32; i += blockDim.y) {
        const int n = n0 + i, k = k0 + threadIdx.x;
        if (n < N && k < K) {
            float h, l;
            split_tf32(tile[threadIdx.x][i], h, l);
            hi_t[static_cast<size_t>(n) * K + k] = h;
            lo_t[static_cast<size_t>(n) * K + k] = l;
        }
    }
}

// ---------------------------------------------------------------------------------------------
// LayerNorm, one warp per row, the row held in registers (NV float4 per lane, D = 128 * NV).
// Two passes like the reference: mean, then the biased variance of (x - mean); eps = 1e-5.
template <int NV>
__device__ __forceinline__ void ln_row_regs(float4 (&xv)[NV], const float* __restrict__ g,
                                            const float* __restrict__ b, int D, int lane,
                                            float* out, float* out_hi, float* out_lo) {
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < NV; ++i) s += (xv[i].x + xv[i].y) + (xv[i].z + xv[i].w);
    const float mean = warp_sum(s) / static_cast<float>(D);
    float v = 0.f;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
        const float a = xv[i].x - mean, bb = xv[i].y - mean, c = xv[i].z - mean,
                    d = xv[i].w - mean;
        v += (a * a + bb * bb) + (c * c + d * d);
    }
    const float var = warp_sum(v) / static_cast<float>(D);
    const float inv_std = 1.0f / sqrtf(var + 1e-5f);
#pragma unroll
    for (int i = 0; i < NV; ++i) {
        const int c0 = (i * 32 + lane) * 4;
        const float4 gg = *reinterpret_cast<const float4*>(g + c0);
        const float4 bv = *reinterpret_cast<const float4*>(b + c0);
        float4 o;
        o.x = gg.x * ((xv[i].x - mean) * inv_std) + bv.x;
        o.y = gg.y * ((xv[i].y - mean) * inv_std) + bv.y;
        o.z = gg.z * ((xv[i].z - mean) * inv_std) + bv.z;
        o.w = gg.w * ((xv[i].w - mean) * inv_std) + bv.w;
        if (out) *reinterpret_cast<float4*>(out + c0) = o;
        if (out_hi) {
            float4 h, l;
            split_tf32(o.x, h.x, l.x);
            split_tf32(o.y, h.y, l.y);
            split_tf32(o.z, h.z, l.z);
            split_tf32(o.w, h.w, l.w);
            *reinterpret_cast<float4*>(out_hi + c0) = h;
            *reinterpret_cast<float4*>(out_lo + c0) = l;
        }
    }
}

template <int NV>
__global__ void layernorm_kernel(const float* __restrict__ x, int ldx,
                                 const float* __restrict__ g, const float* __restrict__ b,
                                 float* out, float* out_hi, float* out_lo, int rows, int D) {
    pdl_trigger();
    pdl_wait();
    const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (row >= rows) return;
    float4 xv[NV];
    const float* xr = x + static_cast<size_t>(row) * ldx;
#pragma unroll
    for (int i = 0; i < NV; ++i) xv[i] = *reinterpret_cast<const float4*>(xr + (i * 32 + lane) * 4);
    const size_t o = static_cast<size_t>(row) * D;
    ln_row_regs<NV>(xv, g, b, D, lane, out ? out + o : nullptr, out_hi ? out_hi + o : nullptr,
                    out_lo ? out_lo + o : nullptr);
}

template <int NV>
__global__ void embed_ln_kernel(const float* __restrict__ table, const int* __restrict__ ids,
                                const float* __restrict__ pe, int pe_rows,
                                const int* __restrict__ slots, const int* __restrict__ pos_by_slot,
                                const int* __restrict__ pos_direct, float* __restrict__ x,
                                const float* __restrict__ g, const float* __restrict__ b,
                                float* out_hi, float* out_lo, int rows, int D, int vocab,
                                int* err) {
    pdl_trigger();
    pdl_wait();
    const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (row >= rows) return;
    int id = ids[row];
    if (id < 0 || id >= vocab) {  // TokenEmbedding::forward throws std::out_of_range here
        if (lane == 0) record_error(err, kDevBadShape);
        id = 0;
    }
    const int pos = pos_by_slot ? pos_by_slot[slots ? slots[row] : row] : pos_direct[row];
    const float* er = table + static_cast<size_t>(id) * D;
    const bool has_pe = pos >= 0 && pos < pe_rows;
    const float* pr = pe + static_cast<size_t>(has_pe ? pos : 0) * D;
    float4 xv[NV];
#pragma unroll
    for (int i = 0; i < NV; ++i) {
        const int c0 = (i * 32 + lane) * 4;
        float4 e = *reinterpret_cast<const float4*>(er + c0);
        if (has_pe) {
            const float4 p = *reinterpret_cast<const float4*>(pr + c0);
            e.x += p.x;
            e.y += p.y;
            e.z += p.z;
            e.w += p.w;
        }
        xv[i] = e;
        *reinterpret_cast<float4*>(x + static_cast<size_t>(row) * D + c0) = e;
    }
    const size_t o = static_cast<size_t>(row) * D;
    ln_row_regs<NV>(xv, g, b, D, lane, nullptr, out_hi + o, out_lo + o);
}

// The decode step's embedding when the first LayerNorm is folded into the Q|K|V GEMM:
// x[r] = table[ids[r]] + pe[pos(r)], its tf32 split, and per 32-column group the statistics
// (sum, squared deviations from the group mean) that the GEMM combines into mean and rstd.
template <int NV>
__global__ void embed_stats_kernel(const float* __restrict__ table, const int* __restrict__ ids,
                                   const float* __restrict__ pe, int pe_rows,
                                   const int* __restrict__ slots, const int* __restrict__ pos_by_slot,
                                   float* __restrict__ x, float* x_hi, float* x_lo,
                                   float2* __restrict__ stats, int rows, int D, int vocab,
                                   int* err) {
    pdl_trigger();
    pdl_wait();
    const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (row >= rows) return;
    int id = ids[row];
    if (id < 0 || id >= vocab) {  // TokenEmbedding::forward throws std::out_of_range here
        if (lane == 0) record_error(err, kDevBadShape);
        id = 0;
    }
    const int pos = pos_by_slot[slots ? slots[row] : row];
    const float* er = table + static_cast<size_t>(id) * D;
    const bool has_pe = pos >= 0 && pos < pe_rows;
    const float* pr = pe + static_cast<size_t>(has_pe ? pos : 0) * D;
    const unsigned seg = 0xFFu << (lane & 24);
#pragma unroll
    for (int i = 0; i < NV; ++i) {
        const int c0 = (i * 32 + lane) * 4;
        float4 e = *reinterpret_cast<const float4*>(er + c0);
        if (has_pe) {
            const float4 p = *reinterpret_cast<const float4*>(pr + c0);
            e.x += p.x;
            e.y += p.y;
            e.z += p.z;
            e.w += p.w;
        }
        const size_t o = static_cast<size_t>(row) * D + c0;
        *reinterpret_cast<float4*>(x + o) = e;
        float4 h, l;
        split_tf32(e.x, h.x, l.x);
        split_tf32(e.y, h.y, l.y);
        split_tf32(e.z, h.z, l.z);
        split_tf32(e.w, h.w, l.w);
        *reinterpret_cast<float4*>(x_hi + o) = h;
        *reinterpret_cast<float4*>(x_lo + o) = l;
        // lanes 8j..8j+7 hold columns [32(4i+j), 32(4i+j) + 32): one group
        float sg = (e.x + e.y) + (e.z + e.w);
        sg += __shfl_xor_sync(seg, sg, 1);
        sg += __shfl_xor_sync(seg, sg, 2);
        sg += __shfl_xor_sync(seg, sg, 4);
        const float mg = sg * (1.0f / 32.0f);
        const float a = e.x - mg, b = e.y - mg, c = e.z - mg, d = e.w - mg;
        float q = (a * a + b * b) + (c * c + d * d);
        q += __shfl_xor_sync(seg, q, 1);
        q += __shfl_xor_sync(seg, q, 2);
        q += __shfl_xor_sync(seg, q, 4);
        if ((lane & 7) == 0)
            stats[static_cast<size_t>(row) * (D >> 5) + (c0 >> 5)] = make_float2(sg, q);
    }
}

// ---------------------------------------------------------------------------------------------
// Decode attention, templated on the head width DH (32 or 64). One CTA per (chunk of a.chunk
// cached rows, head, batch row), 4 warps. A row of one head is DH floats = LPR lanes x float4, so
// a warp covers RPW = 32 / LPR rows per load and the CTA 4 * RPW consecutive rows (contiguous
// bytes in the [slot][head][row][DH] cache). Online softmax per row group of lanes, merged across
// row groups, warps and (through scratch) chunks in a fixed order.
constexpr int kAttnWarps = 4;
constexpr int kAttnUnroll = 4;

__device__ __forceinline__ void merge_into(float& m, float& l, float4& acc, float m2, float l2,
                                           float4 acc2) {
    const float mm = fmaxf(m, m2);
    const float c1 = (m == -INFINITY) ? 0.f : expf(m - mm);
    const float c2 = (m2 == -INFINITY) ? 0.f : expf(m2 - mm);
    l = l * c1 + l2 * c2;
    acc.x = acc.x * c1 + acc2.x * c2;
    acc.y = acc.y * c1 + acc2.y * c2;
    acc.z = acc.z * c1 + acc2.z * c2;
    acc.w = acc.w * c1 + acc2.w * c2;
    m = mm;
}

template <int DH>
__device__ __forceinline__ void write_out(const DecodeAttnArgs& a, int b, int h, int l, float4 o) {
    const size_t off = static_cast<size_t>(b) * a.ldo + h * DH + l * 4;
    if (a.out) *reinterpret_cast<float4*>(a.out + off) = o;
    if (a.out_hi) {
        float4 hi, lo;
        split_tf32(o.x, hi.x, lo.x);
        split_tf32(o.y, hi.y, lo.y);
        split_tf32(o.z, hi.z, lo.z);
        split_tf32(o.w, hi.w, lo.w);
        *reinterpret_cast<float4*>(a.out_hi + off) = hi;
        *reinterpret_cast<float4*>(a.out_lo + off) = lo;
    }
}

template <int DH>
__global__ void __launch_bounds__(kAttnWarps * 32, 8) decode_attention_kernel(const __grid_constant__ DecodeAttnArgs a) {
    constexpr int LPR = DH / 4;        // lanes per cached row
    constexpr int RPW = 32 / LPR;      // rows per warp per load
    constexpr int G = kAttnWarps * RPW;  // consecutive rows per CTA per load
    constexpr unsigned kRowMask = (LPR == 32) ? 0xffffffffu : ((1u << LPR) - 1u);
    pdl_trigger();
    // Before the wait for the preceding kernel: the slot table, the cached lengths and the rows
    // cached before this step were all written before this step's first kernel (the lengths
    // advance only after the step's last GEMM), so the first batch of rows is requested now.
    // The appended row, q and the output are touched only after the wait.
    const int c = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
    const int slot = a.slots ? a.slots[b] : b;
    const int len = a.len_by_slot[slot] + a.len_add;
    // A length the grid and the scratch were not sized for (or past the cache) is refused before
    // any load, append or merge ticket: every CTA of the pair sees the same length and leaves, so
    // the tickets stay at zero and nothing outside the cache is written.
    if (len < a.len_add || len > a.max_len || len > a.cap) {
        if (c == 0 && threadIdx.x == 0) record_error(a.err, kDevAttnLength);
        return;
    }
    const int chunk = a.chunk;
    const int nch = (len + chunk - 1) / chunk;
    // A CTA past the last chunk of its row (the grid is sized for the capacity) touches nothing:
    // it leaves at once instead of holding a slot until the preceding kernel completes.
    if (c >= max(nch, 1)) return;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int rsub = lane / LPR, l = lane % LPR;
    const int r0 = c * chunk;
    const int r1 = min(len, r0 + chunk);
    const int pre_end = min(r1, len - a.len_add);  // rows cached before this step
    float* Kh = a.kc + static_cast<long long>(slot) * a.slot_stride + static_cast<long long>(h) * a.cap * DH;
    float* Vh = a.vc + static_cast<long long>(slot) * a.slot_stride + static_cast<long long>(h) * a.cap * DH;
    float4 kk0[kAttnUnroll], vv0[kAttnUnroll];
    {
        const int base = r0 + warp * RPW + rsub;
#pragma unroll
        for (int u = 0; u < kAttnUnroll; ++u) {
            const int r = base + G * u;
            if (len > 0 && c < nch && r < pre_end) {
                kk0[u] = __ldcs(reinterpret_cast<const float4*>(Kh + static_cast<size_t>(r) * DH + l * 4));
                vv0[u] = __ldcs(reinterpret_cast<const float4*>(Vh + static_cast<size_t>(r) * DH + l * 4));
            } else {
                kk0[u] = make_float4(0.f, 0.f, 0.f, 0.f);
                vv0[u] = kk0[u];
            }
        }
    }
    pdl_wait();
    if (len <= 0) {
        // No cached rows: the reference's softmax over an empty row leaves nothing; output 0.
        if (c == 0 && warp == 0 && rsub == 0) write_out<DH>(a, b, h, l, make_float4(0.f, 0.f, 0.f, 0.f));
        return;
    }
    if (c >= nch) return;
    const float4 q = *reinterpret_cast<const float4*>(a.q + static_cast<size_t>(b) * a.ldq + h * DH + l * 4);

    // Fused KV append: the CTA whose chunk holds the new row writes it (KVCache::append).
    if (a.k_new && (len - 1) / chunk == c) {
        const int t = len - 1;
        if (threadIdx.x < LPR) {
            const float4 kv = *reinterpret_cast<const float4*>(a.k_new + static_cast<size_t>(b) * a.ldkv + h * DH + threadIdx.x * 4);
            *reinterpret_cast<float4*>(Kh + static_cast<size_t>(t) * DH + threadIdx.x * 4) = kv;
        } else if (threadIdx.x < 2 * LPR) {
            const int i = threadIdx.x - LPR;
            const float4 vv = *reinterpret_cast<const float4*>(a.v_new + static_cast<size_t>(b) * a.ldkv + h * DH + i * 4);
            *reinterpret_cast<float4*>(Vh + static_cast<size_t>(t) * DH + i * 4) = vv;
        }
        __syncthreads();
    }

    float m = -INFINITY, lsum = 0.f;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);

    // One batch of kAttnUnroll row groups: scores, online softmax, weighted V.
    auto batch = [&](const float4 (&kk)[kAttnUnroll], const float4 (&vv)[kAttnUnroll], int base) {
        float s[kAttnUnroll];
#pragma unroll
        for (int u = 0; u < kAttnUnroll; ++u) {
            float d = q.x * kk[u].x;
            d = fmaf(q.y, kk[u].y, d);
            d = fmaf(q.z, kk[u].z, d);
            d = fmaf(q.w, kk[u].w, d);
#pragma unroll
            for (int o = LPR / 2; o > 0; o >>= 1) d += __shfl_xor_sync(0xffffffffu, d, o);
            s[u] = (base + G * u < r1) ? d * a.scale : -INFINITY;
        }
        float mu = m;
#pragma unroll
        for (int u = 0; u < kAttnUnroll; ++u) mu = fmaxf(mu, s[u]);
        const float corr = (m == -INFINITY) ? 0.f : expf(m - mu);
        lsum *= corr;
        acc.x *= corr;
        acc.y *= corr;
        acc.z *= corr;
        acc.w *= corr;
#pragma unroll
        for (int u = 0; u < kAttnUnroll; ++u) {
            const float pu = (s[u] == -INFINITY) ? 0.f : expf(s[u] - mu);
            lsum += pu;
            acc.x = fmaf(pu, vv[u].x, acc.x);
            acc.y = fmaf(pu, vv[u].y, acc.y);
            acc.z = fmaf(pu, vv[u].z, acc.z);
            acc.w = fmaf(pu, vv[u].w, acc.w);
        }
        m = mu;
    };
    // The loop bound (gb) is warp-uniform, so every shuffle has all 32 lanes present. The first
    // batch was requested before the wait, except rows appended by this step.
    const int gb0 = r0 + warp * RPW;
    if (gb0 < r1) {
        const int base = gb0 + rsub;
#pragma unroll
        for (int u = 0; u < kAttnUnroll; ++u) {
            const int r = base + G * u;
            if (r >= pre_end && r < r1) {
                kk0[u] = __ldcs(reinterpret_cast<const float4*>(Kh + static_cast<size_t>(r) * DH + l * 4));
                vv0[u] = __ldcs(reinterpret_cast<const float4*>(Vh + static_cast<size_t>(r) * DH + l * 4));
            }
        }
        batch(kk0, vv0, base);
    }
    for (int gb = gb0 + G * kAttnUnroll; gb < r1; gb += G * kAttnUnroll) {
        const int base = gb + rsub;
        float4 kk[kAttnUnroll], vv[kAttnUnroll];
#pragma unroll
        for (int u = 0; u < kAttnUnroll; ++u) {
            const int r = base + G * u;
            if (r < r1) {
                kk[u] = __ldcs(reinterpret_cast<const float4*>(Kh + static_cast<size_t>(r) * DH + l * 4));
                vv[u] = __ldcs(reinterpret_cast<const float4*>(Vh + static_cast<size_t>(r) * DH + l * 4));
            } else {
                kk[u] = make_float4(0.f, 0.f, 0.f, 0.f);
                vv[u] = kk[u];
            }
        }
        batch(kk, vv, base);
    }
    // merge the warp's row groups (lanes l, l+LPR, l+2LPR, ... hold the same output dims)
#pragma unroll
    for (int o = LPR; o < 32; o <<= 1) {
        const float m2 = __shfl_xor_sync(0xffffffffu, m, o);
        const float l2 = __shfl_xor_sync(0xffffffffu, lsum, o);
        float4 a2;
        a2.x = __shfl_xor_sync(0xffffffffu, acc.x, o);
        a2.y = __shfl_xor_sync(0xffffffffu, acc.y, o);
        a2.z = __shfl_xor_sync(0xffffffffu, acc.z, o);
        a2.w = __shfl_xor_sync(0xffffffffu, acc.w, o);
        merge_into(m, lsum, acc, m2, l2, a2);
    }
    __shared__ float sm_m[kAttnWarps], sm_l[kAttnWarps];
    __shared__ float4 sm_acc[kAttnWarps][LPR];
    if (rsub == 0) {
        sm_acc[warp][l] = acc;
        if (l == 0) {
            sm_m[warp] = m;
            sm_l[warp] = lsum;
        }
    }
    __syncthreads();
    if (warp != 0 || rsub != 0) return;
    float M = sm_m[0], L = sm_l[0];
    float4 A = sm_acc[0][l];
#pragma unroll
    for (int w = 1; w < kAttnWarps; ++w) merge_into(M, L, A, sm_m[w], sm_l[w], sm_acc[w][l]);

    if (nch == 1) {
        const float inv = 1.0f / L;
        write_out<DH>(a, b, h, l, make_float4(A.x * inv, A.y * inv, A.z * inv, A.w * inv));
        return;
    }
    // Split-KV: publish this chunk's partial; the last chunk to finish merges them in order.
    constexpr int kPart = DH + 4;  // m, l, 2 pad, DH accumulators
    const int pair = b * a.H + h;
    const int max_ch = (a.max_len + chunk - 1) / chunk;
    float* part = a.ws + (static_cast<size_t>(pair) * max_ch + c) * kPart;
    *reinterpret_cast<float4*>(part + 4 + l * 4) = A;
    if (l == 0) {
        part[0] = M;
        part[1] = L;
    }
    __threadfence();
    __syncwarp(kRowMask);
    int last = 0;
    if (l == 0) last = (atomicAdd(a.tickets + pair, 1) == nch - 1) ? 1 : 0;
    last = __shfl_sync(kRowMask, last, 0);
    if (!last) return;
    __threadfence();
    const float* p0 = a.ws + static_cast<size_t>(pair) * max_ch * kPart;
    M = __ldcg(p0 + 0);
    L = __ldcg(p0 + 1);
    A = __ldcg(reinterpret_cast<const float4*>(p0 + 4 + l * 4));
    for (int j = 1; j < nch; ++j) {
        const float* pj = p0 + static_cast<size_t>(j) * kPart;
        merge_into(M, L, A, __ldcg(pj + 0), __ldcg(pj + 1),
                   __ldcg(reinterpret_cast<const float4*>(pj + 4 + l * 4)));
    }
    const float inv = 1.0f / L;
    write_out<DH>(a, b, h, l, make_float4(A.x * inv, A.y * inv, A.z * inv, A.w * inv));
    if (l == 0) a.tickets[pair] = 0;
}

// ---------------------------------------------------------------------------------------------
// Encoder prefill attention: one thread per query row, 128 query rows per CTA, key/value tiles of
// 32 rows staged in shared memory and read as broadcasts; online softmax in blocks of 16 keys.
constexpr int kPreQ = 128;
constexpr int kPreKT = 32;

template <int DH>
__global__ void __launch_bounds__(kPreQ) prefill_attention_kernel(
    const float* __restrict__ qkv, int D, const int* __restrict__ offsets,
    const int* __restrict__ lens, float* __restrict__ out_hi, float* __restrict__ out_lo,
    float scale) {
    const int s = blockIdx.z, h = blockIdx.y;
    const int S = lens[s];
    const int q0 = blockIdx.x * kPreQ;
    if (q0 >= S) return;
    const int row0 = offsets[s];
    const int i = q0 + threadIdx.x;
    const bool active = i < S;
    const int ld = 3 * D;
    __shared__ __align__(16) float Ks[kPreKT][DH];
    __shared__ __align__(16) float Vs[kPreKT][DH];
    float q[DH], acc[DH];
    if (active) {
        const float* qr = qkv + static_cast<size_t>(row0 + i) * ld + h * DH;
#pragma unroll
        for (int j = 0; j < DH; j += 4) {
            const float4 t = *reinterpret_cast<const float4*>(qr + j);
            q[j] = t.x;
            q[j + 1] = t.y;
            q[j + 2] = t.z;
            q[j + 3] = t.w;
        }
    }
#pragma unroll
    for (int j = 0; j < DH; ++j) acc[j] = 0.f;
    float m = -INFINITY, l = 0.f;
    for (int k0 = 0; k0 < S; k0 += kPreKT) {
        __syncthreads();
        for (int e = threadIdx.x; e < kPreKT * (DH / 4); e += kPreQ) {
            const int r = e / (DH / 4), c4 = (e % (DH / 4)) * 4;
            float4 kv = make_float4(0.f, 0.f, 0.f, 0.f), vv = kv;
            if (k0 + r < S) {
                const float* base = qkv + static_cast<size_t>(row0 + k0 + r) * ld + h * DH + c4;
                kv = *reinterpret_cast<const float4*>(base + D);
                vv = *reinterpret_cast<const float4*>(base + 2 * D);
            }
            *reinterpret_cast<float4*>(&Ks[r][c4]) = kv;
            *reinterpret_cast<float4*>(&Vs[r][c4]) = vv;
        }
        __syncthreads();
        if (!active) continue;
        const int nk = min(kPreKT, S - k0);
        for (int kb = 0; kb < nk; kb += 16) {
            float sc[16];
            float mu = m;
#pragma unroll
            for (int u = 0; u < 16; ++u) {
                float d = 0.f;
#pragma unroll
                for (int j = 0; j < DH; j += 4) {
                    const float4 kk = *reinterpret_cast<const float4*>(&Ks[kb + u][j]);
                    d = fmaf(q[j], kk.x, d);
                    d = fmaf(q[j + 1], kk.y, d);
                    d = fmaf(q[j + 2], kk.z, d);
                    d = fmaf(q[j + 3], kk.w, d);
                }
                sc[u] = (kb + u < nk) ? d * scale : -INFINITY;
                mu = fmaxf(mu, sc[u]);
            }
            const float corr = (m == -INFINITY) ? 0.f : expf(m - mu);
            l *= corr;
#pragma unroll
            for (int j = 0; j < DH; ++j) acc[j] *= corr;
#pragma unroll
            for (int u = 0; u < 16; ++u) {
                const float p = (sc[u] == -INFINITY) ? 0.f : expf(sc[u] - mu);
                l += p;
#pragma unroll
                for (int j = 0; j < DH; j += 4) {
                    const float4 vv = *reinterpret_cast<const float4*>(&Vs[kb + u][j]);
                    acc[j] = fmaf(p, vv.x, acc[j]);
                    acc[j + 1] = fmaf(p, vv.y, acc[j + 1]);
                    acc[j + 2] = fmaf(p, vv.z, acc[j + 2]);
                    acc[j + 3] = fmaf(p, vv.w, acc[j + 3]);
                }
            }
            m = mu;
        }
    }
    if (!active) return;
    const float inv = 1.0f / l;
    const size_t o = static_cast<size_t>(row0 + i) * D + h * DH;
#pragma unroll
    for (int j = 0; j < DH; j += 4) {
        float4 hi, lo;
        split_tf32(acc[j] * inv, hi.x, lo.x);
        split_tf32(acc[j + 1] * inv, hi.y, lo.y);
        split_tf32(acc[j + 2] * inv, hi.z, lo.z);
        split_tf32(acc[j + 3] * inv, hi.w, lo.w);
        *reinterpret_cast<float4*>(out_hi + o + j) = hi;
        *reinterpret_cast<float4*>(out_lo + o + j) = lo;
    }
}

__global__ void advance_kernel(const int* __restrict__ next, int* __restrict__ ids,
                               const int* __restrict__ slots, int* __restrict__ len_by_slot,
                               int B) {
    pdl_trigger();
    pdl_wait();
    const int b = blockIdx.x * blockDim.x + threadIdx.x;
    if (b >= B) return;
    ids[b] = next[b];
    len_by_slot[slots ? slots[b] : b] += 1;
}

}  // namespace

// ---------------------------------------------------------------------------------------------
void launch_split_tf32(const float* x, float* hi, float* lo, size_t n, cudaStream_t st) {
    if (n == 0) return;
    const int threads = 256;
    const size_t blocks = std::min<size_t>((n + threads - 1) / threads, 148 * 16);
    split_kernel<<<static_cast<unsigned>(blocks), threads, 0, st>>>(x, hi, lo, n);
}

void launch_transpose_split(const float* w, int K, int N, float* hi_t, float* lo_t,
                            cudaStream_t st) {
    dim3 grid((N + 31) / 32, (K + 31) / 32);
    transpose_split_kernel<<<grid, dim3(32, 8), 0, st>>>(w, K, N, hi_t, lo_t);
}

#define ADAI_LN_DISPATCH(NV_, KERNEL, ...)                                          \
    switch (NV_) {                                                                  \
        case 1: launch_kernel(KERNEL<1>, grid, block, 0, st, __VA_ARGS__); break;   \
        case 2: launch_kernel(KERNEL<2>, grid, block, 0, st, __VA_ARGS__); break;   \
        case 3: launch_kernel(KERNEL<3>, grid, block, 0, st, __VA_ARGS__); break;   \
        case 4: launch_kernel(KERNEL<4>, grid, block, 0, st, __VA_ARGS__); break;   \
        case 6: launch_kernel(KERNEL<6>, grid, block, 0, st, __VA_ARGS__); break;   \
        case 8: launch_kernel(KERNEL<8>, grid, block, 0, st, __VA_ARGS__); break;   \
        case 12: launch_kernel(KERNEL<12>, grid, block, 0, st, __VA_ARGS__); break; \
        case 16: launch_kernel(KERNEL<16>, grid, block, 0, st, __VA_ARGS__); break; \
        default: break;                                                             \
    }

namespace {
thread_local bool t_launch_pdl = false;
}
bool launch_pdl_enabled() { return t_launch_pdl; }
void set_launch_pdl(bool on) { t_launch_pdl = on; }

bool layernorm_width_supported(int D) {
    if (D % 128) return false;
    const int nv = D / 128;
    return nv == 1 || nv == 2 || nv == 3 || nv == 4 || nv == 6 || nv == 8 || nv == 12 || nv == 16;
}

void launch_layernorm(const float* x, int ldx, const float* g, const float* b, float* out,
                      float* out_hi, float* out_lo, int rows, int D, cudaStream_t st) {
    if (rows <= 0) return;
    const dim3 block(128), grid((rows + 3) / 4);
    ADAI_LN_DISPATCH(D / 128, layernorm_kernel, x, ldx, g, b, out, out_hi, out_lo, rows, D);
}

void launch_embed_ln(const float* table, const int* ids, const float* pe, int pe_rows,
                     const int* slots, const int* pos_by_slot, const int* pos_direct, float* x,
                     const float* g, const float* b, float* out_hi, float* out_lo, int rows,
                     int D, int vocab, int* err, cudaStream_t st) {
    if (rows <= 0) return;
    const dim3 block(128), grid((rows + 3) / 4);
    ADAI_LN_DISPATCH(D / 128, embed_ln_kernel, table, ids, pe, pe_rows, slots, pos_by_slot,
                     pos_direct, x, g, b, out_hi, out_lo, rows, D, vocab, err);
}

void launch_embed_stats(const float* table, const int* ids, const float* pe, int pe_rows,
                        const int* slots, const int* pos_by_slot, float* x, float* x_hi,
                        float* x_lo, float2* stats, int rows, int D, int vocab, int* err,
                        cudaStream_t st) {
    if (rows <= 0) return;
    const dim3 block(128), grid((rows + 3) / 4);
    ADAI_LN_DISPATCH(D / 128, embed_stats_kernel, table, ids, pe, pe_rows, slots, pos_by_slot, x,
                     x_hi, x_lo, stats, rows, D, vocab, err);
}

bool attention_head_dim_supported(int dh) { return dh == 32 || dh == 64; }

size_t decode_attn_ws_floats(int B, int H, int max_len, int head_dim, int chunk) {
    const int max_ch = (std::max(max_len, 1) + chunk - 1) / chunk;
    return static_cast<size_t>(B) * H * max_ch * (head_dim + 4);
}

void launch_decode_attention(const DecodeAttnArgs& a, int* err, cudaStream_t st) {
    if (a.B <= 0) return;
    DecodeAttnArgs args = a;  // chunk: one of the two sizes the scratch is sized for
    args.chunk = (a.chunk == kAttnChunkShort) ? kAttnChunkShort : kAttnChunk;
    args.err = err;
    const int max_ch = (std::max(args.max_len, 1) + args.chunk - 1) / args.chunk;
    dim3 grid(max_ch, args.H, args.B);
    if (a.head_dim == 32)
        launch_kernel(decode_attention_kernel<32>, grid, dim3(kAttnWarps * 32), 0, st, args);
    else
        launch_kernel(decode_attention_kernel<64>, grid, dim3(kAttnWarps * 32), 0, st, args);
}

void launch_prefill_attention(const float* qkv, int D, int H, const int* offsets, const int* lens,
                              int nseq, int max_len, float* out_hi, float* out_lo, float scale,
                              cudaStream_t st) {
    if (nseq <= 0 || max_len <= 0) return;
    dim3 grid((max_len + kPreQ - 1) / kPreQ, H, nseq);
    if (D / H == 32)
        prefill_attention_kernel<32><<<grid, kPreQ, 0, st>>>(qkv, D, offsets, lens, out_hi, out_lo, scale);
    else
        prefill_attention_kernel<64><<<grid, kPreQ, 0, st>>>(qkv, D, offsets, lens, out_hi, out_lo, scale);
}

void launch_advance(const int* next, int* ids, const int* slots, int* len_by_slot, int B,
                    cudaStream_t st) {
    if (B <= 0) return;
    launch_kernel(advance_kernel, dim3((B + 127) / 128), dim3(128), 0, st, next, ids, slots,
                  len_by_slot, B);
}

// Two bounded waits on an mbarrier that nothing arrives at: the first runs out after the spin
// deadline and records its code in the error word; the second sees the word already set and
// gives up at once. Nothing asynchronous is in flight, so the CTA exits cleanly.
__global__ void wait_selftest_kernel(int* err, int* gave_up) {
    __shared__ uint64_t bar;
    if (threadIdx.x != 0) return;
    mbar_init(&bar, 1);
    fence_barrier_init();
    const bool first = mbar_wait(&bar, 0, err, kDevTimeoutAccum);
    const bool second = mbar_wait(&bar, 0, err, kDevTimeoutTmaFull);
    *gave_up = (first ? 0 : 1) + (second ? 0 : 2);
}

void launch_wait_selftest(int* err, int* gave_up, cudaStream_t st) {
    launch_kernel(wait_selftest_kernel, dim3(1), dim3(32), 0, st, err, gave_up);
}

}  // namespace adai_b200
