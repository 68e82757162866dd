// sample.cu — token selection on the device with the reference's sampling rules
// (TextGenerator::generate, src/TextGenerator.cpp:519-565, and the filters at :26-137): the
// min_length mask of next_logits (:197-203), the repetition penalty once per distinct token seen,
// temperature, top-k, top-p, then the argmax (temperature <= 0) or one draw from the slot's own
// std::mt19937 through std::discrete_distribution, as libstdc++ computes both (:145-148).
//
// One CTA of 1024 threads per row. The row is held in shared memory; warp w owns the contiguous
// index range [w*span, (w+1)*span) and reads it 32 consecutive elements at a time, so every pass is
// coalesced and free of bank conflicts and the index order needed for tie ranks and the
// cumulative sum is the (warp, iteration, lane) order.
//
// Where the reference works in float and the device in double (the top-p running sum, the
// cumulative distribution), the two agree except when the decision lies within rounding distance
// of its threshold. Ties at the top-k and top-p cut are kept lowest index first (std::partial_sort
// and std::sort leave their order unspecified).
#include <cfloat>
#include <cmath>

#include "common.cuh"
#include "kernels.h"

namespace adai_b200 {
namespace {

constexpr int kThreads = 1024;
constexpr int kWarps = kThreads / 32;
constexpr unsigned kFull = 0xffffffffu;

// Order-preserving key of a non-NaN float (larger float, larger key); -0 and +0 share one key, as
// they compare equal.
__device__ __forceinline__ unsigned fkey(float f) {
    if (f == 0.0f) f = 0.0f;
    const unsigned u = __float_as_uint(f);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

struct Smem {
    double red_d[kWarps];
    int red_i[kWarps];
    int red_j[kWarps];
    float red_f[kWarps];
    int tie_base[kWarps];
    unsigned mt[624];
    unsigned draw[2];
    double bcast_d;
    int bcast_i;
    float bcast_f;
};

__device__ __forceinline__ double block_sum_d(double v, Smem& s) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(kFull, v, o);
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    __syncthreads();
    if (l == 0) s.red_d[w] = v;
    __syncthreads();
    if (w == 0) {
        // fixed order: warp sums added lane 0 .. 31 by a tree whose shape does not depend on data
        double t = s.red_d[l];
#pragma unroll
        for (int o = 16; o; o >>= 1) t += __shfl_xor_sync(kFull, t, o);
        if (l == 0) s.bcast_d = t;
    }
    __syncthreads();
    return s.bcast_d;
}

__device__ __forceinline__ int block_sum_i(int v, Smem& s) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(kFull, v, o);
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    __syncthreads();
    if (l == 0) s.red_i[w] = v;
    __syncthreads();
    if (w == 0) {
        int t = s.red_i[l];
#pragma unroll
        for (int o = 16; o; o >>= 1) t += __shfl_xor_sync(kFull, t, o);
        if (l == 0) s.bcast_i = t;
    }
    __syncthreads();
    return s.bcast_i;
}

__device__ __forceinline__ float block_max_f(float v, Smem& s) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(kFull, v, o));
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    __syncthreads();
    if (l == 0) s.red_f[w] = v;
    __syncthreads();
    if (w == 0) {
        float t = s.red_f[l];
#pragma unroll
        for (int o = 16; o; o >>= 1) t = fmaxf(t, __shfl_xor_sync(kFull, t, o));
        if (l == 0) s.bcast_f = t;
    }
    __syncthreads();
    return s.bcast_f;
}

// Float sum of the block in a fixed tree order (the reference sums left to right; the difference
// is a common factor of every probability and cancels in the normalised distribution).
__device__ __forceinline__ float block_sum_f(float v, Smem& s) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(kFull, v, o);
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    __syncthreads();
    if (l == 0) s.red_f[w] = v;
    __syncthreads();
    if (w == 0) {
        float t = s.red_f[l];
#pragma unroll
        for (int o = 16; o; o >>= 1) t += __shfl_xor_sync(kFull, t, o);
        if (l == 0) s.bcast_f = t;
    }
    __syncthreads();
    return s.bcast_f;
}

// First index of the maximum over the block (value, index) pairs.
__device__ __forceinline__ int block_argmax(float v, int j, Smem& s) {
#pragma unroll
    for (int o = 16; o; o >>= 1) {
        const float ov = __shfl_xor_sync(kFull, v, o);
        const int oj = __shfl_xor_sync(kFull, j, o);
        if (ov > v || (ov == v && oj < j)) {
            v = ov;
            j = oj;
        }
    }
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    __syncthreads();
    if (l == 0) {
        s.red_f[w] = v;
        s.red_j[w] = j;
    }
    __syncthreads();
    if (w == 0) {
        v = s.red_f[l];
        j = s.red_j[l];
#pragma unroll
        for (int o = 16; o; o >>= 1) {
            const float ov = __shfl_xor_sync(kFull, v, o);
            const int oj = __shfl_xor_sync(kFull, j, o);
            if (ov > v || (ov == v && oj < j)) {
                v = ov;
                j = oj;
            }
        }
        if (l == 0) s.bcast_i = j;
    }
    __syncthreads();
    return s.bcast_i;
}

// MT19937 state refresh (the published recurrence) in three data-parallel phases: entries
// [0,227) read only old words; [227,454) read the new words 227 places back; [454,623) likewise;
// 623 reads the new word 0. Each phase reads into registers before anyone writes.
__device__ void mt_twist_block(unsigned* g, Smem& s) {
    const int t = threadIdx.x;
    for (int i = t; i < 624; i += kThreads) s.mt[i] = g[i];
    __syncthreads();
    auto step = [&](int i) {
        const unsigned y = (s.mt[i] & 0x80000000u) | (s.mt[(i + 1) % 624] & 0x7fffffffu);
        return s.mt[(i + 397) % 624] ^ (y >> 1) ^ ((y & 1u) ? 0x9908b0dfu : 0u);
    };
    const int lo[4] = {0, 227, 454, 623}, hi[4] = {227, 454, 623, 624};
#pragma unroll
    for (int p = 0; p < 4; ++p) {
        const int i = lo[p] + t;
        unsigned v = 0;
        if (i < hi[p]) v = step(i);
        __syncthreads();
        if (i < hi[p]) s.mt[i] = v;
        __syncthreads();
    }
    for (int i = t; i < 624; i += kThreads) g[i] = s.mt[i];
    __syncthreads();
}

__device__ __forceinline__ unsigned mt_temper(unsigned y) {
    y ^= y >> 11;
    y ^= (y << 7) & 0x9d2c5680u;
    y ^= (y << 15) & 0xefc60000u;
    y ^= y >> 18;
    return y;
}

// std::generate_canonical<double, 53>(mt19937) as libstdc++ computes it: two draws,
// (x0 + x1 * 2^32) / 2^64, a result of 1 replaced by the largest double below 1.
__device__ double draw_canonical(unsigned* g, Smem& s) {
    if (threadIdx.x == 0) s.bcast_i = static_cast<int>(g[624]);
    __syncthreads();
    int pos = s.bcast_i;
    __syncthreads();
    for (int d = 0; d < 2; ++d) {
        if (pos >= 624) {
            mt_twist_block(g, s);
            pos = 0;
        }
        if (threadIdx.x == 0) s.draw[d] = mt_temper(g[pos]);
        ++pos;
    }
    if (threadIdx.x == 0) g[624] = static_cast<unsigned>(pos);
    __syncthreads();
    double r = static_cast<double>(s.draw[0]);
    r += static_cast<double>(s.draw[1]) * 4294967296.0;
    r = r / 18446744073709551616.0;
    if (r >= 1.0) r = 0x1.fffffffffffffp-1;
    return r;
}

// Keeps the elements whose key is above `thr`, and of those equal to it the first `need` by index;
// the others become -1e9f. keys(j) computes the key of element j.
template <class KeyFn>
__device__ void keep_above(float* x, int V, int span, unsigned thr, int need, int n_eq, KeyFn keys,
                           Smem& s) {
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    const int base = w * span;
    if (need >= n_eq) {  // no tie to break
        for (int i = 0; i < span; i += 32) {
            const int j = base + i + l;
            if (j < V && keys(j) < thr) x[j] = -1e9f;
        }
        __syncthreads();
        return;
    }
    int cnt = 0;
    for (int i = 0; i < span; i += 32) {
        const int j = base + i + l;
        cnt += __popc(__ballot_sync(kFull, j < V && keys(j) == thr));
    }
    __syncthreads();
    if (l == 0) s.tie_base[w] = cnt;
    __syncthreads();
    if (threadIdx.x == 0) {
        int acc = 0;
        for (int q = 0; q < kWarps; ++q) {
            const int c = s.tie_base[q];
            s.tie_base[q] = acc;
            acc += c;
        }
    }
    __syncthreads();
    int run = s.tie_base[w];
    const unsigned below = (1u << l) - 1u;
    for (int i = 0; i < span; i += 32) {
        const int j = base + i + l;
        const unsigned k = j < V ? keys(j) : 0u;
        const bool eq = j < V && k == thr;
        const unsigned bal = __ballot_sync(kFull, eq);
        const int rank = run + __popc(bal & below);
        run += __popc(bal);
        if (j < V && (k < thr || (eq && rank >= need))) x[j] = -1e9f;
    }
    __syncthreads();
}

// apply_top_k (src/TextGenerator.cpp:41-63): the k-th largest key by bisection over the key bits.
__device__ void top_k_block(float* x, int V, int span, int k, Smem& s) {
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    const int base = w * span;
    auto count_ge = [&](unsigned t) {
        int c = 0;
        for (int i = 0; i < span; i += 32) {
            const int j = base + i + l;
            c += (j < V && fkey(x[j]) >= t) ? 1 : 0;
        }
        return block_sum_i(c, s);
    };
    unsigned thr = 0;
    for (int bit = 31; bit >= 0; --bit) {
        const unsigned cand = thr | (1u << bit);
        if (count_ge(cand) >= k) thr = cand;
    }
    const int n_ge = count_ge(thr);
    const int n_gt = thr == 0xffffffffu ? 0 : count_ge(thr + 1);
    keep_above(x, V, span, thr, k - n_gt, n_ge - n_gt, [&](int j) { return fkey(x[j]); }, s);
}

}  // namespace

__global__ void __launch_bounds__(kThreads, 1) sample_rows_kernel(SampleArgs a) {
    pdl_trigger();
    pdl_wait();
    extern __shared__ __align__(16) float x[];
    __shared__ Smem s;
    const int b = blockIdx.x;
    const int slot = a.slots[b];
    const SampleSlot cfg = a.cfg[slot];
    if (!cfg.enabled) return;
    const int V = a.V;
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    const int span = ((V + kWarps - 1) / kWarps + 31) & ~31;
    const int base = w * span;
    const float* row = a.logits + static_cast<size_t>(b) * a.ld;
    const unsigned* seen = a.seen + static_cast<size_t>(slot) * a.seen_words;
    const int fed = a.fed ? a.fed[b] : -1;
    const bool mask_stop = a.new_tokens[slot] < cfg.min_length;
    const bool penalize = cfg.penalty != 1.0f;
    const bool scale = cfg.temperature > 0.0f && cfg.temperature != 1.0f;

    // next_logits (:177-206): NaN / +inf or no finite value is an error; then the min_length
    // mask, the repetition penalty (:115-136) and the temperature (:26-38), element by element.
    int bad = 0, finite = 0;
    for (int i = 0; i < span; i += 32) {
        const int j = base + i + l;
        if (j >= V) continue;
        float v = row[j];
        bad |= (isnan(v) || v == INFINITY) ? 1 : 0;
        finite |= isfinite(v) ? 1 : 0;
        if (mask_stop && (j == cfg.eos || j == cfg.pad)) v = -INFINITY;
        if (penalize && (j == fed || ((seen[j >> 5] >> (j & 31)) & 1u)))
            v = v > 0.0f ? v / cfg.penalty : v * cfg.penalty;
        if (scale) v = v / cfg.temperature;
        x[j] = v;
    }
    bad = __syncthreads_or(bad);
    finite = __syncthreads_or(finite);
    if (bad || !finite) {
        if (threadIdx.x == 0) {
            if (a.nonfinite) a.nonfinite[b] = 1;
            a.next[b] = 0;
        }
        return;
    }

    if (cfg.top_k > 0 && cfg.top_k < V) top_k_block(x, V, span, cfg.top_k, s);

    if (cfg.top_p < 1.0f) {
        if (cfg.top_p <= 0.0f) {
            top_k_block(x, V, span, 1, s);
        } else {
            // apply_top_p (:66-101): softmax, then the smallest set of most likely tokens whose
            // probability reaches p. The filtered logits are parked in global scratch while the
            // probabilities occupy shared memory.
            float* park = a.scratch + static_cast<size_t>(b) * a.V;
            float mx = -INFINITY;
            for (int i = 0; i < span; i += 32) {
                const int j = base + i + l;
                if (j < V) mx = fmaxf(mx, x[j]);
            }
            mx = block_max_f(mx, s);
            float part = 0.0f;
            for (int i = 0; i < span; i += 32) {
                const int j = base + i + l;
                if (j < V) {
                    park[j] = x[j];
                    const float e = expf(x[j] - mx);
                    x[j] = e;
                    part += e;
                }
            }
            const float sum = block_sum_f(part, s);
            for (int i = 0; i < span; i += 32) {
                const int j = base + i + l;
                if (j < V && sum > 0.0f) x[j] = x[j] / sum;
            }
            __syncthreads();
            // largest probability q (bit pattern; q >= 0) with mass(q_j >= q) >= p
            const double p = cfg.top_p;
            auto mass_ge = [&](unsigned t) {
                double m = 0.0;
                for (int i = 0; i < span; i += 32) {
                    const int j = base + i + l;
                    if (j < V && __float_as_uint(x[j]) >= t) m += static_cast<double>(x[j]);
                }
                return block_sum_d(m, s);
            };
            unsigned thr = 0;
            for (int bit = 30; bit >= 0; --bit) {
                const unsigned cand = thr | (1u << bit);
                if (mass_ge(cand) >= p) thr = cand;
            }
            int n_eq = 0;
            double m_gt = 0.0;
            {
                int ce = 0;
                double mg = 0.0;
                for (int i = 0; i < span; i += 32) {
                    const int j = base + i + l;
                    if (j >= V) continue;
                    const unsigned u = __float_as_uint(x[j]);
                    if (u > thr) mg += static_cast<double>(x[j]);
                    else if (u == thr) ++ce;
                }
                n_eq = block_sum_i(ce, s);
                m_gt = block_sum_d(mg, s);
            }
            int need = n_eq;  // thr == 0: the running sum never reached p, everything is kept
            if (thr != 0) {
                const double q = __uint_as_float(thr);
                const double want = ceil((p - m_gt) / q);
                need = want >= static_cast<double>(n_eq) ? n_eq : max(1, static_cast<int>(want));
            }
            keep_above(x, V, span, thr, need, n_eq,
                       [&](int j) { return __float_as_uint(x[j]); }, s);
            // x holds probabilities with -1e9f where dropped: put the kept logits back
            for (int i = 0; i < span; i += 32) {
                const int j = base + i + l;
                if (j < V && x[j] != -1e9f) x[j] = park[j];
            }
            __syncthreads();
        }
    }

    int tok;
    if (cfg.temperature <= 0.0f) {
        float bv = -INFINITY;
        int bj = 0x7fffffff;
        for (int i = 0; i < span; i += 32) {
            const int j = base + i + l;
            if (j < V && (x[j] > bv || bj == 0x7fffffff)) {
                bv = x[j];
                bj = j;
            }
        }
        tok = block_argmax(bv, bj, s);
    } else {
        // sample_token (:145-148): softmax (Activation::softmax_row), then the first index whose
        // cumulative probability reaches the uniform draw; the last index takes what remains.
        float mx = -INFINITY;
        for (int i = 0; i < span; i += 32) {
            const int j = base + i + l;
            if (j < V) mx = fmaxf(mx, x[j]);
        }
        mx = block_max_f(mx, s);
        float part = 0.0f;
        for (int i = 0; i < span; i += 32) {
            const int j = base + i + l;
            if (j < V) {
                const float e = expf(x[j] - mx);
                x[j] = e;
                part += e;
            }
        }
        const float sum = block_sum_f(part, s);
        double dpart = 0.0;
        for (int i = 0; i < span; i += 32) {
            const int j = base + i + l;
            if (j < V) {
                if (sum > 0.0f) x[j] = x[j] / sum;
                dpart += static_cast<double>(x[j]);
            }
        }
        // warp totals in index order, then the warp holding the crossing walks its range
        double wsum = dpart;
#pragma unroll
        for (int o = 16; o; o >>= 1) wsum += __shfl_xor_sync(kFull, wsum, o);
        __syncthreads();
        if (l == 0) s.red_d[w] = wsum;
        __syncthreads();
        double total = 0.0;
        for (int q = 0; q < kWarps; ++q) total += s.red_d[q];
        const double u = draw_canonical(a.mt + static_cast<size_t>(slot) * kMtWords, s);
        const double target = u * total;
        if (threadIdx.x == 0) s.bcast_i = V - 1;
        __syncthreads();
        double before = 0.0;
        for (int q = 0; q < w; ++q) before += s.red_d[q];
        const double after = before + s.red_d[w];
        if (before < target && after >= target) {  // at most one warp
            double run = before;
            bool done = false;
            for (int i = 0; i < span && !done; i += 32) {
                const int j = base + i + l;
                double v = j < V ? static_cast<double>(x[j]) : 0.0;
                // inclusive scan across the 32 lanes
#pragma unroll
                for (int o = 1; o < 32; o <<= 1) {
                    const double n = __shfl_up_sync(kFull, v, o);
                    if (l >= o) v += n;
                }
                const unsigned hit = __ballot_sync(kFull, j < V && run + v >= target);
                if (hit) {
                    if (l == 0) s.bcast_i = min(base + i + __ffs(hit) - 1, V - 1);
                    done = true;
                }
                run += __shfl_sync(kFull, v, 31);
            }
        } else if (w == 0 && target <= 0.0 && l == 0) {
            s.bcast_i = 0;
        }
        __syncthreads();
        tok = s.bcast_i;
    }
    if (threadIdx.x == 0) {
        a.next[b] = tok;
        a.new_tokens[slot] += 1;
        if (fed >= 0 && fed < V) {
            unsigned* sw = a.seen + static_cast<size_t>(slot) * a.seen_words;
            sw[fed >> 5] |= 1u << (fed & 31);
        }
    }
}

size_t sample_smem_bytes(int V) { return static_cast<size_t>(V) * sizeof(float); }

int sample_max_vocab() {
    static int max_v = [] {
        int dev = 0, optin = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
        const int avail = optin - static_cast<int>(sizeof(Smem)) - 1024;
        return avail > 0 ? avail / static_cast<int>(sizeof(float)) : 0;
    }();
    return max_v;
}

cudaError_t launch_sample_rows(const SampleArgs& a, cudaStream_t st) {
    const size_t smem = sample_smem_bytes(a.V);
    static size_t configured = 0;
    if (smem > configured) {
        cudaError_t e = cudaFuncSetAttribute(sample_rows_kernel,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             static_cast<int>(smem));
        if (e != cudaSuccess) return e;
        configured = smem;
    }
    return launch_kernel(sample_rows_kernel, dim3(a.B), dim3(kThreads), smem, st, a);
}

}  // namespace adai_b200
