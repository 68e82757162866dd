// sample.cu — token selection on the device with the reference's sampling rules
// (TextGenerator::generate, src/TextGenerator.cpp:519-565, and the filters at :26-137): the
// min_length mask of next_logits (:197-203), the repetition penalty once per distinct token seen,
// temperature, top-k, top-p, then the argmax (temperature <= 0) or one draw from the slot's own
// std::mt19937 through std::discrete_distribution, as libstdc++ computes both (:145-148).
//
// One CTA of 1024 threads per row. The row is held in shared memory, padded to 32 equal warp
// ranges: warp w owns the contiguous index range [w*span, (w+1)*span) and reads it 32 consecutive
// elements at a time, so every pass is coalesced and free of bank conflicts, and the index order
// needed for tie ranks and the cumulative sum is the (warp, iteration, lane) order. The padding
// holds values that no pass can select (-inf logits, key 0, probability 0), so the inner loops
// carry no bounds test.
//
// The two cuts are found by radix selection over 32-bit patterns, a byte per pass: top-k over an
// order-preserving key of the logit, top-p over the bit pattern of the probability (which orders
// like the value, as it is never negative), with the mass of each bin summed in fixed point.
// Before a selection the row is rewritten in place as those patterns.
//
// Where the reference works in float and the device in double or fixed point (the top-p running
// sum, the cumulative distribution), the two agree except when the decision lies within rounding
// distance of its threshold. Ties at the top-k and top-p cut are kept lowest index first
// (std::partial_sort and std::sort leave their order unspecified).
#include <cfloat>
#include <cmath>
#include <mutex>

#include "common.cuh"
#include "kernels.h"

namespace adai_b200 {
namespace {

constexpr int kThreads = 1024;
constexpr int kWarps = kThreads / 32;
constexpr unsigned kFull = 0xffffffffu;

// Elements per warp range: a multiple of 32, kWarps ranges cover the vocabulary.
__host__ __device__ inline int span_of(int V) { return ((V + kWarps - 1) / kWarps + 31) & ~31; }

// Order-preserving key of a non-NaN float (larger float, larger key); -0 and +0 share one key, as
// they compare equal. Every key of a float is at least 0x007fffff (that of -inf), so key 0 can
// mark padding.
__device__ __forceinline__ unsigned fkey(float f) {
    if (f == 0.0f) f = 0.0f;
    const unsigned u = __float_as_uint(f);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float key_value(unsigned k) {
    return __uint_as_float((k & 0x80000000u) ? (k & 0x7fffffffu) : ~k);
}

// Reduction slots are double-buffered: a reduction writes one buffer, passes one barrier and reads
// it back; the next reduction writes the other buffer, so a write never meets a read still in
// progress (the barrier of the reduction in between orders them).
struct Smem {
    double rd[2][kWarps];
    int ri[2][kWarps];
    int rj[2][kWarps];
    float rf[2][kWarps];
    int tie_base[kWarps];
    // the filters' radix histograms and the generator refresh are never live at the same time
    union {
        unsigned mt[624];
        struct {
            unsigned c[256];
            unsigned long long m[256];
        } hist;
    };
    unsigned draw[2];
    int bcast_i;
    unsigned long long sel_rem;  // radix selection: the bin one pass picked
    int sel_bin, sel_cnt, sel_ok;
};

template <class T, class Op>
__device__ __forceinline__ T warp_all(T v, Op op) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v = op(v, __shfl_xor_sync(kFull, v, o));
    return v;
}

// Block reductions, one barrier each; every warp folds the 32 warp results itself in a fixed
// order, so all threads return the same value.
__device__ __forceinline__ double bsum_d(double v, Smem& s, int& ph) {
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    auto add = [](double a, double b) { return a + b; };
    v = warp_all(v, add);
    if (l == 0) s.rd[ph][w] = v;
    __syncthreads();
    const double t = warp_all(s.rd[ph][l], add);
    ph ^= 1;
    return t;
}
__device__ __forceinline__ int bsum_i(int v, Smem& s, int& ph) {
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    auto add = [](int a, int b) { return a + b; };
    v = warp_all(v, add);
    if (l == 0) s.ri[ph][w] = v;
    __syncthreads();
    const int t = warp_all(s.ri[ph][l], add);
    ph ^= 1;
    return t;
}
__device__ __forceinline__ float bmax_f(float v, Smem& s, int& ph) {
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    auto mx = [](float a, float b) { return fmaxf(a, b); };
    v = warp_all(v, mx);
    if (l == 0) s.rf[ph][w] = v;
    __syncthreads();
    const float t = warp_all(s.rf[ph][l], mx);
    ph ^= 1;
    return t;
}
// Float sum of the block in a fixed tree order (the reference sums left to right; the difference
// is a common factor of every probability and cancels in the normalised distribution).
__device__ __forceinline__ float bsum_f(float v, Smem& s, int& ph) {
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    auto add = [](float a, float b) { return a + b; };
    v = warp_all(v, add);
    if (l == 0) s.rf[ph][w] = v;
    __syncthreads();
    const float t = warp_all(s.rf[ph][l], add);
    ph ^= 1;
    return t;
}
// First index of the maximum over the block's (value, index) pairs.
__device__ __forceinline__ int bargmax(float v, int j, Smem& s, int& ph) {
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    auto fold = [&]() {
#pragma unroll
        for (int o = 16; o; o >>= 1) {
            const float ov = __shfl_xor_sync(kFull, v, o);
            const int oj = __shfl_xor_sync(kFull, j, o);
            if (ov > v || (ov == v && oj < j)) {
                v = ov;
                j = oj;
            }
        }
    };
    fold();
    if (l == 0) {
        s.rf[ph][w] = v;
        s.rj[ph][w] = j;
    }
    __syncthreads();
    v = s.rf[ph][l];
    j = s.rj[ph][l];
    fold();
    ph ^= 1;
    return j;
}

// MT19937 state refresh (the published recurrence) in data-parallel phases: entries [0,227) read
// only old words; [227,454) read the new words 227 places back; [454,623) likewise; 623 reads the
// new word 0. Each phase reads into registers before anyone writes.
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

// Radix selection over the row's 32-bit patterns (padding 0), most significant byte first. Each
// of four passes histograms the 8-bit digit of the patterns that share the prefix chosen so far
// (counts aggregated per warp with __match_any_sync) and warp 0 walks the 256 bins from the top.
// With kMass a bin also holds the probability mass of its patterns (each pattern is then a
// non-negative float) in fixed point, units of 2^-40, so the sums do not depend on the order of
// the atomic adds. The walk stops at the first bin whose running total reaches `target` (a count,
// or a fixed-point mass). Returns the cut pattern: the target-th largest pattern, or the largest t
// whose mass of patterns >= t reaches target. rem: what is still needed from the patterns equal to
// the cut; n_eq: how many patterns equal it. found is false when the row's total stays below
// target (possible only for masses).
constexpr float kMassScale = 1099511627776.0f;  // 2^40
template <bool kMass>
__device__ unsigned radix_select(const unsigned* xu, int span, unsigned long long target, Smem& s,
                                 unsigned long long& rem, int& n_eq, bool& found) {
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    const int base = w * span + l;
    unsigned prefix = 0;
    rem = target;
    n_eq = 0;
    found = true;
    for (int pass = 0; pass < 4; ++pass) {
        const int shift = 24 - 8 * pass;
        for (int i = threadIdx.x; i < 256; i += kThreads) {
            s.hist.c[i] = 0;
            if (kMass) s.hist.m[i] = 0;
        }
        __syncthreads();
#pragma unroll 4
        for (int i = 0; i < span; i += 32) {
            const unsigned kk = xu[base + i];
            // (masses: a pattern without mass cannot move the walk, so it takes no part)
            const bool in = (pass == 0 || (kk >> (shift + 8)) == prefix) &&
                            (!kMass || __uint_as_float(kk) * kMassScale >= 1.0f);
            const unsigned inmask = __ballot_sync(kFull, in);
            if (in) {
                const unsigned digit = (kk >> shift) & 255u;
                const unsigned peers = __match_any_sync(inmask, digit);
                const bool leader = l == __ffs(peers) - 1;
                if (leader) atomicAdd(&s.hist.c[digit], static_cast<unsigned>(__popc(peers)));
                if (kMass) {
                    // the group's mass in two 32-bit sums that cannot overflow (fx <= 2^40: 20 low
                    // bits and at most 21 high bits per lane, 32 lanes), then one atomic per group
                    const auto fx = static_cast<unsigned long long>(__uint_as_float(kk) * kMassScale);
                    const unsigned lo = __reduce_add_sync(peers, static_cast<unsigned>(fx & 0xFFFFFull));
                    const unsigned hi = __reduce_add_sync(peers, static_cast<unsigned>(fx >> 20));
                    const unsigned long long tot = (static_cast<unsigned long long>(hi) << 20) + lo;
                    if (leader && tot) atomicAdd(&s.hist.m[digit], tot);
                }
            }
        }
        __syncthreads();
        if (w == 0) {  // lane l holds bins 255 - 8l down to 248 - 8l
            unsigned long long v8[8], tot = 0;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const int bin = 255 - 8 * l - j;
                v8[j] = kMass ? s.hist.m[bin] : s.hist.c[bin];
                tot += v8[j];
            }
            unsigned long long incl = tot;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const unsigned long long n = __shfl_up_sync(kFull, incl, o);
                if (l >= o) incl += n;
            }
            const unsigned hit = __ballot_sync(kFull, incl >= rem);
            if (l == 0) s.sel_ok = hit ? 1 : 0;
            if (hit && l == __ffs(hit) - 1) {
                unsigned long long cum = incl - tot;
                for (int j = 0; j < 8; ++j) {
                    if (cum + v8[j] >= rem) {
                        const int bin = 255 - 8 * l - j;
                        s.sel_bin = bin;
                        s.sel_rem = rem - cum;
                        s.sel_cnt = static_cast<int>(s.hist.c[bin]);
                        break;
                    }
                    cum += v8[j];
                }
            }
        }
        __syncthreads();
        if (!s.sel_ok) {
            found = false;
            return 0;
        }
        prefix = (prefix << 8) | static_cast<unsigned>(s.sel_bin);
        rem = s.sel_rem;
        n_eq = s.sel_cnt;
        __syncthreads();  // the next pass rewrites the histogram and the selection
    }
    return prefix;
}

// The exclusive prefix over warps of each warp's count of patterns equal to thr (tie ranks in
// index order), left in s.tie_base.
__device__ void tie_prefix(const unsigned* xu, int span, unsigned thr, Smem& s) {
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    const int base = w * span + l;
    int cnt = 0;
    for (int i = 0; i < span; i += 32) cnt += __popc(__ballot_sync(kFull, xu[base + i] == thr));
    if (l == 0) s.tie_base[w] = cnt;
    __syncthreads();
    if (w == 0) {  // exclusive scan of the 32 warp counts
        const int v = s.tie_base[l];
        int incl = v;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int n = __shfl_up_sync(kFull, incl, o);
            if (l >= o) incl += n;
        }
        s.tie_base[l] = incl - v;
    }
    __syncthreads();
}

// Keeps, of the row's patterns, those above thr and the first `need` (in index order) equal to
// it; writes value(j) for kept elements and -1e9f for the others (-inf on the padding).
template <class ValueFn>
__device__ void keep_cut(float* x, const unsigned* xu, int V, int span, unsigned thr, int need,
                         int n_eq, ValueFn value, Smem& s) {
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    const int base = w * span + l;
    const bool ties = need < n_eq;
    if (ties) tie_prefix(xu, span, thr, s);
    int run = ties ? s.tie_base[w] : 0;
    const unsigned below = (1u << l) - 1u;
#pragma unroll 8
    for (int i = 0; i < span; i += 32) {
        const int j = base + i;
        const unsigned kk = xu[j];
        bool keep = kk > thr || (kk == thr && !ties);
        if (ties) {  // the whole warp takes this branch: the ballot is over all 32 lanes
            const unsigned bal = __ballot_sync(kFull, kk == thr);
            if (kk == thr) keep = run + __popc(bal & below) < need;
            run += __popc(bal);
        }
        const float v = keep ? value(j, kk) : -1e9f;
        x[j] = j >= V ? -INFINITY : v;
    }
    __syncthreads();
}

}  // namespace

__global__ void __launch_bounds__(kThreads, 1) sample_rows_kernel(SampleArgs a) {
    pdl_trigger();
    pdl_wait();
    extern __shared__ __align__(16) float x[];
    unsigned* xu = reinterpret_cast<unsigned*>(x);
    __shared__ Smem s;
    const int b = blockIdx.x;
    const int slot = a.slots[b];
    const SampleSlot cfg = a.cfg[slot];
    if (!cfg.enabled) return;
    const int V = a.V;
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    const int span = span_of(V);
    const int base = w * span + l;  // this thread's element of iteration i is base + i
    const float* row = a.logits + static_cast<size_t>(b) * a.ld;
    const unsigned* seen = a.seen + static_cast<size_t>(slot) * a.seen_words;
    const int fed = a.fed ? a.fed[b] : -1;
    const bool mask_stop = a.new_tokens[slot] < cfg.min_length;
    const bool penalize = cfg.penalty != 1.0f;
    const bool scale = cfg.temperature > 0.0f && cfg.temperature != 1.0f;
    int ph = 0;

    // next_logits (:177-206): NaN / +inf or no finite value is an error; then the min_length
    // mask, the repetition penalty (:115-136) and the temperature (:26-38), element by element.
    int bad = 0, finite = 0;
#pragma unroll 8
    for (int i = 0; i < span; i += 32) {
        const int j = base + i;
        float v = -INFINITY;  // padding
        if (j < V) {
            v = row[j];
            bad |= (isnan(v) || v == INFINITY) ? 1 : 0;
            finite |= isfinite(v) ? 1 : 0;
            if (mask_stop && (j == cfg.eos || j == cfg.pad)) v = -INFINITY;
            if (penalize && (j == fed || ((seen[j >> 5] >> (j & 31)) & 1u)))
                v = v > 0.0f ? v / cfg.penalty : v * cfg.penalty;
            if (scale) v = v / cfg.temperature;
        }
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

    // apply_top_k (:41-63), then apply_top_p's p <= 0 case, which is top-1 (:71-73)
    const int k_top = (cfg.top_k > 0 && cfg.top_k < V) ? cfg.top_k : 0;
    for (int pass = 0; pass < 2; ++pass) {
        const int k = pass == 0 ? ((cfg.top_k > 0 && cfg.top_k < V) ? cfg.top_k : 0)
                                : (cfg.top_p <= 0.0f ? 1 : 0);
        if (k == 0) continue;
        for (int i = 0; i < span; i += 32) {
            const int j = base + i;
            xu[j] = j < V ? fkey(x[j]) : 0u;
        }
        __syncthreads();
        unsigned long long need = 0;
        int n_eq = 0;
        bool found = true;
        const unsigned thr = radix_select<false>(xu, span, static_cast<unsigned long long>(k), s,
                                                 need, n_eq, found);
        keep_cut(x, xu, V, span, thr, static_cast<int>(need), n_eq,
                 [](int, unsigned kk) { return key_value(kk); }, s);
    }

    if (cfg.top_p > 0.0f && cfg.top_p < 1.0f) {
        // apply_top_p (:66-101): softmax, then the smallest set of most likely tokens whose
        // probability reaches p. The filtered logits are parked in global scratch while the
        // probabilities occupy shared memory.
        float* park = a.scratch + static_cast<size_t>(b) * a.V;
        float mx = -INFINITY;
        for (int i = 0; i < span; i += 32) mx = fmaxf(mx, x[base + i]);
        mx = bmax_f(mx, s, ph);
        float part = 0.0f;
#pragma unroll 8
        for (int i = 0; i < span; i += 32) {
            const int j = base + i;
            const float v = x[j];
            if (j < V) park[j] = v;
            const float e = expf(v - mx);  // padding: exp(-inf) = 0
            x[j] = e;
            part += e;
        }
        const float sum = bsum_f(part, s, ph);
        if (sum > 0.0f)
            for (int i = 0; i < span; i += 32) x[base + i] = x[base + i] / sum;
        __syncthreads();
        // The cut: the largest probability pattern t with mass(q >= t) >= p. After top-k at most
        // k tokens carry mass, and a radix selection over them (fixed-point masses, at least one
        // unit so a p below the resolution still keeps the most likely token) takes four cheap
        // passes. Over the whole vocabulary bisection over the pattern's 31 bits with float64
        // block sums is faster.
        unsigned thr = 0;
        int n_eq = 0, need = 0;
        bool found = true;
        if (k_top > 0) {
            const auto target = max(1ull, static_cast<unsigned long long>(
                                              static_cast<double>(cfg.top_p) * static_cast<double>(kMassScale)));
            unsigned long long rem = 0;
            thr = radix_select<true>(xu, span, target, s, rem, n_eq, found);
            if (found) {
                const auto unit = static_cast<unsigned long long>(__uint_as_float(thr) * kMassScale);
                const unsigned long long want = (rem + unit - 1) / unit;  // unit >= 1 here
                need = want >= static_cast<unsigned long long>(n_eq) ? n_eq : max(1, static_cast<int>(want));
            }
        } else {
            const double p = cfg.top_p;
            for (int bit = 30; bit >= 0; --bit) {
                const unsigned cand = thr | (1u << bit);
                double m = 0.0;
#pragma unroll 8
                for (int i = 0; i < span; i += 32) {
                    const unsigned qb = xu[base + i];
                    m += qb >= cand ? static_cast<double>(__uint_as_float(qb)) : 0.0;
                }
                if (bsum_d(m, s, ph) >= p) thr = cand;
            }
            found = thr != 0;
            if (found) {
                int ce = 0;
                double mg = 0.0;
                for (int i = 0; i < span; i += 32) {
                    const unsigned qb = xu[base + i];
                    if (qb > thr) mg += static_cast<double>(__uint_as_float(qb));
                    ce += qb == thr ? 1 : 0;
                }
                n_eq = bsum_i(ce, s, ph);
                const double m_gt = bsum_d(mg, s, ph);
                const double want = ceil((p - m_gt) / static_cast<double>(__uint_as_float(thr)));
                need = want >= static_cast<double>(n_eq) ? n_eq : max(1, static_cast<int>(want));
            }
        }
        if (!found) {  // the running sum never reached p: everything is kept
#pragma unroll 8
            for (int i = 0; i < span; i += 32) {
                const int j = base + i;
                x[j] = j < V ? park[j] : -INFINITY;
            }
            __syncthreads();
        } else {
            keep_cut(x, xu, V, span, thr, need, n_eq, [&](int j, unsigned) { return park[j]; }, s);
        }
    }

    int tok;
    if (cfg.temperature <= 0.0f) {
        // argmax (:151-153): first maximum; padding (-inf, higher index) never wins
        float bv = x[base];
        int bj = base;
        for (int i = 32; i < span; i += 32)
            if (x[base + i] > bv) {
                bv = x[base + i];
                bj = base + i;
            }
        tok = bargmax(bv, bj, s, ph);
    } else {
        // sample_token (:145-148): softmax (Activation::softmax_row), then the first index whose
        // cumulative probability reaches the uniform draw; the last index takes what remains.
        float mx = -INFINITY;
        for (int i = 0; i < span; i += 32) mx = fmaxf(mx, x[base + i]);
        mx = bmax_f(mx, s, ph);
        float part = 0.0f;
        for (int i = 0; i < span; i += 32) {
            const float e = expf(x[base + i] - mx);
            x[base + i] = e;
            part += e;
        }
        const float sum = bsum_f(part, s, ph);
        double dpart = 0.0;
        for (int i = 0; i < span; i += 32) {
            float q = x[base + i];
            if (sum > 0.0f) q = q / sum;
            x[base + i] = q;
            dpart += static_cast<double>(q);
        }
        // warp totals in index order, then the warp holding the crossing walks its range
        const double wsum = warp_all(dpart, [](double u, double v) { return u + v; });
        if (l == 0) s.rd[ph][w] = wsum;
        __syncthreads();
        double total = 0.0, before = 0.0;
        for (int q = 0; q < kWarps; ++q) {
            const double t = s.rd[ph][q];
            if (q < w) before += t;
            total += t;
        }
        const double after = before + s.rd[ph][w];
        ph ^= 1;
        const double u = draw_canonical(a.mt + static_cast<size_t>(slot) * kMtWords, s);
        const double target = u * total;
        if (threadIdx.x == 0) s.bcast_i = target <= 0.0 ? 0 : V - 1;
        __syncthreads();
        if (before < target && after >= target) {  // at most one warp
            // The warp's range is span / 32 chunks of 32 consecutive elements, taken 32 at a
            // time: lane l sums chunk g0 + l (reading element (t + l) & 31 at step t, so the 32
            // lanes hit 32 different banks), a scan over the chunk sums finds the chunk of the
            // crossing, and a scan inside it the element.
            const int wbase = w * span;
            const int nchunk = span / 32;
            double run0 = before;
            for (int g0 = 0; g0 < nchunk; g0 += 32) {
                const int c = g0 + l;
                double csum = 0.0;
                if (c < nchunk) {
                    const float* c0 = x + wbase + c * 32;
                    for (int t = 0; t < 32; ++t) csum += static_cast<double>(c0[(t + l) & 31]);
                }
                double incl = csum;
#pragma unroll
                for (int o = 1; o < 32; o <<= 1) {
                    const double n = __shfl_up_sync(kFull, incl, o);
                    if (l >= o) incl += n;
                }
                const unsigned chit = __ballot_sync(kFull, c < nchunk && run0 + incl >= target);
                if (chit) {
                    const int cl = __ffs(chit) - 1;
                    const double run = run0 + __shfl_sync(kFull, incl - csum, cl);
                    const int j0 = wbase + (g0 + cl) * 32;
                    double v = static_cast<double>(x[j0 + l]);
#pragma unroll
                    for (int o = 1; o < 32; o <<= 1) {
                        const double n = __shfl_up_sync(kFull, v, o);
                        if (l >= o) v += n;
                    }
                    const unsigned hit = __ballot_sync(kFull, j0 + l < V && run + v >= target);
                    if (hit && l == 0) s.bcast_i = min(j0 + __ffs(hit) - 1, V - 1);
                    break;
                }
                run0 += __shfl_sync(kFull, incl, 31);
            }
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

size_t sample_smem_bytes(int V) {
    return static_cast<size_t>(kWarps) * span_of(V) * sizeof(float);
}

int sample_max_vocab() {
    static int max_v = [] {
        int dev = 0, optin = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
        const int avail = optin - static_cast<int>(sizeof(Smem)) - 1024;
        // the padded row is kWarps ranges of a multiple of 32 elements
        return avail > 0 ? avail / static_cast<int>(sizeof(float)) / (kWarps * 32) * (kWarps * 32)
                         : 0;
    }();
    return max_v;
}

// The kernel's shared-memory limit, raised once per device (a process may drive several GPUs)
// to what the largest accepted vocabulary needs.
cudaError_t prepare_sample_attr() {
    static std::mutex mu;
    static unsigned long long done_mask = 0;
    int dev = 0;
    cudaGetDevice(&dev);
    std::lock_guard<std::mutex> lock(mu);
    if (dev < 64 && (done_mask & (1ull << dev))) return cudaSuccess;
    const cudaError_t e = cudaFuncSetAttribute(sample_rows_kernel,
                                               cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               static_cast<int>(sample_smem_bytes(sample_max_vocab())));
    if (e == cudaSuccess && dev < 64) done_mask |= 1ull << dev;
    return e;
}

cudaError_t launch_sample_rows(const SampleArgs& a, cudaStream_t st) {
    const cudaError_t e = prepare_sample_attr();
    if (e != cudaSuccess) return e;
    return launch_kernel(sample_rows_kernel, dim3(a.B), dim3(kThreads), sample_smem_bytes(a.V), st, a);
}

}  // namespace adai_b200
