// gemm_tc.cu — fp32-accurate GEMM on the 5th-generation tensor cores (sm_100a).
//
// Replaces the reference's Matrix::operator* / matrix_multiply_gpu (src/Matrix.cpp:212-277,
// src/gpu/MatrixGPU.cu:351-370, cuBLAS SGEMM) for the stacked decode projections (Q/K/V/O,
// cross-attention, FFN, LM head) and the encoder prefill.
//
// Precision: 3xTF32. Each fp32 operand x is split into hi = tf32(x) and lo = tf32(x - hi)
// (round to nearest); the product is accumulated in fp32 in TMEM as
//     A*W ~= A_lo*W_hi + A_hi*W_lo + A_hi*W_hi,
// the published error-corrected TF32 scheme (Ootomo & Yokota, 2022), which keeps the result
// within a few fp32 ulps of an fp32 GEMM. The weights are split once at upload (stored W^T,
// K-major, hi and lo planes); activations arrive already split by the kernel that produced them.
//
// Structure (one CTA = one 128 x BN output tile, or one K-slice of it):
//   warp 0    TMA producer: 4 boxes per stage (A_hi, A_lo 128x32; W_hi, W_lo BNx32), 128B swizzle
//   warp 1    TMEM allocator + single-thread tcgen05.mma issuer (3 MMAs per K=8 step)
//   warps 2-5 epilogue: tcgen05.ld 32 rows x 16 columns per warp, fused bias / GELU / residual /
//             tf32 split of the output / KV-cache scatter / first-maximum argmax partials.
// Split-K writes fp32 partial tiles to scratch; the last CTA of a tile (ticket counter) sums the
// partials in split order 0..S-1 — deterministic — and runs the epilogue. No cluster multicast.
#include <algorithm>
#include <cstdio>
#include <cstring>
#include <mutex>

#include "common.cuh"
#include "kernels.h"

namespace adai_b200 {

namespace {

constexpr int kBM = 128;
constexpr int kBK = 32;  // fp32 elements per 128-byte swizzled row
constexpr int kThreads = 192;
constexpr int kATileBytes = kBM * kBK * 4;  // 16 KB
constexpr size_t kSmemLimit = 227 * 1024;
constexpr size_t kSmemReserve = 1024 /*alignment slack*/ + 256 /*barriers*/;

struct __align__(64) GemmKParams {
    CUtensorMap a_hi, a_lo, b_hi, b_lo;
    int M, N, K;
    int bn, stages, kb_per_split, splits, n_tiles, m_tiles, total_kb;
    uint32_t idesc, tmem_cols;
    GemmEpilogue epi;
    float* ws;
    int* tickets;
    float* arg_val;
    int* arg_idx;
    int* err;
};

constexpr int kArgNone = 0x7FFFFFFF;

struct ArgState {
    float best;
    int idx;
    int nf;
};

__device__ __forceinline__ void st4(float* p, float a, float b, float c, float d) {
    *reinterpret_cast<float4*>(p) = make_float4(a, b, c, d);
}

// Epilogue on 16 consecutive accumulator columns [col, col+16) of one output row.
__device__ __forceinline__ void epilogue16(const GemmKParams& p, int row, int col, float (&v)[16],
                                           ArgState& as) {
    const GemmEpilogue& e = p.epi;
    const int N = p.N;
    const bool full = col + 16 <= N;
    if (e.flags & kEpiBias) {
#pragma unroll
        for (int j = 0; j < 16; ++j)
            if (full || col + j < N) v[j] += __ldg(e.bias + col + j);
    }
    if (e.flags & kEpiGelu) {
#pragma unroll
        for (int j = 0; j < 16; ++j) v[j] = gelu_tanh(v[j]);
    }
    if (e.flags & kEpiResid) {
        const float* r = e.resid + static_cast<size_t>(row) * e.ldr + col;
#pragma unroll
        for (int j = 0; j < 16; ++j)
            if (full || col + j < N) v[j] = r[j] + v[j];
    }
    if (e.flags & kEpiArgmax) {
#pragma unroll
        for (int j = 0; j < 16; ++j) {
            if (full || col + j < N) {
                const float x = v[j];
                if (isnan(x) || x == INFINITY) as.nf = 1;
                if (x > as.best) {
                    as.best = x;
                    as.idx = col + j;
                }
            }
        }
    }
    const bool vec = full && ((col & 3) == 0);
    if (e.flags & kEpiStore) {
        float* o = e.out + static_cast<size_t>(row) * e.ldo + col;
        if (vec && ((e.ldo & 3) == 0)) {
#pragma unroll
            for (int j = 0; j < 16; j += 4) st4(o + j, v[j], v[j + 1], v[j + 2], v[j + 3]);
        } else {
#pragma unroll
            for (int j = 0; j < 16; ++j)
                if (col + j < N) o[j] = v[j];
        }
    }
    if (e.flags & kEpiSplit) {
        float* oh = e.out_hi + static_cast<size_t>(row) * e.lds + col;
        float* ol = e.out_lo + static_cast<size_t>(row) * e.lds + col;
        float h[16], l[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) split_tf32(v[j], h[j], l[j]);
        if (vec && ((e.lds & 3) == 0)) {
#pragma unroll
            for (int j = 0; j < 16; j += 4) {
                st4(oh + j, h[j], h[j + 1], h[j + 2], h[j + 3]);
                st4(ol + j, l[j], l[j + 1], l[j + 2], l[j + 3]);
            }
        } else {
#pragma unroll
            for (int j = 0; j < 16; ++j)
                if (col + j < N) {
                    oh[j] = h[j];
                    ol[j] = l[j];
                }
        }
    }
    if (e.flags & kEpiKvScatter) {
        // 16-column chunks never straddle a head (head width 64) nor the K/V boundary (d_model).
        const int kv = col / e.d_model;
        const int cc = col - kv * e.d_model;
        const int h = cc >> 6, j0 = cc & 63;
        const int slot = e.row_slot[row], t = e.row_pos[row];
        float* dst = (kv ? e.vc : e.kc) + static_cast<long long>(slot) * e.slot_stride +
                     (static_cast<long long>(h) * e.cap + t) * 64 + j0;
#pragma unroll
        for (int j = 0; j < 16; j += 4) st4(dst + j, v[j], v[j + 1], v[j + 2], v[j + 3]);
    }
}

__device__ __forceinline__ void epi_bar() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

__global__ void __launch_bounds__(kThreads, 1) gemm_3xtf32_kernel(const __grid_constant__ GemmKParams p) {
    // An earlier kernel on this context already failed: do nothing rather than wait on it.
    if (p.err && *reinterpret_cast<volatile int*>(p.err) != 0) return;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    const int bn = p.bn;
    const int stages = p.stages;
    const int b_tile_bytes = bn * kBK * 4;
    const int stage_bytes = 2 * kATileBytes + 2 * b_tile_bytes;
    uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + static_cast<size_t>(stages) * stage_bytes);
    uint64_t* empty_bar = full_bar + stages;
    uint64_t* accum_bar = empty_bar + stages;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(accum_bar + 1);
    int* last_flag = reinterpret_cast<int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int nt = blockIdx.x, mt = blockIdx.y, split = blockIdx.z;
    const int m0 = mt * kBM, n0 = nt * bn;
    const int kb0 = split * p.kb_per_split;
    const int kb1 = min(p.total_kb, kb0 + p.kb_per_split);
    const int nkb = kb1 - kb0;

    if (warp == 0 && lane == 0) {
        tma_prefetch_desc(&p.a_hi);
        tma_prefetch_desc(&p.a_lo);
        tma_prefetch_desc(&p.b_hi);
        tma_prefetch_desc(&p.b_lo);
        for (int s = 0; s < stages; ++s) {
            mbar_init(&full_bar[s], 1);
            mbar_init(&empty_bar[s], 1);
        }
        mbar_init(accum_bar, 1);
        fence_barrier_init();
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, p.tmem_cols);
        tmem_relinquish();
    }
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    if (warp == 0) {
        if (lane == 0 && nkb > 0) {
            for (int i = 0; i < nkb; ++i) {
                const int s = i % stages;
                const uint32_t round = static_cast<uint32_t>(i / stages);
                if (!mbar_wait(&empty_bar[s], (round & 1u) ^ 1u, p.err, kDevTimeoutSmemEmpty)) break;
                uint8_t* st = smem + static_cast<size_t>(s) * stage_bytes;
                mbar_arrive_expect_tx(&full_bar[s], static_cast<uint32_t>(stage_bytes));
                const int kx = (kb0 + i) * kBK;
                tma_load_2d(st, &p.a_hi, &full_bar[s], kx, m0);
                tma_load_2d(st + kATileBytes, &p.a_lo, &full_bar[s], kx, m0);
                tma_load_2d(st + 2 * kATileBytes, &p.b_hi, &full_bar[s], kx, n0);
                tma_load_2d(st + 2 * kATileBytes + b_tile_bytes, &p.b_lo, &full_bar[s], kx, n0);
            }
        }
    } else if (warp == 1) {
        if (lane == 0 && nkb > 0) {
            bool ok = true;
            for (int i = 0; i < nkb && ok; ++i) {
                const int s = i % stages;
                const uint32_t round = static_cast<uint32_t>(i / stages);
                if (!mbar_wait(&full_bar[s], round & 1u, p.err, kDevTimeoutTmaFull)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t st = smem_u32(smem + static_cast<size_t>(s) * stage_bytes);
                const uint32_t a_hi = st, a_lo = st + kATileBytes;
                const uint32_t b_hi = st + 2 * kATileBytes, b_lo = b_hi + b_tile_bytes;
#pragma unroll
                for (int kk = 0; kk < kBK / 8; ++kk) {
                    const uint32_t off = kk * 32;  // 8 tf32 = 32 bytes along the swizzled row
                    const uint32_t acc = (i > 0 || kk > 0) ? 1u : 0u;
                    // small terms first, then the dominant hi*hi product
                    mma_tf32(tmem_base, smem_desc_k_sw128(a_lo + off), smem_desc_k_sw128(b_hi + off),
                             p.idesc, acc);
                    mma_tf32(tmem_base, smem_desc_k_sw128(a_hi + off), smem_desc_k_sw128(b_lo + off),
                             p.idesc, 1u);
                    mma_tf32(tmem_base, smem_desc_k_sw128(a_hi + off), smem_desc_k_sw128(b_hi + off),
                             p.idesc, 1u);
                }
                mma_commit(&empty_bar[s]);
            }
            if (ok) mma_commit(accum_bar);
        }
    } else {
        // ---------------- epilogue warps 2..5 ----------------
        const int q = warp & 3;  // TMEM lane quarter this warp may access
        const int row_local = q * 32 + lane;
        const int row = m0 + row_local;
        const bool row_ok = row < p.M;
        const bool have = nkb > 0 && mbar_wait(accum_bar, 0, p.err, kDevTimeoutAccum);
        tc_fence_after();
        ArgState as{-INFINITY, kArgNone, 0};
        const uint32_t taddr = tmem_base + (static_cast<uint32_t>(q * 32) << 16);
        if (p.splits == 1) {
            for (int c0 = 0; c0 < bn; c0 += 16) {
                float v[16];
                if (have) {
                    tmem_ld_16(taddr + c0, v);
                } else {
#pragma unroll
                    for (int j = 0; j < 16; ++j) v[j] = 0.f;
                }
                if (row_ok && n0 + c0 < p.N) epilogue16(p, row, n0 + c0, v, as);
            }
        } else {
            const size_t tile_elems = static_cast<size_t>(kBM) * bn;
            float* ws_mine = p.ws + (static_cast<size_t>(split * p.m_tiles + mt) * p.n_tiles + nt) * tile_elems +
                             static_cast<size_t>(row_local) * bn;
            for (int c0 = 0; c0 < bn; c0 += 16) {
                float v[16];
                if (have) {
                    tmem_ld_16(taddr + c0, v);
                } else {
#pragma unroll
                    for (int j = 0; j < 16; ++j) v[j] = 0.f;
                }
#pragma unroll
                for (int j = 0; j < 16; j += 4) st4(ws_mine + c0 + j, v[j], v[j + 1], v[j + 2], v[j + 3]);
            }
            __threadfence();
            epi_bar();
            const int ticket_id = mt * p.n_tiles + nt;
            if (threadIdx.x == 64) {
                const int t = atomicAdd(p.tickets + ticket_id, 1);
                *last_flag = (t == p.splits - 1) ? 1 : 0;
            }
            epi_bar();
            if (*last_flag) {
                __threadfence();
                for (int c0 = 0; c0 < bn; c0 += 16) {
                    float v[16];
#pragma unroll
                    for (int j = 0; j < 16; ++j) v[j] = 0.f;
                    for (int s = 0; s < p.splits; ++s) {
                        const float* src = p.ws + (static_cast<size_t>(s * p.m_tiles + mt) * p.n_tiles + nt) * tile_elems +
                                           static_cast<size_t>(row_local) * bn + c0;
#pragma unroll
                        for (int j = 0; j < 16; j += 4) {
                            const float4 t4 = __ldcg(reinterpret_cast<const float4*>(src + j));
                            v[j] += t4.x;
                            v[j + 1] += t4.y;
                            v[j + 2] += t4.z;
                            v[j + 3] += t4.w;
                        }
                    }
                    if (row_ok && n0 + c0 < p.N) epilogue16(p, row, n0 + c0, v, as);
                }
                if (threadIdx.x == 64) p.tickets[ticket_id] = 0;
            }
        }
        if (p.epi.flags & kEpiArgmax) {
            // splits == 1 here (host-enforced). Partial of this N tile, then the last tile of the
            // row block reduces the partials in tile order (first maximum wins).
            if (row_ok) {
                p.arg_val[static_cast<size_t>(row) * p.n_tiles + nt] = as.best;
                p.arg_idx[static_cast<size_t>(row) * p.n_tiles + nt] =
                    (as.idx & 0x7FFFFFFF) | (as.nf ? static_cast<int>(0x80000000u) : 0);
            }
            __threadfence();
            epi_bar();
            if (threadIdx.x == 64) {
                const int t = atomicAdd(p.tickets + mt, 1);
                *last_flag = (t == p.n_tiles - 1) ? 1 : 0;
            }
            epi_bar();
            if (*last_flag) {
                __threadfence();
                if (row_ok) {
                    float best = -INFINITY;
                    int idx = kArgNone, nf = 0;
                    for (int t = 0; t < p.n_tiles; ++t) {
                        const float bv = __ldcg(p.arg_val + static_cast<size_t>(row) * p.n_tiles + t);
                        const int bi = __ldcg(p.arg_idx + static_cast<size_t>(row) * p.n_tiles + t);
                        nf |= (bi >> 31) & 1;
                        const int ii = bi & 0x7FFFFFFF;
                        if (ii != kArgNone && bv > best) {
                            best = bv;
                            idx = ii;
                        }
                    }
                    p.epi.next_ids[row] = (idx == kArgNone) ? -1 : idx;
                    if (p.epi.nonfinite) p.epi.nonfinite[row] = (nf || idx == kArgNone) ? 1 : 0;
                }
                if (threadIdx.x == 64) p.tickets[mt] = 0;
            }
        }
        tc_fence_before();
    }
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, p.tmem_cols);
    }
}

// ---------------------------------------------------------------------------------------------
// Host side
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    });
    return fn;
}

bool make_map(CUtensorMap* map, const float* base, int K, int rows, int box_rows) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return false;
    if ((reinterpret_cast<uintptr_t>(base) & 15) != 0 || (K & 3) != 0) return false;
    cuuint64_t dims[2] = {static_cast<cuuint64_t>(K), static_cast<cuuint64_t>(rows)};
    cuuint64_t strides[1] = {static_cast<cuuint64_t>(K) * 4};
    cuuint32_t box[2] = {static_cast<cuuint32_t>(kBK), static_cast<cuuint32_t>(box_rows)};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(base), dims, strides,
                    box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

size_t stage_bytes_for(int bn) { return 2 * static_cast<size_t>(kATileBytes) + 2 * static_cast<size_t>(bn) * kBK * 4; }

}  // namespace

bool tensor_map_api_available() { return encode_fn() != nullptr; }

GemmPlan gemm_plan(int M, int N, int K, int flags, int num_sms) {
    GemmPlan best;
    double best_t = 1e300;
    const int m_tiles = (M + kBM - 1) / kBM;
    const int total_kb = (K + kBK - 1) / kBK;
    const int n16 = (N + 15) / 16 * 16;
    const int cands[] = {256, 224, 192, 160, 128, 96, 64, 48, 32, 16};
    for (int bn : cands) {
        if (bn > n16 && bn != 16) {
            // a tile wider than the matrix only wastes work; keep the smallest that covers it
            bool smaller_covers = false;
            for (int b2 : cands)
                if (b2 < bn && b2 >= n16) smaller_covers = true;
            if (smaller_covers) continue;
        }
        const int n_tiles = (N + bn - 1) / bn;
        const int tiles = m_tiles * n_tiles;
        const int max_split = (flags & (kEpiArgmax)) ? 1 : std::min(16, total_kb);
        for (int s = 1; s <= max_split; ++s) {
            const int kbc = (total_kb + s - 1) / s;
            const int s_eff = (total_kb + kbc - 1) / kbc;
            if (s_eff != s) continue;
            const long long ctas = static_cast<long long>(tiles) * s_eff;
            const long long waves = (ctas + num_sms - 1) / num_sms;
            // per-CTA time ~ fixed cost + per K-block cost (MMA ~ bn, A tile ~ constant)
            double t = static_cast<double>(waves) * (40.0 + kbc * (bn + 96.0));
            if (s_eff > 1) t += 3.0 * s_eff * bn / 16.0 + 30.0;
            if (t < best_t - 1e-9) {
                best_t = t;
                best.bn = bn;
                best.splits = s_eff;
                best.kb_per_split = kbc;
                best.m_tiles = m_tiles;
                best.n_tiles = n_tiles;
            }
        }
    }
    const size_t sb = stage_bytes_for(best.bn);
    int stages = static_cast<int>((kSmemLimit - kSmemReserve) / sb);
    stages = std::max(1, std::min(stages, 8));
    stages = std::min(stages, std::max(1, best.kb_per_split));
    best.stages = stages;
    best.smem_bytes = stages * sb + kSmemReserve;
    // Keep (CTAs resident per SM) x (TMEM columns per CTA) <= 512: pad the shared-memory request
    // so that no more CTAs fit on an SM than its tensor memory can hold at once.
    uint32_t cols = 32;
    while (cols < static_cast<uint32_t>(best.bn)) cols <<= 1;
    const size_t max_ctas = 512 / cols;
    const size_t sm_bytes = 228 * 1024;
    const size_t min_smem = sm_bytes / (max_ctas + 1) + 1;  // max_ctas + 1 CTAs must not fit
    if (best.smem_bytes < min_smem) best.smem_bytes = min_smem;
    return best;
}

size_t gemm_ws_floats(const GemmPlan& p) {
    return p.splits > 1 ? static_cast<size_t>(p.splits) * p.m_tiles * p.n_tiles * kBM * p.bn : 0;
}

size_t gemm_arg_entries(const GemmPlan& p) {
    return static_cast<size_t>(p.m_tiles) * kBM * p.n_tiles;
}

int gemm_launch(const TcActs& a, int M, const TcWeight& w, const GemmEpilogue& epi,
                const GemmPlan& plan, const GemmScratch& scratch, int* err, cudaStream_t st) {
    {
        // The attribute is per device; set it once for each device this process launches on.
        static std::mutex mu;
        static unsigned long long done_mask = 0;
        int dev = 0;
        cudaGetDevice(&dev);
        std::lock_guard<std::mutex> lock(mu);
        if (dev < 64 && !(done_mask & (1ull << dev))) {
            const cudaError_t e = cudaFuncSetAttribute(
                gemm_3xtf32_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                static_cast<int>(kSmemLimit));
            if (e != cudaSuccess) return static_cast<int>(e);
            done_mask |= (1ull << dev);
        }
    }
    if (M <= 0 || w.N <= 0 || w.K <= 0 || a.K != w.K) return cudaErrorInvalidValue;
    if (a.rows_alloc < plan.m_tiles * kBM) return cudaErrorInvalidValue;
    if (plan.bn % 16 || plan.bn < 16 || plan.bn > 256) return cudaErrorInvalidValue;
    if ((epi.flags & kEpiArgmax) && plan.splits != 1) return cudaErrorInvalidValue;
    if (plan.splits > 1 && (scratch.ws == nullptr || scratch.ws_floats < gemm_ws_floats(plan) ||
                            scratch.n_tickets < plan.m_tiles * plan.n_tiles))
        return cudaErrorInvalidValue;
    if ((epi.flags & kEpiArgmax) &&
        (scratch.arg_val == nullptr || scratch.arg_entries < gemm_arg_entries(plan) ||
         scratch.n_tickets < plan.m_tiles || epi.next_ids == nullptr))
        return cudaErrorInvalidValue;
    if ((epi.flags & kEpiKvScatter) && (epi.d_model % 64 != 0 || w.N != 2 * epi.d_model))
        return cudaErrorInvalidValue;
    const int n_rows_alloc = (w.N + 255) / 256 * 256;

    GemmKParams p{};
    if (!make_map(&p.a_hi, a.hi, a.K, a.rows_alloc, kBM) ||
        !make_map(&p.a_lo, a.lo, a.K, a.rows_alloc, kBM) ||
        !make_map(&p.b_hi, w.hi, w.K, n_rows_alloc, plan.bn) ||
        !make_map(&p.b_lo, w.lo, w.K, n_rows_alloc, plan.bn))
        return cudaErrorInvalidValue;
    p.M = M;
    p.N = w.N;
    p.K = w.K;
    p.bn = plan.bn;
    p.stages = plan.stages;
    p.kb_per_split = plan.kb_per_split;
    p.splits = plan.splits;
    p.n_tiles = plan.n_tiles;
    p.m_tiles = plan.m_tiles;
    p.total_kb = (w.K + kBK - 1) / kBK;
    p.idesc = idesc_tf32(kBM, plan.bn);
    uint32_t cols = 32;
    while (cols < static_cast<uint32_t>(plan.bn)) cols <<= 1;
    p.tmem_cols = cols;
    p.epi = epi;
    p.ws = scratch.ws;
    p.tickets = scratch.tickets;
    p.arg_val = scratch.arg_val;
    p.arg_idx = scratch.arg_idx;
    p.err = err;
    dim3 grid(plan.n_tiles, plan.m_tiles, plan.splits);
    gemm_3xtf32_kernel<<<grid, kThreads, plan.smem_bytes, st>>>(p);
    return static_cast<int>(cudaGetLastError());
}

}  // namespace adai_b200
