// gemm_tc.cu — fp32-accurate GEMM on the 5th-generation tensor cores (sm_100a).
//
// Replaces the reference's Matrix::operator* / matrix_multiply_gpu (src/Matrix.cpp:212-277,
// src/gpu/MatrixGPU.cu:351-370, cuBLAS SGEMM) for the stacked decode projections (Q/K/V/O,
// cross-attention, FFN, LM head) and the encoder prefill.
//
// Precision: 3xTF32. Each fp32 operand x is split into hi = tf32(x) and lo = tf32(x - hi)
// (round to nearest); the product is accumulated as
//     A*W ~= A_hi*W_hi + (A_lo*W_hi + A_hi*W_lo),
// the published error-corrected TF32 scheme (Ootomo & Yokota, 2022). The weights are split once
// at upload (stored W^T, K-major, hi and lo planes); activations arrive already split by the
// kernel that produced them. The tensor core's accumulation does not round to nearest, so a long
// K sum kept in one TMEM accumulator drifts toward zero; here the accumulator is promoted to
// fp32 registers chunk by chunk (double-buffered TMEM, hi*hi and correction terms in separate
// accumulators), which keeps the error at or below an fp32 FMA chain.
//
// One CTA computes one 128 x BN output tile over one K-slice:
//   warp 0    TMA producer: 4 boxes per stage (A_hi, A_lo 128x32; W_hi, W_lo BNx32), 128B swizzle
//   warp 1    TMEM allocator + tcgen05.mma issuer of A_hi*W_hi
//   warps 6-7 tcgen05.mma issuers of the correction terms (one warp for both at BN = 128), each
//             into its own TMEM accumulator
//   warps 2-5 promote finished TMEM chunks into fp32 registers (one output row per thread), and
//             with two TMEM buffers four more warps after the issuers, each pair of warps on one
//             TMEM lane quarter splitting the row's columns
// Two variants: 224-column tiles (the LM head, one wave of CTAs) keep a single TMEM buffer, so the
// K slice is one chunk that the epilogue streams to shared memory 16 columns at a time; and the
// op-level product of a small fp32 A (kEpiAFp32) lets TMA bring the raw A box into a third plane
// of each stage, where two more warps split it into A_hi / A_lo before the MMAs read them.
// Split-K: the S K-slices of a tile are the S CTAs of one thread-block cluster. Each CTA stages
// its partial tile in its own shared memory and ships the rows it does not own to their owners
// with one bulk copy per owner (cp.async.bulk shared::cta -> shared::cluster, completing on the
// owner's mbarrier); every CTA then sums its 128/S rows over the S slots in rank order 0..S-1
// (deterministic) and runs the fused epilogue with coalesced float4 stores:
// folded LayerNorm / bias / GELU / residual / fp32 store / tf32 split of the output / row
// statistics for the next folded LayerNorm / KV-cache scatter / first-maximum argmax partials
// (the LM head). The epilogue is a template parameter so each
// instantiation carries only its own code. No TMA multicast anywhere.
#include <algorithm>
#include <cstdio>
#include <cstring>
#include <cstdlib>
#include <map>
#include <mutex>
#include <tuple>

#include "common.cuh"
#include "kernels.h"

namespace adai_b200 {

namespace {

constexpr int kBM = 128;
constexpr int kBK = 32;  // fp32 elements per 128-byte swizzled row

// The three MMAs of a 3xTF32 k-step are issued by up to three threads of different warps, each
// into its own TMEM accumulator: a single thread issuing tcgen05.mma back to back, with the
// barrier wait, fence and commit of every K block, is limited by its own issue rate (measured on
// B200: about 35 ns per MMA and 0.3 us per K block of synchronisation), while a second issuing
// warp nearly doubles the tensor core's rate for N <= 64.
// Accumulators: 0 = A_hi*B_hi, 1 = A_lo*B_hi (and A_hi*B_lo when there are two), 2 = A_hi*B_lo.
// Two TMEM buffers of kNAcc x BN columns must fit the 512 columns of an SM.
template <int BN>
struct GemmShape {
    static constexpr int kNAcc = (6 * BN <= 512) ? 3 : 2;
    // TMEM buffers of the accumulators: two (chunks promoted while the next one accumulates), or
    // one for tiles too wide for two (224 columns, the LM head): the K slice is then one chunk.
    static constexpr int kTBufs = (2 * kNAcc * BN <= 512) ? 2 : 1;
    // warp 0 TMA producer, warp 1 issuer 0, warps 2-5 epilogue, warps 6 .. kIssuerEnd-1 further
    // issuers; with two TMEM buffers four more epilogue warps follow, so that two warps share
    // each TMEM lane quarter, each promoting half of the tile's columns.
    static constexpr int kIssuerEnd = 6 + kNAcc - 1;
    static constexpr int kEpiWarps = (kTBufs == 2) ? 8 : 4;
    static constexpr int kWarps = kIssuerEnd + kEpiWarps - 4;
    static constexpr int kThreads = 32 * kWarps;
};
int threads_for(int bn, int flags = 0) {
    const int conv = (flags & kEpiAFp32) ? 64 : 0;  // the fp32-A converter warps
    switch (bn) {
        case 32: return GemmShape<32>::kThreads + conv;
        case 64: return GemmShape<64>::kThreads + conv;
        case 224: return GemmShape<224>::kThreads + conv;
        default: return GemmShape<128>::kThreads + conv;
    }
}
int nacc_for(int bn) { return (6 * bn <= 512) ? 3 : 2; }
constexpr int kATileBytes = kBM * kBK * 4;  // 16 KB
constexpr size_t kSmemLimit = 227 * 1024;
constexpr size_t kSmemReserve = 1024 /*alignment slack*/ + 256 /*barriers*/ + 1024 /*row mean, rstd*/;
constexpr int kMaxCluster = 16;  // 8 is portable; 16 is used only where the device can place it

// The epilogue flag sets the decode step and the op-level entry points use.
constexpr int kEpiSetStore = kEpiStore;
constexpr int kEpiSetResid = kEpiStore | kEpiResid;
constexpr int kEpiSetFfnUp = kEpiBias | kEpiGelu | kEpiSplit;
constexpr int kEpiSetFfnDown = kEpiBias | kEpiResid | kEpiStore;
constexpr int kEpiSetHead = kEpiBias | kEpiArgmax;
constexpr int kEpiSetHeadLogits = kEpiBias | kEpiArgmax | kEpiStore;
constexpr int kEpiSetScatter = kEpiKvScatter;
// The decode step's variants with the LayerNorm folded into the consuming GEMM: the GEMMs that
// update the residual stream also write its tf32 split and row statistics.
constexpr int kEpiSetStoreLn = kEpiBias | kEpiStore | kEpiLnFold;
constexpr int kEpiSetResidStats = kEpiStore | kEpiResid | kEpiSplit | kEpiRowStats;
constexpr int kEpiSetFfnUpLn = kEpiBias | kEpiGelu | kEpiSplit | kEpiLnFold;
constexpr int kEpiSetFfnDownStats = kEpiBias | kEpiResid | kEpiStore | kEpiSplit | kEpiRowStats;
constexpr int kEpiSetHeadLn = kEpiBias | kEpiArgmax | kEpiLnFold;
constexpr int kEpiSetHeadLogitsLn = kEpiBias | kEpiArgmax | kEpiStore | kEpiLnFold;
// The op-level product with A in fp32, split inside the GEMM.
constexpr int kEpiSetStoreAF = kEpiStore | kEpiAFp32;

// Warps of a launch: the shape's, plus two converter warps when A arrives in fp32.
template <int BN, int EPI>
struct GemmWarps {
    static constexpr bool kAF = (EPI & kEpiAFp32) != 0;
    static constexpr int kConvWarps = kAF ? 2 : 0;
    static constexpr int kWarps = GemmShape<BN>::kWarps + kConvWarps;
    static constexpr int kThreads = 32 * kWarps;
};

struct __align__(64) GemmKParams {
    CUtensorMap a_hi, a_lo, b_hi, b_lo;
    int M, N, K;
    int stages, kb_per_split, splits, n_tiles, m_tiles, total_kb, chunk_kb, rows_per;
    int pair_commit;  // 1: the MMA issuers free the stages two at a time (even stage counts)
    uint32_t idesc, tmem_cols;
    GemmEpilogue epi;
    int* tickets;
    unsigned long long* arg_key;
    int* arg_nf;
    int* err;
};

constexpr int kArgNone = 0x7FFFFFFF;

// First-maximum argmax across CTAs as one 64-bit atomicMax per row: the high word orders like
// the float (sign-magnitude bits mapped to an unsigned order; -0 folded into +0 so the two
// compare equal, as they do in the reference's `>`), the low word is the complemented column,
// so equal values resolve to the lowest column. Zero means "no candidate": every finite value
// and +inf map to a non-zero high word.
__device__ __forceinline__ unsigned long long arg_key_of(float v, int col) {
    const uint32_t u = __float_as_uint(v == 0.f ? 0.f : v);
    const uint32_t ord = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
    return (static_cast<unsigned long long>(ord) << 32) | (0xFFFFFFFFu - static_cast<uint32_t>(col));
}
__device__ __forceinline__ int arg_col_of(unsigned long long key) {
    return static_cast<int>(0xFFFFFFFFu - static_cast<uint32_t>(key & 0xFFFFFFFFull));
}

struct ArgState {
    float best;
    int idx;
    int nf;
};

__device__ __forceinline__ void st4(float* p, float4 v) { *reinterpret_cast<float4*>(p) = v; }

// Epilogue on 4 consecutive output columns [col, col+4) of one row (col % 4 == 0, col < N);
// returns the final values (after the residual add). mean / rstd: the row's LayerNorm
// statistics (kEpiLnFold only).
template <int EPI>
__device__ __forceinline__ float4 epilogue4(const GemmKParams& p, int row, int col, float4 acc,
                                            ArgState& as, float mean = 0.f, float rstd = 0.f) {
    const GemmEpilogue& e = p.epi;
    const int nv = min(4, p.N - col);
    float v[4] = {acc.x, acc.y, acc.z, acc.w};
    if constexpr ((EPI & kEpiLnFold) != 0) {
        // sum_k LN(x)_k W_kn = rstd * (sum_k x_k gamma_k W_kn - mean * ln_c1[n]) + (beta W)_n
        float c1[4] = {0.f, 0.f, 0.f, 0.f};
        if (nv == 4) {
            const float4 c4 = __ldg(reinterpret_cast<const float4*>(e.ln_c1 + col));
            c1[0] = c4.x;
            c1[1] = c4.y;
            c1[2] = c4.z;
            c1[3] = c4.w;
        } else {
#pragma unroll
            for (int j = 0; j < 4; ++j)
                if (j < nv) c1[j] = __ldg(e.ln_c1 + col + j);
        }
#pragma unroll
        for (int j = 0; j < 4; ++j) v[j] = rstd * fmaf(-mean, c1[j], v[j]);
    }
    if constexpr ((EPI & kEpiBias) != 0) {
        if (nv == 4) {
            const float4 b4 = __ldg(reinterpret_cast<const float4*>(e.bias + col));
            v[0] += b4.x;
            v[1] += b4.y;
            v[2] += b4.z;
            v[3] += b4.w;
        } else {
#pragma unroll
            for (int j = 0; j < 4; ++j)
                if (j < nv) v[j] += __ldg(e.bias + col + j);
        }
    }
    if constexpr ((EPI & kEpiGelu) != 0) {
#pragma unroll
        for (int j = 0; j < 4; ++j) v[j] = gelu_tanh(v[j]);
    }
    if constexpr ((EPI & kEpiResid) != 0) {
        const float* r = e.resid + static_cast<size_t>(row) * e.ldr + col;
        if (nv == 4 && (e.ldr & 3) == 0) {
            const float4 rv = *reinterpret_cast<const float4*>(r);
            v[0] = rv.x + v[0];
            v[1] = rv.y + v[1];
            v[2] = rv.z + v[2];
            v[3] = rv.w + v[3];
        } else {
#pragma unroll
            for (int j = 0; j < 4; ++j)
                if (j < nv) v[j] = r[j] + v[j];
        }
    }
    if constexpr ((EPI & kEpiArgmax) != 0) {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            if (j < nv) {
                const float x = v[j];
                if (isnan(x) || x == INFINITY) as.nf = 1;
                if (x > as.best) {  // strictly greater: the first maximum in column order wins
                    as.best = x;
                    as.idx = col + j;
                }
            }
        }
    }
    if constexpr ((EPI & kEpiStore) != 0) {
        float* o = e.out + static_cast<size_t>(row) * e.ldo + col;
        if (nv == 4 && (e.ldo & 3) == 0) {
            st4(o, make_float4(v[0], v[1], v[2], v[3]));
        } else {
#pragma unroll
            for (int j = 0; j < 4; ++j)
                if (j < nv) o[j] = v[j];
        }
    }
    if constexpr ((EPI & kEpiSplit) != 0) {
        float h[4], l[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) split_tf32(v[j], h[j], l[j]);
        float* oh = e.out_hi + static_cast<size_t>(row) * e.lds + col;
        float* ol = e.out_lo + static_cast<size_t>(row) * e.lds + col;
        if (nv == 4 && (e.lds & 3) == 0) {
            st4(oh, make_float4(h[0], h[1], h[2], h[3]));
            st4(ol, make_float4(l[0], l[1], l[2], l[3]));
        } else {
#pragma unroll
            for (int j = 0; j < 4; ++j)
                if (j < nv) {
                    oh[j] = h[j];
                    ol[j] = l[j];
                }
        }
    }
    if constexpr ((EPI & kEpiKvScatter) != 0) {
        // columns [0, D) are K, [D, 2D) are V; a 4-column group never straddles a head.
        const int kv = col / e.d_model;
        const int cc = col - kv * e.d_model;
        const int h = cc / e.head_dim, j0 = cc - h * e.head_dim;
        const int slot = e.row_slot[row], t = e.row_pos[row];
        float* dst = (kv ? e.vc : e.kc) + static_cast<long long>(slot) * e.slot_stride +
                     (static_cast<long long>(h) * e.cap + t) * e.head_dim + j0;
        st4(dst, make_float4(v[0], v[1], v[2], v[3]));
    }
    return make_float4(v[0], v[1], v[2], v[3]);
}

// Combines the K / 32 group statistics (sum, squared deviations from the group mean) of one row,
// contiguous at st, in group order (the parallel-variance combination of Chan et al.):
// LayerNorm's mean and 1 / sqrt(biased variance + 1e-5), as LayerNorm::forward computes them
// from the whole row. K is a multiple of 64 (two groups per 16-byte load).
__device__ __forceinline__ void ln_row_stats(const float2* __restrict__ st, int K, float& mean,
                                             float& rstd) {
    const float4* s4 = reinterpret_cast<const float4*>(st);
    const int pairs = K >> 6;
    float sum = 0.f;
#pragma unroll 8
    for (int t = 0; t < pairs; ++t) {
        const float4 g = __ldg(s4 + t);
        sum += g.x;
        sum += g.z;
    }
    mean = sum / static_cast<float>(K);
    float m2 = 0.f;
#pragma unroll 8
    for (int t = 0; t < pairs; ++t) {
        const float4 g = __ldg(s4 + t);
        const float d0 = g.x * (1.0f / 32.0f) - mean, d1 = g.z * (1.0f / 32.0f) - mean;
        m2 += g.y + 32.0f * d0 * d0;
        m2 += g.w + 32.0f * d1 * d1;
    }
    rstd = 1.0f / sqrtf(m2 / static_cast<float>(K) + 1e-5f);
}

// Group statistics of 32 consecutive values of one row, held as one float4 by each of 8
// consecutive lanes (lane % 8 == 0 holds the first four): written by that lane.
__device__ __forceinline__ void row_group_stats(float4 v, float2* dst, int lane) {
    const unsigned seg = 0xFFu << (lane & 24);
    float s = (v.x + v.y) + (v.z + v.w);
    s += __shfl_xor_sync(seg, s, 1);
    s += __shfl_xor_sync(seg, s, 2);
    s += __shfl_xor_sync(seg, s, 4);
    const float mg = s * (1.0f / 32.0f);
    const float a = v.x - mg, b = v.y - mg, c = v.z - mg, d = v.w - mg;
    float q = (a * a + b * b) + (c * c + d * d);
    q += __shfl_xor_sync(seg, q, 1);
    q += __shfl_xor_sync(seg, q, 2);
    q += __shfl_xor_sync(seg, q, 4);
    if ((lane & 7) == 0) *dst = make_float2(s, q);
}

template <int BN, int EPI>
__global__ void __launch_bounds__(GemmWarps<BN, EPI>::kThreads, 1) gemm_3xtf32_kernel(const __grid_constant__ GemmKParams p) {
    constexpr int kThreads = GemmWarps<BN, EPI>::kThreads;
    constexpr int kWarps = GemmWarps<BN, EPI>::kWarps;
    constexpr bool kAF = GemmWarps<BN, EPI>::kAF;
    constexpr int kNAcc = GemmShape<BN>::kNAcc;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    constexpr bool kArgmax = (EPI & kEpiArgmax) != 0;
    constexpr int b_tile_bytes = BN * kBK * 4;
    // kAF: a third A plane per stage holds the raw fp32 box TMA brings
    constexpr int stage_bytes = (kAF ? 3 : 2) * kATileBytes + 2 * b_tile_bytes;
    constexpr int raw_off = 2 * kATileBytes + 2 * b_tile_bytes;  // kAF: the raw A box in a stage
    constexpr int kChunks = BN / 4;  // float4 columns per output row
    const int stages = p.stages;
    const int S = p.splits;
    const int rows_per = p.rows_per;  // 128 / S: output rows each cluster rank finishes
    const size_t pipe_bytes = static_cast<size_t>(stages) * stage_bytes;
    // Once the mainloop is over the pipeline buffers hold, from their start: this CTA's partial
    // tile, [128 rows][BN] fp32 with float4 columns XOR-swizzled by (row & 7) (conflict-free row
    // writes and column reads), then with S > 1 the peers' partials of this rank's rows,
    // [S slots][rows_per][BN], same swizzle (rows_per is a multiple of 8). Peers write there
    // only after the cluster barrier that follows this CTA's last pipeline use.
    constexpr size_t stage_tile_bytes = static_cast<size_t>(kBM) * BN * 4;
    uint8_t* stage_out = smem;
    uint8_t* recv = smem + stage_tile_bytes;
    const size_t recv_bytes = (S > 1) ? static_cast<size_t>(S) * rows_per * BN * 4 : 0;
    const size_t region_bytes = max(pipe_bytes, stage_tile_bytes + recv_bytes);
    uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + region_bytes);
    uint64_t* empty_bar = full_bar + stages;
    uint64_t* tfull_bar = empty_bar + stages;  // [2] chunk accumulated in TMEM buffer b
    uint64_t* tempty_bar = tfull_bar + 2;      // [2] TMEM buffer b drained by the epilogue
    uint64_t* recv_bar = tempty_bar + 2;       // peers' partials have landed in `recv`
    uint64_t* done_bar = recv_bar + 1;         // [3] every MMA issuer i issued has completed
    uint64_t* a_ready = done_bar + 3;          // [stages] kAF: the converters split the stage's A
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(a_ready + (kAF ? stages : 0));
    int* last_flag = reinterpret_cast<int*>(tmem_slot + 1);
    // LayerNorm mean / rstd of the tile's rows (kEpiLnFold), after the 256 bytes of barriers
    float* ln_mean = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(full_bar) + 256);
    float* ln_rstd = ln_mean + kBM;

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int nt = blockIdx.x, mt = blockIdx.y;
    const int rank = (S > 1) ? static_cast<int>(cluster_ctarank()) : 0;
    const int m0 = mt * kBM, n0 = nt * BN;
    const int kb0 = rank * p.kb_per_split;
    const int kb1 = min(p.total_kb, kb0 + p.kb_per_split);
    const int nkb = max(0, kb1 - kb0);
    const int CK = p.chunk_kb;
    const int nchunks = (nkb + CK - 1) / CK;
    const int n_first = min(stages, nkb);  // stages filled before the first wait for an empty one
    // Each weight box is read by one CTA once: its lines go first when L2 needs room.
    const uint64_t w_policy = (warp == 0 && lane == 0) ? l2_policy_evict_first() : 0;
    // The activation boxes are read by every N tile's CTA: kept longest.
    const uint64_t a_policy = (warp == 0 && lane == 0) ? l2_policy_evict_last() : 0;
    // kAF: one raw A box instead of the two split planes
    constexpr uint32_t tx_bytes = (kAF ? 1 : 2) * kATileBytes + 2 * b_tile_bytes;

    if (warp == 0 && lane == 0) {
        tma_prefetch_desc(&p.a_hi);
        if constexpr (!kAF) tma_prefetch_desc(&p.a_lo);
        tma_prefetch_desc(&p.b_hi);
        tma_prefetch_desc(&p.b_lo);
        for (int s = 0; s < stages; ++s) {
            mbar_init(&full_bar[s], 1);
            mbar_init(&empty_bar[s], kNAcc);  // one commit per MMA issuer
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&tfull_bar[b], kNAcc);  // one commit per MMA issuer
            mbar_init(&tempty_bar[b], GemmShape<BN>::kEpiWarps);  // one arrival per epilogue warp
        }
        mbar_init(recv_bar, 1);
        for (int r = 0; r < 3; ++r) mbar_init(&done_bar[r], 1);
        if constexpr (kAF)
            for (int s = 0; s < stages; ++s) mbar_init(&a_ready[s], GemmWarps<BN, EPI>::kConvWarps);
        if (S > 1)  // the phase completes once every peer's rows have arrived
            mbar_arrive_expect_tx(recv_bar, static_cast<uint32_t>((S - 1) * rows_per * BN * 4));
        fence_barrier_init();
        // Weights are constant: the first stages' weight boxes are requested as soon as their
        // barriers exist (before the tensor-memory allocation and the CTA barrier), the
        // activation boxes only after the wait for the preceding kernel.
        for (int i = 0; i < n_first; ++i) {
            uint8_t* st = smem + static_cast<size_t>(i) * stage_bytes;
            mbar_arrive_expect_tx(&full_bar[i], tx_bytes);
            const int kx = (kb0 + i) * kBK;
            tma_load_2d_hint(st + 2 * kATileBytes, &p.b_hi, &full_bar[i], kx, n0, w_policy);
            tma_load_2d_hint(st + 2 * kATileBytes + b_tile_bytes, &p.b_lo, &full_bar[i], kx, n0, w_policy);
        }
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, p.tmem_cols);
        tmem_relinquish();
    }
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    const uint32_t stage_s = smem_u32(stage_out);
    const uint32_t recv_s = smem_u32(recv);

    if (warp == 0) {
        if (lane == 0 && nkb > 0) {
            // (the first stages' weight boxes are on their way: see the barrier set-up)
            pdl_wait();
            for (int i = 0; i < n_first; ++i) {
                uint8_t* st = smem + static_cast<size_t>(i) * stage_bytes;
                const int kx = (kb0 + i) * kBK;
                if constexpr (kAF) {
                    tma_load_2d(st + raw_off, &p.a_hi, &full_bar[i], kx, m0);  // raw fp32 A
                } else {
                    tma_load_2d_hint(st, &p.a_hi, &full_bar[i], kx, m0, a_policy);
                    tma_load_2d_hint(st + kATileBytes, &p.a_lo, &full_bar[i], kx, m0, a_policy);
                }
            }
            int issued = n_first;
            for (int i = n_first; i < nkb; ++i) {
                const int s = i % stages;
                const uint32_t round = static_cast<uint32_t>(i / stages);
                // Stage s last held K block i - stages; with paired commits an even block's stage
                // is freed by the commit of the odd block after it (the next stage, same round).
                const int se = (p.pair_commit && !(s & 1)) ? s + 1 : s;
                if (!mbar_wait(&empty_bar[se], (round & 1u) ^ 1u, p.err, kDevTimeoutSmemEmpty)) break;
                uint8_t* st = smem + static_cast<size_t>(s) * stage_bytes;
                mbar_arrive_expect_tx(&full_bar[s], tx_bytes);
                const int kx = (kb0 + i) * kBK;
                if constexpr (kAF) {
                    tma_load_2d(st + raw_off, &p.a_hi, &full_bar[s], kx, m0);
                } else {
                    tma_load_2d_hint(st, &p.a_hi, &full_bar[s], kx, m0, a_policy);
                    tma_load_2d_hint(st + kATileBytes, &p.a_lo, &full_bar[s], kx, m0, a_policy);
                }
                tma_load_2d_hint(st + 2 * kATileBytes, &p.b_hi, &full_bar[s], kx, n0, w_policy);
                tma_load_2d_hint(st + 2 * kATileBytes + b_tile_bytes, &p.b_lo, &full_bar[s], kx, n0, w_policy);
                ++issued;
            }
            // No copy may still be landing in shared memory when the CTA moves on, also after an
            // abort: drain the last load of every stage (immediate when the MMAs consumed them).
            for (int i = max(0, issued - stages); i < issued; ++i)
                mbar_wait_drain(&full_bar[i % stages], static_cast<uint32_t>(i / stages) & 1u,
                                p.err, kDevTimeoutTmaFull);
        }
        if (S > 1) cluster_arrive_one();  // no copy of this CTA lands in its pipeline any more
    } else if (kAF && warp >= GemmShape<BN>::kWarps) {
        // ---- kAF converters: the stage's raw A box (as TMA wrote it, 128-byte swizzled) ->
        // A_hi and A_lo at the same offsets of their planes (the split is elementwise) ----
        constexpr int kConv = GemmWarps<BN, EPI>::kConvWarps;
        constexpr int kVec = kATileBytes / 16;
        const int cw = warp - GemmShape<BN>::kWarps;
        const uint32_t smem0 = smem_u32(smem);
        int s = 0;
        uint32_t phase = 0;
        for (int i = 0; i < nkb; ++i) {
            // every lane waits, so that each sees the copy's bytes
            const bool got = mbar_wait(&full_bar[s], phase, p.err, kDevTimeoutTmaFull);
            if (!__all_sync(0xffffffffu, got)) break;
            const uint32_t st = smem0 + static_cast<uint32_t>(s * stage_bytes);
#pragma unroll 4
            for (int v = cw * 32 + lane; v < kVec; v += 32 * kConv) {
                const uint32_t o = static_cast<uint32_t>(v * 16);
                const float4 x = ld_shared_f4(st + raw_off + o);
                float h0, h1, h2, h3, l0, l1, l2, l3;
                split_tf32(x.x, h0, l0);
                split_tf32(x.y, h1, l1);
                split_tf32(x.z, h2, l2);
                split_tf32(x.w, h3, l3);
                st_shared_f4(st + o, h0, h1, h2, h3);
                st_shared_f4(st + kATileBytes + o, l0, l1, l2, l3);
            }
            fence_proxy_async_smem();  // the tensor core reads both planes through the async proxy
            __syncwarp();
            if (lane == 0) mbar_arrive(&a_ready[s]);
            if (++s == stages) {
                s = 0;
                phase ^= 1u;
            }
        }
        if (S > 1) cluster_arrive_one();  // done with the raw A planes
    } else if (warp == 1 || (warp >= 6 && warp < GemmShape<BN>::kIssuerEnd)) {
        // ---- MMA issuers: role 0 (warp 1), 1 (warp 6), 2 (warp 7) ----
        const int role = (warp == 1) ? 0 : warp - 5;
        if (lane == 0 && nkb > 0) {
            bool ok = true;
            int i = 0, s = 0;
            uint32_t phase = 0;  // parity of stage s's current fill
            const uint32_t smem0 = smem_u32(smem);
            constexpr int kTB = GemmShape<BN>::kTBufs;
            for (int c = 0; c < nchunks && ok; ++c) {
                const int b = c % kTB;
                const uint32_t use = static_cast<uint32_t>(c / kTB);
                if (c >= kTB && !mbar_wait(&tempty_bar[b], (use - 1u) & 1u, p.err, kDevTimeoutAccum)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t t_acc = tmem_base + static_cast<uint32_t>((b * kNAcc + role) * BN);
                const int kend = min(nkb, (c + 1) * CK);
                for (; i < kend; ++i) {
                    // kAF: the converters waited for the copy and split A
                    if (!mbar_wait(kAF ? &a_ready[s] : &full_bar[s], phase, p.err, kDevTimeoutTmaFull)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    // Descriptors of the stage's planes; a k-step moves the start address by 32
                    // bytes, i.e. +2 in the descriptor's address field.
                    const uint32_t st = smem0 + static_cast<uint32_t>(s * stage_bytes);
                    const uint64_t d_ahi = smem_desc_k_sw128(st);
                    const uint64_t d_alo = smem_desc_k_sw128(st + kATileBytes);
                    const uint64_t d_bhi = smem_desc_k_sw128(st + 2 * kATileBytes);
                    const uint64_t d_blo = smem_desc_k_sw128(st + 2 * kATileBytes + b_tile_bytes);
                    const uint32_t first = (i == c * CK) ? 0u : 1u;  // 0: overwrite the accumulator
#pragma unroll
                    for (int kk = 0; kk < kBK / 8; ++kk) {
                        const uint64_t o = static_cast<uint64_t>(kk * 2);
                        const uint32_t acc = (kk == 0) ? first : 1u;
                        if (role == 0) {
                            mma_tf32(t_acc, d_ahi + o, d_bhi + o, p.idesc, acc);
                        } else if (role == 1) {
                            mma_tf32(t_acc, d_alo + o, d_bhi + o, p.idesc, acc);
                            if constexpr (kNAcc == 2) mma_tf32(t_acc, d_ahi + o, d_blo + o, p.idesc, 1u);
                        } else {
                            mma_tf32(t_acc, d_ahi + o, d_blo + o, p.idesc, acc);
                        }
                    }
                    // one commit per two K blocks with paired commits: it tracks both blocks' MMAs
                    if (!p.pair_commit || (i & 1)) mma_commit(&empty_bar[s]);
                    if (++s == stages) {
                        s = 0;
                        phase ^= 1u;
                    }
                }
                if (ok) mma_commit(&tfull_bar[b]);
            }
            // Tensor memory is released after the CTA barrier below: every MMA issued here must
            // have completed by then, also when the loop was aborted.
            mma_commit(&done_bar[role]);
            mbar_wait_drain(&done_bar[role], 0, p.err, kDevTimeoutAccum);
        }
        if (S > 1) cluster_arrive_one();  // every MMA of this issuer has read its operands
    } else {
        // ---- warps 2..5 (and kIssuerEnd..): promote each finished chunk into fp32 registers,
        // one row per thread; with eight such warps each owns half of the row's columns ----
        // These warps write only the staging tile, which the peers' partials do not overlap, so
        // they arrive on the cluster barrier at once.
        if (S > 1) cluster_arrive_one();
        pdl_wait();  // the epilogue reads and writes data of earlier kernels
        const int q = warp & 3;  // TMEM lane quarter this warp may access
        const int row_local = q * 32 + lane;
        constexpr int kCols = BN / (GemmShape<BN>::kEpiWarps / 4);  // columns one warp promotes
        const int c_lo = (warp < 6) ? 0 : kCols;
        if constexpr ((EPI & kEpiLnFold) != 0) {
            if (c_lo == 0) {  // one warp of the two per lane quarter
                float mean = 0.f, rstd = 0.f;
                if (m0 + row_local < p.M)
                    ln_row_stats(p.epi.row_stats + static_cast<size_t>(m0 + row_local) * (p.K >> 5),
                                 p.K, mean, rstd);
                ln_mean[row_local] = mean;
                ln_rstd[row_local] = rstd;
            }
        }
        const uint32_t taddr = tmem_base + (static_cast<uint32_t>(q * 32) << 16);
        // This row of the partial tile goes to the staging tile (in the pipeline buffers, free
        // once every MMA that read them has completed), float4 columns XOR-swizzled by row.
        const uint32_t row_s = stage_s + static_cast<uint32_t>(row_local * BN * 4);
        const int sw = row_local & 7;
        if constexpr (GemmShape<BN>::kTBufs == 1) {
            // One TMEM buffer and one chunk (the host guarantees nchunks <= 1): the accumulators
            // stream to the staging tile 16 columns at a time, no register copy of the row.
            static_assert(GemmShape<BN>::kNAcc == 2, "wide tiles keep two accumulators");
            int ok = (nchunks == 1) ? 1 : 0;
            if (lane == 0 && ok) ok = mbar_wait(&tfull_bar[0], 0, p.err, kDevTimeoutAccum) ? 1 : 0;
            ok = __shfl_sync(0xffffffffu, ok, 0);
            if (ok) tc_fence_after();
#pragma unroll 2
            for (int c0 = 0; c0 < BN; c0 += 16) {
                float vb[16], vs[16];
                if (ok) {
                    tmem_ld_16x2(taddr + c0, taddr + BN + c0, vb, vs);
                } else {
#pragma unroll
                    for (int j = 0; j < 16; ++j) vb[j] = vs[j] = 0.f;
                }
#pragma unroll
                for (int g = 0; g < 4; ++g) {
                    const int ch = c0 / 4 + g;
                    st_shared_f4(row_s + static_cast<uint32_t>((ch ^ sw) * 16), vb[4 * g] + vs[4 * g],
                                 vb[4 * g + 1] + vs[4 * g + 1], vb[4 * g + 2] + vs[4 * g + 2],
                                 vb[4 * g + 3] + vs[4 * g + 3]);
                }
            }
            tc_fence_before();
        } else {
            float acc[kCols];
#pragma unroll
            for (int j = 0; j < kCols; ++j) acc[j] = 0.f;
            for (int c = 0; c < nchunks; ++c) {
                const int b = c & 1;
                int ok = 1;
                if (lane == 0)
                    ok = mbar_wait(&tfull_bar[b], static_cast<uint32_t>(c >> 1) & 1u, p.err, kDevTimeoutAccum) ? 1 : 0;
                ok = __shfl_sync(0xffffffffu, ok, 0);
                if (!ok) break;
                tc_fence_after();
                const uint32_t t_big = taddr + static_cast<uint32_t>(b * kNAcc * BN + c_lo);
#pragma unroll
                for (int c0 = 0; c0 < kCols; c0 += 16) {
                    float vb[16], vs[16];
                    tmem_ld_16x2(t_big + c0, t_big + BN + c0, vb, vs);
                    if constexpr (kNAcc == 3) {
                        float v2[16];
                        tmem_ld_16(t_big + 2 * BN + c0, v2);
#pragma unroll
                        for (int j = 0; j < 16; ++j) acc[c0 + j] += vb[j] + (vs[j] + v2[j]);
                    } else {
#pragma unroll
                        for (int j = 0; j < 16; ++j) acc[c0 + j] += vb[j] + vs[j];
                    }
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&tempty_bar[b]);
            }
#pragma unroll
            for (int ch = 0; ch < kCols / 4; ++ch)
                st_shared_f4(row_s + static_cast<uint32_t>(((c_lo / 4 + ch) ^ sw) * 16), acc[4 * ch],
                             acc[4 * ch + 1], acc[4 * ch + 2], acc[4 * ch + 3]);
        }
        if (S > 1) fence_proxy_async_smem();  // the rows leave by bulk copy (async proxy)
    }
    __syncwarp();
    __syncthreads();  // staging tile complete
    // The next kernel in the stream may begin its own prologue (it waits before touching data).
    // Not earlier: an attention kernel's CTAs fit beside this one and would start streaming their
    // cached rows while the K loop still needs the memory system (measured slower).
    pdl_trigger();
    if (warp == 1) {  // accumulators drained: give the tensor memory back early
        tc_fence_after();
        tmem_dealloc(tmem_base, p.tmem_cols);
    }
    if (S > 1) {
        // Peers may write into this CTA's buffers once every thread of the cluster has arrived:
        // each thread arrived when its role was done with the pipeline buffers (the TMA loads
        // landed, the MMAs completed, the converters finished), after the receive barrier's
        // initialisation.
        cluster_wait_all();
        if (threadIdx.x == 0) {
            // rows [o*rows_per, (o+1)*rows_per) of this partial go to rank o, slot `rank`
            const uint32_t bytes = static_cast<uint32_t>(rows_per * BN * 4);
            for (int o = 0; o < S; ++o) {
                if (o == rank) continue;
                const uint32_t src = stage_s + static_cast<uint32_t>(o) * bytes;
                const uint32_t dst = dsmem_addr(recv_s + static_cast<uint32_t>(rank) * bytes, o);
                const uint32_t bar = dsmem_addr(smem_u32(recv_bar), o);
                bulk_copy_to_peer(dst, src, bytes, bar);
            }
            bulk_commit();
        }
        if constexpr ((EPI & kEpiResid) != 0) {
            // The epilogue's residual rows (written by earlier kernels: every thread is past the
            // CTA barrier that follows the epilogue warps' wait for them) are requested into L1
            // while the peers' partials travel.
            constexpr int kLines = (BN * 4 + 127) / 128;
            const int rl0 = rank * rows_per;
            const int rn = max(0, min(kBM, rl0 + rows_per) - rl0);
            for (int it = threadIdx.x; it < rn * kLines; it += kThreads) {
                const int row = m0 + rl0 + it / kLines;
                const int col = n0 + (it % kLines) * 32;
                if (row < p.M && col < p.N)
                    prefetch_l1(p.epi.resid + static_cast<size_t>(row) * p.epi.ldr + col);
            }
        }
        // Peers' rows of this rank are here. After an abort elsewhere still drain: no copy may
        // land in this CTA's memory after it exits.
        if (!mbar_wait(recv_bar, 0, p.err, kDevTimeoutAccum))
            mbar_wait_drain(recv_bar, 0, p.err, kDevTimeoutAccum);
    }

    // ---- sum the S slots in rank order and run the fused epilogue on this rank's rows ----
    const int r_lo = rank * rows_per;
    const int r_cnt = max(0, min(kBM, r_lo + rows_per) - r_lo);
    auto slot_addr = [&](int s, int r, int ch) -> uint32_t {
        const uint32_t phys = static_cast<uint32_t>((ch ^ (r & 7)) * 16);
        return (s == rank) ? stage_s + static_cast<uint32_t>((r_lo + r) * BN * 4) + phys
                           : recv_s + static_cast<uint32_t>((s * rows_per + r) * BN * 4) + phys;
    };
    if constexpr (!kArgmax) {
        // flattened (row, float4 column) items; consecutive threads write consecutive columns
        for (int it = threadIdx.x; it < r_cnt * kChunks; it += kThreads) {
            const int r = it / kChunks, ch = it - r * kChunks;
            const int row = m0 + r_lo + r;
            const int col = n0 + ch * 4;
            // a row's 32-column group is 8 consecutive items (threads): all skip or none do
            if (row >= p.M || col >= p.N) continue;
            float4 a4 = ld_shared_f4(slot_addr(0, r, ch));
            for (int s = 1; s < S; ++s) {
                const float4 t = ld_shared_f4(slot_addr(s, r, ch));
                a4.x += t.x;
                a4.y += t.y;
                a4.z += t.z;
                a4.w += t.w;
            }
            ArgState unused{0.f, 0, 0};
            float mean = 0.f, rstd = 0.f;
            if constexpr ((EPI & kEpiLnFold) != 0) {
                mean = ln_mean[r_lo + r];
                rstd = ln_rstd[r_lo + r];
            }
            const float4 v = epilogue4<EPI>(p, row, col, a4, unused, mean, rstd);
            if constexpr ((EPI & kEpiRowStats) != 0)
                row_group_stats(v, p.epi.row_stats + static_cast<size_t>(row) * (p.N >> 5) + (col >> 5),
                                lane);
        }
    } else {
        // one row per warp, so the row's first maximum over this tile is a warp reduction
        for (int r = warp; r < r_cnt; r += kWarps) {
            const int row = m0 + r_lo + r;
            if (row >= p.M) break;
            ArgState as{-INFINITY, kArgNone, 0};
            float mean = 0.f, rstd = 0.f;
            if constexpr ((EPI & kEpiLnFold) != 0) {
                mean = ln_mean[r_lo + r];
                rstd = ln_rstd[r_lo + r];
            }
            for (int ch = lane; ch < kChunks; ch += 32) {
                const int col = n0 + ch * 4;
                if (col >= p.N) break;
                float4 a4 = ld_shared_f4(slot_addr(0, r, ch));
                for (int s = 1; s < S; ++s) {
                    const float4 t = ld_shared_f4(slot_addr(s, r, ch));
                    a4.x += t.x;
                    a4.y += t.y;
                    a4.z += t.z;
                    a4.w += t.w;
                }
                epilogue4<EPI>(p, row, col, a4, as, mean, rstd);
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                const float ov = __shfl_xor_sync(0xffffffffu, as.best, o);
                const int oi = __shfl_xor_sync(0xffffffffu, as.idx, o);
                const int onf = __shfl_xor_sync(0xffffffffu, as.nf, o);
                if (ov > as.best || (ov == as.best && oi < as.idx)) {
                    as.best = ov;
                    as.idx = oi;
                }
                as.nf |= onf;
            }
            if (lane == 0) {
                if (as.idx != kArgNone) atomicMax(p.arg_key + row, arg_key_of(as.best, as.idx));
                if (as.nf) atomicOr(p.arg_nf + row, 1);
            }
        }
        // The last CTA of this row block to finish (n_tiles x S arrive) reads every row's key,
        // which by then holds the first maximum over the whole row, and hands the keys and
        // flags back at zero for the next launch.
        __threadfence();
        __syncthreads();
        if (threadIdx.x == 0) {
            const int t = atomicAdd(p.tickets + mt, 1);
            *last_flag = (t == p.n_tiles * S - 1) ? 1 : 0;
        }
        __syncthreads();
        if (*last_flag) {
            __threadfence();
            for (int rl = threadIdx.x; rl < kBM; rl += kThreads) {
                const int row = m0 + rl;
                if (row >= p.M) break;
                const unsigned long long key = atomicExch(p.arg_key + row, 0ull);
                const int nf = atomicExch(p.arg_nf + row, 0);
                p.epi.next_ids[row] = key ? arg_col_of(key) : -1;
                if (p.epi.nonfinite) p.epi.nonfinite[row] = (nf || key == 0ull) ? 1 : 0;
            }
            if (threadIdx.x == 0) p.tickets[mt] = 0;
        }
    }
    // Outgoing bulk copies must have read the staging tile before this CTA's memory is released.
    if (S > 1 && threadIdx.x == 0) bulk_wait_reads();
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

// Tensor map of a row-major fp32 matrix [rows, cols] with row stride ld (floats), box 32 x box_rows,
// 128-byte swizzle; reads past cols or rows fill with zero.
bool make_map_ld(CUtensorMap* map, const float* base, int cols, int ld, int rows, int box_rows) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return false;
    if ((reinterpret_cast<uintptr_t>(base) & 15) != 0 || (ld & 3) != 0 || cols > ld) return false;
    cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
    cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld) * 4};
    cuuint32_t box[2] = {static_cast<cuuint32_t>(kBK), static_cast<cuuint32_t>(box_rows)};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(base), dims, strides,
                    box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

bool make_map(CUtensorMap* map, const float* base, int K, int rows, int box_rows) {
    return make_map_ld(map, base, K, K, rows, box_rows);
}

size_t stage_bytes_for(int bn) {
    return 2 * static_cast<size_t>(kATileBytes) + 2 * static_cast<size_t>(bn) * kBK * 4;
}

int rows_per_for(int s) { return (kBM + s - 1) / s; }

// Receive buffer for the peers' partials (none without a cluster: the staging tile reuses the
// pipeline buffers).
size_t recv_bytes_for(int bn, int s) {
    return s > 1 ? static_cast<size_t>(s) * rows_per_for(s) * bn * 4 : 0;
}

// Two TMEM buffers (one when two do not fit), each with one accumulator of BN columns per MMA
// issuer.
int tbufs_for(int bn) { return (2 * nacc_for(bn) * bn <= 512) ? 2 : 1; }
uint32_t tmem_cols_for(int bn) {
    uint32_t cols = 32;
    while (cols < static_cast<uint32_t>(tbufs_for(bn) * nacc_for(bn) * bn)) cols <<= 1;
    return cols;
}

typedef void (*GemmKernelFn)(GemmKParams);

template <int BN>
GemmKernelFn kernel_for_epi(int flags) {
    switch (flags) {
        case kEpiSetStore: return gemm_3xtf32_kernel<BN, kEpiSetStore>;
        case kEpiSetResid: return gemm_3xtf32_kernel<BN, kEpiSetResid>;
        case kEpiSetFfnUp: return gemm_3xtf32_kernel<BN, kEpiSetFfnUp>;
        case kEpiSetFfnDown: return gemm_3xtf32_kernel<BN, kEpiSetFfnDown>;
        case kEpiSetHead: return gemm_3xtf32_kernel<BN, kEpiSetHead>;
        case kEpiSetHeadLogits: return gemm_3xtf32_kernel<BN, kEpiSetHeadLogits>;
        case kEpiSetScatter: return gemm_3xtf32_kernel<BN, kEpiSetScatter>;
        case kEpiSetStoreLn: return gemm_3xtf32_kernel<BN, kEpiSetStoreLn>;
        case kEpiSetResidStats: return gemm_3xtf32_kernel<BN, kEpiSetResidStats>;
        case kEpiSetFfnUpLn: return gemm_3xtf32_kernel<BN, kEpiSetFfnUpLn>;
        case kEpiSetFfnDownStats: return gemm_3xtf32_kernel<BN, kEpiSetFfnDownStats>;
        case kEpiSetHeadLn: return gemm_3xtf32_kernel<BN, kEpiSetHeadLn>;
        case kEpiSetHeadLogitsLn: return gemm_3xtf32_kernel<BN, kEpiSetHeadLogitsLn>;
        case kEpiSetStoreAF: return gemm_3xtf32_kernel<BN, kEpiSetStoreAF>;
        default: return nullptr;
    }
}

constexpr int kTileWidths[] = {32, 64, 128};  // the time model's candidates
// 224-column tiles exist for the LM head only (143 tiles of a 32000-word vocabulary: one wave).
constexpr int kWideTile = 224;

GemmKernelFn kernel_for(int bn, int flags) {
    switch (bn) {
        case 32: return kernel_for_epi<32>(flags);
        case 64: return kernel_for_epi<64>(flags);
        case 128: return kernel_for_epi<128>(flags);
        case kWideTile:
            switch (flags) {
                case kEpiSetHead: return gemm_3xtf32_kernel<kWideTile, kEpiSetHead>;
                case kEpiSetHeadLogits: return gemm_3xtf32_kernel<kWideTile, kEpiSetHeadLogits>;
                case kEpiSetHeadLn: return gemm_3xtf32_kernel<kWideTile, kEpiSetHeadLn>;
                case kEpiSetHeadLogitsLn: return gemm_3xtf32_kernel<kWideTile, kEpiSetHeadLogitsLn>;
                default: return nullptr;
            }
        default: return nullptr;
    }
}

// Sets the shared-memory attribute of every instantiation once per device.
cudaError_t prepare_device_attrs() {
    static std::mutex mu;
    static unsigned long long done_mask = 0;
    int dev = 0;
    cudaGetDevice(&dev);
    std::lock_guard<std::mutex> lock(mu);
    if (dev >= 64 || (done_mask & (1ull << dev))) return cudaSuccess;
    const int sets[] = {kEpiSetStore,       kEpiSetResid,   kEpiSetFfnUp,        kEpiSetFfnDown,
                        kEpiSetHead,        kEpiSetHeadLogits, kEpiSetScatter,   kEpiSetStoreLn,
                        kEpiSetResidStats,  kEpiSetFfnUpLn, kEpiSetFfnDownStats, kEpiSetHeadLn,
                        kEpiSetHeadLogitsLn, kEpiSetStoreAF};
    for (int bn : {32, 64, 128, kWideTile})
        for (int f : sets) {
            GemmKernelFn k = kernel_for(bn, f);
            if (k == nullptr) continue;
            cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 static_cast<int>(kSmemLimit));
            if (e == cudaSuccess)
                e = cudaFuncSetAttribute(k, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
            if (e != cudaSuccess) return e;
        }
    done_mask |= (1ull << dev);
    return cudaSuccess;
}

// How many clusters of `s` CTAs with `smem` bytes each the current device can hold at once.
int max_active_clusters(int bn, int s, size_t smem) {
    static std::mutex mu;
    static std::map<std::tuple<int, int, int, size_t>, int> cache;
    int dev = 0;
    cudaGetDevice(&dev);
    const auto key = std::make_tuple(dev, bn, s, smem);
    std::lock_guard<std::mutex> lock(mu);
    auto it = cache.find(key);
    if (it != cache.end()) return it->second;
    int n = 0;
    if (prepare_device_attrs() == cudaSuccess) {
        cudaLaunchConfig_t cfg{};
        cfg.gridDim = dim3(1, 1, s);
        cfg.blockDim = dim3(threads_for(bn));
        cfg.dynamicSmemBytes = smem;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = 1;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = s;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        if (cudaOccupancyMaxActiveClusters(&n, kernel_for(bn, kEpiSetStore), &cfg) != cudaSuccess) n = 0;
        cudaGetLastError();
    }
    cache[key] = n;
    return n;
}

// The pipeline buffers, reused after the mainloop for the partial tile and the peers' partials.
size_t smem_for(int bn, int s, int stages) {
    const size_t after = static_cast<size_t>(kBM) * bn * 4 + recv_bytes_for(bn, s);
    return std::max(stages * stage_bytes_for(bn), after) + kSmemReserve;
}

}  // namespace

bool tensor_map_api_available() { return encode_fn() != nullptr; }

int gemm_cluster_capacity(int bn, int splits, int stages) {
    return max_active_clusters(bn, splits, smem_for(bn, splits, stages));
}

// Picks the N tile and the cluster split of K from a time model fitted to measurements on B200
// (ns): each CTA pays a fixed ~2.5 us (launch, prologue, first load, epilogue) plus its bytes —
// the weight tile (HBM) and the activation tile (L2, re-read once per N tile) — at the rate one
// SM ingests (~70 GB/s when all SMs pull), or its MMAs if slower; clusters that do not fit on
// the device at once run in waves.
//
// Decode projections (one 128-row tile) of the supported model widths use plans measured on B200
// instead: candidate (N tile, cluster split, stages, promotion chunk) sets were timed for each
// shape, alone and inside the captured decode step (where the overlap of consecutive launches
// decides: plans that fill every SM leave the next launch no room to start early), and the
// fastest kept. The model mispredicts these latency-bound launches by up to 1.5x (K = 4096:
// split 8 with 128-wide tiles runs in 18.9 us against 28.7 us for its pick).
struct MeasuredPlan {
    int n, k, bn, splits, stages, chunk_kb;
};
constexpr MeasuredPlan kMeasuredPlans[] = {
    // d_model 1024, d_ff 4096, vocab 32000
    {3072, 1024, 128, 4, 3, 8},
    {1024, 1024, 32, 4, 4, 8},
    {4096, 1024, 128, 4, 3, 8},
    {1024, 4096, 128, 8, 3, 8},
    {32000, 1024, kWideTile, 1, 2, 32},  // LM head: 143 tiles, one wave, one TMEM chunk
    {32000, 1024, 128, 1, 3, 8},
    // d_model 512, d_ff 2048, vocab 16000
    {1536, 512, 64, 4, 2, 4},
    {2048, 512, 64, 4, 2, 4},
    {16000, 512, 128, 1, 3, 8},
    // d_model 128, d_ff 512
    {384, 128, 32, 2, 2, 2},
    {128, 128, 32, 2, 2, 2},
    {512, 128, 32, 2, 2, 2},
    {128, 512, 32, 8, 2, 2},
};

// Keep (CTAs resident per SM) x (TMEM columns per CTA) <= 512: the smallest shared-memory request
// that lets no more CTAs fit on an SM than its tensor memory can hold at once.
size_t tmem_bound_smem(int bn) {
    const size_t max_ctas = 512 / tmem_cols_for(bn);
    return 228 * 1024 / (max_ctas + 1) + 1;  // max_ctas + 1 CTAs must not fit
}

// Fills kb_per_split, tile counts and the shared-memory request of a plan whose bn, splits and
// stages are set; false if it does not fit or its clusters cannot be placed.
bool complete_plan(GemmPlan& p, int M, int N, int K) {
    const int total_kb = (K + kBK - 1) / kBK;
    if (p.splits < 1 || p.splits > std::min(kMaxCluster, total_kb) || kBM % p.splits) return false;
    p.kb_per_split = (total_kb + p.splits - 1) / p.splits;
    if ((total_kb + p.kb_per_split - 1) / p.kb_per_split != p.splits) return false;
    p.m_tiles = (M + kBM - 1) / kBM;
    p.n_tiles = (N + p.bn - 1) / p.bn;
    p.stages = std::max(1, std::min(p.stages, p.kb_per_split));
    p.chunk_kb = std::max(1, std::min(p.chunk_kb, p.kb_per_split));
    if (tbufs_for(p.bn) == 1) p.chunk_kb = p.kb_per_split;  // one TMEM buffer: one chunk
    p.smem_bytes = std::max(smem_for(p.bn, p.splits, p.stages), tmem_bound_smem(p.bn));
    if (p.smem_bytes > kSmemLimit) return false;
    if (p.splits > 1 && max_active_clusters(p.bn, p.splits, p.smem_bytes) <= 0) return false;
    return true;
}

GemmPlan gemm_plan(int M, int N, int K, int flags, int num_sms) {
    GemmPlan best;
    double best_t = 1e300;
    const int m_tiles = (M + kBM - 1) / kBM;
    const int total_kb = (K + kBK - 1) / kBK;
    bool measured = false;
    // ADAI_B200_GEMM_PLANS="N:K:bn:splits:stages:chunk,..." replaces the plan of every (N, K) it
    // names, whatever M (plan tuning; the measured table below holds one-row-tile plans only).
    {
        if (const char* env = std::getenv("ADAI_B200_GEMM_PLANS")) {
            const char* q = env;
            while (*q && !measured) {
                MeasuredPlan mp{};
                int used = 0;
                if (std::sscanf(q, "%d:%d:%d:%d:%d:%d%n", &mp.n, &mp.k, &mp.bn, &mp.splits,
                                &mp.stages, &mp.chunk_kb, &used) != 6)
                    break;
                q += used;
                if (*q == ',') ++q;
                if (mp.n != N || mp.k != K || kernel_for(mp.bn, flags) == nullptr) continue;
                GemmPlan p;
                p.bn = mp.bn;
                p.splits = mp.splits;
                p.stages = mp.stages;
                p.chunk_kb = mp.chunk_kb;
                if (complete_plan(p, M, N, K)) {
                    best = p;
                    measured = true;
                }
            }
        }
    }
    if (m_tiles == 1 && !measured) {
        for (const MeasuredPlan& mp : kMeasuredPlans) {
            if (mp.n != N || mp.k != K || kernel_for(mp.bn, flags) == nullptr) continue;
            GemmPlan p;
            p.bn = mp.bn;
            p.splits = mp.splits;
            p.stages = mp.stages;
            p.chunk_kb = mp.chunk_kb;
            if (complete_plan(p, M, N, K)) {
                best = p;
                measured = true;
            }
            break;
        }
    }
    const int n16 = (N + 15) / 16 * 16;
    for (int bn : kTileWidths) {
        if (measured) break;
        if (bn > n16 && bn != kTileWidths[0]) {
            bool narrower_covers = false;
            for (int b2 : kTileWidths)
                if (b2 < bn && b2 >= n16) narrower_covers = true;
            if (narrower_covers) continue;
        }
        const int n_tiles = (N + bn - 1) / bn;
        const int tiles = m_tiles * n_tiles;
        for (int s = 1; s <= std::min(kMaxCluster, total_kb); ++s) {
            const int kbc = (total_kb + s - 1) / s;
            if ((total_kb + kbc - 1) / kbc != s) continue;
            if (s > 1 && (kBM % s) != 0) continue;  // whole rows per rank
            const size_t sb = stage_bytes_for(bn);
            if (smem_for(bn, s, 1) > kSmemLimit) continue;
            int stages = static_cast<int>((kSmemLimit - kSmemReserve) / sb);
            stages = std::max(1, std::min({stages, 8, kbc}));
            const size_t smem = smem_for(bn, s, stages);
            const long long ctas = static_cast<long long>(tiles) * s;
            long long waves;
            if (s > 1) {
                const int cap = max_active_clusters(bn, s, smem);
                if (cap <= 0) continue;
                waves = (static_cast<long long>(tiles) + cap - 1) / cap;
            } else {
                waves = (ctas + num_sms - 1) / num_sms;
            }
            const long long active = std::min<long long>(ctas, num_sms);
            // One SM keeps ~`stages` boxes in flight against ~1.7 us of load latency; all SMs
            // together are capped near 9.5 TB/s (L2 + HBM) and the weights alone by HBM.
            const double ingest = std::min({static_cast<double>(stages) * sb / 1700.0, 150.0,
                                            9500.0 / static_cast<double>(active)});  // B/ns
            const double bytes_kb = static_cast<double>(sb);                       // A + W tiles
            const double mma_ns = 24576.0 * bn / 7400.0;
            const double per_kb = std::max(bytes_kb / ingest, mma_ns);
            const double hbm_floor = static_cast<double>(N) * K * 8.0 / 6500.0;    // W hi + lo
            const double t = std::max(static_cast<double>(waves) * (2500.0 + kbc * per_kb + 60.0 * s),
                                      hbm_floor + 2500.0);
            if (t < best_t - 1e-9) {
                best_t = t;
                best.bn = bn;
                best.splits = s;
                best.kb_per_split = kbc;
                best.m_tiles = m_tiles;
                best.n_tiles = n_tiles;
                best.stages = stages;
                best.smem_bytes = smem;
            }
        }
    }
    // Promotion chunk: the accumulators move to fp32 registers after every 4 K blocks (128 k, 16
    // MMA steps; 8 blocks in some measured plans). The tensor core's accumulation into TMEM does
    // not round to nearest, so its error grows with the steps between promotions; 16-32 steps
    // keep it at the size of the fp32 in-order CPU product's own rounding, while each promotion
    // costs a TMEM round trip that stalls the MMA issue (one-block chunks measured up to ~25%
    // slower per K block).
    if (!measured) best.chunk_kb = std::min(best.kb_per_split, 4);
    best.smem_bytes = std::max(best.smem_bytes, tmem_bound_smem(best.bn));
    return best;
}

size_t gemm_ws_floats(const GemmPlan&) { return 0; }

size_t gemm_arg_rows(const GemmPlan& p) { return static_cast<size_t>(p.m_tiles) * kBM; }

int gemm_launch(const TcActs& a, int M, const TcWeight& w, const GemmEpilogue& epi,
                const GemmPlan& plan, const GemmScratch& scratch, int* err, cudaStream_t st) {
    const cudaError_t ae = prepare_device_attrs();
    if (ae != cudaSuccess) return static_cast<int>(ae);
    if (M <= 0 || w.N <= 0 || w.K <= 0 || a.K != w.K) return cudaErrorInvalidValue;
    if (a.rows_alloc < plan.m_tiles * kBM) return cudaErrorInvalidValue;
    GemmKernelFn kern = kernel_for(plan.bn, epi.flags);
    if (kern == nullptr || plan.chunk_kb < 1 || plan.stages < 1) return cudaErrorInvalidValue;
    if (plan.splits < 1 || plan.splits > kMaxCluster || (plan.splits > 1 && kBM % plan.splits))
        return cudaErrorInvalidValue;
    if (tbufs_for(plan.bn) == 1 && plan.chunk_kb < plan.kb_per_split) return cudaErrorInvalidValue;
    if (plan.smem_bytes > kSmemLimit ||
        plan.smem_bytes < smem_for(plan.bn, plan.splits, plan.stages))
        return cudaErrorInvalidValue;
    if ((epi.flags & kEpiArgmax) &&
        (scratch.arg_key == nullptr || scratch.arg_nf == nullptr ||
         scratch.arg_rows < gemm_arg_rows(plan) ||
         scratch.n_tickets < plan.m_tiles || epi.next_ids == nullptr))
        return cudaErrorInvalidValue;
    if ((epi.flags & kEpiKvScatter) &&
        (epi.head_dim % 4 != 0 || epi.d_model % epi.head_dim != 0 || w.N != 2 * epi.d_model))
        return cudaErrorInvalidValue;
    if ((epi.flags & kEpiRowStats) &&
        (epi.row_stats == nullptr || epi.stats_ld < M || w.N % 64 != 0))
        return cudaErrorInvalidValue;
    if ((epi.flags & kEpiLnFold) &&
        (epi.row_stats == nullptr || epi.ln_c1 == nullptr || epi.stats_ld < M || w.K % 64 != 0 ||
         (reinterpret_cast<uintptr_t>(epi.row_stats) & 15) != 0 ||
         (reinterpret_cast<uintptr_t>(epi.ln_c1) & 15) != 0))
        return cudaErrorInvalidValue;
    // fp32 A: a third A plane per stage (the raw box) and a third barrier per stage; as many
    // stages as then fit
    const bool af = (epi.flags & kEpiAFp32) != 0;
    GemmPlan pl = plan;
    if (af) {
        if (a.fp32 == nullptr || a.k_valid <= 0 || a.k_valid > w.K || a.rows < M)
            return cudaErrorInvalidValue;
        auto smem_af = [&](int st) {
            return std::max(static_cast<size_t>(st) * (stage_bytes_for(pl.bn) + kATileBytes),
                            smem_for(pl.bn, pl.splits, 1) - kSmemReserve) + kSmemReserve;
        };
        while (pl.stages > 1 && (smem_af(pl.stages) > kSmemLimit || 3 * pl.stages + 8 > 31)) --pl.stages;
        pl.smem_bytes = std::max(pl.smem_bytes, smem_af(pl.stages));
        if (pl.smem_bytes > kSmemLimit) return cudaErrorInvalidValue;
    }
    // barriers (2 per stage + 8, or 3 per stage + 8), the TMEM slot and the ticket flag share 256
    // bytes
    if (((af ? 3 : 2) * pl.stages + 8) * 8 + 8 > 256) return cudaErrorInvalidValue;
    const int n_rows_alloc = (w.N + 255) / 256 * 256;

    GemmKParams p{};
    const bool amaps = af ? make_map_ld(&p.a_hi, a.fp32, a.k_valid, a.lda, a.rows, kBM)
                          : (make_map(&p.a_hi, a.hi, a.K, a.rows_alloc, kBM) &&
                             make_map(&p.a_lo, a.lo, a.K, a.rows_alloc, kBM));
    if (!amaps ||
        !make_map(&p.b_hi, w.hi, w.K, n_rows_alloc, plan.bn) ||
        !make_map(&p.b_lo, w.lo, w.K, n_rows_alloc, plan.bn))
        return cudaErrorInvalidValue;
    p.M = M;
    p.N = w.N;
    p.K = w.K;
    p.stages = pl.stages;
    p.pair_commit = (pl.stages % 2 == 0 && pl.stages >= 4) ? 1 : 0;
    p.kb_per_split = plan.kb_per_split;
    p.splits = plan.splits;
    p.rows_per = rows_per_for(plan.splits);
    p.n_tiles = plan.n_tiles;
    p.m_tiles = plan.m_tiles;
    p.total_kb = (w.K + kBK - 1) / kBK;
    p.chunk_kb = plan.chunk_kb;
    p.idesc = idesc_tf32(kBM, plan.bn);
    p.tmem_cols = tmem_cols_for(plan.bn);
    p.epi = epi;
    p.tickets = scratch.tickets;
    p.arg_key = scratch.arg_key;
    p.arg_nf = scratch.arg_nf;
    p.err = err;

    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(plan.n_tiles, plan.m_tiles, plan.splits);
    cfg.blockDim = dim3(threads_for(plan.bn, epi.flags));
    cfg.dynamicSmemBytes = pl.smem_bytes;
    cfg.stream = st;
    cudaLaunchAttribute attr[2];
    int na = 0;
    if (plan.splits > 1) {
        attr[na].id = cudaLaunchAttributeClusterDimension;
        attr[na].val.clusterDim.x = 1;
        attr[na].val.clusterDim.y = 1;
        attr[na].val.clusterDim.z = plan.splits;
        ++na;
    }
    if (launch_pdl_enabled()) {
        attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[na].val.programmaticStreamSerializationAllowed = 1;
        ++na;
    }
    cfg.attrs = attr;
    cfg.numAttrs = na;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, p);
    if (e != cudaSuccess) return static_cast<int>(e);
    return static_cast<int>(cudaGetLastError());
}

}  // namespace adai_b200
