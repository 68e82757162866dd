// prefill_tc.cu — encoder self-attention (LLMEncoder prefill, src/EncoderBlock.cpp:34-77, all-ones
// mask) on the 5th-generation tensor cores, 3xTF32, flash-style: per (128-query block, head,
// sequence) one CTA streams its sequence's keys in blocks of 64, S = Q K^T and O += P V both as
// tcgen05.mma into tensor memory, the online softmax in registers in between.
//
// Operands come split (x = hi + lo, tf32 each) and K-major, in the canonical 128-byte swizzled
// layout TMA writes: Q and K straight from the split Q|K|V rows, V from a per-head transposed copy
// (V^T [head * DH + d][column]) whose sequences start at 32-column boundaries, so that every box
// starts on a 16-byte boundary. P is written by the softmax warps in the same swizzled layout.
//
// Warp roles (320 threads): warp 0 issues the TMA loads, warp 1 the MMAs, warps 2-9 run the
// softmax and the output, two warps per TMEM lane quarter (32 query rows): each reads the whole S
// block of its rows and takes the row maximum (both halves get the same value), then half h
// exponentiates key columns [32h, 32h + 32), writes that 32-column atom of P and folds output
// dimensions [h DH/2, (h+1) DH/2). The two halves' row sums are added once at the end. Every wait
// is bounded.
#include <mutex>

#include "common.cuh"
#include "kernels.h"

namespace adai_b200 {
namespace {

constexpr int kPBM = 128;       // queries per CTA
constexpr int kPBN = 64;        // keys per block
constexpr int kPThreads = 320;
constexpr uint32_t kAtomRows128 = 128 * 128;  // bytes of a [128 rows x 32 floats] swizzled atom

struct __align__(64) PrefillParams {
    CUtensorMap q_hi, q_lo, k_hi, k_lo, v_hi, v_lo;
    const int* offsets;  // first row of each sequence
    const int* lens;     // rows of each sequence
    const int* vcol;     // first V^T column of each sequence (multiple of 32)
    float* out_hi;       // [rows, D] split output
    float* out_lo;
    int D;
    float scale;
    int* err;
};

template <int DH>
struct PrefillLayout {
    static constexpr int kAtomsD = DH / 32;                       // 32-float atoms along head dims
    static constexpr uint32_t kQ = 2u * kAtomsD * 128 * 128;      // Q hi, lo
    static constexpr uint32_t kK = 2u * kAtomsD * kPBN * 128;     // K hi, lo
    static constexpr uint32_t kVStage = 2u * (kPBN / 32) * DH * 128;  // V^T hi, lo of one block
    static constexpr uint32_t kV = 2u * kVStage;                   // two blocks in flight
    static constexpr uint32_t kP = 2u * (kPBN / 32) * 128 * 128;  // P hi, lo
    static constexpr uint32_t kBytes = kQ + kK + kV + kP + 1024 /* barriers */ + 1024 /* align */;
    // TMEM: two S buffers (hi*hi and correction, kPBN columns each) and one O (DH each).
    static constexpr uint32_t kTmemCols = 512;
};

template <int DH>
__global__ void __launch_bounds__(kPThreads, 1) prefill_attention_tc_kernel(const __grid_constant__ PrefillParams p) {
    using L = PrefillLayout<DH>;
    extern __shared__ uint8_t praw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(praw) + 1023) & ~uintptr_t(1023));
    const int qb = blockIdx.x, h = blockIdx.y, s = blockIdx.z;
    const int S = p.lens[s];
    if (qb * kPBM >= S) return;
    const int row0 = p.offsets[s];
    const int nkb = (S + kPBN - 1) / kPBN;

    uint8_t* q_s = smem;                  // [hi|lo][atom][128 rows x 128 B]
    uint8_t* k_s = q_s + L::kQ;           // [hi|lo][atom][64 rows x 128 B]
    uint8_t* v_s = k_s + L::kK;           // [hi|lo][key atom][DH rows x 128 B]
    uint8_t* p_s = v_s + L::kV;           // [hi|lo][key atom][128 rows x 128 B]
    uint64_t* bars = reinterpret_cast<uint64_t*>(p_s + L::kP);
    uint64_t* q_full = bars + 0;
    uint64_t* k_full = bars + 1;
    uint64_t* k_empty = bars + 2;
    uint64_t* v_full = bars + 3;   // [2] V^T stage
    uint64_t* v_empty = bars + 5;  // [2]
    uint64_t* s_full = bars + 7;   // [2] S buffer
    uint64_t* s_empty = bars + 9;  // [2]
    uint64_t* p_full = bars + 11;
    uint64_t* o_full = bars + 12;
    uint64_t* o_empty = bars + 13;
    uint64_t* done = bars + 14;
    uint64_t* pair_end = bars + 15;  // [4] both halves of a lane quarter have left their row sums
    constexpr int kBars = 19;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + kBars);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        tma_prefetch_desc(&p.q_hi);
        tma_prefetch_desc(&p.k_hi);
        tma_prefetch_desc(&p.v_hi);
        // arrivals per phase: the producer (expect_tx) or one tcgen05.commit, except the barriers
        // the eight softmax warps arrive on (one arrival per warp) and the quarters' end-of-row
        // exchanges (one per thread of the two warps)
        for (int i = 0; i < kBars; ++i) {
            const bool softmax = (bars + i == s_empty || bars + i == s_empty + 1 || bars + i == p_full ||
                                  bars + i == o_empty);
            const bool pair = bars + i >= pair_end;
            mbar_init(&bars[i], pair ? 64 : (softmax ? 8 : 1));
        }
        fence_barrier_init();
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, L::kTmemCols);
        tmem_relinquish();
    }
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    // TMEM columns: S buffer b at b * 2 * kPBN (hi*hi) and + kPBN (correction); O at 4 * kPBN.
    const uint32_t t_o = tmem + 4 * kPBN;

    if (warp == 0) {
        // lane 0 streams Q and the K blocks, lane 1 the V^T blocks (two stages), each on its own
        // barriers, so that a block's K is requested as soon as S of the previous block is done
        // and its V while the previous P V is still running.
        if (lane == 0) {
            mbar_arrive_expect_tx(q_full, L::kQ);
            for (int a = 0; a < L::kAtomsD; ++a) {
                tma_load_2d(q_s + a * kAtomRows128, &p.q_hi, q_full, h * DH + 32 * a, row0 + qb * kPBM);
                tma_load_2d(q_s + (L::kAtomsD + a) * kAtomRows128, &p.q_lo, q_full, h * DH + 32 * a, row0 + qb * kPBM);
            }
            int issued = 0;
            for (int j = 0; j < nkb; ++j) {
                if (j > 0 && !mbar_wait(k_empty, (j - 1) & 1, p.err, kDevTimeoutSmemEmpty)) break;
                mbar_arrive_expect_tx(k_full, L::kK);
                for (int a = 0; a < L::kAtomsD; ++a) {
                    tma_load_2d(k_s + a * (kPBN * 128), &p.k_hi, k_full, p.D + h * DH + 32 * a, row0 + j * kPBN);
                    tma_load_2d(k_s + (L::kAtomsD + a) * (kPBN * 128), &p.k_lo, k_full, p.D + h * DH + 32 * a, row0 + j * kPBN);
                }
                ++issued;
            }
            // Nothing may land in shared memory after the CTA moves on.
            mbar_wait_drain(q_full, 0, p.err, kDevTimeoutTmaFull);
            if (issued) mbar_wait_drain(k_full, (issued - 1) & 1, p.err, kDevTimeoutTmaFull);
        } else if (lane == 1) {
            int issued = 0;
            for (int j = 0; j < nkb; ++j) {
                const int st = j & 1;
                if (j >= 2 && !mbar_wait(v_empty + st, ((j >> 1) - 1) & 1, p.err, kDevTimeoutSmemEmpty)) break;
                mbar_arrive_expect_tx(v_full + st, L::kVStage);
                uint8_t* vb = v_s + st * L::kVStage;
                for (int a = 0; a < kPBN / 32; ++a) {
                    const int x = p.vcol[s] + j * kPBN + 32 * a;
                    tma_load_2d(vb + a * (DH * 128), &p.v_hi, v_full + st, x, h * DH);
                    tma_load_2d(vb + (kPBN / 32 + a) * (DH * 128), &p.v_lo, v_full + st, x, h * DH);
                }
                ++issued;
            }
            for (int j = (issued > 2 ? issued - 2 : 0); j < issued; ++j)
                mbar_wait_drain(v_full + (j & 1), static_cast<uint32_t>(j >> 1) & 1u, p.err, kDevTimeoutTmaFull);
        }
    } else if (warp == 1) {
        if (lane == 0) {
            constexpr uint32_t idesc_s = idesc_tf32(128, kPBN);
            constexpr uint32_t idesc_o = idesc_tf32(128, DH);
            const uint32_t qs = smem_u32(q_s), ks = smem_u32(k_s), vs = smem_u32(v_s), ps = smem_u32(p_s);
            bool ok = mbar_wait(q_full, 0, p.err, kDevTimeoutTmaFull);
            // S_j = Q K_j^T into S buffer j % 2
            auto issue_s = [&](int j) -> bool {
                const int b = j & 1;
                if (j >= 2 && !mbar_wait(s_empty + b, ((j >> 1) - 1) & 1, p.err, kDevTimeoutAccum)) return false;
                if (!mbar_wait(k_full, j & 1, p.err, kDevTimeoutTmaFull)) return false;
                tc_fence_after();
                const uint32_t t_big = tmem + b * 2 * kPBN, t_small = t_big + kPBN;
#pragma unroll
                for (int kk = 0; kk < DH / 8; ++kk) {
                    const int a = kk / 4;
                    const uint32_t off = (kk % 4) * 32;
                    const uint32_t qh = qs + a * kAtomRows128 + off, ql = qs + (L::kAtomsD + a) * kAtomRows128 + off;
                    const uint32_t kh = ks + a * (kPBN * 128) + off, kl = ks + (L::kAtomsD + a) * (kPBN * 128) + off;
                    const uint32_t acc = kk ? 1u : 0u;
                    mma_tf32(t_small, smem_desc_k_sw128(ql), smem_desc_k_sw128(kh), idesc_s, acc);
                    mma_tf32(t_small, smem_desc_k_sw128(qh), smem_desc_k_sw128(kl), idesc_s, 1u);
                    mma_tf32(t_big, smem_desc_k_sw128(qh), smem_desc_k_sw128(kh), idesc_s, acc);
                }
                mma_commit(s_full + b);
                mma_commit(k_empty);
                return true;
            };
            if (ok) ok = issue_s(0);
            for (int j = 0; j < nkb && ok; ++j) {
                if (j + 1 < nkb && !issue_s(j + 1)) {
                    ok = false;
                    break;
                }
                // O_j = P_j V_j once the softmax has written P_j and consumed O_{j-1}
                if (!mbar_wait(p_full, j & 1, p.err, kDevTimeoutAccum) ||
                    !mbar_wait(v_full + (j & 1), (j >> 1) & 1, p.err, kDevTimeoutTmaFull) ||
                    (j > 0 && !mbar_wait(o_empty, (j - 1) & 1, p.err, kDevTimeoutAccum))) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t t_big = t_o, t_small = t_o + DH;
                const uint32_t vst = vs + (j & 1) * L::kVStage;
#pragma unroll
                for (int kk = 0; kk < kPBN / 8; ++kk) {
                    const int a = kk / 4;
                    const uint32_t off = (kk % 4) * 32;
                    const uint32_t ph = ps + a * kAtomRows128 + off, pl = ps + (kPBN / 32 + a) * kAtomRows128 + off;
                    const uint32_t vh = vst + a * (DH * 128) + off, vl = vst + (kPBN / 32 + a) * (DH * 128) + off;
                    const uint32_t acc = kk ? 1u : 0u;
                    mma_tf32(t_small, smem_desc_k_sw128(pl), smem_desc_k_sw128(vh), idesc_o, acc);
                    mma_tf32(t_small, smem_desc_k_sw128(ph), smem_desc_k_sw128(vl), idesc_o, 1u);
                    mma_tf32(t_big, smem_desc_k_sw128(ph), smem_desc_k_sw128(vh), idesc_o, acc);
                }
                mma_commit(o_full);
                mma_commit(v_empty + (j & 1));
            }
            mma_commit(done);
            mbar_wait_drain(done, 0, p.err, kDevTimeoutAccum);
        }
    } else {
        // ---- warps 2..9: one query row per thread, two warps (halves) per row ----
        const int qq = warp & 3;
        const int hf = (warp - 2) >> 2;
        constexpr int HD = DH / 2;     // output dimensions of this half
        constexpr int HC = kPBN / 2;   // key columns of this half (one 32-float P atom)
        const int row = qq * 32 + lane;  // row within the query block = TMEM lane
        const uint32_t lane_off = static_cast<uint32_t>(qq * 32) << 16;
        float o[HD];
#pragma unroll
        for (int d = 0; d < HD; ++d) o[d] = 0.f;
        float m = -INFINITY, l = 0.f, corr_prev = 0.f;
        bool ok = true;
        const uint32_t ps = smem_u32(p_s);
        // P row `row` inside a [128 x 32 floats] swizzled atom: 16-byte chunk c sits at (c ^ (row & 7)).
        const uint32_t p_row = static_cast<uint32_t>(row) * 128;
        const int sw = row & 7;
        for (int j = 0; j < nkb && ok; ++j) {
            const int b = j & 1;
            int got = 1;
            if (lane == 0) got = mbar_wait(s_full + b, (j >> 1) & 1, p.err, kDevTimeoutAccum) ? 1 : 0;
            got = __shfl_sync(0xffffffffu, got, 0);
            if (!got) {
                ok = false;
                break;
            }
            tc_fence_after();
            // the block maximum over all kPBN columns; this half's columns kept for the exponentials
            const int kvalid = S - j * kPBN;  // keys of this block inside the sequence
            const uint32_t t_big = tmem + lane_off + b * 2 * kPBN;
            float mx = m;
            float sc[HC];
#pragma unroll
            for (int c0 = 0; c0 < kPBN; c0 += 16) {
                float vb[16], vsm[16];
                tmem_ld_16x2(t_big + c0, t_big + kPBN + c0, vb, vsm);
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                    const float v = (c0 + i < kvalid) ? (vb[i] + vsm[i]) * p.scale : -INFINITY;
                    mx = fmaxf(mx, v);
                    if (c0 / HC == hf) sc[(c0 % HC) + i] = v;
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(s_empty + b);
            const float corr = (m == -INFINITY) ? 0.f : expf(m - mx);
            float psum = 0.f;
#pragma unroll
            for (int i = 0; i < HC; ++i) {
                sc[i] = (sc[i] == -INFINITY) ? 0.f : expf(sc[i] - mx);
                psum += sc[i];
            }
            l = l * corr + psum;
            m = mx;
            // O_{j-1} is done (so is every read of the P buffer): fold it in, then write P_j.
            if (j > 0) {
                if (lane == 0) got = mbar_wait(o_full, (j - 1) & 1, p.err, kDevTimeoutAccum) ? 1 : 0;
                got = __shfl_sync(0xffffffffu, got, 0);
                if (!got) {
                    ok = false;
                    break;
                }
                tc_fence_after();
#pragma unroll
                for (int c0 = 0; c0 < HD; c0 += 16) {
                    float vb[16], vsm[16];
                    tmem_ld_16x2(t_o + lane_off + hf * HD + c0, t_o + lane_off + DH + hf * HD + c0, vb, vsm);
#pragma unroll
                    for (int i = 0; i < 16; ++i) o[c0 + i] = o[c0 + i] * corr_prev + (vb[i] + vsm[i]);
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(o_empty);
            }
            corr_prev = corr;
            {
                const uint32_t hi_atom = ps + hf * kAtomRows128 + p_row;
                const uint32_t lo_atom = ps + (kPBN / 32 + hf) * kAtomRows128 + p_row;
#pragma unroll
                for (int c = 0; c < 8; ++c) {
                    float h4[4], l4[4];
#pragma unroll
                    for (int e = 0; e < 4; ++e) split_tf32(sc[c * 4 + e], h4[e], l4[e]);
                    const uint32_t off = static_cast<uint32_t>((c ^ sw) * 16);
                    st_shared_f4(hi_atom + off, h4[0], h4[1], h4[2], h4[3]);
                    st_shared_f4(lo_atom + off, l4[0], l4[1], l4[2], l4[3]);
                }
            }
            fence_proxy_async_smem();  // P is read by the tensor cores (async proxy)
            __syncwarp();
            if (lane == 0) mbar_arrive(p_full);
        }
        if (ok) {
            int got = 1;
            if (lane == 0) got = mbar_wait(o_full, (nkb - 1) & 1, p.err, kDevTimeoutAccum) ? 1 : 0;
            got = __shfl_sync(0xffffffffu, got, 0);
            if (got) {
                tc_fence_after();
#pragma unroll
                for (int c0 = 0; c0 < HD; c0 += 16) {
                    float vb[16], vsm[16];
                    tmem_ld_16x2(t_o + lane_off + hf * HD + c0, t_o + lane_off + DH + hf * HD + c0, vb, vsm);
#pragma unroll
                    for (int i = 0; i < 16; ++i) o[c0 + i] = o[c0 + i] * corr_prev + (vb[i] + vsm[i]);
                }
                // The last P V has completed, so the P buffer is free: the two halves of each row
                // leave their partial sums there and take the other's.
                float* lx = reinterpret_cast<float*>(p_s);
                lx[hf * kPBM + row] = l;
                mbar_arrive(pair_end + qq);
                if (mbar_wait(pair_end + qq, 0, p.err, kDevTimeoutAccum)) {
                    const float l_all = l + lx[(1 - hf) * kPBM + row];
                    const int q = qb * kPBM + row;
                    if (q < S) {
                        const float inv = 1.0f / l_all;
                        const size_t base = static_cast<size_t>(row0 + q) * p.D + h * DH + hf * HD;
#pragma unroll
                        for (int d = 0; d < HD; d += 4) {
                            float4 hi, lo;
                            split_tf32(o[d] * inv, hi.x, lo.x);
                            split_tf32(o[d + 1] * inv, hi.y, lo.y);
                            split_tf32(o[d + 2] * inv, hi.z, lo.z);
                            split_tf32(o[d + 3] * inv, hi.w, lo.w);
                            *reinterpret_cast<float4*>(p.out_hi + base + d) = hi;
                            *reinterpret_cast<float4*>(p.out_lo + base + d) = lo;
                        }
                    }
                }
            }
        }
        tc_fence_before();
    }
    __syncwarp();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, L::kTmemCols);
    }
}

// [32 x 32] tiles of the V columns of the Q|K|V rows, written transposed and split into
// V^T [head * DH + d][vcol(row)] (hi and lo).
__global__ void prefill_vt_kernel(const float* __restrict__ qkv, int rows, int D,
                                  const int* __restrict__ row_vcol, int ldv,
                                  float* __restrict__ vt_hi, float* __restrict__ vt_lo) {
    __shared__ float tile[32][33];
    const int r0 = blockIdx.x * 32, c0 = blockIdx.y * 32;  // c over the D value columns
    for (int i = threadIdx.y; i < 32; i += blockDim.y) {
        const int r = r0 + i, cc = c0 + threadIdx.x;
        tile[i][threadIdx.x] = (r < rows && cc < D) ? qkv[static_cast<size_t>(r) * 3 * D + 2 * D + cc] : 0.f;
    }
    __syncthreads();
    for (int i = threadIdx.y; i < 32; i += blockDim.y) {
        const int cc = c0 + i, r = r0 + threadIdx.x;
        if (cc < D && r < rows) {
            float hi, lo;
            split_tf32(tile[threadIdx.x][i], hi, lo);
            const size_t dst = static_cast<size_t>(cc) * ldv + row_vcol[r];
            vt_hi[dst] = hi;
            vt_lo[dst] = lo;
        }
    }
}

__global__ void split_rows_kernel(const float* __restrict__ x, size_t n, float* __restrict__ hi,
                                  float* __restrict__ lo) {
    for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<size_t>(gridDim.x) * blockDim.x) {
        float h, l;
        split_tf32(x[i], h, l);
        hi[i] = h;
        lo[i] = l;
    }
}

typedef CUresult (*EncodeTiledFnP)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*,
                                   CUtensorMapInterleave, CUtensorMapSwizzle, CUtensorMapL2promotion,
                                   CUtensorMapFloatOOBfill);

bool make_map_p(CUtensorMap* map, const float* base, int cols, int rows, int box_rows) {
    static EncodeTiledFnP fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFnP>(f);
    });
    if (!fn || (reinterpret_cast<uintptr_t>(base) & 15) || (cols & 3)) return false;
    cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
    cuuint64_t strides[1] = {static_cast<cuuint64_t>(cols) * 4};
    cuuint32_t box[2] = {32, static_cast<cuuint32_t>(box_rows)};
    cuuint32_t estr[2] = {1, 1};
    return fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(base), dims, strides, box, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int DH>
cudaError_t prepare_prefill_attr() {
    static std::mutex mu;
    static unsigned long long done_mask = 0;
    int dev = 0;
    cudaGetDevice(&dev);
    std::lock_guard<std::mutex> lock(mu);
    if (dev >= 64 || (done_mask & (1ull << dev))) return cudaSuccess;
    const cudaError_t e = cudaFuncSetAttribute(prefill_attention_tc_kernel<DH>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               static_cast<int>(PrefillLayout<DH>::kBytes));
    if (e == cudaSuccess) done_mask |= (1ull << dev);
    return e;
}

}  // namespace

bool prefill_tc_supported(int head_dim) { return head_dim == 32 || head_dim == 64; }

int launch_prefill_attention_tc(const PrefillTcArgs& a, cudaStream_t st) {
    if (a.nseq <= 0 || a.max_len <= 0) return 0;
    if (!prefill_tc_supported(a.head_dim)) return static_cast<int>(cudaErrorInvalidValue);
    split_rows_kernel<<<static_cast<int>(std::min<size_t>((static_cast<size_t>(a.rows) * 3 * a.D + 255) / 256, 148 * 16)),
                        256, 0, st>>>(a.qkv, static_cast<size_t>(a.rows) * 3 * a.D, a.qkv_hi, a.qkv_lo);
    prefill_vt_kernel<<<dim3((a.rows + 31) / 32, (a.D + 31) / 32), dim3(32, 8), 0, st>>>(
        a.qkv, a.rows, a.D, a.row_vcol, a.ldv, a.vt_hi, a.vt_lo);
    PrefillParams p{};
    const int DHv = a.head_dim;
    if (!make_map_p(&p.q_hi, a.qkv_hi, 3 * a.D, a.rows, kPBM) || !make_map_p(&p.q_lo, a.qkv_lo, 3 * a.D, a.rows, kPBM) ||
        !make_map_p(&p.k_hi, a.qkv_hi, 3 * a.D, a.rows, kPBN) || !make_map_p(&p.k_lo, a.qkv_lo, 3 * a.D, a.rows, kPBN) ||
        !make_map_p(&p.v_hi, a.vt_hi, a.ldv, a.D, DHv) || !make_map_p(&p.v_lo, a.vt_lo, a.ldv, a.D, DHv))
        return static_cast<int>(cudaErrorInvalidValue);
    p.offsets = a.offsets;
    p.lens = a.lens;
    p.vcol = a.seq_vcol;
    p.out_hi = a.out_hi;
    p.out_lo = a.out_lo;
    p.D = a.D;
    p.scale = a.scale;
    p.err = a.err;
    const dim3 grid((a.max_len + kPBM - 1) / kPBM, a.D / DHv, a.nseq);
    cudaError_t e;
    if (DHv == 64) {
        if ((e = prepare_prefill_attr<64>()) != cudaSuccess) return static_cast<int>(e);
        prefill_attention_tc_kernel<64><<<grid, kPThreads, PrefillLayout<64>::kBytes, st>>>(p);
    } else {
        if ((e = prepare_prefill_attr<32>()) != cudaSuccess) return static_cast<int>(e);
        prefill_attention_tc_kernel<32><<<grid, kPThreads, PrefillLayout<32>::kBytes, st>>>(p);
    }
    return static_cast<int>(cudaGetLastError());
}

}  // namespace adai_b200
