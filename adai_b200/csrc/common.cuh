// common.cuh — shared device helpers for the sm_100a kernels: bounded mbarrier waits, TMA,
// tcgen05 (TMEM allocation, MMA, loads) and the 3xTF32 operand split.
//
// Every spin in these kernels is bounded: a wait that runs past its deadline records an error
// code in the context's device error word and returns false, and the caller leaves its loop.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace adai_b200 {

// Device error codes written into the context's error word (first writer wins).
enum DeviceError : int {
    kDevOk = 0,
    kDevTimeoutTmaFull = 101,   // MMA warp gave up waiting for a TMA stage
    kDevTimeoutSmemEmpty = 102, // producer gave up waiting for a free stage
    kDevTimeoutAccum = 103,     // epilogue gave up waiting for the accumulator
    kDevBadShape = 110,
    kDevAttnLength = 111,       // a cached length outside [0, max_len] or past the capacity
};

// Wait deadline for any device-side spin (nanoseconds of %globaltimer).
constexpr unsigned long long kSpinTimeoutNs = 2000000000ull;  // 2 s

__device__ __forceinline__ unsigned long long globaltimer_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ void record_error(int* err, int code) {
    if (err) atomicCAS(err, 0, code);
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---------------------------------------------------------------------------------------------
// mbarrier
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_barrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t addr, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(addr), "r"(parity)
        : "memory");
    return ok != 0;
}

// Bounded wait for the phase with the given parity to complete. Gives up after kSpinTimeoutNs
// (recording `code`), or at once when another thread of the context has already recorded an
// error, so one failure does not make every later wait run to its deadline.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* err, int code) {
    const uint32_t addr = smem_u32(bar);
    if (mbar_try_wait(addr, parity)) return true;
    const unsigned long long t0 = globaltimer_ns();
    while (true) {
        for (int i = 0; i < 256; ++i)
            if (mbar_try_wait(addr, parity)) return true;
        if (err && *reinterpret_cast<volatile int*>(err) != 0) return false;
        if (globaltimer_ns() - t0 > kSpinTimeoutNs) {
            record_error(err, code);
            return false;
        }
    }
}

// Bounded wait used to drain this CTA's own asynchronous work (copies landing in its shared
// memory, MMAs still running on its tensor memory) before it frees those resources or exits. It
// ignores the error word, so an aborted CTA still lets its in-flight operations finish; it gives
// up (recording `code`) only after its own deadline.
constexpr unsigned long long kDrainTimeoutNs = 1000000000ull;  // 1 s
__device__ __forceinline__ bool mbar_wait_drain(uint64_t* bar, uint32_t parity, int* err, int code) {
    const uint32_t addr = smem_u32(bar);
    if (mbar_try_wait(addr, parity)) return true;
    const unsigned long long t0 = globaltimer_ns();
    while (true) {
        for (int i = 0; i < 256; ++i)
            if (mbar_try_wait(addr, parity)) return true;
        if (globaltimer_ns() - t0 > kDrainTimeoutNs) {
            record_error(err, code);
            return false;
        }
    }
}

// ---------------------------------------------------------------------------------------------
// Thread-block clusters: rank, barrier, and loads from a peer CTA's shared memory (DSMEM).
__device__ __forceinline__ uint32_t cluster_ctarank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}

// Every thread of every CTA of the cluster must execute this (warp-converged).
__device__ __forceinline__ void cluster_sync_all() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\t"
                 "barrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// Split form of the cluster barrier: arrive early, wait later (both by every thread, in order).
__device__ __forceinline__ void cluster_arrive_all() {
    asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
}
// Arrival of one thread on the cluster barrier, from divergent code: each thread of every CTA
// of the cluster arrives once (here or with cluster_arrive_all) before it waits.
__device__ __forceinline__ void cluster_arrive_one() {
    asm volatile("barrier.cluster.arrive.release;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait_all() {
    asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// 16-byte shared-memory load / store at a shared-window address.
__device__ __forceinline__ float4 ld_shared_f4(uint32_t addr) {
    float4 v;
    asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                 : "r"(addr)
                 : "memory");
    return v;
}
__device__ __forceinline__ void st_shared_f4(uint32_t addr, float a, float b, float c, float d) {
    asm volatile("st.shared.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "f"(a), "f"(b), "f"(c),
                 "f"(d)
                 : "memory");
}

// Make this thread's generic-proxy shared-memory writes visible to the async proxy (bulk copies).
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Bulk copy of `bytes` (multiple of 16) from this CTA's shared memory to another CTA's shared
// memory in the cluster; completion is signalled as transaction bytes on the destination CTA's
// mbarrier. dst and bar are shared::cluster addresses.
__device__ __forceinline__ void bulk_copy_to_peer(uint32_t dst_cluster, uint32_t src_cta,
                                                  uint32_t bytes, uint32_t bar_cluster) {
    asm volatile(
        "cp.async.bulk.shared::cluster.shared::cta.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
        ::"r"(dst_cluster), "r"(src_cta), "r"(bytes), "r"(bar_cluster)
        : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// Waits until the source reads of every committed bulk copy of this thread are done.
__device__ __forceinline__ void bulk_wait_reads() {
    asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}

// Programmatic dependent launch: wait for the preceding kernel's completion (and its memory) /
// allow the next kernel in the stream to start launching. No-ops without the launch attribute.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// shared::cluster address of the same shared-memory location in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t dsmem_addr(uint32_t local_smem_addr, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(local_smem_addr), "r"(rank));
    return r;
}

__device__ __forceinline__ float4 ld_dsmem_f4(uint32_t cluster_addr) {
    float4 v;
    asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                 : "r"(cluster_addr)
                 : "memory");
    return v;
}

// ---------------------------------------------------------------------------------------------
// TMA (tiled tensor copies, no multicast)
// Request the 128-byte line holding `ptr` into L1 (no register result, no wait).
__device__ __forceinline__ void prefetch_l1(const void* ptr) {
    asm volatile("prefetch.global.L1 [%0];" ::"l"(reinterpret_cast<uint64_t>(ptr)));
}
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// 2-D tiled load of the box at (x = inner coordinate, y) into shared memory; completion is
// signalled on `bar` as transaction bytes. x * element size must be a multiple of 16 bytes.
__device__ __forceinline__ void tma_load_2d(void* smem_dst, const CUtensorMap* map, uint64_t* bar,
                                            int x, int y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(smem_dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y)
        : "memory");
}

// The same with an L2 cache policy (from l2_policy_evict_first / createpolicy).
__device__ __forceinline__ void tma_load_2d_hint(void* smem_dst, const CUtensorMap* map, uint64_t* bar,
                                                 int x, int y, uint64_t policy) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
        " [%0], [%1, {%3, %4}], [%2], %5;" ::"r"(smem_u32(smem_dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y), "l"(policy)
        : "memory");
}

// An L2 policy under which the lines a load brings in are the first to be evicted (data read once).
// An L2 policy under which the lines a load brings in are kept longest (data read many times).
__device__ __forceinline__ uint64_t l2_policy_evict_last() {
    uint64_t policy;
    asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(policy));
    return policy;
}
__device__ __forceinline__ uint64_t l2_policy_evict_first() {
    uint64_t policy;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(policy));
    return policy;
}

// ---------------------------------------------------------------------------------------------
// tcgen05
__device__ __forceinline__ void tmem_alloc(uint32_t* smem_result, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(smem_result)),
                 "r"(ncols)
                 : "memory");
}

__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
                 : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem] * B[smem]^T, kind::tf32, one CTA. accumulate = 0 overwrites D.
__device__ __forceinline__ void mma_tf32(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                         uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// Arrive on `bar` once every tcgen05.mma issued so far by this thread has completed.
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
    asm volatile(
        "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
            smem_u32(bar))
        : "memory");
}

// tcgen05.ld writes its destination registers asynchronously: they hold the data only after
// tcgen05.wait::ld. The load(s) and the wait are therefore one asm statement, so the compiler
// never sees the outputs (nor reuses their registers) before the wait has completed.
//
// 32 lanes x 16 columns of 32-bit accumulator: thread i of the warp gets row (lane base + i),
// columns [col, col+16).
__device__ __forceinline__ void tmem_ld_16(uint32_t taddr, float (&v)[16]) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,"
        "%14,%15}, [%16];\n\t"
        "tcgen05.wait::ld.sync.aligned;"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
          "=r"(r[14]), "=r"(r[15])
        : "r"(taddr)
        : "memory");
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// Two 32x32b.x16 loads (e.g. the hi*hi and the correction accumulators of the same columns) in
// flight together, one wait.
__device__ __forceinline__ void tmem_ld_16x2(uint32_t taddr_a, uint32_t taddr_b, float (&va)[16],
                                             float (&vb)[16]) {
    uint32_t a[16], b[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,"
        "%14,%15}, [%32];\n\t"
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,"
        "%28,%29,%30,%31}, [%33];\n\t"
        "tcgen05.wait::ld.sync.aligned;"
        : "=r"(a[0]), "=r"(a[1]), "=r"(a[2]), "=r"(a[3]), "=r"(a[4]), "=r"(a[5]), "=r"(a[6]),
          "=r"(a[7]), "=r"(a[8]), "=r"(a[9]), "=r"(a[10]), "=r"(a[11]), "=r"(a[12]), "=r"(a[13]),
          "=r"(a[14]), "=r"(a[15]), "=r"(b[0]), "=r"(b[1]), "=r"(b[2]), "=r"(b[3]), "=r"(b[4]),
          "=r"(b[5]), "=r"(b[6]), "=r"(b[7]), "=r"(b[8]), "=r"(b[9]), "=r"(b[10]), "=r"(b[11]),
          "=r"(b[12]), "=r"(b[13]), "=r"(b[14]), "=r"(b[15])
        : "r"(taddr_a), "r"(taddr_b)
        : "memory");
#pragma unroll
    for (int i = 0; i < 16; ++i) {
        va[i] = __uint_as_float(a[i]);
        vb[i] = __uint_as_float(b[i]);
    }
}

// Shared-memory matrix descriptor for a K-major operand stored in the canonical 128-byte
// swizzled layout (rows of 128 bytes, 8-row swizzle atoms 1024 bytes apart). The tile base must be
// 1024-byte aligned; stepping K inside the 128-byte row moves the start address.
__device__ __forceinline__ uint64_t smem_desc_k_sw128(uint32_t saddr) {
    uint64_t d = 0;
    d |= static_cast<uint64_t>((saddr & 0x3FFFF) >> 4);          // start address  [0,14)
    d |= static_cast<uint64_t>(16 >> 4) << 16;                   // LBO (unused)   [16,30)
    d |= static_cast<uint64_t>(1024 >> 4) << 32;                 // SBO = 1024 B   [32,46)
    d |= static_cast<uint64_t>(1) << 46;                         // version = 1    [46,48)
    d |= static_cast<uint64_t>(2) << 61;                         // SWIZZLE_128B   [61,64)
    return d;
}

// Instruction descriptor: kind::tf32, fp32 accumulate, A and B K-major, M = 128, N = n.
__host__ __device__ constexpr uint32_t idesc_tf32(int m, int n) {
    return (1u << 4)                                  // D format F32
           | (2u << 7)                                // A format TF32
           | (2u << 10)                               // B format TF32
           | (0u << 15) | (0u << 16)                  // K-major A, K-major B
           | (static_cast<uint32_t>(n >> 3) << 17)    // N >> 3
           | (static_cast<uint32_t>(m >> 4) << 24);   // M >> 4
}

// ---------------------------------------------------------------------------------------------
// 3xTF32 operand split: x = hi + lo with hi = tf32(x), lo = tf32(x - hi), both stored as fp32
// bit patterns whose low 13 mantissa bits are zero (round-to-nearest-away, cvt.rna).
__device__ __forceinline__ float tf32_rna(float x) {
    uint32_t r;
    asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
    return __uint_as_float(r);
}

__device__ __forceinline__ void split_tf32(float x, float& hi, float& lo) {
    hi = tf32_rna(x);
    lo = tf32_rna(x - hi);
}

// GELU, tanh approximation with the reference constants (src/ActivationConstants.hpp:18-19).
__device__ __forceinline__ float gelu_tanh(float x) {
    const float cube = x * x * x;
    const float inner = 0.7978845608f * (x + 0.044715f * cube);
    return 0.5f * x * (1.0f + tanhf(inner));
}

}  // namespace adai_b200
