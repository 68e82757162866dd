// kernels.h — host-side launch interface of the sm_100a kernels (internal to libadai_b200.so).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>
#include <utility>

namespace adai_b200 {

// ------------------------------------------------------------------------------------------
// Programmatic dependent launch. While enabled on the calling thread, every launch below asks
// for programmatic stream serialization: the kernel may start its prologue while the preceding
// kernel finishes; each kernel waits (griddepcontrol.wait) before touching data of earlier
// kernels. The decode step enables it around the launches it captures into its CUDA graph.
bool launch_pdl_enabled();
void set_launch_pdl(bool on);

struct ScopedPdl {
    bool prev;
    explicit ScopedPdl(bool on) : prev(launch_pdl_enabled()) { set_launch_pdl(on); }
    ~ScopedPdl() { set_launch_pdl(prev); }
};

template <typename... KArgs, typename... Args>
cudaError_t launch_kernel(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                          cudaStream_t st, Args&&... args) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    if (launch_pdl_enabled()) {
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
    }
    return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// ------------------------------------------------------------------------------------------
// 3xTF32 tcgen05 GEMM: out[M,N] = epilogue(A[M,K] * W[K,N]) with A given as its tf32 split
// (A_hi, A_lo, row-major [M,K]) and W given transposed and split (W_hi, W_lo, row-major [N,K]).
enum GemmFlags : int {
    kEpiBias = 1,       // + bias[n]
    kEpiGelu = 2,       // GELU-tanh after the bias
    kEpiResid = 4,      // resid[m,n] + (...)
    kEpiStore = 8,      // write fp32 out[m,n]
    kEpiSplit = 16,     // write the tf32 split of the result to out_hi / out_lo
    kEpiArgmax = 32,    // per-row first maximum -> next_ids (and the non-finite flag)
    kEpiKvScatter = 64, // columns [0,D) -> K cache, [D,2D) -> V cache at (row_slot, row_pos)
    // Per output row and 32-column group: (sum, sum of squared deviations from the group mean)
    // -> row_stats[row * (N / 32) + col / 32] (N a multiple of 64). Written by the GEMMs that
    // produce the residual stream, for the LayerNorm the next GEMM folds in.
    kEpiRowStats = 128,
    // LayerNorm folded into this GEMM: A holds the split of the un-normalised rows x, W holds
    // diag(gamma) W, and the result is rstd * (acc - mean * ln_c1[n]) before the bias, where
    // ln_c1 = column sums of diag(gamma) W and the bias holds beta W (+ the layer's own bias).
    // mean / rstd per row come from the K / 32 group statistics in row_stats.
    kEpiLnFold = 256,
    // Not an epilogue: A arrives in fp32 (TcActs::fp32, row stride lda); TMA brings its boxes
    // raw and two converter warps split them into tf32 hi / lo in shared memory (the op-level
    // entry points: one launch instead of a split kernel and the GEMM).
    kEpiAFp32 = 512,
};

struct GemmEpilogue {
    int flags = 0;
    const float* bias = nullptr;
    const float* resid = nullptr;
    int ldr = 0;
    float* out = nullptr;
    int ldo = 0;
    float* out_hi = nullptr;
    float* out_lo = nullptr;
    int lds = 0;
    // argmax
    int* next_ids = nullptr;
    int* nonfinite = nullptr;
    // kv scatter
    float* kc = nullptr;
    float* vc = nullptr;
    long long slot_stride = 0;  // floats between slots
    int cap = 0;                // rows per (slot, head)
    int head_dim = 64;
    int d_model = 0;
    const int* row_slot = nullptr;
    const int* row_pos = nullptr;
    // row statistics (kEpiRowStats writes, kEpiLnFold reads): float2 [stats_ld rows][width / 32]
    float2* row_stats = nullptr;
    int stats_ld = 0;  // rows allocated
    const float* ln_c1 = nullptr;  // kEpiLnFold: [N]
};

// A prepared right-hand operand: W^T split into hi/lo, [N, K] row-major, device memory.
struct TcWeight {
    int K = 0, N = 0;
    float* hi = nullptr;
    float* lo = nullptr;
};

// A left-hand operand: the tf32 split of A, [rows_alloc, K] row-major, device memory.
struct TcActs {
    int K = 0, rows_alloc = 0;
    const float* hi = nullptr;
    const float* lo = nullptr;
    // kEpiAFp32: A itself, [rows, k_valid] row-major with row stride lda (a multiple of 4, base
    // 16-byte aligned); rows past `rows` and columns past k_valid read as zero
    const float* fp32 = nullptr;
    int lda = 0, k_valid = 0, rows = 0;
};

struct GemmPlan {
    int bn = 128;
    int splits = 1;
    int stages = 3;
    int kb_per_split = 0;
    int chunk_kb = 1;  // K blocks accumulated in TMEM before promotion to fp32 registers
    int m_tiles = 1, n_tiles = 1;
    size_t smem_bytes = 0;
};

// Scratch a GEMM launch may use: split-K partial tiles and per-tile tickets (zeroed at creation;
// every launch leaves them zero again), argmax partials.
struct GemmScratch {
    float* ws = nullptr;
    size_t ws_floats = 0;
    int* tickets = nullptr;
    int n_tickets = 0;
    // LM-head argmax: per output row the running first maximum as one 64-bit key (the value's
    // order-preserving bits above the complemented column) and a non-finite flag. Both start at
    // zero; the last CTA of each row block reads them back and leaves them at zero.
    unsigned long long* arg_key = nullptr;
    int* arg_nf = nullptr;
    size_t arg_rows = 0;
};

GemmPlan gemm_plan(int M, int N, int K, int flags, int num_sms);
size_t gemm_ws_floats(const GemmPlan& p);
size_t gemm_arg_rows(const GemmPlan& p);

// Encodes (or reuses) the tensor maps and launches. Returns a cudaError_t-style code: 0 ok,
// cudaErrorInvalidValue for shapes the kernel cannot take.
int gemm_launch(const TcActs& a, int M, const TcWeight& w, const GemmEpilogue& epi,
                const GemmPlan& plan, const GemmScratch& scratch, int* err, cudaStream_t st);

bool tensor_map_api_available();
// Clusters of `splits` GEMM CTAs (tile width bn, `stages` pipeline stages) the device holds at once.
int gemm_cluster_capacity(int bn, int splits, int stages);

// ------------------------------------------------------------------------------------------
// Row kernels
void launch_split_tf32(const float* x, float* hi, float* lo, size_t n, cudaStream_t st);
void launch_transpose_split(const float* w, int K, int N, float* hi_t, float* lo_t,
                            cudaStream_t st);
// LayerNorm (two-pass, eps 1e-5) of `rows` rows of x (row stride ldx); writes any of out / the
// split (out_hi, out_lo), row stride D.
void launch_layernorm(const float* x, int ldx, const float* g, const float* b, float* out,
                      float* out_hi, float* out_lo, int rows, int D, cudaStream_t st);
// x[r] = table[ids[r]] + pe[pos(r)] (no positional row when pos >= pe_rows), then LayerNorm.
// pos(r) = pos_by_slot ? pos_by_slot[slots[r]] : pos_direct[r].
void launch_embed_ln(const float* table, const int* ids, const float* pe, int pe_rows,
                     const int* slots, const int* pos_by_slot, const int* pos_direct, float* x,
                     const float* g, const float* b, float* out_hi, float* out_lo, int rows,
                     int D, int vocab, int* err, cudaStream_t st);
// x[r] = table[ids[r]] + pe[pos_by_slot[slots[r]]] (no positional row when pos >= pe_rows),
// its tf32 split, and the row statistics of kEpiRowStats (the decode step's first LayerNorm is
// folded into the Q|K|V GEMM).
void launch_embed_stats(const float* table, const int* ids, const float* pe, int pe_rows,
                        const int* slots, const int* pos_by_slot, float* x, float* x_hi,
                        float* x_lo, float2* stats, int rows, int D, int vocab, int* err,
                        cudaStream_t st);

// ------------------------------------------------------------------------------------------
// Attention
struct DecodeAttnArgs {
    const float* q = nullptr;  // row b at q + b*ldq; head h at + h*head_dim
    int ldq = 0;
    const float* k_new = nullptr;  // self-attention append source (null: no append)
    const float* v_new = nullptr;
    int ldkv = 0;
    float* kc = nullptr;  // this layer's cache: [slot][H][cap][head_dim]
    float* vc = nullptr;
    long long slot_stride = 0;
    int cap = 0;
    const int* slots = nullptr;        // [B] slot of each batch row (null: row b is slot b)
    const int* len_by_slot = nullptr;  // rows already cached per slot
    int len_add = 0;                   // 1 for self-attention (the appended row)
    float* out = nullptr;              // optional fp32 [B, ldo]
    float* out_hi = nullptr;           // optional split
    float* out_lo = nullptr;
    int ldo = 0;
    int B = 0, H = 0;
    int head_dim = 64;  // 32 or 64
    int max_len = 0;  // upper bound of len over the batch (sizes the grid)
    float scale = 0.f;
    float* ws = nullptr;  // split-KV partials
    int* tickets = nullptr;
    int chunk = 256;  // cached rows per CTA: kAttnChunk or kAttnChunkShort
    int* err = nullptr;  // device error word: a length outside [0, max_len] records kDevAttnLength
};
constexpr int kAttnChunk = 256;       // cached rows per CTA (default)
constexpr int kAttnChunkShort = 128;  // the decode step's cross-attention
bool attention_head_dim_supported(int head_dim);
// split-KV partials: per (b, h, chunk) m, l, 2 pad, head_dim accumulators
size_t decode_attn_ws_floats(int B, int H, int max_len, int head_dim, int chunk = kAttnChunk);
void launch_decode_attention(const DecodeAttnArgs& a, int* err, cudaStream_t st);

// Encoder self-attention on the tensor cores (prefill_tc.cu). qkv [rows, 3D] fp32 is split into
// qkv_hi/lo and its V columns transposed into vt_hi/lo [D, ldv]: row r of sequence s lands in
// column row_vcol[r] = seq_vcol[s] + position, seq_vcol multiples of 32.
struct PrefillTcArgs {
    const float* qkv = nullptr;
    float* qkv_hi = nullptr;
    float* qkv_lo = nullptr;
    float* vt_hi = nullptr;
    float* vt_lo = nullptr;
    int ldv = 0;
    const int* row_vcol = nullptr;
    const int* seq_vcol = nullptr;
    const int* offsets = nullptr;
    const int* lens = nullptr;
    int nseq = 0, max_len = 0, rows = 0, D = 0, head_dim = 64;
    float* out_hi = nullptr;
    float* out_lo = nullptr;
    float scale = 0.f;
    int* err = nullptr;
};
bool prefill_tc_supported(int head_dim);
int launch_prefill_attention_tc(const PrefillTcArgs& a, cudaStream_t st);

// Row and elementwise operations of the reference backend table (backend_ops.cu).
void launch_softmax_rows(float* data, int rows, int cols, cudaStream_t st);
void launch_layernorm_rows(const float* x, float* y, float* xn, const float* g, const float* b,
                           float* mean, float* rstd, int rows, int cols, float eps, cudaStream_t st);
void launch_add_row_bias(const float* m, const float* bias, float* out, int rows, int cols,
                         cudaStream_t st);
void launch_activation(float* data, size_t n, int type, cudaStream_t st);  // 0 ReLU 1 sigmoid 2 tanh 3 GELU
void launch_embed_pe(const float* table, const int* ids, const float* pe, int pe_rows, int pos_offset,
                     float* out, int n, int d, int vocab, int* err, cudaStream_t st);

// Encoder self-attention over ragged sequences: qkv [rows, 3D]; sequence s holds rows
// [offsets[s], offsets[s] + lens[s]); out split [rows, D].
void launch_prefill_attention(const float* qkv, int D, int H, const int* offsets, const int* lens,
                              int nseq, int max_len, float* out_hi, float* out_lo, float scale,
                              cudaStream_t st);

// Decode-loop bookkeeping: ids[b] = next[b]; len_by_slot[slots[b]] += 1.
void launch_advance(const int* next, int* ids, const int* slots, int* len_by_slot, int B,
                    cudaStream_t st);

// Diagnostic: one CTA makes a bounded device wait run out (error code kDevTimeoutAccum in *err)
// and a second wait return at once because the error word is set; *gave_up = 3 when both gave up.
void launch_wait_selftest(int* err, int* gave_up, cudaStream_t st);

// ---- token selection with the reference's sampling rules (sample.cu) ----
// Per-slot configuration (GenerationConfig's sampling fields, src/TextGenerator.hpp:65-82).
struct SampleSlot {
    float temperature = 1.0f, top_p = 1.0f, penalty = 1.0f;
    int top_k = 0, min_length = 0, eos = 3, pad = 0;
    int enabled = 0;  // 0: the row keeps the step's fused argmax
};
constexpr int kMtWords = 640;  // per slot: std::mt19937 state [624] + read position, padded
struct SampleArgs {
    const float* logits = nullptr;  // [B, ld]
    int ld = 0;
    const int* slots = nullptr;     // [B]
    const int* fed = nullptr;       // [B] token fed this step (counts as seen), or null
    int* next = nullptr;            // [B] chosen token (rows whose slot is disabled untouched)
    int* nonfinite = nullptr;       // [B] set to 1 for NaN / +inf / all -inf rows, or null
    const SampleSlot* cfg = nullptr;  // [slots]
    unsigned* mt = nullptr;         // [slots][kMtWords]
    unsigned* seen = nullptr;       // [slots][seen_words] bit per token id
    int seen_words = 0;
    int* new_tokens = nullptr;      // [slots] steps sampled since the slot was configured
    float* scratch = nullptr;       // [B, V] (top-p parks the filtered row here)
    int B = 0, V = 0;
};
int sample_max_vocab();
cudaError_t launch_sample_rows(const SampleArgs& a, cudaStream_t st);

}  // namespace adai_b200
