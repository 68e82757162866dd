// engine.cu — host runtime behind the C ABI (include/adai_b200.h): per-GPU context, model
// upload, KV-cache arena, encoder prefill, the stacked decode step and its CUDA-graph replay.
//
// Reference behaviour this mirrors:
//   GPUManager (src/gpu/GPUUtils.hpp:98-530): one device, one stream, a memory budget.
//   GPUDecoderKVCache (src/gpu/MatrixGPU.hpp:563-623): fixed-capacity per-layer caches.
//   LLMDecoder::gpu_decode_step (src/Decoder.cpp:566-608) / forward_with_cache (:210-287), for B
//   stacked sequences instead of one: embed + PE, L pre-LN blocks, final LN, LM head, argmax.
//   LLMEncoder::encode_with_mask (src/LLMEncoder.cpp:120-142) + CrossAttention's first-call K/V.
#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <limits>
#include <map>
#include <memory>
#include <mutex>
#include <random>
#include <set>
#include <stdexcept>
#include <string>
#include <thread>
#include <tuple>
#include <vector>

#include "../../include/adai_b200.h"
#include "common.cuh"
#include "checkpoint.h"
#include "kernels.h"
#include "trace.h"

using namespace adai_b200;

namespace adai_b200 {
bool layernorm_width_supported(int D);
}

namespace {

thread_local std::string g_last_error;

struct Status : std::runtime_error {
    int code;
    Status(int c, const std::string& m) : std::runtime_error(m), code(c) {}
};

[[noreturn]] void fail(int code, const std::string& msg) { throw Status(code, msg); }

void cuda_ok(cudaError_t e, const char* what) {
    if (e != cudaSuccess)
        fail(ADAI_B200_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

void launch_ok(int e, const char* what) {
    if (e != 0) fail(ADAI_B200_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(static_cast<cudaError_t>(e)));
}

template <class Fn>
int guarded(Fn&& fn) {
    try {
        fn();
        g_last_error.clear();
        return ADAI_B200_OK;
    } catch (const Status& s) {
        g_last_error = s.what();
        return s.code;
    } catch (const std::bad_alloc&) {
        g_last_error = "host allocation failed";
        return ADAI_B200_ERR_CUDA;
    } catch (const CheckpointIoError& e) {
        g_last_error = e.what();
        return ADAI_B200_ERR_IO;
    } catch (const std::invalid_argument& e) {
        g_last_error = e.what();
        return ADAI_B200_ERR_INVALID_ARGUMENT;
    } catch (const std::exception& e) {
        g_last_error = e.what();
        return ADAI_B200_ERR_CUDA;
    }
}

inline int round_up(int x, int m) { return (x + m - 1) / m * m; }

double wait_timeout_seconds() {
    const char* s = std::getenv("ADAI_B200_WAIT_TIMEOUT_SECONDS");
    if (s && *s) {
        const double v = std::atof(s);
        if (v > 0) return v;
    }
    return 120.0;
}

constexpr int kEncRows = 16384;  // encoder prefill rows per chunk

}  // namespace

// ---------------------------------------------------------------------------------------------
struct EncLayerW {
    const float *ln1g, *ln1b, *ln2g, *ln2b, *b1, *b2;
    TcWeight qkv, o, w1, w2;
};
struct DecLayerW {
    const float *ln1g, *ln1b, *ln2g, *ln2b, *ln3g, *ln3b, *b1, *b2;
    TcWeight qkv, o, cq, ckv, co, w1, w2;
    // qkv, cq and w1 hold diag(gamma) W of the LayerNorm before them (kEpiLnFold): the column
    // sums of that product and the bias beta W (+ b1 for w1)
    float *qkv_c1 = nullptr, *qkv_bias = nullptr, *cq_c1 = nullptr, *cq_bias = nullptr,
          *w1_c1 = nullptr, *w1_bias = nullptr;
};

struct Model {
    adai_b200_model_desc d{};
    float* pe = nullptr;
    float* enc_embed = nullptr;
    float* dec_embed = nullptr;
    const float *enc_lnf_g = nullptr, *enc_lnf_b = nullptr, *dec_lnf_g = nullptr,
                *dec_lnf_b = nullptr, *head_b = nullptr;
    std::vector<EncLayerW> enc;
    std::vector<DecLayerW> dec;
    TcWeight head;  // diag(final gamma) W_out; head_c1 / head_bias as for the layers' folded W
    float *head_c1 = nullptr, *head_bias = nullptr;
    std::vector<void*> owned;
};

struct StepBufs {
    int rows = 0;  // allocated rows (multiple of 128)
    float *x = nullptr, *nrm_hi = nullptr, *nrm_lo = nullptr, *qkv = nullptr, *attn_hi = nullptr,
          *attn_lo = nullptr, *qc = nullptr, *h_hi = nullptr, *h_lo = nullptr,
          *logits = nullptr;
    float2* ln_stats = nullptr;  // [rows][d_model / 32] residual-stream group statistics
    int *ids = nullptr, *next = nullptr, *slots = nullptr, *nonfinite = nullptr,
        *nonfinite_any = nullptr;
};

struct EncBufs {
    int rows = 0;
    float *x = nullptr, *nrm_hi = nullptr, *nrm_lo = nullptr, *qkv = nullptr, *attn_hi = nullptr,
          *attn_lo = nullptr, *h_hi = nullptr, *h_lo = nullptr, *out = nullptr;
    int *ids = nullptr, *row_slot = nullptr, *row_pos = nullptr, *offsets = nullptr,
        *lens = nullptr;
    // tensor-core prefill attention: split Q|K|V rows and the transposed V columns
    float *qkv_hi = nullptr, *qkv_lo = nullptr, *vt_hi = nullptr, *vt_lo = nullptr;
    int ldv = 0;
    int *row_vcol = nullptr, *seq_vcol = nullptr;
};

struct adai_b200_kv {
    int max_slots = 0, self_cap = 0, cross_cap = 0, L = 0, H = 0, dh = 64;
    float *self_k = nullptr, *self_v = nullptr, *cross_k = nullptr, *cross_v = nullptr;
    int *d_self_len = nullptr, *d_cross_len = nullptr;
    int* d_hist = nullptr;  // [max_slots][self_cap]: the argmax produced at each position
    std::vector<int> self_len, cross_len;
    std::vector<char> encoded;  // the slot holds an encoder output (possibly of no rows)
    // sampling state per slot (allocated on first use): configuration, std::mt19937, the set of
    // token ids already in the sequence (one bit each), steps sampled since configured
    SampleSlot* d_samp = nullptr;
    unsigned* d_mt = nullptr;
    unsigned* d_seen = nullptr;
    int* d_new_tokens = nullptr;
    int seen_words = 0, samp_vocab = 0;
    std::vector<char> samp_on;
    long long self_slot_stride() const { return static_cast<long long>(H) * self_cap * dh; }
    long long cross_slot_stride() const { return static_cast<long long>(H) * cross_cap * dh; }
    float* self_k_layer(int l) const { return self_k + static_cast<size_t>(l) * max_slots * self_slot_stride(); }
    float* self_v_layer(int l) const { return self_v + static_cast<size_t>(l) * max_slots * self_slot_stride(); }
    float* cross_k_layer(int l) const { return cross_k + static_cast<size_t>(l) * max_slots * cross_slot_stride(); }
    float* cross_v_layer(int l) const { return cross_v + static_cast<size_t>(l) * max_slots * cross_slot_stride(); }
};

struct adai_b200_weight {
    TcWeight w;
    int K = 0;     // the caller's inner dimension
    int Kpad = 0;  // K rounded up to a multiple of 4 (16-byte rows for TMA)
};

struct GraphKey {
    const adai_b200_kv* kv;
    int B;
    int flags;
    bool operator<(const GraphKey& o) const {
        return std::tie(kv, B, flags) < std::tie(o.kv, o.B, o.flags);
    }
};

enum StepFlags { kStepLogits = 1, kStepAdvanceIds = 2, kStepSample = 4 };

// Per-launch CUDA-event spans of a profiled (eager) decode step, with the algorithmic bytes and
// flops of each launch, grouped by kernel class (adai_b200_kernel_class in the header).
struct Span {
    cudaEvent_t a, b;
    int cls;
    double bytes, flops;
};
struct Profiler {
    std::vector<Span> spans;
    double sum_self_rows = 0;   // sum over the batch of rows attended by self-attention
    double sum_cross_rows = 0;  // ... by cross-attention
};

struct adai_b200_ctx {
    int device = 0;
    int num_sms = 148;
    cudaStream_t stream = nullptr;
    size_t mem_cap = 0, mem_used = 0;
    std::map<void*, size_t> allocs;
    int* d_err = nullptr;
    bool unusable = false;
    std::unique_ptr<Model> model;
    std::set<adai_b200_kv*> kvs;
    StepBufs sb;
    EncBufs eb;
    GemmScratch gs;
    float* attn_ws = nullptr;
    size_t attn_ws_floats = 0;
    int* attn_tickets = nullptr;
    int attn_n_tickets = 0;
    float *op_a_hi = nullptr, *op_a_lo = nullptr;
    size_t op_a_floats = 0;
    float* op_c = nullptr;  // packed output of op-level GEMMs whose C is not float4-aligned
    size_t op_c_floats = 0;
    float* samp_park = nullptr;  // [rows, V]: top-p parks the filtered logits here
    size_t samp_park_floats = 0;
    int* h_pin = nullptr;  // pinned staging for ids / slots / lengths
    int* h_err = nullptr;  // pinned copy of the device error word, read back by sync()
    cudaEvent_t sync_ev = nullptr;
    size_t h_pin_ints = 0;
    std::map<GraphKey, cudaGraphExec_t> graphs;
    std::map<GraphKey, int> graph_kernels;
    Profiler* prof = nullptr;
    double last_decode_ms = 0.0;
    int last_kernels_per_step = 0;
    adai_b200_trace::WorkTrace trace;  // last work queued, for failed waits (trace.h)

    void* dalloc(size_t bytes) {
        if (bytes == 0) bytes = 16;
        if (mem_cap && mem_used + bytes > mem_cap)
            fail(ADAI_B200_ERR_CUDA, "device memory budget (mem_fraction) exceeded: need " +
                                         std::to_string(bytes) + " more bytes, " +
                                         std::to_string(mem_cap - mem_used) + " left");
        void* p = nullptr;
        cuda_ok(cudaMalloc(&p, bytes), "cudaMalloc");
        allocs[p] = bytes;
        mem_used += bytes;
        return p;
    }
    template <class T>
    T* dalloc_t(size_t n) {
        return static_cast<T*>(dalloc(n * sizeof(T)));
    }
    template <class T>
    T* dzalloc_t(size_t n) {
        T* p = dalloc_t<T>(n);
        cuda_ok(cudaMemsetAsync(p, 0, n * sizeof(T), stream), "cudaMemset");
        return p;
    }
    void dfree(void* p) {
        if (!p) return;
        auto it = allocs.find(p);
        if (it != allocs.end()) {
            mem_used -= it->second;
            allocs.erase(it);
        }
        cudaFree(p);
    }
    void clear_graphs() {
        for (auto& kvp : graphs) cudaGraphExecDestroy(kvp.second);
        graphs.clear();
        graph_kernels.clear();
    }
    void check_usable() const {
        if (unusable)
            fail(ADAI_B200_ERR_STATE, "context is unusable after an earlier device timeout or fault");
    }
    int* pinned(size_t n) {
        if (n > h_pin_ints) {
            // copies queued from the old buffer must finish before it is released
            cuda_ok(cudaStreamSynchronize(stream), "sync before staging growth");
            if (h_pin) cudaFreeHost(h_pin);
            h_pin = nullptr;
            h_pin_ints = 0;
            cuda_ok(cudaMallocHost(&h_pin, n * sizeof(int)), "cudaMallocHost");
            h_pin_ints = n;
        }
        return h_pin;
    }
    bool capturing() const {
        cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
        return cudaStreamIsCapturing(stream, &cs) == cudaSuccess && cs != cudaStreamCaptureStatusNone;
    }
    // Records a launch about to be queued. With ADAI_B200_SYNC=kernel[:N] it first waits for the
    // work already queued (before every Nth launch), so a failure is reported against the kernel
    // that ran; never inside a stream capture.
    void note(const char* kernel) {
        if (capturing()) return;  // recorded into a graph, not queued: its replay is noted
        const adai_b200_trace::Settings& st = adai_b200_trace::settings();
        if (st.mode == adai_b200_trace::kSyncKernel) {
            const unsigned long long n = trace.seq.load(std::memory_order_relaxed);
            if (n > 0 && (st.every <= 1 || n % st.every == 0)) sync(wait_timeout_seconds());
        }
        trace.note_kernel(kernel);
    }
    std::string last_work() const { return "; last GPU work queued: " + trace.describe(); }
    // Bounded host wait (GPU_WAIT_TIMEOUT_SECONDS semantics), then the device error word.
    void sync(double timeout_s) {
        // the error word comes back with the work (no second round trip after the wait)
        cuda_ok(cudaMemcpyAsync(h_err, d_err, sizeof(int), cudaMemcpyDeviceToHost, stream),
                "read error word");
        cudaEvent_t ev = sync_ev;
        cuda_ok(cudaEventRecord(ev, stream), "cudaEventRecord");
        const auto t0 = std::chrono::steady_clock::now();
        while (true) {
            const cudaError_t q = cudaEventQuery(ev);
            if (q == cudaSuccess) break;
            if (q != cudaErrorNotReady) {
                unusable = true;
                fail(ADAI_B200_ERR_CUDA,
                     std::string("device error: ") + cudaGetErrorString(q) + last_work());
            }
            const double el =
                std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
            if (el > timeout_s) {
                unusable = true;
                fail(ADAI_B200_ERR_TIMEOUT,
                     "device wait exceeded " + std::to_string(timeout_s) + " s" + last_work());
            }
            std::this_thread::yield();
        }
        const int herr = *h_err;
        if (herr != 0) {
            cuda_ok(cudaMemset(d_err, 0, sizeof(int)), "clear error word");
            if (herr >= 101 && herr <= 103) {
                unusable = true;
                fail(ADAI_B200_ERR_TIMEOUT, "a kernel gave up waiting (code " +
                                                std::to_string(herr) + ")" + last_work());
            }
            fail(ADAI_B200_ERR_OUT_OF_RANGE,
                 "a kernel rejected its input (code " + std::to_string(herr) + ")" + last_work());
        }
    }

    // ------------------------------------------------------------------------------------------
    void ensure_gemm_scratch(const GemmPlan& p) {
        const size_t ws = gemm_ws_floats(p);
        const int tk = p.m_tiles * p.n_tiles;
        const size_t ar = gemm_arg_rows(p);
        if (ws > gs.ws_floats || tk > gs.n_tickets || ar > gs.arg_rows) {
            cuda_ok(cudaStreamSynchronize(stream), "sync before scratch growth");
            clear_graphs();
            if (ws > gs.ws_floats) {
                dfree(gs.ws);
                gs.ws_floats = std::max(ws, gs.ws_floats * 2);
                gs.ws = dalloc_t<float>(gs.ws_floats);
            }
            if (tk > gs.n_tickets) {
                dfree(gs.tickets);
                gs.n_tickets = std::max(tk, 1024);
                gs.tickets = dzalloc_t<int>(gs.n_tickets);
            }
            if (ar > gs.arg_rows) {
                dfree(gs.arg_key);
                dfree(gs.arg_nf);
                gs.arg_rows = std::max(ar, gs.arg_rows * 2);
                gs.arg_key = dzalloc_t<unsigned long long>(gs.arg_rows);
                gs.arg_nf = dzalloc_t<int>(gs.arg_rows);
            }
        }
    }
    void ensure_attn_scratch(int B, int H, int max_len, int dh) {
        // the decode step's cross-attention uses the shorter chunk: the most partials per row
        const size_t f = decode_attn_ws_floats(B, H, max_len, dh, kAttnChunkShort);
        const int tk = B * H;
        if (f > attn_ws_floats || tk > attn_n_tickets) {
            cuda_ok(cudaStreamSynchronize(stream), "sync before scratch growth");
            clear_graphs();
            if (f > attn_ws_floats) {
                dfree(attn_ws);
                attn_ws_floats = f;
                attn_ws = dalloc_t<float>(f);
            }
            if (tk > attn_n_tickets) {
                dfree(attn_tickets);
                attn_n_tickets = tk;
                attn_tickets = dzalloc_t<int>(tk);
            }
        }
    }

    void ensure_sample_park(size_t floats) {
        if (floats <= samp_park_floats) return;
        cuda_ok(cudaStreamSynchronize(stream), "sync before scratch growth");
        clear_graphs();
        dfree(samp_park);
        samp_park = dalloc_t<float>(floats);
        samp_park_floats = floats;
    }

    void gemm(const TcActs& a, int M, const TcWeight& w, const GemmEpilogue& e,
              const char* what = "gemm_3xtf32_kernel") {
        const GemmPlan p = gemm_plan(M, w.N, w.K, e.flags, num_sms);
        ensure_gemm_scratch(p);
        note(what);
        launch_ok(gemm_launch(a, M, w, e, p, gs, d_err, stream), "gemm launch");
    }
};

namespace {

// Runs `fn` (which enqueues launches on the context stream) between two recorded events when a
// profiled step is being recorded; otherwise just runs it.
template <class Fn>
void timed(adai_b200_ctx* c, int cls, double bytes, double flops, Fn&& fn) {
    if (!c->prof) {
        fn();
        return;
    }
    Span sp{};
    sp.cls = cls;
    sp.bytes = bytes;
    sp.flops = flops;
    cuda_ok(cudaEventCreate(&sp.a), "cudaEventCreate");
    cuda_ok(cudaEventCreate(&sp.b), "cudaEventCreate");
    cuda_ok(cudaEventRecord(sp.a, c->stream), "cudaEventRecord");
    fn();
    cuda_ok(cudaEventRecord(sp.b, c->stream), "cudaEventRecord");
    c->prof->spans.push_back(sp);
}

// guarded() for an entry point that queues GPU work: its phase tag and NVTX range around `fn`,
// and with ADAI_B200_SYNC=step or kernel a bounded wait for that work before it returns.
template <class Fn>
int traced(adai_b200_ctx* c, const char* phase, Fn&& fn) {
    return guarded([&] {
        adai_b200_trace::PhaseScope ps(c ? &c->trace : nullptr, phase);
        fn();
        if (c && !c->unusable && adai_b200_trace::settings().mode != adai_b200_trace::kSyncOff)
            c->sync(wait_timeout_seconds());
    });
}

double gemm_bytes(double M, double N, double K) { return 4.0 * (M * K + K * N + M * N); }
double gemm_flops(double M, double N, double K) { return 2.0 * M * N * K; }

// ---------------------------------------------------------------------------------------------
// Model upload
TcWeight make_tc_weight(adai_b200_ctx* c, std::vector<void*>& owned, int K, int N) {
    TcWeight w;
    w.K = K;
    w.N = N;
    const size_t rows = static_cast<size_t>(round_up(N, 256));
    w.hi = c->dzalloc_t<float>(rows * K);
    w.lo = c->dzalloc_t<float>(rows * K);
    owned.push_back(w.hi);
    owned.push_back(w.lo);
    return w;
}

// Transposes + splits host W [K, Nsub] into rows [row0, row0+Nsub) of w (W^T layout).
void fill_tc_weight(adai_b200_ctx* c, float* staging, const TcWeight& w, int row0, const float* host,
                    int K, int Nsub) {
    const size_t bytes = static_cast<size_t>(K) * Nsub * sizeof(float);
    cuda_ok(cudaMemcpyAsync(staging, host, bytes, cudaMemcpyHostToDevice, c->stream), "upload");
    c->note("transpose_split_kernel");
    launch_transpose_split(staging, K, Nsub, w.hi + static_cast<size_t>(row0) * K,
                           w.lo + static_cast<size_t>(row0) * K, c->stream);
    cuda_ok(cudaGetLastError(), "transpose-split");
    cuda_ok(cudaStreamSynchronize(c->stream), "upload sync");  // staging is reused
}

// Folds the LayerNorm (gamma g, beta b, both [K]) that precedes W [K, N] into it, in place:
// W <- diag(g) W, c1[n] = sum_k (diag(g) W)[k][n], bias[n] = sum_k b[k] W[k][n] (+ extra[n]),
// the sums in double over the fp32 products the GEMM multiplies.
__global__ void fold_layernorm_kernel(float* __restrict__ w, int K, int N, const float* __restrict__ g,
                                      const float* __restrict__ b, const float* __restrict__ extra,
                                      float* __restrict__ c1, float* __restrict__ bias) {
    const int n = blockIdx.x * blockDim.x + threadIdx.x;
    if (n >= N) return;
    double s1 = 0.0, s0 = extra ? static_cast<double>(extra[n]) : 0.0;
    for (int k = 0; k < K; ++k) {
        float* p = w + static_cast<size_t>(k) * N + n;
        const float wk = *p;
        const float ws = g[k] * wk;
        *p = ws;
        s1 += static_cast<double>(ws);
        s0 += static_cast<double>(b[k]) * static_cast<double>(wk);
    }
    c1[n] = static_cast<float>(s1);
    bias[n] = static_cast<float>(s0);
}

// fill_tc_weight for a W that a LayerNorm (g, b on the device) precedes: see
// fold_layernorm_kernel; c1 / bias receive columns [row0, row0 + Nsub).
void fill_tc_weight_folded(adai_b200_ctx* c, float* staging, const TcWeight& w, int row0,
                           const float* host, int K, int Nsub, const float* g, const float* b,
                           const float* extra, float* c1, float* bias) {
    const size_t bytes = static_cast<size_t>(K) * Nsub * sizeof(float);
    cuda_ok(cudaMemcpyAsync(staging, host, bytes, cudaMemcpyHostToDevice, c->stream), "upload");
    c->note("fold_layernorm_kernel");
    fold_layernorm_kernel<<<(Nsub + 127) / 128, 128, 0, c->stream>>>(staging, K, Nsub, g, b, extra,
                                                                     c1 + row0, bias + row0);
    cuda_ok(cudaGetLastError(), "fold-layernorm");
    c->note("transpose_split_kernel");
    launch_transpose_split(staging, K, Nsub, w.hi + static_cast<size_t>(row0) * K,
                           w.lo + static_cast<size_t>(row0) * K, c->stream);
    cuda_ok(cudaGetLastError(), "transpose-split");
    cuda_ok(cudaStreamSynchronize(c->stream), "upload sync");  // staging is reused
}

float* upload_vec(adai_b200_ctx* c, std::vector<void*>& owned, const float* host, size_t n) {
    float* d = c->dalloc_t<float>(n);
    owned.push_back(d);
    cuda_ok(cudaMemcpyAsync(d, host, n * sizeof(float), cudaMemcpyHostToDevice, c->stream),
            "upload");
    return d;
}

float* alloc_vec(adai_b200_ctx* c, std::vector<void*>& owned, size_t n) {
    float* d = c->dzalloc_t<float>(n);
    owned.push_back(d);
    return d;
}

void free_model(adai_b200_ctx* c) {
    if (!c->model) return;
    cudaStreamSynchronize(c->stream);
    for (void* p : c->model->owned) c->dfree(p);
    c->model.reset();
    c->clear_graphs();
}

void validate_desc(const adai_b200_model_desc* d) {
    if (!d) fail(ADAI_B200_ERR_INVALID_ARGUMENT, "null model description");
    if (d->vocab <= 0 || d->d_model <= 0 || d->n_heads <= 0 || d->d_ff <= 0 ||
        d->enc_layers < 0 || d->dec_layers <= 0 || d->max_seq <= 0)
        fail(ADAI_B200_ERR_INVALID_ARGUMENT, "model dimensions must be positive");
    if (d->d_model % d->n_heads || !attention_head_dim_supported(d->d_model / d->n_heads))
        fail(ADAI_B200_ERR_INVALID_ARGUMENT, "d_model / n_heads must be 32 or 64 (head widths of the attention kernels)");
    if (!layernorm_width_supported(d->d_model))
        fail(ADAI_B200_ERR_INVALID_ARGUMENT, "d_model must be 128 * {1,2,3,4,6,8,12,16}");
    if (d->d_ff % 16 || d->vocab % 4)
        fail(ADAI_B200_ERR_INVALID_ARGUMENT, "d_ff must be a multiple of 16 and vocab of 4");
}

int tensor_count(const adai_b200_model_desc* d) {
    return 1 + 12 * d->enc_layers + 2 + 1 + 18 * d->dec_layers + 2 + 2;
}

// PositionalEncoding table, src/PositionalEncoding.cpp:13-32.
std::vector<float> pe_table_host(int max_len, int D) {
    std::vector<float> t(static_cast<size_t>(max_len) * D);
    for (int pos = 0; pos < max_len; ++pos)
        for (int i = 0; i < D; ++i) {
            const float angle = static_cast<float>(pos) /
                                std::pow(10000.0f, (2.0f * static_cast<float>(i / 2)) / static_cast<float>(D));
            t[static_cast<size_t>(pos) * D + i] = (i % 2 == 0) ? std::sin(angle) : std::cos(angle);
        }
    return t;
}

// ---------------------------------------------------------------------------------------------
void ensure_step_bufs(adai_b200_ctx* c, int rows_needed) {
    const Model& m = *c->model;
    const int R = round_up(std::max(rows_needed, 1), 128);
    if (c->sb.rows >= R) return;
    cuda_ok(cudaStreamSynchronize(c->stream), "sync");
    c->clear_graphs();
    StepBufs& s = c->sb;
    // slots / ids and next / nonfinite_any are two allocations each (see below)
    for (void* p : {(void*)s.x, (void*)s.nrm_hi, (void*)s.nrm_lo, (void*)s.qkv, (void*)s.attn_hi,
                    (void*)s.attn_lo, (void*)s.qc, (void*)s.h_hi, (void*)s.h_lo, (void*)s.logits,
                    (void*)s.slots, (void*)s.next, (void*)s.nonfinite, (void*)s.ln_stats})
        c->dfree(p);
    const size_t D = m.d.d_model, F = m.d.d_ff, V = m.d.vocab;
    s.rows = R;
    s.x = c->dzalloc_t<float>(R * D);
    s.nrm_hi = c->dzalloc_t<float>(R * D);
    s.nrm_lo = c->dzalloc_t<float>(R * D);
    s.qkv = c->dzalloc_t<float>(R * 3 * D);
    s.attn_hi = c->dzalloc_t<float>(R * D);
    s.attn_lo = c->dzalloc_t<float>(R * D);
    s.qc = c->dzalloc_t<float>(R * D);
    s.h_hi = c->dzalloc_t<float>(R * F);
    s.h_lo = c->dzalloc_t<float>(R * F);
    s.logits = c->dzalloc_t<float>(R * V);
    // [slots R | ids R] and [next R | nonfinite_any]: one copy each way per decode step
    s.slots = c->dzalloc_t<int>(2 * static_cast<size_t>(R));
    s.ids = s.slots + R;
    s.next = c->dzalloc_t<int>(R + 1);
    s.nonfinite_any = s.next + R;
    s.nonfinite = c->dzalloc_t<int>(R);
    s.ln_stats = c->dzalloc_t<float2>(R * (D / 32));
}

void ensure_enc_bufs(adai_b200_ctx* c) {
    if (c->eb.rows) return;
    const Model& m = *c->model;
    const int R = kEncRows;
    EncBufs& e = c->eb;
    const size_t D = m.d.d_model, F = m.d.d_ff;
    e.rows = R;
    e.x = c->dzalloc_t<float>(R * D);
    e.nrm_hi = c->dzalloc_t<float>(R * D);
    e.nrm_lo = c->dzalloc_t<float>(R * D);
    e.qkv = c->dzalloc_t<float>(R * 3 * D);
    e.attn_hi = c->dzalloc_t<float>(R * D);
    e.attn_lo = c->dzalloc_t<float>(R * D);
    e.h_hi = c->dzalloc_t<float>(R * F);
    e.h_lo = c->dzalloc_t<float>(R * F);
    e.out = c->dzalloc_t<float>(R * D);
    e.ids = c->dzalloc_t<int>(R);
    e.row_slot = c->dzalloc_t<int>(R);
    e.row_pos = c->dzalloc_t<int>(R);
    e.offsets = c->dzalloc_t<int>(R);
    e.lens = c->dzalloc_t<int>(R);
    if (prefill_tc_supported(D / m.d.n_heads)) {
        e.ldv = 2 * R + 32;  // sequences start on 32-column boundaries: at most 31 padding each
        e.qkv_hi = c->dzalloc_t<float>(R * 3 * D);
        e.qkv_lo = c->dzalloc_t<float>(R * 3 * D);
        e.vt_hi = c->dzalloc_t<float>(D * static_cast<size_t>(e.ldv));
        e.vt_lo = c->dzalloc_t<float>(D * static_cast<size_t>(e.ldv));
        e.row_vcol = c->dzalloc_t<int>(R);
        e.seq_vcol = c->dzalloc_t<int>(R);
    }
}

void free_enc_bufs(adai_b200_ctx* c) {
    EncBufs& e = c->eb;
    for (void* p : {(void*)e.x, (void*)e.nrm_hi, (void*)e.nrm_lo, (void*)e.qkv, (void*)e.attn_hi,
                    (void*)e.attn_lo, (void*)e.h_hi, (void*)e.h_lo, (void*)e.out, (void*)e.ids,
                    (void*)e.row_slot, (void*)e.row_pos, (void*)e.offsets, (void*)e.lens,
                    (void*)e.qkv_hi, (void*)e.qkv_lo, (void*)e.vt_hi, (void*)e.vt_lo,
                    (void*)e.row_vcol, (void*)e.seq_vcol})
        c->dfree(p);
    e = EncBufs{};
}

void free_step_bufs(adai_b200_ctx* c) {
    StepBufs& s = c->sb;
    // slots / ids and next / nonfinite_any are two allocations each (see below)
    for (void* p : {(void*)s.x, (void*)s.nrm_hi, (void*)s.nrm_lo, (void*)s.qkv, (void*)s.attn_hi,
                    (void*)s.attn_lo, (void*)s.qc, (void*)s.h_hi, (void*)s.h_lo, (void*)s.logits,
                    (void*)s.slots, (void*)s.next, (void*)s.nonfinite, (void*)s.ln_stats})
        c->dfree(p);
    s = StepBufs{};
}

TcActs acts(const float* hi, const float* lo, int K, int rows_alloc) {
    TcActs a;
    a.hi = hi;
    a.lo = lo;
    a.K = K;
    a.rows_alloc = rows_alloc;
    return a;
}

SampleArgs sample_args(adai_b200_ctx* c, adai_b200_kv* kv, int B, const float* logits, int ld,
                       const int* fed, int* next, int* nonfinite) {
    SampleArgs a;
    a.logits = logits;
    a.ld = ld;
    a.slots = c->sb.slots;
    a.fed = fed;
    a.next = next;
    a.nonfinite = nonfinite;
    a.cfg = kv->d_samp;
    a.mt = kv->d_mt;
    a.seen = kv->d_seen;
    a.seen_words = kv->seen_words;
    a.new_tokens = kv->d_new_tokens;
    a.scratch = c->samp_park;
    a.B = B;
    a.V = c->model->d.vocab;
    return a;
}

// Enqueues one stacked decode step for rows 0..B-1 of the step buffers (ids in sb.ids, slots in
// sb.slots). The graph captured from this is replayed by decode_step / generate.
void record_step(adai_b200_ctx* c, adai_b200_kv* kv, int B, int flags) {
    const Model& m = *c->model;
    StepBufs& s = c->sb;
    const int D = m.d.d_model, F = m.d.d_ff, H = m.d.n_heads, L = m.d.dec_layers;
    const int R = s.rows;
    const float scale = 1.0f / std::sqrt(static_cast<float>(D / H));
    cudaStream_t st = c->stream;
    const double Bd = B, Dd = D, Fd = F;
    // Every LayerNorm is folded into the GEMM that consumes it (kEpiLnFold): the kernels that
    // write the residual stream x also write its tf32 split (into nrm_hi / nrm_lo) and its
    // per-32-column group statistics (kEpiRowStats), from which that GEMM takes mean and rstd.
    const double ln_bytes = 3.0 * Bd * Dd * 4.0;
    timed(c, ADAI_B200_KC_NORM, ln_bytes, 0, [&] {
        c->note("embed_stats_kernel");
        launch_embed_stats(m.dec_embed, s.ids, m.pe, m.d.max_seq, s.slots, kv->d_self_len, s.x,
                           s.nrm_hi, s.nrm_lo, s.ln_stats, B, D, m.d.vocab, c->d_err, st);
    });
    auto ln_fold = [&](GemmEpilogue& e, const float* c1, const float* bias) {
        e.flags |= kEpiLnFold | kEpiBias;
        e.ln_c1 = c1;
        e.bias = bias;
        e.row_stats = s.ln_stats;
        e.stats_ld = R;
    };
    auto x_stats = [&](GemmEpilogue& e) {  // x written: also its split and group statistics
        e.flags |= kEpiSplit | kEpiRowStats;
        e.out_hi = s.nrm_hi;
        e.out_lo = s.nrm_lo;
        e.lds = D;
        e.row_stats = s.ln_stats;
        e.stats_ld = R;
    };
    const double self_bytes = c->prof ? (2.0 * c->prof->sum_self_rows * Dd * 4.0 + 4.0 * Bd * Dd * 4.0) : 0;
    const double cross_bytes = c->prof ? (2.0 * c->prof->sum_cross_rows * Dd * 4.0 + 2.0 * Bd * Dd * 4.0) : 0;
    const TcActs a_nrm = acts(s.nrm_hi, s.nrm_lo, D, R);
    const TcActs a_attn = acts(s.attn_hi, s.attn_lo, D, R);
    const TcActs a_h = acts(s.h_hi, s.h_lo, F, R);
    for (int l = 0; l < L; ++l) {
        const DecLayerW& w = m.dec[l];
        {  // Q|K|V of the new token
            GemmEpilogue e;
            e.flags = kEpiStore;
            e.out = s.qkv;
            e.ldo = 3 * D;
            ln_fold(e, w.qkv_c1, w.qkv_bias);
            timed(c, ADAI_B200_KC_GEMM, gemm_bytes(Bd, 3 * Dd, Dd), gemm_flops(Bd, 3 * Dd, Dd),
                  [&] { c->gemm(a_nrm, B, w.qkv, e, "gemm_3xtf32_kernel (decoder self Q|K|V)"); });
        }
        {  // masked self-attention over the cache, the new K/V appended first
            DecodeAttnArgs a;
            a.q = s.qkv;
            a.ldq = 3 * D;
            a.k_new = s.qkv + D;
            a.v_new = s.qkv + 2 * D;
            a.ldkv = 3 * D;
            a.kc = kv->self_k_layer(l);
            a.vc = kv->self_v_layer(l);
            a.slot_stride = kv->self_slot_stride();
            a.cap = kv->self_cap;
            a.slots = s.slots;
            a.len_by_slot = kv->d_self_len;
            a.len_add = 1;
            a.out_hi = s.attn_hi;
            a.out_lo = s.attn_lo;
            a.ldo = D;
            a.B = B;
            a.H = H;
            a.head_dim = D / H;
            a.max_len = kv->self_cap;
            a.scale = scale;
            a.ws = c->attn_ws;
            a.tickets = c->attn_tickets;
            timed(c, ADAI_B200_KC_SELF_ATTN, self_bytes, 0, [&] {
                c->note("decode_attention_kernel (self, append)");
                launch_decode_attention(a, c->d_err, st);
            });
        }
        {  // x = x + attn W_o
            GemmEpilogue e;
            e.flags = kEpiStore | kEpiResid;
            e.resid = s.x;
            e.ldr = D;
            e.out = s.x;
            e.ldo = D;
            x_stats(e);
            timed(c, ADAI_B200_KC_GEMM, gemm_bytes(Bd, Dd, Dd), gemm_flops(Bd, Dd, Dd),
                  [&] { c->gemm(a_attn, B, w.o, e, "gemm_3xtf32_kernel (decoder self W_o)"); });
        }
        {  // cross-attention query of LN2(x)
            GemmEpilogue e;
            e.flags = kEpiStore;
            e.out = s.qc;
            e.ldo = D;
            ln_fold(e, w.cq_c1, w.cq_bias);
            timed(c, ADAI_B200_KC_GEMM, gemm_bytes(Bd, Dd, Dd), gemm_flops(Bd, Dd, Dd),
                  [&] { c->gemm(a_nrm, B, w.cq, e, "gemm_3xtf32_kernel (decoder cross Q)"); });
        }
        {
            DecodeAttnArgs a;
            a.q = s.qc;
            a.ldq = D;
            a.kc = kv->cross_k_layer(l);
            a.vc = kv->cross_v_layer(l);
            a.slot_stride = kv->cross_slot_stride();
            a.cap = kv->cross_cap;
            a.slots = s.slots;
            a.len_by_slot = kv->d_cross_len;
            a.len_add = 0;
            a.chunk = kAttnChunkShort;  // 128-row chunks: more CTAs over the longer source rows
            a.out_hi = s.attn_hi;
            a.out_lo = s.attn_lo;
            a.ldo = D;
            a.B = B;
            a.H = H;
            a.head_dim = D / H;
            a.max_len = kv->cross_cap;
            a.scale = scale;
            a.ws = c->attn_ws;
            a.tickets = c->attn_tickets;
            timed(c, ADAI_B200_KC_CROSS_ATTN, cross_bytes, 0, [&] {
                c->note("decode_attention_kernel (cross)");
                launch_decode_attention(a, c->d_err, st);
            });
        }
        {
            GemmEpilogue e;
            e.flags = kEpiStore | kEpiResid;
            e.resid = s.x;
            e.ldr = D;
            e.out = s.x;
            e.ldo = D;
            x_stats(e);
            timed(c, ADAI_B200_KC_GEMM, gemm_bytes(Bd, Dd, Dd), gemm_flops(Bd, Dd, Dd),
                  [&] { c->gemm(a_attn, B, w.co, e, "gemm_3xtf32_kernel (decoder cross W_o)"); });
        }
        {  // h = GELU(LN3(x) W1 + b1), written as its tf32 split for the next GEMM
            GemmEpilogue e;
            e.flags = kEpiGelu | kEpiSplit;
            e.out_hi = s.h_hi;
            e.out_lo = s.h_lo;
            e.lds = F;
            ln_fold(e, w.w1_c1, w.w1_bias);
            timed(c, ADAI_B200_KC_GEMM, gemm_bytes(Bd, Fd, Dd), gemm_flops(Bd, Fd, Dd),
                  [&] { c->gemm(a_nrm, B, w.w1, e, "gemm_3xtf32_kernel (decoder FFN W1)"); });
        }
        {  // x = x + (h W2 + b2)
            GemmEpilogue e;
            e.flags = kEpiBias | kEpiResid | kEpiStore;
            e.bias = w.b2;
            e.resid = s.x;
            e.ldr = D;
            e.out = s.x;
            e.ldo = D;
            x_stats(e);
            timed(c, ADAI_B200_KC_GEMM, gemm_bytes(Bd, Dd, Fd), gemm_flops(Bd, Dd, Fd),
                  [&] { c->gemm(a_h, B, w.w2, e, "gemm_3xtf32_kernel (decoder FFN W2)"); });
        }
    }
    {  // logits = x W_out + b, first maximum per row
        GemmEpilogue e;
        e.flags = kEpiArgmax | ((flags & (kStepLogits | kStepSample)) ? kEpiStore : 0);
        ln_fold(e, m.head_c1, m.head_bias);  // the decoder's final LayerNorm
        e.out = s.logits;
        e.ldo = m.d.vocab;
        e.next_ids = s.next;
        e.nonfinite = s.nonfinite;
        const double Vd = m.d.vocab;
        timed(c, ADAI_B200_KC_HEAD, 4.0 * (Bd * Dd + Dd * Vd), gemm_flops(Bd, Vd, Dd),
              [&] { c->gemm(a_nrm, B, m.head, e, "gemm_3xtf32_kernel (LM head + argmax)"); });
    }
    if (flags & kStepSample) {  // rows whose slot samples replace the argmax (sample.cu)
        const SampleArgs a = sample_args(c, kv, B, s.logits, m.d.vocab, s.ids, s.next, s.nonfinite);
        timed(c, ADAI_B200_KC_OTHER, 4.0 * Bd * m.d.vocab, 0, [&] {
            c->note("sample_rows_kernel");
            cuda_ok(launch_sample_rows(a, st), "sample launch");
        });
    }
}

__global__ void record_and_advance_kernel(const int* __restrict__ next, int* __restrict__ ids,
                                          const int* __restrict__ slots, int* __restrict__ self_len,
                                          int* __restrict__ hist, int hist_ld,
                                          const int* __restrict__ nonfinite, int* __restrict__ nf_any,
                                          int B, int feed_back) {
    pdl_trigger();
    pdl_wait();
    const int b = blockIdx.x * blockDim.x + threadIdx.x;
    if (b >= B) return;
    const int slot = slots[b];
    const int pos = self_len[slot];
    if (hist) hist[static_cast<size_t>(slot) * hist_ld + pos] = next[b];
    if (nonfinite[b]) atomicOr(nf_any, 1);
    if (feed_back) ids[b] = next[b];
    self_len[slot] = pos + 1;
}

// Sizes the scratch a decode step of B rows needs (allocation cannot happen inside a capture).
void presize_step_scratch(adai_b200_ctx* c, adai_b200_kv* kv, int B, int flags) {
    const Model& m = *c->model;
    if (flags & kStepSample) c->ensure_sample_park(static_cast<size_t>(B) * m.d.vocab);
    const int D = m.d.d_model, F = m.d.d_ff;
    for (const auto& sh : {std::make_tuple(3 * D, D, 0), std::make_tuple(D, D, 0),
                           std::make_tuple(F, D, 0), std::make_tuple(D, F, 0),
                           std::make_tuple(m.d.vocab, D, (int)kEpiArgmax)})
        c->ensure_gemm_scratch(gemm_plan(B, std::get<0>(sh), std::get<1>(sh), std::get<2>(sh), c->num_sms));
    c->ensure_attn_scratch(B, m.d.n_heads, std::max(kv->self_cap, kv->cross_cap), kv->dh);
}

cudaGraphExec_t get_graph(adai_b200_ctx* c, adai_b200_kv* kv, int B, int flags) {
    const GraphKey key{kv, B, flags};
    auto it = c->graphs.find(key);
    if (it != c->graphs.end()) return it->second;
    presize_step_scratch(c, kv, B, flags);
    cuda_ok(cudaStreamSynchronize(c->stream), "sync before capture");
    cudaGraph_t g;
    cuda_ok(cudaStreamBeginCapture(c->stream, cudaStreamCaptureModeThreadLocal), "begin capture");
    try {
        // The step's kernels overlap their prologues with the previous kernel's tail (PDL edges
        // in the graph); each waits for its predecessor before touching data.
        ScopedPdl pdl(true);
        record_step(c, kv, B, flags);
        cuda_ok(launch_kernel(record_and_advance_kernel, dim3((B + 127) / 128), dim3(128), 0,
                              c->stream, c->sb.next, c->sb.ids, c->sb.slots, kv->d_self_len,
                              kv->d_hist, kv->self_cap, c->sb.nonfinite, c->sb.nonfinite_any, B,
                              (flags & kStepAdvanceIds) ? 1 : 0),
                "advance launch");
    } catch (...) {
        cudaGraph_t dummy;
        cudaStreamEndCapture(c->stream, &dummy);
        if (dummy) cudaGraphDestroy(dummy);
        throw;
    }
    cuda_ok(cudaStreamEndCapture(c->stream, &g), "end capture");
    size_t n_nodes = 0;
    cuda_ok(cudaGraphGetNodes(g, nullptr, &n_nodes), "graph nodes");
    c->graph_kernels[key] = static_cast<int>(n_nodes);
    cudaGraphExec_t ge;
    cuda_ok(cudaGraphInstantiate(&ge, g, 0), "graph instantiate");
    cudaGraphDestroy(g);
    c->graphs[key] = ge;
    return ge;
}

// Queues one decode step: replays the step's CUDA graph, or, with ADAI_B200_SYNC=kernel, queues
// its kernels one by one without a graph so that each launch is waited for and named.
void run_step(adai_b200_ctx* c, adai_b200_kv* kv, int B, int flags) {
    if (adai_b200_trace::settings().mode != adai_b200_trace::kSyncKernel) {
        cudaGraphExec_t g = get_graph(c, kv, B, flags);
        c->note("decode step (CUDA graph)");
        cuda_ok(cudaGraphLaunch(g, c->stream), "graph launch");
        return;
    }
    presize_step_scratch(c, kv, B, flags);
    record_step(c, kv, B, flags);
    c->note("record_and_advance_kernel");
    record_and_advance_kernel<<<(B + 127) / 128, 128, 0, c->stream>>>(
        c->sb.next, c->sb.ids, c->sb.slots, kv->d_self_len, kv->d_hist, kv->self_cap,
        c->sb.nonfinite, c->sb.nonfinite_any, B, (flags & kStepAdvanceIds) ? 1 : 0);
    cuda_ok(cudaGetLastError(), "advance launch");
}

void check_ctx(adai_b200_ctx* c) {
    if (!c) fail(ADAI_B200_ERR_INVALID_ARGUMENT, "null context");
    c->check_usable();
    cuda_ok(cudaSetDevice(c->device), "cudaSetDevice");
}

void check_kv(adai_b200_ctx* c, adai_b200_kv* kv) {
    if (!kv || !c->kvs.count(kv)) fail(ADAI_B200_ERR_INVALID_ARGUMENT, "unknown KV arena");
}

void check_model(adai_b200_ctx* c) {
    if (!c->model) fail(ADAI_B200_ERR_STATE, "no model uploaded");
}

// kStepSample when a row of the batch belongs to a slot configured for sampling.
int sample_flag(const adai_b200_kv* kv, int B, const int* slots) {
    if (kv->samp_on.empty()) return 0;
    for (int b = 0; b < B; ++b)
        if (kv->samp_on[slots[b]]) return kStepSample;
    return 0;
}

// Validates the batch of a decode step and stages slots/ids into the step buffers.
void stage_batch(adai_b200_ctx* c, adai_b200_kv* kv, int B, const int* slots, const int* ids,
                 int steps) {
    if (B <= 0 || B > kv->max_slots)
        fail(ADAI_B200_ERR_INVALID_ARGUMENT, "batch must be in [1, max_slots]");
    if (!slots || !ids) fail(ADAI_B200_ERR_INVALID_ARGUMENT, "null slots or ids");
    std::vector<char> seen(kv->max_slots, 0);
    for (int b = 0; b < B; ++b) {
        const int s = slots[b];
        if (s < 0 || s >= kv->max_slots)
            fail(ADAI_B200_ERR_OUT_OF_RANGE, "slot " + std::to_string(s) + " out of range");
        if (seen[s]) fail(ADAI_B200_ERR_INVALID_ARGUMENT, "slot " + std::to_string(s) + " repeated in one batch");
        seen[s] = 1;
        if (!kv->encoded[s])
            fail(ADAI_B200_ERR_STATE, "slot " + std::to_string(s) + " has no encoder output (call adai_b200_encode first)");
        if (kv->self_len[s] + steps > kv->self_cap)
            fail(ADAI_B200_ERR_OUT_OF_RANGE, "self-attention cache of slot " + std::to_string(s) +
                                                 " full (capacity " + std::to_string(kv->self_cap) + ")");
        if (ids[b] < 0 || ids[b] >= c->model->d.vocab)
            fail(ADAI_B200_ERR_OUT_OF_RANGE, "Token ID " + std::to_string(ids[b]) + " out of range [0, " +
                                                 std::to_string(c->model->d.vocab) + ")");
    }
    ensure_step_bufs(c, B);
    // slots into [0, B), ids into [R, R + B) of the [slots R | ids R] block, in one copy
    const size_t R = static_cast<size_t>(c->sb.rows);
    int* pin = c->pinned(R + B);
    std::memcpy(pin, slots, B * sizeof(int));
    std::memcpy(pin + R, ids, B * sizeof(int));
    cuda_ok(cudaMemcpyAsync(c->sb.slots, pin, (R + B) * sizeof(int), cudaMemcpyHostToDevice, c->stream),
            "H2D slots and ids");
}

}  // namespace

// =============================================================================================
// C ABI
extern "C" {

const char* adai_b200_last_error(void) { return g_last_error.c_str(); }

int adai_b200_ctx_create(int device, float mem_fraction, adai_b200_ctx** out) {
    return guarded([&] {
        if (!out) fail(ADAI_B200_ERR_INVALID_ARGUMENT, "null output handle");
        *out = nullptr;
        int n = 0;
        if (cudaGetDeviceCount(&n) != cudaSuccess || n == 0)
            fail(ADAI_B200_ERR_NO_DEVICE, "no CUDA device");
        if (device < 0 || device >= n) fail(ADAI_B200_ERR_OUT_OF_RANGE, "device index out of range");
        if (mem_fraction < 0.f || mem_fraction > 1.f)
            fail(ADAI_B200_ERR_INVALID_ARGUMENT, "mem_fraction must be in [0, 1]");
        cudaDeviceProp prop;
        cuda_ok(cudaGetDeviceProperties(&prop, device), "cudaGetDeviceProperties");
        if (prop.major != 10)
            fail(ADAI_B200_ERR_NO_DEVICE, std::string("device ") + prop.name +
                                              " is not sm_100 (this library is built for sm_100a only)");
        if (!tensor_map_api_available())
            fail(ADAI_B200_ERR_NO_DEVICE, "cuTensorMapEncodeTiled unavailable in the driver");
        cuda_ok(cudaSetDevice(device), "cudaSetDevice");
        auto c = std::make_unique<adai_b200_ctx>();
        c->device = device;
        c->num_sms = prop.multiProcessorCount;
        if (mem_fraction > 0.f) c->mem_cap = static_cast<size_t>(static_cast<double>(prop.totalGlobalMem) * mem_fraction);
        cuda_ok(cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking), "cudaStreamCreate");
        c->d_err = c->dzalloc_t<int>(1);
        cuda_ok(cudaHostAlloc(reinterpret_cast<void**>(&c->h_err), sizeof(int), cudaHostAllocDefault),
                "cudaHostAlloc");
        *c->h_err = 0;
        cuda_ok(cudaEventCreateWithFlags(&c->sync_ev, cudaEventDisableTiming), "cudaEventCreate");
        cuda_ok(cudaStreamSynchronize(c->stream), "sync");
        *out = c.release();
    });
}

int adai_b200_ctx_destroy(adai_b200_ctx* c) {
    return guarded([&] {
        if (!c) return;
        cudaSetDevice(c->device);
        cudaStreamSynchronize(c->stream);
        c->clear_graphs();
        for (auto& kvp : c->allocs) cudaFree(kvp.first);
        c->allocs.clear();
        for (adai_b200_kv* kv : c->kvs) delete kv;
        c->kvs.clear();
        if (c->h_pin) cudaFreeHost(c->h_pin);
        if (c->h_err) cudaFreeHost(c->h_err);
        if (c->sync_ev) cudaEventDestroy(c->sync_ev);
        cudaStreamDestroy(c->stream);
        delete c;
    });
}

int adai_b200_ctx_synchronize(adai_b200_ctx* c, double timeout_seconds) {
    return guarded([&] {
        check_ctx(c);
        c->sync(timeout_seconds > 0 ? timeout_seconds : wait_timeout_seconds());
    });
}

int adai_b200_ctx_check_wait_timeout(adai_b200_ctx* c, double* waited_seconds) {
    return traced(c, "adai_b200_ctx_check_wait_timeout", [&] {
        check_ctx(c);
        int* gave_up = c->dzalloc_t<int>(1);
        const auto t0 = std::chrono::steady_clock::now();
        try {
            c->note("wait_selftest_kernel");
            launch_wait_selftest(c->d_err, gave_up, c->stream);
            cuda_ok(cudaGetLastError(), "wait self-test launch");
            int h = 0;
            cuda_ok(cudaMemcpyAsync(&h, gave_up, sizeof(int), cudaMemcpyDeviceToHost, c->stream), "D2H");
            c->sync(wait_timeout_seconds());  // reads the error word: fails with the timeout
            fail(ADAI_B200_ERR_STATE, "the device wait did not report its timeout (gave_up " +
                                          std::to_string(h) + ")");
        } catch (...) {
            if (waited_seconds)
                *waited_seconds = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
            c->dfree(gave_up);
            throw;
        }
    });
}

int adai_b200_ctx_last_work(adai_b200_ctx* c, char* buf, int buf_len, unsigned long long* launches) {
    return guarded([&] {
        if (!c) fail(ADAI_B200_ERR_INVALID_ARGUMENT, "null context");
        if (launches) *launches = c->trace.seq.load(std::memory_order_relaxed);
        if (buf && buf_len > 0) {
            const std::string w = c->trace.describe();
            const size_t n = std::min(w.size(), static_cast<size_t>(buf_len - 1));
            std::memcpy(buf, w.data(), n);
            buf[n] = '\0';
        }
    });
}

int adai_b200_debug_sync_parse(const char* value, int* mode, unsigned* every) {
    return guarded([&] {
        if (!mode || !every) fail(ADAI_B200_ERR_INVALID_ARGUMENT, "null output");
        std::string problem;
        if (!adai_b200_trace::parse_sync(value, mode, every, &problem))
            fail(ADAI_B200_ERR_INVALID_ARGUMENT, problem);
    });
}

int adai_b200_debug_configure(int mode, unsigned every, const char* trace_file) {
    return guarded([&] {
        if (mode < adai_b200_trace::kSyncOff || mode > adai_b200_trace::kSyncKernel)
            fail(ADAI_B200_ERR_INVALID_ARGUMENT, "mode must be 0 (off), 1 (step) or 2 (kernel)");
        if (every < 1 || every > 1000000)
            fail(ADAI_B200_ERR_INVALID_ARGUMENT, "every must be in [1, 1000000]");
        adai_b200_trace::Settings st;
        st.mode = mode;
        st.every = every;
        if (trace_file) st.trace_file = trace_file;
        adai_b200_trace::set_settings(st);
    });
}

int adai_b200_debug_settings(int* mode, unsigned* every) {
    return guarded([&] {
        if (!mode || !every) fail(ADAI_B200_ERR_INVALID_ARGUMENT, "null output");
        const adai_b200_trace::Settings& st = adai_b200_trace::settings();
        *mode = st.mode;
        *every = st.every;
    });
}

int adai_b200_ctx_memory(adai_b200_ctx* c, unsigned long long* bytes) {
    return guarded([&] {
        if (!c || !bytes) fail(ADAI_B200_ERR_INVALID_ARGUMENT, "null argument");
        *bytes = c->mem_used;
    });
}

void* adai_b200_ctx_stream(adai_b200_ctx* c) { return c ? static_cast<void*>(c->stream) : nullptr; }

int adai_b200_model_tensor_count(const adai_b200_model_desc* d) { return d ? tensor_count(d) : -1; }

int adai_b200_model_upload(adai_b200_ctx* c, const adai_b200_model_desc* d,
                           const float* const* t, const float* pe_table) {
    return traced(c, "adai_b200_model_upload", [&] {
        check_ctx(c);
        validate_desc(d);
        if (!t) fail(ADAI_B200_ERR_INVALID_ARGUMENT, "null tensor list");
        for (int i = 0; i < tensor_count(d); ++i)
            if (!t[i]) fail(ADAI_B200_ERR_INVALID_ARGUMENT, "tensor " + std::to_string(i) + " is null");
        for (adai_b200_kv* kv : c->kvs)
            if (kv->L != d->dec_layers || kv->H != d->n_heads)
                fail(ADAI_B200_ERR_STATE, "an existing KV arena does not match this model");
        for (adai_b200_kv* kv : c->kvs)  // sampling state is per vocabulary: slots go back to argmax
            if (kv->samp_vocab != d->vocab) std::fill(kv->samp_on.begin(), kv->samp_on.end(), 0);
        free_model(c);
        free_enc_bufs(c);
        free_step_bufs(c);
        auto m = std::make_unique<Model>();
        m->d = *d;
        const int V = d->vocab, D = d->d_model, F = d->d_ff;
        auto& own = m->owned;
        const size_t max_mat = std::max<size_t>({static_cast<size_t>(V) * D, static_cast<size_t>(D) * F});
        float* staging = c->dalloc_t<float>(max_mat);
        try {
            int k = 0;
            m->enc_embed = upload_vec(c, own, t[k++], static_cast<size_t>(V) * D);
            m->enc.resize(d->enc_layers);
            for (int i = 0; i < d->enc_layers; ++i) {
                EncLayerW& e = m->enc[i];
                e.ln1g = upload_vec(c, own, t[k++], D);
                e.ln1b = upload_vec(c, own, t[k++], D);
                e.qkv = make_tc_weight(c, own, D, 3 * D);
                fill_tc_weight(c, staging, e.qkv, 0, t[k++], D, D);
                fill_tc_weight(c, staging, e.qkv, D, t[k++], D, D);
                fill_tc_weight(c, staging, e.qkv, 2 * D, t[k++], D, D);
                e.o = make_tc_weight(c, own, D, D);
                fill_tc_weight(c, staging, e.o, 0, t[k++], D, D);
                e.ln2g = upload_vec(c, own, t[k++], D);
                e.ln2b = upload_vec(c, own, t[k++], D);
                e.w1 = make_tc_weight(c, own, D, F);
                fill_tc_weight(c, staging, e.w1, 0, t[k++], D, F);
                e.b1 = upload_vec(c, own, t[k++], F);
                e.w2 = make_tc_weight(c, own, F, D);
                fill_tc_weight(c, staging, e.w2, 0, t[k++], F, D);
                e.b2 = upload_vec(c, own, t[k++], D);
            }
            m->enc_lnf_g = upload_vec(c, own, t[k++], D);
            m->enc_lnf_b = upload_vec(c, own, t[k++], D);
            m->dec_embed = upload_vec(c, own, t[k++], static_cast<size_t>(V) * D);
            m->dec.resize(d->dec_layers);
            for (int i = 0; i < d->dec_layers; ++i) {
                DecLayerW& w = m->dec[i];
                w.ln1g = upload_vec(c, own, t[k++], D);
                w.ln1b = upload_vec(c, own, t[k++], D);
                w.qkv = make_tc_weight(c, own, D, 3 * D);
                w.qkv_c1 = alloc_vec(c, own, 3 * D);
                w.qkv_bias = alloc_vec(c, own, 3 * D);
                for (int j = 0; j < 3; ++j)
                    fill_tc_weight_folded(c, staging, w.qkv, j * D, t[k++], D, D, w.ln1g, w.ln1b,
                                          nullptr, w.qkv_c1, w.qkv_bias);
                w.o = make_tc_weight(c, own, D, D);
                fill_tc_weight(c, staging, w.o, 0, t[k++], D, D);
                w.ln2g = upload_vec(c, own, t[k++], D);
                w.ln2b = upload_vec(c, own, t[k++], D);
                w.cq = make_tc_weight(c, own, D, D);
                w.cq_c1 = alloc_vec(c, own, D);
                w.cq_bias = alloc_vec(c, own, D);
                fill_tc_weight_folded(c, staging, w.cq, 0, t[k++], D, D, w.ln2g, w.ln2b, nullptr,
                                      w.cq_c1, w.cq_bias);
                w.ckv = make_tc_weight(c, own, D, 2 * D);
                fill_tc_weight(c, staging, w.ckv, 0, t[k++], D, D);
                fill_tc_weight(c, staging, w.ckv, D, t[k++], D, D);
                w.co = make_tc_weight(c, own, D, D);
                fill_tc_weight(c, staging, w.co, 0, t[k++], D, D);
                w.ln3g = upload_vec(c, own, t[k++], D);
                w.ln3b = upload_vec(c, own, t[k++], D);
                w.w1 = make_tc_weight(c, own, D, F);
                const float* w1_host = t[k++];
                w.b1 = upload_vec(c, own, t[k++], F);
                w.w1_c1 = alloc_vec(c, own, F);
                w.w1_bias = alloc_vec(c, own, F);
                fill_tc_weight_folded(c, staging, w.w1, 0, w1_host, D, F, w.ln3g, w.ln3b, w.b1,
                                      w.w1_c1, w.w1_bias);
                w.w2 = make_tc_weight(c, own, F, D);
                fill_tc_weight(c, staging, w.w2, 0, t[k++], F, D);
                w.b2 = upload_vec(c, own, t[k++], D);
            }
            m->dec_lnf_g = upload_vec(c, own, t[k++], D);
            m->dec_lnf_b = upload_vec(c, own, t[k++], D);
            m->head = make_tc_weight(c, own, D, V);
            const float* head_host = t[k++];
            m->head_b = upload_vec(c, own, t[k++], V);
            m->head_c1 = alloc_vec(c, own, V);
            m->head_bias = alloc_vec(c, own, V);
            fill_tc_weight_folded(c, staging, m->head, 0, head_host, D, V, m->dec_lnf_g,
                                  m->dec_lnf_b, m->head_b, m->head_c1, m->head_bias);
            std::vector<float> pe;
            if (!pe_table) {
                pe = pe_table_host(d->max_seq, D);
                pe_table = pe.data();
            }
            m->pe = upload_vec(c, own, pe_table, static_cast<size_t>(d->max_seq) * D);
            cuda_ok(cudaStreamSynchronize(c->stream), "upload sync");
        } catch (...) {
            c->dfree(staging);
            for (void* p : own) c->dfree(p);
            throw;
        }
        c->dfree(staging);
        c->model = std::move(m);
    });
}

int adai_b200_checkpoint_config(const char* dir, adai_b200_model_desc* out) {
    return guarded([&] {
        if (!dir || !out) fail(ADAI_B200_ERR_INVALID_ARGUMENT, "null argument");
        *out = read_checkpoint_config(dir);
    });
}

int adai_b200_checkpoint_special_tokens(const char* path, int* bos, int* eos, int* pad) {
    return guarded([&] {
        if (!path) fail(ADAI_B200_ERR_INVALID_ARGUMENT, "null argument");
        int b = 0, e = 0, p = 0;
        read_checkpoint_special_tokens(path, &b, &e, &p);
        if (bos) *bos = b;
        if (eos) *eos = e;
        if (pad) *pad = p;
    });
}

int adai_b200_checkpoint_read(const char* dir, const adai_b200_model_desc* d, float* const* t) {
    return guarded([&] {
        if (!dir || !t) fail(ADAI_B200_ERR_INVALID_ARGUMENT, "null argument");
        validate_desc(d);
        const int n = tensor_count(d);
        std::vector<float*> out(t, t + n);
        for (int i = 0; i < n; ++i)
            if (!out[i]) fail(ADAI_B200_ERR_INVALID_ARGUMENT, "tensor " + std::to_string(i) + " is null");
        read_checkpoint_tensors(dir, *d, out);
    });
}

int adai_b200_model_load(adai_b200_ctx* c, const char* dir, const adai_b200_model_desc* expect) {
    return traced(c, "adai_b200_model_load", [&] {
        check_ctx(c);
        if (!dir) fail(ADAI_B200_ERR_INVALID_ARGUMENT, "null checkpoint directory");
        const adai_b200_model_desc d = read_checkpoint_config(dir);
        if (expect && std::memcmp(expect, &d, sizeof d) != 0)
            fail(ADAI_B200_ERR_INVALID_ARGUMENT,
                 "architecture mismatch between the checkpoint " + std::string(dir) + " (vocab " +
                     std::to_string(d.vocab) + ", d_model " + std::to_string(d.d_model) + ", heads " +
                     std::to_string(d.n_heads) + ", d_ff " + std::to_string(d.d_ff) + ", layers " +
                     std::to_string(d.enc_layers) + "+" + std::to_string(d.dec_layers) +
                     ", max_length " + std::to_string(d.max_seq) + ") and the expected model");
        validate_desc(&d);
        const std::vector<size_t> sizes = upload_tensor_sizes(d);
        std::vector<std::vector<float>> host(sizes.size());
        std::vector<float*> ptr(sizes.size());
        for (size_t i = 0; i < sizes.size(); ++i) {
            host[i].resize(sizes[i]);
            ptr[i] = host[i].data();
        }
        read_checkpoint_tensors(dir, d, ptr);
        std::vector<const float*> cptr(ptr.begin(), ptr.end());
        const int rc = adai_b200_model_upload(c, &d, cptr.data(), nullptr);
        if (rc != ADAI_B200_OK) fail(rc, g_last_error);
    });
}

int adai_b200_kv_create(adai_b200_ctx* c, int max_slots, int self_cap, int cross_cap,
                        adai_b200_kv** out) {
    return traced(c, "adai_b200_kv_create", [&] {
        check_ctx(c);
        check_model(c);
        if (!out) fail(ADAI_B200_ERR_INVALID_ARGUMENT, "null output handle");
        if (max_slots <= 0 || self_cap <= 0 || cross_cap <= 0)
            fail(ADAI_B200_ERR_INVALID_ARGUMENT, "KV arena sizes must be positive");
        const Model& m = *c->model;
        auto kv = std::make_unique<adai_b200_kv>();
        kv->max_slots = max_slots;
        kv->self_cap = self_cap;
        kv->cross_cap = cross_cap;
        kv->L = m.d.dec_layers;
        kv->H = m.d.n_heads;
        kv->dh = m.d.d_model / m.d.n_heads;
        const size_t self_n = static_cast<size_t>(kv->L) * max_slots * kv->self_slot_stride();
        const size_t cross_n = static_cast<size_t>(kv->L) * max_slots * kv->cross_slot_stride();
        std::vector<void*> got;
        try {
            kv->self_k = c->dalloc_t<float>(self_n);
            got.push_back(kv->self_k);
            kv->self_v = c->dalloc_t<float>(self_n);
            got.push_back(kv->self_v);
            kv->cross_k = c->dalloc_t<float>(cross_n);
            got.push_back(kv->cross_k);
            kv->cross_v = c->dalloc_t<float>(cross_n);
            got.push_back(kv->cross_v);
            kv->d_self_len = c->dzalloc_t<int>(max_slots);
            got.push_back(kv->d_self_len);
            kv->d_cross_len = c->dzalloc_t<int>(max_slots);
            got.push_back(kv->d_cross_len);
            kv->d_hist = c->dzalloc_t<int>(static_cast<size_t>(max_slots) * self_cap);
            got.push_back(kv->d_hist);
        } catch (...) {
            for (void* p : got) c->dfree(p);
            throw;
        }
        kv->self_len.assign(max_slots, 0);
        kv->cross_len.assign(max_slots, 0);
        kv->encoded.assign(max_slots, 0);
        cuda_ok(cudaStreamSynchronize(c->stream), "sync");
        c->kvs.insert(kv.get());
        *out = kv.release();
    });
}

int adai_b200_kv_destroy(adai_b200_ctx* c, adai_b200_kv* kv) {
    return guarded([&] {
        if (!c) fail(ADAI_B200_ERR_INVALID_ARGUMENT, "null context");
        check_kv(c, kv);
        cudaSetDevice(c->device);
        cudaStreamSynchronize(c->stream);
        c->clear_graphs();
        for (void* p : {(void*)kv->self_k, (void*)kv->self_v, (void*)kv->cross_k,
                        (void*)kv->cross_v, (void*)kv->d_self_len, (void*)kv->d_cross_len,
                        (void*)kv->d_hist, (void*)kv->d_samp, (void*)kv->d_mt, (void*)kv->d_seen,
                        (void*)kv->d_new_tokens})
            c->dfree(p);
        c->kvs.erase(kv);
        delete kv;
    });
}

int adai_b200_kv_reset(adai_b200_ctx* c, adai_b200_kv* kv, int slot) {
    return traced(c, "adai_b200_kv_reset", [&] {
        check_ctx(c);
        check_kv(c, kv);
        if (slot < 0 || slot >= kv->max_slots) fail(ADAI_B200_ERR_OUT_OF_RANGE, "slot out of range");
        kv->self_len[slot] = 0;
        kv->cross_len[slot] = 0;
        kv->encoded[slot] = 0;
        cuda_ok(cudaMemsetAsync(kv->d_self_len + slot, 0, sizeof(int), c->stream), "memset");
        cuda_ok(cudaMemsetAsync(kv->d_cross_len + slot, 0, sizeof(int), c->stream), "memset");
        if (kv->d_samp) {  // back to the fused argmax
            kv->samp_on[slot] = 0;
            cuda_ok(cudaMemsetAsync(kv->d_samp + slot, 0, sizeof(SampleSlot), c->stream), "memset");
        }
        c->sync(wait_timeout_seconds());
    });
}

int adai_b200_kv_clear_self(adai_b200_ctx* c, adai_b200_kv* kv, int slot) {
    return traced(c, "adai_b200_kv_clear_self", [&] {
        check_ctx(c);
        check_kv(c, kv);
        if (slot < 0 || slot >= kv->max_slots) fail(ADAI_B200_ERR_OUT_OF_RANGE, "slot out of range");
        kv->self_len[slot] = 0;
        cuda_ok(cudaMemsetAsync(kv->d_self_len + slot, 0, sizeof(int), c->stream), "memset");
        c->sync(wait_timeout_seconds());
    });
}

int adai_b200_kv_length(adai_b200_ctx* c, adai_b200_kv* kv, int slot, int* self_len,
                        int* cross_len) {
    return guarded([&] {
        if (!c) fail(ADAI_B200_ERR_INVALID_ARGUMENT, "null context");
        check_kv(c, kv);
        if (slot < 0 || slot >= kv->max_slots) fail(ADAI_B200_ERR_OUT_OF_RANGE, "slot out of range");
        if (self_len) *self_len = kv->self_len[slot];
        if (cross_len) *cross_len = kv->cross_len[slot];
    });
}

int adai_b200_encode(adai_b200_ctx* c, adai_b200_kv* kv, int n, const int* slots, const int* ids,
                     const int* src_lens, float* enc_out) {
    return traced(c, "adai_b200_encode", [&] {
        check_ctx(c);
        check_model(c);
        check_kv(c, kv);
        const Model& m = *c->model;
        if (n <= 0 || !slots || !ids || !src_lens) fail(ADAI_B200_ERR_INVALID_ARGUMENT, "empty or null request list");
        std::vector<char> seen(kv->max_slots, 0);
        long long total = 0;
        for (int i = 0; i < n; ++i) {
            if (slots[i] < 0 || slots[i] >= kv->max_slots) fail(ADAI_B200_ERR_OUT_OF_RANGE, "slot out of range");
            if (seen[slots[i]]) fail(ADAI_B200_ERR_INVALID_ARGUMENT, "slot repeated in one encode call");
            seen[slots[i]] = 1;
            // No lower bound, as in the reference: an empty source has no encoder rows, and
            // cross-attention over no rows contributes zeros.
            if (src_lens[i] < 0) fail(ADAI_B200_ERR_INVALID_ARGUMENT, "negative source length");
            // LLMEncoder::encode_with_mask refuses more than max_seq_length ids (src/LLMEncoder.cpp:106-116)
            if (src_lens[i] > m.d.max_seq)
                fail(ADAI_B200_ERR_INVALID_ARGUMENT, std::to_string(src_lens[i]) + " tokens exceed max_seq_length " + std::to_string(m.d.max_seq));
            if (src_lens[i] > kv->cross_cap) fail(ADAI_B200_ERR_OUT_OF_RANGE, "source longer than the cross-attention cache");
            total += src_lens[i];
        }
        for (long long r = 0; r < total; ++r)
            if (ids[r] < 0 || ids[r] >= m.d.vocab)
                fail(ADAI_B200_ERR_OUT_OF_RANGE, "Token ID " + std::to_string(ids[r]) + " out of range [0, " + std::to_string(m.d.vocab) + ")");
        ensure_enc_bufs(c);
        EncBufs& e = c->eb;
        const int D = m.d.d_model, F = m.d.d_ff, H = m.d.n_heads;
        const float scale = 1.0f / std::sqrt(static_cast<float>(D / H));
        cudaStream_t st = c->stream;
        long long row_base = 0;
        int i0 = 0;
        while (i0 < n) {
            int i1 = i0, rows = 0;
            while (i1 < n && rows + src_lens[i1] <= e.rows) rows += src_lens[i1++];
            if (i1 == i0)
                fail(ADAI_B200_ERR_INVALID_ARGUMENT, "a source of " + std::to_string(src_lens[i0]) +
                                                         " ids exceeds the encoder's row buffer");
            const int nseq = i1 - i0;
            if (rows == 0) {  // only empty sources in this chunk: nothing to compute
                for (int i = i0; i < i1; ++i) {
                    kv->cross_len[slots[i]] = 0;
                    kv->self_len[slots[i]] = 0;
                    kv->encoded[slots[i]] = 1;
                }
                i0 = i1;
                continue;
            }
            int max_len = 0;
            int* pin = c->pinned(static_cast<size_t>(rows) * 4 + 3 * static_cast<size_t>(nseq));
            int* p_ids = pin;
            int* p_slot = pin + rows;
            int* p_pos = pin + 2 * rows;
            int* p_vcol = pin + 3 * rows;
            int* p_off = pin + 4 * rows;
            int* p_len = p_off + nseq;
            int* p_svcol = p_len + nseq;
            int r = 0, vcol = 0;
            for (int i = i0; i < i1; ++i) {
                p_off[i - i0] = r;
                p_len[i - i0] = src_lens[i];
                p_svcol[i - i0] = vcol;
                max_len = std::max(max_len, src_lens[i]);
                for (int t = 0; t < src_lens[i]; ++t, ++r) {
                    p_ids[r] = ids[row_base + r];
                    p_slot[r] = slots[i];
                    p_pos[r] = t;
                    p_vcol[r] = vcol + t;
                }
                vcol = round_up(vcol + src_lens[i], 32);
            }
            // The tensor-core attention needs every sequence's transposed V to start on a
            // 32-column boundary; a chunk of very many short sources may not fit its buffer.
            const bool tc_attn = e.vt_hi != nullptr && vcol <= e.ldv;
            if (tc_attn) {
                cuda_ok(cudaMemcpyAsync(e.row_vcol, p_vcol, rows * sizeof(int), cudaMemcpyHostToDevice, st), "H2D");
                cuda_ok(cudaMemcpyAsync(e.seq_vcol, p_svcol, nseq * sizeof(int), cudaMemcpyHostToDevice, st), "H2D");
            }
            cuda_ok(cudaMemcpyAsync(e.ids, p_ids, rows * sizeof(int), cudaMemcpyHostToDevice, st), "H2D");
            cuda_ok(cudaMemcpyAsync(e.row_slot, p_slot, rows * sizeof(int), cudaMemcpyHostToDevice, st), "H2D");
            cuda_ok(cudaMemcpyAsync(e.row_pos, p_pos, rows * sizeof(int), cudaMemcpyHostToDevice, st), "H2D");
            cuda_ok(cudaMemcpyAsync(e.offsets, p_off, nseq * sizeof(int), cudaMemcpyHostToDevice, st), "H2D");
            cuda_ok(cudaMemcpyAsync(e.lens, p_len, nseq * sizeof(int), cudaMemcpyHostToDevice, st), "H2D");
            const int Le = m.d.enc_layers;
            c->note("embed_ln_kernel");
            launch_embed_ln(m.enc_embed, e.ids, m.pe, m.d.max_seq, nullptr, nullptr, e.row_pos, e.x,
                            Le ? m.enc[0].ln1g : m.enc_lnf_g, Le ? m.enc[0].ln1b : m.enc_lnf_b,
                            e.nrm_hi, e.nrm_lo, rows, D, m.d.vocab, c->d_err, st);
            if (Le == 0) {  // the embedding row LayerNorm'd by final_norm is the encoder output
                c->note("layernorm_kernel (encoder final)");
                launch_layernorm(e.x, D, m.enc_lnf_g, m.enc_lnf_b, e.out, e.nrm_hi, e.nrm_lo, rows, D, st);
            }
            const TcActs a_nrm = acts(e.nrm_hi, e.nrm_lo, D, e.rows);
            const TcActs a_attn = acts(e.attn_hi, e.attn_lo, D, e.rows);
            const TcActs a_h = acts(e.h_hi, e.h_lo, F, e.rows);
            for (int l = 0; l < Le; ++l) {
                const EncLayerW& w = m.enc[l];
                GemmEpilogue q;
                q.flags = kEpiStore;
                q.out = e.qkv;
                q.ldo = 3 * D;
                c->gemm(a_nrm, rows, w.qkv, q, "gemm_3xtf32_kernel (encoder Q|K|V)");
                if (tc_attn) {
                    PrefillTcArgs pa;
                    pa.qkv = e.qkv;
                    pa.qkv_hi = e.qkv_hi;
                    pa.qkv_lo = e.qkv_lo;
                    pa.vt_hi = e.vt_hi;
                    pa.vt_lo = e.vt_lo;
                    pa.ldv = e.ldv;
                    pa.row_vcol = e.row_vcol;
                    pa.seq_vcol = e.seq_vcol;
                    pa.offsets = e.offsets;
                    pa.lens = e.lens;
                    pa.nseq = nseq;
                    pa.max_len = max_len;
                    pa.rows = rows;
                    pa.D = D;
                    pa.head_dim = D / H;
                    pa.out_hi = e.attn_hi;
                    pa.out_lo = e.attn_lo;
                    pa.scale = scale;
                    pa.err = c->d_err;
                    c->note("prefill_attention_tc_kernel");
                    launch_ok(launch_prefill_attention_tc(pa, st), "prefill attention launch");
                } else {
                    c->note("prefill_attention_kernel");
                    launch_prefill_attention(e.qkv, D, H, e.offsets, e.lens, nseq, max_len, e.attn_hi,
                                             e.attn_lo, scale, st);
                }
                GemmEpilogue o;
                o.flags = kEpiStore | kEpiResid;
                o.resid = e.x;
                o.ldr = D;
                o.out = e.x;
                o.ldo = D;
                c->gemm(a_attn, rows, w.o, o, "gemm_3xtf32_kernel (encoder W_o)");
                c->note("layernorm_kernel (encoder LN2)");
                launch_layernorm(e.x, D, w.ln2g, w.ln2b, nullptr, e.nrm_hi, e.nrm_lo, rows, D, st);
                GemmEpilogue f1;
                f1.flags = kEpiBias | kEpiGelu | kEpiSplit;
                f1.bias = w.b1;
                f1.out_hi = e.h_hi;
                f1.out_lo = e.h_lo;
                f1.lds = F;
                c->gemm(a_nrm, rows, w.w1, f1, "gemm_3xtf32_kernel (encoder FFN W1)");
                GemmEpilogue f2;
                f2.flags = kEpiBias | kEpiResid | kEpiStore;
                f2.bias = w.b2;
                f2.resid = e.x;
                f2.ldr = D;
                f2.out = e.x;
                f2.ldo = D;
                c->gemm(a_h, rows, w.w2, f2, "gemm_3xtf32_kernel (encoder FFN W2)");
                const bool last = l + 1 == Le;
                c->note("layernorm_kernel (encoder LN1 / final)");
                launch_layernorm(e.x, D, last ? m.enc_lnf_g : m.enc[l + 1].ln1g,
                                 last ? m.enc_lnf_b : m.enc[l + 1].ln1b, last ? e.out : nullptr,
                                 e.nrm_hi, e.nrm_lo, rows, D, st);
            }
            // Cross-attention K/V of every decoder layer, scattered into the slot's cache rows.
            for (int l = 0; l < m.d.dec_layers; ++l) {
                GemmEpilogue s;
                s.flags = kEpiKvScatter;
                s.kc = kv->cross_k_layer(l);
                s.vc = kv->cross_v_layer(l);
                s.slot_stride = kv->cross_slot_stride();
                s.cap = kv->cross_cap;
                s.head_dim = D / H;
                s.d_model = D;
                s.row_slot = e.row_slot;
                s.row_pos = e.row_pos;
                c->gemm(a_nrm, rows, m.dec[l].ckv, s, "gemm_3xtf32_kernel (cross K|V scatter)");
            }
            if (enc_out)
                cuda_ok(cudaMemcpyAsync(enc_out + row_base * D, e.out, static_cast<size_t>(rows) * D * sizeof(float),
                                        cudaMemcpyDeviceToHost, st), "D2H encoder output");
            for (int i = i0; i < i1; ++i) {
                kv->cross_len[slots[i]] = src_lens[i];
                kv->self_len[slots[i]] = 0;
                kv->encoded[slots[i]] = 1;
            }
            c->sync(wait_timeout_seconds());
            row_base += rows;
            i0 = i1;
        }
        // Device copies of the per-slot lengths.
        int* pin = c->pinned(2 * static_cast<size_t>(kv->max_slots));
        std::memcpy(pin, kv->self_len.data(), kv->max_slots * sizeof(int));
        std::memcpy(pin + kv->max_slots, kv->cross_len.data(), kv->max_slots * sizeof(int));
        cuda_ok(cudaMemcpyAsync(kv->d_self_len, pin, kv->max_slots * sizeof(int), cudaMemcpyHostToDevice, st), "H2D");
        cuda_ok(cudaMemcpyAsync(kv->d_cross_len, pin + kv->max_slots, kv->max_slots * sizeof(int), cudaMemcpyHostToDevice, st), "H2D");
        c->sync(wait_timeout_seconds());
    });
}

int adai_b200_decode_step(adai_b200_ctx* c, adai_b200_kv* kv, int B, const int* slots,
                          const int* ids, int* next_ids, float* logits) {
    return traced(c, "adai_b200_decode_step", [&] {
        check_ctx(c);
        check_model(c);
        check_kv(c, kv);
        if (!next_ids) fail(ADAI_B200_ERR_INVALID_ARGUMENT, "null next_ids");
        stage_batch(c, kv, B, slots, ids, 1);
        const int flags = (logits ? kStepLogits : 0) | sample_flag(kv, B, slots);
        cuda_ok(cudaMemsetAsync(c->sb.nonfinite_any, 0, sizeof(int), c->stream), "memset");
        run_step(c, kv, B, flags);
        // next ids and the non-finite flag: [next R | flag], one copy
        const size_t R = static_cast<size_t>(c->sb.rows);
        int* pin = c->pinned(R + 1);
        cuda_ok(cudaMemcpyAsync(pin, c->sb.next, (R + 1) * sizeof(int), cudaMemcpyDeviceToHost, c->stream),
                "D2H ids and flag");
        if (logits)
            cuda_ok(cudaMemcpyAsync(logits, c->sb.logits, static_cast<size_t>(B) * c->model->d.vocab * sizeof(float),
                                    cudaMemcpyDeviceToHost, c->stream), "D2H logits");
        c->sync(wait_timeout_seconds());
        for (int b = 0; b < B; ++b) kv->self_len[slots[b]] += 1;
        std::memcpy(next_ids, pin, B * sizeof(int));
        if (pin[R]) fail(ADAI_B200_ERR_NONFINITE, "the model returned non-finite logits");
    });
}

int adai_b200_generate(adai_b200_ctx* c, adai_b200_kv* kv, int B, const int* slots,
                       const int* first_ids, int steps, int* out_ids) {
    return traced(c, "adai_b200_generate", [&] {
        check_ctx(c);
        check_model(c);
        check_kv(c, kv);
        if (steps <= 0 || !out_ids) fail(ADAI_B200_ERR_INVALID_ARGUMENT, "steps must be positive, out_ids non-null");
        stage_batch(c, kv, B, slots, first_ids, steps);
        std::vector<int> pos0(B);
        for (int b = 0; b < B; ++b) pos0[b] = kv->self_len[slots[b]];
        const int flags = kStepAdvanceIds | sample_flag(kv, B, slots);
        if (adai_b200_trace::settings().mode != adai_b200_trace::kSyncKernel)
            get_graph(c, kv, B, flags);  // captured before the timed region
        cuda_ok(cudaMemsetAsync(c->sb.nonfinite_any, 0, sizeof(int), c->stream), "memset");
        cudaEvent_t e0, e1;
        cuda_ok(cudaEventCreate(&e0), "cudaEventCreate");
        cuda_ok(cudaEventCreate(&e1), "cudaEventCreate");
        cuda_ok(cudaEventRecord(e0, c->stream), "cudaEventRecord");
        for (int s = 0; s < steps; ++s) run_step(c, kv, B, flags);
        cuda_ok(cudaEventRecord(e1, c->stream), "cudaEventRecord");
        c->sync(wait_timeout_seconds() + 1e-3 * steps);
        float ms = 0.f;
        cuda_ok(cudaEventElapsedTime(&ms, e0, e1), "cudaEventElapsedTime");
        cudaEventDestroy(e0);
        cudaEventDestroy(e1);
        c->last_decode_ms = ms;
        const auto gk = c->graph_kernels.find(GraphKey{kv, B, flags});
        c->last_kernels_per_step = gk != c->graph_kernels.end() ? gk->second : 0;
        for (int b = 0; b < B; ++b) kv->self_len[slots[b]] += steps;
        int nf = 0;
        cuda_ok(cudaMemcpy(&nf, c->sb.nonfinite_any, sizeof(int), cudaMemcpyDeviceToHost), "D2H flag");
        for (int b = 0; b < B; ++b)
            cuda_ok(cudaMemcpy(out_ids + static_cast<size_t>(b) * steps,
                               kv->d_hist + static_cast<size_t>(slots[b]) * kv->self_cap + pos0[b],
                               steps * sizeof(int), cudaMemcpyDeviceToHost), "D2H ids");
        if (nf) fail(ADAI_B200_ERR_NONFINITE, "the model returned non-finite logits");
    });
}

}  // extern "C"

// ---- sampling ----------------------------------------------------------------------------------
namespace {

// std::mt19937(seed): the published MT19937 initialisation; the read position starts past the
// end, so the first draw refreshes the state (as the standard engine does).
void mt_seed_host(unsigned seed, unsigned* st) {
    st[0] = seed;
    for (unsigned i = 1; i < 624; ++i) st[i] = 1812433253u * (st[i - 1] ^ (st[i - 1] >> 30)) + i;
    st[624] = 624;
}

void ensure_kv_sampling(adai_b200_ctx* c, adai_b200_kv* kv) {
    const int V = c->model->d.vocab;
    if (kv->d_samp && kv->samp_vocab == V) return;
    cuda_ok(cudaStreamSynchronize(c->stream), "sync");
    c->clear_graphs();
    for (void* p : {(void*)kv->d_samp, (void*)kv->d_mt, (void*)kv->d_seen, (void*)kv->d_new_tokens})
        c->dfree(p);
    kv->d_samp = nullptr;
    kv->d_mt = kv->d_seen = nullptr;
    kv->d_new_tokens = nullptr;
    const size_t n = kv->max_slots;
    kv->seen_words = (V + 31) / 32;
    kv->d_samp = c->dzalloc_t<SampleSlot>(n);
    kv->d_mt = c->dzalloc_t<unsigned>(n * kMtWords);
    kv->d_seen = c->dzalloc_t<unsigned>(n * kv->seen_words);
    kv->d_new_tokens = c->dzalloc_t<int>(n);
    kv->samp_vocab = V;
    kv->samp_on.assign(n, 0);
}

void check_slot(const adai_b200_kv* kv, int slot) {
    if (slot < 0 || slot >= kv->max_slots)
        fail(ADAI_B200_ERR_OUT_OF_RANGE, "slot " + std::to_string(slot) + " out of range");
}

}  // namespace

extern "C" {

int adai_b200_kv_set_sampling(adai_b200_ctx* c, adai_b200_kv* kv, int slot,
                              const adai_b200_sampling* cfg, const int* history, int n_history) {
    return traced(c, "adai_b200_kv_set_sampling", [&] {
        check_ctx(c);
        check_model(c);
        check_kv(c, kv);
        check_slot(kv, slot);
        if (!cfg) {
            if (kv->d_samp) {
                kv->samp_on[slot] = 0;
                cuda_ok(cudaMemsetAsync(kv->d_samp + slot, 0, sizeof(SampleSlot), c->stream), "memset");
                c->sync(wait_timeout_seconds());
            }
            return;
        }
        if (n_history < 0 || (n_history > 0 && !history))
            fail(ADAI_B200_ERR_INVALID_ARGUMENT, "history must hold n_history >= 0 ids");
        if (!std::isfinite(cfg->temperature) || !std::isfinite(cfg->top_p))
            fail(ADAI_B200_ERR_INVALID_ARGUMENT, "temperature and top_p must be finite");
        if (!std::isfinite(cfg->repetition_penalty) || !(cfg->repetition_penalty > 0.0f))
            fail(ADAI_B200_ERR_INVALID_ARGUMENT, "repetition_penalty must be finite and positive");
        const int V = c->model->d.vocab;
        if (V > sample_max_vocab())
            fail(ADAI_B200_ERR_INVALID_ARGUMENT, "vocabulary of " + std::to_string(V) +
                                                     " exceeds the device sampler's " +
                                                     std::to_string(sample_max_vocab()));
        ensure_kv_sampling(c, kv);
        SampleSlot h;
        h.temperature = cfg->temperature;
        h.top_p = cfg->top_p;
        h.penalty = cfg->repetition_penalty;
        h.top_k = cfg->top_k;
        h.min_length = cfg->min_length;
        h.eos = cfg->eos_token_id;
        h.pad = cfg->pad_token_id;
        h.enabled = 1;
        const unsigned seed = cfg->seed ? cfg->seed : std::random_device{}();
        std::vector<unsigned> mt(kMtWords, 0u);
        mt_seed_host(seed, mt.data());
        std::vector<unsigned> seen(kv->seen_words, 0u);
        for (int i = 0; i < n_history; ++i)
            if (history[i] >= 0 && history[i] < V) seen[history[i] >> 5] |= 1u << (history[i] & 31);
        cudaStream_t st = c->stream;
        cuda_ok(cudaMemcpyAsync(kv->d_samp + slot, &h, sizeof(h), cudaMemcpyHostToDevice, st), "H2D");
        cuda_ok(cudaMemcpyAsync(kv->d_mt + static_cast<size_t>(slot) * kMtWords, mt.data(),
                                kMtWords * sizeof(unsigned), cudaMemcpyHostToDevice, st), "H2D");
        cuda_ok(cudaMemcpyAsync(kv->d_seen + static_cast<size_t>(slot) * kv->seen_words, seen.data(),
                                seen.size() * sizeof(unsigned), cudaMemcpyHostToDevice, st), "H2D");
        cuda_ok(cudaMemsetAsync(kv->d_new_tokens + slot, 0, sizeof(int), st), "memset");
        c->sync(wait_timeout_seconds());
        kv->samp_on[slot] = 1;
    });
}

int adai_b200_kv_sampling_state(adai_b200_ctx* c, adai_b200_kv* kv, int slot, unsigned* mt_state,
                                int* new_tokens) {
    return traced(c, "adai_b200_kv_sampling_state", [&] {
        check_ctx(c);
        check_kv(c, kv);
        check_slot(kv, slot);
        if (kv->samp_on.empty() || !kv->samp_on[slot])
            fail(ADAI_B200_ERR_STATE, "slot " + std::to_string(slot) + " is not configured for sampling");
        c->sync(wait_timeout_seconds());
        if (mt_state)
            cuda_ok(cudaMemcpy(mt_state, kv->d_mt + static_cast<size_t>(slot) * kMtWords,
                               625 * sizeof(unsigned), cudaMemcpyDeviceToHost), "D2H");
        if (new_tokens)
            cuda_ok(cudaMemcpy(new_tokens, kv->d_new_tokens + slot, sizeof(int), cudaMemcpyDeviceToHost), "D2H");
    });
}

int adai_b200_sample_logits(adai_b200_ctx* c, adai_b200_kv* kv, int B, const int* slots,
                            const int* fed_ids, const float* logits, int ld, int* next_ids) {
    return traced(c, "adai_b200_sample_logits", [&] {
        check_ctx(c);
        check_model(c);
        check_kv(c, kv);
        const int V = c->model->d.vocab;
        if (B <= 0 || B > kv->max_slots) fail(ADAI_B200_ERR_INVALID_ARGUMENT, "batch must be in [1, max_slots]");
        if (!slots || !logits || !next_ids || ld < V)
            fail(ADAI_B200_ERR_INVALID_ARGUMENT, "need slots, logits with ld >= vocab, next_ids");
        std::vector<char> dup(kv->max_slots, 0);
        for (int b = 0; b < B; ++b) {
            check_slot(kv, slots[b]);
            if (dup[slots[b]]) fail(ADAI_B200_ERR_INVALID_ARGUMENT, "slot repeated in one batch");
            dup[slots[b]] = 1;
            if (kv->samp_on.empty() || !kv->samp_on[slots[b]])
                fail(ADAI_B200_ERR_STATE, "slot " + std::to_string(slots[b]) + " is not configured for sampling");
            if (fed_ids && (fed_ids[b] < 0 || fed_ids[b] >= V))
                fail(ADAI_B200_ERR_OUT_OF_RANGE, "Token ID " + std::to_string(fed_ids[b]) + " out of range");
        }
        if (kv->samp_vocab != V) fail(ADAI_B200_ERR_STATE, "sampling state was made for another vocabulary");
        ensure_step_bufs(c, B);
        c->ensure_sample_park(static_cast<size_t>(B) * V);
        int* pin = c->pinned(3 * static_cast<size_t>(B));
        std::memcpy(pin, slots, B * sizeof(int));
        if (fed_ids) std::memcpy(pin + B, fed_ids, B * sizeof(int));
        cudaStream_t st = c->stream;
        cuda_ok(cudaMemcpyAsync(c->sb.slots, pin, B * sizeof(int), cudaMemcpyHostToDevice, st), "H2D slots");
        if (fed_ids)
            cuda_ok(cudaMemcpyAsync(c->sb.ids, pin + B, B * sizeof(int), cudaMemcpyHostToDevice, st), "H2D ids");
        cuda_ok(cudaMemsetAsync(c->sb.nonfinite, 0, B * sizeof(int), st), "memset");
        const SampleArgs a = sample_args(c, kv, B, logits, ld, fed_ids ? c->sb.ids : nullptr,
                                         c->sb.next, c->sb.nonfinite);
        c->note("sample_rows_kernel");
        cuda_ok(launch_sample_rows(a, st), "sample launch");
        cuda_ok(cudaMemcpyAsync(pin, c->sb.next, B * sizeof(int), cudaMemcpyDeviceToHost, st), "D2H");
        cuda_ok(cudaMemcpyAsync(pin + 2 * B, c->sb.nonfinite, B * sizeof(int), cudaMemcpyDeviceToHost, st), "D2H");
        c->sync(wait_timeout_seconds());
        std::memcpy(next_ids, pin, B * sizeof(int));
        for (int b = 0; b < B; ++b)
            if (pin[2 * B + b])
                fail(ADAI_B200_ERR_NONFINITE, "TextGenerator: the model returned non-finite logits");
    });
}

// ---- op level ----------------------------------------------------------------------------------
namespace {
// A [m, k] operand of the op-level GEMMs, times alpha, as its tf32 pair in the layout the GEMM
// streams: [rows_alloc, kpad] row-major, zero padded. op(A)[r][c] is a[r * lda + c], or
// a[c * lda + r] when trans.
__global__ void pack_split_a_kernel(const float* __restrict__ a, int lda, int trans, int m, int k,
                                    float alpha, float* __restrict__ hi, float* __restrict__ lo,
                                    int kpad, int rows_alloc) {
    // The GEMM that follows (programmatic dependent launch) may start its prologue and weight
    // loads now; it reads hi / lo only after this grid has completed.
    pdl_trigger();
    if (!trans && k == kpad && (kpad & 3) == 0 && (lda & 3) == 0 &&
        (reinterpret_cast<uintptr_t>(a) & 15) == 0) {
        // row-major A with whole 16-byte rows: four elements per thread
        const int q = kpad >> 2;
        const size_t n4 = static_cast<size_t>(rows_alloc) * q;
        for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n4;
             i += static_cast<size_t>(gridDim.x) * blockDim.x) {
            const int r = static_cast<int>(i / q), c4 = static_cast<int>(i - static_cast<size_t>(r) * q);
            float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
            if (r < m) v = *reinterpret_cast<const float4*>(a + static_cast<size_t>(r) * lda + c4 * 4);
            float4 h, l;
            split_tf32(alpha * v.x, h.x, l.x);
            split_tf32(alpha * v.y, h.y, l.y);
            split_tf32(alpha * v.z, h.z, l.z);
            split_tf32(alpha * v.w, h.w, l.w);
            reinterpret_cast<float4*>(hi)[i] = h;
            reinterpret_cast<float4*>(lo)[i] = l;
        }
        return;
    }
    const size_t n = static_cast<size_t>(rows_alloc) * kpad;
    for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<size_t>(gridDim.x) * blockDim.x) {
        const int r = static_cast<int>(i / kpad), cc = static_cast<int>(i % kpad);
        float v = 0.f;
        if (r < m && cc < k)
            v = alpha * (trans ? a[static_cast<size_t>(cc) * lda + r] : a[static_cast<size_t>(r) * lda + cc]);
        float h, l;
        split_tf32(v, h, l);
        hi[i] = h;
        lo[i] = l;
    }
}
// B [k, n] row-major (row stride ldb) -> B^T hi/lo [n, kpad], through a shared-memory tile.
__global__ void transpose_split_pad_kernel(const float* __restrict__ w, int ldb, int K, int N, int Kpad,
                                           float* __restrict__ hi_t, float* __restrict__ lo_t) {
    __shared__ float tile[32][33];
    const int n0 = blockIdx.x * 32, k0 = blockIdx.y * 32;
    for (int i = threadIdx.y; i < 32; i += blockDim.y) {
        const int k = k0 + i, nn = n0 + threadIdx.x;
        tile[i][threadIdx.x] = (k < K && nn < N) ? w[static_cast<size_t>(k) * ldb + nn] : 0.f;
    }
    __syncthreads();
    for (int i = threadIdx.y; i < 32; i += blockDim.y) {
        const int nn = n0 + i, k = k0 + threadIdx.x;
        if (nn < N && k < Kpad) {
            float h, l;
            split_tf32(tile[threadIdx.x][i], h, l);
            hi_t[static_cast<size_t>(nn) * Kpad + k] = h;
            lo_t[static_cast<size_t>(nn) * Kpad + k] = l;
        }
    }
}
// B stored transposed ([n, k], row stride ldb): already the B^T layout, split and padded.
__global__ void copy_split_pad_kernel(const float* __restrict__ w, int ldb, int K, int N, int Kpad,
                                      float* __restrict__ hi_t, float* __restrict__ lo_t) {
    const size_t total = static_cast<size_t>(N) * Kpad;
    for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<size_t>(gridDim.x) * blockDim.x) {
        const int nn = static_cast<int>(i / Kpad), k = static_cast<int>(i % Kpad);
        const float v = (k < K) ? w[static_cast<size_t>(nn) * ldb + k] : 0.f;
        float h, l;
        split_tf32(v, h, l);
        hi_t[i] = h;
        lo_t[i] = l;
    }
}

int blocks_for(size_t n) { return static_cast<int>(std::min<size_t>((n + 255) / 256, 148 * 16)); }

adai_b200_weight* prepare_weight(adai_b200_ctx* c, const float* B, int k, int n, int ldb = -1,
                                 bool trans_b = false) {
    if (!B || k <= 0 || n <= 0) fail(ADAI_B200_ERR_INVALID_ARGUMENT, "bad weight shape");
    if (ldb < 0) ldb = trans_b ? k : n;
    if (ldb < (trans_b ? k : n)) fail(ADAI_B200_ERR_INVALID_ARGUMENT, "ldb is smaller than a row of B");
    auto w = std::make_unique<adai_b200_weight>();
    const int kpad = round_up(k, 4);
    const size_t rows = static_cast<size_t>(round_up(n, 256));
    w->K = k;
    w->Kpad = kpad;
    w->w.K = kpad;
    w->w.N = n;
    w->w.hi = c->dzalloc_t<float>(rows * kpad);
    w->w.lo = c->dzalloc_t<float>(rows * kpad);
    c->note(trans_b ? "copy_split_pad_kernel" : "transpose_split_pad_kernel");
    if (trans_b) {
        copy_split_pad_kernel<<<blocks_for(static_cast<size_t>(n) * kpad), 256, 0, c->stream>>>(
            B, ldb, k, n, kpad, w->w.hi, w->w.lo);
    } else {
        dim3 grid((n + 31) / 32, (kpad + 31) / 32);
        transpose_split_pad_kernel<<<grid, dim3(32, 8), 0, c->stream>>>(B, ldb, k, n, kpad, w->w.hi, w->w.lo);
    }
    cuda_ok(cudaGetLastError(), "weight split");
    return w.release();
}

void free_weight(adai_b200_ctx* c, adai_b200_weight* w) {
    c->dfree(w->w.hi);
    c->dfree(w->w.lo);
    delete w;
}

// C[m, n] (row stride ldc) = alpha op(A) W. The fused epilogue stores float4 rows, so an output
// that is not 16-byte aligned with ldc % 4 == 0 goes through a packed buffer and a 2-D copy.
void gemm_run(adai_b200_ctx* c, int m, const float* A, int lda, bool trans_a, float alpha,
              const adai_b200_weight* w, float* C, int ldc) {
    if (m <= 0 || !A || !C) fail(ADAI_B200_ERR_INVALID_ARGUMENT, "bad GEMM arguments");
    const int k = w->K, n = w->w.N, kpad = w->Kpad;
    if (lda < (trans_a ? m : k)) fail(ADAI_B200_ERR_INVALID_ARGUMENT, "lda is smaller than a row of A");
    if (ldc < n) fail(ADAI_B200_ERR_INVALID_ARGUMENT, "ldc is smaller than a row of C");
    const int rows_alloc = round_up(m, 128);
    const size_t need = static_cast<size_t>(rows_alloc) * kpad;
    const bool direct = reinterpret_cast<uintptr_t>(C) % 16 == 0 && ldc % 4 == 0;
    // Up to two 128-row tiles of A in its own layout (rows 16-byte aligned) are split inside the
    // GEMM, one launch, when N is at most 8192. Larger, transposed, scaled or unaligned A goes
    // through the split kernel; so do wide products, where the extra shared-memory plane for the
    // raw A box costs a pipeline stage (measured on B200: 128 x 1024 x 32000 took 91.5 us split
    // inside against 66.2 us with the split kernel).
    const bool fused_split = !trans_a && alpha == 1.0f && rows_alloc <= 256 && n <= 8192 &&
                             lda % 4 == 0 && reinterpret_cast<uintptr_t>(A) % 16 == 0;
    const int ldp = round_up(n, 4);
    const size_t need_c = direct ? 0 : static_cast<size_t>(m) * ldp;
    if ((!fused_split && need > c->op_a_floats) || need_c > c->op_c_floats) {
        cuda_ok(cudaStreamSynchronize(c->stream), "sync");
        if (!fused_split && need > c->op_a_floats) {
            c->dfree(c->op_a_hi);
            c->dfree(c->op_a_lo);
            c->op_a_hi = c->op_a_lo = nullptr;
            c->op_a_floats = 0;
            c->op_a_hi = c->dalloc_t<float>(need);
            c->op_a_lo = c->dalloc_t<float>(need);
            c->op_a_floats = need;
        }
        if (need_c > c->op_c_floats) {
            c->dfree(c->op_c);
            c->op_c = nullptr;
            c->op_c_floats = 0;
            c->op_c = c->dalloc_t<float>(need_c);
            c->op_c_floats = need_c;
        }
    }
    GemmEpilogue e;
    e.flags = kEpiStore;
    e.out = direct ? C : c->op_c;
    e.ldo = direct ? ldc : ldp;
    if (fused_split) {
        TcActs a;
        a.K = kpad;
        a.rows_alloc = rows_alloc;
        a.fp32 = A;
        a.lda = lda;
        a.k_valid = k;
        a.rows = m;
        e.flags |= kEpiAFp32;
        c->gemm(a, m, w->w, e, "gemm_3xtf32_kernel (A split inside)");
    } else {
        c->note("pack_split_a_kernel");
        pack_split_a_kernel<<<blocks_for(need), 256, 0, c->stream>>>(A, lda, trans_a ? 1 : 0, m, k, alpha,
                                                                     c->op_a_hi, c->op_a_lo, kpad, rows_alloc);
        cuda_ok(cudaGetLastError(), "split");
        c->gemm(acts(c->op_a_hi, c->op_a_lo, kpad, rows_alloc), m, w->w, e);
    }
    if (!direct)
        cuda_ok(cudaMemcpy2DAsync(C, static_cast<size_t>(ldc) * sizeof(float), c->op_c,
                                  static_cast<size_t>(ldp) * sizeof(float), static_cast<size_t>(n) * sizeof(float),
                                  static_cast<size_t>(m), cudaMemcpyDeviceToDevice, c->stream),
                "copy out");
}
}  // namespace

int adai_b200_weight_create(adai_b200_ctx* c, const float* B, int k, int n, adai_b200_weight** out) {
    return traced(c, "adai_b200_weight_create", [&] {
        check_ctx(c);
        if (!out) fail(ADAI_B200_ERR_INVALID_ARGUMENT, "null output handle");
        *out = prepare_weight(c, B, k, n);
    });
}

int adai_b200_weight_destroy(adai_b200_ctx* c, adai_b200_weight* w) {
    return guarded([&] {
        if (!c || !w) fail(ADAI_B200_ERR_INVALID_ARGUMENT, "null argument");
        cudaSetDevice(c->device);
        cudaStreamSynchronize(c->stream);
        free_weight(c, w);
    });
}

int adai_b200_sgemm_prepared(adai_b200_ctx* c, int m, const float* A, const adai_b200_weight* w, float* C) {
    return traced(c, "adai_b200_sgemm_prepared", [&] {
        check_ctx(c);
        if (!w) fail(ADAI_B200_ERR_INVALID_ARGUMENT, "null weight");
        gemm_run(c, m, A, w->K, false, 1.0f, w, C, w->w.N);
    });
}

int adai_b200_sgemm(adai_b200_ctx* c, int m, int n, int k, const float* A, const float* B, float* C) {
    return traced(c, "adai_b200_sgemm", [&] {
        check_ctx(c);
        adai_b200_weight* w = prepare_weight(c, B, k, n);
        try {
            gemm_run(c, m, A, k, false, 1.0f, w, C, n);
        } catch (...) {
            cudaStreamSynchronize(c->stream);
            free_weight(c, w);
            throw;
        }
        cuda_ok(cudaStreamSynchronize(c->stream), "sync");
        free_weight(c, w);
    });
}

int adai_b200_decode_attention(adai_b200_ctx* c, int B, int H, int head_dim, int capacity,
                               const float* q, const float* k_new, const float* v_new,
                               float* k_cache, float* v_cache, const int* lens, int max_len,
                               float* out) {
    return traced(c, "adai_b200_decode_attention", [&] {
        check_ctx(c);
        if (B <= 0 || H <= 0 || capacity <= 0 || !q || !k_cache || !v_cache || !lens || !out)
            fail(ADAI_B200_ERR_INVALID_ARGUMENT, "bad attention arguments");
        if (!attention_head_dim_supported(head_dim))
            fail(ADAI_B200_ERR_INVALID_ARGUMENT, "head_dim must be 32 or 64");
        if ((k_new == nullptr) != (v_new == nullptr))
            fail(ADAI_B200_ERR_INVALID_ARGUMENT, "k_new and v_new must both be given or both be null");
        for (const void* p : {(const void*)q, (const void*)k_new, (const void*)v_new,
                              (const void*)k_cache, (const void*)v_cache, (const void*)out})
            if (reinterpret_cast<uintptr_t>(p) % 16)
                fail(ADAI_B200_ERR_INVALID_ARGUMENT, "attention buffers must be 16-byte aligned");
        const int add = k_new ? 1 : 0;
        if (max_len < 0 || max_len + add > capacity)
            fail(ADAI_B200_ERR_OUT_OF_RANGE, "max_len exceeds the cache capacity");
        c->ensure_attn_scratch(B, H, max_len + add, head_dim);
        const int D = H * head_dim;
        DecodeAttnArgs a;
        a.q = q;
        a.ldq = D;
        a.k_new = k_new;
        a.v_new = v_new;
        a.ldkv = D;
        a.kc = k_cache;
        a.vc = v_cache;
        a.slot_stride = static_cast<long long>(H) * capacity * head_dim;
        a.cap = capacity;
        a.slots = nullptr;
        a.len_by_slot = lens;
        a.len_add = add;
        a.out = out;
        a.ldo = D;
        a.B = B;
        a.H = H;
        a.head_dim = head_dim;
        a.max_len = max_len + add;
        a.scale = 1.0f / std::sqrt(static_cast<float>(head_dim));
        a.ws = c->attn_ws;
        a.tickets = c->attn_tickets;
        c->note("decode_attention_kernel");
        launch_decode_attention(a, c->d_err, c->stream);
        cuda_ok(cudaGetLastError(), "attention launch");
    });
}

int adai_b200_ctx_last_timing(adai_b200_ctx* c, double* decode_ms, int* kernels_per_step) {
    return guarded([&] {
        if (!c) fail(ADAI_B200_ERR_INVALID_ARGUMENT, "null context");
        if (decode_ms) *decode_ms = c->last_decode_ms;
        if (kernels_per_step) *kernels_per_step = c->last_kernels_per_step;
    });
}

int adai_b200_profile_step(adai_b200_ctx* c, adai_b200_kv* kv, int B, const int* slots,
                           const int* ids, int n_classes, double* ms, double* bytes,
                           double* flops, int* launches) {
    return traced(c, "adai_b200_profile_step", [&] {
        check_ctx(c);
        check_model(c);
        check_kv(c, kv);
        if (n_classes < ADAI_B200_KC_COUNT || !ms || !bytes || !flops || !launches)
            fail(ADAI_B200_ERR_INVALID_ARGUMENT, "need ADAI_B200_KC_COUNT entries in every output array");
        stage_batch(c, kv, B, slots, ids, 1);
        const int flags = sample_flag(kv, B, slots);
        presize_step_scratch(c, kv, B, flags);
        Profiler prof;
        for (int b = 0; b < B; ++b) {
            prof.sum_self_rows += kv->self_len[slots[b]] + 1;
            prof.sum_cross_rows += kv->cross_len[slots[b]];
        }
        c->prof = &prof;
        try {
            record_step(c, kv, B, flags);
            timed(c, ADAI_B200_KC_OTHER, 0, 0, [&] {
                c->note("record_and_advance_kernel");
                record_and_advance_kernel<<<(B + 127) / 128, 128, 0, c->stream>>>(
                    c->sb.next, c->sb.ids, c->sb.slots, kv->d_self_len, kv->d_hist, kv->self_cap,
                    c->sb.nonfinite, c->sb.nonfinite_any, B, 0);
            });
            c->prof = nullptr;
            c->sync(wait_timeout_seconds());
        } catch (...) {
            c->prof = nullptr;
            cudaStreamSynchronize(c->stream);
            for (auto& sp : prof.spans) {
                cudaEventDestroy(sp.a);
                cudaEventDestroy(sp.b);
            }
            throw;
        }
        for (int k = 0; k < n_classes; ++k) {
            ms[k] = bytes[k] = flops[k] = 0;
            launches[k] = 0;
        }
        for (auto& sp : prof.spans) {
            float t = 0.f;
            cuda_ok(cudaEventElapsedTime(&t, sp.a, sp.b), "cudaEventElapsedTime");
            ms[sp.cls] += t;
            bytes[sp.cls] += sp.bytes;
            flops[sp.cls] += sp.flops;
            launches[sp.cls] += 1;
            cudaEventDestroy(sp.a);
            cudaEventDestroy(sp.b);
        }
        for (int b = 0; b < B; ++b) kv->self_len[slots[b]] += 1;
    });
}

int adai_b200_layernorm(adai_b200_ctx* c, const float* x, const float* gamma, const float* beta,
                        float* out, int rows, int D) {
    return traced(c, "adai_b200_layernorm", [&] {
        check_ctx(c);
        if (!x || !gamma || !beta || !out || rows <= 0) fail(ADAI_B200_ERR_INVALID_ARGUMENT, "bad LayerNorm arguments");
        if (!layernorm_width_supported(D)) fail(ADAI_B200_ERR_INVALID_ARGUMENT, "D must be 128 * {1,2,3,4,6,8,12,16}");
        c->note("layernorm_kernel");
        launch_layernorm(x, D, gamma, beta, out, nullptr, nullptr, rows, D, c->stream);
        cuda_ok(cudaGetLastError(), "layernorm launch");
    });
}

// ---- the decode-path entries of the reference backend table (adai::gpu::matrix_*_gpu) ----------
int adai_b200_gemm_strided(adai_b200_ctx* c, int trans_a, int trans_b, int m, int n, int k,
                           float alpha, const float* a, int lda, const float* b, int ldb, float* out,
                           int ldc) {
    return traced(c, "adai_b200_gemm_strided", [&] {
        check_ctx(c);
        if (m <= 0 || n <= 0) return;  // nothing to write, as the reference returns early
        if (!out || ldc < n) fail(ADAI_B200_ERR_INVALID_ARGUMENT, "bad output of the strided GEMM");
        if (k <= 0) {  // an empty inner dimension: C = 0
            cuda_ok(cudaMemset2DAsync(out, static_cast<size_t>(ldc) * sizeof(float), 0,
                                      static_cast<size_t>(n) * sizeof(float), static_cast<size_t>(m),
                                      c->stream),
                    "zero C");
            return;
        }
        if (!a || !b) fail(ADAI_B200_ERR_INVALID_ARGUMENT, "null operand");
        adai_b200_weight* w = prepare_weight(c, b, k, n, ldb, trans_b != 0);
        try {
            gemm_run(c, m, a, lda, trans_a != 0, alpha, w, out, ldc);
        } catch (...) {
            cudaStreamSynchronize(c->stream);
            free_weight(c, w);
            throw;
        }
        cuda_ok(cudaStreamSynchronize(c->stream), "sync");
        free_weight(c, w);
    });
}

int adai_b200_softmax_rows(adai_b200_ctx* c, float* data, int rows, int cols) {
    return traced(c, "adai_b200_softmax_rows", [&] {
        check_ctx(c);
        if (rows < 0 || cols < 0 || (rows && cols && !data)) fail(ADAI_B200_ERR_INVALID_ARGUMENT, "bad softmax arguments");
        c->note("softmax_rows_kernel");
        launch_softmax_rows(data, rows, cols, c->stream);
        cuda_ok(cudaGetLastError(), "softmax launch");
    });
}

int adai_b200_layernorm_fwd(adai_b200_ctx* c, const float* x, float* y, float* x_normed,
                            const float* gamma, const float* beta, float* mean, float* rstd,
                            int rows, int cols, float eps) {
    return traced(c, "adai_b200_layernorm_fwd", [&] {
        check_ctx(c);
        if (rows < 0 || cols <= 0 || (rows && (!x || !y || !gamma || !beta)))
            fail(ADAI_B200_ERR_INVALID_ARGUMENT, "bad LayerNorm arguments");
        c->note("layernorm_rows_kernel");
        launch_layernorm_rows(x, y, x_normed, gamma, beta, mean, rstd, rows, cols, eps, c->stream);
        cuda_ok(cudaGetLastError(), "layernorm launch");
    });
}

int adai_b200_add_row_bias(adai_b200_ctx* c, const float* m, const float* bias, float* out, int rows,
                           int cols) {
    return traced(c, "adai_b200_add_row_bias", [&] {
        check_ctx(c);
        if (rows < 0 || cols <= 0 || (rows && (!m || !bias || !out)))
            fail(ADAI_B200_ERR_INVALID_ARGUMENT, "bad bias arguments");
        c->note("add_row_bias_kernel");
        launch_add_row_bias(m, bias, out, rows, cols, c->stream);
        cuda_ok(cudaGetLastError(), "bias launch");
    });
}

int adai_b200_activation(adai_b200_ctx* c, float* data, int size, int type) {
    return traced(c, "adai_b200_activation", [&] {
        check_ctx(c);
        if (size < 0 || (size && !data)) fail(ADAI_B200_ERR_INVALID_ARGUMENT, "bad activation arguments");
        if (type < 0 || type > 3) fail(ADAI_B200_ERR_INVALID_ARGUMENT, "activation type must be 0..3");
        c->note("activation_kernel");
        launch_activation(data, static_cast<size_t>(size), type, c->stream);
        cuda_ok(cudaGetLastError(), "activation launch");
    });
}

int adai_b200_embedding_gather_add_pe(adai_b200_ctx* c, const float* table, const int* ids,
                                      const float* pe, int pe_rows, int pos_offset, float* out, int n,
                                      int d, int vocab) {
    return traced(c, "adai_b200_embedding_gather_add_pe", [&] {
        check_ctx(c);
        if (n < 0 || d <= 0 || (n && (!table || !ids || !out)))
            fail(ADAI_B200_ERR_INVALID_ARGUMENT, "bad embedding arguments");
        c->note("embed_pe_kernel");
        launch_embed_pe(table, ids, pe, pe_rows, pos_offset, out, n, d,
                        vocab > 0 ? vocab : std::numeric_limits<int>::max(), c->d_err, c->stream);
        cuda_ok(cudaGetLastError(), "embedding launch");
    });
}

}  // extern "C"

// ---------------------------------------------------------------------------------------------
// Decode attention with static scratch: adai_b200_decode_attention for callers that must not
// allocate device memory at call time. The split-KV partials and the per-(sequence, head) merge
// tickets live in one fixed array that is part of this library's device image, so the call
// itself neither allocates nor frees: it suits a host that has handed all free device memory to
// its own pool up front (nothing is left for a late cudaMalloc, and a cudaMalloc would also
// stall the device while its streams are busy), or that forbids allocation on its serving path.
// The price is a hard size limit and one shared buffer per device: calls that overlap in time
// on the same device (two streams, two contexts, two threads) race on it and corrupt each
// other's results. Serializing the host calls is not enough, because each call only queues its
// kernel: calls on different streams must also be ordered on the device (one stream, events, or
// a device synchronize between them). A cached length outside [0, max_len] is refused by the
// kernel itself (the call then fails at the next synchronize with ADAI_B200_ERR_OUT_OF_RANGE) and
// leaves the merge counters at zero.
static constexpr size_t kStaticAttnScratchBytes = size_t(16) << 20;  // per device
static constexpr size_t kStaticAttnTicketBytes = size_t(64) << 10;   // first part: tickets
static constexpr int kStaticAttnMaxPairs = static_cast<int>(kStaticAttnTicketBytes / sizeof(int));

static __device__ __align__(256) unsigned char g_static_attn_scratch[kStaticAttnScratchBytes];

namespace {

constexpr int kStaticMaxDevices = 64;
std::mutex g_static_attn_mu;
// Per device, the array address whose merge counters this process has zeroed. A device reset
// reloads the module; its array then shows up at a fresh lookup and is zeroed again if its address
// differs (a reloaded module's array starts zeroed in any case).
void* g_static_attn_zeroed[kStaticMaxDevices] = {};

// The scratch array's address on the current device, looked up on every call (the lookup is a
// host-side table read). The first call on a device zeroes the merge counters (every launch hands
// them back at zero) and waits for that before it returns, so a later call on any stream of the
// device is ordered after it. `device` must be the current device.
unsigned char* static_attn_scratch(int device, cudaStream_t st) {
    if (device < 0 || device >= kStaticMaxDevices)
        fail(ADAI_B200_ERR_INVALID_ARGUMENT, "device index out of range for the static scratch table");
    void* p = nullptr;
    cuda_ok(cudaGetSymbolAddress(&p, g_static_attn_scratch), "cudaGetSymbolAddress(static attention scratch)");
    std::lock_guard<std::mutex> lock(g_static_attn_mu);
    if (g_static_attn_zeroed[device] != p) {
        cuda_ok(cudaMemsetAsync(p, 0, kStaticAttnTicketBytes, st), "zero static attention tickets");
        cuda_ok(cudaStreamSynchronize(st), "wait for the static attention tickets to be zeroed");
        g_static_attn_zeroed[device] = p;
    }
    return static_cast<unsigned char*>(p);
}

}  // namespace

extern "C" {

int adai_b200_decode_attention_static(adai_b200_ctx* c, int B, int H, int head_dim, int capacity,
                                      const float* q, const float* k_new, const float* v_new,
                                      float* k_cache, float* v_cache, const int* lens, int max_len,
                                      float* out) {
    return traced(c, "adai_b200_decode_attention_static", [&] {
        check_ctx(c);
        if (B <= 0 || H <= 0 || capacity <= 0 || !q || !k_cache || !v_cache || !lens || !out)
            fail(ADAI_B200_ERR_INVALID_ARGUMENT, "bad attention arguments");
        if (!attention_head_dim_supported(head_dim))
            fail(ADAI_B200_ERR_INVALID_ARGUMENT, "head_dim must be 32 or 64");
        if ((k_new == nullptr) != (v_new == nullptr))
            fail(ADAI_B200_ERR_INVALID_ARGUMENT, "k_new and v_new must both be given or both be null");
        for (const void* p : {(const void*)q, (const void*)k_new, (const void*)v_new,
                              (const void*)k_cache, (const void*)v_cache, (const void*)out})
            if (reinterpret_cast<uintptr_t>(p) % 16)
                fail(ADAI_B200_ERR_INVALID_ARGUMENT, "attention buffers must be 16-byte aligned");
        const int add = k_new ? 1 : 0;
        if (max_len < 0 || max_len + add > capacity)
            fail(ADAI_B200_ERR_OUT_OF_RANGE, "max_len exceeds the cache capacity");
        const long long pairs = static_cast<long long>(B) * H;
        const size_t part_bytes = decode_attn_ws_floats(B, H, max_len + add, head_dim) * sizeof(float);
        const size_t part_max = kStaticAttnScratchBytes - kStaticAttnTicketBytes;
        if (pairs > kStaticAttnMaxPairs || part_bytes > part_max) {
            char msg[256];
            std::snprintf(msg, sizeof msg,
                          "static attention scratch too small: B*H = %lld (max %d) and %zu bytes of "
                          "split partials (max %zu); use adai_b200_decode_attention",
                          pairs, kStaticAttnMaxPairs, part_bytes, part_max);
            fail(ADAI_B200_ERR_OUT_OF_RANGE, msg);
        }
        unsigned char* base = static_attn_scratch(c->device, c->stream);
        const int D = H * head_dim;
        DecodeAttnArgs a;
        a.q = q;
        a.ldq = D;
        a.k_new = k_new;
        a.v_new = v_new;
        a.ldkv = D;
        a.kc = k_cache;
        a.vc = v_cache;
        a.slot_stride = static_cast<long long>(H) * capacity * head_dim;
        a.cap = capacity;
        a.slots = nullptr;
        a.len_by_slot = lens;
        a.len_add = add;
        a.out = out;
        a.ldo = D;
        a.B = B;
        a.H = H;
        a.head_dim = head_dim;
        a.max_len = max_len + add;
        a.scale = 1.0f / std::sqrt(static_cast<float>(head_dim));
        a.tickets = reinterpret_cast<int*>(base);
        a.ws = reinterpret_cast<float*>(base + kStaticAttnTicketBytes);
        c->note("decode_attention_kernel");
        launch_decode_attention(a, c->d_err, c->stream);
        cuda_ok(cudaGetLastError(), "attention launch");
    });
}

}  // extern "C"
