// Test infrastructure, not product code: a C driver over the reference's own CPU decode path.
//
// It is compiled together with the reference sources (oracle/Makefile, target `ref`) into
// oracle/_ref/libadai_ref.so. The driver builds the reference objects (LLMEncoder, LLMDecoder,
// LanguageModelHead — the same trio benchmarks/GpuDecodeBenchmark.cpp:250-310 drives), installs the
// caller's seeded weights through their public setters, and runs the reference arithmetic
// (Matrix::operator*, LayerNorm::forward, Activation::gelu/softmax, the cached forward passes).
// Only tests/, the fixture generator and bench.py's CPU baseline leg load it.
//
// Weight order (row-major fp32, shapes as the reference setters take them) — the same order the
// product's adai_b200_model_upload() uses:
//   enc.embed[V,D]
//   per encoder layer: ln1.g[D] ln1.b[D] wq wk wv wo [D,D] ln2.g ln2.b w1[D,F] b1[F] w2[F,D] b2[D]
//   enc.lnf.g enc.lnf.b
//   dec.embed[V,D]
//   per decoder layer: ln1.g ln1.b sa.wq sa.wk sa.wv sa.wo ln2.g ln2.b ca.wq ca.wk ca.wv ca.wo
//                      ln3.g ln3.b w1 b1 w2 b2
//   dec.lnf.g dec.lnf.b
//   head.w[D,V] head.b[V]

#include <algorithm>
#include <chrono>
#include <cstring>
#include <functional>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

#include <omp.h>

#include "Activation.hpp"
#include "BinaryIO.hpp"
#include "Decoder.hpp"
#include "KVCache.hpp"
#include "LanguageModelHead.hpp"
#include "LayerNorm.hpp"
#include "Matrix.hpp"
#include "PositionalEncoding.hpp"
#include "TextGenerator.hpp"
#include "encoder.hpp"

namespace {

thread_local std::string g_err;

Matrix from_flat(const float* p, int rows, int cols) {
    Matrix m(rows, cols);
    for (int i = 0; i < rows; ++i)
        std::memcpy(m.data[i].data(), p + static_cast<size_t>(i) * cols, sizeof(float) * cols);
    return m;
}

void to_flat(const Matrix& m, float* p) {
    for (int i = 0; i < m.rows; ++i)
        std::memcpy(p + static_cast<size_t>(i) * m.cols, m.data[i].data(), sizeof(float) * m.cols);
}

struct RefModel {
    int V, D, H, F, Le, L, max_seq;
    std::unique_ptr<LLMEncoder> enc;
    std::unique_ptr<LLMDecoder> dec;
    std::unique_ptr<LanguageModelHead> head;
};

template <class Fn>
int guarded(Fn&& fn) {
    try {
        fn();
        return 0;
    } catch (const std::exception& e) {
        g_err = e.what();
        return -1;
    }
}

int first_max(const std::vector<float>& row) {
    return static_cast<int>(std::max_element(row.begin(), row.end()) - row.begin());
}

}  // namespace

extern "C" {

const char* ref_last_error() { return g_err.c_str(); }

const char* ref_matmul_kernel() { return Matrix::cpu_matmul_kernel(); }

// cfg = {vocab, d_model, n_heads, d_ff, enc_layers, dec_layers, max_seq}
int ref_model_create(const int* cfg, const float* const* t, void** out) {
    return guarded([&] {
        auto m = std::make_unique<RefModel>();
        m->V = cfg[0];
        m->D = cfg[1];
        m->H = cfg[2];
        m->F = cfg[3];
        m->Le = cfg[4];
        m->L = cfg[5];
        m->max_seq = cfg[6];
        const int V = m->V, D = m->D, F = m->F;
        m->enc = std::make_unique<LLMEncoder>(V, D, m->Le, m->H, F, m->max_seq);
        m->dec = std::make_unique<LLMDecoder>(V, D, m->L, m->H, F, m->max_seq, 0);
        m->head = std::make_unique<LanguageModelHead>(D, V);
        int k = 0;
        auto next = [&](int r, int c) { return from_flat(t[k++], r, c); };
        m->enc->get_token_embedding()->set_embeddings(next(V, D));
        for (int i = 0; i < m->Le; ++i) {
            EncoderBlock* b = m->enc->get_encoder_block(i);
            b->get_norm1()->set_gamma(next(1, D));
            b->get_norm1()->set_beta(next(1, D));
            MultiHeadAttention* a = b->get_self_attention();
            a->set_Wq(next(D, D));
            a->set_Wk(next(D, D));
            a->set_Wv(next(D, D));
            a->set_Wo(next(D, D));
            b->get_norm2()->set_gamma(next(1, D));
            b->get_norm2()->set_beta(next(1, D));
            FeedForward* f = b->get_feed_forward();
            f->set_W1(next(D, F));
            f->set_b1(next(1, F));
            f->set_W2(next(F, D));
            f->set_b2(next(1, D));
        }
        m->enc->get_final_norm()->set_gamma(next(1, D));
        m->enc->get_final_norm()->set_beta(next(1, D));
        m->dec->get_token_embedding()->set_embeddings(next(V, D));
        for (int i = 0; i < m->L; ++i) {
            DecoderBlock* b = m->dec->get_decoder_block(i);
            b->get_norm1()->set_gamma(next(1, D));
            b->get_norm1()->set_beta(next(1, D));
            MultiHeadAttention* sa = b->get_self_attention();
            sa->set_Wq(next(D, D));
            sa->set_Wk(next(D, D));
            sa->set_Wv(next(D, D));
            sa->set_Wo(next(D, D));
            b->get_norm2()->set_gamma(next(1, D));
            b->get_norm2()->set_beta(next(1, D));
            CrossAttention* ca = b->get_cross_attention();
            ca->set_Wq(next(D, D));
            ca->set_Wk(next(D, D));
            ca->set_Wv(next(D, D));
            ca->set_Wo(next(D, D));
            b->get_norm3()->set_gamma(next(1, D));
            b->get_norm3()->set_beta(next(1, D));
            FeedForward* f = b->get_feed_forward();
            f->set_W1(next(D, F));
            f->set_b1(next(1, F));
            f->set_W2(next(F, D));
            f->set_b2(next(1, D));
        }
        m->dec->get_final_norm()->set_gamma(next(1, D));
        m->dec->get_final_norm()->set_beta(next(1, D));
        m->head->set_W_output(next(D, V));
        m->head->set_bias(next(1, V));
        *out = m.release();
    });
}

void ref_model_destroy(void* h) { delete static_cast<RefModel*>(h); }

// Encoder prefill: LLMEncoder::encode_with_mask with an all-ones mask (src/LLMEncoder.cpp:120-142).
int ref_encode(void* h, const int* ids, int S, float* enc_out) {
    return guarded([&] {
        auto* m = static_cast<RefModel*>(h);
        std::vector<int> v(ids, ids + S);
        Matrix mask(S, S);
        for (auto& row : mask.data) std::fill(row.begin(), row.end(), 1.0f);
        to_flat(m->enc->encode_with_mask(v, mask), enc_out);
    });
}

// One request the way the reference serves it: encoder once, then one cached decoder step per token
// (LLMDecoder::forward_with_cache, src/Decoder.cpp:210-287) -> LanguageModelHead::forward -> first
// maximum (TextGenerator::argmax, src/TextGenerator.cpp:151-153), no stop tokens. With `forced`
// non-null, step s feeds forced[s] instead of its own argmax (teacher forcing for lockstep parity).
// logits: [steps, V] or null. enc_s / dec_s: wall seconds of the encoder and of the decode loop.
int ref_generate(void* h, const int* src, int S, int bos, int steps, const int* forced,
                 int* out_ids, float* logits, double* enc_s, double* dec_s) {
    return guarded([&] {
        auto* m = static_cast<RefModel*>(h);
        using clk = std::chrono::steady_clock;
        auto t0 = clk::now();
        std::vector<int> v(src, src + S);
        Matrix mask(S, S);
        for (auto& row : mask.data) std::fill(row.begin(), row.end(), 1.0f);
        Matrix enc = m->enc->encode_with_mask(v, mask);
        auto t1 = clk::now();
        DecoderKVCache cache(m->L);
        int tok = bos;
        for (int s = 0; s < steps; ++s) {
            Matrix x = m->dec->forward_with_cache({tok}, cache, &enc, true);
            Matrix lg = m->head->forward(x);
            const std::vector<float>& row = lg.data[lg.rows - 1];
            out_ids[s] = first_max(row);
            if (logits) std::memcpy(logits + static_cast<size_t>(s) * m->V, row.data(),
                                    sizeof(float) * m->V);
            tok = forced ? forced[s] : out_ids[s];
        }
        auto t2 = clk::now();
        if (enc_s) *enc_s = std::chrono::duration<double>(t1 - t0).count();
        if (dec_s) *dec_s = std::chrono::duration<double>(t2 - t1).count();
    });
}

// ref_generate that also returns, per step, the decoder's output row (after its final LayerNorm,
// src/Decoder.cpp:284), which LanguageModelHead::forward turns into the logits as hidden * W_output
// + bias (src/LanguageModelHead.cpp:49-69). hidden: [steps, D]. logit_sum / top2: per step, the
// float64 sum of the logits row and its two largest values (either may be null). These are what the
// long-run fixtures keep: the logits follow from the hidden rows with the same in-order product.
int ref_generate_hidden(void* h, const int* src, int S, int bos, int steps, const int* forced,
                        int* out_ids, float* hidden, double* logit_sum, float* top2) {
    return guarded([&] {
        auto* m = static_cast<RefModel*>(h);
        std::vector<int> v(src, src + S);
        Matrix mask(S, S);
        for (auto& row : mask.data) std::fill(row.begin(), row.end(), 1.0f);
        Matrix enc = m->enc->encode_with_mask(v, mask);
        DecoderKVCache cache(m->L);
        int tok = bos;
        for (int s = 0; s < steps; ++s) {
            Matrix x = m->dec->forward_with_cache({tok}, cache, &enc, true);
            Matrix lg = m->head->forward(x);
            const std::vector<float>& row = lg.data[lg.rows - 1];
            out_ids[s] = first_max(row);
            if (hidden) std::memcpy(hidden + static_cast<size_t>(s) * m->D, x.data[x.rows - 1].data(),
                                    sizeof(float) * m->D);
            if (logit_sum) {
                double acc = 0.0;
                for (float f : row) acc += static_cast<double>(f);
                logit_sum[s] = acc;
            }
            if (top2) {
                std::vector<float> c(row);
                std::partial_sort(c.begin(), c.begin() + 2, c.end(), std::greater<float>());
                top2[2 * s] = c[0];
                top2[2 * s + 1] = c[1];
            }
            tok = forced ? forced[s] : out_ids[s];
        }
    });
}

// The same greedy loop with the wall time of every decode step (decoder + head + argmax) in
// step_s[s]; the encoder time in *enc_s. Used to time the reference CPU path per token.
int ref_generate_timed(void* h, const int* src, int S, int bos, int steps, int* out_ids,
                       double* step_s, double* enc_s) {
    return guarded([&] {
        auto* m = static_cast<RefModel*>(h);
        using clk = std::chrono::steady_clock;
        auto t0 = clk::now();
        std::vector<int> v(src, src + S);
        Matrix mask(S, S);
        for (auto& row : mask.data) std::fill(row.begin(), row.end(), 1.0f);
        Matrix enc = m->enc->encode_with_mask(v, mask);
        if (enc_s) *enc_s = std::chrono::duration<double>(clk::now() - t0).count();
        DecoderKVCache cache(m->L);
        int tok = bos;
        for (int s = 0; s < steps; ++s) {
            auto a = clk::now();
            Matrix x = m->dec->forward_with_cache({tok}, cache, &enc, true);
            Matrix lg = m->head->forward(x);
            out_ids[s] = first_max(lg.data[lg.rows - 1]);
            step_s[s] = std::chrono::duration<double>(clk::now() - a).count();
            tok = out_ids[s];
        }
    });
}

// ref_generate_timed with a host thread count per step: before step s the OpenMP team size is set
// to threads[s] (0: unchanged), so one run gives both the all-core and the one-thread rate of the
// reference's decode after a single encoder pass (which runs on the first step's team). The team
// size is restored afterwards.
int ref_generate_timed_threads(void* h, const int* src, int S, int bos, int steps,
                               const int* threads, int* out_ids, double* step_s, double* enc_s) {
    const int saved = omp_get_max_threads();
    const int rc = guarded([&] {
        auto* m = static_cast<RefModel*>(h);
        using clk = std::chrono::steady_clock;
        if (threads && steps > 0 && threads[0] > 0) omp_set_num_threads(threads[0]);
        auto t0 = clk::now();
        std::vector<int> v(src, src + S);
        Matrix mask(S, S);
        for (auto& row : mask.data) std::fill(row.begin(), row.end(), 1.0f);
        Matrix enc = m->enc->encode_with_mask(v, mask);
        if (enc_s) *enc_s = std::chrono::duration<double>(clk::now() - t0).count();
        DecoderKVCache cache(m->L);
        int tok = bos;
        for (int s = 0; s < steps; ++s) {
            if (threads && threads[s] > 0) omp_set_num_threads(threads[s]);
            auto a = clk::now();
            Matrix x = m->dec->forward_with_cache({tok}, cache, &enc, true);
            Matrix lg = m->head->forward(x);
            out_ids[s] = first_max(lg.data[lg.rows - 1]);
            step_s[s] = std::chrono::duration<double>(clk::now() - a).count();
            tok = out_ids[s];
        }
    });
    omp_set_num_threads(saved);
    return rc;
}

// One decoder step over a caller-supplied encoder output, returning the final-LN hidden row and
// the logits row; used for the decode-step fixtures at a chosen position. pre_ids are the tokens
// fed before (positions 0..n_pre-1); the step feeds `tok` at position n_pre.
int ref_decode_after(void* h, const float* enc_out, int S, const int* pre_ids, int n_pre, int tok,
                     float* hidden, float* logits) {
    return guarded([&] {
        auto* m = static_cast<RefModel*>(h);
        Matrix enc = from_flat(enc_out, S, m->D);
        DecoderKVCache cache(m->L);
        for (int i = 0; i < n_pre; ++i) m->dec->forward_with_cache({pre_ids[i]}, cache, &enc, true);
        Matrix x = m->dec->forward_with_cache({tok}, cache, &enc, true);
        Matrix lg = m->head->forward(x);
        if (hidden) to_flat(x, hidden);
        if (logits) to_flat(lg, logits);
    });
}

// C[M,N] = A[M,K] * B[K,N] through Matrix::operator* (src/Matrix.cpp:212-277).
int ref_matmul(const float* A, const float* B, float* C, int M, int K, int N) {
    return guarded([&] { to_flat(from_flat(A, M, K) * from_flat(B, K, N), C); });
}

// LayerNorm::forward with the given gamma/beta (src/LayerNorm.cpp:56-109).
int ref_layernorm(const float* x, const float* g, const float* b, float* out, int rows, int D) {
    return guarded([&] {
        LayerNorm ln(D);
        ln.set_gamma(from_flat(g, 1, D));
        ln.set_beta(from_flat(b, 1, D));
        to_flat(ln.forward(from_flat(x, rows, D)), out);
    });
}

int ref_gelu(const float* x, float* out, int n) {
    return guarded([&] { to_flat(Activation::gelu(from_flat(x, 1, n)), out); });
}

int ref_softmax_rows(const float* x, float* out, int rows, int cols) {
    return guarded([&] { to_flat(Activation::softmax(from_flat(x, rows, cols)), out); });
}

int ref_pe_table(int max_len, int D, float* out) {
    return guarded([&] { to_flat(PositionalEncoding(max_len, D).get_encoding(), out); });
}

// Single-query attention over one sequence's cache, every head, with the reference's per-head
// Matrix arithmetic (src/MultiHeadAttention.cpp:336-367): scores = (Q_h * K_h^T).scale(1/sqrt(dk)),
// Activation::softmax, * V_h, scattered into the head's columns. q [D], K/V [T, D] row-major.
int ref_attention_single(const float* q, const float* K, const float* Vv, int T, int D, int H,
                         float* out) {
    return guarded([&] {
        const int dk = D / H;
        Matrix Q = from_flat(q, 1, D);
        Matrix Km = from_flat(K, T, D);
        Matrix Vm = from_flat(Vv, T, D);
        const float scale = 1.0f / std::sqrt(static_cast<float>(dk));
        for (int h = 0; h < H; ++h) {
            Matrix Qh(1, dk), Kh(T, dk), Vh(T, dk);
            for (int j = 0; j < dk; ++j) Qh.data[0][j] = Q.data[0][h * dk + j];
            for (int t = 0; t < T; ++t)
                for (int j = 0; j < dk; ++j) {
                    Kh.data[t][j] = Km.data[t][h * dk + j];
                    Vh.data[t][j] = Vm.data[t][h * dk + j];
                }
            Matrix scores = (Qh * Kh.transpose()).scale(scale);
            Matrix w = Activation::softmax(scores);
            Matrix o = w * Vh;
            for (int j = 0; j < dk; ++j) out[h * dk + j] = o.data[0][j];
        }
    });
}

// The model's weights in the reference's own checkpoint files, as EncoderDecoderModel::save_model
// (src/EncoderDecoderModel.cpp:960-985) writes them: prefix.config through adai::binio with the
// format marker and version that save_model writes, then the encoder's, decoder's and head's own
// save_weights (which write their per-component files). The tokenizer's prefix.vocab is not
// written (it is not part of the decode arithmetic).
int ref_model_save(void* h, const char* prefix, int bos, int eos, int pad) {
    return guarded([&] {
        auto* m = static_cast<RefModel*>(h);
        const std::string p(prefix);
        adai::binio::Writer cfg(p + ".config");
        cfg.value(static_cast<int32_t>(-20260721), "format marker");
        cfg.value(static_cast<int32_t>(2), "format version");
        for (int field : {m->V, m->D, m->Le, m->L, m->H, m->F, m->max_seq, bos, eos, pad})
            cfg.value(field, "architecture");
        cfg.close();
        m->enc->save_weights(p + ".encoder");
        m->dec->save_weights(p + ".decoder");
        m->head->save_weights(p + ".lm_head");
    });
}

// TextGenerator::generate (src/TextGenerator.cpp:519-565) with every filter, over logits the caller
// supplies: the model function returns row (tokens generated so far) of logits [steps, V], so the
// sampler sees exactly these rows. fcfg = {temperature, top_p, repetition_penalty};
// icfg = {top_k, min_length, eos_token_id, pad_token_id, bos_token_id}. seed != 0 seeds the
// generator's mt19937 as TextGenerator(config, seed) does. prompt (n_prompt tokens) are the start
// tokens ({bos} when empty). out receives the whole generated sequence, start tokens included;
// *n_out its length (capacity n_prompt + steps, or steps + 1 when the prompt is empty).
int ref_sample_generate(const float* logits, int V, int steps, const float* fcfg, const int* icfg,
                        unsigned int seed, const int* prompt, int n_prompt, int* out, int* n_out) {
    return guarded([&] {
        TextGenerator::GenerationConfig cfg;
        cfg.max_length = steps;
        cfg.temperature = fcfg[0];
        cfg.top_p = fcfg[1];
        cfg.repetition_penalty = fcfg[2];
        cfg.top_k = icfg[0];
        cfg.min_length = icfg[1];
        cfg.eos_token_id = icfg[2];
        cfg.pad_token_id = icfg[3];
        cfg.bos_token_id = icfg[4];
        cfg.num_beams = 1;
        TextGenerator gen(cfg, seed);
        const int start = n_prompt > 0 ? n_prompt : 1;
        TextGenerator::ModelForwardFn fn = [&](const std::vector<int>& toks) {
            const size_t step = toks.size() - static_cast<size_t>(start);
            if (step >= static_cast<size_t>(steps)) throw std::runtime_error("past the last logits row");
            return from_flat(logits + step * static_cast<size_t>(V), 1, V);
        };
        std::vector<int> p(prompt, prompt + std::max(n_prompt, 0));
        std::vector<int> got = gen.generate(fn, p);
        std::copy(got.begin(), got.end(), out);
        *n_out = static_cast<int>(got.size());
    });
}

}  // extern "C"
