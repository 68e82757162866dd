/*
 * adai_oracle.h — CPU restatement of the reference's batched-decode arithmetic.
 *
 * TEST INFRASTRUCTURE ONLY. tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg are
 * the only callers; the product (adai_b200/libadai_b200.so) never links or calls it.
 *
 * Every routine restates one reference routine in plain C, in fp32, in the reference's summation
 * order, and cites the file:line it follows (paths inside the kerfbit/adai source tree).
 * Pinned by tests/test_oracle.py against the reference itself (oracle/_ref, built from the
 * reference sources by oracle/Makefile) and against the committed fixtures in tests/golden/.
 *
 * Model weight order: identical to adai_b200_model_upload() (include/adai_b200.h).
 */
#ifndef ADAI_ORACLE_H
#define ADAI_ORACLE_H

#ifdef __cplusplus
extern "C" {
#endif

/* C[M,N] = A[M,K] B[K,N], each C[i][j] an in-order fused multiply-add chain over k starting from
 * 0 — the arithmetic of matmul_tile_avx2 (src/Matrix.cpp:75-91) under Matrix::operator*
 * (src/Matrix.cpp:212-277). */
void orc_matmul(const float* A, const float* B, float* C, int M, int K, int N);

/* LayerNorm::forward (src/LayerNorm.cpp:56-109): two-pass mean / biased variance, eps 1e-5. */
void orc_layernorm(const float* x, const float* g, const float* b, float* out, int rows, int D);

/* Activation::gelu, tanh approximation (src/Activation.cpp:69-86, src/ActivationConstants.hpp). */
void orc_gelu(const float* x, float* out, int n);

/* Activation::softmax_row (src/Activation.cpp:12-31). */
void orc_softmax_row(const float* in, float* out, int n);

/* PositionalEncoding table (src/PositionalEncoding.cpp:13-32). out [max_len, D]. */
void orc_pe_table(int max_len, int D, float* out);

/* Single-query attention over one sequence's K/V [T, D], all heads (src/MultiHeadAttention.cpp:
 * 336-367; CrossAttention is the same arithmetic, src/CrossAttention.cpp:432-455). */
void orc_attention_single(const float* q, const float* K, const float* V, int T, int D, int H,
                          float* out);

/* First index of the maximum (TextGenerator::argmax, src/TextGenerator.cpp:151-153). */
int orc_argmax(const float* v, int n);

/* ---- whole-model path ---- */
typedef struct orc_model orc_model;

/* cfg = {vocab, d_model, n_heads, d_ff, enc_layers, dec_layers, max_seq}; tensors in the upload
 * order. The model keeps pointers: the caller keeps the weights alive. Returns NULL on bad cfg. */
orc_model* orc_model_create(const int* cfg, const float* const* tensors);
void orc_model_destroy(orc_model* m);

/* LLMEncoder::encode_with_mask with an all-ones mask (src/LLMEncoder.cpp:120-142). */
int orc_encode(orc_model* m, const int* ids, int S, float* enc_out);

/* Greedy cached decode of one request (src/Decoder.cpp:210-287, src/LanguageModelHead.cpp:49-69,
 * src/TextGenerator.cpp:151-153), no stop tokens; forced != NULL teacher-forces step s with
 * forced[s]. logits [steps, V] may be NULL. */
int orc_generate(orc_model* m, const int* src, int S, int bos, int steps, const int* forced,
                 int* out_ids, float* logits);

/* ---- sampling (TextGenerator::generate, src/TextGenerator.cpp:519-565) ----
 * fcfg = {temperature, top_p, repetition_penalty}; icfg = {top_k, min_length, eos_token_id,
 * pad_token_id, bos_token_id} (GenerationConfig, src/TextGenerator.hpp:65-82). */

/* std::mt19937 state: st[0..623] and the read position st[624]. */
void orc_mt_seed(unsigned int* st, unsigned int seed);
unsigned int orc_mt_next(unsigned int* st);
/* std::generate_canonical<double, 53>(mt19937) as libstdc++ computes it (two draws). */
double orc_canonical(unsigned int* st);

/* One token from one logits row [V]: next_logits' checks and min_length mask, the repetition
 * penalty over seen[] (1 = token already in the sequence), temperature, top-k, top-p, then the
 * argmax (temperature <= 0) or a draw from std::discrete_distribution. Returns the token, -1 for
 * NaN/+inf logits, -2 when every logit is -inf. *margin (may be NULL) is how far the decision was
 * from changing: the smallest of the relative gap at the top-k cut, the distance of the running
 * probability sum from p at the top-p cut, the relative gap between the two best values (argmax),
 * and the distance of the uniform draw from its interval's ends (sampling); 0 at ties whose order
 * the reference leaves unspecified. */
int orc_sample_next(const float* logits, int V, const float* fcfg, const int* icfg,
                    const unsigned char* seen, int new_tokens, unsigned int* st, double* margin);

/* TextGenerator(config, seed).generate(fn, prompt) where fn returns row (new tokens so far) of
 * logits [steps, V]: stops after EOS or PAD. out (capacity max(n_prompt, 1) + steps) receives the
 * start tokens and the new ones; margins[s] the margin of step s. Returns the length of out, or a
 * negative orc_sample_next status. */
int orc_sample_generate(const float* logits, int V, int steps, const float* fcfg, const int* icfg,
                        unsigned int seed, const int* prompt, int n_prompt, int* out, double* margins);

#ifdef __cplusplus
}
#endif
#endif
