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

#ifdef __cplusplus
}
#endif
#endif
