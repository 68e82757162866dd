/*
 * adai_b200.h — C ABI of the B200 (sm_100a) batched KV-cached decode step.
 *
 * Drop-in target: the GPU decode path of kerfbit/adai (paths below are inside that source tree).
 * Plain C types only (pointers, ints, floats); no CUDA or C++ types cross this boundary except
 * the opaque handles. Every call returns an adai_b200_status; adai_b200_last_error() gives the
 * message of the last failure on the calling thread.
 *
 * Threading: one context per GPU, used by one host thread at a time (the reference serialises its
 * GPU path the same way: EncoderDecoderModel::model_mutex_, src/EncoderDecoderModel.cpp:366 and
 * :1476, and the cuBLAS mutex, src/gpu/MatrixGPU.cu:356). Several contexts on several GPUs may be
 * driven from several threads at once; nothing is shared between contexts except the scratch
 * array of adai_b200_decode_attention_static (one per device).
 *
 * Layouts: host tensors are row-major fp32 exactly as the reference Matrix holds them
 * (src/Matrix.hpp:32); weights are W[in, out] as the reference setters take them.
 */
#ifndef ADAI_B200_H
#define ADAI_B200_H

#if defined(__GNUC__)
#define ADAI_B200_API __attribute__((visibility("default")))
#else
#define ADAI_B200_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
    ADAI_B200_OK = 0,
    ADAI_B200_ERR_INVALID_ARGUMENT = 1, /* std::invalid_argument in the reference */
    ADAI_B200_ERR_OUT_OF_RANGE = 2,     /* std::out_of_range (capacity, token id, slot) */
    ADAI_B200_ERR_CUDA = 3,             /* a CUDA runtime error (std::runtime_error, CUDA_CHECK) */
    ADAI_B200_ERR_TIMEOUT = 4,          /* a bounded wait expired; the context is marked unusable */
    ADAI_B200_ERR_NONFINITE = 5,        /* NaN/+inf logits (TextGenerator::next_logits throws) */
    ADAI_B200_ERR_STATE = 6,            /* call order (no model, context unusable, ...) */
    ADAI_B200_ERR_NO_DEVICE = 7,        /* no sm_100 device / the tensor-map API is missing */
    ADAI_B200_ERR_IO = 8                /* a checkpoint file cannot be opened or read */
} adai_b200_status;

typedef struct adai_b200_ctx adai_b200_ctx;
typedef struct adai_b200_kv adai_b200_kv;
typedef struct adai_b200_weight adai_b200_weight;

/* Model shape: the constructor arguments of LLMEncoder (src/encoder.hpp:90), LLMDecoder
 * (src/Decoder.hpp:125) and LanguageModelHead. */
typedef struct {
    int vocab;
    int d_model;
    int n_heads;    /* d_model / n_heads must be 32 or 64 */
    int d_ff;
    int enc_layers;
    int dec_layers;
    int max_seq;    /* positional-encoding table rows (PositionalEncoding(max_seq, d_model)) */
} adai_b200_model_desc;

/* Message of the last failed call on this thread ("" if none). */
ADAI_B200_API const char* adai_b200_last_error(void);

/* ---- context (replaces GPUManager: one device, one stream; src/gpu/GPUUtils.hpp:98-530) ---- */

/* Creates a context on `device`. mem_fraction in (0, 1] caps the device memory the context will
 * allocate (GPU_MEMORY_FRACTION, config.conf:262-300); 0 means no cap. */
ADAI_B200_API int adai_b200_ctx_create(int device, float mem_fraction, adai_b200_ctx** out);
ADAI_B200_API int adai_b200_ctx_destroy(adai_b200_ctx* ctx);
/* Bounded host wait for all queued work (GPUDebugSync wait with GPU_WAIT_TIMEOUT_SECONDS,
 * src/gpu/GPUDebugSync.cpp:236-244). On expiry returns ADAI_B200_ERR_TIMEOUT and marks the
 * context unusable (the reference marks the device lost). */
ADAI_B200_API int adai_b200_ctx_synchronize(adai_b200_ctx* ctx, double timeout_seconds);
/* Diagnostic of the timeout path (GPU_WAIT_TIMEOUT_SECONDS semantics, src/gpu/GPUDebugSync.cpp):
 * runs one device-side bounded wait on a barrier that nothing completes. The wait gives up after
 * its 2 s limit and records its code, a second wait returns at once because the error is already
 * recorded, and the kernel ends normally (no fault). The call then returns ADAI_B200_ERR_TIMEOUT
 * and the context is unusable, as after any device timeout; any other status means the path is
 * broken. waited_seconds (may be NULL) receives the host's wall time for the call. */
ADAI_B200_API int adai_b200_ctx_check_wait_timeout(adai_b200_ctx* ctx, double* waited_seconds);
/* The last GPU work this context queued, as "<seq> <phase> <kernel>": seq counts the launches
 * queued so far, phase is the entry point that queued the last one, kernel its name (a replayed
 * decode step is one launch, "decode step (CUDA graph)"). Replaces describe_last_gpu_work() over
 * the tag every reference kernel entry point stores (note_gpu_kernel,
 * src/gpu/GPUDebugSync.cpp:246-253); a failed or timed-out wait appends the same text to
 * adai_b200_last_error(). `buf` receives at most buf_len - 1 characters and a NUL; launches (may
 * be NULL) receives seq. */
ADAI_B200_API int adai_b200_ctx_last_work(adai_b200_ctx* ctx, char* buf, int buf_len,
                                          unsigned long long* launches);
/* Debug-sync settings of the process (ADAI_GPU_SYNC / ADAI_GPU_TRACE_FILE,
 * src/gpu/GPUDebugSync.hpp:5-22), read from ADAI_B200_SYNC (else ADAI_GPU_SYNC) and
 * ADAI_B200_TRACE_FILE (else ADAI_GPU_TRACE_FILE) on first use:
 *   mode 0 (off), 1 (step: every entry point waits for its work before it returns), 2 (kernel:
 *   also wait before every `every`-th launch, and the decode step runs its kernels one by one
 *   instead of replaying its graph, so a failure names the kernel that ran);
 *   trace_file: "<seq> <phase> <kernel>" of the last launch, rewritten in place.
 * Every wait is the bounded one of adai_b200_ctx_synchronize. */
/* Parses an ADAI_B200_SYNC value: "off", "step", "kernel" or "kernel:N" (1 <= N <= 1000000);
 * NULL or "" is off. A value it cannot read returns ADAI_B200_ERR_INVALID_ARGUMENT (mode stays
 * 0), as parse_gpu_debug_settings records a problem and keeps the default. Host only. */
ADAI_B200_API int adai_b200_debug_sync_parse(const char* value, int* mode, unsigned* every);
/* Replaces the process's settings (tools and tests; set_gpu_debug_settings_for_testing).
 * trace_file may be NULL (no file). */
ADAI_B200_API int adai_b200_debug_configure(int mode, unsigned every, const char* trace_file);
/* The process's current settings (mode, every). Host only. */
ADAI_B200_API int adai_b200_debug_settings(int* mode, unsigned* every);
/* Device bytes this context holds. */
ADAI_B200_API int adai_b200_ctx_memory(adai_b200_ctx* ctx, unsigned long long* bytes);
/* The CUDA stream (as void*) the context launches on. */
ADAI_B200_API void* adai_b200_ctx_stream(adai_b200_ctx* ctx);

/* ---- model weights ---- */

/* Number of tensors adai_b200_model_upload expects for `desc`. */
ADAI_B200_API int adai_b200_model_tensor_count(const adai_b200_model_desc* desc);

/* Copies the model to the device (host fp32 row-major). Tensor order:
 *   enc.embed[V,D]
 *   per encoder layer: ln1.g[D] ln1.b[D] wq wk wv wo[D,D] ln2.g ln2.b w1[D,F] b1[F] w2[F,D] b2[D]
 *   enc.lnf.g enc.lnf.b
 *   dec.embed[V,D]
 *   per decoder layer: ln1.g ln1.b sa.wq sa.wk sa.wv sa.wo ln2.g ln2.b ca.wq ca.wk ca.wv ca.wo
 *                      ln3.g ln3.b w1 b1 w2 b2
 *   dec.lnf.g dec.lnf.b head.w[D,V] head.b[V]
 * i.e. the setters MultiHeadAttention::set_W* (src/MultiHeadAttention.cpp:630-652),
 * CrossAttention::set_W* (src/CrossAttention.cpp:717-739), FeedForward::set_W1/b1/W2/b2
 * (src/FeedForward.hpp:201-212), LayerNorm::set_gamma/set_beta (src/LayerNorm.cpp:218-234),
 * TokenEmbedding::set_embeddings (src/TokenEmbedding.hpp:259), LanguageModelHead::set_W_output /
 * set_bias (src/LanguageModelHead.cpp:145-160). Weights are copied; a later change on the host
 * needs a new upload (the reference's refresh_gpu_mirror, src/MultiHeadAttention.cpp:654-660).
 * pe_table [max_seq, d_model] may be NULL: the table of src/PositionalEncoding.cpp:13-32 is then
 * computed on the host. Replaces the previous model, if any. */
ADAI_B200_API int adai_b200_model_upload(adai_b200_ctx* ctx, const adai_b200_model_desc* desc,
                           const float* const* tensors, const float* pe_table);

/* ---- checkpoints (host only, no device needed unless stated). `path` is either
 * (1) a SafeTensors directory (ModelSerializer::export_safetensors / import_safetensors,
 *     src/ModelSerializer.cpp:243-391 and :395-579): path/config.json and path/model.safetensors,
 *     T5-style tensor names, projections stored [out, in], F32; or
 * (2) the prefix given to the reference's EncoderDecoderModel::save_model (src/EncoderDecoderModel.cpp:
 *     960-985): path.config, path.encoder, path.decoder, path.lm_head and the per-component files
 *     the encoder and decoder write beside them, in the adai::binio layout (src/BinaryIO.cpp).
 * The format is told by which of path/config.json and path.config exists. ----
 * Reads the model shape. */
ADAI_B200_API int adai_b200_checkpoint_config(const char* path, adai_b200_model_desc* out);
/* The checkpoint's BOS, EOS and PAD ids (config.json: decoder_start_token_id, eos_token_id,
 * pad_token_id; path.config: its last three fields). Any output may be NULL. */
ADAI_B200_API int adai_b200_checkpoint_special_tokens(const char* path, int* bos, int* eos,
                                                      int* pad);
/* Reads the tensors into caller buffers, in the order and layouts of adai_b200_model_upload.
 * SafeTensors: projections back to W[in, out]; a file with no model.decoder.embed_tokens.weight
 * gives the decoder model.shared.weight, and one with no final LayerNorm gives gamma 1 / beta 0,
 * as the reference's import does; tensors not used here are ignored.
 * save_model files: every file is checked as the reference's loaders check it (each dimension,
 * no trailing bytes); an encoder without its own token_emb / final_norm files takes the shared
 * path_token_emb.bin / path_final_norm.bin, as the reference does for older checkpoints
 * (src/LLMEncoder.cpp:326-349). Final LayerNorm files must hold epsilon 1e-5 (the kernels' value,
 * the reference's default), and decoder blocks with a gated world-model or hippocampal path are
 * refused.
 * Errors: ADAI_B200_ERR_INVALID_ARGUMENT naming the tensor or file (missing tensor, wrong shape or
 * dimension, dtype other than F32, trailing data, bad format marker), ADAI_B200_ERR_IO (a file that
 * is missing, unreadable or cut short). */
ADAI_B200_API int adai_b200_checkpoint_read(const char* path, const adai_b200_model_desc* desc,
                                            float* const* tensors);
/* adai_b200_checkpoint_config + adai_b200_checkpoint_read + adai_b200_model_upload. When expect
 * is non-NULL the checkpoint's shape must equal it (the reference's architecture checks,
 * src/ModelSerializer.cpp:410-432, src/EncoderDecoderModel.cpp:1030-1047), else
 * ADAI_B200_ERR_INVALID_ARGUMENT. */
ADAI_B200_API int adai_b200_model_load(adai_b200_ctx* ctx, const char* path,
                                       const adai_b200_model_desc* expect);

/* ---- KV cache arena (replaces GPUDecoderKVCache, src/gpu/MatrixGPU.hpp:563-623, and the CPU
 * DecoderKVCache, src/KVCache.hpp:155-245) ----
 * `max_slots` sequences, each with dec_layers self caches of `self_capacity` rows and cross
 * caches of `cross_capacity` rows (fixed capacity, as GPUKVCache's max_seq_length). */
ADAI_B200_API int adai_b200_kv_create(adai_b200_ctx* ctx, int max_slots, int self_capacity, int cross_capacity,
                        adai_b200_kv** out);
ADAI_B200_API int adai_b200_kv_destroy(adai_b200_ctx* ctx, adai_b200_kv* kv);
/* DecoderKVCache::clear() for one slot (self and cross). */
ADAI_B200_API int adai_b200_kv_reset(adai_b200_ctx* ctx, adai_b200_kv* kv, int slot);
/* DecoderKVCache::clear_self_attention() for one slot (src/KVCache.hpp:190-196): the decoder
 * restarts at position 0 over the same encoder output. */
ADAI_B200_API int adai_b200_kv_clear_self(adai_b200_ctx* ctx, adai_b200_kv* kv, int slot);
/* Rows currently cached for a slot (DecoderKVCache::current_length, src/KVCache.hpp:235-244). */
ADAI_B200_API int adai_b200_kv_length(adai_b200_ctx* ctx, adai_b200_kv* kv, int slot, int* self_len,
                        int* cross_len);

/* ---- encoder prefill + cross K/V (LLMEncoder::encode_with_mask, src/LLMEncoder.cpp:120-142,
 * with CrossAttention's first-call K/V projection, src/CrossAttention.cpp:388-413) ----
 * n requests; request i has src_lens[i] source ids (concatenated in ids) and is placed in slot
 * slots[i], whose self cache is cleared. Host arrays. Optionally returns the encoder output
 * [sum(src_lens), d_model] (enc_out may be NULL). A source may be empty, as in the reference
 * (only max_seq bounds it, src/LLMEncoder.cpp:106-122): it has no encoder rows, and the slot's
 * cross-attention contributes zeros. */
ADAI_B200_API int adai_b200_encode(adai_b200_ctx* ctx, adai_b200_kv* kv, int n, const int* slots,
                     const int* ids, const int* src_lens, float* enc_out);

/* ---- one stacked decode step (LLMDecoder::forward_with_cache, src/Decoder.cpp:210-287, for B
 * sequences at once; LanguageModelHead::forward, src/LanguageModelHead.cpp:49-69; greedy
 * TextGenerator::argmax, src/TextGenerator.cpp:151-153) ----
 * Feeds ids[b] to sequence slots[b], appends one row to its self caches and returns the first
 * maximum of its logits in next_ids[b]. logits [B, vocab] may be NULL. Host arrays; the call
 * waits for the result. Fails with ADAI_B200_ERR_NONFINITE where the reference's
 * TextGenerator::next_logits would throw (NaN or +inf logit, or every logit -inf). */
ADAI_B200_API int adai_b200_decode_step(adai_b200_ctx* ctx, adai_b200_kv* kv, int B, const int* slots,
                          const int* ids, int* next_ids, float* logits);

/* Greedy decode of `steps` tokens for B sequences, all on the device: the step is captured once
 * in a CUDA graph and replayed, the argmax fed back on the device. first_ids[b] is the first
 * token fed (BOS = 2 for a fresh request); out_ids [B, steps] receives step s's argmax in column
 * s. Host arrays. The same arithmetic as `steps` calls of adai_b200_decode_step. */
ADAI_B200_API int adai_b200_generate(adai_b200_ctx* ctx, adai_b200_kv* kv, int B, const int* slots,
                       const int* first_ids, int steps, int* out_ids);

/* ---- sampling (TextGenerator::generate, src/TextGenerator.cpp:519-565; GenerationConfig,
 * src/TextGenerator.hpp:65-82) ----
 * A slot configured with adai_b200_kv_set_sampling picks its tokens, in adai_b200_decode_step and
 * adai_b200_generate alike, by the reference's rules instead of the plain argmax: min_length keeps
 * EOS and PAD out while fewer new tokens exist (:197-203); the repetition penalty divides positive
 * and multiplies other logits of every distinct token already in the sequence (:115-136); then
 * temperature (:26-38), top-k (:41-63), top-p (:66-101); temperature <= 0 takes the first maximum
 * of the filtered logits, otherwise the token is drawn from their softmax with the slot's own
 * std::mt19937 through std::discrete_distribution as GCC's libstdc++ computes it (:145-148).
 * Every strategy of the reference is a setting of these fields: generate_greedy (:209) is
 * temperature <= 0, generate_sampling (:398) top_k 0 and top_p 1, generate_top_k (:438) top_p 1,
 * generate_nucleus (:475) top_k 0. Exactly tied values at the top-k / top-p cut are kept lowest
 * index first (the reference's std::partial_sort / std::sort leave that order unspecified). */
typedef struct adai_b200_sampling {
    float temperature;        /* <= 0: argmax of the filtered logits; 1: unscaled */
    int top_k;                /* <= 0 or >= vocab: off */
    float top_p;              /* >= 1: off; <= 0: the single most likely token */
    float repetition_penalty; /* 1: off; must be finite and positive */
    int min_length;           /* new tokens before EOS / PAD may be chosen */
    int eos_token_id;         /* masked while below min_length (3 in the reference) */
    int pad_token_id;         /* masked while below min_length (0 in the reference) */
    unsigned int seed;        /* std::mt19937 seed; 0 draws one from std::random_device */
} adai_b200_sampling;

/* Configures slot `slot` for sampling (cfg NULL: back to the fused argmax, as after
 * adai_b200_kv_reset), seeds its generator and resets its count of new tokens. history holds the
 * ids already in the sequence before the first token fed (the reference's start tokens beyond the
 * one fed first; may be NULL when n_history is 0). Each step then counts the id fed as part of the
 * sequence, so after the usual BOS feed the penalty set is exactly the reference's `generated`.
 * The whole logits row is held in shared memory: vocab is limited to 56 320 (55 Ki). */
ADAI_B200_API int adai_b200_kv_set_sampling(adai_b200_ctx* ctx, adai_b200_kv* kv, int slot,
                                            const adai_b200_sampling* cfg, const int* history,
                                            int n_history);

/* The slot's generator state (625 words: std::mt19937's 624 state words, then the read position)
 * and its count of sampled steps. Either output may be NULL. */
ADAI_B200_API int adai_b200_kv_sampling_state(adai_b200_ctx* ctx, adai_b200_kv* kv, int slot,
                                              unsigned int* mt_state, int* new_tokens);

/* Op level: picks one token per row of device logits [B, ld] (ld >= vocab) for slots[b] (each
 * configured for sampling), with fed_ids[b] (host; may be NULL) counted into the sequence first,
 * exactly as a decode step does after its LM head. Advances the slots' generators and counts.
 * next_ids: host. Fails with ADAI_B200_ERR_NONFINITE for a NaN / +inf row or one without a finite
 * value (TextGenerator::next_logits, :177-206). */
ADAI_B200_API int adai_b200_sample_logits(adai_b200_ctx* ctx, adai_b200_kv* kv, int B,
                                          const int* slots, const int* fed_ids,
                                          const float* logits, int ld, int* next_ids);

/* ---- op level: stacked GEMM (Matrix::operator*, src/Matrix.cpp:212-277; matrix_multiply_gpu,
 * src/gpu/MatrixGPU.hpp:100 and src/gpu/MatrixGPU.cu:351-370) ----
 * C[m,n] = A[m,k] B[k,n], fp32 in and out, 3xTF32 on the tensor cores. Device pointers on the
 * context's stream; asynchronous. B is prepared (transposed and split) on every call; use
 * adai_b200_weight_create + adai_b200_sgemm_prepared to prepare it once. */
ADAI_B200_API int adai_b200_sgemm(adai_b200_ctx* ctx, int m, int n, int k, const float* A, const float* B,
                    float* C);
/* Prepares B [k, n] (device pointer) once for repeated products. */
ADAI_B200_API int adai_b200_weight_create(adai_b200_ctx* ctx, const float* B, int k, int n,
                            adai_b200_weight** out);
ADAI_B200_API int adai_b200_weight_destroy(adai_b200_ctx* ctx, adai_b200_weight* w);
ADAI_B200_API int adai_b200_sgemm_prepared(adai_b200_ctx* ctx, int m, const float* A, const adai_b200_weight* w,
                             float* C);

/* ---- op level: single-token attention over a KV cache with the append fused in
 * (MultiHeadAttention::forward_with_cache, src/MultiHeadAttention.cpp:278-395, per-head math
 * :336-367; KVCache::append, src/KVCache.hpp:99-128) ----
 * B sequences, H heads of width head_dim (32 or 64), D = H * head_dim. Cache layout
 * [B][H][capacity][head_dim] (K and V). All pointers are 16-byte aligned device pointers (rows
 * are read and written as float4). lens[b] rows are cached
 * for sequence b (max_len >= every lens[b]); when k_new/v_new [B, D] are non-NULL they are
 * appended at row lens[b] first and attention runs over lens[b] + 1 rows (lens is not updated).
 * q [B, D]; out [B, D]. Asynchronous on the context's stream. */
ADAI_B200_API int adai_b200_decode_attention(adai_b200_ctx* ctx, int B, int H, int head_dim,
                                             int capacity, const float* q, const float* k_new,
                                             const float* v_new, float* k_cache, float* v_cache,
                                             const int* lens, int max_len, float* out);

/* No counterpart in the reference. adai_b200_decode_attention for callers that must not allocate
 * device memory at call time: a host that has reserved all free device memory for its own pool,
 * or a serving loop that forbids allocation (a device allocation can stall every stream of the
 * device). Same arguments, same arithmetic and same results as adai_b200_decode_attention, but
 * the split-KV scratch is a fixed 16 MiB array inside this library's device image (per device),
 * so the call allocates and frees nothing.
 * Limits: B * H <= 16384, and the split partials, B * H * ceil((max_len + appended) / 256) *
 * (head_dim + 4) floats, must fit in 16 MiB - 64 KiB (B = 256, H = 16, head_dim = 64 fits while
 * max_len + appended <= 3840); larger calls return ADAI_B200_ERR_OUT_OF_RANGE and launch nothing.
 * The first call on each device does a one-time setup (zeroes the array's merge counters on
 * ctx's stream and waits for that); make that first call before any stream capture.
 * The array is shared by every caller on a device: calls that overlap in time on one device race
 * and corrupt each other's results. Serializing the host calls is not enough (each call only
 * queues a kernel): calls on different streams or contexts of one device must also be ordered on
 * the device (one stream, events, or a synchronize between them).
 * A lens[b] outside [0, max_len] is refused by the kernel: that pair computes nothing, and the
 * next adai_b200_ctx_synchronize returns ADAI_B200_ERR_OUT_OF_RANGE (also for
 * adai_b200_decode_attention). */
ADAI_B200_API int adai_b200_decode_attention_static(adai_b200_ctx* ctx, int B, int H, int head_dim,
                                                    int capacity, const float* q,
                                                    const float* k_new, const float* v_new,
                                                    float* k_cache, float* v_cache,
                                                    const int* lens, int max_len, float* out);

/* ---- op level: LayerNorm (LayerNorm::forward, src/LayerNorm.cpp:56-109; the reference GPU
 * kernel matrix_layer_norm_fwd_gpu, src/gpu/MatrixGPU.hpp:140) ----
 * out[rows, D] = gamma * (x - mean) / sqrt(var + 1e-5) + beta. Device pointers; D a multiple of
 * 128 up to 2048. */
ADAI_B200_API int adai_b200_layernorm(adai_b200_ctx* ctx, const float* x, const float* gamma, const float* beta,
                        float* out, int rows, int D);

/* ---- the decode-path entries of the reference GPU backend table (adai::gpu::matrix_*_gpu,
 * src/gpu/MatrixGPU.hpp:43-201), for callers of that table outside the fused decode step. Device
 * pointers, row-major, on the context's stream. include/adai_b200_backend.hpp gives them the
 * reference's own C++ signatures. ---- */
/* C[m, n] (row stride ldc) = alpha * op(A) * op(B); op(A) is m x k (A stored k x m when trans_a),
 * op(B) is k x n (B stored n x k when trans_b); beta = 0 (matrix_gemm_strided_gpu,
 * src/gpu/MatrixGPU.hpp:92-100). 3xTF32 on the tensor cores; waits for completion. */
ADAI_B200_API int adai_b200_gemm_strided(adai_b200_ctx* ctx, int trans_a, int trans_b, int m, int n,
                                         int k, float alpha, const float* a, int lda,
                                         const float* b, int ldb, float* c, int ldc);
/* In-place row softmax, Activation::softmax_row semantics (src/Activation.cpp:12-31): a row whose
 * exponentials sum to 0 is left unnormalised (matrix_softmax_rows_gpu). */
ADAI_B200_API int adai_b200_softmax_rows(adai_b200_ctx* ctx, float* data, int rows, int cols);
/* y = gamma * (x - mean) * rstd + beta per row, any width; x_normed, mean, rstd may be NULL
 * (matrix_layer_norm_fwd_gpu, src/gpu/MatrixGPU.hpp:147-149). */
ADAI_B200_API int adai_b200_layernorm_fwd(adai_b200_ctx* ctx, const float* x, float* y,
                                          float* x_normed, const float* gamma, const float* beta,
                                          float* mean, float* rstd, int rows, int cols, float eps);
/* out[r, c] = m[r, c] + bias[c] (matrix_add_row_bias_gpu). */
ADAI_B200_API int adai_b200_add_row_bias(adai_b200_ctx* ctx, const float* m, const float* bias,
                                         float* out, int rows, int cols);
/* In place: type 0 ReLU, 1 sigmoid, 2 tanh, 3 GELU (tanh form), the ActivationType values of
 * src/gpu/MatrixGPU.hpp:27 (matrix_apply_activation_gpu). */
ADAI_B200_API int adai_b200_activation(adai_b200_ctx* ctx, float* data, int size, int type);
/* out[i, :] = table[ids[i], :] + pe[pos_offset + i, :], no positional row past pe_rows or when pe
 * is NULL (embedding_gather_add_pe_gpu, src/gpu/MatrixGPU.hpp:182-185). With vocab > 0 an id
 * outside [0, vocab) is reported by the next synchronisation as ADAI_B200_ERR_OUT_OF_RANGE. */
ADAI_B200_API int adai_b200_embedding_gather_add_pe(adai_b200_ctx* ctx, const float* table,
                                                    const int* ids, const float* pe, int pe_rows,
                                                    int pos_offset, float* out, int n, int d,
                                                    int vocab);
/* The context the adai::gpu::matrix_*_gpu functions of include/adai_b200_backend.hpp run on (one
 * per process, as the reference's GPUManager singleton; NULL unbinds). */
ADAI_B200_API int adai_b200_backend_bind(adai_b200_ctx* ctx);

/* ---- measurement ----
 * Device time (CUDA events on the context stream, around the graph replays) of the decode loop
 * of the last adai_b200_generate call, and the kernels one replayed step launches. The reference
 * reports the same figure as ms/token from its decode benchmark
 * (benchmarks/GpuDecodeBenchmark.cpp:383-420). */
ADAI_B200_API int adai_b200_ctx_last_timing(adai_b200_ctx* ctx, double* decode_ms,
                                            int* kernels_per_step);

typedef enum {
    ADAI_B200_KC_GEMM = 0,       /* stacked projections: Q|K|V, W_o, cross W_q / W_o, FFN */
    ADAI_B200_KC_SELF_ATTN = 1,  /* decode self-attention with the fused KV append */
    ADAI_B200_KC_CROSS_ATTN = 2, /* decode cross-attention over the encoder K/V */
    ADAI_B200_KC_NORM = 3,       /* LayerNorms, embedding + positional row */
    ADAI_B200_KC_HEAD = 4,       /* LM head GEMM with the fused argmax */
    ADAI_B200_KC_OTHER = 5,      /* step bookkeeping */
    ADAI_B200_KC_COUNT = 6
} adai_b200_kernel_class;

/* Runs one decode step like adai_b200_decode_step (ids fed, one row appended per sequence) but
 * launched eagerly with a CUDA event pair around every kernel, and returns per kernel class the
 * summed device time (ms), the algorithmic bytes and flops the launches had to move / compute
 * (GEMM: 4(MK+KN+MN) bytes, 2MNK flops; attention: the K/V rows read, q read, output written)
 * and the launch count. Arrays hold n_classes >= ADAI_B200_KC_COUNT entries. */
ADAI_B200_API int adai_b200_profile_step(adai_b200_ctx* ctx, adai_b200_kv* kv, int B,
                                         const int* slots, const int* ids, int n_classes,
                                         double* ms, double* bytes, double* flops,
                                         int* launches);

#ifdef __cplusplus
}
#endif
#endif /* ADAI_B200_H */
