/*
 * adai_oracle.c — CPU restatement of the reference's decode-path arithmetic, in plain C.
 *
 * TEST INFRASTRUCTURE ONLY (see adai_oracle.h). Pinned against the reference build
 * (oracle/_ref/libadai_ref.so) and the fixtures in tests/golden/ by tests/test_oracle.py.
 *
 * Each function restates the cited reference routine in fp32 and in the reference's order of
 * operations; the only intended differences are the ones -ffast-math allows the reference
 * compiler (vectorised reductions in LayerNorm/softmax), which stay far inside the parity
 * tolerance |a-b| <= 1e-5 + 1e-4|b|.
 */
#include "adai_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

/* src/Matrix.cpp:75-91 (matmul_tile_avx2): for each k in order, c[j] = fma(a[k], b[k][j], c[j]);
 * src/Matrix.cpp:258-274 tiles rows x 256-column blocks; the per-element sum order is the same
 * for every tiling, so rows run in parallel here without changing any result. */
void orc_matmul(const float* A, const float* B, float* C, int M, int K, int N) {
    long long work = (long long)M * K * N;
#pragma omp parallel for schedule(static) if (work > (1LL << 18) && M > 1)
    for (int i = 0; i < M; ++i) {
        float* c = C + (size_t)i * N;
        const float* a = A + (size_t)i * K;
        for (int j = 0; j < N; ++j) c[j] = 0.0f;
        for (int k = 0; k < K; ++k) {
            const float av = a[k];
            const float* b = B + (size_t)k * N;
            for (int j = 0; j < N; ++j) c[j] = fmaf(av, b[j], c[j]);
        }
    }
}

/* src/LayerNorm.cpp:56-109 and src/LayerNorm.hpp:70 (eps = 1e-5). */
void orc_layernorm(const float* x, const float* g, const float* b, float* out, int rows, int D) {
    for (int i = 0; i < rows; ++i) {
        const float* r = x + (size_t)i * D;
        float* o = out + (size_t)i * D;
        float mean = 0.0f;
        for (int j = 0; j < D; ++j) mean += r[j];
        mean /= (float)D;
        float var = 0.0f;
        for (int j = 0; j < D; ++j) {
            float d = r[j] - mean;
            var += d * d;
        }
        var /= (float)D;
        float inv_std = 1.0f / sqrtf(var + 1e-5f);
        for (int j = 0; j < D; ++j) o[j] = g[j] * ((r[j] - mean) * inv_std) + b[j];
    }
}

/* src/Activation.cpp:69-86 with src/ActivationConstants.hpp:18-19. */
void orc_gelu(const float* x, float* out, int n) {
    for (int i = 0; i < n; ++i) {
        float v = x[i];
        float cube = v * v * v;
        float inner = 0.7978845608f * (v + 0.044715f * cube);
        out[i] = 0.5f * v * (1.0f + tanhf(inner));
    }
}

/* src/Activation.cpp:12-31: max-subtracted exp, divided by the sum unless the sum is <= 0. */
void orc_softmax_row(const float* in, float* out, int n) {
    if (n <= 0) return;
    float mx = in[0];
    for (int j = 1; j < n; ++j) mx = in[j] > mx ? in[j] : mx;
    float sum = 0.0f;
    for (int j = 0; j < n; ++j) {
        out[j] = expf(in[j] - mx);
        sum += out[j];
    }
    if (sum > 0.0f)
        for (int j = 0; j < n; ++j) out[j] /= sum;
}

/* src/PositionalEncoding.cpp:13-32. */
void orc_pe_table(int max_len, int D, float* out) {
    for (int pos = 0; pos < max_len; ++pos)
        for (int i = 0; i < D; ++i) {
            float angle = (float)pos / powf(10000.0f, (2.0f * (float)(i / 2)) / (float)D);
            out[(size_t)pos * D + i] = (i % 2 == 0) ? sinf(angle) : cosf(angle);
        }
}

/* src/MultiHeadAttention.cpp:336-367: per head h, scores = (Q_h K_h^T) * (1/sqrt(dk)) with each
 * score an in-order fma chain over the head's dk columns (Matrix::operator*), softmax_row, then
 * out_h = weights * V_h (again an in-order fma chain over t). */
void orc_attention_single(const float* q, const float* K, const float* V, int T, int D, int H,
                          float* out) {
    const int dk = D / H;
    const float scale = 1.0f / sqrtf((float)dk);
    float* s = (float*)malloc(sizeof(float) * (size_t)(T > 0 ? T : 1));
    float* w = (float*)malloc(sizeof(float) * (size_t)(T > 0 ? T : 1));
    for (int h = 0; h < H; ++h) {
        const int c0 = h * dk;
        for (int t = 0; t < T; ++t) {
            float acc = 0.0f;
            const float* kr = K + (size_t)t * D + c0;
            for (int j = 0; j < dk; ++j) acc = fmaf(q[c0 + j], kr[j], acc);
            s[t] = acc * scale;
        }
        orc_softmax_row(s, w, T);
        for (int j = 0; j < dk; ++j) out[c0 + j] = 0.0f;
        for (int t = 0; t < T; ++t) {
            const float* vr = V + (size_t)t * D + c0;
            for (int j = 0; j < dk; ++j) out[c0 + j] = fmaf(w[t], vr[j], out[c0 + j]);
        }
    }
    free(s);
    free(w);
}

/* Encoder self-attention (src/MultiHeadAttention.cpp:176-240): every query row attends over all
 * S rows (the all-ones mask never fires); Q/K/V [S, D]. */
static void attention_full(const float* Q, const float* K, const float* V, int S, int D, int H,
                           float* out) {
    for (int i = 0; i < S; ++i)
        orc_attention_single(Q + (size_t)i * D, K, V, S, D, H, out + (size_t)i * D);
}

int orc_argmax(const float* v, int n) {
    int best = 0;
    for (int j = 1; j < n; ++j)
        if (v[j] > v[best]) best = j;
    return best;
}

/* ------------------------------------------------------------------------------------------ */

typedef struct {
    const float *ln1g, *ln1b, *wq, *wk, *wv, *wo, *ln2g, *ln2b, *w1, *b1, *w2, *b2;
} enc_layer;

typedef struct {
    const float *ln1g, *ln1b, *sq, *sk, *sv, *so, *ln2g, *ln2b, *cq, *ck, *cv, *co, *ln3g, *ln3b,
        *w1, *b1, *w2, *b2;
} dec_layer;

struct orc_model {
    int V, D, H, F, Le, L, max_seq;
    const float *enc_embed, *enc_lnf_g, *enc_lnf_b, *dec_embed, *dec_lnf_g, *dec_lnf_b, *head_w,
        *head_b;
    enc_layer* enc;
    dec_layer* dec;
    float* pe;
};

orc_model* orc_model_create(const int* cfg, const float* const* t) {
    if (cfg[0] <= 0 || cfg[1] <= 0 || cfg[2] <= 0 || cfg[1] % cfg[2] != 0 || cfg[3] <= 0 ||
        cfg[4] < 0 || cfg[5] <= 0 || cfg[6] <= 0)
        return NULL;
    orc_model* m = (orc_model*)calloc(1, sizeof(orc_model));
    m->V = cfg[0];
    m->D = cfg[1];
    m->H = cfg[2];
    m->F = cfg[3];
    m->Le = cfg[4];
    m->L = cfg[5];
    m->max_seq = cfg[6];
    int k = 0;
    m->enc_embed = t[k++];
    m->enc = (enc_layer*)calloc((size_t)(m->Le > 0 ? m->Le : 1), sizeof(enc_layer));
    for (int i = 0; i < m->Le; ++i) {
        enc_layer* e = &m->enc[i];
        e->ln1g = t[k++]; e->ln1b = t[k++];
        e->wq = t[k++]; e->wk = t[k++]; e->wv = t[k++]; e->wo = t[k++];
        e->ln2g = t[k++]; e->ln2b = t[k++];
        e->w1 = t[k++]; e->b1 = t[k++]; e->w2 = t[k++]; e->b2 = t[k++];
    }
    m->enc_lnf_g = t[k++];
    m->enc_lnf_b = t[k++];
    m->dec_embed = t[k++];
    m->dec = (dec_layer*)calloc((size_t)m->L, sizeof(dec_layer));
    for (int i = 0; i < m->L; ++i) {
        dec_layer* d = &m->dec[i];
        d->ln1g = t[k++]; d->ln1b = t[k++];
        d->sq = t[k++]; d->sk = t[k++]; d->sv = t[k++]; d->so = t[k++];
        d->ln2g = t[k++]; d->ln2b = t[k++];
        d->cq = t[k++]; d->ck = t[k++]; d->cv = t[k++]; d->co = t[k++];
        d->ln3g = t[k++]; d->ln3b = t[k++];
        d->w1 = t[k++]; d->b1 = t[k++]; d->w2 = t[k++]; d->b2 = t[k++];
    }
    m->dec_lnf_g = t[k++];
    m->dec_lnf_b = t[k++];
    m->head_w = t[k++];
    m->head_b = t[k++];
    m->pe = (float*)malloc(sizeof(float) * (size_t)m->max_seq * m->D);
    orc_pe_table(m->max_seq, m->D, m->pe);
    return m;
}

void orc_model_destroy(orc_model* m) {
    if (!m) return;
    free(m->enc);
    free(m->dec);
    free(m->pe);
    free(m);
}

/* FeedForward::forward (src/FeedForward.cpp:66-108): h = gelu(x W1 + b1); y = h W2 + b2. */
static void ffn(const float* x, int rows, int D, int F, const float* w1, const float* b1,
                const float* w2, const float* b2, float* y, float* hbuf) {
    orc_matmul(x, w1, hbuf, rows, D, F);
    for (int i = 0; i < rows; ++i)
        for (int j = 0; j < F; ++j) hbuf[(size_t)i * F + j] += b1[j];
    orc_gelu(hbuf, hbuf, rows * F);
    orc_matmul(hbuf, w2, y, rows, F, D);
    for (int i = 0; i < rows; ++i)
        for (int j = 0; j < D; ++j) y[(size_t)i * D + j] += b2[j];
}

int orc_encode(orc_model* m, const int* ids, int S, float* out) {
    const int D = m->D, F = m->F, H = m->H;
    /* no lower bound: an empty source encodes to no rows, and cross-attention over no rows gives
     * zeros (src/LLMEncoder.cpp:106-122 checks only the upper bound) */
    if (S < 0 || S > m->max_seq) return -1;
    if (S == 0) return 0;
    for (int i = 0; i < S; ++i)
        if (ids[i] < 0 || ids[i] >= m->V) return -1;
    size_t n = (size_t)S * D;
    float* x = (float*)malloc(sizeof(float) * n);
    float* nrm = (float*)malloc(sizeof(float) * n);
    float* q = (float*)malloc(sizeof(float) * n);
    float* k = (float*)malloc(sizeof(float) * n);
    float* v = (float*)malloc(sizeof(float) * n);
    float* a = (float*)malloc(sizeof(float) * n);
    float* o = (float*)malloc(sizeof(float) * n);
    float* h = (float*)malloc(sizeof(float) * (size_t)S * F);
    /* TokenEmbedding::forward + PositionalEncoding::forward (src/LLMEncoder.cpp:129-133) */
    for (int i = 0; i < S; ++i)
        for (int j = 0; j < D; ++j)
            x[(size_t)i * D + j] = m->enc_embed[(size_t)ids[i] * D + j] + m->pe[(size_t)i * D + j];
    /* EncoderBlock::forward (src/EncoderBlock.cpp:34-77), pre-LN */
    for (int l = 0; l < m->Le; ++l) {
        const enc_layer* e = &m->enc[l];
        orc_layernorm(x, e->ln1g, e->ln1b, nrm, S, D);
        orc_matmul(nrm, e->wq, q, S, D, D);
        orc_matmul(nrm, e->wk, k, S, D, D);
        orc_matmul(nrm, e->wv, v, S, D, D);
        attention_full(q, k, v, S, D, H, a);
        orc_matmul(a, e->wo, o, S, D, D);
        for (size_t i = 0; i < n; ++i) x[i] = x[i] + o[i];
        orc_layernorm(x, e->ln2g, e->ln2b, nrm, S, D);
        ffn(nrm, S, D, F, e->w1, e->b1, e->w2, e->b2, o, h);
        for (size_t i = 0; i < n; ++i) x[i] = x[i] + o[i];
    }
    orc_layernorm(x, m->enc_lnf_g, m->enc_lnf_b, out, S, D);
    free(x); free(nrm); free(q); free(k); free(v); free(a); free(o); free(h);
    return 0;
}

int orc_generate(orc_model* m, const int* src, int S, int bos, int steps, const int* forced,
                 int* out_ids, float* logits) {
    const int D = m->D, F = m->F, H = m->H, V = m->V, L = m->L;
    if (steps <= 0) return 0;
    float* enc = (float*)malloc(sizeof(float) * (size_t)S * D);
    if (orc_encode(m, src, S, enc) != 0) {
        free(enc);
        return -1;
    }
    /* DecoderKVCache (src/KVCache.hpp:155-245): per layer, self K/V grow by one row per step;
     * cross K/V = enc W_k / enc W_v, computed on the first step (src/CrossAttention.cpp:388-413). */
    float* selfk = (float*)malloc(sizeof(float) * (size_t)L * steps * D);
    float* selfv = (float*)malloc(sizeof(float) * (size_t)L * steps * D);
    float* crossk = (float*)malloc(sizeof(float) * (size_t)L * S * D);
    float* crossv = (float*)malloc(sizeof(float) * (size_t)L * S * D);
    for (int l = 0; l < L; ++l) {
        orc_matmul(enc, m->dec[l].ck, crossk + (size_t)l * S * D, S, D, D);
        orc_matmul(enc, m->dec[l].cv, crossv + (size_t)l * S * D, S, D, D);
    }
    float *x = malloc(sizeof(float) * D), *nrm = malloc(sizeof(float) * D),
          *q = malloc(sizeof(float) * D), *a = malloc(sizeof(float) * D),
          *o = malloc(sizeof(float) * D), *h = malloc(sizeof(float) * F),
          *lg = malloc(sizeof(float) * V);
    int tok = bos;
    for (int s = 0; s < steps; ++s) {
        if (tok < 0 || tok >= V) {
            tok = -1;
            break;
        }
        /* src/Decoder.cpp:224-243: embedding + PE row of the absolute position (none past the
         * table) */
        for (int j = 0; j < D; ++j) {
            x[j] = m->dec_embed[(size_t)tok * D + j];
            if (s < m->max_seq) x[j] += m->pe[(size_t)s * D + j];
        }
        for (int l = 0; l < L; ++l) {
            const dec_layer* d = &m->dec[l];
            float* K = selfk + (size_t)l * steps * D;
            float* Vv = selfv + (size_t)l * steps * D;
            /* DecoderBlock::forward_with_cache (src/DecoderBlock.cpp:239-309) */
            orc_layernorm(x, d->ln1g, d->ln1b, nrm, 1, D);
            orc_matmul(nrm, d->sq, q, 1, D, D);
            orc_matmul(nrm, d->sk, K + (size_t)s * D, 1, D, D);
            orc_matmul(nrm, d->sv, Vv + (size_t)s * D, 1, D, D);
            orc_attention_single(q, K, Vv, s + 1, D, H, a);
            orc_matmul(a, d->so, o, 1, D, D);
            for (int j = 0; j < D; ++j) x[j] = x[j] + o[j];
            orc_layernorm(x, d->ln2g, d->ln2b, nrm, 1, D);
            orc_matmul(nrm, d->cq, q, 1, D, D);
            orc_attention_single(q, crossk + (size_t)l * S * D, crossv + (size_t)l * S * D, S, D,
                                 H, a);
            orc_matmul(a, d->co, o, 1, D, D);
            for (int j = 0; j < D; ++j) x[j] = x[j] + o[j];
            orc_layernorm(x, d->ln3g, d->ln3b, nrm, 1, D);
            ffn(nrm, 1, D, F, d->w1, d->b1, d->w2, d->b2, o, h);
            for (int j = 0; j < D; ++j) x[j] = x[j] + o[j];
        }
        orc_layernorm(x, m->dec_lnf_g, m->dec_lnf_b, nrm, 1, D);
        /* LanguageModelHead::forward (src/LanguageModelHead.cpp:49-69) */
        orc_matmul(nrm, m->head_w, lg, 1, D, V);
        for (int j = 0; j < V; ++j) lg[j] += m->head_b[j];
        out_ids[s] = orc_argmax(lg, V);
        if (logits) memcpy(logits + (size_t)s * V, lg, sizeof(float) * V);
        tok = forced ? forced[s] : out_ids[s];
    }
    free(enc); free(selfk); free(selfv); free(crossk); free(crossv);
    free(x); free(nrm); free(q); free(a); free(o); free(h); free(lg);
    return tok < 0 ? -1 : 0;
}

/* ------------------------------------------------------------------------------------------ */
/* Sampling: TextGenerator::generate (src/TextGenerator.cpp:519-565) and the filters it applies
 * (:26-137), with the generator's std::mt19937 and std::discrete_distribution as GCC's libstdc++
 * implements them (the reference is built with g++; TextGenerator.hpp:95).                      */

/* MT19937 (Matsumoto and Nishimura, 1998): the published initialisation and recurrence with the
 * std::mt19937 parameters. st[0..623] is the state, st[624] the read position. */
void orc_mt_seed(unsigned int* st, unsigned int seed) {
    st[0] = seed;
    for (unsigned int i = 1; i < 624; ++i) st[i] = 1812433253u * (st[i - 1] ^ (st[i - 1] >> 30)) + i;
    st[624] = 624;
}

static void mt_twist(unsigned int* mt) {
    for (int i = 0; i < 624; ++i) {
        const unsigned int y = (mt[i] & 0x80000000u) | (mt[(i + 1) % 624] & 0x7fffffffu);
        mt[i] = mt[(i + 397) % 624] ^ (y >> 1) ^ ((y & 1u) ? 0x9908b0dfu : 0u);
    }
}

unsigned int orc_mt_next(unsigned int* st) {
    if (st[624] >= 624) {
        mt_twist(st);
        st[624] = 0;
    }
    unsigned int y = st[st[624]++];
    y ^= y >> 11;
    y ^= (y << 7) & 0x9d2c5680u;
    y ^= (y << 15) & 0xefc60000u;
    y ^= y >> 18;
    return y;
}

/* std::generate_canonical<double, 53> over a 32-bit engine, as libstdc++ computes it: two draws
 * x0, x1; (x0 + x1 * 2^32) / 2^64 in double; a result that rounds to 1 becomes the largest double
 * below 1. */
double orc_canonical(unsigned int* st) {
    double s = (double)orc_mt_next(st);
    s += (double)orc_mt_next(st) * 4294967296.0;
    double r = s / 18446744073709551616.0;
    if (r >= 1.0) r = nextafter(1.0, 0.0);
    return r;
}

static double dmin(double a, double b) { return a < b ? a : b; }

/* Keeps the k largest values and sets the rest to -1e9f (apply_top_k, src/TextGenerator.cpp:41-63).
 * Values tied at the k-th place are kept lowest index first (std::partial_sort leaves that order
 * unspecified; *margin drops to 0 there). *margin also takes the gap between the k-th and the
 * (k+1)-th largest value, relative to the k-th. */
static void keep_top(float* x, int V, int k, double* margin) {
    int* ord = (int*)malloc(sizeof(int) * V);
    for (int j = 0; j < V; ++j) ord[j] = j;
    /* selection by descending value, ascending index among equals */
    for (int r = 0; r < k + 1 && r < V; ++r) {
        int best = r;
        for (int q = r + 1; q < V; ++q) {
            const int a = ord[q], b = ord[best];
            if (x[a] > x[b] || (x[a] == x[b] && a < b)) best = q;
        }
        const int t = ord[r]; ord[r] = ord[best]; ord[best] = t;
    }
    if (k < V) {
        const double vk = x[ord[k - 1]], vn = x[ord[k]];
        const double gap = (vk - vn) / (fabs(vk) > 1e-30 ? fabs(vk) : 1e-30);
        *margin = dmin(*margin, gap);
    }
    unsigned char* keep = (unsigned char*)calloc(V, 1);
    for (int r = 0; r < k; ++r) keep[ord[r]] = 1;
    for (int j = 0; j < V; ++j)
        if (!keep[j]) x[j] = -1e9f;
    free(keep);
    free(ord);
}

static const float* g_sort_key;
static int by_prob_desc(const void* pa, const void* pb) {
    const int a = *(const int*)pa, b = *(const int*)pb;
    if (g_sort_key[a] > g_sort_key[b]) return -1;
    if (g_sort_key[a] < g_sort_key[b]) return 1;
    return a < b ? -1 : (a > b);
}

/* apply_top_p (src/TextGenerator.cpp:66-101): softmax, tokens by descending probability, a float
 * running sum until it reaches p; the rest -1e9f. *margin takes the distance of the float64
 * running sum from p on both sides of the cut, and 0 when the float and float64 sums cut at
 * different places or when equal probabilities straddle the cut. */
static void keep_nucleus(float* x, int V, float p, double* margin) {
    float* pr = (float*)malloc(sizeof(float) * V);
    int* ord = (int*)malloc(sizeof(int) * V);
    orc_softmax_row(x, pr, V);
    for (int j = 0; j < V; ++j) ord[j] = j;
    g_sort_key = pr;
    qsort(ord, V, sizeof(int), by_prob_desc);
    float cum = 0.0f;
    double dcum = 0.0;
    int n_f = -1, n_d = -1;
    for (int r = 0; r < V; ++r) {
        const double prev = dcum;
        cum += pr[ord[r]];
        dcum += pr[ord[r]];
        if (n_f < 0 && cum >= p) n_f = r;
        if (n_d < 0 && dcum >= p) {
            n_d = r;
            *margin = dmin(*margin, dmin(dcum - p, p - prev));
        }
    }
    if (n_f != n_d) *margin = 0.0;
    const int last = n_f < 0 ? V - 1 : n_f;
    if (last + 1 < V && pr[ord[last]] == pr[ord[last + 1]]) *margin = 0.0;
    float* y = (float*)malloc(sizeof(float) * V);
    for (int j = 0; j < V; ++j) y[j] = -1e9f;
    for (int r = 0; r <= last; ++r) y[ord[r]] = x[ord[r]];
    memcpy(x, y, sizeof(float) * V);
    free(y);
    free(ord);
    free(pr);
}

int orc_sample_next(const float* logits, int V, const float* fcfg, const int* icfg,
                    const unsigned char* seen, int new_tokens, unsigned int* st, double* margin_out) {
    const float T = fcfg[0], top_p = fcfg[1], pen = fcfg[2];
    const int top_k = icfg[0], min_len = icfg[1], eos = icfg[2], pad = icfg[3];
    double margin = INFINITY;
    int any_finite = 0;
    for (int j = 0; j < V; ++j) {
        if (isnan(logits[j]) || logits[j] == INFINITY) return -1;  /* next_logits :186-190 */
        any_finite |= isfinite(logits[j]);
    }
    if (!any_finite) return -2;  /* :192-194 */
    float* x = (float*)malloc(sizeof(float) * V);
    memcpy(x, logits, sizeof(float) * V);
    if (new_tokens < min_len) {  /* :197-203 */
        if (eos >= 0 && eos < V) x[eos] = -INFINITY;
        if (pad >= 0 && pad < V) x[pad] = -INFINITY;
    }
    if (pen != 1.0f)  /* apply_repetition_penalty :115-136, once per distinct token */
        for (int j = 0; j < V; ++j)
            if (seen[j]) x[j] = x[j] > 0 ? x[j] / pen : x[j] * pen;
    if (T > 0.0f && T != 1.0f)  /* apply_temperature :26-38 */
        for (int j = 0; j < V; ++j) x[j] = x[j] / T;
    if (top_k > 0 && top_k < V) keep_top(x, V, top_k, &margin);
    if (top_p < 1.0f) {
        if (top_p <= 0.0f) keep_top(x, V, 1, &margin);
        else keep_nucleus(x, V, top_p, &margin);
    }
    int tok;
    if (T <= 0.0f) {  /* argmax (:151-153): first maximum */
        tok = orc_argmax(x, V);
        float second = -INFINITY;
        for (int j = 0; j < V; ++j)
            if (j != tok && x[j] > second) second = x[j];
        const double top = x[tok];
        margin = dmin(margin, (top - second) / (fabs(top) > 1e-30 ? fabs(top) : 1e-30));
    } else {  /* sample_token (:145-148): std::discrete_distribution over softmax(x) */
        float* pr = (float*)malloc(sizeof(float) * V);
        double* cp = (double*)malloc(sizeof(double) * V);
        orc_softmax_row(x, pr, V);
        double sum = 0.0;
        for (int j = 0; j < V; ++j) sum += (double)pr[j];
        double acc = 0.0;
        for (int j = 0; j < V; ++j) {
            acc += (double)pr[j] / sum;
            cp[j] = acc;
        }
        cp[V - 1] = 1.0;
        const double u = orc_canonical(st);
        int lo = 0, hi = V;  /* lower_bound: first cp >= u */
        while (lo < hi) {
            const int mid = (lo + hi) / 2;
            if (cp[mid] < u) lo = mid + 1;
            else hi = mid;
        }
        tok = lo;
        const double below = tok > 0 ? cp[tok - 1] : 0.0;
        margin = dmin(margin, dmin(u - below, cp[tok] - u));
        free(cp);
        free(pr);
    }
    free(x);
    if (margin_out) *margin_out = margin;
    return tok;
}

int orc_sample_generate(const float* logits, int V, int steps, const float* fcfg, const int* icfg,
                        unsigned int seed, const int* prompt, int n_prompt, int* out, double* margins) {
    const int bos = icfg[4], eos = icfg[2], pad = icfg[3];
    unsigned int st[625];
    orc_mt_seed(st, seed);
    unsigned char* seen = (unsigned char*)calloc(V, 1);
    int n = 0;
    if (n_prompt > 0) {
        for (int i = 0; i < n_prompt; ++i) out[n++] = prompt[i];
    } else {
        out[n++] = bos;
    }
    for (int i = 0; i < n; ++i)
        if (out[i] >= 0 && out[i] < V) seen[out[i]] = 1;
    for (int s = 0; s < steps; ++s) {
        double m = 0.0;
        const int tok = orc_sample_next(logits + (size_t)s * V, V, fcfg, icfg, seen, s, st, &m);
        if (tok < 0) {
            free(seen);
            return tok;
        }
        if (margins) margins[s] = m;
        out[n++] = tok;
        seen[tok] = 1;
        if (tok == eos || tok == pad) break;  /* is_stop_token, src/SpecialTokens.hpp:162-164 */
    }
    free(seen);
    return n;
}
