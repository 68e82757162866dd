// adai_b200_reference.hpp — the reference-side half of the binding: compiled inside the
// kerfbit/adai build (its src/ folder on the include path), it walks a model's components through
// their public getters and hands the weights to adai_b200_model_upload in the order that call
// documents, which is the order of the reference's own setters.
//
//   std::vector<std::vector<float>> keep;
//   auto tensors = adai_b200::tensors_in_upload_order(model, keep);   // EncoderDecoderModel&
//   ctx.upload(adai_b200::model_desc(model), tensors);                 // adai_b200::Context
//
// The component overload (LLMEncoder, LLMDecoder, LanguageModelHead) serves hosts that hold the
// three pieces directly, as benchmarks/GpuDecodeBenchmark.cpp does. The EncoderDecoderModel
// overloads are compiled when ADAI_B200_ENCODER_DECODER_MODEL is defined (they include
// EncoderDecoderModel.hpp and so need the rest of the reference's headers on the include path).
#ifndef ADAI_B200_REFERENCE_HPP
#define ADAI_B200_REFERENCE_HPP

#include <vector>

#include "Decoder.hpp"            // LLMDecoder, DecoderBlock (src/Decoder.hpp:125, :328-337)
#include "LanguageModelHead.hpp"  // get_W_output / get_bias (src/LanguageModelHead.hpp:154-158)
#include "adai_b200.h"
#include "encoder.hpp"            // LLMEncoder, EncoderBlock (src/encoder.hpp:90, :258-270)

namespace adai_b200 {

// Copies a reference Matrix (one heap vector per row, src/Matrix.hpp:32) into one row-major
// buffer owned by `keep`; returns its data pointer.
inline const float* flat_copy(const Matrix& m, std::vector<std::vector<float>>& keep) {
    std::vector<float> v;
    v.reserve(static_cast<size_t>(m.rows) * static_cast<size_t>(m.cols));
    for (int i = 0; i < m.rows; ++i) v.insert(v.end(), m.data[i].begin(), m.data[i].end());
    keep.push_back(std::move(v));
    return keep.back().data();
}

// The host tensors of adai_b200_model_upload, in its order: encoder embedding; per encoder layer
// LN1 gamma/beta, Wq Wk Wv Wo, LN2 gamma/beta, W1 b1 W2 b2; encoder final LN; decoder embedding;
// per decoder layer LN1, self-attention Wq Wk Wv Wo, LN2, cross-attention Wq Wk Wv Wo, LN3,
// W1 b1 W2 b2; decoder final LN; head W_output and bias. `keep` owns the copies (reserve is
// called so that the returned pointers stay valid).
inline std::vector<const float*> tensors_in_upload_order(LLMEncoder& enc, LLMDecoder& dec,
                                                         LanguageModelHead& head,
                                                         std::vector<std::vector<float>>& keep) {
    const int le = enc.get_num_layers(), ld = dec.get_num_layers();
    keep.clear();
    keep.reserve(static_cast<size_t>(1 + 12 * le + 2 + 1 + 18 * ld + 4));
    std::vector<const float*> t;
    auto add = [&](const Matrix& m) { t.push_back(flat_copy(m, keep)); };
    auto add_ln = [&](LayerNorm* n) {
        add(n->get_gamma());
        add(n->get_beta());
    };
    auto add_ffn = [&](FeedForward* f) {
        add(f->get_W1());
        add(f->get_b1());
        add(f->get_W2());
        add(f->get_b2());
    };
    add(enc.get_token_embedding()->get_embeddings());
    for (int i = 0; i < le; ++i) {
        EncoderBlock* b = enc.get_encoder_block(i);
        add_ln(b->get_norm1());
        MultiHeadAttention* a = b->get_self_attention();
        add(a->get_Wq());
        add(a->get_Wk());
        add(a->get_Wv());
        add(a->get_Wo());
        add_ln(b->get_norm2());
        add_ffn(b->get_feed_forward());
    }
    add_ln(enc.get_final_norm());
    add(dec.get_token_embedding()->get_embeddings());
    for (int i = 0; i < ld; ++i) {
        DecoderBlock* b = dec.get_decoder_block(i);
        add_ln(b->get_norm1());
        MultiHeadAttention* sa = b->get_self_attention();
        add(sa->get_Wq());
        add(sa->get_Wk());
        add(sa->get_Wv());
        add(sa->get_Wo());
        add_ln(b->get_norm2());
        CrossAttention* ca = b->get_cross_attention();
        add(ca->get_Wq());
        add(ca->get_Wk());
        add(ca->get_Wv());
        add(ca->get_Wo());
        add_ln(b->get_norm3());
        add_ffn(b->get_feed_forward());
    }
    add_ln(dec.get_final_norm());
    add(head.get_W_output());
    add(head.get_bias());
    return t;
}

#ifdef ADAI_B200_ENCODER_DECODER_MODEL
}  // namespace adai_b200
#include "EncoderDecoderModel.hpp"
namespace adai_b200 {

// EncoderDecoderModel's shape getters (src/EncoderDecoderModel.hpp:690-721).
inline adai_b200_model_desc model_desc(const EncoderDecoderModel& m) {
    adai_b200_model_desc d{};
    d.vocab = m.get_vocab_size();
    d.d_model = m.get_d_model();
    d.n_heads = m.get_num_heads();
    d.d_ff = m.get_d_ff();
    d.enc_layers = m.get_encoder_layers();
    d.dec_layers = m.get_decoder_layers();
    d.max_seq = m.get_max_seq_length();
    return d;
}

// The model's components (get_encoder / get_decoder / get_lm_head, src/EncoderDecoderModel.hpp:
// 728-736) in upload order.
inline std::vector<const float*> tensors_in_upload_order(EncoderDecoderModel& m,
                                                         std::vector<std::vector<float>>& keep) {
    return tensors_in_upload_order(*m.get_encoder(), *m.get_decoder(), *m.get_lm_head(), keep);
}
#endif

}  // namespace adai_b200

#endif  // ADAI_B200_REFERENCE_HPP
