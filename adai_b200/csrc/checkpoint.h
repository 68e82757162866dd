// checkpoint.h — reading the reference's checkpoints (host side, no device work).
//
// Two formats, told apart by what exists at `path`:
// * a SafeTensors directory: path/config.json (model shape) and path/model.safetensors (an 8-byte
//   little-endian header length, a JSON header naming each tensor's dtype, shape and byte range,
//   then the raw data), as ModelSerializer::export_safetensors writes them
//   (src/ModelSerializer.cpp:243-395; container layout :111-160);
// * the reference's own save_model(path) files: path.config, path.encoder, path.decoder,
//   path.lm_head and the per-component files beside them (src/EncoderDecoderModel.cpp:960-985),
//   in the adai::binio layout (src/BinaryIO.cpp).
#pragma once

#include <cstddef>
#include <stdexcept>
#include <string>
#include <vector>

#include "../../include/adai_b200.h"

namespace adai_b200 {

// A checkpoint file that cannot be opened or read (as opposed to one whose content is invalid,
// which is std::invalid_argument).
struct CheckpointIoError : std::runtime_error {
    using std::runtime_error::runtime_error;
};

// Model shape: from path/config.json (keys vocab_size, d_model, d_ff, num_heads, num_layers,
// num_decoder_layers, max_length), or from path.config (format marker, version >= 2, then
// vocab, d_model, encoder and decoder layers, heads, d_ff, max length, BOS, EOS, PAD). Throws
// std::invalid_argument on malformed content, CheckpointIoError if nothing can be read.
adai_b200_model_desc read_checkpoint_config(const std::string& path);

// The checkpoint's BOS / EOS / PAD ids (config.json's decoder_start_token_id, eos_token_id,
// pad_token_id; path.config's last three fields).
void read_checkpoint_special_tokens(const std::string& path, int* bos, int* eos, int* pad);

// Element counts of the tensors of adai_b200_model_upload, in its order.
std::vector<size_t> upload_tensor_sizes(const adai_b200_model_desc& d);

// Reads the tensors into `out` (one host buffer per upload tensor, sized as
// upload_tensor_sizes).
// SafeTensors: the checkpoint's [out, in] projection matrices become the reference's in-memory
// W[in, out]. The decoder embedding falls back to model.shared.weight and the final LayerNorms to
// gamma 1 / beta 0 when the file has none, as the reference's import does
// (src/ModelSerializer.cpp:474-487, :518-525, :565-572); tensors it does not use are ignored.
// save_model files: each file is checked as the reference's loader checks it (every dimension,
// no trailing bytes); the encoder's embedding and final norm fall back to the shared
// path_token_emb.bin / path_final_norm.bin of checkpoints written before the encoder-specific
// names (src/LLMEncoder.cpp:326-349). Final LayerNorms must carry epsilon 1e-5, and decoder
// blocks with a gated world-model or hippocampal path are refused (the decode step has neither).
// Throws std::invalid_argument for invalid content (naming the tensor or file) and
// CheckpointIoError for missing, unreadable or truncated files.
void read_checkpoint_tensors(const std::string& path, const adai_b200_model_desc& d,
                             const std::vector<float*>& out);

}  // namespace adai_b200
