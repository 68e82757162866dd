// checkpoint.h — reading the reference's SafeTensors checkpoints (host side, no device work).
//
// A checkpoint directory holds config.json (model shape) and model.safetensors (an 8-byte
// little-endian header length, a JSON header naming each tensor's dtype, shape and byte range,
// then the raw data), as the reference's ModelSerializer::export_safetensors writes them
// (src/ModelSerializer.cpp:243-395; container layout :111-160).
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

// Model shape from <dir>/config.json (keys vocab_size, d_model, d_ff, num_heads, num_layers,
// num_decoder_layers, max_length). Throws std::invalid_argument on a missing or malformed key,
// CheckpointIoError if the file cannot be read.
adai_b200_model_desc read_checkpoint_config(const std::string& dir);

// Element counts of the tensors of adai_b200_model_upload, in its order.
std::vector<size_t> upload_tensor_sizes(const adai_b200_model_desc& d);

// Reads <dir>/model.safetensors into `out` (one host buffer per upload tensor, sized as
// upload_tensor_sizes), converting the checkpoint's [out, in] projection matrices to the
// reference's in-memory W[in, out]. The decoder embedding falls back to model.shared.weight and
// the final LayerNorms to gamma 1 / beta 0 when the file has none, as the reference's import
// does (src/ModelSerializer.cpp:474-487, :518-525, :565-572); tensors it does not use are
// ignored. Throws std::invalid_argument naming the tensor for a missing tensor, a wrong shape or a
// dtype other than F32, and CheckpointIoError for I/O errors.
void read_checkpoint_tensors(const std::string& dir, const adai_b200_model_desc& d,
                             const std::vector<float*>& out);

}  // namespace adai_b200
