"""Writing SafeTensors checkpoints in the reference's layout, so that weights held in Python (the
seeded synthetic models, or weights converted from elsewhere) can be loaded the way a reference
checkpoint is (`Context.load`, `adai_b200_model_load`).

The layout is the one ModelSerializer::export_safetensors writes (src/ModelSerializer.cpp:243-391).
config.json carries the T5-style shape keys, and model.safetensors the tensors under T5-style
names. Projection matrices are stored [out, in], transposed from the reference's right-multiplied
W[in, out]. Vectors and embedding tables are stored as they are, all as F32. The container is an
8-byte little-endian header length, a JSON header padded with spaces to a multiple of 8 bytes, then
the data in header order (:111-160).
"""
from __future__ import annotations

import json
import os
import struct

import numpy as np

from .config import ModelConfig
from .synth import tensor_specs


def checkpoint_names(cfg: ModelConfig) -> list[tuple[str, bool]]:
    """(checkpoint name, stored transposed) of every upload tensor, in upload order."""
    names: list[tuple[str, bool]] = [("model.shared.weight", False)]
    for i in range(cfg.enc_layers):
        b = f"model.encoder.block.{i}"
        names += [(f"{b}.layer.0.layer_norm.weight", False), (f"{b}.layer.0.layer_norm.bias", False)]
        names += [(f"{b}.layer.0.SelfAttention.{p}.weight", True) for p in "qkvo"]
        names += [(f"{b}.layer.1.layer_norm.weight", False), (f"{b}.layer.1.layer_norm.bias", False),
                  (f"{b}.layer.1.DenseReluDense.wi.weight", True),
                  (f"{b}.layer.1.DenseReluDense.wi.bias", False),
                  (f"{b}.layer.1.DenseReluDense.wo.weight", True),
                  (f"{b}.layer.1.DenseReluDense.wo.bias", False)]
    names += [("model.encoder.final_layer_norm.weight", False),
              ("model.encoder.final_layer_norm.bias", False),
              ("model.decoder.embed_tokens.weight", False)]
    for i in range(cfg.dec_layers):
        b = f"model.decoder.block.{i}"
        names += [(f"{b}.layer.0.layer_norm.weight", False), (f"{b}.layer.0.layer_norm.bias", False)]
        names += [(f"{b}.layer.0.SelfAttention.{p}.weight", True) for p in "qkvo"]
        names += [(f"{b}.layer.1.layer_norm.weight", False), (f"{b}.layer.1.layer_norm.bias", False)]
        names += [(f"{b}.layer.1.EncDecAttention.{p}.weight", True) for p in "qkvo"]
        names += [(f"{b}.layer.2.layer_norm.weight", False), (f"{b}.layer.2.layer_norm.bias", False),
                  (f"{b}.layer.2.DenseReluDense.wi.weight", True),
                  (f"{b}.layer.2.DenseReluDense.wi.bias", False),
                  (f"{b}.layer.2.DenseReluDense.wo.weight", True),
                  (f"{b}.layer.2.DenseReluDense.wo.bias", False)]
    names += [("model.decoder.final_layer_norm.weight", False),
              ("model.decoder.final_layer_norm.bias", False),
              ("lm_head.weight", True), ("lm_head.bias", False)]
    return names


def write_safetensors(path: str, tensors: list[tuple[str, np.ndarray]],
                      metadata: dict[str, str] | None = None) -> None:
    """A SafeTensors file of F32 tensors, in the given order."""
    header: dict = {"__metadata__": dict(metadata or {})}
    off = 0
    for name, a in tensors:
        n = int(a.size) * 4
        header[name] = {"dtype": "F32", "shape": [int(s) for s in a.shape],
                        "data_offsets": [off, off + n]}
        off += n
    h = json.dumps(header, separators=(",", ":")).encode()
    h += b" " * (-len(h) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)))
        f.write(h)
        for _, a in tensors:
            f.write(np.ascontiguousarray(a, dtype="<f4").tobytes())


def write_checkpoint(directory: str, cfg: ModelConfig, weights: list[np.ndarray], bos: int = 2,
                     eos: int = 3, pad: int = 0) -> None:
    """Writes `weights` (upload order, the reference's in-memory layouts) as
    <directory>/model.safetensors + <directory>/config.json."""
    specs = tensor_specs(cfg)
    if len(weights) != len(specs):
        raise ValueError(f"model needs {len(specs)} tensors, got {len(weights)}")
    tensors = []
    for (name, transposed), (_, shape), w in zip(checkpoint_names(cfg), specs, weights):
        w = np.asarray(w, np.float32)
        if w.shape != shape:
            raise ValueError(f"{name}: shape {w.shape}, expected {shape}")
        tensors.append((name, w.T if transposed else w))
    os.makedirs(directory, exist_ok=True)
    write_safetensors(os.path.join(directory, "model.safetensors"), tensors,
                      {"format": "pt", "adai_version": "1.0", "model_type": "t5"})
    config = {
        "architectures": ["T5ForConditionalGeneration"], "model_type": "t5", "adai_native": True,
        "vocab_size": cfg.vocab, "d_model": cfg.d_model, "d_ff": cfg.d_ff,
        "d_kv": cfg.d_model // cfg.n_heads, "num_heads": cfg.n_heads,
        "num_layers": cfg.enc_layers, "num_decoder_layers": cfg.dec_layers,
        "max_length": cfg.max_seq, "decoder_start_token_id": bos, "eos_token_id": eos,
        "pad_token_id": pad, "feed_forward_proj": "gelu", "torch_dtype": "float32",
    }
    with open(os.path.join(directory, "config.json"), "w") as f:
        json.dump(config, f, indent=2)
        f.write("\n")
