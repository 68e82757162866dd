"""Seeded synthetic weights and inputs for the encoder-decoder decode path.

The tensor order and shapes are the model-upload order of the C-ABI (adai_b200_model_upload in
include/adai_b200.h), which is also the order the reference's public setters are called in
(MultiHeadAttention::set_W*, CrossAttention::set_W*, FeedForward::set_W1/b1/W2/b2,
LayerNorm::set_gamma/set_beta, TokenEmbedding::set_embeddings, LanguageModelHead::set_W_output /
set_bias). Two weight schemes, each drawn from one numpy PCG64 stream in that order:

* "xavier": every matrix Xavier-uniform U(+-sqrt(6/(fan_in+fan_out))), the embedding tables
  included (the benchmark workloads' weights).
* "reference": the distributions of the reference's own constructors, which make a sequence's
  greedy tokens depend on its source: token embeddings N(0, 1) (TokenEmbedding::kInitStd,
  src/TokenEmbedding.cpp:15-24), attention projections N(0, 2/d_model)
  (src/MultiHeadAttention.cpp:66-72, src/CrossAttention.cpp:84-90), W1 N(0, 2/d_model) and
  W2 N(0, 2/d_ff) (src/FeedForward.cpp:28-50), the head N(0, 2/(d_model + vocab))
  (src/LanguageModelHead.cpp:30-32). Under "xavier" the embedding rows are far smaller than the
  positional rows, so every source gives nearly the same greedy stream.

LayerNorm gamma = 1, beta = 0 and biases = 0 unless `affine` asks for random ones (parity tests
use random ones so every bias and affine path is exercised).
"""
from __future__ import annotations

import numpy as np

from .config import ModelConfig


def tensor_specs(cfg: ModelConfig) -> list[tuple[str, tuple[int, ...]]]:
    """(name, shape) of every tensor in upload order."""
    V, D, F = cfg.vocab, cfg.d_model, cfg.d_ff
    out: list[tuple[str, tuple[int, ...]]] = [("enc.embed", (V, D))]
    for i in range(cfg.enc_layers):
        p = f"enc.{i}."
        out += [(p + "ln1.g", (D,)), (p + "ln1.b", (D,)),
                (p + "attn.wq", (D, D)), (p + "attn.wk", (D, D)), (p + "attn.wv", (D, D)),
                (p + "attn.wo", (D, D)),
                (p + "ln2.g", (D,)), (p + "ln2.b", (D,)),
                (p + "ffn.w1", (D, F)), (p + "ffn.b1", (F,)), (p + "ffn.w2", (F, D)),
                (p + "ffn.b2", (D,))]
    out += [("enc.lnf.g", (D,)), ("enc.lnf.b", (D,)), ("dec.embed", (V, D))]
    for i in range(cfg.dec_layers):
        p = f"dec.{i}."
        out += [(p + "ln1.g", (D,)), (p + "ln1.b", (D,)),
                (p + "sa.wq", (D, D)), (p + "sa.wk", (D, D)), (p + "sa.wv", (D, D)),
                (p + "sa.wo", (D, D)),
                (p + "ln2.g", (D,)), (p + "ln2.b", (D,)),
                (p + "ca.wq", (D, D)), (p + "ca.wk", (D, D)), (p + "ca.wv", (D, D)),
                (p + "ca.wo", (D, D)),
                (p + "ln3.g", (D,)), (p + "ln3.b", (D,)),
                (p + "ffn.w1", (D, F)), (p + "ffn.b1", (F,)), (p + "ffn.w2", (F, D)),
                (p + "ffn.b2", (D,))]
    out += [("dec.lnf.g", (D,)), ("dec.lnf.b", (D,)), ("head.w", (D, V)), ("head.b", (V,))]
    return out


def _reference_std(cfg: ModelConfig, name: str) -> float:
    D, F, V = cfg.d_model, cfg.d_ff, cfg.vocab
    if name.endswith("embed"):
        return 1.0
    if name == "head.w":
        return float(np.sqrt(2.0 / (D + V)))
    if name.endswith("ffn.w2"):
        return float(np.sqrt(2.0 / F))
    return float(np.sqrt(2.0 / D))


def make_weights(cfg: ModelConfig, seed: int = 0, affine: bool = False,
                 scheme: str = "xavier") -> list[np.ndarray]:
    """Weights in upload order, C-contiguous float32 (scheme "xavier" or "reference")."""
    if scheme not in ("xavier", "reference"):
        raise ValueError(f"unknown weight scheme {scheme!r}")
    rng = np.random.default_rng(seed)
    out = []
    for name, shape in tensor_specs(cfg):
        if len(shape) == 2 and scheme == "reference":
            w = rng.standard_normal(shape, dtype=np.float32)
            w *= np.float32(_reference_std(cfg, name))
        elif len(shape) == 2:
            bound = np.float32(np.sqrt(6.0 / (shape[0] + shape[1])))
            w = rng.random(shape, dtype=np.float32)
            w *= np.float32(2.0) * bound
            w -= bound
        elif name.endswith(".g"):
            w = (rng.uniform(0.5, 1.5, shape).astype(np.float32) if affine
                 else np.ones(shape, np.float32))
        else:
            w = (rng.uniform(-0.1, 0.1, shape).astype(np.float32) if affine
                 else np.zeros(shape, np.float32))
        out.append(np.ascontiguousarray(w))
    return out


def make_sources(cfg: ModelConfig, batch: int, src_len: tuple[int, int], seed: int = 0
                 ) -> list[np.ndarray]:
    """Per-sequence source token ids, uniform in [4, vocab) (ids 0-3 are PAD/UNK/BOS/EOS,
    src/SpecialTokens.hpp:55-61); lengths uniform in [lo, hi]."""
    rng = np.random.default_rng(seed + 1)
    lo, hi = src_len
    lens = rng.integers(lo, hi + 1, size=batch) if hi > lo else np.full(batch, lo)
    return [rng.integers(4, cfg.vocab, size=int(n)).astype(np.int32) for n in lens]


def weights_digest(weights: list[np.ndarray]) -> str:
    """Short digest of a weight set, stored beside fixtures so generator drift is caught."""
    import hashlib
    h = hashlib.sha256()
    for w in weights:
        h.update(np.ascontiguousarray(w).view(np.uint8).tobytes()[:4096])
        h.update(np.float64(w.astype(np.float64).sum()).tobytes())
    return h.hexdigest()[:16]
