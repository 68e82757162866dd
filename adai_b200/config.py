"""Model and workload shapes of the encoder-decoder decode path.

ModelConfig mirrors the constructor arguments of the reference model
(LLMEncoder(vocab, d_model, layers, heads, d_ff, max_seq), src/encoder.hpp:90;
LLMDecoder(vocab, d_model, layers, heads, d_ff, max_seq, 0), src/Decoder.hpp:125;
LanguageModelHead(d_model, vocab)). The named workloads below are the five synthetic
workloads this library is measured and parity-tested on.
"""
from __future__ import annotations

from dataclasses import dataclass, field


@dataclass(frozen=True)
class ModelConfig:
    vocab: int
    d_model: int
    n_heads: int
    d_ff: int
    enc_layers: int
    dec_layers: int
    max_seq: int

    def __post_init__(self):
        if self.d_model % self.n_heads:
            raise ValueError("d_model must be a multiple of n_heads")

    @property
    def head_dim(self) -> int:
        return self.d_model // self.n_heads

    def as_cfg(self) -> list[int]:
        """The 7-int config array of the C-ABI (adai_b200_model_desc order)."""
        return [self.vocab, self.d_model, self.n_heads, self.d_ff, self.enc_layers,
                self.dec_layers, self.max_seq]

    # ---- algorithmic work per decoded token (GEMM FLOPs) and per step (weight bytes) ----
    def decode_gemm_flops_per_token(self) -> int:
        D, F, V, L = self.d_model, self.d_ff, self.vocab, self.dec_layers
        # per layer: Wq Wk Wv Wo (self) + Wq Wo (cross) = 6 D^2, FFN 2 D F; head D V
        return 2 * (L * (6 * D * D + 2 * D * F) + D * V)

    def decoder_weight_bytes(self) -> int:
        D, F, V, L = self.d_model, self.d_ff, self.vocab, self.dec_layers
        return 4 * (L * (6 * D * D + 2 * D * F) + D * V)


@dataclass(frozen=True)
class Workload:
    name: str
    model: ModelConfig
    batch: int                 # sequences decoded together (per GPU for the serving workload)
    src_len: tuple[int, int]   # source length range [lo, hi] (lo == hi: fixed)
    steps: int                 # greedy decode steps
    notes: str = ""
    extra: dict = field(default_factory=dict)


TINY = ModelConfig(vocab=4096, d_model=128, n_heads=4, d_ff=512, enc_layers=2, dec_layers=2,
                   max_seq=128)
MID = ModelConfig(vocab=16000, d_model=512, n_heads=8, d_ff=2048, enc_layers=6, dec_layers=6,
                  max_seq=512)
LARGE = ModelConfig(vocab=32000, d_model=1024, n_heads=16, d_ff=4096, enc_layers=12,
                    dec_layers=12, max_seq=1024)

WORKLOADS = {
    "tiny-encdec-b8-s64-t32": Workload("tiny-encdec-b8-s64-t32", TINY, 8, (64, 64), 32),
    "mid-encdec-b64-s256-t128": Workload("mid-encdec-b64-s256-t128", MID, 64, (256, 256), 128),
    "large-encdec-b128-s128to1024-t256": Workload(
        "large-encdec-b128-s128to1024-t256", LARGE, 128, (128, 1024), 256,
        notes="128 sequences per GPU; batch 1024 over 8 GPUs"),
    # the same 1024 sequences (same seed) on one GPU: the strong-scaling reference point
    "large-encdec-b1024-s128to1024-t256": Workload(
        "large-encdec-b1024-s128to1024-t256", LARGE, 1024, (128, 1024), 256,
        notes="1024 sequences per GPU (about 130 GB of KV caches)"),
}

# Stacked-GEMM sweep shapes (M rows x K -> N) and the KV-attention op workload.
GEMM_SWEEP_M = (64, 256, 1024, 4096)
GEMM_SWEEP_KN = ((512, 1536), (512, 2048), (2048, 512), (512, 16000))
ATTN_OP = dict(batch=256, heads=16, head_dim=64, capacity=2048, len_lo=256, len_hi=2048, steps=64)
