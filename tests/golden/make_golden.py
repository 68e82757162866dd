"""Generates tests/golden/reference_outputs.npz from the reference's own CPU implementation.

Runs the reference build (oracle/_ref/libadai_ref.so, made by `make -C oracle ref` from the
reference sources) on seeded inputs and stores its outputs. The inputs are regenerated from the
seeds by the tests, so only outputs (and digests of the inputs) are committed.

    python tests/golden/make_golden.py

Known-answer cases restated from the reference's tests (kerfbit/adai):
  * GEMM shapes of tests/matrix_simd_test.cpp:290-319 (tiled GEMM vs scalar, tol 1e-5 + 1e-5 sum|ab|)
  * softmax rows of tests/matrixgpu_td003_test.cpp:234-249 ([0,0] -> [.5,.5], [0,ln 3] -> [.25,.75])
  * GELU (tests/matrixgpu_td003_test.cpp:448), LayerNorm, the positional table
    (tests/positionalencoding_test.cpp:437), per-head cached attention
    (tests/multiheadattention_test.cpp:363), argmax lowest index on ties
    (tests/matrixgpu_td003_test.cpp:478)
  * a cached greedy decode of the tiny encoder-decoder (the lockstep check of
    benchmarks/GpuDecodeBenchmark.cpp:347-375)
"""
from __future__ import annotations

import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

from adai_b200.config import TINY  # noqa: E402
from adai_b200.synth import make_sources, make_weights, weights_digest  # noqa: E402
from oracle.pyoracle import Ref  # noqa: E402

OUT = os.path.join(os.path.dirname(os.path.abspath(__file__)), "reference_outputs.npz")

GEMM_SHAPES = [(1, 512, 2000), (8, 512, 700), (3, 1000, 300), (64, 512, 513), (17, 300, 257),
               (2, 100, 100)]
DECODE_SEQS, DECODE_SRC, DECODE_STEPS, DECODE_LOGIT_STEPS = 3, 16, 12, 4


def gemm_inputs(i, M, K, N):
    rng = np.random.default_rng(1000 + i)
    return (rng.standard_normal((M, K)).astype(np.float32),
            rng.standard_normal((K, N)).astype(np.float32))


def small_inputs():
    rng = np.random.default_rng(7)
    return dict(
        ln_x=rng.standard_normal((4, 128)).astype(np.float32) * 3 + 1,
        ln_g=rng.uniform(0.5, 1.5, 128).astype(np.float32),
        ln_b=rng.uniform(-0.1, 0.1, 128).astype(np.float32),
        gelu_x=np.linspace(-6, 6, 97).astype(np.float32),
        att_q=rng.standard_normal(128).astype(np.float32),
        att_k=rng.standard_normal((40, 128)).astype(np.float32),
        att_v=rng.standard_normal((40, 128)).astype(np.float32),
    )


def main():
    ref = Ref()
    out = {"matmul_kernel": np.array(ref.matmul_kernel())}
    for i, (M, K, N) in enumerate(GEMM_SHAPES):
        A, B = gemm_inputs(i, M, K, N)
        out[f"gemm_{i}"] = ref.matmul(A, B)
    s = small_inputs()
    out["ln"] = ref.layernorm(s["ln_x"], s["ln_g"], s["ln_b"])
    out["gelu"] = ref.gelu(s["gelu_x"])
    out["softmax_kat"] = ref.softmax_rows(np.array([[0, 0], [0, np.log(3.0)]], np.float32))
    out["pe_64x128"] = ref.pe_table(64, 128)
    out["attn"] = ref.attention_single(s["att_q"], s["att_k"], s["att_v"], 4)

    w = make_weights(TINY, seed=0, affine=True)
    out["tiny_weights_digest"] = np.array(weights_digest(w))
    srcs = make_sources(TINY, DECODE_SEQS, (DECODE_SRC, DECODE_SRC), seed=0)
    model = ref.model(TINY, w)
    ids, logits = [], []
    for src in srcs:
        i_, l_ = model.generate(src, DECODE_STEPS, want_logits=True)
        ids.append(i_)
        logits.append(l_[:DECODE_LOGIT_STEPS])
    out["tiny_ids"] = np.stack(ids)
    out["tiny_logits"] = np.stack(logits)
    out["tiny_enc0"] = model.encode(srcs[0])
    np.savez_compressed(OUT, **out)
    print("wrote", OUT, os.path.getsize(OUT), "bytes")


if __name__ == "__main__":
    main()
