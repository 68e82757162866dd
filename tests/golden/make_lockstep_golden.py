"""Generates tests/golden/large_lockstep.npz: a full-length greedy decode of the large
encoder-decoder by the reference's own CPU implementation.

The large model (d_model 1024, 16 heads, 12+12 layers, d_ff 4096, vocab 32000) with weights
drawn like the reference's constructors draw them (adai_b200.synth, scheme "reference", random
LayerNorm affine parameters and biases) decodes 8 sources whose lengths span the serving
workload's range 128-1024 (one of exactly 1024) for 256 greedy steps, through oracle/_ref
(the reference sources built by `make -C oracle ref`; encoder once, LLMDecoder::forward_with_cache
per token, LanguageModelHead::forward, first maximum, no stop tokens).

Stored per sequence and step: the greedy id, the decoder's output row (after its final LayerNorm),
the float64 sequential sum of the logits row and its two largest logits. The logits themselves
(8 x 256 x 32000 floats) are not stored: the tests rebuild them as hidden * W_output + bias with
the oracle's in-order product, which is bit-identical to the reference's Matrix::operator*
(tests/test_oracle.py), and check every rebuilt row against the stored sum and top two.
The weights and sources are regenerated from their seeds by the tests.

    python tests/golden/make_lockstep_golden.py      # about 15 minutes on 8 host cores

The eight sequences run in parallel worker processes, one OpenMP thread each.
"""
from __future__ import annotations

import multiprocessing as mp
import os
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

OUT = os.path.join(os.path.dirname(os.path.abspath(__file__)), "large_lockstep.npz")

LARGE_SEED = 4
LARGE_SRC_LENS = (1024, 128, 896, 256, 640, 384, 768, 512)
LARGE_STEPS = 256


def large_inputs():
    """(weights, sources) of the large lockstep case."""
    from adai_b200.config import LARGE
    from adai_b200.synth import make_weights
    w = make_weights(LARGE, LARGE_SEED, affine=True, scheme="reference")
    rng = np.random.default_rng(LARGE_SEED + 100)
    srcs = [rng.integers(4, LARGE.vocab, size=n).astype(np.int32) for n in LARGE_SRC_LENS]
    return w, srcs


def _worker(i):
    os.environ["OMP_NUM_THREADS"] = "1"
    from adai_b200.config import LARGE
    from oracle.pyoracle import Ref
    w, srcs = large_inputs()
    m = Ref().model(LARGE, w)
    t0 = time.time()
    ids, hid, sums, top2 = m.generate_hidden(srcs[i], LARGE_STEPS)
    return i, ids, hid, sums, top2, time.time() - t0


def main():
    from adai_b200.synth import weights_digest
    w, srcs = large_inputs()
    n = len(srcs)
    res = [None] * n
    os.environ["OMP_NUM_THREADS"] = "1"  # inherited by the spawned workers
    ctx = mp.get_context("spawn")
    with ctx.Pool(min(n, os.cpu_count() or 1)) as pool:
        for i, ids, hid, sums, top2, dt in pool.imap_unordered(_worker, range(n)):
            res[i] = (ids, hid, sums, top2)
            print(f"sequence {i}: source {len(srcs[i])}, {dt:.0f} s, ids {ids[:8].tolist()}",
                  flush=True)
    np.savez_compressed(
        OUT,
        ids=np.stack([r[0] for r in res]),
        hidden=np.stack([r[1] for r in res]),
        logit_sum=np.stack([r[2] for r in res]),
        top2=np.stack([r[3] for r in res]),
        src_lens=np.array(LARGE_SRC_LENS, np.int32),
        weights_digest=np.array(weights_digest(w)),
    )
    print("wrote", OUT, os.path.getsize(OUT), "bytes")


if __name__ == "__main__":
    main()
