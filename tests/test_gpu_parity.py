"""Full-length greedy parity of the batched decode step against the reference build.

The reference (oracle/_ref: its own sources, built by oracle/Makefile) decodes each sequence on
the CPU; the device decodes them stacked in one batch, in lockstep (tests/lockstep.py). Weights
are drawn like the reference's constructors draw them (scheme "reference"), with random LayerNorm
affine parameters and biases, so each source gives its own greedy stream: the tests assert that
the streams differ, and a negative control shows that handing a sequence another sequence's
source (and so its cross K/V) fails the logit check.

* mid encoder-decoder (d_model 512, 6+6 layers, vocab 16000): 8 sequences x all 128 steps of the
  mid workload (sources of 256 ids), the reference run live in worker processes.
* large encoder-decoder (d_model 1024, 12+12 layers, vocab 32000): 8 sequences x all 256 steps,
  sources of 128-1024 ids (one of 1024). The reference's run takes about 15 minutes of host time,
  so its ids and hidden rows are a committed fixture (tests/golden/make_lockstep_golden.py); the
  logits are rebuilt from them with the oracle's in-order product, bit for bit (checked against
  the stored row sums and top two).

Tolerance: |gpu - cpu| <= 1e-5 + 1e-4 |cpu| for every logit; argmax differences only at near ties.
"""
import os

import numpy as np
import pytest

from adai_b200.api import Context
from adai_b200.config import LARGE, MID
from adai_b200.synth import make_sources, make_weights, tensor_specs, weights_digest
from oracle.pyoracle import Ref
from tests.golden.make_lockstep_golden import LARGE_STEPS, OUT as LARGE_FIXTURE, large_inputs
from tests.lockstep import (LockstepReport, compare_row, distinct_stream_pairs, gpu_lockstep,
                            reference_generate_parallel)

pytestmark = pytest.mark.gpu

MID_SEED = 11
MID_SEQS, MID_SRC, MID_STEPS = 8, 256, 128


@pytest.fixture(scope="module")
def mid_reference():
    assert Ref.available(), "the reference build (oracle/_ref/libadai_ref.so) is missing"
    srcs = make_sources(MID, MID_SEQS, (MID_SRC, MID_SRC), MID_SEED)
    ids, logits = reference_generate_parallel("MID", MID_SEED, "reference", srcs, MID_STEPS)
    return srcs, ids, logits


@pytest.fixture(scope="module")
def mid_ctx():
    with Context(0) as c:
        c.upload(MID, make_weights(MID, MID_SEED, affine=True, scheme="reference"))
        yield c


def test_mid_full_lockstep_against_reference(mid_reference, mid_ctx):
    srcs, ids, logits = mid_reference
    frac = distinct_stream_pairs(ids)
    print(f"mid: {frac:.2f} of sequence pairs have different greedy streams")
    assert frac >= 0.5
    kv = mid_ctx.kv_arena(MID_SEQS, MID_STEPS, MID_SRC)
    slots = [3, 0, 7, 1, 6, 2, 5, 4]  # slots out of batch order
    rep = gpu_lockstep(kv, slots, srcs, ids, lambda t: logits[:, t], MID_STEPS)
    kv.close()
    print("mid lockstep against the reference build:", rep.summary())
    assert rep.steps == MID_SEQS * MID_STEPS
    assert rep.worst <= 1.0, rep.summary()
    assert all(tie for *_, tie in rep.mismatches), rep.mismatches


def test_swapped_sources_fail_the_logit_check(mid_reference, mid_ctx):
    # Negative control: sequences 0 and 1 are encoded from each other's source, so each reads the
    # other's cross K/V; the lockstep check must reject both at once and pass the others.
    srcs, ids, logits = mid_reference
    swapped = [srcs[1], srcs[0], srcs[2], srcs[3]]
    kv = mid_ctx.kv_arena(4, 8, MID_SRC)
    kv.encode([0, 1, 2, 3], swapped)
    reps = [LockstepReport() for _ in range(4)]
    feed = np.full(4, 2, np.int32)
    for t in range(4):
        nxt, lg = kv.decode_step([0, 1, 2, 3], feed, want_logits=True)
        for i in range(4):
            compare_row(reps[i], i, t, lg[i], logits[i, t], nxt[i], ids[i, t])
        feed = ids[:4, t].astype(np.int32)
    kv.close()
    print("swapped sources, worst tolerance ratio per sequence:",
          [round(r.worst, 3) for r in reps])
    assert reps[0].worst > 10.0 and reps[1].worst > 10.0
    assert reps[2].worst <= 1.0 and reps[3].worst <= 1.0


def test_large_full_lockstep_against_reference(port):
    assert os.path.exists(LARGE_FIXTURE), "tests/golden/large_lockstep.npz is missing"
    g = np.load(LARGE_FIXTURE)
    w, srcs = large_inputs()
    assert weights_digest(w) == str(g["weights_digest"]), "weight generator drifted"
    assert [len(s) for s in srcs] == g["src_lens"].tolist()
    ids, hidden = g["ids"], g["hidden"]
    n, steps = ids.shape
    assert steps == LARGE_STEPS and max(len(s) for s in srcs) == 1024
    frac = distinct_stream_pairs(ids)
    print(f"large: {frac:.2f} of sequence pairs have different greedy streams")
    assert frac >= 0.5
    names = [nm for nm, _ in tensor_specs(LARGE)]
    W = w[names.index("head.w")]
    bias = w[names.index("head.b")]
    # The reference's logits: LanguageModelHead::forward = hidden * W_output + bias
    # (src/LanguageModelHead.cpp:49-69), rebuilt with the oracle's in-order product.
    logits = np.empty((n, steps, LARGE.vocab), np.float32)
    for i in range(n):
        rec = port.matmul(hidden[i], W)
        rec += bias
        np.testing.assert_array_equal(np.cumsum(rec.astype(np.float64), axis=1)[:, -1],
                                      g["logit_sum"][i])
        np.testing.assert_array_equal(-np.sort(-rec, axis=1)[:, :2], g["top2"][i])
        logits[i] = rec
    with Context(0) as c:
        c.upload(LARGE, w)
        kv = c.kv_arena(n, steps, 1024)
        slots = [5, 2, 7, 0, 3, 6, 1, 4]
        rep = gpu_lockstep(kv, slots, srcs, ids, lambda t: logits[:, t], steps)
        kv.close()
    print("large lockstep against the reference build:", rep.summary())
    assert rep.steps == n * steps
    assert rep.worst <= 1.0, rep.summary()
    assert all(tie for *_, tie in rep.mismatches), rep.mismatches
