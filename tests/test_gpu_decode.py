"""The stacked decode step end to end through the C ABI, against the CPU oracle.

The bar (from the decode-path specification): greedy token ids identical to the reference CPU
path, logits within |gpu - cpu| <= 1e-5 + 1e-4 |cpu|. Checked in lockstep (each step fed the
oracle's own token, as benchmarks/GpuDecodeBenchmark.cpp:347-375 does) so that one near-tie
cannot cascade, and free-running (greedy, ids fed back on the device) for whole generations.
"""
import numpy as np
import pytest

from adai_b200.api import Context, StateError
from adai_b200.config import LARGE, MID, TINY
from adai_b200.synth import make_sources, make_weights
from tests.conftest import tol_ratio
from tests.golden.make_golden import DECODE_LOGIT_STEPS, DECODE_SEQS, DECODE_SRC, DECODE_STEPS

pytestmark = pytest.mark.gpu

BOS = 2


def near_tie(logits_row, tol_abs):
    top2 = np.sort(logits_row)[-2:]
    return (top2[1] - top2[0]) <= 2 * tol_abs


def lockstep(kv, cfg, model, slots, srcs, steps):
    """Feeds every sequence the oracle's greedy tokens; returns the worst tolerance ratio over
    all logits and the list of (seq, step) where the argmax differed."""
    want = [model.generate(s, steps, want_logits=True) for s in srcs]
    kv.encode(slots, srcs)
    worst, mismatch = 0.0, []
    feed = np.full(len(srcs), BOS, np.int32)
    for t in range(steps):
        nxt, lg = kv.decode_step(slots, feed, want_logits=True)
        for i in range(len(srcs)):
            wid, wlg = want[i][0][t], want[i][1][t]
            worst = max(worst, tol_ratio(lg[i], wlg))
            if nxt[i] != wid:
                mismatch.append((i, t, near_tie(wlg, np.abs(lg[i] - wlg).max())))
            feed[i] = wid
    return worst, mismatch


@pytest.fixture(scope="module")
def tiny(ctx):
    w = make_weights(TINY, 0, affine=True)
    ctx.upload(TINY, w)
    return w


def test_encoder_output_matches_oracle(ctx, port, tiny, golden):
    kv = ctx.kv_arena(4, 64, 64)
    srcs = make_sources(TINY, DECODE_SEQS, (DECODE_SRC, DECODE_SRC), 0)
    out = kv.encode([0, 1, 2], srcs, want_output=True)
    assert tol_ratio(out[:DECODE_SRC], golden["tiny_enc0"]) <= 1.0
    m = port.model(TINY, tiny)
    for i, s in enumerate(srcs):
        assert tol_ratio(out[i * DECODE_SRC:(i + 1) * DECODE_SRC], m.encode(s)) <= 1.0
    kv.close()


def test_tiny_lockstep_against_golden(ctx, tiny, golden):
    kv = ctx.kv_arena(DECODE_SEQS, 32, 32)
    srcs = make_sources(TINY, DECODE_SEQS, (DECODE_SRC, DECODE_SRC), 0)
    kv.encode(list(range(DECODE_SEQS)), srcs)
    feed = np.full(DECODE_SEQS, BOS, np.int32)
    for t in range(DECODE_STEPS):
        nxt, lg = kv.decode_step(list(range(DECODE_SEQS)), feed, want_logits=True)
        np.testing.assert_array_equal(nxt, golden["tiny_ids"][:, t])
        if t < DECODE_LOGIT_STEPS:
            assert tol_ratio(lg, golden["tiny_logits"][:, t]) <= 1.0
        feed = golden["tiny_ids"][:, t].astype(np.int32)
    kv.close()


def test_tiny_workload_free_running_greedy(ctx, port, tiny):
    # The tiny encoder-decoder workload: batch 8, source length 64, 32 greedy tokens.
    srcs = make_sources(TINY, 8, (64, 64), 0)
    kv = ctx.kv_arena(8, 40, 64)
    kv.encode(list(range(8)), srcs)
    got = kv.generate(list(range(8)), [BOS] * 8, 32)
    m = port.model(TINY, tiny)
    for i, s in enumerate(srcs):
        np.testing.assert_array_equal(got[i], m.generate(s, 32)[0])
    assert kv.length(3) == (32, 64)
    kv.close()


def test_generate_equals_repeated_decode_step(ctx, tiny):
    srcs = make_sources(TINY, 5, (10, 40), 9)
    slots = [4, 0, 7, 2, 5]   # non-contiguous slots, ragged sources
    kv1 = ctx.kv_arena(8, 24, 64)
    kv1.encode(slots, srcs)
    g = kv1.generate(slots, [BOS] * 5, 20)
    kv2 = ctx.kv_arena(8, 24, 64)
    kv2.encode(slots, srcs)
    feed = np.full(5, BOS, np.int32)
    for t in range(20):
        nxt, _ = kv2.decode_step(slots, feed)
        np.testing.assert_array_equal(nxt, g[:, t])
        feed = nxt
    kv1.close()
    kv2.close()


def test_ragged_batch_lockstep_with_random_affine(ctx, port, tiny):
    srcs = make_sources(TINY, 6, (1, 64), 21)
    kv = ctx.kv_arena(6, 16, 64)
    worst, mism = lockstep(kv, TINY, port.model(TINY, tiny), [5, 3, 1, 0, 2, 4], srcs, 16)
    assert worst <= 1.0, worst
    assert all(tie for _, _, tie in mism), mism
    kv.close()


@pytest.mark.parametrize("offset", [4.0, 16.0])
def test_folded_layernorm_on_rows_with_a_large_mean(port, offset):
    # The decode step folds each LayerNorm into the GEMM after it, which subtracts
    # mean * colsum(diag(gamma) W) from the product of the raw rows: the cancellation grows with
    # |mean| / std of a row. A decoder embedding shifted by `offset` gives every residual row a
    # mean of about offset against a spread below 1.
    from adai_b200.synth import tensor_specs
    w = make_weights(TINY, 13, affine=True)
    names = [n for n, _ in tensor_specs(TINY)]
    w[names.index("dec.embed")] = w[names.index("dec.embed")] + np.float32(offset)
    with Context(0) as c:
        c.upload(TINY, w)
        srcs = make_sources(TINY, 4, (8, 48), 13)
        kv = c.kv_arena(4, 16, 64)
        worst, mism = lockstep(kv, TINY, port.model(TINY, w), [0, 1, 2, 3], srcs, 12)
        print(f"row mean offset {offset}: worst tolerance ratio {worst:.4f}")
        assert worst <= 1.0, worst
        assert all(tie for _, _, tie in mism), mism
        kv.close()


def test_mid_model_lockstep(port):
    # Mid encoder-decoder (d_model 512, 8 heads, 6+6 layers, d_ff 2048, vocab 16000); 4 of the
    # workload's 64 sequences (source length 256), 12 steps.
    with Context(0) as c:
        w = make_weights(MID, 1)
        c.upload(MID, w)
        srcs = make_sources(MID, 4, (256, 256), 1)
        kv = c.kv_arena(4, 16, 256)
        worst, mism = lockstep(kv, MID, port.model(MID, w), [0, 1, 2, 3], srcs, 12)
        print(f"mid lockstep: worst tolerance ratio {worst:.4f}")
        assert worst <= 1.0, worst
        assert all(tie for _, _, tie in mism), mism
        kv.close()


def test_large_model_lockstep(port):
    # Large encoder-decoder (d_model 1024, 16 heads, 12+12 layers, d_ff 4096, vocab 32000); two
    # sequences with sources of 130 and 300 ids (the workload's range is 128-1024), 4 steps.
    with Context(0) as c:
        w = make_weights(LARGE, 2)
        c.upload(LARGE, w)
        srcs = make_sources(LARGE, 2, (128, 300), 2)
        kv = c.kv_arena(2, 8, 1024)
        worst, mism = lockstep(kv, LARGE, port.model(LARGE, w), [0, 1], srcs, 4)
        print(f"large lockstep: worst tolerance ratio {worst:.4f}")
        assert worst <= 1.0, worst
        assert all(tie for _, _, tie in mism), mism
        kv.close()


def test_errors_follow_reference_exceptions(ctx, tiny):
    kv = ctx.kv_arena(2, 2, 16)
    with pytest.raises(StateError):          # no encoder output yet
        kv.decode_step([0], [BOS])
    src = make_sources(TINY, 1, (8, 8), 0)
    kv.encode([0], src)
    with pytest.raises(IndexError):          # TokenEmbedding: id out of range
        kv.decode_step([0], [TINY.vocab])
    with pytest.raises(IndexError):          # slot out of range
        kv.decode_step([2], [BOS])
    with pytest.raises(ValueError):          # one slot twice in a batch
        kv.encode([1, 1], src * 2)
    with pytest.raises(ValueError):          # encoder input longer than max_seq_length
        kv.encode([1], [np.arange(4, 4 + TINY.max_seq + 1) % TINY.vocab])
    kv.decode_step([0], [BOS])
    kv.decode_step([0], [BOS])
    with pytest.raises(IndexError):          # self-attention cache full
        kv.decode_step([0], [BOS])
    kv.reset(0)
    assert kv.length(0) == (0, 0)
    kv.close()


def test_lm_head_argmax_first_maximum_and_nonfinite():
    """The fused LM-head argmax returns the first maximum (TextGenerator::argmax's strict `>`,
    src/TextGenerator.cpp:151-153) when equal maxima sit in the same N tile and in other tiles,
    and a NaN or +inf logit, or a row of -inf, fails the step as next_logits throws
    (src/TextGenerator.cpp:177-206)."""
    from adai_b200.api import NonFiniteLogits
    srcs = make_sources(TINY, 3, (5, 20), 9)
    base = make_weights(TINY, 5, affine=True)
    with Context(0) as c:
        def run(weights):
            c.upload(TINY, weights)
            kv = c.kv_arena(3, 4, 32)
            kv.encode([0, 1, 2], srcs)
            return kv
        w = [a.copy() for a in base]
        hw, hb = w[-2], w[-1]                  # head.w [D, V], head.b [V]
        for col in (9, 4000, 4095):            # same tile as 5, later tiles, the last column
            hw[:, col] = hw[:, 5]
        hb[[5, 9, 4000, 4095]] = 60.0
        kv = run(w)
        nxt, lg = kv.decode_step([0, 1, 2], [BOS] * 3, want_logits=True)
        assert (lg[:, 5] == lg[:, 9]).all() and (lg[:, 5] == lg[:, 4000]).all()
        assert (lg[:, 5] == lg[:, 4095]).all()
        assert nxt.tolist() == [5, 5, 5]
        assert (kv.generate([0, 1, 2], [5] * 3, 3) == 5).all()
        kv.close()
        for bad in ("nan", "inf", "all-neg-inf"):
            w = [a.copy() for a in base]
            if bad == "all-neg-inf":
                w[-1][:] = -np.inf
            else:
                w[-1][7] = float(bad)
            kv = run(w)
            with pytest.raises(NonFiniteLogits):
                kv.decode_step([0, 1, 2], [BOS] * 3)
            kv.close()


def test_decoding_past_the_positional_table(port):
    # Past max_seq_length no positional row is added (src/Decoder.cpp:230-242); 20 steps with a
    # 12-row table, lockstep against the oracle.
    from adai_b200.config import ModelConfig
    cfg = ModelConfig(vocab=512, d_model=128, n_heads=2, d_ff=256, enc_layers=1, dec_layers=2,
                      max_seq=12)
    with Context(0) as c:
        w = make_weights(cfg, 8, affine=True)
        c.upload(cfg, w)
        srcs = make_sources(cfg, 3, (4, 12), 8)
        kv = c.kv_arena(3, 24, 12)
        worst, mism = lockstep(kv, cfg, port.model(cfg, w), [0, 1, 2], srcs, 20)
        assert worst <= 1.0, worst
        assert all(tie for _, _, tie in mism), mism
        kv.close()


def test_device_wait_timeout_reaches_the_host():
    # A device-side bounded wait on a barrier nothing completes gives up after its 2 s limit and
    # records its code; the host reports the timeout and refuses further work on that context
    # (GPU_WAIT_TIMEOUT_SECONDS semantics). No fault is involved: the kernel ends normally, and a
    # new context on the same device works.
    c = Context(0)
    waited = c.check_wait_timeout()
    assert 1.5 < waited < 30.0, waited         # one 2 s deadline; the second wait returns at once
    with pytest.raises(StateError, match="unusable"):
        c.upload(TINY, make_weights(TINY, 0))
    c.close()
    with Context(0) as fresh:
        fresh.upload(TINY, make_weights(TINY, 0))
        kv = fresh.kv_arena(1, 4, 8)
        kv.encode([0], make_sources(TINY, 1, (8, 8), 0))
        assert kv.generate([0], [BOS], 2).shape == (1, 2)
        kv.close()


def test_wide_batch_one_attention_cta_per_head(ctx, port, tiny):
    # 160 sequences x 4 heads: enough (sequence, head) pairs that each attention CTA takes every
    # cached row of its pair (no split-KV merge); ragged sources, lockstep with the oracle.
    B = 160
    srcs = make_sources(TINY, B, (4, 48), 13)
    kv = ctx.kv_arena(B, 12, 48)
    worst, mismatch = lockstep(kv, TINY, port.model(TINY, tiny), list(range(B)), srcs, 6)
    kv.close()
    assert worst <= 1.0, worst
    assert all(tie for _, _, tie in mismatch), mismatch


def test_empty_sources_decode_like_the_oracle(ctx, port, tiny):
    # An empty source (no encoder rows, cross-attention contributes zeros) mixed into a batch,
    # and a batch whose sources are all empty (nothing to encode).
    srcs = make_sources(TINY, 4, (5, 30), 17)
    srcs[1] = np.zeros(0, np.int32)
    kv = ctx.kv_arena(4, 10, 32)
    worst, mismatch = lockstep(kv, TINY, port.model(TINY, tiny), [0, 1, 2, 3], srcs, 8)
    assert kv.length(1) == (8, 0)
    kv.close()
    assert worst <= 1.0, worst
    assert all(tie for _, _, tie in mismatch), mismatch
    kv = ctx.kv_arena(2, 10, 32)
    empties = [np.zeros(0, np.int32)] * 2
    worst, mismatch = lockstep(kv, TINY, port.model(TINY, tiny), [0, 1], empties, 8)
    kv.close()
    assert worst <= 1.0, worst
    assert not mismatch, mismatch
    kv = ctx.kv_arena(1, 4, 8)
    with pytest.raises(StateError):  # never encoded: refused, as before
        kv.decode_step([0], [BOS])
    kv.close()


def test_maximum_source_length_and_last_vocabulary_id(ctx, port, tiny):
    # A source of exactly max_seq_length ids (the largest LLMEncoder accepts) decodes in lockstep
    # with the oracle; the last id of the vocabulary is a valid decoder input.
    m = port.model(TINY, tiny)
    src = [(np.arange(TINY.max_seq, dtype=np.int32) * 37 + 4) % TINY.vocab]
    kv = ctx.kv_arena(1, 8, TINY.max_seq)
    worst, mismatch = lockstep(kv, TINY, m, [0], src, 6)
    assert worst <= 1.0, worst
    assert all(tie for _, _, tie in mismatch), mismatch
    kv.reset(0)
    kv.encode([0], src)
    nxt, lg = kv.decode_step([0], [TINY.vocab - 1], want_logits=True)
    want_ids, want_lg = m.generate(src[0], 1, bos=TINY.vocab - 1, want_logits=True)
    assert tol_ratio(lg[0], want_lg[0]) <= 1.0
    assert nxt[0] == want_ids[0] or near_tie(want_lg[0], np.abs(lg[0] - want_lg[0]).max())
    kv.close()
