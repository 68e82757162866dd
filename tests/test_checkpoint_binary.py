"""The reference's own checkpoint files (EncoderDecoderModel::save_model, src/EncoderDecoderModel.cpp:
960-985), written here by the reference's code (oracle/_ref: LLMEncoder / LLMDecoder /
LanguageModelHead::save_weights), read by the library's native reader.

Cases follow the reference's tests of this format: the round trip (tests/decoder_test.cpp:733,
tests/crossattention_test.cpp:1361), a short read, trailing data and a missing file
(tests/binaryio_test.cpp:35-65), dimension mismatches (tests/decoder_test.cpp:711,
tests/crossattention_test.cpp:1468), the format marker (src/EncoderDecoderModel.cpp:987-1013), the
pre-TD-538 encoder fallback (src/LLMEncoder.cpp:326-349) and gated decoder paths
(tests/decoderblock_test.cpp:1731).
"""
import os
import shutil
import struct

import numpy as np
import pytest

from adai_b200 import TINY
from adai_b200.api import checkpoint_config, checkpoint_special_tokens, read_checkpoint
from adai_b200.config import ModelConfig
from adai_b200.synth import make_sources, make_weights
from oracle.pyoracle import Ref

SMALL = ModelConfig(vocab=300, d_model=128, n_heads=2, d_ff=96, enc_layers=2, dec_layers=2,
                    max_seq=40)


@pytest.fixture(scope="module")
def ref():
    if not Ref.available():
        pytest.skip("reference build absent (make -C oracle ref)")
    return Ref()


@pytest.fixture(scope="module")
def saved(ref, tmp_path_factory):
    d = tmp_path_factory.mktemp("binckpt")
    w = make_weights(SMALL, 21, affine=True)
    m = ref.model(SMALL, w)
    prefix = str(d / "model")
    m.save(prefix, bos=7, eos=8, pad=9)
    return prefix, w


def clone(prefix, dst_dir):
    """Copies every file of the checkpoint at `prefix` into dst_dir; returns the new prefix."""
    src_dir, stem = os.path.split(prefix)
    os.makedirs(dst_dir, exist_ok=True)
    for f in os.listdir(src_dir):
        if f.startswith(stem):
            shutil.copy(os.path.join(src_dir, f), os.path.join(dst_dir, f))
    return os.path.join(dst_dir, stem)


def test_files_are_the_save_model_layout(saved):
    prefix, _ = saved
    names = sorted(os.listdir(os.path.dirname(prefix)))
    for want in ["model.config", "model.encoder", "model.decoder", "model.lm_head",
                 "model_encoder_token_emb.bin", "model_encoder_final_norm.bin",
                 "model_encoder_block_1.bin", "model_encoder_block_1_attention.bin",
                 "model_encoder_block_1_feedforward.bin", "model_token_emb.bin",
                 "model_final_norm.bin", "model_decoder_block_1.bin",
                 "model_decoder_block_1.bin.self_attn", "model_decoder_block_1.bin.cross_attn",
                 "model_decoder_block_1.bin.ff"]:
        assert want in names, (want, names)


def test_config_and_special_tokens(saved):
    prefix, _ = saved
    assert checkpoint_config(prefix) == SMALL
    assert checkpoint_special_tokens(prefix) == (7, 8, 9)


def test_round_trip_bit_exact(saved):
    prefix, w = saved
    got = read_checkpoint(prefix, SMALL)
    assert len(got) == len(w)
    for i, (a, b) in enumerate(zip(got, w)):
        np.testing.assert_array_equal(a.reshape(b.shape), b, err_msg=f"tensor {i}")


def test_pre_td538_encoder_takes_the_shared_files(saved, tmp_path):
    # Checkpoints written before the encoder-specific names hold only model_token_emb.bin and
    # model_final_norm.bin (the decoder's); the reference loads those for the encoder too.
    prefix, w = saved
    p = clone(prefix, str(tmp_path / "old"))
    os.remove(p + "_encoder_token_emb.bin")
    os.remove(p + "_encoder_final_norm.bin")
    got = read_checkpoint(p, SMALL)
    n_enc = 1 + 12 * SMALL.enc_layers
    dec_embed = w[n_enc + 2]
    np.testing.assert_array_equal(got[0].reshape(dec_embed.shape), dec_embed)
    np.testing.assert_array_equal(got[n_enc], w[-4])      # decoder final norm gamma
    np.testing.assert_array_equal(got[n_enc + 1], w[-3])  # and beta


def _patch(path, offset, fmt, value):
    with open(path, "r+b") as f:
        f.seek(offset)
        f.write(struct.pack(fmt, value))


def test_truncated_trailing_and_missing_files(saved, tmp_path):
    prefix, _ = saved
    p = clone(prefix, str(tmp_path / "t"))
    f = p + "_decoder_block_0.bin.ff"
    data = open(f, "rb").read()
    open(f, "wb").write(data[:-5])
    with pytest.raises(OSError, match="Truncated"):
        read_checkpoint(p, SMALL)
    open(f, "wb").write(data + b"\0")
    with pytest.raises(ValueError, match="trailing data"):
        read_checkpoint(p, SMALL)
    open(f, "wb").write(data)
    os.remove(p + ".lm_head")
    with pytest.raises(OSError, match="lm_head"):
        read_checkpoint(p, SMALL)
    with pytest.raises(OSError, match="no checkpoint"):
        checkpoint_config(str(tmp_path / "nothing"))


def test_dimension_and_architecture_mismatches(saved, tmp_path):
    prefix, _ = saved
    p = clone(prefix, str(tmp_path / "d"))
    _patch(p + "_encoder_block_1_attention.bin", 4, "<i", 4)      # num_heads 2 -> 4
    with pytest.raises(ValueError, match="num_heads"):
        read_checkpoint(p, SMALL)
    p = clone(prefix, str(tmp_path / "e"))
    _patch(p + ".decoder", 0, "<i", 301)                          # vocab in the decoder header
    with pytest.raises(ValueError, match="vocab_size"):
        read_checkpoint(p, SMALL)
    other = ModelConfig(SMALL.vocab, SMALL.d_model, SMALL.n_heads, SMALL.d_ff, SMALL.enc_layers,
                        SMALL.dec_layers, SMALL.max_seq + 1)
    with pytest.raises(ValueError, match="architecture mismatch"):
        read_checkpoint(prefix, other)


def test_format_marker_version_epsilon_and_gated_paths(saved, tmp_path):
    prefix, _ = saved
    p = clone(prefix, str(tmp_path / "m"))
    _patch(p + ".config", 0, "<i", 1234)
    with pytest.raises(ValueError, match="format marker"):
        checkpoint_config(p)
    p = clone(prefix, str(tmp_path / "v"))
    _patch(p + ".config", 4, "<i", 1)
    with pytest.raises(ValueError, match="format_version"):
        checkpoint_config(p)
    p = clone(prefix, str(tmp_path / "eps"))
    _patch(p + "_final_norm.bin", 4, "<f", 1e-6)                  # LayerNorm epsilon
    with pytest.raises(ValueError, match="epsilon"):
        read_checkpoint(p, SMALL)
    p = clone(prefix, str(tmp_path / "g"))
    blk = p + "_decoder_block_1.bin"
    data = bytearray(open(blk, "rb").read())
    assert data[-2:] == b"\0\0"                                   # both gated-path flags clear
    # world-model path present: its flag, its gate value, then the hippocampal flag
    open(blk, "wb").write(bytes(data[:-2]) + b"\x01" + struct.pack("<f", 0.5) + b"\x00")
    with pytest.raises(ValueError, match="world-model"):
        read_checkpoint(p, SMALL)


@pytest.mark.gpu
def test_reference_checkpoint_loads_and_decodes_like_the_oracle(ref, tmp_path, port):
    from adai_b200 import Context
    w = make_weights(TINY, 8, affine=True)
    prefix = str(tmp_path / "m")
    ref.model(TINY, w).save(prefix)
    srcs = make_sources(TINY, 3, (5, 30), 8)
    with Context(0) as c:
        assert c.load(prefix, expect=TINY) == TINY
        kv = c.kv_arena(3, 8, 32)
        kv.encode([0, 1, 2], srcs)
        got = kv.generate([0, 1, 2], [2, 2, 2], 8)
        kv.close()
    m = port.model(TINY, w)
    for i, s in enumerate(srcs):
        np.testing.assert_array_equal(got[i], m.generate(s, 8)[0])
