"""SafeTensors checkpoints in the reference's layout (ModelSerializer, src/ModelSerializer.cpp):
the library's reader against the Python writer, and the reference serializer tests' cases
(tests/model_serializer_test.cpp): round trip, a file with only the shared embedding, unknown keys
ignored, a missing required tensor, an architecture mismatch. The last case needs a device, so
it runs on the GPU, where the loaded model also decodes like the oracle.
"""
import json
import os
import struct

import numpy as np
import pytest

from adai_b200 import TINY
from adai_b200.api import checkpoint_config, read_checkpoint
from adai_b200.checkpoint import checkpoint_names, write_checkpoint, write_safetensors
from adai_b200.config import ModelConfig
from adai_b200.synth import make_sources, make_weights, tensor_specs

SMALL = ModelConfig(vocab=512, d_model=128, n_heads=2, d_ff=256, enc_layers=1, dec_layers=2,
                    max_seq=40)


def _read_raw(path):
    with open(path, "rb") as f:
        n = struct.unpack("<Q", f.read(8))[0]
        header = json.loads(f.read(n))
        data = f.read()
    out = {}
    for k, v in header.items():
        if k == "__metadata__":
            continue
        a, b = v["data_offsets"]
        out[k] = np.frombuffer(data[a:b], "<f4").reshape(v["shape"])
    return out


def _rewrite(src_dir, dst_dir, edit):
    """Copies a checkpoint, letting `edit` change the name -> tensor dict."""
    raw = _read_raw(os.path.join(src_dir, "model.safetensors"))
    edit(raw)
    os.makedirs(dst_dir, exist_ok=True)
    write_safetensors(os.path.join(dst_dir, "model.safetensors"), list(raw.items()))
    with open(os.path.join(src_dir, "config.json")) as f:
        cfg = f.read()
    with open(os.path.join(dst_dir, "config.json"), "w") as f:
        f.write(cfg)


@pytest.fixture(scope="module")
def ckpt(tmp_path_factory):
    d = str(tmp_path_factory.mktemp("ckpt"))
    w = make_weights(SMALL, 11, affine=True)
    write_checkpoint(d, SMALL, w)
    return d, w


def test_config_round_trip(ckpt):
    d, _ = ckpt
    assert checkpoint_config(d) == SMALL


def test_tensors_round_trip_bit_exact(ckpt):
    d, w = ckpt
    got = read_checkpoint(d)
    assert len(got) == len(w)
    for (name, _), a, b in zip(tensor_specs(SMALL), got, w):
        assert a.shape == b.shape, name
        assert np.array_equal(a, b), name


def test_layout_follows_the_reference_export(ckpt):
    d, w = ckpt
    raw = _read_raw(os.path.join(d, "model.safetensors"))
    names = checkpoint_names(SMALL)
    assert set(raw) == {n for n, _ in names}
    for (name, transposed), a in zip(names, w):
        np.testing.assert_array_equal(raw[name], a.T if transposed else a)
    # projections are [out, in] (HF convention), e.g. wi is [d_ff, d_model]
    assert raw["model.decoder.block.1.layer.2.DenseReluDense.wi.weight"].shape == (256, 128)
    assert raw["lm_head.weight"].shape == (512, 128)


def test_only_shared_embedding_goes_to_both(ckpt, tmp_path):
    d, w = ckpt
    _rewrite(d, str(tmp_path), lambda r: r.pop("model.decoder.embed_tokens.weight"))
    got = read_checkpoint(str(tmp_path))
    i_dec = [n for n, _ in tensor_specs(SMALL)].index("dec.embed")
    np.testing.assert_array_equal(got[i_dec], w[0])


def test_missing_final_norms_default_to_identity(ckpt, tmp_path):
    d, _ = ckpt

    def drop(r):
        for k in [k for k in r if "final_layer_norm" in k]:
            r.pop(k)
    _rewrite(d, str(tmp_path), drop)
    got = dict(zip([n for n, _ in tensor_specs(SMALL)], read_checkpoint(str(tmp_path))))
    for p in ("enc.lnf", "dec.lnf"):
        np.testing.assert_array_equal(got[p + ".g"], np.ones(128, np.float32))
        np.testing.assert_array_equal(got[p + ".b"], np.zeros(128, np.float32))


def test_unknown_tensor_keys_are_ignored(ckpt, tmp_path):
    d, w = ckpt

    def add(r):
        r["encoder.block.0.layer.0.SelfAttention.relative_attention_bias.weight"] = np.ones((32, 2), np.float32)
    _rewrite(d, str(tmp_path), add)
    got = read_checkpoint(str(tmp_path))
    assert all(np.array_equal(a, b) for a, b in zip(got, w))


def test_missing_required_tensor_is_named(ckpt, tmp_path):
    d, _ = ckpt
    gone = "model.decoder.block.1.layer.1.EncDecAttention.v.weight"
    _rewrite(d, str(tmp_path), lambda r: r.pop(gone))
    with pytest.raises(ValueError, match="required tensor missing: " + gone.replace(".", r"\.")):
        read_checkpoint(str(tmp_path))


def test_wrong_shape_and_dtype_are_rejected(ckpt, tmp_path):
    d, _ = ckpt
    _rewrite(d, str(tmp_path / "shape"), lambda r: r.update({"lm_head.bias": np.zeros(511, np.float32)}))
    with pytest.raises(ValueError, match="lm_head.bias"):
        read_checkpoint(str(tmp_path / "shape"))
    # an F16 tensor: rewrite the header's dtype and halve the byte range of the last tensor
    src = os.path.join(d, "model.safetensors")
    with open(src, "rb") as f:
        n = struct.unpack("<Q", f.read(8))[0]
        header = json.loads(f.read(n))
        data = f.read()
    header["lm_head.bias"]["dtype"] = "F16"
    h = json.dumps(header).encode()
    h += b" " * (-len(h) % 8)
    os.makedirs(tmp_path / "f16")
    with open(tmp_path / "f16" / "model.safetensors", "wb") as f:
        f.write(struct.pack("<Q", len(h)) + h + data)
    with open(tmp_path / "f16" / "config.json", "w") as f:
        f.write(open(os.path.join(d, "config.json")).read())
    with pytest.raises(ValueError, match="F16"):
        read_checkpoint(str(tmp_path / "f16"))


def test_malformed_files_fail_cleanly(ckpt, tmp_path):
    d, _ = ckpt
    with pytest.raises(OSError):
        checkpoint_config(str(tmp_path / "absent"))
    os.makedirs(tmp_path / "bad")
    with open(tmp_path / "bad" / "config.json", "w") as f:
        f.write('{"vocab_size": 512, "d_model": ')
    with pytest.raises(ValueError, match="malformed JSON"):
        checkpoint_config(str(tmp_path / "bad"))
    for blob in (b"", struct.pack("<Q", 1 << 40), struct.pack("<Q", 4) + b"{}"):
        with open(tmp_path / "bad" / "model.safetensors", "wb") as f:
            f.write(blob)
        with pytest.raises(ValueError):
            read_checkpoint(str(tmp_path / "bad"), SMALL)
    with open(os.path.join(d, "model.safetensors"), "rb") as f:
        whole = f.read()
    with open(tmp_path / "bad" / "model.safetensors", "wb") as f:
        f.write(whole[: len(whole) - 100])   # data cut short: ranges now outside the file
    with pytest.raises(ValueError, match="outside the file"):
        read_checkpoint(str(tmp_path / "bad"), SMALL)


@pytest.mark.gpu
def test_loaded_checkpoint_decodes_like_the_oracle(tmp_path, port):
    from adai_b200 import Context
    w = make_weights(TINY, 7, affine=True)
    write_checkpoint(str(tmp_path), TINY, w)
    srcs = make_sources(TINY, 3, (5, 30), 7)
    with Context(0) as c:
        assert c.load(str(tmp_path), expect=TINY) == TINY
        kv = c.kv_arena(3, 8, 32)
        kv.encode([0, 1, 2], srcs)
        got = kv.generate([0, 1, 2], [2, 2, 2], 8)
        kv.close()
        wrong = ModelConfig(TINY.vocab, TINY.d_model, TINY.n_heads, TINY.d_ff, TINY.enc_layers,
                            TINY.dec_layers + 1, TINY.max_seq)
        with pytest.raises(ValueError, match="architecture mismatch"):
            c.load(str(tmp_path), expect=wrong)
    m = port.model(TINY, w)
    for i, s in enumerate(srcs):
        np.testing.assert_array_equal(got[i], m.generate(s, 8)[0])
