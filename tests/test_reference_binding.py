"""The reference-side half of the binding, built against the reference's own sources (CPU).

* include/adai_b200_reference.hpp walks the reference's LLMEncoder / LLMDecoder /
  LanguageModelHead through their public getters into adai_b200_model_upload's tensor order.
  tests/cpp/upload_order.cpp (built by `make -C oracle binding` against the reference objects)
  initialises the three components with the reference's own random draws, writes the walked
  tensors and the reference's own greedy decode; here the tensors replay through the oracle in
  upload order, and the ids and logits must match.
* tests/cpp/backend_table.cpp compiles against the reference's src/gpu/MatrixGPU.hpp and links to
  libadai_b200.so (`make -C oracle boundary`): untouched callers of the matrix_*_gpu table resolve
  every symbol they use. The GPU test runs that program (tests/test_gpu_backend.py).
"""
import os
import subprocess

import numpy as np
import pytest

from adai_b200.config import ModelConfig
from adai_b200.synth import tensor_specs
from tests.conftest import ROOT, tol_ratio

REF = os.environ.get("ADAI_REFERENCE", "/root/reference")
OUT = os.path.join(ROOT, "oracle", "_ref")
have_reference = pytest.mark.skipif(not os.path.isdir(os.path.join(REF, "src")),
                                    reason="reference sources not on this host")

SMALL = ModelConfig(vocab=512, d_model=128, n_heads=4, d_ff=256, enc_layers=1, dec_layers=2,
                    max_seq=64)


def _make(target):
    subprocess.run(["make", "-s", "-C", os.path.join(ROOT, "oracle"), target, f"REF={REF}"],
                   check=True, timeout=900)


@have_reference
def test_upload_order_walk_replays_the_reference_decode(tmp_path, port):
    _make("binding")
    cfg, steps = SMALL, 8
    src = list(range(5, 5 + 29, 1))
    out = str(tmp_path / "walk.bin")
    subprocess.run([os.path.join(OUT, "upload_order"), out] +
                   [str(v) for v in cfg.as_cfg()[:6]] + [str(cfg.max_seq), str(steps)] +
                   [str(v) for v in src], check=True, timeout=300, capture_output=True)
    with open(out, "rb") as f:
        n = int(np.fromfile(f, np.int32, 1)[0])
        tensors = []
        for _ in range(n):
            c = int(np.fromfile(f, np.int64, 1)[0])
            tensors.append(np.fromfile(f, np.float32, c))
        st = int(np.fromfile(f, np.int32, 1)[0])
        ids = np.fromfile(f, np.int32, st)
        logits = np.fromfile(f, np.float32, st * cfg.vocab).reshape(st, cfg.vocab)
    specs = tensor_specs(cfg)
    assert n == len(specs)
    weights = []
    for (name, shape), t in zip(specs, tensors):
        assert t.size == int(np.prod(shape)), name
        weights.append(t.reshape(shape))
    got_ids, got_lg = port.model(cfg, weights).generate(np.asarray(src, np.int32), steps,
                                                        want_logits=True)
    np.testing.assert_array_equal(got_ids, ids)
    assert tol_ratio(got_lg, logits) <= 1.0


@have_reference
def test_backend_table_builds_against_the_reference_header():
    _make("boundary")
    exe = os.path.join(OUT, "backend_table_refhdr")
    assert os.path.exists(exe)
    undefined = subprocess.run(["nm", "-C", "--undefined-only", exe], check=True,
                               capture_output=True, text=True).stdout
    for fn in ("matrix_multiply_gpu", "matrix_gemm_strided_gpu", "matrix_softmax_rows_gpu",
               "matrix_layer_norm_fwd_gpu", "matrix_add_row_bias_gpu",
               "matrix_apply_activation_gpu", "embedding_gather_add_pe_gpu"):
        assert f"adai::gpu::{fn}(" in undefined, fn
    exported = subprocess.run(["nm", "-C", "-D", "--defined-only",
                               os.path.join(ROOT, "adai_b200", "libadai_b200.so")],
                              check=True, capture_output=True, text=True).stdout
    for ln in undefined.splitlines():
        if "adai::gpu::" in ln:
            assert ln.split(" U ", 1)[1].strip() in exported, ln
