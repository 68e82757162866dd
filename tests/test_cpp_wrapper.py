"""include/adai_b200.hpp, the C++ wrapper a reference-side C++ host would use: it compiles against
the C ABI, maps status codes to the reference's exception types, and its BatchGenerator (the
stacked counterpart of BatchedInferenceEngine::process_batch, src/BatchedInferenceEngine.hpp:465-537)
returns what TextGenerator::generate_greedy returns per request (src/TextGenerator.cpp:209-233)."""
import os
import shutil
import subprocess

import numpy as np
import pytest

from adai_b200 import TINY
from adai_b200.synth import make_sources, make_weights
from tests.conftest import ROOT

SRC = os.path.join(ROOT, "tests", "cpp", "batch_generate.cpp")
LIBDIR = os.path.join(ROOT, "adai_b200")
STOP = (3, 0)  # EOS, PAD: adai::is_stop_token (src/SpecialTokens.hpp:162-164)


@pytest.fixture(scope="module")
def driver(tmp_path_factory):
    gxx = shutil.which("g++")
    if gxx is None:
        pytest.skip("no C++ compiler")
    out = str(tmp_path_factory.mktemp("cpp") / "batch_generate")
    subprocess.run([gxx, "-std=c++17", "-O1", "-Wall", "-Wextra", "-Werror",
                    "-I" + os.path.join(ROOT, "include"), SRC, "-L" + LIBDIR, "-ladai_b200",
                    "-Wl,-rpath," + LIBDIR, "-o", out], check=True)
    return out


def test_wrapper_refuses_without_device(driver):
    torch = pytest.importorskip("torch")
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    got = subprocess.run([driver], check=True, capture_output=True, text=True).stdout
    assert got.startswith("no-device: runtime_error:"), got


def _write_requests(path, cfg, weights, slots, reqs):
    with open(path, "wb") as f:
        np.asarray(list(cfg.as_cfg()) + [len(weights)], np.int32).tofile(f)
        for w in weights:
            np.asarray([w.size], np.int64).tofile(f)
            np.ascontiguousarray(w, np.float32).tofile(f)
        np.asarray([slots, len(reqs)], np.int32).tofile(f)
        for max_len, src in reqs:
            np.asarray([max_len, len(src)], np.int32).tofile(f)
            np.asarray(src, np.int32).tofile(f)


def _greedy(model, src, max_len):
    ids, _ = model.generate(src, max_len)
    out = [2]
    for t in ids.tolist():
        out.append(t)
        if t in STOP:
            break
    return out


@pytest.mark.gpu
def test_batch_generator_matches_oracle(driver, tmp_path, port):
    w = make_weights(TINY, 3, affine=True)
    srcs = make_sources(TINY, 7, (5, 40), 3)
    lens = [12, 1, 20, 0, 7, 20, 3]
    reqs = list(zip(lens, srcs))
    reqs.insert(2, (5, [4, 5, TINY.vocab + 9]))   # out-of-vocabulary id: this request alone fails
    path = str(tmp_path / "req.bin")
    _write_requests(path, TINY, w, 3, reqs)      # 3 slots: the requests run in three waves
    out = subprocess.run([driver, path], check=True, capture_output=True, text=True,
                         timeout=300).stdout.splitlines()
    assert len(out) == len(reqs)
    model = port.model(TINY, w)
    for i, (max_len, src) in enumerate(reqs):
        head, rest = out[i].split(":", 1)
        assert int(head) == i
        if i == 2:
            assert rest.startswith(" error:"), out[i]
            continue
        got = [int(t) for t in rest.split()]
        want = _greedy(model, src, max_len) if max_len > 0 else [2]
        assert got == want, (i, got, want)
