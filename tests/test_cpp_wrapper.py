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
        for rq in reqs:
            max_len, src = rq[0], rq[1]
            smp = rq[2] if len(rq) > 2 else None
            np.asarray([max_len, len(src)], np.int32).tofile(f)
            np.asarray(src, np.int32).tofile(f)
            np.asarray([0 if smp is None else 1], np.int32).tofile(f)
            if smp is not None:
                np.asarray([smp["temperature"]], np.float32).tofile(f)
                np.asarray([smp["top_k"]], np.int32).tofile(f)
                np.asarray([smp["top_p"], smp["repetition_penalty"]], np.float32).tofile(f)
                np.asarray([smp["min_length"], 3, 0], np.int32).tofile(f)
                np.asarray([smp["seed"]], np.uint32).tofile(f)


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


def _smp(temperature=1.0, top_k=0, top_p=1.0, repetition_penalty=1.0, min_length=0, seed=1):
    return dict(temperature=temperature, top_k=top_k, top_p=top_p,
                repetition_penalty=repetition_penalty, min_length=min_length, seed=seed)


@pytest.mark.gpu
def test_batch_generator_sampled_requests(driver, tmp_path, port):
    """Sampled and greedy requests mixed in one continuously admitted batch. Each sampled request
    is replayed alone through the Python API with the same configuration and seed, feeding the
    tokens the C++ run produced: the device must choose the same tokens (its own generator per
    request), and the sampler restatement must agree on them wherever its margin allows."""
    from adai_b200.api import Context, Sampling
    from oracle.pyoracle import sampling_cfg
    w = make_weights(TINY, 4, affine=True)
    srcs = make_sources(TINY, 6, (8, 40), 4)
    cfgs = [_smp(temperature=0.8, top_k=40, seed=11), None,
            _smp(temperature=1.2, top_p=0.9, repetition_penalty=1.3, seed=12),
            _smp(temperature=0.0, repetition_penalty=1.5, min_length=4, seed=13),
            _smp(temperature=1.0, min_length=30, seed=14), _smp(temperature=0.6, seed=15)]
    lens = [16, 10, 24, 12, 30, 20]
    reqs = [(lens[i], srcs[i], cfgs[i]) for i in range(6)]
    path = str(tmp_path / "req.bin")
    _write_requests(path, TINY, w, 3, reqs)
    out = subprocess.run([driver, path], check=True, capture_output=True, text=True,
                         timeout=300).stdout.splitlines()
    got = [[int(t) for t in line.split(":", 1)[1].split()] for line in out]
    model = port.model(TINY, w)
    assert got[1] == _greedy(model, srcs[1], lens[1])
    ctx = Context(0)
    ctx.upload(TINY, w)
    kv = ctx.kv_arena(1, 48, 64)
    checked = total = 0
    for i, c in enumerate(cfgs):
        if c is None:
            continue
        seq = got[i]
        assert seq[0] == 2 and len(seq) >= 2
        stopped = seq[-1] in STOP
        assert len(seq) - 1 == lens[i] or stopped
        assert all(t not in STOP for t in seq[1:-1])
        if stopped:  # min_length keeps EOS / PAD out of the first min_length new tokens
            assert len(seq) - 1 > c["min_length"]
        kv.reset(0)
        kv.encode([0], [srcs[i]])
        kv.set_sampling(0, Sampling.make(**c))
        fcfg, icfg = sampling_cfg(**{k: v for k, v in c.items() if k != "seed"})
        st = port.mt_seed(c["seed"])
        seen = np.zeros(TINY.vocab, np.uint8)
        for s in range(len(seq) - 1):
            nxt, lg = kv.decode_step([0], [seq[s]], want_logits=True)
            assert nxt[0] == seq[s + 1], (i, s)
            seen[seq[s]] = 1
            tok, m = port.sample_next(lg[0], (fcfg, icfg), seen, s, st)
            total += 1
            if m > 1e-6:
                assert tok == seq[s + 1], (i, s, tok, seq[s + 1], m)
                checked += 1
    assert checked >= 0.8 * total, (checked, total)
    kv.close()
    ctx.close()


@pytest.mark.gpu
def test_batched_inference_engine_submit_matches_oracle(driver, tmp_path, port):
    """adai_b200::BatchedInferenceEngine (include/adai_b200_engine.hpp), the reference's
    BatchedInferenceEngine::submit -> std::future<std::string> contract
    (src/BatchedInferenceEngine.hpp:242-272): ten greedy requests submitted from three threads at
    once, collected into batches of at most four and decoded on 3 slots; each future's text is the
    request's greedy ids without special tokens (TextGenerator::generate_text's decode with
    skip_special_tokens), checked against the oracle. A request with decoder seed text fails alone,
    and a submit after shutdown() is refused."""
    w = make_weights(TINY, 17, affine=True, scheme="reference")
    srcs = make_sources(TINY, 9, (4, 48), 17)
    lens = [12, 3, 20, 7, 1, 16, 9, 5, 11]
    reqs = list(zip(lens, srcs))
    reqs.insert(4, (6, [-1]))   # submitted with decoder seed text: refused by the engine
    path = str(tmp_path / "req.bin")
    _write_requests(path, TINY, w, 3, reqs)
    out = subprocess.run([driver, path, "engine"], check=True, capture_output=True, text=True,
                         timeout=300).stdout.splitlines()
    assert len(out) == len(reqs) + 1, out
    model = port.model(TINY, w)
    texts = []
    for i, (max_len, src) in enumerate(reqs):
        head, rest = out[i].split(":", 1)
        assert int(head) == i
        if i == 4:
            assert rest.startswith(" error:") and "decoder seed text" in rest, out[i]
            continue
        want = " ".join(str(t) for t in _greedy(model, src, max_len) if t >= 4)
        assert rest[1:] == want, (i, rest, want)
        texts.append(want)
    assert len(set(texts)) > len(texts) // 2     # the requests do not all decode alike
    assert out[-1].endswith("refused_after_shutdown 1"), out[-1]
    assert "requests 10 " in out[-1], out[-1]
