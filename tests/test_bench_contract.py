"""bench.py's command-line contract on the CPU: the reference arm's JSON line (the reference CPU
path timed on the host cores, on the tiny encoder-decoder workload so it ends in seconds) and the
sampling option parser."""
import json
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import bench  # noqa: E402


def test_parse_sampling():
    assert bench.parse_sampling("") == {}
    got = bench.parse_sampling("temperature=0.8, top_k=50,top_p=0.95,repetition_penalty=1.1,min_length=3")
    assert got == {"temperature": 0.8, "top_k": 50, "top_p": 0.95, "repetition_penalty": 1.1,
                   "min_length": 3}
    assert isinstance(got["top_k"], int) and isinstance(got["min_length"], int)


def test_reference_arm_json_line():
    env = dict(os.environ, OMP_NUM_THREADS="2")
    r = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference",
                        "--workload", "tiny-encdec-b8-s64-t32", "--steps", "3", "--warmup", "1"],
                       capture_output=True, text=True, timeout=600, cwd=ROOT, env=env)
    assert r.returncode == 0, r.stderr[-2000:]
    line = json.loads(r.stdout.strip().splitlines()[-1])
    if "unavailable" in line:
        pytest.skip(line["unavailable"])
    assert line["impl"] == "reference"
    for k in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step",
              "higher_is_better", "scaling", "vs_baseline", "dtype", "data", "config",
              "cpu_baseline", "e2e"):
        assert k in line, k
    assert line["value"] > 0 and line["unit"] == "tokens/s" and line["higher_is_better"] is True
    assert line["metric"] == "batched greedy decode tokens/s (tiny-encdec-b8-s64-t32, fp32)"
    assert bench.metric_for(bench.WORKLOADS[bench.DEFAULT_WORKLOAD]) == bench.METRIC
    cb = line["cpu_baseline"]
    assert cb["kind"] in ("reference", "port") and cb["cores"] >= 1 and cb["value"] == line["value"]
    e2e = line["e2e"]
    assert e2e["value"] == line["value"] and e2e["h2d_bytes_per_step"] == 0
    assert e2e["d2h_bytes_per_step"] == 0
    assert line["config"]["workload"] == "tiny-encdec-b8-s64-t32"

