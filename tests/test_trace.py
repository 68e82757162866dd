"""Debug-sync settings and the work trace, host side (no GPU): the counterpart of the reference's
GPUDebugSync settings (src/gpu/GPUDebugSync.hpp:5-22, parse_gpu_debug_settings)."""
import os
import subprocess
import sys

import pytest

from adai_b200 import api
from tests.conftest import ROOT


@pytest.mark.parametrize("value,want", [
    (None, (0, 1)), ("", (0, 1)), ("off", (0, 1)), ("0", (0, 1)), ("step", (1, 1)),
    ("kernel", (2, 1)), ("kernel:1", (2, 1)), ("kernel:8", (2, 8)), ("kernel:1000000", (2, 1000000)),
])
def test_sync_values(value, want):
    assert api.debug_sync_parse(value) == want


@pytest.mark.parametrize("value", ["kernel:0", "kernel:", "kernel:-3", "kernel:8x", "kernel:1000001",
                                   "Kernel", "steps", "on"])
def test_sync_values_that_cannot_be_read(value):
    with pytest.raises(ValueError, match="ADAI_B200_SYNC"):
        api.debug_sync_parse(value)


def test_configure_round_trip_and_bounds():
    before = api.debug_settings()
    try:
        api.debug_configure(api.SYNC_KERNEL, 4)
        assert api.debug_settings() == (2, 4)
        api.debug_configure(api.SYNC_STEP)
        assert api.debug_settings() == (1, 1)
        with pytest.raises(ValueError):
            api.debug_configure(3)
        with pytest.raises(ValueError):
            api.debug_configure(api.SYNC_KERNEL, 0)
        assert api.debug_settings() == (1, 1)  # a rejected call changes nothing
    finally:
        api.debug_configure(*before)


def _settings_in_child(env):
    code = "from adai_b200 import api; print(*api.debug_settings())"
    full = {k: v for k, v in os.environ.items()
            if k not in ("ADAI_B200_SYNC", "ADAI_GPU_SYNC", "ADAI_B200_TRACE_FILE",
                         "ADAI_GPU_TRACE_FILE")}
    full.update(env)
    r = subprocess.run([sys.executable, "-c", code], cwd=ROOT, env=full, capture_output=True,
                       text=True, timeout=120, check=True)
    return tuple(int(v) for v in r.stdout.split()), r.stderr


def test_settings_come_from_the_environment_once():
    assert _settings_in_child({"ADAI_B200_SYNC": "kernel:16"})[0] == (2, 16)
    # the reference's own variable is honoured when the library's is unset
    assert _settings_in_child({"ADAI_GPU_SYNC": "step"})[0] == (1, 1)
    assert _settings_in_child({"ADAI_B200_SYNC": "off", "ADAI_GPU_SYNC": "step"})[0] == (0, 1)
    got, err = _settings_in_child({"ADAI_B200_SYNC": "everything"})
    assert got == (0, 1) and "debug sync stays off" in err


def test_last_work_needs_a_context():
    with pytest.raises(ValueError):
        api.check(api.load().adai_b200_ctx_last_work(None, None, 0, None))
