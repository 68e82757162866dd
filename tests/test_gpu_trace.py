"""The work trace on the device path: every launch is named, ADAI_B200_SYNC=kernel runs the decode
step kernel by kernel (no graph) with the same results, and a failed wait names the last work
(GPUDebugSync's last-kernel tag, src/gpu/GPUDebugSync.cpp:246-253)."""
import numpy as np
import pytest

from adai_b200 import api
from adai_b200.api import Context
from adai_b200.config import TINY
from adai_b200.synth import make_sources, make_weights

pytestmark = pytest.mark.gpu

BOS = 2


@pytest.fixture
def restore_settings():
    before = api.debug_settings()
    yield
    api.debug_configure(*before)


def _generate(c, srcs, steps):
    kv = c.kv_arena(len(srcs), steps + 1, 64)
    slots = list(range(len(srcs)))
    kv.encode(slots, srcs)
    ids = kv.generate(slots, [BOS] * len(srcs), steps)
    kv.close()
    return ids


def test_kernel_sync_names_every_launch_and_matches_the_graph(restore_settings, tmp_path):
    srcs = make_sources(TINY, 3, (9, 40), 5)
    steps = 4
    with Context(0) as c:
        c.upload(TINY, make_weights(TINY, 0, scheme="reference"))
        api.debug_configure(api.SYNC_OFF)
        want = _generate(c, srcs, steps)
        work, n_graph = c.last_work()
        assert work.endswith("adai_b200_generate decode step (CUDA graph)"), work
        trace = tmp_path / "trace.txt"
        api.debug_configure(api.SYNC_KERNEL, 1, str(trace))
        got = _generate(c, srcs, steps)
        work, n = c.last_work()
        api.debug_configure(api.SYNC_OFF)
    np.testing.assert_array_equal(got, want)
    assert work.endswith("adai_b200_generate record_and_advance_kernel"), work
    assert trace.read_text() == work + "\n"
    # one step: embedding, per layer 6 GEMMs + 2 attention launches, LM head, advance
    per_step = 1 + 8 * TINY.dec_layers + 1 + 1
    assert n - n_graph >= steps * per_step, (n, n_graph)


def test_step_sync_on_an_op_entry(restore_settings, torch_cuda):
    torch = torch_cuda
    api.debug_configure(api.SYNC_STEP)
    with Context(0) as c:
        a = torch.randn(64, 96, device="cuda")
        b = torch.randn(96, 80, device="cuda")
        out = torch.empty(64, 80, device="cuda")
        api.check(c.lib.adai_b200_sgemm(c.h, 64, 80, 96, a.data_ptr(), b.data_ptr(),
                                        out.data_ptr()))
        work, _ = c.last_work()
        ref = (a.double() @ b.double()).float()
    assert " adai_b200_sgemm gemm_3xtf32_kernel" in work, work
    assert torch.allclose(out, ref, rtol=1e-4, atol=1e-4)


def test_a_failed_wait_names_the_last_work():
    # The bounded device wait of adai_b200_ctx_check_wait_timeout gives up after 2 s (no fault);
    # the timeout message carries the last work queued.
    c = Context(0)
    c.check_wait_timeout()
    msg = api.load().adai_b200_last_error().decode()
    assert "last GPU work queued" in msg and "wait_selftest_kernel" in msg, msg
    assert "adai_b200_ctx_check_wait_timeout" in msg, msg
    c.close()
