"""adai_b200_decode_attention_static, the decode-attention entry point that allocates nothing (its
split-KV scratch is a fixed per-device array in the library's device image), against the
allocating adai_b200_decode_attention on the same inputs, several calls in a row (each call
reuses the merge counters the previous one handed back), against the oracle's per-head attention
directly, its size limit, and a call whose cached length exceeds max_len (refused by the kernel,
after which the next call still matches).

Tolerance: |static - allocating| <= 1e-5 + 1e-4 |allocating| elementwise, the decode-path bound;
the appended cache rows must be identical.
"""
import numpy as np
import pytest

from tests.conftest import tol_ok

pytestmark = pytest.mark.gpu


def _inputs(torch, seed, B, H, dh, cap, lens, append):
    g = torch.Generator(device="cuda").manual_seed(seed)
    D = H * dh
    kc = torch.randn((B, H, cap, dh), generator=g, device="cuda")
    vc = torch.randn((B, H, cap, dh), generator=g, device="cuda")
    q = torch.randn((B, D), generator=g, device="cuda")
    kn = torch.randn((B, D), generator=g, device="cuda") if append else None
    vn = torch.randn((B, D), generator=g, device="cuda") if append else None
    dl = torch.from_numpy(np.asarray(lens, np.int32)).cuda()
    return kc, vc, q, kn, vn, dl


def _run(fn, torch, B, H, dh, cap, kc, vc, q, kn, vn, dl, max_len):
    kc, vc = kc.clone(), vc.clone()
    out = torch.empty((B, H * dh), device="cuda")
    ptr = (lambda t: None if t is None else t.data_ptr())
    fn(B, H, cap, q.data_ptr(), ptr(kn), ptr(vn), kc.data_ptr(), vc.data_ptr(), dl.data_ptr(),
       max_len, out.data_ptr(), head_dim=dh)
    return out, kc, vc


@pytest.mark.parametrize("calls", [[(64, True, 21), (64, True, 22), (64, False, 23), (32, True, 24)]])
def test_static_scratch_matches_allocating_entry_point(ctx, torch_cuda, calls):
    torch = torch_cuda
    B, H, cap = 6, 4, 1100
    for dh, append, seed in calls:
        # lengths on both sides of the 256-row split boundary: single-chunk and merged sequences
        lens = [0, 1, 255, 256, 700, 1098][:B]
        max_len = max(lens)
        kc, vc, q, kn, vn, dl = _inputs(torch, seed, B, H, dh, cap, lens, append)
        torch.cuda.synchronize()
        want, kc_a, vc_a = _run(ctx.decode_attention, torch, B, H, dh, cap, kc, vc, q, kn, vn, dl,
                                max_len)
        got, kc_b, vc_b = _run(ctx.decode_attention_static, torch, B, H, dh, cap, kc, vc, q, kn,
                               vn, dl, max_len)
        ctx.synchronize()
        torch.cuda.synchronize()
        assert tol_ok(got.cpu().numpy(), want.cpu().numpy()), (dh, append, seed)
        assert torch.equal(kc_a, kc_b) and torch.equal(vc_a, vc_b)


def test_static_scratch_matches_oracle(ctx, torch_cuda, port):
    # The reference's per-head cached attention (src/MultiHeadAttention.cpp:336-367), restated by
    # the oracle, on each sequence's appended cache.
    torch = torch_cuda
    B, H, dh, cap = 4, 4, 64, 700
    lens = [0, 255, 256, 600]
    kc, vc, q, kn, vn, dl = _inputs(torch, 31, B, H, dh, cap, lens, True)
    torch.cuda.synchronize()
    got, kc_b, vc_b = _run(ctx.decode_attention_static, torch, B, H, dh, cap, kc, vc, q, kn, vn,
                           dl, max(lens))
    ctx.synchronize()
    got = got.cpu().numpy()
    kc_h, vc_h, q_h = kc_b.cpu().numpy(), vc_b.cpu().numpy(), q.cpu().numpy()
    for b in range(B):
        t = lens[b] + 1
        K = kc_h[b, :, :t, :].transpose(1, 0, 2).reshape(t, H * dh)
        V = vc_h[b, :, :t, :].transpose(1, 0, 2).reshape(t, H * dh)
        assert tol_ok(got[b], port.attention_single(q_h[b], K, V, H)), b


def test_static_scratch_refuses_a_length_past_max_len(ctx, torch_cuda):
    # lens[2] = 900 > max_len = 600: the kernel refuses that pair before any load, append or merge
    # counter and the synchronize reports it; the counters stay at zero, so the next call on the
    # shared array matches the allocating entry point.
    torch = torch_cuda
    B, H, dh, cap = 4, 4, 64, 1024
    bad = [10, 300, 900, 600]
    kc, vc, q, kn, vn, dl = _inputs(torch, 41, B, H, dh, cap, bad, True)
    torch.cuda.synchronize()
    with pytest.raises(IndexError, match="code 111"):
        _run(ctx.decode_attention_static, torch, B, H, dh, cap, kc, vc, q, kn, vn, dl, 600)
        ctx.synchronize()
    good = [10, 300, 599, 600]
    kc, vc, q, kn, vn, dl = _inputs(torch, 42, B, H, dh, cap, good, True)
    torch.cuda.synchronize()
    want, _, _ = _run(ctx.decode_attention, torch, B, H, dh, cap, kc, vc, q, kn, vn, dl, 600)
    got, _, _ = _run(ctx.decode_attention_static, torch, B, H, dh, cap, kc, vc, q, kn, vn, dl, 600)
    ctx.synchronize()
    torch.cuda.synchronize()
    assert tol_ok(got.cpu().numpy(), want.cpu().numpy())


def test_static_scratch_rejects_oversized_calls(ctx, torch_cuda):
    torch = torch_cuda
    B, H, dh, cap = 3277, 5, 64, 2          # B * H = 16385, one more (sequence, head) than fits
    kc, vc, q, kn, vn, dl = _inputs(torch, 5, B, H, dh, cap, [0] * B, True)
    out = torch.empty((B, H * dh), device="cuda")
    torch.cuda.synchronize()
    with pytest.raises(IndexError, match="static attention scratch too small"):
        ctx.decode_attention_static(B, H, cap, q.data_ptr(), kn.data_ptr(), vn.data_ptr(),
                                    kc.data_ptr(), vc.data_ptr(), dl.data_ptr(), 0,
                                    out.data_ptr(), head_dim=dh)
    ctx.synchronize()
