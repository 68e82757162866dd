"""GPU op parity through the C ABI: 3xTF32 tcgen05 GEMM, decode attention with the fused KV
append, LayerNorm — each against the CPU oracle (oracle/adai_oracle.c) on the same seeded inputs.

Tolerances: GEMM elements within 1e-5 + 1e-5 * sum_k |a_ik b_kj| of the float64 product (the
bound of the reference's tests/matrix_simd_test.cpp:290-319) and of the oracle; attention and
LayerNorm within |gpu - oracle| <= 1e-5 + 1e-4 |oracle| (the decode-path parity bound).
"""
import numpy as np
import pytest

from adai_b200.config import ATTN_OP, GEMM_SWEEP_KN, GEMM_SWEEP_M
from tests.conftest import tol_ok, tol_ratio
from tests.golden.make_golden import GEMM_SHAPES, gemm_inputs

pytestmark = pytest.mark.gpu


def dev(torch, a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def gemm_gpu(ctx, torch, A, B):
    M, K = A.shape
    N = B.shape[1]
    dA, dB = dev(torch, A), dev(torch, B)
    dC = torch.empty((M, N), dtype=torch.float32, device="cuda")
    torch.cuda.synchronize()
    ctx.sgemm(M, N, K, dA.data_ptr(), dB.data_ptr(), dC.data_ptr())
    ctx.synchronize()
    return dC.cpu().numpy()


def gemm_bound(A, B):
    return 1e-5 + 1e-5 * (np.abs(A).astype(np.float64) @ np.abs(B).astype(np.float64))


@pytest.mark.parametrize("i", range(len(GEMM_SHAPES)))
def test_gemm_simd_test_shapes(ctx, torch_cuda, port, golden, i):
    M, K, N = GEMM_SHAPES[i]
    A, B = gemm_inputs(i, M, K, N)
    got = gemm_gpu(ctx, torch_cuda, A, B)
    exact = A.astype(np.float64) @ B.astype(np.float64)
    bound = gemm_bound(A, B)
    assert np.all(np.abs(got - exact) <= bound)
    assert np.all(np.abs(got - golden[f"gemm_{i}"]) <= 2 * bound)


@pytest.mark.parametrize("M", [64, 256])
@pytest.mark.parametrize("KN", GEMM_SWEEP_KN)
def test_gemm_sweep_shapes_vs_oracle(ctx, torch_cuda, port, M, KN):
    K, N = KN
    rng = np.random.default_rng(M * 7 + K + N)
    A = rng.standard_normal((M, K)).astype(np.float32)
    B = rng.standard_normal((K, N)).astype(np.float32)
    got = gemm_gpu(ctx, torch_cuda, A, B)
    assert np.all(np.abs(got - port.matmul(A, B)) <= 2 * gemm_bound(A, B))


@pytest.mark.parametrize("M", GEMM_SWEEP_M)
@pytest.mark.parametrize("KN", GEMM_SWEEP_KN)
def test_gemm_full_sweep_sampled_rows(ctx, torch_cuda, M, KN):
    # Full-size sweep: every element is computed on the GPU; 48 rows are checked in float64.
    K, N = KN
    torch = torch_cuda
    g = torch.Generator(device="cuda").manual_seed(M + K * 3 + N)
    dA = torch.randn((M, K), generator=g, device="cuda", dtype=torch.float32)
    dB = torch.randn((K, N), generator=g, device="cuda", dtype=torch.float32)
    dC = torch.empty((M, N), dtype=torch.float32, device="cuda")
    torch.cuda.synchronize()
    ctx.sgemm(M, N, K, dA.data_ptr(), dB.data_ptr(), dC.data_ptr())
    ctx.synchronize()
    rows = np.unique(np.random.default_rng(M).integers(0, M, 48))
    A = dA[rows].cpu().numpy()
    B = dB.cpu().numpy()
    exact = A.astype(np.float64) @ B.astype(np.float64)
    got = dC[rows].cpu().numpy()
    assert np.all(np.abs(got - exact) <= gemm_bound(A, B))
    assert np.isfinite(dC.sum().item())


def test_gemm_is_deterministic_and_prepared_weight_matches(ctx, torch_cuda):
    torch = torch_cuda
    rng = np.random.default_rng(5)
    A = rng.standard_normal((128, 4096)).astype(np.float32)
    B = rng.standard_normal((4096, 1024)).astype(np.float32)   # split-K shape at M=128
    first = gemm_gpu(ctx, torch, A, B)
    second = gemm_gpu(ctx, torch, A, B)
    np.testing.assert_array_equal(first, second)
    dA, dB = dev(torch, A), dev(torch, B)
    dC = torch.empty((128, 1024), dtype=torch.float32, device="cuda")
    torch.cuda.synchronize()
    w = ctx.weight(dB.data_ptr(), 4096, 1024)
    w.matmul(128, dA.data_ptr(), dC.data_ptr())
    ctx.synchronize()
    np.testing.assert_array_equal(dC.cpu().numpy(), first)
    w.close()


def test_gemm_odd_inner_dimension(ctx, torch_cuda):
    rng = np.random.default_rng(11)
    A = rng.standard_normal((33, 101)).astype(np.float32)
    B = rng.standard_normal((101, 70)).astype(np.float32)
    got = gemm_gpu(ctx, torch_cuda, A, B)
    exact = A.astype(np.float64) @ B.astype(np.float64)
    assert np.all(np.abs(got - exact) <= gemm_bound(A, B))


@pytest.mark.parametrize("m,n,k,lda,off", [(64, 1536, 512, 512, 0), (200, 96, 70, 72, 0),
                                           (1, 33, 5, 8, 0), (256, 128, 1024, 1028, 0),
                                           (64, 96, 40, 44, 1), (257, 64, 64, 64, 0)])
def test_gemm_split_inside_the_gemm_matches_the_split_kernel(ctx, torch_cuda, m, n, k, lda, off):
    # Up to 256 rows of untransposed, unscaled A with 16-byte aligned rows are split into tf32 hi
    # and lo inside the GEMM (TMA brings the fp32 box, converter warps split it); a transposed A
    # takes the separate split kernel. Both must give the same bits: the same split, the same
    # products. Covered: rows past M, columns past K (K not a multiple of 32), and an A that the
    # inside split does not take (a base 4 bytes off 16-byte alignment, more than 256 rows).
    torch = torch_cuda
    g = torch.Generator(device="cuda").manual_seed(m * 7 + k)
    buf = torch.randn(m * lda + 4, device="cuda", generator=g)
    A = buf[off:off + m * lda].view(m, lda)
    B = torch.randn(k, n, device="cuda", generator=g)
    C1 = torch.empty(m, n, device="cuda")
    C2 = torch.empty(m, n, device="cuda")
    ctx.gemm_strided(0, 0, m, n, k, 1.0, A.data_ptr(), lda, B.data_ptr(), n, C1.data_ptr(), n)
    At = A[:, :k].t().contiguous()  # [k, m]
    ctx.gemm_strided(1, 0, m, n, k, 1.0, At.data_ptr(), m, B.data_ptr(), n, C2.data_ptr(), n)
    torch.cuda.synchronize()
    assert torch.equal(C1, C2)
    a64, b64 = A[:, :k].double().cpu().numpy(), B.double().cpu().numpy()
    bound = 1e-5 + 1e-5 * (np.abs(a64) @ np.abs(b64))
    assert np.all(np.abs(C1.double().cpu().numpy() - a64 @ b64) <= bound)


@pytest.mark.parametrize("m", [64, 300])
@pytest.mark.parametrize("n,k,plan", [
    (96, 224, "96:224:32:1:4:2"),      # 7 K blocks (odd) over 4 stages, 2-block chunks
    (128, 470, "128:470:64:2:4:4"),    # 2-way split-K, 8 + 7 K blocks, ragged last K block
    (64, 1024, "64:1024:32:1:4:8"),    # 32 K blocks: every stage refilled 7 times
])
def test_gemm_forced_pipeline_plans(ctx, torch_cuda, monkeypatch, m, n, k, plan):
    # Plans with four stages, where the MMA issuers free the stages two at a time, forced through
    # ADAI_B200_GEMM_PLANS (read at each call): odd K-block counts per split leave an even last
    # block with no commit of its own. 64 rows take the in-GEMM split of an fp32 A (converter
    # warps), 300 rows the separate split kernel.
    monkeypatch.setenv("ADAI_B200_GEMM_PLANS", plan)
    rng = np.random.default_rng(m + n + k)
    A = rng.standard_normal((m, k)).astype(np.float32)
    B = rng.standard_normal((k, n)).astype(np.float32)
    got = gemm_gpu(ctx, torch_cuda, A, B)
    exact = A.astype(np.float64) @ B.astype(np.float64)
    assert np.all(np.abs(got - exact) <= gemm_bound(A, B))


# ---------------------------------------------------------------------------------------------
def attention_case(ctx, torch, port, lens, H, cap, append, seed, dh=64):
    rng = np.random.default_rng(seed)
    B = len(lens)
    D = H * dh
    kc = rng.standard_normal((B, H, cap, dh)).astype(np.float32)
    vc = rng.standard_normal((B, H, cap, dh)).astype(np.float32)
    q = rng.standard_normal((B, D)).astype(np.float32)
    kn = rng.standard_normal((B, D)).astype(np.float32)
    vn = rng.standard_normal((B, D)).astype(np.float32)
    lens = np.asarray(lens, np.int32)
    d = {k: dev(torch, v) for k, v in dict(kc=kc, vc=vc, q=q, kn=kn, vn=vn, lens=lens).items()}
    out = torch.empty((B, D), dtype=torch.float32, device="cuda")
    torch.cuda.synchronize()
    ctx.decode_attention(B, H, cap, d["q"].data_ptr(),
                         d["kn"].data_ptr() if append else None,
                         d["vn"].data_ptr() if append else None,
                         d["kc"].data_ptr(), d["vc"].data_ptr(), d["lens"].data_ptr(),
                         int(lens.max()), out.data_ptr(), head_dim=dh)
    ctx.synchronize()
    got = out.cpu().numpy()
    kc_after = d["kc"].cpu().numpy()
    worst = 0.0
    for b in range(B):
        L = int(lens[b])
        K = kc[b].transpose(1, 0, 2)[:L].reshape(L, D)   # [T, H*64] row-major like the reference
        V = vc[b].transpose(1, 0, 2)[:L].reshape(L, D)
        if append:
            K = np.vstack([K, kn[b][None]])
            V = np.vstack([V, vn[b][None]])
            np.testing.assert_array_equal(kc_after[b, :, L, :], kn[b].reshape(H, dh))
        want = port.attention_single(q[b], K, V, H)
        worst = max(worst, tol_ratio(got[b], want))
    return worst


@pytest.mark.parametrize("dh", [32, 64])
@pytest.mark.parametrize("append", [False, True])
def test_decode_attention_ragged_lengths(ctx, torch_cuda, port, append, dh):
    lens = [1, 7, 255, 256, 257, 600, 1023] if not append else [0, 6, 255, 256, 511, 900, 1022]
    r = attention_case(ctx, torch_cuda, port, lens, H=4, cap=1024, append=append, seed=3, dh=dh)
    assert r <= 1.0, r


def test_decode_attention_kv_op_workload(ctx, torch_cuda, port):
    # The KV-attention op workload (batch 256, 16 heads, capacity 2048, lengths U[256, 2048]) at
    # full size on the GPU; 12 sequences are checked against the oracle.
    torch = torch_cuda
    cfg = ATTN_OP
    B, H, cap = cfg["batch"], cfg["heads"], cfg["capacity"]
    D = H * 64
    rng = np.random.default_rng(42)
    lens = rng.integers(cfg["len_lo"], cfg["len_hi"], size=B).astype(np.int32)  # room to append
    g = torch.Generator(device="cuda").manual_seed(42)
    kc = torch.randn((B, H, cap, 64), generator=g, device="cuda")
    vc = torch.randn((B, H, cap, 64), generator=g, device="cuda")
    q = torch.randn((B, D), generator=g, device="cuda")
    kn = torch.randn((B, D), generator=g, device="cuda")
    vn = torch.randn((B, D), generator=g, device="cuda")
    dl = torch.from_numpy(lens).cuda()
    out = torch.empty((B, D), device="cuda")
    check = np.unique(np.concatenate([np.argsort(lens)[[0, 1, -1, -2]],
                                      rng.integers(0, B, 8)]))
    before = {int(b): (kc[b].cpu().numpy(), vc[b].cpu().numpy()) for b in check}
    torch.cuda.synchronize()
    ctx.decode_attention(B, H, cap, q.data_ptr(), kn.data_ptr(), vn.data_ptr(), kc.data_ptr(),
                         vc.data_ptr(), dl.data_ptr(), int(lens.max()), out.data_ptr())
    ctx.synchronize()
    got = out.cpu().numpy()
    qn, knn, vnn = q.cpu().numpy(), kn.cpu().numpy(), vn.cpu().numpy()
    for b in check:
        L = int(lens[b])
        K = np.vstack([before[b][0].transpose(1, 0, 2)[:L].reshape(L, D), knn[b][None]])
        V = np.vstack([before[b][1].transpose(1, 0, 2)[:L].reshape(L, D), vnn[b][None]])
        r = tol_ratio(got[b], port.attention_single(qn[b], K, V, H))
        assert r <= 1.0, (b, L, r)


def test_layernorm_op(ctx, torch_cuda, port):
    torch = torch_cuda
    rng = np.random.default_rng(8)
    for D in (128, 512, 1024):
        x = (rng.standard_normal((37, D)) * 2 + 0.5).astype(np.float32)
        g = rng.uniform(0.5, 1.5, D).astype(np.float32)
        b = rng.uniform(-0.2, 0.2, D).astype(np.float32)
        dx, dg, db = dev(torch, x), dev(torch, g), dev(torch, b)
        out = torch.empty_like(dx)
        torch.cuda.synchronize()
        ctx.layernorm(dx.data_ptr(), dg.data_ptr(), db.data_ptr(), out.data_ptr(), 37, D)
        ctx.synchronize()
        assert tol_ok(out.cpu().numpy(), port.layernorm(x, g, b))
