"""The decode-path entries of the reference backend table (adai::gpu::matrix_*_gpu,
src/gpu/MatrixGPU.hpp:43-201) through the C ABI, against the CPU oracle / numpy on the same inputs,
and the same functions through their C++ reference signatures (include/adai_b200_backend.hpp).

Tolerances: GEMM elements within 1e-5 + 1e-5 sum_k |alpha a b| of the oracle (the bound of the
reference's tests/matrix_simd_test.cpp:290-319); softmax / LayerNorm / GELU within
1e-5 + 1e-4 |oracle| (the decode-path bound); sigmoid and tanh within 4 ulp of float64; bias add,
ReLU and the embedding gather exact.
"""
import os
import shutil
import subprocess

import numpy as np
import pytest

from tests.conftest import ROOT, tol_ok

pytestmark = pytest.mark.gpu


def dev(torch, a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


@pytest.mark.parametrize("trans_a,trans_b", [(0, 0), (1, 0), (0, 1), (1, 1)])
def test_gemm_strided_views_and_transposes(ctx, torch_cuda, port, trans_a, trans_b):
    torch = torch_cuda
    rng = np.random.default_rng(31 + 2 * trans_a + trans_b)
    m, n, k, alpha = 37, 70, 129, 0.125
    A = rng.standard_normal((k, m) if trans_a else (m, k)).astype(np.float32)
    B = rng.standard_normal((n, k) if trans_b else (k, n)).astype(np.float32)
    # views into wider matrices: 5 extra columns on every operand, C starts one float in (unaligned)
    Aw = np.zeros((A.shape[0], A.shape[1] + 5), np.float32)
    Aw[:, 3:3 + A.shape[1]] = A
    Bw = np.zeros((B.shape[0], B.shape[1] + 5), np.float32)
    Bw[:, 2:2 + B.shape[1]] = B
    dA, dB = dev(torch, Aw), dev(torch, Bw)
    dC = torch.full((m, n + 7), 7.0, device="cuda")
    torch.cuda.synchronize()
    ctx.gemm_strided(trans_a, trans_b, m, n, k, alpha, dA.data_ptr() + 12, Aw.shape[1],
                     dB.data_ptr() + 8, Bw.shape[1], dC.data_ptr() + 4, n + 7)
    ctx.synchronize()
    got = dC.cpu().numpy()
    opA = A.T if trans_a else A
    opB = B.T if trans_b else B
    want = port.matmul(np.ascontiguousarray(alpha * opA), np.ascontiguousarray(opB))
    bound = 1e-5 + 1e-5 * (np.abs(alpha * opA).astype(np.float64) @ np.abs(opB).astype(np.float64))
    assert np.all(np.abs(got[:, 1:1 + n] - want) <= bound)
    assert np.all(got[:, 0] == 7.0) and np.all(got[:, 1 + n:] == 7.0)   # nothing outside C


def test_gemm_strided_empty_inner_dimension_zeroes_c(ctx, torch_cuda):
    torch = torch_cuda
    dC = torch.full((4, 8), 3.0, device="cuda")
    torch.cuda.synchronize()
    ctx.gemm_strided(0, 0, 4, 6, 0, 1.0, 0, 1, 0, 6, dC.data_ptr(), 8)
    ctx.synchronize()
    got = dC.cpu().numpy()
    assert np.all(got[:, :6] == 0) and np.all(got[:, 6:] == 3.0)


def test_softmax_rows_follows_the_cpu_definition(ctx, torch_cuda, port):
    torch = torch_cuda
    rng = np.random.default_rng(5)
    x = (rng.standard_normal((9, 1000)) * 4).astype(np.float32)
    x[3, :] = -np.inf
    x[3, 17] = 2.0                      # one finite entry: probability 1 there
    x[4, :5] = 80.0                     # large values: the maximum is subtracted first
    d = dev(torch, x)
    torch.cuda.synchronize()
    ctx.softmax_rows(d.data_ptr(), 9, 1000)
    ctx.synchronize()
    assert tol_ok(d.cpu().numpy(), port.softmax_rows(x))


@pytest.mark.parametrize("cols", [300, 1024, 4097])
def test_layernorm_fwd_any_width_with_statistics(ctx, torch_cuda, port, cols):
    torch = torch_cuda
    rng = np.random.default_rng(cols)
    x = (rng.standard_normal((11, cols)) * 3 + 1.5).astype(np.float32)
    g = rng.uniform(0.5, 1.5, cols).astype(np.float32)
    b = rng.uniform(-0.3, 0.3, cols).astype(np.float32)
    dx, dg, db = dev(torch, x), dev(torch, g), dev(torch, b)
    y, xn = torch.empty_like(dx), torch.empty_like(dx)
    mean, rstd = torch.empty(11, device="cuda"), torch.empty(11, device="cuda")
    torch.cuda.synchronize()
    ctx.layernorm_fwd(dx.data_ptr(), y.data_ptr(), xn.data_ptr(), dg.data_ptr(), db.data_ptr(),
                      mean.data_ptr(), rstd.data_ptr(), 11, cols, 1e-5)
    ctx.synchronize()
    assert tol_ok(y.cpu().numpy(), port.layernorm(x, g, b))
    x64 = x.astype(np.float64)
    mu = x64.mean(axis=1)
    rs = 1.0 / np.sqrt(((x64 - mu[:, None]) ** 2).mean(axis=1) + 1e-5)
    assert tol_ok(mean.cpu().numpy(), mu) and tol_ok(rstd.cpu().numpy(), rs)
    assert tol_ok(xn.cpu().numpy(), (x64 - mu[:, None]) * rs[:, None])


def test_add_row_bias_and_activations(ctx, torch_cuda, port):
    torch = torch_cuda
    rng = np.random.default_rng(9)
    m = (rng.standard_normal((13, 77)) * 3).astype(np.float32)
    bias = rng.standard_normal(77).astype(np.float32)
    dm, dbias = dev(torch, m), dev(torch, bias)
    out = torch.empty_like(dm)
    torch.cuda.synchronize()
    ctx.add_row_bias(dm.data_ptr(), dbias.data_ptr(), out.data_ptr(), 13, 77)
    ctx.synchronize()
    np.testing.assert_array_equal(out.cpu().numpy(), m + bias)
    x = (rng.standard_normal(4099) * 4).astype(np.float32)
    x64 = x.astype(np.float64)
    for kind in range(4):
        d = dev(torch, x)
        torch.cuda.synchronize()
        ctx.activation(d.data_ptr(), x.size, kind)
        ctx.synchronize()
        got = d.cpu().numpy()
        if kind == 0:
            np.testing.assert_array_equal(got, np.maximum(x, 0))
        elif kind == 3:
            assert tol_ok(got, port.gelu(x))
        else:
            want = 1 / (1 + np.exp(-x64)) if kind == 1 else np.tanh(x64)
            assert np.all(np.abs(got - want) <= 4 * np.spacing(np.abs(want).astype(np.float32)) + 1e-30)


def test_embedding_gather_add_pe(ctx, torch_cuda):
    torch = torch_cuda
    rng = np.random.default_rng(4)
    V, d, pe_rows = 50, 96, 6
    table = rng.standard_normal((V, d)).astype(np.float32)
    pe = rng.standard_normal((pe_rows, d)).astype(np.float32)
    ids = np.array([3, 0, 49, 7, 7, 12, 1, 2], np.int32)
    dt, dp, di = dev(torch, table), dev(torch, pe), dev(torch, ids)
    for pos_offset, use_pe in [(0, True), (3, True), (0, False)]:
        out = torch.empty((8, d), device="cuda")
        torch.cuda.synchronize()
        ctx.embedding_gather_add_pe(dt.data_ptr(), di.data_ptr(), dp.data_ptr() if use_pe else None,
                                    pe_rows, pos_offset, out.data_ptr(), 8, d, V)
        ctx.synchronize()
        want = table[ids].copy()
        if use_pe:
            for i in range(8):
                if pos_offset + i < pe_rows:
                    want[i] += pe[pos_offset + i]
        np.testing.assert_array_equal(out.cpu().numpy(), want)
    bad = dev(torch, np.array([1, V], np.int32))
    out = torch.empty((2, d), device="cuda")
    torch.cuda.synchronize()
    ctx.embedding_gather_add_pe(dt.data_ptr(), bad.data_ptr(), None, 0, 0, out.data_ptr(), 2, d, V)
    with pytest.raises(IndexError):      # TokenEmbedding::forward throws std::out_of_range
        ctx.synchronize()


def test_reference_signatures_link_and_run(tmp_path):
    gxx = shutil.which("g++")
    if gxx is None:
        pytest.skip("no C++ compiler")
    cuda = "/usr/local/cuda"
    exe = str(tmp_path / "backend_table")
    lib = os.path.join(ROOT, "adai_b200")
    subprocess.run([gxx, "-std=c++17", "-O1", "-Wall", "-Werror", "-I" + os.path.join(ROOT, "include"),
                    "-I" + cuda + "/include", os.path.join(ROOT, "tests", "cpp", "backend_table.cpp"),
                    "-L" + lib, "-ladai_b200", "-Wl,-rpath," + lib, "-L" + cuda + "/lib64", "-lcudart",
                    "-o", exe], check=True)
    r = subprocess.run([exe], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "all ok" in r.stdout, r.stdout


def test_program_built_against_the_reference_header_runs():
    # oracle/_ref/backend_table_refhdr: the same program compiled against the reference's own
    # src/gpu/MatrixGPU.hpp (oracle/Makefile, target `boundary`, built where the reference sources
    # are; it travels with the built library). Its calls resolve to libadai_b200.so.
    exe = os.path.join(ROOT, "oracle", "_ref", "backend_table_refhdr")
    if not os.path.exists(exe):
        pytest.skip("built only where the reference sources are (make -C oracle boundary)")
    r = subprocess.run([exe], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "all ok" in r.stdout, r.stdout


def test_softmax_known_answers(ctx, torch_cuda):
    # tests/matrixgpu_td003_test.cpp:234-249: [0, 0] -> [0.5, 0.5]; [0, ln 3] -> [0.25, 0.75]
    torch = torch_cuda
    d = dev(torch, np.array([[0.0, 0.0], [0.0, np.log(3.0)]], np.float32))
    torch.cuda.synchronize()
    ctx.softmax_rows(d.data_ptr(), 2, 2)
    ctx.synchronize()
    got = d.cpu().numpy()
    assert abs(got[0, 0] - 0.5) <= 1e-4 and abs(got[0, 1] - 0.5) <= 1e-4
    assert abs(got[1, 0] - 0.25) <= 1e-3 and abs(got[1, 1] - 0.75) <= 1e-3


def test_strided_gemm_known_answers(ctx, torch_cuda):
    # tests/matrixgpu_td003_test.cpp:396-446: sin / cos operands viewed inside wider rows, every
    # transpose combination, against a float64 host product within 1e-4; columns outside the
    # output view keep their value.
    torch = torch_cuda
    m, n, k, a_off, b_off, c_off, alpha = 3, 5, 4, 2, 1, 3, 0.75
    for trans_a in (False, True):
        for trans_b in (False, True):
            a_rows, a_cols = (k, m) if trans_a else (m, k)
            b_rows, b_cols = (n, k) if trans_b else (k, n)
            lda, ldb, ldc = a_cols + 4, b_cols + 3, n + 6
            a = np.sin(0.37 * np.arange(a_rows * lda, dtype=np.float32)).astype(np.float32)
            b = np.cos(0.23 * np.arange(b_rows * ldb, dtype=np.float32)).astype(np.float32)
            da, db = dev(torch, a), dev(torch, b)
            dc = torch.full((m * ldc,), 99.0, device="cuda")
            torch.cuda.synchronize()
            ctx.gemm_strided(trans_a, trans_b, m, n, k, alpha, da.data_ptr() + 4 * a_off, lda,
                             db.data_ptr() + 4 * b_off, ldb, dc.data_ptr() + 4 * c_off, ldc)
            ctx.synchronize()
            out = dc.cpu().numpy().reshape(m, ldc)
            A = a.reshape(a_rows, lda)[:, a_off:a_off + a_cols].astype(np.float64)
            B = b.reshape(b_rows, ldb)[:, b_off:b_off + b_cols].astype(np.float64)
            ref = alpha * ((A.T if trans_a else A) @ (B.T if trans_b else B))
            assert np.all(np.abs(out[:, c_off:c_off + n] - ref) <= 1e-4), (trans_a, trans_b)
            assert np.all(out[:, :c_off] == 99.0)
