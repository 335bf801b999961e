"""Products against the oracle: matmul, matmul_add and
matmul_transposed_add in f32 (rel 1e-5*sqrt(K)) and f16/bf16 (half
precision tolerance of the f32-accumulated, once-rounded result,
src/compact.rs:232-253); matvec and vecmat."""
from __future__ import annotations

import numpy as np
import pytest

import oracle as O
from tensorcrate_b200 import cuda
from tensorcrate_b200 import _native as N
from util import DTYPES, uniform

pytestmark = pytest.mark.gpu

SHAPES = [(1, 1, 1), (7, 5, 3), (96, 96, 96), (128, 64, 256), (129, 200, 257), (256, 512, 384), (300, 1024, 520),
          (1024, 1024, 1024), (256, 4096, 512), (130, 2048, 264)]  # the last two split K


def _tol(dtype, k):
    return {"f32": 1e-5 * np.sqrt(k), "f16": 2.0 ** -10 * 2, "bf16": 2.0 ** -7 * 2}[dtype]


def _run(dtype, transposed, m, k, n, accumulate, seed):
    a_shape = (k, m) if transposed == N.TRANS_LEFT else (m, k)
    b_shape = (n, k) if transposed == N.TRANS_RIGHT else (k, n)
    a = O.narrow(uniform(a_shape, seed), dtype)
    b = O.narrow(uniform(b_shape, seed + 1), dtype)
    c0 = O.narrow(uniform((m, n), seed + 2), dtype)
    da, db = cuda.CudaStorage.store(a, dtype), cuda.CudaStorage.store(b, dtype)
    dc = cuda.CudaStorage.store(c0, dtype) if accumulate else None
    got = O.widen(cuda.Cuda.matmul(da, db, m, k, n, transposed, dc).as_slice(), dtype)
    want = O.widen(O.matmul(dtype, transposed, m, k, n, a, b, c0 if accumulate else None, accumulate), dtype)
    return got, want


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("m,k,n", SHAPES)
def test_matmul(device, dtype, m, k, n):
    got, want = _run(dtype, N.TRANS_NONE, m, k, n, False, m + k + n)
    scale = max(1.0, float(np.max(np.abs(want))))
    assert np.max(np.abs(got - want)) <= _tol(dtype, k) * scale


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("transposed", [N.TRANS_NONE, N.TRANS_LEFT, N.TRANS_RIGHT])
@pytest.mark.parametrize("m,k,n", [(7, 5, 3), (130, 96, 72), (256, 320, 512), (256, 2048, 512)])
def test_transposed_accumulating_products(device, dtype, transposed, m, k, n):
    """The tape's backward products (tape/mod.rs:1195-1216)."""
    got, want = _run(dtype, transposed, m, k, n, True, 3 * m + k)
    scale = max(1.0, float(np.max(np.abs(want))))
    assert np.max(np.abs(got - want)) <= _tol(dtype, k) * scale


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("rows,cols", [(1, 1), (7, 13), (1024, 1024), (333, 4096)])
def test_matvec_and_vecmat(device, dtype, rows, cols):
    m = O.narrow(uniform((rows, cols), 1), dtype)
    x = O.narrow(uniform(cols, 2), dtype)
    y0 = O.narrow(uniform(rows, 3), dtype)
    dm, dx = cuda.CudaStorage.store(m, dtype), cuda.CudaStorage.store(x, dtype)
    got = O.widen(cuda.Cuda.matvec(dm, dx, rows, cols).as_slice(), dtype)
    want = np.empty(rows, m.dtype)
    O.call("orc_matvec", O.DTYPES[dtype], rows, cols, O.ptr(m), O.ptr(x), O.ptr(want), 0)
    want = O.widen(want, dtype)
    assert np.max(np.abs(got - want)) <= _tol(dtype, cols) * max(1.0, np.max(np.abs(want)))
    dy = cuda.CudaStorage.store(y0, dtype)
    got = O.widen(cuda.Cuda.matvec(dm, dx, rows, cols, addend=dy).as_slice(), dtype)
    want = y0.copy()
    O.call("orc_matvec", O.DTYPES[dtype], rows, cols, O.ptr(m), O.ptr(x), O.ptr(want), 1)
    want = O.widen(want, dtype)
    assert np.max(np.abs(got - want)) <= _tol(dtype, cols) * max(1.0, np.max(np.abs(want)))
    v = O.narrow(uniform(rows, 4), dtype)
    dv = cuda.CudaStorage.store(v, dtype)
    got = O.widen(cuda.Cuda.vecmat(dv, dm, rows, cols).as_slice(), dtype)
    want = np.empty(cols, m.dtype)
    O.call("orc_vecmat", O.DTYPES[dtype], rows, cols, O.ptr(v), O.ptr(m), O.ptr(want))
    want = O.widen(want, dtype)
    assert np.max(np.abs(got - want)) <= _tol(dtype, rows) * max(1.0, np.max(np.abs(want)))


def _sampled_rows_check(dtype, m, k, n, transposed, rows, seed):
    """Full-size products checked on a sample of output rows: the oracle's
    i-p-j rows are independent, so a band of rows is the whole product's."""
    a_shape = (k, m) if transposed == N.TRANS_LEFT else (m, k)
    b_shape = (n, k) if transposed == N.TRANS_RIGHT else (k, n)
    a = O.narrow(uniform(a_shape, seed), dtype)
    b = O.narrow(uniform(b_shape, seed + 1), dtype)
    da, db = cuda.CudaStorage.store(a, dtype), cuda.CudaStorage.store(b, dtype)
    got = O.widen(cuda.Cuda.matmul(da, db, m, k, n, transposed).as_slice(), dtype).reshape(m, n)
    a_rm = np.ascontiguousarray(a.reshape(a_shape).T) if transposed == N.TRANS_LEFT else a.reshape(m, k)
    b_rm = np.ascontiguousarray(b.reshape(b_shape).T) if transposed == N.TRANS_RIGHT else b.reshape(k, n)
    for r0 in rows:
        band = np.zeros(16 * n, dtype=O.STORE[dtype])
        O.call("orc_matmul_rows", O.DTYPES[dtype], 16, k, n, O.ptr(np.ascontiguousarray(a_rm[r0:r0 + 16])),
               O.ptr(b_rm), O.ptr(band), 0, 0, 16)
        want = O.widen(band, dtype).reshape(16, n)
        assert np.max(np.abs(got[r0:r0 + 16] - want)) <= _tol(dtype, k) * max(1.0, np.max(np.abs(want))), r0
    status = C.c_int(0)
    N.call("tc_device_status", C.byref(status))


import ctypes as C  # noqa: E402


@pytest.mark.parametrize("transposed", [N.TRANS_NONE, N.TRANS_LEFT, N.TRANS_RIGHT])
def test_bf16_2048_cubed_sampled(device, transposed):
    _sampled_rows_check("bf16", 2048, 2048, 2048, transposed, [0, 640, 2032], 7)


def test_bf16_config5_8192_sampled(device):
    """Config 5's middle size, M=N=K=8192, uniform[-1,1], checked on 48 rows."""
    _sampled_rows_check("bf16", 8192, 8192, 8192, N.TRANS_NONE, [0, 4096, 8176], 11)


def test_no_gemm_wait_gave_up(device):
    fault = C.c_int(0)
    N.call("tc_device_status", C.byref(fault))
    assert fault.value == 0


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("transposed", [N.TRANS_NONE, N.TRANS_LEFT, N.TRANS_RIGHT])
def test_outer_products(device, dtype, transposed):
    """An inner dimension of one (the tape's b ⊗ ones, tape/mod.rs:1000-1005):
    one rounding of an exact product, so f16/bf16 match bit for bit."""
    for (m, n) in [(4096, 2048), (7, 13)]:
        for accumulate in (False, True):
            got, want = _run(dtype, transposed, m, 1, n, accumulate, m + n)
            if dtype == "f32":
                assert np.max(np.abs(got - want)) <= 2 ** -22 * max(1.0, np.max(np.abs(want)))
            else:
                assert np.array_equal(got, want)


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("m,k,n", [(7, 5, 3), (130, 96, 72), (256, 320, 512), (4096, 1024, 264), (128, 8, 256),
                                   (1024, 4096, 256)])
@pytest.mark.parametrize("relu", [True, False])
def test_matmul_epilogue_matches_the_separate_operations(device, dtype, m, k, n, relu):
    """tc_matmul_epilogue (Kernels::matmul_epilogue, kernels.rs:1137-1150)
    for a dense layer's programs: forward A = P + bias[row], H = max(A, 0);
    backward P * MaxShare(A, 0).  It must give the bits of the separate
    operations the tape runs: the product (tc_matmul), then each
    elementwise operation rounded in turn."""
    a = O.narrow(uniform((m, k), m + k), dtype)
    b = O.narrow(uniform((k, n), n + 1), dtype)
    bias = O.narrow(uniform(m, 9), dtype)
    share_src = O.narrow(np.round(uniform((m, n), 4) * 2) / 2, dtype)  # negative, zero and positive entries
    da, db, dbias, dshare = (cuda.CudaStorage.store(x, dtype) for x in (a, b, bias, share_src))
    product = cuda.Cuda.matmul(da, db, m, k, n).as_slice()
    pw = O.widen(product, dtype).reshape(m, n)
    want_a = O.narrow(pw + O.widen(bias, dtype)[:, None], dtype).reshape(-1)
    want_h = O.narrow(np.maximum(O.widen(want_a, dtype), np.float32(0)), dtype)
    sw = O.widen(share_src, dtype).reshape(m, n)
    share = np.where(sw > 0, 1.0, np.where(sw < 0, 0.0, 0.5)).astype(np.float32)
    want_s = O.narrow(pw * share, dtype).reshape(-1)
    code = N.DTYPES[dtype]
    got = cuda.CudaStorage(dtype, m * n)
    got_h = cuda.CudaStorage(dtype, m * n) if relu else None
    N.call("tc_matmul_epilogue", code, N.TRANS_NONE, m, k, n, da.ptr, db.ptr, None, dbias.ptr, got.ptr,
           got_h.ptr if relu else None, None)
    assert np.array_equal(got.as_slice(), want_a)
    if relu:
        assert np.array_equal(got_h.as_slice(), want_h)
    N.call("tc_matmul_epilogue", code, N.TRANS_NONE, m, k, n, da.ptr, db.ptr, dshare.ptr, None, got.ptr, None, None)
    assert np.array_equal(got.as_slice(), want_s)
    N.call("tc_matmul_epilogue", code, N.TRANS_NONE, m, k, n, da.ptr, db.ptr, None, None, got.ptr, None, None)
    assert np.array_equal(got.as_slice(), product)
