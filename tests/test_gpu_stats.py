"""Moments and distribution functions through the C ABI (vector_moments,
matrix_moments, matrix_axis_moments, vector/matrix/matrix_axis
_distribution; kernels.rs:1035-1070), against the oracle.

Parity: moments are sums (rel 1e-5·√K; exact on the integral filler's
means); the distribution functions are f64 evaluations rounded once, held
to 1 step of the element type from the oracle's (CUDA's f64 exp/log/sqrt
and the C library's differ by an f64 ulp at most, which moves a rounded
result by one step only at a rounding boundary)."""
from __future__ import annotations

import numpy as np
import pytest

import oracle as O
from tensorcrate_b200 import _native as N
from tensorcrate_b200 import cuda
from util import DTYPES, expand, integral, kats, normal, steps, uniform

pytestmark = pytest.mark.gpu


def moments_gpu(a, dtype):
    out = cuda.CudaStorage(dtype, 2)
    src = cuda.CudaStorage.store(a, dtype) if a.size else None
    N.call("tc_moments", N.DTYPES[dtype], src.ptr if src else None, a.size, out.ptr, None)
    return out.as_slice()


@pytest.mark.parametrize("k", kats("moments"), ids=lambda k: k["id"])
def test_moments_worked_examples(device, k):
    a = np.array(expand(k["input"]), np.float32)
    got = moments_gpu(a, "f32")
    want = np.array(expand(k["expect"]), np.float32)
    assert np.array_equal(got, want, equal_nan=True)


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("n", [1, 7, 1000, (1 << 20) + 7])
def test_moments_match_the_oracle(device, dtype, n):
    a = O.narrow(normal(n, 3) + np.float32(2.0), dtype)
    got = O.widen(moments_gpu(a, dtype), dtype).astype(np.float64)
    want = np.empty(2, a.dtype)
    O.call("orc_moments", O.DTYPES[dtype], O.ptr(a), n, O.ptr(want))
    want = O.widen(want, dtype).astype(np.float64)
    rel = 1e-5 * np.sqrt(n) + (0 if dtype == "f32" else (2.0 ** -7 if dtype == "bf16" else 2.0 ** -10))
    # f16's deviation sum of a million values overflows to inf on both sides
    same_inf = np.isinf(got) & (got == want)
    with np.errstate(invalid="ignore"):  # inf - inf where both overflowed
        close = np.abs(got - want) <= rel * np.maximum(np.abs(want), 1.0)
    assert np.all(same_inf | close)


@pytest.mark.parametrize("dtype", DTYPES)
def test_moments_of_the_integral_filler_have_the_hosts_mean(device, dtype):
    n = 1 << 16
    a = O.narrow(integral(n), dtype)
    got = moments_gpu(a, dtype)
    want = np.empty(2, a.dtype)
    O.call("orc_moments", O.DTYPES[dtype], O.ptr(a), n, O.ptr(want))
    assert got[0] == want[0]


@pytest.mark.parametrize("k", kats("axis_moments"), ids=lambda k: k["id"])
def test_axis_moments_worked_examples(device, k):
    a = cuda.CudaStorage.store(np.array(k["input"], np.float32), "f32")
    r, c = k["shape"]
    extent = r if k["axis"] == N.ROWS else c
    means, devs = cuda.CudaStorage("f32", extent), cuda.CudaStorage("f32", extent)
    N.call("tc_axis_moments", N.F32, r, c, k["axis"], a.ptr, means.ptr, devs.ptr, None)
    want = k.get("expect_means") or [np.float32(v) for v in k["expect_means_f64"]]
    assert list(means.as_slice()) == list(np.array(want, np.float32))


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("shape", [(64, 1000), (1000, 64), (1, 5000), (5000, 1), (3, 0)])
@pytest.mark.parametrize("axis", [N.ROWS, N.COLUMNS])
def test_axis_moments_match_the_oracle(device, dtype, shape, axis):
    r, c = shape
    a = O.narrow(uniform(r * c, 4) * np.float32(3.0) + np.float32(1.0), dtype)
    extent, depth = (r, c) if axis == N.ROWS else (c, r)
    src = cuda.CudaStorage.store(a, dtype) if a.size else None
    means, devs = cuda.CudaStorage(dtype, extent), cuda.CudaStorage(dtype, extent)
    N.call("tc_axis_moments", N.DTYPES[dtype], r, c, axis, src.ptr if src else None, means.ptr, devs.ptr, None)
    wm, wd = np.empty(extent, a.dtype), np.empty(extent, a.dtype)
    O.call("orc_axis_moments", O.DTYPES[dtype], r, c, axis, O.ptr(a), O.ptr(wm), O.ptr(wd))
    rel = 1e-5 * np.sqrt(max(depth, 1)) + (0 if dtype == "f32" else (2.0 ** -7 if dtype == "bf16" else 2.0 ** -10))
    for got, want in ((means, wm), (devs, wd)):
        g = O.widen(got.as_slice(), dtype).astype(np.float64)
        w = O.widen(want, dtype).astype(np.float64)
        if depth == 0:
            assert np.all(np.isnan(g))
        else:
            assert np.all(np.abs(g - w) <= rel * np.maximum(np.abs(w), 1.0))


def _inputs(family, statistic, n, seed):
    rng = np.random.default_rng(seed)
    if statistic == N.PPF:
        x = rng.uniform(0.0, 1.0, n)
        x[:4] = [0.0, 1.0, 1e-6, 1.0 - 1e-6]
        x[4:6] = [1.5, -0.25]  # outside [0, 1]: NaN
        return x.astype(np.float32)
    if family == N.NORMAL:
        return (rng.standard_normal(n) * 4.0).astype(np.float32)
    x = rng.uniform(-0.5, 6.0, n)
    x[:2] = [0.0, -1.0]
    return x.astype(np.float32)


CASES = [(f, s, p) for f, params in ((N.NORMAL, [(0.5, 2.0), (0.0, 1.0), (1.0, -1.0)]),
                                     (N.INVERSE_GAUSSIAN, [(1.0, 1.0), (2.0, 0.5), (0.5, 20.0), (1.0, 1e6)]))
         for s in (N.PDF, N.CDF, N.PPF) for p in params]


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("family,statistic,params", CASES)
def test_distribution_matches_the_oracle(device, dtype, family, statistic, params):
    n = 3001
    a = O.narrow(_inputs(family, statistic, n, 7 + statistic), dtype)
    # the parameters as element-type values
    p0, p1 = (float(v) for v in O.widen(O.narrow(np.array(params, np.float32), dtype), dtype))
    src, out = cuda.CudaStorage.store(a, dtype), cuda.CudaStorage(dtype, n)
    N.call("tc_distribution", N.DTYPES[dtype], family, statistic, src.ptr, n, p0, p1, out.ptr, None)
    want = np.empty_like(a)
    O.call("orc_distribution", O.DTYPES[dtype], family, statistic, O.ptr(a), n, p0, p1, O.ptr(want))
    assert int(np.max(steps(out.as_slice(), want, dtype))) <= 1


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("axis", [N.ROWS, N.COLUMNS])
@pytest.mark.parametrize("family", [N.NORMAL, N.INVERSE_GAUSSIAN])
def test_axis_distribution_matches_the_oracle(device, dtype, axis, family):
    r, c = 37, 53
    extent = r if axis == N.ROWS else c
    rng = np.random.default_rng(5)
    first = O.narrow(rng.uniform(0.5, 2.0, extent).astype(np.float32), dtype)
    second = O.narrow(rng.uniform(0.5, 3.0, extent).astype(np.float32), dtype)
    for statistic in (N.PDF, N.CDF, N.PPF):
        a = O.narrow(_inputs(family, statistic, r * c, 9 + statistic), dtype)
        src, out = cuda.CudaStorage.store(a, dtype), cuda.CudaStorage(dtype, r * c)
        df, ds = cuda.CudaStorage.store(first, dtype), cuda.CudaStorage.store(second, dtype)
        N.call("tc_axis_distribution", N.DTYPES[dtype], r, c, axis, family, statistic, src.ptr, df.ptr, ds.ptr,
               out.ptr, None)
        want = np.empty_like(a)
        O.call("orc_axis_distribution", O.DTYPES[dtype], r, c, axis, family, statistic, O.ptr(a), O.ptr(first),
               O.ptr(second), O.ptr(want))
        assert int(np.max(steps(out.as_slice(), want, dtype))) <= 1, statistic
