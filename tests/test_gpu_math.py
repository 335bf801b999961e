"""The other vector methods of Kernels<T> through the C ABI: vector_unary
and vector_unary_dual (kernels.rs:876, 891; Host 1257-1304), vector_power
and vector_power_scalar (kernels.rs:884-888), vector_prefix_sum
(kernels.rs:870; vector.rs:578-589) and vector_sort (kernels.rs:873;
vector.rs:874-886), each against the oracle on the same seeded inputs.

Parity: sort is a permutation (same bits, as tests/ordering.rs:411-418 asks
of the Metal tier); the prefix sum is exact on the integral filler and
within an f32 sum's rounding otherwise; the analytic functions and powers
within 2 ulp of the element type (the transcendental bound)."""
from __future__ import annotations

import numpy as np
import pytest

import oracle as O
from tensorcrate_b200 import _native as N
from tensorcrate_b200 import cuda
from util import DTYPES, bits_of, integral, normal, steps, uniform

pytestmark = pytest.mark.gpu


def _domain(f, n, seed):
    x = uniform(n, seed)
    if f in (N.ARCSIN, N.ARCCOS):
        return x * np.float32(0.95)
    if f in (N.LN, N.SQRT):
        return np.abs(x) * np.float32(4.0) + np.float32(0.01)
    if f in (N.EXP, N.SINH, N.COSH):
        return x * np.float32(8.0)
    return x * np.float32(3.0)


FUNCS = list(range(14))
EXACT = [np.sin, np.cos, np.tan, lambda v: 1 / np.cos(v), lambda v: 1 / np.sin(v), np.arcsin, np.arccos, np.arctan,
         np.exp, np.log, np.sinh, np.cosh, np.tanh, np.sqrt]


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("f", FUNCS)
def test_unary_matches_the_oracle(device, dtype, f):
    """f32: within 2 ulp of the exact value (3 for sec and csc, a quotient
    of a 2-ulp function), so within twice that of the oracle, whose C library
    functions carry their own 2-ulp bound; the root is exact.  f16/bf16:
    both sides round an f32 value within those bounds, so they agree within
    2 steps of the element type."""
    n = 4099
    x = O.narrow(_domain(f, n, 40 + f), dtype)
    got = cuda.Cuda.vector_unary(cuda.CudaStorage.store(x, dtype), f).as_slice()
    want = np.empty_like(x)
    O.call("orc_unary", O.DTYPES[dtype], f, O.ptr(x), O.ptr(want), n)
    bound = 0 if f == N.SQRT else (3 if f in (N.SEC, N.CSC) else 2)
    if dtype == "f32":
        exact = EXACT[f](x.astype(np.float64))
        ulp = np.spacing(np.abs(exact).astype(np.float32)).astype(np.float64)
        assert float(np.max(np.abs(got.astype(np.float64) - exact) / ulp)) <= bound + 0.5
        assert int(np.max(steps(got, want, dtype))) <= 2 * bound
    else:
        assert int(np.max(steps(got, want, dtype))) <= min(bound, 2)


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("f", FUNCS)
def test_unary_dual_matches_the_oracle(device, dtype, f):
    """(f(x), f'(x)·t): the value as vector_unary; the tangent composes up
    to four rounded operations on 2-ulp functions on each side, so it is
    held to 8 steps of f32 (4 of f16/bf16) from the oracle's."""
    n = 2053
    x = O.narrow(_domain(f, n, 60 + f), dtype)
    t = O.narrow(uniform(n, 80 + f), dtype)
    xv, tv = cuda.CudaStorage.store(x, dtype), cuda.CudaStorage.store(t, dtype)
    got_v, got_t = cuda.Cuda.vector_unary_dual(xv, tv, f)
    want_v, want_t = np.empty_like(x), np.empty_like(x)
    O.call("orc_unary_dual", O.DTYPES[dtype], f, O.ptr(x), O.ptr(t), O.ptr(want_v), O.ptr(want_t), n)
    bound = 0 if f == N.SQRT else (3 if f in (N.SEC, N.CSC) else 2)
    assert int(np.max(steps(got_v.as_slice(), want_v, dtype))) <= (2 * bound if dtype == "f32" else min(bound, 2))
    if dtype == "f32" and f == N.TANH:
        # 1 - tanh² cancels near |tanh| = 1: a 2-ulp difference in tanh
        # moves it by up to about 2^-22 absolutely, whatever its size.
        g, w = got_t.as_slice().astype(np.float64), want_t.astype(np.float64)
        ulp = np.spacing(np.abs(want_t)).astype(np.float64)
        assert np.all(np.abs(g - w) <= 8 * ulp + 2.0 ** -20 * np.abs(t.astype(np.float64)))
    else:
        assert int(np.max(steps(got_t.as_slice(), want_t, dtype))) <= (8 if dtype == "f32" else 4)


@pytest.mark.parametrize("dtype", DTYPES)
def test_power_and_power_scalar_match_the_oracle(device, dtype):
    n = 5003
    a = O.narrow(np.abs(uniform(n, 7)) * np.float32(3.0) + np.float32(0.05), dtype)
    b = O.narrow(uniform(n, 8) * np.float32(4.0), dtype)
    da, db = cuda.CudaStorage.store(a, dtype), cuda.CudaStorage.store(b, dtype)
    got = cuda.Cuda.vector_power(da, db).as_slice()
    want = np.empty_like(a)
    O.call("orc_power", O.DTYPES[dtype], O.ptr(a), O.ptr(b), O.ptr(want), n)
    assert int(np.max(steps(got, want, dtype))) <= 2
    for scalar, left in ((2.5, False), (1.75, True), (-3.0, False)):
        got = cuda.Cuda.vector_power_scalar(da, scalar, left).as_slice()
        O.call("orc_power_scalar", O.DTYPES[dtype], O.ptr(a), scalar, int(left), O.ptr(want), n)
        assert int(np.max(steps(got, want, dtype))) <= 2, (scalar, left)


SCAN_SIZES = [1, 5, 17, 2048, 2049, 100_003, (1 << 20) + 3, 9_000_001]


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("n", SCAN_SIZES)
def test_prefix_sum_of_the_integral_filler_is_exact(device, dtype, n):
    """Every partial sum of the filler is a small integer, exact in f32 in
    any order, so the scan must give the Host's bits."""
    a = O.narrow(integral(n), dtype)
    got = cuda.Cuda.vector_prefix_sum(cuda.CudaStorage.store(a, dtype)).as_slice()
    want = np.empty_like(a)
    O.call("orc_prefix_sum", O.DTYPES[dtype], O.ptr(a), O.ptr(want), n)
    assert np.array_equal(got, want)


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("n", [1000, (1 << 20) + 3, 9_000_001])
def test_prefix_sum_of_normal_values_within_sum_rounding(device, dtype, n):
    """N(0,1) values: the tree of f32 additions differs from the Host's
    serial chain; both are within n·2^-24·Σ|x| of the exact prefix, so they
    are held to that bound plus one rounding to the element type."""
    a = O.narrow(normal(n, 11), dtype)
    got = O.widen(cuda.Cuda.vector_prefix_sum(cuda.CudaStorage.store(a, dtype)).as_slice(), dtype)
    want_bits = np.empty_like(a)
    O.call("orc_prefix_sum", O.DTYPES[dtype], O.ptr(a), O.ptr(want_bits), n)
    want = O.widen(want_bits, dtype).astype(np.float64)
    x = O.widen(a, dtype).astype(np.float64)
    bound = 2.0 * np.log2(n) * 2.0 ** -24 * np.cumsum(np.abs(x)) + 2.0 * 2.0 ** -24 * n * np.abs(x).mean()
    half = 0.0 if dtype == "f32" else (2.0 ** -7 if dtype == "bf16" else 2.0 ** -10) * np.abs(want)
    err = np.abs(got.astype(np.float64) - want)
    assert np.all(err <= bound + half + 1e-30)


def test_prefix_sum_of_nothing_is_nothing(device):
    out = cuda.CudaStorage("f32", 0)
    N.call("tc_prefix_sum", N.F32, None, out.ptr, 0, None)


def _awkward(n, seed, dtype):
    x = normal(n, seed)
    rng = np.random.default_rng(seed + 1)
    specials = np.array([np.nan, -np.nan, np.inf, -np.inf, 0.0, -0.0], np.float32)
    at = rng.choice(n, size=max(1, n // 50), replace=False)
    x[at] = specials[rng.integers(0, len(specials), size=at.size)]
    # repeated values, so equal keys meet in the sort
    x[: n // 4] = np.round(x[: n // 4] * 4) / 4
    return O.narrow(x, dtype)


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("n", [1, 7, 1000, 4096, 4097, (1 << 20) + 1])
@pytest.mark.parametrize("order", [N.ASCENDING, N.DESCENDING])
def test_sort_matches_the_oracle_bit_for_bit(device, dtype, n, order):
    a = _awkward(n, 21, dtype)
    got = cuda.Cuda.vector_sort(cuda.CudaStorage.store(a, dtype), order).as_slice()
    want = np.empty_like(a)
    O.call("orc_sort", O.DTYPES[dtype], order, O.ptr(a), O.ptr(want), n)
    assert np.array_equal(bits_of(got, dtype), bits_of(want, dtype))


@pytest.mark.parametrize("dtype", DTYPES)
def test_sort_of_few_distinct_values(device, dtype):
    """Every key in a handful of digits: the radix passes' counts pile into
    few bins and each tile's ranks run long."""
    rng = np.random.default_rng(5)
    a = O.narrow(rng.choice(np.array([1.0, -2.5, 0.0, 3.0], np.float32), size=300001), dtype)
    for order in (N.ASCENDING, N.DESCENDING):
        got = cuda.Cuda.vector_sort(cuda.CudaStorage.store(a, dtype), order).as_slice()
        want = np.empty_like(a)
        O.call("orc_sort", O.DTYPES[dtype], order, O.ptr(a), O.ptr(want), a.size)
        assert np.array_equal(bits_of(got, dtype), bits_of(want, dtype))


@pytest.mark.parametrize("dtype", DTYPES)
def test_sort_in_place(device, dtype):
    """tc_sort with out == a: the first pass reads the values before any pass
    writes `out`."""
    a = _awkward(70001, 23, dtype)
    buf = cuda.CudaStorage.store(a, dtype)
    N.call("tc_sort", N.DTYPES[dtype], N.DESCENDING, buf.ptr, buf.ptr, a.size, None)
    want = np.empty_like(a)
    O.call("orc_sort", O.DTYPES[dtype], N.DESCENDING, O.ptr(a), O.ptr(want), a.size)
    assert np.array_equal(bits_of(buf.as_slice(), dtype), bits_of(want, dtype))


def test_sort_orders_nans_and_zeros_like_the_host(device):
    """tests/ordering.rs:422-440: -NaN first, -0.0 before +0.0, +NaN last."""
    bits = np.array([0x7FC00000, 0, 0x80000000, 0xFFC00000, 0x3F800000, 0xFF800000, 0x40200000], np.uint32)
    a = bits.view(np.float32)
    for order in (N.ASCENDING, N.DESCENDING):
        got = cuda.Cuda.vector_sort(cuda.CudaStorage.store(a, "f32"), order).as_slice().view(np.uint32)
        want = np.empty_like(a)
        O.call("orc_sort", O.DTYPES["f32"], order, O.ptr(a), O.ptr(want), a.size)
        assert list(got) == list(want.view(np.uint32))
    asc = cuda.Cuda.vector_sort(cuda.CudaStorage.store(a, "f32"), N.ASCENDING).as_slice().view(np.uint32)
    assert [int(b) for b in asc] == [0xFFC00000, 0xFF800000, 0x80000000, 0, 0x3F800000, 0x40200000, 0x7FC00000]
