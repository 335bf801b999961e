"""Same-shape elementwise, scalar broadcast, comparisons, clamp and the
broadcasting strided binary against the oracle.  Bit-exact for add, sub,
mul, div, rem and every comparison (north star); power within 2 ulp."""
from __future__ import annotations

import numpy as np
import pytest

import oracle as O
from tensorcrate_b200 import cuda
from tensorcrate_b200 import _native as N
from util import DTYPES, integral, normal

pytestmark = pytest.mark.gpu

ARITH = [N.ADD, N.SUB, N.MUL, N.DIV, N.REM]
COMPARES = list(range(7))


def _specials(dtype):
    v = np.array([0.0, -0.0, 1.0, -1.0, np.inf, -np.inf, np.nan, 3.5, -2.25, 1e-30, 65504.0, 1e30], np.float32)
    return O.narrow(v, dtype)


def _inputs(dtype, n, seed):
    a = O.narrow(normal(n, seed) * 3, dtype)
    b = O.narrow(normal(n, seed + 1) * 3, dtype)
    sp = _specials(dtype)
    a[: sp.size * sp.size] = np.repeat(sp, sp.size)[: min(a.size, sp.size * sp.size)]
    b[: sp.size * sp.size] = np.tile(sp, sp.size)[: min(b.size, sp.size * sp.size)]
    # some exact ties, for the comparisons
    b[200:260] = a[200:260]
    return a, b


def _bits_equal(got, want, dtype):
    g, w = O.widen(got, dtype), O.widen(want, dtype)
    both_nan = np.isnan(g) & np.isnan(w)
    return bool(np.all((got == want) | both_nan))


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("n", [1, 7, 1000, 4099, 65536 * 3 + 5])
def test_same_shape_arithmetic_and_compare(device, dtype, n):
    a, b = _inputs(dtype, max(n, 300), 10)
    a, b = a[:n].copy(), b[:n].copy()
    da, db = cuda.CudaStorage.store(a, dtype), cuda.CudaStorage.store(b, dtype)
    for op in ARITH:
        got = cuda.Cuda.vector_elementwise(da, db, op).as_slice()
        want = np.empty_like(a)
        O.call("orc_elementwise", O.DTYPES[dtype], op, O.ptr(a), O.ptr(b), O.ptr(want), n)
        assert _bits_equal(got, want, dtype), f"op {op}"
    for cmp in COMPARES:
        got = cuda.Cuda.vector_compare(da, db, cmp).as_slice()
        want = np.empty_like(a)
        O.call("orc_compare", O.DTYPES[dtype], cmp, O.ptr(a), O.ptr(b), O.ptr(want), n)
        if cmp in (N.MIN, N.MAX):
            # the sign of a zero when -0 meets +0 is not pinned (kernels.rs:96-103)
            g, w = O.widen(got, dtype), O.widen(want, dtype)
            ok = (g == w) | (np.isnan(g) & np.isnan(w))
            assert ok.all(), f"compare {cmp}"
        else:
            assert np.array_equal(got, want), f"compare {cmp}"


@pytest.mark.parametrize("dtype", DTYPES)
def test_scalar_forms_and_clamp(device, dtype):
    n = 5003
    a, _ = _inputs(dtype, n, 20)
    da = cuda.CudaStorage.store(a, dtype)
    for scalar in (0.0, -1.5, 3.0):
        for left in (False, True):
            for op in ARITH:
                got = cuda.Cuda.vector_broadcast(da, scalar, op, left).as_slice()
                want = np.empty_like(a)
                O.call("orc_broadcast_scalar", O.DTYPES[dtype], op, O.ptr(a), scalar, int(left), O.ptr(want), n)
                assert _bits_equal(got, want, dtype)
            for cmp in COMPARES:
                got = cuda.Cuda.vector_compare_scalar(da, scalar, cmp, left).as_slice()
                want = np.empty_like(a)
                O.call("orc_compare_scalar", O.DTYPES[dtype], cmp, O.ptr(a), scalar, int(left), O.ptr(want), n)
                g, w = O.widen(got, dtype), O.widen(want, dtype)
                assert np.all((g == w) | (np.isnan(g) & np.isnan(w)))
    got = cuda.Cuda.vector_clamp(da, -1.0, 2.0).as_slice()
    want = np.empty_like(a)
    O.call("orc_clamp", O.DTYPES[dtype], O.ptr(a), -1.0, 2.0, O.ptr(want), n)
    assert np.array_equal(O.widen(got, dtype), O.widen(want, dtype))


def _strided(dtype, kind, op, shape, a, a_off, a_str, b, b_off, b_str):
    da, db = cuda.CudaStorage.store(a, dtype), cuda.CudaStorage.store(b, dtype)
    va = cuda.TensorView(da, list(shape), list(a_str), a_off)
    vb = cuda.TensorView(db, list(shape), list(b_str), b_off)
    got = cuda.Cuda.strided_binary(va, vb, kind, op).as_slice()
    want = O.strided_binary(dtype, kind, op, shape, a, a_off, a_str, b, b_off, b_str)
    return got, want


@pytest.mark.parametrize("dtype", DTYPES)
def test_broadcast_binary_layouts(device, dtype):
    """tensor_ops.rs:71-91 through strided_binary: bias broadcasts, scalar
    broadcasts, permuted and sliced operands."""
    rng = np.random.default_rng(30)
    cases = []
    # [B, T, F] + [F] (config 2's layout), odd and even inner extents
    for F in (1024, 1000, 7):
        shape = [3, 5, F]
        cases.append((shape, [5 * F, F, 1], 0, [0, 0, 1], 0))
    # a column broadcast and a leading-axis broadcast
    cases.append(([6, 9], [9, 1], 0, [1, 0], 0))
    cases.append(([4, 6, 9], [54, 9, 1], 0, [0, 9, 1], 0))
    # a transposed operand, and an offset slice
    cases.append(([7, 5], [1, 7], 0, [5, 1], 0))
    cases.append(([3, 4, 5], [40, 5, 1], 13, [20, 5, 1], 3))
    for shape, a_str, a_off, b_str, b_off in cases:
        na = a_off + sum((e - 1) * s for e, s in zip(shape, a_str)) + 1
        nb = b_off + sum((e - 1) * s for e, s in zip(shape, b_str)) + 1
        a = O.narrow(normal(na, int(rng.integers(1000))), dtype)
        b = O.narrow(normal(nb, int(rng.integers(1000))), dtype)
        for kind, ops in ((N.PAIR_ARITHMETIC, ARITH), (N.PAIR_COMPARE, COMPARES)):
            for op in ops:
                got, want = _strided(dtype, kind, op, shape, a, a_off, a_str, b, b_off, b_str)
                assert _bits_equal(got, want, dtype), (shape, kind, op)


@pytest.mark.parametrize("dtype", DTYPES)
def test_power_within_two_ulp(device, dtype):
    shape = [4, 257]
    a = O.narrow(np.abs(normal(4 * 257, 5)) * 2 + 0.01, dtype)
    b = O.narrow(normal(257, 6), dtype)
    got, want = _strided(dtype, N.PAIR_POWER, 0, shape, a, 0, [257, 1], b, 0, [0, 1])
    g, w = O.widen(got, dtype).astype(np.float64), O.widen(want, dtype).astype(np.float64)
    ulp = {"f32": 2.0 ** -23, "f16": 2.0 ** -10, "bf16": 2.0 ** -7}[dtype]
    assert np.all(np.abs(g - w) <= 2 * ulp * np.abs(w) + 1e-38)


def test_config2_broadcast_at_full_size(device):
    """Config 2's broadcast ops on f32 [64,512,1024] + [1,1,1024]: exact
    against the oracle on a row sample, and a checksum of the whole."""
    shape = [64, 512, 1024]
    x = normal(shape, 1).reshape(-1)
    bias = normal([1024], 2)
    t = cuda.Tensor(cuda.CudaStorage.store(x, "f32"), shape)
    b = cuda.Tensor(cuda.CudaStorage.store(bias, "f32"), [1, 1, 1024])
    for kind, op, f in [(N.PAIR_ARITHMETIC, N.ADD, lambda u, v: u + v), (N.PAIR_ARITHMETIC, N.MUL, lambda u, v: u * v),
                        (N.PAIR_COMPARE, N.GREATER, lambda u, v: (u > v).astype(np.float32))]:
        out = cuda.elementwise(t, b, kind, op).storage.as_slice()
        want = f(x.reshape(-1, 1024), bias).reshape(-1)
        assert np.array_equal(out, want)
