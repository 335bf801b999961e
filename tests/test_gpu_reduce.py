"""Axis reductions and arg-reductions against the oracle, on the shapes the
reference tests (tests/broadcast_reduce.rs:388-416, 700-812): every subset of
axes, permuted views, leading and trailing axes, long slices.  With the
integral filler every sum is exact, so sums match bit for bit; min, max and
arg always do; N(0,1) data check sums within rel 1e-5*sqrt(K)."""
from __future__ import annotations

import itertools

import numpy as np
import pytest

import oracle as O
from tensorcrate_b200 import cuda
from tensorcrate_b200 import _native as N
from util import DTYPES, integral, normal

pytestmark = pytest.mark.gpu

FOLDS = [(N.AXIS_FOLD, N.SUM), (N.AXIS_FOLD, N.RMIN), (N.AXIS_FOLD, N.RMAX), (N.AXIS_MEAN, 0), (N.AXIS_VARIANCE, 0)]


def _check(dtype, shape, x, offset, strides, exact: bool, tol: float):
    s = cuda.CudaStorage.store(x, dtype)
    view = cuda.TensorView(s, list(shape), list(strides), offset)
    rank = len(shape)
    for r in range(1, rank + 1):
        for axes in itertools.combinations(range(rank), r):
            axes = list(axes)
            depth = int(np.prod([shape[a] for a in axes]))
            for kind, op in FOLDS:
                divisor = depth - 1 if kind == N.AXIS_VARIANCE else 0
                if kind == N.AXIS_VARIANCE and divisor == 0:
                    continue
                got = O.widen(cuda.Cuda.reduce_axes(view, axes, kind, op, divisor).as_slice(), dtype)
                want = O.widen(O.reduce_axes(dtype, shape, x, offset, strides, axes, kind, op, divisor), dtype)
                # With the integral filler every sum is exact in f32, so a
                # fold and a mean agree bit for bit; a variance's deviations
                # from a fractional mean do not.
                if (exact and kind != N.AXIS_VARIANCE) or (kind == N.AXIS_FOLD and op != N.SUM):
                    assert np.array_equal(got, want), (axes, kind, op)
                else:
                    scale = np.abs(want) + 1.0
                    assert np.all(np.abs(got - want) <= tol * np.sqrt(depth) * scale), (axes, kind, op)
    for axis in range(rank):
        for op in (N.RMAX, N.RMIN):
            got = cuda.Cuda.arg_reduce(view, axis, op).as_slice()
            want = O.arg_reduce(dtype, shape, x, offset, strides, axis, op)
            assert np.array_equal(got, want), (axis, op)


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("shape", [[2, 3, 4, 5], [3, 2, 5, 70], [80, 3, 2, 4]])
def test_every_subset_with_the_integral_filler(device, dtype, shape):
    n = int(np.prod(shape))
    x = O.narrow(integral(n), dtype)
    _check(dtype, shape, x, 0, cuda.contiguous_strides(shape), exact=True, tol=1e-5)


@pytest.mark.parametrize("dtype", DTYPES)
def test_permuted_and_offset_views(device, dtype):
    shape = [2, 3, 4, 5]
    x = O.narrow(integral(200), dtype)
    base = cuda.contiguous_strides(shape)
    perm = [3, 1, 0, 2]
    _check(dtype, [shape[p] for p in perm], x, 7, [base[p] for p in perm], exact=True, tol=1e-5)


@pytest.mark.parametrize("shape,axis", [([100, 1100], 0), ([1100, 100], 1), ([100, 1100], 1), ([1100, 100], 0)])
def test_long_slices_match_exactly(device, shape, axis):
    """tests/broadcast_reduce.rs:789-812: exact sums, maxima and argmaxima."""
    x = integral(int(np.prod(shape)))
    s = cuda.CudaStorage.store(x, "f32")
    st = cuda.contiguous_strides(shape)
    v = cuda.TensorView(s, shape, st, 0)
    for kind, op in [(N.AXIS_FOLD, N.SUM), (N.AXIS_FOLD, N.RMAX)]:
        got = cuda.Cuda.reduce_axes(v, [axis], kind, op, 0).as_slice()
        assert np.array_equal(got, O.reduce_axes("f32", shape, x, 0, st, [axis], kind, op, 0))
    got = cuda.Cuda.arg_reduce(v, axis, N.RMAX).as_slice()
    assert np.array_equal(got, O.arg_reduce("f32", shape, x, 0, st, axis, N.RMAX))


@pytest.mark.parametrize("dtype", DTYPES)
def test_normal_data_within_tolerance(device, dtype):
    shape = [16, 33, 1024]
    x = O.narrow(normal(shape, 9).reshape(-1), dtype)
    tol = {"f32": 1e-5, "f16": 2e-3, "bf16": 1e-2}[dtype]
    st = cuda.contiguous_strides(shape)
    s = cuda.CudaStorage.store(x, dtype)
    v = cuda.TensorView(s, shape, st, 0)
    for axes in ([2], [0, 2], [1], [0, 1, 2]):
        depth = int(np.prod([shape[a] for a in axes]))
        for kind, op in FOLDS:
            divisor = depth if kind == N.AXIS_VARIANCE else 0
            got = O.widen(cuda.Cuda.reduce_axes(v, axes, kind, op, divisor).as_slice(), dtype)
            want = O.widen(O.reduce_axes(dtype, shape, x, 0, st, axes, kind, op, divisor), dtype)
            if kind == N.AXIS_FOLD and op != N.SUM:
                assert np.array_equal(got, want)
            else:
                xa = np.abs(O.widen(x, dtype)).reshape(shape)
                mass = xa.sum(axis=tuple(axes)).reshape(-1) / np.sqrt(depth)
                assert np.all(np.abs(got - want) <= tol * np.sqrt(depth) * (np.abs(want) + mass + 1e-6)), (axes, kind)


def test_config2_reductions_at_full_size(device):
    """Config 2's reductions on f32 [64,512,1024] N(0,1): sum/mean/var over
    axis 2, max/min over (0,2), argmax over axis 1 — against the oracle."""
    shape = [64, 512, 1024]
    x = normal(shape, 1).reshape(-1)
    st = cuda.contiguous_strides(shape)
    s = cuda.CudaStorage.store(x, "f32")
    v = cuda.TensorView(s, shape, st, 0)
    for kind, op, axes, div in [(N.AXIS_FOLD, N.SUM, [2], 0), (N.AXIS_MEAN, 0, [2], 0),
                                (N.AXIS_VARIANCE, 0, [2], 1024), (N.AXIS_FOLD, N.RMAX, [0, 2], 0),
                                (N.AXIS_FOLD, N.RMIN, [0, 2], 0)]:
        got = cuda.Cuda.reduce_axes(v, axes, kind, op, div).as_slice()
        want = O.reduce_axes("f32", shape, x, 0, st, axes, kind, op, div)
        if op in (N.RMAX, N.RMIN):
            assert np.array_equal(got, want)
        else:
            assert np.all(np.abs(got - want) <= 1e-5 * 32 * (np.abs(want) + 1)), (kind, op)
    got = cuda.Cuda.arg_reduce(v, 1, N.RMAX).as_slice()
    assert np.array_equal(got, O.arg_reduce("f32", shape, x, 0, st, 1, N.RMAX))


def test_empty_and_degenerate_front_end(device):
    """tests/broadcast_reduce.rs:451-493: empty slices give the identity or
    NaN; one element has no sample variance."""
    empty = cuda.Tensor(cuda.CudaStorage("f32", 0), [2, 0, 3])
    assert np.array_equal(empty.sum_axes(1).to_numpy(), np.zeros([2, 3], np.float32))
    assert np.all(empty.max_axes(1, keep_dims=True).to_numpy() == -np.inf)
    assert np.all(empty.min_axes(1).to_numpy() == np.inf)
    assert np.all(np.isnan(empty.mean_axes(1).to_numpy()))
    assert empty.sum_axes(2).shape == [2, 0]
    single = cuda.Tensor.from_numpy(integral(3).reshape(3, 1), "f32")
    assert np.all(np.isnan(single.var_axes(1, sample=True).to_numpy()))
    assert np.array_equal(single.var_axes(1, sample=False).to_numpy(), np.zeros(3, np.float32))


@pytest.mark.parametrize("dtype", DTYPES)
def test_whole_vector_fold_and_dot(device, dtype):
    n = 100003
    x = O.narrow(integral(n), dtype)
    y = O.narrow(integral(n, 5), dtype)
    dx, dy = cuda.CudaStorage.store(x, dtype), cuda.CudaStorage.store(y, dtype)
    for op in (N.SUM, N.RMIN, N.RMAX):
        got = O.widen(cuda.Cuda.vector_reduce(dx, op).as_slice(), dtype)
        want = np.empty(1, x.dtype)
        O.call("orc_vector_reduce", O.DTYPES[dtype], op, O.ptr(x), n, O.ptr(want))
        assert np.array_equal(got, O.widen(want, dtype))
    got = O.widen(cuda.Cuda.dot(dx, dy).as_slice(), dtype)
    want = np.empty(1, x.dtype)
    O.call("orc_dot", O.DTYPES[dtype], O.ptr(x), O.ptr(y), n, O.ptr(want))
    assert np.array_equal(got, O.widen(want, dtype))


@pytest.mark.parametrize("dtype", DTYPES)
def test_streamed_reductions_of_long_runs(device, dtype):
    """Slices of contiguous runs, more than 8 MB in all, including the split
    shares merged for a fold over (0, 2)."""
    import ctypes as C
    shape = [64, 64, 1024]
    n = int(np.prod(shape))
    x = O.narrow(integral(n), dtype)
    st = cuda.contiguous_strides(shape)
    s = cuda.CudaStorage.store(x, dtype)
    v = cuda.TensorView(s, shape, st, 0)
    for kind, op, axes, div in [(N.AXIS_FOLD, N.SUM, [2], 0), (N.AXIS_MEAN, 0, [2], 0),
                                (N.AXIS_VARIANCE, 0, [2], 1023), (N.AXIS_FOLD, N.RMAX, [0, 2], 0),
                                (N.AXIS_FOLD, N.RMIN, [0, 2], 0), (N.AXIS_FOLD, N.SUM, [0, 2], 0)]:
        got = O.widen(cuda.Cuda.reduce_axes(v, axes, kind, op, div).as_slice(), dtype)
        want = O.widen(O.reduce_axes(dtype, shape, x, 0, st, axes, kind, op, div), dtype)
        if kind == N.AXIS_VARIANCE:
            assert np.all(np.abs(got - want) <= 1e-5 * 32 * (np.abs(want) + 1)), (kind, op, axes)
        else:
            assert np.array_equal(got, want), (kind, op, axes)
    for axis in (2, 1):
        got = cuda.Cuda.arg_reduce(v, axis, N.RMAX).as_slice()
        assert np.array_equal(got, O.arg_reduce(dtype, shape, x, 0, st, axis, N.RMAX))
    fault = C.c_int(0)
    N.call("tc_device_status", C.byref(fault))
    assert fault.value == 0


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("shape", [[3, 2049, 1028], [40, 300, 2048], [1, 7, 4096], [512, 4, 1024]])
def test_column_reductions_split_across_blocks(device, dtype, shape):
    """Folds over axis 1 with the results side by side (the columns path):
    every block streams an equal range of rows, so a tile's rows may be
    shared by several blocks whose partials merge in block order.  Ragged
    tiles (1028 columns) and short slices (7 rows) included; the integral
    filler makes every sum exact."""
    n = int(np.prod(shape))
    x = O.narrow(integral(n), dtype)
    st = cuda.contiguous_strides(shape)
    v = cuda.TensorView(cuda.CudaStorage.store(x, dtype), shape, st, 0)
    for kind, op in [(N.AXIS_FOLD, N.SUM), (N.AXIS_FOLD, N.RMIN), (N.AXIS_FOLD, N.RMAX), (N.AXIS_MEAN, 0)]:
        got = O.widen(cuda.Cuda.reduce_axes(v, [1], kind, op, 0).as_slice(), dtype)
        want = O.widen(O.reduce_axes(dtype, shape, x, 0, st, [1], kind, op, 0), dtype)
        assert np.array_equal(got, want), (kind, op)
    for op in (N.RMAX, N.RMIN):
        got = cuda.Cuda.arg_reduce(v, 1, op).as_slice()
        assert np.array_equal(got, O.arg_reduce(dtype, shape, x, 0, st, 1, op)), op


@pytest.mark.parametrize("dtype", DTYPES)
def test_column_arg_reductions_with_nans_ties_and_signed_zeros(device, dtype):
    """arg_reduce down the rows (the columns path): NaNs are passed over, a
    column of only NaNs answers 0, ties keep the first row, -0 and +0 tie,
    and infinities count (strided.rs:186-225)."""
    rows, cols = 700, 1024
    x = (integral(rows * cols) % 5).reshape(rows, cols)  # many ties
    x[::7, :] = np.nan
    x[:, 3] = np.nan                                      # all NaN
    x[:, 5] = 0.0
    x[1::2, 5] = -0.0                                     # signed zeros only
    x[:, 9] = -np.inf
    x[650:, 9] = np.nan
    x[:, 11] = np.inf
    x[:, 12] = np.nan
    x[699, 12] = -3.0                                     # the last row the only number
    x = O.narrow(x.reshape(-1), dtype)
    shape, st = [rows, cols], [cols, 1]
    v = cuda.TensorView(cuda.CudaStorage.store(x, dtype), shape, st, 0)
    for op in (N.RMAX, N.RMIN):
        got = cuda.Cuda.arg_reduce(v, 0, op).as_slice()
        assert np.array_equal(got, O.arg_reduce(dtype, shape, x, 0, st, 0, op)), op


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("shape,axes,offset_perm", [
    ([1 << 22], [0], None),            # one long slice: the split variance, the run-splitting sum
    ([100000, 3], [0], None),          # three long strided columns
    ([7, 8, 4096], [0, 2], None),      # eight slices, each 7 runs of 4096
    ([8, 4096, 6], [0, 1], [1, 2, 0]),  # a permuted view: 8 slices of 24576 over two folded axes
    ([3, 50001], [1], None),           # three contiguous slices, rows off the 16-byte boundary
])
def test_few_long_slices(device, dtype, shape, axes, offset_perm):
    """Few slices of 16384+ elements: the variance splits each slice into
    chunks over the whole machine (one pass merging the chunks' sums and
    squared deviations for contiguous slices, two passes otherwise) and a
    single long run's sum is split between warps; both against the oracle
    within the f32 sum bound (the integral filler makes folds and means
    exact)."""
    n = int(np.prod(shape))
    for fill, exact in ((integral(n), True), (normal(n, 17) + np.float32(3.0), False)):
        x = O.narrow(fill, dtype)
        strides = cuda.contiguous_strides(shape)
        view_shape = shape
        if offset_perm is not None:
            view_shape = [shape[a] for a in offset_perm]
            strides = [strides[a] for a in offset_perm]
        s = cuda.CudaStorage.store(x, dtype)
        view = cuda.TensorView(s, list(view_shape), list(strides), 0)
        depth = int(np.prod([view_shape[a] for a in axes]))
        for kind, op in ((N.AXIS_FOLD, N.SUM), (N.AXIS_MEAN, 0), (N.AXIS_VARIANCE, 0), (N.AXIS_FOLD, N.RMAX)):
            divisor = depth - 1 if kind == N.AXIS_VARIANCE else 0
            got = O.widen(cuda.Cuda.reduce_axes(view, axes, kind, op, divisor).as_slice(), dtype)
            want = O.widen(O.reduce_axes(dtype, view_shape, x, 0, strides, axes, kind, op, divisor), dtype)
            if (exact and kind != N.AXIS_VARIANCE) or op == N.RMAX:
                assert np.array_equal(got, want), (kind, op)
            else:
                half = 0 if dtype == "f32" else (2.0 ** -7 if dtype == "bf16" else 2.0 ** -10)
                scale = np.abs(want) + 1.0
                same_inf = np.isinf(got) & (got == want)  # f16 sums of millions overflow on both sides
                with np.errstate(invalid="ignore"):
                    close = np.abs(got - want) <= (1e-5 * np.sqrt(depth) + half) * scale
                assert np.all(same_inf | close), (kind, op)
