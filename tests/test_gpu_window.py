"""The windowed matrix methods through the C ABI: correlate and its two
gradients (kernels.rs:998-1023; Host 1514-1573, 1720-1788), pad and flip
(kernels.rs:1025-1028; Host 1531-1542, 1575-1601), against the oracle.

Parity: a thread per output walks the taps in the Host's order with
rounded products and sums, so those results are the Host's bits; the
shared-output path (4096 taps or more, few outputs) is held to an f32 sum's
rounding; pad and flip move bits.  The worked examples of tests/conv.rs
run through the GPU as well."""
from __future__ import annotations

import numpy as np
import pytest

import oracle as O
from tensorcrate_b200 import _native as N
from tensorcrate_b200 import cuda
from util import DTYPES, kats, uniform

pytestmark = pytest.mark.gpu


def _store(x, dtype):
    return cuda.CudaStorage.store(x, dtype)


def correlate_gpu(x, w, shape, wshape, flip, dtype):
    (r, c), (wr, wc) = shape, wshape
    out = cuda.CudaStorage(dtype, (r - wr + 1) * (c - wc + 1))
    dx, dw = _store(x, dtype), _store(w, dtype)  # held until the result is read
    N.call("tc_correlate", N.DTYPES[dtype], r, c, wr, wc, int(flip), dx.ptr, dw.ptr, out.ptr, None)
    return out.as_slice()


def correlate_oracle(x, w, shape, wshape, flip, dtype):
    (r, c), (wr, wc) = shape, wshape
    out = np.empty((r - wr + 1) * (c - wc + 1), x.dtype)
    O.call("orc_correlate", O.DTYPES[dtype], r, c, wr, wc, int(flip), O.ptr(x), O.ptr(w), O.ptr(out))
    return out


@pytest.mark.parametrize("k", kats("correlate"), ids=lambda k: k["id"])
def test_correlate_worked_examples(device, k):
    x, w = np.array(k["input"], np.float32), np.array(k["window"], np.float32)
    got = correlate_gpu(x, w, k["shape"], k["window_shape"], k["flip"], "f32")
    assert list(got) == k["expect"]


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("shape,wshape", [((8, 9), (3, 2)), ((64, 100), (5, 7)), ((1, 1), (1, 1)),
                                          ((33, 257), (33, 1)), ((300, 40), (1, 40)), ((60, 60), (60, 60)),
                                          ((40, 136), (5, 5)), ((21, 203), (3, 8)), ((19, 64), (4, 6)),
                                          ((12, 40), (2, 9))])
@pytest.mark.parametrize("flip", [False, True])
def test_correlate_is_the_hosts_bits(device, dtype, shape, wshape, flip):
    x = O.narrow(uniform(shape[0] * shape[1], 1), dtype)
    w = O.narrow(uniform(wshape[0] * wshape[1], 2), dtype)
    got = correlate_gpu(x, w, shape, wshape, flip, dtype)
    want = correlate_oracle(x, w, shape, wshape, flip, dtype)
    assert np.array_equal(got, want)


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_correlate_with_more_taps_than_shared_memory_holds(device, dtype):
    """A 65x65 window (4225 taps, more than the 4096 staged in shared memory)
    over enough outputs (136 x 939) for the thread-per-outputs kernel, which
    then reads the taps through L1: still the Host's bits.  The output rows
    are not a multiple of the 8 outputs a thread takes."""
    shape, wshape = (200, 1003), (65, 65)
    x = O.narrow(uniform(shape[0] * shape[1], 11), dtype)
    w = O.narrow(uniform(wshape[0] * wshape[1], 12), dtype)
    assert np.array_equal(correlate_gpu(x, w, shape, wshape, False, dtype),
                          correlate_oracle(x, w, shape, wshape, False, dtype))


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("forward_flip", [False, True])
def test_correlate_input_gradient_with_more_taps_than_shared_memory_holds(device, dtype, forward_flip):
    """The input gradient through a 65x65 window (taps read through L1):
    the Host's bits, out-of-range taps skipped as the Host skips them."""
    (ar, ac), (wr, wc) = (70, 83), (65, 65)
    adj = O.narrow(uniform(ar * ac, 13), dtype)
    w = O.narrow(uniform(wr * wc, 14), dtype)
    rows, cols = ar + wr - 1, ac + wc - 1
    out = cuda.CudaStorage(dtype, rows * cols)
    dadj, dw = _store(adj, dtype), _store(w, dtype)
    N.call("tc_correlate_input_gradient", N.DTYPES[dtype], ar, ac, wr, wc, int(forward_flip), dadj.ptr, dw.ptr,
           out.ptr, None)
    want = np.empty(rows * cols, adj.dtype)
    O.call("orc_correlate_input_gradient", O.DTYPES[dtype], ar, ac, wr, wc, int(forward_flip), O.ptr(adj), O.ptr(w),
           O.ptr(want))
    assert np.array_equal(out.as_slice(), want)


@pytest.mark.parametrize("dtype", DTYPES)
def test_window_gradient_with_many_taps_within_sum_rounding(device, dtype):
    """The window gradient of a 300x300 input (a 298x298 adjoint, 88804
    taps per output): a block per output, a tree of partial sums."""
    r = c = 300
    ar = ac = 298
    x = O.narrow(uniform(r * c, 3), dtype)
    adj = O.narrow(uniform(ar * ac, 4), dtype)
    out = cuda.CudaStorage(dtype, 9)
    dx, dadj = _store(x, dtype), _store(adj, dtype)
    N.call("tc_correlate_window_gradient", N.DTYPES[dtype], r, c, ar, ac, dx.ptr, dadj.ptr, out.ptr, None)
    got = O.widen(out.as_slice(), dtype).astype(np.float64)
    want = O.widen(correlate_oracle(x, adj, (r, c), (ar, ac), False, dtype), dtype).astype(np.float64)
    xs, ads = O.widen(x, dtype).reshape(r, c), O.widen(adj, dtype).reshape(ar, ac)
    scale = np.array([np.sum(np.abs(xs[a:a + ar, b:b + ac] * ads)) for a in range(3) for b in range(3)])
    taps = ar * ac
    tol = 2.0 * np.sqrt(taps) * 2.0 ** -24 * scale * 8
    half = 0.0 if dtype == "f32" else (2.0 ** -7 if dtype == "bf16" else 2.0 ** -10) * np.abs(want)
    assert np.all(np.abs(got - want) <= tol + half)


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("ashape,wshape", [((30, 40), (3, 5)), ((2, 3), (5, 4)), ((17, 1), (1, 1)),
                                           ((64, 64), (7, 7)), ((50, 132), (5, 5)), ((19, 77), (3, 8)),
                                           ((33, 64), (2, 4)), ((9, 40), (3, 9))])
@pytest.mark.parametrize("forward_flip", [False, True])
def test_correlate_input_gradient_is_the_hosts_bits(device, dtype, ashape, wshape, forward_flip):
    (ar, ac), (wr, wc) = ashape, wshape
    adj = O.narrow(uniform(ar * ac, 5), dtype)
    w = O.narrow(uniform(wr * wc, 6), dtype)
    rows, cols = ar + wr - 1, ac + wc - 1
    out = cuda.CudaStorage(dtype, rows * cols)
    dadj, dw = _store(adj, dtype), _store(w, dtype)
    N.call("tc_correlate_input_gradient", N.DTYPES[dtype], ar, ac, wr, wc, int(forward_flip), dadj.ptr, dw.ptr,
           out.ptr, None)
    want = np.empty(rows * cols, adj.dtype)
    O.call("orc_correlate_input_gradient", O.DTYPES[dtype], ar, ac, wr, wc, int(forward_flip), O.ptr(adj), O.ptr(w),
           O.ptr(want))
    assert np.array_equal(out.as_slice(), want)


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("shape,pad", [((2, 2), (1, 1)), ((7, 5), (2, 3)), ((7, 5), (0, 0)), ((0, 4), (2, 1)),
                                       ((1000, 1000), (3, 9)), ((64, 256), (5, 8)), ((0, 16), (2, 8)),
                                       ((33, 1024), (0, 16))])
def test_pad_moves_bits(device, dtype, shape, pad):
    (r, c), (pr, pc) = shape, pad
    x = O.narrow(uniform(max(1, r * c), 7)[: r * c], dtype)
    out = cuda.CudaStorage(dtype, (r + 2 * pr) * (c + 2 * pc))
    src = _store(x, dtype) if r * c else None
    N.call("tc_pad", N.DTYPES[dtype], r, c, pr, pc, src.ptr if src else None, out.ptr, None)
    want = np.empty((r + 2 * pr) * (c + 2 * pc), x.dtype)
    O.call("orc_pad", O.DTYPES[dtype], r, c, pr, pc, O.ptr(x), O.ptr(want))
    assert np.array_equal(out.as_slice(), want)


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("shape", [(2, 2), (1, 1), (7, 5), (1000, 1001)])
def test_flip_moves_bits_and_is_an_involution(device, dtype, shape):
    r, c = shape
    x = O.narrow(uniform(r * c, 8), dtype)
    once = cuda.CudaStorage(dtype, r * c)
    dx = _store(x, dtype)
    N.call("tc_flip", N.DTYPES[dtype], r, c, dx.ptr, once.ptr, None)
    want = np.empty_like(x)
    O.call("orc_flip", O.DTYPES[dtype], r, c, O.ptr(x), O.ptr(want))
    assert np.array_equal(once.as_slice(), want)
    twice = cuda.CudaStorage(dtype, r * c)
    N.call("tc_flip", N.DTYPES[dtype], r, c, once.ptr, twice.ptr, None)
    assert np.array_equal(twice.as_slice(), x)


def test_correlate_rejects_a_window_that_does_not_fit(device):
    x = _store(np.zeros(6, np.float32), "f32")
    out = cuda.CudaStorage("f32", 1)
    assert N.lib().tc_correlate(N.F32, 2, 3, 3, 1, 0, x.ptr, x.ptr, out.ptr, None) == N.EINVAL


def test_trait_surface_matches_the_oracle(device):
    """The Cuda mirror of the trait methods (cuda.Cuda.correlate, pad, flip,
    the gradients, moments and distributions) on one small case each."""
    x = np.arange(20, dtype=np.float32).reshape(4, 5) / 7
    w = np.array([[1.0, -2.0], [0.5, 3.0]], np.float32)
    dx, dw = _store(x.ravel(), "f32"), _store(w.ravel(), "f32")
    got = cuda.Cuda.correlate(dx, (4, 5), dw, (2, 2), True).as_slice()
    assert np.array_equal(got, correlate_oracle(x.ravel(), w.ravel(), (4, 5), (2, 2), True, "f32"))
    adj = _store(np.ones(12, np.float32), "f32")
    gw = cuda.Cuda.correlate_window_gradient(dx, (4, 5), adj, (3, 4)).as_slice()
    assert np.array_equal(gw, correlate_oracle(x.ravel(), np.ones(12, np.float32), (4, 5), (3, 4), False, "f32"))
    gi = cuda.Cuda.correlate_input_gradient(adj, (3, 4), dw, (2, 2), False).as_slice()
    want = np.empty(20, np.float32)
    O.call("orc_correlate_input_gradient", O.DTYPES["f32"], 3, 4, 2, 2, 0, O.ptr(np.ones(12, np.float32)),
           O.ptr(w.ravel()), O.ptr(want))
    assert np.array_equal(gi, want)
    assert np.array_equal(cuda.Cuda.flip(dx, (4, 5)).as_slice(), x.ravel()[::-1])
    assert np.array_equal(cuda.Cuda.pad(dx, (4, 5), 1, 2).as_slice().reshape(6, 9), np.pad(x, ((1, 1), (2, 2))))
    m = cuda.Cuda.vector_moments(dx).as_slice()
    assert abs(m[0] - x.mean()) <= 1e-6 and abs(m[1] - ((x - x.mean()) ** 2).sum()) <= 1e-4
    means, devs = cuda.Cuda.matrix_axis_moments(dx, (4, 5), N.COLUMNS)
    assert np.allclose(means.as_slice(), x.mean(axis=0), atol=1e-6)
    cdf = cuda.Cuda.vector_distribution(dx, N.NORMAL, N.CDF, (1.0, 2.0)).as_slice()
    want = np.empty(20, np.float32)
    O.call("orc_distribution", O.DTYPES["f32"], N.NORMAL, N.CDF, O.ptr(x.ravel()), 20, 1.0, 2.0, O.ptr(want))
    assert np.array_equal(cdf, want)
