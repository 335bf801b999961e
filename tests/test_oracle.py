"""The oracle pinned: every known answer the reference's tests and docs state
for the hot path (tests/golden/reference_kats.json), plus the oracle's
agreement with plain numpy/f64 arithmetic where the reference's own test
strategy uses a naive index-arithmetic reference (tests/broadcast_reduce.rs:
1-3, tests/nd_tensor.rs:1-4).  CPU only."""
from __future__ import annotations

import itertools

import numpy as np
import pytest

import oracle as O
from util import DTYPES, expand, integral, kats, normal, same_floats, uniform

SUM, RMIN, RMAX = 0, 1, 2


def _input(k):
    vals = np.array(expand(k["input"]), dtype=np.float32)
    return O.narrow(vals, k["dtype"])


@pytest.mark.parametrize("k", kats("reduce"), ids=lambda k: k["id"])
def test_reduce_kats(k):
    x = _input(k)
    shape = k["shape"]
    strides = [int(np.prod(shape[a + 1:], dtype=np.int64)) for a in range(len(shape))]
    got = O.reduce_axes(k["dtype"], shape, x, 0, strides, k["axes"], k["reduction"], k["op"], k["divisor"])
    assert same_floats(O.widen(got, k["dtype"]), expand(k["expect"])), k["source"]


@pytest.mark.parametrize("k", kats("arg"), ids=lambda k: k["id"])
def test_arg_kats(k):
    x = _input(k)
    shape = k["shape"]
    strides = [int(np.prod(shape[a + 1:], dtype=np.int64)) for a in range(len(shape))]
    got = O.arg_reduce(k["dtype"], shape, x, 0, strides, k["axis"], k["op"])
    assert list(got) == k["expect"], k["source"]


@pytest.mark.parametrize("k", kats("walk"), ids=lambda k: k["id"])
def test_walk_kats(k):
    n = int(np.prod(k["shape"], dtype=np.int64)) if k["shape"] else 1
    out = np.zeros(max(n, 1), dtype=np.uint64)
    O.call("orc_walk", len(k["shape"]), O.sizes(k["shape"]), k["offset"], O.sizes(k["strides"]), O.ptr(out))
    assert list(out[: len(k["expect"])]) == k["expect"]
    if not k["expect"]:
        assert 0 in k["shape"]


@pytest.mark.parametrize("k", kats("coalesce"), ids=lambda k: k["id"])
def test_coalesce_kats(k):
    import ctypes as C
    rank = C.c_uint32()
    shape = (C.c_size_t * 6)()
    strides = (C.c_size_t * 18)()
    flat = [s for op in k["strides"] for s in op]
    O.call("orc_coalesce", len(k["shape"]), O.sizes(k["shape"]), len(k["strides"]), O.sizes(flat), C.byref(rank),
           shape, strides)
    assert list(shape[: rank.value]) == k["expect_shape"]
    assert [list(strides[o * rank.value:(o + 1) * rank.value]) for o in range(len(k["strides"]))] == \
        k["expect_strides"]


@pytest.mark.parametrize("k", kats("broadcast_shape"), ids=lambda k: k["id"])
def test_broadcast_shape_kats(k):
    import ctypes as C
    rank = C.c_uint32()
    out = (C.c_size_t * 6)()
    st = O.status("orc_broadcast_shape", len(k["left"]), O.sizes(k["left"]), len(k["right"]), O.sizes(k["right"]),
                  C.byref(rank), out)
    if k["expect"] is None:
        assert st != 0
    else:
        assert st == 0 and list(out[: rank.value]) == k["expect"]


@pytest.mark.parametrize("k", kats("broadcast_strides"), ids=lambda k: k["id"])
def test_broadcast_strides_kats(k):
    out = (O.C.c_size_t * 6)() if hasattr(O, "C") else None
    import ctypes as C
    out = (C.c_size_t * 6)()
    st = O.status("orc_broadcast_strides", len(k["shape"]), O.sizes(k["shape"]), O.sizes(k["strides"]),
                  len(k["target"]), O.sizes(k["target"]), out)
    if k["expect"] is None:
        assert st != 0
    else:
        assert st == 0 and list(out[: len(k["target"])]) == k["expect"]


@pytest.mark.parametrize("k", kats("reach"), ids=lambda k: k["id"])
def test_reach_kats(k):
    # reach decides whether a copy stays inside its storage: a source of
    # exactly `reach` elements is accepted and one fewer is refused.
    n = int(np.prod(k["shape"], dtype=np.int64)) if k["shape"] else 1
    src = np.zeros(max(k["expect"], 1), dtype=np.float32)
    dst = np.zeros(max(n, 1), dtype=np.float32)
    assert O.status("orc_strided_copy", 4, len(k["shape"]), O.sizes(k["shape"]), O.ptr(src), k["expect"],
                    k["offset"], O.sizes(k["strides"]), O.ptr(dst)) == 0
    if k["expect"] > 0:
        assert O.status("orc_strided_copy", 4, len(k["shape"]), O.sizes(k["shape"]), O.ptr(src), k["expect"] - 1,
                        k["offset"], O.sizes(k["strides"]), O.ptr(dst)) != 0


@pytest.mark.parametrize("k", kats("strided_copy"), ids=lambda k: k["id"])
def test_strided_copy_kats(k):
    src = np.array(k["input"], dtype=np.uint32)
    got = O.strided_copy(src, k["shape"], k["offset"], k["strides"])
    assert list(got) == k["expect"]


@pytest.mark.parametrize("k", kats("assemble"), ids=lambda k: k["id"])
def test_assemble_kats(k):
    import ctypes as C
    from tensorcrate_b200._native import Region
    src = np.array(k["input"], dtype=np.uint32)
    regs = (Region * len(k["regions"]))()
    for r, d in zip(regs, k["regions"]):
        r.source, r.source_len, r.rank = src.ctypes.data, src.size, len(d["shape"])
        for a in range(len(d["shape"])):
            r.shape[a], r.from_strides[a], r.to_strides[a] = d["shape"][a], d["from_strides"][a], d["to_strides"][a]
        r.from_offset, r.to_offset = d["from_offset"], d["to_offset"]
    out = np.zeros(k["length"], dtype=np.uint32)
    O.call("orc_assemble", 4, O.ptr(out), k["length"], C.addressof(regs), len(k["regions"]))
    assert list(out) == k["expect"]


@pytest.mark.parametrize("k", kats("elementwise"), ids=lambda k: k["id"])
def test_elementwise_kats(k):
    a, b = O.narrow(expand(k["a"]), k["dtype"]), O.narrow(expand(k["b"]), k["dtype"])
    out = np.empty_like(a)
    O.call("orc_elementwise", O.DTYPES[k["dtype"]], k["op"], O.ptr(a), O.ptr(b), O.ptr(out), a.size)
    assert same_floats(O.widen(out, k["dtype"]), expand(k["expect"]))


@pytest.mark.parametrize("k", kats("prefix_sum"), ids=lambda k: k["id"])
def test_prefix_sum_kats(k):
    a = O.narrow(expand(k["input"]), k["dtype"])
    out = np.empty_like(a)
    O.call("orc_prefix_sum", O.DTYPES[k["dtype"]], O.ptr(a), O.ptr(out), a.size)
    assert same_floats(O.widen(out, k["dtype"]), expand(k["expect"]))


@pytest.mark.parametrize("k", kats("sort"), ids=lambda k: k["id"])
def test_sort_kats(k):
    if k["input_bits"] is not None:
        a = np.array(k["input_bits"], np.uint32).view(np.float32)
    else:
        a = O.narrow(expand(k["input"]), k["dtype"])
    out = np.empty_like(a)
    O.call("orc_sort", O.DTYPES[k["dtype"]], k["order"], O.ptr(a), O.ptr(out), a.size)
    if "expect_bits" in k:
        bits = out.view(np.uint32)
        for i, want in k["expect_bits"].items():
            assert int(bits[int(i)]) == want, i
    else:
        assert same_floats(O.widen(out, k["dtype"]), expand(k["expect"]))


def test_sort_matches_numpy_on_distinct_values():
    """Away from NaNs and signed zeros the total order is the numeric one."""
    a = normal(10000, 5)
    for order in (0, 1):
        out = np.empty_like(a)
        O.call("orc_sort", O.DTYPES["f32"], order, O.ptr(a), O.ptr(out), a.size)
        want = np.sort(a) if order == 0 else np.sort(a)[::-1]
        assert np.array_equal(out, want)


def test_prefix_sum_of_the_integral_filler_is_exact():
    a = integral(100000)
    out = np.empty_like(a)
    O.call("orc_prefix_sum", O.DTYPES["f32"], O.ptr(a), O.ptr(out), a.size)
    assert np.array_equal(out, np.cumsum(a.astype(np.float64)).astype(np.float32))


@pytest.mark.parametrize("k", kats("correlate"), ids=lambda k: k["id"])
def test_correlate_kats(k):
    x, w = np.array(k["input"], np.float32), np.array(k["window"], np.float32)
    (r, c), (wr, wc) = k["shape"], k["window_shape"]
    out = np.empty((r - wr + 1) * (c - wc + 1), np.float32)
    O.call("orc_correlate", O.DTYPES["f32"], r, c, wr, wc, k["flip"], O.ptr(x), O.ptr(w), O.ptr(out))
    assert list(out) == k["expect"]


@pytest.mark.parametrize("k", kats("pad") + kats("flip"), ids=lambda k: k["id"])
def test_pad_and_flip_kats(k):
    x = np.array(k["input"], np.float32)
    r, c = k["shape"]
    if k["kind"] == "pad":
        pr, pc = k["pad"]
        out = np.empty((r + 2 * pr) * (c + 2 * pc), np.float32)
        O.call("orc_pad", O.DTYPES["f32"], r, c, pr, pc, O.ptr(x), O.ptr(out))
    else:
        out = np.empty(r * c, np.float32)
        O.call("orc_flip", O.DTYPES["f32"], r, c, O.ptr(x), O.ptr(out))
    assert list(out) == list(map(float, k["expect"]))


def test_convolution_is_correlation_with_the_window_flipped():
    """tests/conv.rs:118-126."""
    x, w = uniform(4 * 5, 3), uniform(2 * 3, 4)
    conv, flipped, corr = np.empty(3 * 3, np.float32), np.empty(6, np.float32), np.empty(3 * 3, np.float32)
    O.call("orc_correlate", O.DTYPES["f32"], 4, 5, 2, 3, 1, O.ptr(x), O.ptr(w), O.ptr(conv))
    O.call("orc_flip", O.DTYPES["f32"], 2, 3, O.ptr(w), O.ptr(flipped))
    O.call("orc_correlate", O.DTYPES["f32"], 4, 5, 2, 3, 0, O.ptr(x), O.ptr(flipped), O.ptr(corr))
    assert np.array_equal(conv, corr)


def test_correlate_gradients_match_numpy():
    """The window gradient is the input correlated with the adjoint, and the
    input gradient the full correlation: both against f64 numpy sums."""
    x, w, adj = uniform((6, 7), 5), uniform((3, 2), 6), uniform((4, 6), 7)
    got = np.empty((6, 7), np.float32)
    O.call("orc_correlate_input_gradient", O.DTYPES["f32"], 4, 6, 3, 2, 0, O.ptr(adj), O.ptr(w), O.ptr(got))
    want = np.zeros((6, 7))
    for i in range(4):
        for j in range(6):
            want[i:i + 3, j:j + 2] += adj[i, j] * w.astype(np.float64)
    assert np.allclose(got, want, atol=1e-5)
    gw = np.empty((3, 2), np.float32)
    O.call("orc_correlate", O.DTYPES["f32"], 6, 7, 4, 6, 0, O.ptr(x), O.ptr(adj), O.ptr(gw))
    want_w = np.array([[np.sum(x[a:a + 4, b:b + 6].astype(np.float64) * adj) for b in range(2)] for a in range(3)])
    assert np.allclose(gw, want_w, atol=1e-5)


@pytest.mark.parametrize("k", kats("moments"), ids=lambda k: k["id"])
def test_moments_kats(k):
    a = np.array(expand(k["input"]), np.float32)
    out = np.empty(2, np.float32)
    O.call("orc_moments", O.DTYPES["f32"], O.ptr(a), a.size, O.ptr(out))
    assert same_floats(out, expand(k["expect"]))


@pytest.mark.parametrize("k", kats("axis_moments"), ids=lambda k: k["id"])
def test_axis_moments_kats(k):
    a = np.array(k["input"], np.float32)
    r, c = k["shape"]
    extent = r if k["axis"] == 0 else c
    means, devs = np.empty(extent, np.float32), np.empty(extent, np.float32)
    O.call("orc_axis_moments", O.DTYPES["f32"], r, c, k["axis"], O.ptr(a), O.ptr(means), O.ptr(devs))
    want = k.get("expect_means") or [np.float32(v) for v in k["expect_means_f64"]]
    assert list(means) == list(np.array(want, np.float32))


@pytest.mark.parametrize("k", kats("distribution"), ids=lambda k: k["id"])
def test_distribution_kats(k):
    """In f64, as tests/statistics.rs checks them: within 1e-14 relative
    (max(|want|, 1)) of the published value, or the stated tolerance."""
    got = O.lib().orc_evaluate_f64(k["family"], k["statistic"], _value_of(k["x"]), k["params"][0], k["params"][1])
    want = _value_of(k["expect_f64"])
    if np.isnan(want) or np.isinf(want):
        assert (np.isnan(got) and np.isnan(want)) or got == want
    else:
        assert abs(got - want) <= k.get("tol", 1e-14) * max(abs(want), 1.0)


def test_distribution_rounds_the_f64_value_once():
    """The f32/f16/bf16 results are the f64 value rounded once, to nearest."""
    x = np.array([0.5, 0.95, 0.975, 0.99, 0.001, 0.999, 0.3, 0.7], np.float32)
    for dtype in ("f32", "f16", "bf16"):
        xs = O.narrow(x, dtype)
        out = np.empty_like(xs)
        O.call("orc_distribution", O.DTYPES[dtype], 0, 2, O.ptr(xs), xs.size, 0.0, 1.0, O.ptr(out))
        exact = np.array([O.lib().orc_evaluate_f64(0, 2, float(v), 0.0, 1.0) for v in O.widen(xs, dtype)])
        if dtype == "f32":
            assert np.array_equal(out, exact.astype(np.float32))
        elif dtype == "f16":
            assert np.array_equal(out.view(np.float16), exact.astype(np.float16))
        else:
            got = O.widen(out, dtype).astype(np.float64)
            assert np.array_equal(np.isinf(got), np.isinf(exact))
            nz = (got != 0) & np.isfinite(got)
            ulp = np.exp2(np.floor(np.log2(np.abs(got[nz]))) - 7)
            assert np.all(np.abs(got[nz] - exact[nz]) <= 0.5 * ulp)


def test_normal_quantile_inverts_the_cdf():
    """tests/statistics.rs:120-143: cdf(ppf(p)) = p within 1e-13 across the
    interval and 1e-12 far into the tail."""
    ev = O.lib().orc_evaluate_f64
    for i in range(1, 10000, 7):
        p = i / 10000.0
        assert abs(ev(0, 1, ev(0, 2, p, 0.0, 1.0), 0.0, 1.0) - p) <= 1e-13 * max(p, 1.0)
    for p in (1e-300, 1e-100, 1e-20, 1e-8, 1e-3):
        assert abs(ev(0, 1, ev(0, 2, p, 0.0, 1.0), 0.0, 1.0) - p) <= 1e-12 * max(p, 1.0)


def test_inverse_gaussian_quantile_inverts_its_cdf():
    """tests/statistics.rs:146-165: the solved quantile round-trips within
    1e-12 for the reference's five parameter pairs."""
    ev = O.lib().orc_evaluate_f64
    for mean, shape in ((1.0, 1.0), (1.0, 3.0), (2.0, 0.5), (0.5, 20.0), (1.0, 100.0)):
        for i in range(1, 500, 3):
            p = i / 500.0
            x = ev(1, 2, p, mean, shape)
            assert abs(ev(1, 1, x, mean, shape) - p) <= 1e-12 * max(p, 1.0), (mean, shape, p)


def _value_of(v):
    return expand([v])[0]


def test_sgd_kat():
    (k,) = kats("sgd")
    p, g = np.array(k["p"], np.float32), np.array(k["g"], np.float32)
    O.call("orc_sgd", 0, 2, O.ptr(p), O.ptr(g), k["rate"])
    want = [np.float32(1.0) - np.float32(0.05), np.float32(-2.0) - np.float32(0.4)]
    assert list(p) == want


@pytest.mark.parametrize("k", kats("adam_first"), ids=lambda k: k["id"])
def test_adam_first_step_kat(k):
    coef = O.adam_coefficients("f32", k["rate"], 0.9, 0.999, 1e-8, 1)
    p, g = np.array(k["p"], np.float32), np.array(k["g"], np.float32)
    m, v = np.zeros_like(p), np.zeros_like(p)
    O.call("orc_adam", 0, 1, O.ptr(p), O.ptr(g), O.ptr(m), O.ptr(v), 0, *coef)
    assert abs(p[0] - k["expect"][0]) <= k["tol"]


def test_bf16_adam_default_beta2_rounds_to_one():
    """Real::from_f64(0.999) in bf16 is 1.0, so Adam's second correction is
    1/(1 - 1) = inf and the reference's bf16 update is NaN (optim.rs:1029-1035,
    1110-1124).  The oracle reproduces it."""
    coef = O.adam_coefficients("bf16", 1e-3, 0.9, 0.999, 1e-8, 1)
    assert coef[2] == 1.0 and np.isinf(coef[5])
    p = O.narrow(np.array([0.5], np.float32), "bf16")
    g = O.narrow(np.array([0.25], np.float32), "bf16")
    m, v = np.zeros_like(p), np.zeros_like(p)
    O.call("orc_adam", 2, 1, O.ptr(p), O.ptr(g), O.ptr(m), O.ptr(v), 0, *coef)
    assert np.isnan(O.widen(p, "bf16")[0])


# --- the oracle against naive index arithmetic --------------------------------
def _numpy_view(x, shape, offset, strides):
    idx = offset + sum(np.arange(e).reshape([-1 if a == d else 1 for d in range(len(shape))]) * s
                       for a, (e, s) in enumerate(zip(shape, strides)))
    return x[idx] if shape else x[offset:offset + 1].reshape(())


@pytest.mark.parametrize("perm", [(2, 0, 3, 1), (0, 3, 1, 2), (3, 2, 1, 0)])
def test_strided_copy_matches_index_arithmetic(perm):
    shape = [2, 3, 4, 5]
    x = integral(120)
    strides = [60, 20, 5, 1]
    pshape, pstrides = [shape[a] for a in perm], [strides[a] for a in perm]
    got = O.strided_copy(x, pshape, 0, pstrides)
    want = np.transpose(x.reshape(shape), perm).reshape(-1)
    assert np.array_equal(got, want)


@pytest.mark.parametrize("dtype", DTYPES)
def test_reductions_over_every_subset_match_f64(dtype):
    """tests/broadcast_reduce.rs:388-400: every subset of axes, integral
    filler, so sums are exact."""
    shape = [2, 3, 4, 5]
    x = O.narrow(integral(120), dtype)
    xf = O.widen(x, dtype).reshape(shape).astype(np.float64)
    strides = [60, 20, 5, 1]
    for r in range(1, 5):
        for axes in itertools.combinations(range(4), r):
            axes = list(axes)
            got = O.widen(O.reduce_axes(dtype, shape, x, 0, strides, axes, 0, SUM, 0), dtype)
            want = xf.sum(axis=tuple(axes)).reshape(-1)
            assert np.array_equal(got, O.widen(O.narrow(want, dtype), dtype))
            got = O.widen(O.reduce_axes(dtype, shape, x, 0, strides, axes, 0, RMAX, 0), dtype)
            assert np.array_equal(got, xf.max(axis=tuple(axes)).reshape(-1))


def test_matmul_matches_f64_within_tolerance():
    rng = np.random.default_rng(0)
    for m, k, n in [(1, 1, 1), (3, 5, 7), (33, 17, 9), (96, 96, 96), (8, 64, 13)]:
        a = rng.uniform(-1, 1, (m, k)).astype(np.float32)
        b = rng.uniform(-1, 1, (k, n)).astype(np.float32)
        got = O.matmul("f32", 0, m, k, n, a, b).reshape(m, n)
        want = a.astype(np.float64) @ b.astype(np.float64)
        assert np.max(np.abs(got - want)) <= 1e-5 * np.sqrt(k) * max(1.0, np.max(np.abs(want)))


def test_bf16_matmul_rounds_once():
    """compact::matmul (src/compact.rs:232-253): widen, f32 product, round once."""
    rng = np.random.default_rng(1)
    m, k, n = 16, 32, 24
    a = O.narrow(rng.uniform(-1, 1, (m, k)), "bf16")
    b = O.narrow(rng.uniform(-1, 1, (k, n)), "bf16")
    got = O.widen(O.matmul("bf16", 0, m, k, n, a, b), "bf16").reshape(m, n)
    exact = O.widen(a, "bf16").reshape(m, k).astype(np.float64) @ O.widen(b, "bf16").reshape(k, n).astype(np.float64)
    assert np.max(np.abs(got - exact)) <= 2 ** -8 * np.max(np.abs(exact)) + 1e-6


def test_transposed_products_equal_explicit_transpose():
    rng = np.random.default_rng(2)
    m, k, n = 7, 9, 11
    a = rng.uniform(-1, 1, (k, m)).astype(np.float32)
    b = rng.uniform(-1, 1, (k, n)).astype(np.float32)
    left = O.matmul("f32", 1, m, k, n, a, b)
    plain = O.matmul("f32", 0, m, k, n, np.ascontiguousarray(a.T), b)
    assert np.array_equal(left, plain)
    bt = rng.uniform(-1, 1, (n, k)).astype(np.float32)
    a2 = rng.uniform(-1, 1, (m, k)).astype(np.float32)
    right = O.matmul("f32", 2, m, k, n, a2, bt)
    assert np.array_equal(right, O.matmul("f32", 0, m, k, n, a2, np.ascontiguousarray(bt.T)))


def test_f16_conversion_matches_numpy_for_finite_values():
    x = normal(100000, 7) * np.float32(300.0)
    x = np.concatenate([x, np.array([65504, 65520, 1e-8, 6e-8, -3e-5, 0.0, -0.0], np.float32)])
    assert np.array_equal(O.narrow(x, "f16"), x.astype(np.float16).view(np.uint16))


def test_bf16_conversion_is_nearest_even():
    u = np.array([0x3F808000, 0x3F818000, 0x3F80C000, 0x3F804000, 0x7F7FFFFF, 0x7FC00001], np.uint32)
    got = O.narrow(u.view(np.float32), "bf16")
    assert list(got) == [0x3F80, 0x3F82, 0x3F81, 0x3F80, 0x7F80, 0x7FC0]


def test_strided_binary_matches_numpy_broadcast():
    shape = [4, 3, 5]
    x = uniform(shape, 3)
    bias = uniform([5], 4)
    got = O.strided_binary("f32", 0, 0, shape, x.reshape(-1), 0, [15, 5, 1], bias, 0, [0, 0, 1])
    assert np.array_equal(got, (x + bias).reshape(-1))
