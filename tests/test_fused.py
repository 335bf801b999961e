"""Fused elementwise programs (Kernels::fused, kernels.rs:1077-1082; the
bytecode of fused/mod.rs:290-313) through tc_fused, against the oracle's
restatement of the Host interpreter (fused/mod.rs:4055-4260).  The oracle's
interpreter is pinned first against the oracle's own unfused kernels (the
Sgd and Adam programs, elementwise and broadcast programs) on the CPU."""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

import oracle as O
from tensorcrate_b200 import _native as N
from util import DTYPES, normal, uniform

I = N


def ins(code, dst=0, a=0, b=0, op=0, slot=0, value=0.0):
    x = N.Instr()
    x.code, x.dst, x.a, x.b, x.op, x.slot, x.value = code, dst, a, b, op, slot, value
    return x


def load(dst, slot):
    return ins(N.I_LOAD, dst=dst, slot=slot)


def const(dst, value):
    return ins(N.I_CONST, dst=dst, value=value)


def binary(dst, op, a, b):
    return ins(N.I_BINARY, dst=dst, a=a, b=b, op=op)


def unary(dst, op, a):
    return ins(N.I_UNARY, dst=dst, a=a, op=op)


def cmp(dst, op, a, b):
    return ins(N.I_CMP, dst=dst, a=a, b=b, op=op)


def store(src, slot):
    return ins(N.I_STORE, a=src, slot=slot)


def place(ptr, dtype, rows, cols, offset=0, col_step=1, row_step=None):
    """A place reading `rows` rows `row_step` apart (default: in order)."""
    p = N.Place()
    p.data, p.dtype, p.lead, p.offset, p.col_step = ptr, N.DTYPES[dtype], 1, offset, col_step
    p.dims[0], p.steps[0] = rows, cols if row_step is None else row_step
    return p


def run_oracle(dtype, rows, cols, code, places_host, outs_host, out_dtypes):
    """orc_fused over host arrays: places_host = [(array, dtype, offset, col_step, row_step)]."""
    pl = (N.Place * len(places_host))(*[place(a.ctypes.data, d, rows, cols, o, cs, rs)
                                         for a, d, o, cs, rs in places_host])
    code_arr = (N.Instr * len(code))(*code)
    outs = (C.c_void_p * len(outs_host))(*[o.ctypes.data for o in outs_host])
    dts = (C.c_int * len(out_dtypes))(*[N.DTYPES[d] for d in out_dtypes])
    O.call("orc_fused", O.DTYPES[dtype], rows, cols, C.cast(code_arr, C.c_void_p), len(code), C.cast(pl, C.c_void_p),
           len(places_host), C.cast(outs, C.c_void_p), C.cast(dts, C.c_void_p), len(outs_host))


def test_oracle_interpreter_matches_the_oracle_sgd_and_adam():
    """The oracle's interpreter, fed the programs Sgd and Adam build
    (optim.rs:773-787, 1048-1099), gives the oracle's optimizer results."""
    for dtype in DTYPES:
        n = 1000
        p0 = O.narrow(normal(n, 1), dtype)
        g = O.narrow(normal(n, 2) * 0.1, dtype)
        rate = float(O.widen(O.narrow(np.array([1e-2], np.float32), dtype), dtype)[0])
        want = p0.copy()
        O.call("orc_sgd", O.DTYPES[dtype], n, O.ptr(want), O.ptr(g), rate)
        got = np.empty_like(p0)
        code = [load(0, 0), load(1, 1), const(2, rate), binary(3, N.MUL, 1, 2), binary(4, N.SUB, 0, 3), store(4, 0)]
        run_oracle(dtype, 1, n, code, [(p0, dtype, 0, 1, n), (g, dtype, 0, 1, n)], [got], [dtype])
        assert np.array_equal(got, want)
        beta2 = 0.99 if dtype == "bf16" else 0.999
        coef = O.adam_coefficients(dtype, 1e-3, 0.9, beta2, 1e-8, 2)
        m0, v0 = O.narrow(normal(n, 3) * 0.01, dtype), O.narrow(np.abs(normal(n, 4)) * 1e-4, dtype)
        wp, wm, wv = p0.copy(), m0.copy(), v0.copy()
        O.call("orc_adam", O.DTYPES[dtype], n, O.ptr(wp), O.ptr(g), O.ptr(wm), O.ptr(wv), 1, *coef)
        outs = [np.empty_like(p0) for _ in range(3)]
        run_oracle(dtype, 1, n, adam_program(dtype, coef),
                   [(p0, dtype, 0, 1, n), (g, dtype, 0, 1, n), (m0, dtype, 0, 1, n), (v0, dtype, 0, 1, n)],
                   outs, [dtype] * 3)
        for got_x, want_x in zip(outs, (wp, wm, wv)):
            assert np.array_equal(got_x, want_x), dtype


def adam_program(dtype, coef):
    """Adam's resumed-step program in the order optim.rs:1048-1099 builds it."""
    rate, b1, b2, eps, c1, c2 = coef
    one = lambda x: float(O.widen(O.narrow(np.array([x], np.float32), dtype), dtype)[0])
    s1, s2 = one(1.0 - np.float32(b1)), one(1.0 - np.float32(b2))
    return [load(0, 0), load(1, 1), load(2, 2), load(3, 3),
            const(4, s1), binary(5, N.MUL, 1, 4),            # fresh_first = g*(1-b1)
            binary(6, N.MUL, 1, 1),                          # squared
            const(7, s2), binary(8, N.MUL, 6, 7),            # fresh_second
            const(9, b1), binary(10, N.MUL, 2, 9), binary(11, N.ADD, 10, 5),   # first
            const(9, b2), binary(10, N.MUL, 3, 9), binary(12, N.ADD, 10, 8),   # second
            const(9, c1), binary(13, N.MUL, 11, 9),          # first*c1
            const(9, c2), binary(14, N.MUL, 12, 9), unary(14, N.SQRT, 14),
            const(9, eps), binary(14, N.ADD, 14, 9), binary(13, N.DIV, 13, 14),
            const(9, rate), binary(13, N.MUL, 13, 9), binary(0, N.SUB, 0, 13),
            store(0, 0), store(11, 1), store(12, 2)]


def test_oracle_interpreter_matches_elementwise_and_broadcast():
    rows, cols = 7, 300
    for dtype in DTYPES:
        x = O.narrow(normal(rows * cols, 5), dtype)
        bias = O.narrow(normal(cols, 6), dtype)
        want = np.empty_like(x)
        O.call("orc_strided_binary", O.DTYPES[dtype], N.PAIR_ARITHMETIC, N.MUL, 2, O.sizes([rows, cols]), O.ptr(x),
               x.size, 0, O.sizes([cols, 1]), O.ptr(bias), bias.size, 0, O.sizes([0, 1]), O.ptr(want))
        got = np.empty_like(x)
        run_oracle(dtype, rows, cols, [load(0, 0), load(1, 1), binary(2, N.MUL, 0, 1), store(2, 0)],
                   [(x, dtype, 0, 1, cols), (bias, dtype, 0, 1, 0)], [got], [dtype])
        assert np.array_equal(got, want)


# ---------------------------------------------------------------------------
# GPU: tc_fused against the oracle
# ---------------------------------------------------------------------------
def run_gpu(dtype, rows, cols, code, places_dev, out_dev, out_dtypes):
    from tensorcrate_b200 import cuda
    pl = (N.Place * len(places_dev))(*[place(s.ptr, d, rows, cols, o, cs, rs) for s, d, o, cs, rs in places_dev])
    code_arr = (N.Instr * len(code))(*code)
    outs = (C.c_void_p * len(out_dev))(*[o.ptr for o in out_dev])
    dts = (C.c_int * len(out_dtypes))(*[N.DTYPES[d] for d in out_dtypes])
    N.call("tc_fused", N.DTYPES[dtype], rows, cols, code_arr, len(code), pl, len(places_dev), outs, dts,
           len(out_dev), None)
    cuda.synchronize()


def same_bits(a, b, dtype):
    wa, wb = O.widen(a, dtype), O.widen(b, dtype)
    return bool(np.all((a == b) | (np.isnan(wa) & np.isnan(wb))))


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", DTYPES)
def test_fused_programs_match_the_oracle(device, dtype):
    """Arithmetic, remainders, comparisons, min/max, a row-broadcast load, a
    permuted (transposed) load, a second storage type (an f32 input and an
    f32 output of a 16-bit program), square roots: bit for bit."""
    from tensorcrate_b200 import cuda
    rows, cols = 96, 130
    x = O.narrow(normal(rows * cols, 11), dtype)
    y = O.narrow(uniform(rows * cols, 12) * 3, dtype)
    bias = O.narrow(normal(cols, 13), dtype)
    xt = np.ascontiguousarray(x.reshape(rows, cols).T).reshape(-1)   # read back through a transposed place
    w32 = normal(rows * cols, 14)                                     # an f32 storage
    code = [load(0, 0), load(1, 1), load(2, 2), load(3, 3), load(4, 4),
            binary(5, N.ADD, 0, 2), binary(5, N.MUL, 5, 1), binary(6, N.DIV, 5, 1), binary(7, N.REM, 6, 1),
            cmp(8, N.GREATER, 0, 1), cmp(9, N.MAX, 7, 3), cmp(10, N.MAX_SHARE, 0, 4), cmp(11, N.MIN, 9, 4),
            binary(12, N.SUB, 3, 0),                                   # the transposed load equals x: exact zeros
            unary(13, N.SQRT, 1), const(14, 0.75), binary(13, N.MUL, 13, 14), binary(13, N.ADD, 13, 4),
            store(5, 0), store(7, 1), store(8, 2), store(11, 3), store(10, 4), store(12, 5), store(13, 6)]
    out_dtypes = [dtype, dtype, dtype, dtype, dtype, dtype, "f32"]
    host_places = [(x, dtype, 0, 1, cols), (y, dtype, 0, 1, cols), (bias, dtype, 0, 1, 0),
                   (xt, dtype, 0, rows, 1), (w32, "f32", 0, 1, cols)]
    want = [np.empty(rows * cols, O.STORE[d] if d != "f32" else np.float32) for d in out_dtypes]
    run_oracle(dtype, rows, cols, code, host_places, want, out_dtypes)
    dev_places = [(cuda.CudaStorage.store(a, d), d, o, cs, rs) for a, d, o, cs, rs in host_places]
    got = [cuda.CudaStorage(d, rows * cols) for d in out_dtypes]
    run_gpu(dtype, rows, cols, code, dev_places, got, out_dtypes)
    for k, (g, w, d) in enumerate(zip(got, want, out_dtypes)):
        assert same_bits(g.as_slice(), w, d), k


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", DTYPES)
def test_fused_adam_program_matches_the_adam_kernel(device, dtype):
    """Adam's program run by the interpreter gives the bits of tc_adam (the
    dedicated kernel).  Its results go to fresh outputs: written in place,
    tc_fused would recognise the update and run tc_adam itself."""
    from tensorcrate_b200 import cuda
    n = 5000
    beta2 = 0.99 if dtype == "bf16" else 0.999
    coef = O.adam_coefficients(dtype, 1e-3, 0.9, beta2, 1e-8, 2)
    p0 = O.narrow(normal(n, 21), dtype)
    g = O.narrow(normal(n, 22) * 0.1, dtype)
    m0, v0 = O.narrow(normal(n, 23) * 0.01, dtype), O.narrow(np.abs(normal(n, 24)) * 1e-4, dtype)
    a = {k: cuda.CudaStorage.store(v, dtype) for k, v in (("p", p0), ("g", g), ("m", m0), ("v", v0))}
    b = {k: cuda.CudaStorage.store(v, dtype) for k, v in (("p", p0), ("g", g), ("m", m0), ("v", v0))}
    N.call("tc_adam", N.DTYPES[dtype], n, a["p"].ptr, a["g"].ptr, a["m"].ptr, a["v"].ptr, 1, *coef, None)
    places = [(b[k], dtype, 0, 1, n) for k in ("p", "g", "m", "v")]
    fresh = {k: cuda.CudaStorage(dtype, n) for k in ("p", "m", "v")}
    run_gpu(dtype, 1, n, adam_program(dtype, coef), places, [fresh["p"], fresh["m"], fresh["v"]], [dtype] * 3)
    for k in ("p", "m", "v"):
        assert same_bits(a[k].as_slice(), fresh[k].as_slice(), dtype), k


@pytest.mark.gpu
def test_fused_transcendentals_within_two_ulp(device):
    """Unary Analytic functions of an f32 program: within 2 ulp of the
    exactly rounded value (f64), sec and csc within 3 (two roundings)."""
    from tensorcrate_b200 import cuda
    n = 4096
    x = uniform(n, 31).astype(np.float32) * 0.9
    funcs = [(N.SIN, np.sin), (N.COS, np.cos), (N.TAN, np.tan), (N.SEC, lambda v: 1 / np.cos(v)),
             (N.CSC, lambda v: 1 / np.sin(v)), (N.ARCSIN, np.arcsin), (N.ARCCOS, np.arccos),
             (N.ARCTAN, np.arctan), (N.EXP, np.exp), (N.LN, lambda v: np.log(np.abs(v) + 0.1)),
             (N.SINH, np.sinh), (N.COSH, np.cosh), (N.TANH, np.tanh), (N.SQRT, lambda v: np.sqrt(np.abs(v)))]
    xs = cuda.CudaStorage.store(x, "f32")
    absx = cuda.CudaStorage.store(np.abs(x) + np.float32(0.1), "f32")
    for op, f in funcs:
        src = absx if op == N.LN else xs
        arg = np.abs(x) + np.float32(0.1) if op == N.LN else x
        if op == N.SQRT:
            src, arg = cuda.CudaStorage.store(np.abs(x), "f32"), np.abs(x)
        out = cuda.CudaStorage("f32", n)
        run_gpu("f32", 1, n, [load(0, 0), unary(1, op, 0), store(1, 0)], [(src, "f32", 0, 1, n)], [out], ["f32"])
        got = out.as_slice().astype(np.float64)
        exact = (np.log(arg.astype(np.float64)) if op == N.LN else f(arg.astype(np.float64)))
        ulp = np.spacing(np.abs(exact).astype(np.float32)).astype(np.float64)
        limit = 0.0 if op == N.SQRT else (3.0 if op in (N.SEC, N.CSC) else 2.0)
        err = np.abs(got - exact) / ulp
        assert np.max(err) <= limit + 0.5, (op, float(np.max(err)))


# ---- row statistics, sums and row moments (kernels.rs:1090-1135) -----------

def layer_norm_program():
    """(x - mean) / sqrt(deviations * 0.5) of each row: the doc example of
    Builder::row_statistic (fused/mod.rs:1808-1827).  Place 0 is x, places
    1 and 2 its row mean and deviations."""
    return [load(0, 0), load(1, 1), load(2, 2), const(3, 0.5), binary(4, N.MUL, 2, 3), unary(5, N.SQRT, 4),
            binary(6, N.SUB, 0, 1), binary(7, N.DIV, 6, 5), store(7, 0)]


def _stats_places(ptr, dtype, rows, cols):
    x = place(ptr, dtype, rows, cols)
    blank = N.Place()
    return (N.Place * 3)(x, blank, blank)


STATS = (N.RowStatistic * 2)(N.RowStatistic(0, 1, N.ROW_MEAN), N.RowStatistic(0, 2, N.ROW_DEVIATIONS))


def _with_statistics_oracle(dtype, x, rows, cols, code):
    out = np.empty(rows * cols, x.dtype)
    pl = _stats_places(x.ctypes.data, dtype, rows, cols)
    code_arr = (N.Instr * len(code))(*code)
    outs = (C.c_void_p * 1)(out.ctypes.data)
    dts = (C.c_int * 1)(N.DTYPES[dtype])
    O.call("orc_fused_with_statistics", O.DTYPES[dtype], rows, cols, C.cast(code_arr, C.c_void_p), len(code),
           C.cast(pl, C.c_void_p), 3, C.cast(STATS, C.c_void_p), 2, C.cast(outs, C.c_void_p), C.cast(dts, C.c_void_p), 1)
    return out


def test_oracle_layer_norm_doc_example():
    """fused/mod.rs:1822-1826: [[1, 3], [10, 20]] normalizes to [[-1, 1], [-1, 1]]."""
    x = np.array([1.0, 3.0, 10.0, 20.0], np.float32)
    assert list(_with_statistics_oracle("f32", x, 2, 2, layer_norm_program())) == [-1.0, 1.0, -1.0, 1.0]


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("rows,cols", [(2, 2), (64, 1000), (1000, 64), (7, 1), (3, 4099), (37, 131), (3, 20001),
                                       (5, 4096)])
def test_fused_with_statistics_matches_the_oracle(device, dtype, rows, cols):
    """The row statistics are sums in another order (rel 1e-5·√cols), so
    the normalized values agree within that for f32, and within a step of
    the element type for f16/bf16; the 2x2 doc example is exact.  The
    shapes take each row width the kernel has (8 lanes, a warp or a block
    per row), with the row kept on chip (4096 and 4099 columns: more than
    48 KB of shared memory with the register file) and, at 20001 columns,
    read again from memory."""
    from tensorcrate_b200 import cuda
    x_host = np.array([1.0, 3.0, 10.0, 20.0], np.float32) if (rows, cols) == (2, 2) else normal(rows * cols, 12)
    x = O.narrow(x_host * np.float32(3.0) + np.float32(1.0) if (rows, cols) != (2, 2) else x_host, dtype)
    dx, out = cuda.CudaStorage.store(x, dtype), cuda.CudaStorage(dtype, rows * cols)
    code = layer_norm_program()
    code_arr = (N.Instr * len(code))(*code)
    pl = _stats_places(dx.ptr, dtype, rows, cols)
    outs = (C.c_void_p * 1)(out.ptr)
    dts = (C.c_int * 1)(N.DTYPES[dtype])
    N.call("tc_fused_with_statistics", N.DTYPES[dtype], rows, cols, C.cast(code_arr, C.c_void_p), len(code),
           C.cast(pl, C.c_void_p), 3, C.cast(STATS, C.c_void_p), 2, C.cast(outs, C.c_void_p),
           C.cast(dts, C.c_void_p), 1, None)
    want = _with_statistics_oracle(dtype, x, rows, cols, code)
    got = out.as_slice()
    if (rows, cols) == (2, 2):
        assert list(O.widen(got, dtype)) == [-1.0, 1.0, -1.0, 1.0]
    if cols == 1:
        # one element per row: zero deviation, 0/0
        assert np.all(np.isnan(O.widen(got, dtype)))
        return
    g, w = O.widen(got, dtype).astype(np.float64), O.widen(want, dtype).astype(np.float64)
    if dtype == "f32":
        assert np.all(np.abs(g - w) <= 1e-5 * np.sqrt(cols) * np.maximum(np.abs(w), 1.0))
    else:
        from util import steps
        assert int(np.max(steps(got, want, dtype))) <= 2


def sum_program():
    """x * y + 1: place 0 is x, place 1 is y."""
    return [load(0, 0), load(1, 1), binary(2, N.MUL, 0, 1), const(3, 1.0), binary(4, N.ADD, 2, 3), store(4, 0)]


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("rows,cols", [(100, 300), (3000, 7), (1, 5000), (5000, 1), (2048, 1024), (37, 1027)])
@pytest.mark.parametrize("axis", [N.ROWS, N.COLUMNS])
def test_fused_sum_matches_the_oracle(device, dtype, rows, cols, axis):
    """A program's output summed along an axis without being stored, against
    the Host's definition (the output, then matvec/vecmat with ones): sums in
    another order, rel 1e-5·√K, plus a step of the element type."""
    from tensorcrate_b200 import cuda
    n = rows * cols
    x, y = O.narrow(uniform(n, 13), dtype), O.narrow(uniform(n, 14), dtype)
    dx, dy = cuda.CudaStorage.store(x, dtype), cuda.CudaStorage.store(y, dtype)
    results = rows if axis == N.ROWS else cols
    out = cuda.CudaStorage(dtype, results)
    code = sum_program()
    code_arr = (N.Instr * len(code))(*code)
    pl = (N.Place * 2)(place(dx.ptr, dtype, rows, cols), place(dy.ptr, dtype, rows, cols))
    N.call("tc_fused_sum", N.DTYPES[dtype], rows, cols, C.cast(code_arr, C.c_void_p), len(code),
           C.cast(pl, C.c_void_p), 2, axis, out.ptr, None)
    want = np.empty(results, x.dtype)
    hpl = (N.Place * 2)(place(x.ctypes.data, dtype, rows, cols), place(y.ctypes.data, dtype, rows, cols))
    O.call("orc_fused_sum", O.DTYPES[dtype], rows, cols, C.cast(code_arr, C.c_void_p), len(code),
           C.cast(hpl, C.c_void_p), 2, axis, O.ptr(want))
    depth = cols if axis == N.ROWS else rows
    g, w = O.widen(out.as_slice(), dtype).astype(np.float64), O.widen(want, dtype).astype(np.float64)
    rel = 1e-5 * np.sqrt(depth) + (0 if dtype == "f32" else (2.0 ** -7 if dtype == "bf16" else 2.0 ** -10))
    assert np.all(np.abs(g - w) <= rel * np.maximum(np.abs(w), 1.0))


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("stored", ["f32", "bf16"])
def test_row_moments_through_a_transposing_place(device, dtype, stored):
    """row_moments of the transpose of a stored [cols x rows] matrix, read
    through a place (col_step = rows, row step 1), converting the storage
    type to the program's type first."""
    from tensorcrate_b200 import cuda
    rows, cols = 300, 517
    src = O.narrow(normal(rows * cols, 15) + np.float32(0.5), stored)
    dsrc = cuda.CudaStorage.store(src, stored)
    pl = place(dsrc.ptr, stored, rows, cols, col_step=rows, row_step=1)
    means, devs = cuda.CudaStorage(dtype, rows), cuda.CudaStorage(dtype, rows)
    N.call("tc_row_moments", N.DTYPES[dtype], C.byref(pl), rows, cols, means.ptr, devs.ptr, None)
    hpl = place(src.ctypes.data, stored, rows, cols, col_step=rows, row_step=1)
    store_t = np.float32 if dtype == "f32" else np.uint16
    wm, wd = np.empty(rows, store_t), np.empty(rows, store_t)
    O.call("orc_row_moments", O.DTYPES[dtype], C.byref(hpl), rows, cols, O.ptr(wm), O.ptr(wd))
    rel = 1e-5 * np.sqrt(cols) + (0 if dtype == "f32" else (2.0 ** -7 if dtype == "bf16" else 2.0 ** -10))
    for got, want in ((means, wm), (devs, wd)):
        g, w = O.widen(got.as_slice(), dtype).astype(np.float64), O.widen(want, dtype).astype(np.float64)
        assert np.all(np.abs(g - w) <= rel * np.maximum(np.abs(w), 1.0))


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("m,k,n", [(128, 256, 192), (33, 70, 17), (512, 1024, 768)])
def test_matmul_program_matches_the_oracle(device, dtype, m, k, n):
    """Kernels::matmul_epilogue with a program of its own: tanh(P) * 0.5 +
    bias[col], the product as input 0 and a per-column bias as input 1 (a
    place that repeats one row).  The product itself is a GEMM (half-
    precision tolerance for f16/bf16, the 3xTF32 bound for f32), which the
    program carries through."""
    from tensorcrate_b200 import cuda
    a, b = O.narrow(uniform(m * k, 21), dtype), O.narrow(uniform(k * n, 22), dtype)
    bias = O.narrow(uniform(n, 23), dtype)
    da, db, dbias = (cuda.CudaStorage.store(x, dtype) for x in (a, b, bias))
    out = cuda.CudaStorage(dtype, m * n)
    code = [load(0, 0), unary(1, N.TANH, 0), const(2, 0.5), binary(3, N.MUL, 1, 2), load(4, 1),
            binary(5, N.ADD, 3, 4), store(5, 0)]
    code_arr = (N.Instr * len(code))(*code)
    pl = (N.Place * 2)(place(None, dtype, m, n), place(dbias.ptr, dtype, m, n, row_step=0))
    outs = (C.c_void_p * 1)(out.ptr)
    dts = (C.c_int * 1)(N.DTYPES[dtype])
    N.call("tc_matmul_program", N.DTYPES[dtype], m, k, n, da.ptr, db.ptr, C.cast(code_arr, C.c_void_p), len(code),
           C.cast(pl, C.c_void_p), 2, C.cast(outs, C.c_void_p), C.cast(dts, C.c_void_p), 1, None)
    want = np.empty(m * n, a.dtype)
    hpl = (N.Place * 2)(place(None, dtype, m, n), place(bias.ctypes.data, dtype, m, n, row_step=0))
    houts = (C.c_void_p * 1)(want.ctypes.data)
    O.call("orc_matmul_program", O.DTYPES[dtype], m, k, n, O.ptr(a), O.ptr(b), C.cast(code_arr, C.c_void_p),
           len(code), C.cast(hpl, C.c_void_p), 2, C.cast(houts, C.c_void_p), C.cast(dts, C.c_void_p), 1)
    g, w = O.widen(out.as_slice(), dtype).astype(np.float64), O.widen(want, dtype).astype(np.float64)
    tol = 1e-5 * np.sqrt(k) if dtype == "f32" else (2.0 ** -6 if dtype == "bf16" else 2.0 ** -9)
    assert np.all(np.abs(g - w) <= tol * np.maximum(np.abs(w), 1.0))


def _through_the_file(code):
    """The same program with a constant into an otherwise unused register
    before every instruction: no instruction reads the one just before it,
    so every value travels through the interpreter's register file."""
    out = []
    for i in code:
        out += [const(15, 0.0), i]
    return out


FORWARDING = [load(0, 0), load(1, 1),
              binary(2, N.MUL, 1, 1),        # the next instruction's operands both forwarded; y read again later
              unary(3, N.EXP, 2),            # a transcendental: its operand must be in the file
              binary(4, N.ADD, 3, 0),        # its result read from the file, x from the file
              store(4, 0),                   # a forwarded store
              binary(0, N.SUB, 0, 1),        # after a store: nothing forwarded; a register overwritten by itself
              unary(5, N.SIN, 0),            # a transcendental of the value just made
              unary(5, N.COS, 5),            # and of its own result, in place
              binary(6, N.MUL, 5, 2),        # r2 from the file long after it was made
              cmp(6, N.MAX, 6, 6),           # both operands forwarded, written back to its own register
              unary(7, N.SQRT, 6),           # the root takes its operand forwarded
              binary(7, N.ADD, 7, 6),        # r7 forwarded, r6 (read again) from the file
              store(6, 1), store(7, 2)]


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", DTYPES)
def test_forwarded_values_match_the_register_file(device, dtype):
    """The interpreter keeps a result that only the next instruction reads in
    registers and writes the rest to its register file: the same program
    with every value forced through the file gives the same bits, through
    the flat kernel and both summing kernels (rows and columns)."""
    from tensorcrate_b200 import cuda
    rows, cols = 37, 203
    x = O.narrow(uniform(rows * cols, 31), dtype)
    y = O.narrow(uniform(rows * cols, 32), dtype)
    places = [(cuda.CudaStorage.store(x, dtype), dtype, 0, 1, cols), (cuda.CudaStorage.store(y, dtype), dtype, 0, 1, cols)]
    results = []
    for code in (FORWARDING, _through_the_file(FORWARDING)):
        outs = [cuda.CudaStorage(dtype, rows * cols) for _ in range(3)]
        run_gpu(dtype, rows, cols, code, places, outs, [dtype] * 3)
        results.append([o.as_slice() for o in outs])
    for k, (a, b) in enumerate(zip(*results)):
        assert same_bits(a, b, dtype), k
    one_store = FORWARDING[:5] + [binary(4, N.MUL, 4, 2), store(4, 0)]
    pl = (N.Place * 2)(*[place(s.ptr, d, rows, cols, o, cs, rs) for s, d, o, cs, rs in places])
    for axis, n in ((N.ROWS, rows), (N.COLUMNS, cols)):
        sums = []
        for code in (one_store, _through_the_file(one_store)):
            out = cuda.CudaStorage(dtype, n)
            code_arr = (N.Instr * len(code))(*code)
            N.call("tc_fused_sum", N.DTYPES[dtype], rows, cols, code_arr, len(code), pl, 2, axis, out.ptr, None)
            sums.append(out.as_slice())
        assert same_bits(sums[0], sums[1], dtype), axis


def test_oracle_runs_the_rules_programs_as_their_formulas():
    """The programs the optimizer tests build for Momentum, Nesterov, AdaGrad
    and RmsProp (optim.rs:826-846, 892-904, 948-964) compute the rules'
    formulas: the oracle's interpreter against numpy's f32 arithmetic in the
    same order (f32: every operation rounds once either way)."""
    from test_gpu_optim import _in, _rule_program
    n, f = 1000, np.float32
    p, g, s = normal(n, 61), normal(n, 62) * f(0.1), np.abs(normal(n, 63)) * f(0.01)
    rate = _in("f32", 0.01)
    for rule in ("momentum", "nesterov", "adagrad", "rmsprop"):
        c = _in("f32", 1e-8) if rule == "adagrad" else _in("f32", 0.9)
        code = _rule_program("momentum" if rule == "nesterov" else rule, "f32", rate, c, nesterov=rule == "nesterov")
        got_p, got_s = np.empty_like(p), np.empty_like(s)
        run_oracle("f32", 1, n, code, [(g, "f32", 0, 1, n), (p, "f32", 0, 1, n), (s, "f32", 0, 1, n)],
                   [got_p, got_s], ["f32", "f32"])
        k, r, eps = f(c), f(rate), f(_in("f32", 1e-8))
        if rule in ("momentum", "nesterov"):
            want_s = s * k + g
            step = want_s if rule == "momentum" else g + want_s * k
            want_p = p - step * r
        else:
            want_s = s + g * g if rule == "adagrad" else s * k + (g * g) * (f(1) - k)
            want_p = p - (g / (np.sqrt(want_s) + (k if rule == "adagrad" else eps))) * r
        assert np.array_equal(got_s, want_s.astype(f)), rule
        assert np.array_equal(got_p, want_p.astype(f)), rule
