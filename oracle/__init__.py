"""ctypes binding of the oracle (oracle/_build/liboracle.so).

TEST INFRASTRUCTURE ONLY: the CPU restatement of tensorcrate's Host backend
that the CUDA backend is checked against, and the timed CPU baseline.  Only
tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg import it;
the product never does.  See oracle/oracle.h for what each function
restates.
"""
from __future__ import annotations

import ctypes as C
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "_build" / "liboracle.so"

_sz, _p, _i, _u32, _d = C.c_size_t, C.c_void_p, C.c_int, C.c_uint32, C.c_double
_szp, _u32p = C.POINTER(C.c_size_t), C.POINTER(C.c_uint32)

SIGNATURES = {
    "orc_coalesce": [_u32, _szp, _u32, _szp, _u32p, _szp, _szp],
    "orc_broadcast_shape": [_u32, _szp, _u32, _szp, _u32p, _szp],
    "orc_broadcast_strides": [_u32, _szp, _szp, _u32, _szp, _szp],
    "orc_walk": [_u32, _szp, _sz, _szp, _p],
    "orc_strided_copy": [_sz, _u32, _szp, _p, _sz, _sz, _szp, _p],
    "orc_strided_write": [_sz, _p, _sz, _p],
    "orc_assemble": [_sz, _p, _sz, _p, _sz],
    "orc_elementwise": [_i, _i, _p, _p, _p, _sz],
    "orc_broadcast_scalar": [_i, _i, _p, _d, _i, _p, _sz],
    "orc_compare": [_i, _i, _p, _p, _p, _sz],
    "orc_compare_scalar": [_i, _i, _p, _d, _i, _p, _sz],
    "orc_clamp": [_i, _p, _d, _d, _p, _sz],
    "orc_vector_reduce": [_i, _i, _p, _sz, _p],
    "orc_dot": [_i, _p, _p, _sz, _p],
    "orc_strided_binary": [_i, _i, _i, _u32, _szp, _p, _sz, _sz, _szp, _p, _sz, _sz, _szp, _p],
    "orc_reduce_axes": [_i, _u32, _szp, _p, _sz, _sz, _szp, _u32, _u32p, _i, _i, _sz, _p],
    "orc_arg_reduce": [_i, _u32, _szp, _p, _sz, _sz, _szp, _u32, _i, _u32p],
    "orc_matmul": [_i, _i, _sz, _sz, _sz, _p, _p, _p, _i],
    "orc_matmul_rows": [_i, _sz, _sz, _sz, _p, _p, _p, _i, _sz, _sz],
    "orc_matvec": [_i, _sz, _sz, _p, _p, _p, _i],
    "orc_vecmat": [_i, _sz, _sz, _p, _p, _p],
    "orc_transpose": [_i, _sz, _sz, _p, _p],
    "orc_adam": [_i, _sz, _p, _p, _p, _p, _i, _d, _d, _d, _d, _d, _d],
    "orc_sgd": [_i, _sz, _p, _p, _d],
    "orc_fused": [_i, _sz, _sz, _p, _u32, _p, _u32, _p, _p, _u32],
    "orc_unary": [_i, _i, _p, _p, _sz],
    "orc_unary_dual": [_i, _i, _p, _p, _p, _p, _sz],
    "orc_prefix_sum": [_i, _p, _p, _sz],
    "orc_sort": [_i, _i, _p, _p, _sz],
    "orc_power": [_i, _p, _p, _p, _sz],
    "orc_power_scalar": [_i, _p, _d, _i, _p, _sz],
    "orc_correlate": [_i, _sz, _sz, _sz, _sz, _i, _p, _p, _p],
    "orc_correlate_input_gradient": [_i, _sz, _sz, _sz, _sz, _i, _p, _p, _p],
    "orc_pad": [_i, _sz, _sz, _sz, _sz, _p, _p],
    "orc_flip": [_i, _sz, _sz, _p, _p],
    "orc_moments": [_i, _p, _sz, _p],
    "orc_axis_moments": [_i, _sz, _sz, _i, _p, _p, _p],
    "orc_distribution": [_i, _i, _i, _p, _sz, _d, _d, _p],
    "orc_axis_distribution": [_i, _sz, _sz, _i, _i, _i, _p, _p, _p, _p],
    "orc_row_moments": [_i, _p, _sz, _sz, _p, _p],
    "orc_fused_with_statistics": [_i, _sz, _sz, _p, _u32, _p, _u32, _p, _u32, _p, _p, _u32],
    "orc_fused_sum": [_i, _sz, _sz, _p, _u32, _p, _u32, _i, _p],
    "orc_matmul_program": [_i, _sz, _sz, _sz, _p, _p, _p, _u32, _p, _u32, _p, _p, _u32],
    "orc_adam_coefficients": [_i, _d, _d, _d, _d, _u32, C.POINTER(C.c_double)],
    "orc_mlp_params": [_p, _u32, _p, _p, _i],
    "orc_mlp_grads": [_p, _u32, _p, _p],
    "orc_mlp_step": [_p, _p, _p, _p, _i],
}

DTYPES = {"f32": 0, "f16": 1, "bf16": 2}
STORE = {"f32": np.float32, "f16": np.uint16, "bf16": np.uint16, "u32": np.uint32}

_lib = None


def build() -> Path:
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    return LIB_PATH


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        sources = [HERE / "oracle.cpp", HERE / "oracle.h", HERE / "Makefile"]
        if not LIB_PATH.exists() or any(f.stat().st_mtime > LIB_PATH.stat().st_mtime for f in sources if f.exists()):
            build()
        h = C.CDLL(str(LIB_PATH))
        for name, args in SIGNATURES.items():
            fn = getattr(h, name)
            fn.argtypes, fn.restype = args, C.c_int
        h.orc_narrow.argtypes = [_i, _p, _p, _sz]
        h.orc_narrow.restype = None
        h.orc_widen.argtypes = [_i, _p, _p, _sz]
        h.orc_widen.restype = None
        h.orc_mlp_create.argtypes = [_i, _u32, _u32p, _u32, _u32, _d, _d, _d, _d]
        h.orc_mlp_create.restype = _p
        h.orc_mlp_destroy.argtypes = [_p]
        h.orc_mlp_destroy.restype = None
        h.orc_evaluate_f64.argtypes = [_i, _i, _d, _d, _d]
        h.orc_evaluate_f64.restype = _d
        h.orc_set_threads.argtypes = [_i]
        h.orc_set_threads.restype = None
        h.orc_set_matmul_threads.argtypes = [_i]
        h.orc_set_matmul_threads.restype = None
        _lib = h
    return _lib


def call(name: str, *args) -> None:
    st = getattr(lib(), name)(*args)
    if st != 0:
        raise RuntimeError(f"{name} failed with status {st}")


def status(name: str, *args) -> int:
    return getattr(lib(), name)(*args)


def sizes(values):
    values = [int(v) for v in values]
    return (_sz * max(1, len(values)))(*values)


def u32s(values):
    values = [int(v) for v in values]
    return (_u32 * max(1, len(values)))(*values)


def ptr(a: np.ndarray) -> C.c_void_p:
    """The array's address as a ctypes pointer that keeps the array alive
    while the pointer lives (a bare integer would let a temporary array be
    freed before the call reads it)."""
    return a.ctypes.data_as(C.c_void_p)


def narrow(values, dtype: str) -> np.ndarray:
    """f32 -> storage of `dtype`, rounded as crate half rounds."""
    x = np.ascontiguousarray(values, dtype=np.float32)
    if dtype == "f32":
        return x.copy()
    out = np.empty(x.shape, dtype=np.uint16)
    lib().orc_narrow(DTYPES[dtype], ptr(x), ptr(out), x.size)
    return out


def widen(values, dtype: str) -> np.ndarray:
    x = np.ascontiguousarray(values, dtype=STORE[dtype])
    if dtype == "f32":
        return x.astype(np.float32)
    out = np.empty(x.shape, dtype=np.float32)
    lib().orc_widen(DTYPES[dtype], ptr(x), ptr(out), x.size)
    return out


def set_threads(n: int) -> None:
    lib().orc_set_threads(int(n))


def set_matmul_threads(n: int) -> None:
    """Threads for the oracle's large products (tests only: the same bits as
    the Host's single thread, in a cache-blocked loop nest)."""
    lib().orc_set_matmul_threads(int(n))


# --- convenience wrappers returning numpy arrays ---------------------------
def strided_copy(src: np.ndarray, shape, offset, strides) -> np.ndarray:
    n = int(np.prod(shape, dtype=np.int64)) if shape else 1
    out = np.empty(n, dtype=src.dtype)
    call("orc_strided_copy", src.itemsize, len(shape), sizes(shape), ptr(src), src.size, offset, sizes(strides),
         ptr(out))
    return out


def strided_binary(dtype, kind, op, shape, a, a_off, a_str, b, b_off, b_str) -> np.ndarray:
    n = int(np.prod(shape, dtype=np.int64)) if shape else 1
    out = np.empty(n, dtype=STORE[dtype])
    call("orc_strided_binary", DTYPES[dtype], kind, op, len(shape), sizes(shape), ptr(a), a.size, a_off,
         sizes(a_str), ptr(b), b.size, b_off, sizes(b_str), ptr(out))
    return out


def reduce_axes(dtype, shape, x, offset, strides, axes, kind, op, divisor) -> np.ndarray:
    results = int(np.prod([e for a, e in enumerate(shape) if a not in axes], dtype=np.int64))
    out = np.empty(results, dtype=STORE[dtype])
    call("orc_reduce_axes", DTYPES[dtype], len(shape), sizes(shape), ptr(x), x.size, offset, sizes(strides),
         len(axes), u32s(axes), kind, op, divisor, ptr(out))
    return out


def arg_reduce(dtype, shape, x, offset, strides, axis, op) -> np.ndarray:
    results = int(np.prod([e for a, e in enumerate(shape) if a != axis], dtype=np.int64))
    out = np.empty(results, dtype=np.uint32)
    call("orc_arg_reduce", DTYPES[dtype], len(shape), sizes(shape), ptr(x), x.size, offset, sizes(strides),
         axis, op, out.ctypes.data_as(_u32p))
    return out


def matmul(dtype, transposed, rows, inner, cols, a, b, c=None, accumulate=False) -> np.ndarray:
    out = np.zeros(rows * cols, dtype=STORE[dtype]) if c is None else np.array(c, dtype=STORE[dtype]).reshape(-1)
    call("orc_matmul", DTYPES[dtype], transposed, rows, inner, cols, ptr(np.ascontiguousarray(a)),
         ptr(np.ascontiguousarray(b)), ptr(out), int(accumulate))
    return out


def adam_coefficients(dtype, rate, b1, b2, eps, step) -> list[float]:
    out = (C.c_double * 6)()
    call("orc_adam_coefficients", DTYPES[dtype], rate, b1, b2, eps, step, out)
    return list(out)
