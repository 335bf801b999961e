"""ctypes binding of the C ABI in include/tccuda.h (libtccuda.so).

The library is the product: there is no CPU or Python fallback.  Loading
fails loudly if tensorcrate_b200/_lib/libtccuda.so has not been built
(`python -m tensorcrate_b200.build`).
"""
from __future__ import annotations

import ctypes as C
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "_lib" / "libtccuda.so"

# Status codes, element types and operation enums (include/tccuda.h).
OK, EINVAL, ERANGE, ENOMEM, ECUDA, ENCCL, ETIMEOUT, ENOTSUP = range(8)
F32, F16, BF16, U32 = 0, 1, 2, 3
DTYPES = {"f32": F32, "f16": F16, "bf16": BF16, "u32": U32}
ADD, SUB, MUL, DIV, REM = range(5)
MIN, MAX, MAX_SHARE, LESS, LESS_EQUAL, GREATER, GREATER_EQUAL = range(7)
SUM, RMIN, RMAX = range(3)
PAIR_ARITHMETIC, PAIR_COMPARE, PAIR_POWER = range(3)
AXIS_FOLD, AXIS_MEAN, AXIS_VARIANCE = range(3)
TRANS_NONE, TRANS_LEFT, TRANS_RIGHT = range(3)
MAX_RANK = 6

_sz = C.c_size_t
_p = C.c_void_p
_i = C.c_int
_u32 = C.c_uint32
_d = C.c_double
_szp = C.POINTER(C.c_size_t)
_u32p = C.POINTER(C.c_uint32)


class Region(C.Structure):
    """tc_region: one block of an assemble or strided write."""

    _fields_ = [
        ("source", _p),
        ("source_len", _sz),
        ("rank", _u32),
        ("shape", _sz * MAX_RANK),
        ("from_offset", _sz),
        ("from_strides", _sz * MAX_RANK),
        ("to_offset", _sz),
        ("to_strides", _sz * MAX_RANK),
    ]


class Instr(C.Structure):
    """tc_instr: one instruction of a fused program."""

    _fields_ = [("code", C.c_uint8), ("dst", C.c_uint8), ("a", C.c_uint8), ("b", C.c_uint8), ("op", C.c_uint8),
                ("slot", C.c_uint8), ("reserved", C.c_uint16), ("value", C.c_float)]


class Place(C.Structure):
    """tc_place: where one load of a fused program reads."""

    _fields_ = [("data", _p), ("dtype", C.c_int), ("lead", _u32), ("offset", _sz), ("col_step", _sz),
                ("dims", _sz * (MAX_RANK - 1)), ("steps", _sz * (MAX_RANK - 1))]


I_LOAD, I_CONST, I_BINARY, I_UNARY, I_CMP, I_STORE = range(6)
(SIN, COS, TAN, SEC, CSC, ARCSIN, ARCCOS, ARCTAN, EXP, LN, SINH, COSH, TANH, SQRT) = range(14)
ASCENDING, DESCENDING = range(2)
ROWS, COLUMNS = range(2)
NORMAL, INVERSE_GAUSSIAN = range(2)
PDF, CDF, PPF = range(3)


class RowStatistic(C.Structure):
    """tc_row_statistic: loads of `into_place` read a statistic of each row
    of `of_place`."""

    _fields_ = [("of_place", _u32), ("into_place", _u32), ("statistic", C.c_int)]


ROW_MEAN, ROW_DEVIATIONS = range(2)


class AdamTensor(C.Structure):
    """tc_adam_tensor: one parameter of a tc_adam_multi call."""

    _fields_ = [("p", _p), ("g", _p), ("m", _p), ("v", _p), ("n", _sz)]


# name -> argtypes; every function returns int status.
SIGNATURES = {
    "tc_last_error": [C.c_char_p, _sz],
    "tc_set_device": [_i],
    "tc_device_count": [C.POINTER(_i)],
    "tc_sm_count": [C.POINTER(_i)],
    "tc_ctx_create": [_i, C.POINTER(_p)],
    "tc_ctx_stream": [_p, C.POINTER(_p)],
    "tc_ctx_device": [_p, C.POINTER(_i)],
    "tc_ctx_destroy": [_p],
    "tc_malloc": [C.POINTER(_p), _sz],
    "tc_malloc_async": [C.POINTER(_p), _sz, _p],
    "tc_free": [_p],
    "tc_free_async": [_p, _p],
    "tc_alloc_counts": [C.POINTER(C.c_uint64), C.POINTER(C.c_uint64)],
    "tc_pool_trim": [],
    "tc_host_alloc": [C.POINTER(_p), _sz],
    "tc_host_free": [_p],
    "tc_memcpy_h2d": [_p, _p, _sz, _p],
    "tc_memcpy_d2h": [_p, _p, _sz, _p],
    "tc_memcpy_d2d": [_p, _p, _sz, _p],
    "tc_memset": [_p, _i, _sz, _p],
    "tc_stream_sync": [_p],
    "tc_strided_copy": [_sz, _u32, _szp, _p, _sz, _sz, _szp, _p, _p],
    "tc_strided_write": [_sz, _p, _sz, C.POINTER(Region), _p],
    "tc_assemble": [_sz, _p, _sz, C.POINTER(Region), _sz, _p],
    "tc_elementwise": [_i, _i, _p, _p, _p, _sz, _p],
    "tc_broadcast_scalar": [_i, _i, _p, _d, _i, _p, _sz, _p],
    "tc_compare": [_i, _i, _p, _p, _p, _sz, _p],
    "tc_compare_scalar": [_i, _i, _p, _d, _i, _p, _sz, _p],
    "tc_clamp": [_i, _p, _d, _d, _p, _sz, _p],
    "tc_vector_reduce": [_i, _i, _p, _sz, _p, _p],
    "tc_dot": [_i, _p, _p, _sz, _p, _p],
    "tc_prefix_sum": [_i, _p, _p, _sz, _p],
    "tc_sort": [_i, _i, _p, _p, _sz, _p],
    "tc_unary": [_i, _i, _p, _p, _sz, _p],
    "tc_unary_dual": [_i, _i, _p, _p, _p, _p, _sz, _p],
    "tc_power": [_i, _p, _p, _p, _sz, _p],
    "tc_power_scalar": [_i, _p, _d, _i, _p, _sz, _p],
    "tc_correlate": [_i, _sz, _sz, _sz, _sz, _i, _p, _p, _p, _p],
    "tc_correlate_window_gradient": [_i, _sz, _sz, _sz, _sz, _p, _p, _p, _p],
    "tc_correlate_input_gradient": [_i, _sz, _sz, _sz, _sz, _i, _p, _p, _p, _p],
    "tc_pad": [_i, _sz, _sz, _sz, _sz, _p, _p, _p],
    "tc_flip": [_i, _sz, _sz, _p, _p, _p],
    "tc_moments": [_i, _p, _sz, _p, _p],
    "tc_axis_moments": [_i, _sz, _sz, _i, _p, _p, _p, _p],
    "tc_distribution": [_i, _i, _i, _p, _sz, _d, _d, _p, _p],
    "tc_axis_distribution": [_i, _sz, _sz, _i, _i, _i, _p, _p, _p, _p, _p],
    "tc_strided_binary": [_i, _i, _i, _u32, _szp, _p, _sz, _sz, _szp, _p, _sz, _sz, _szp, _p, _p],
    "tc_reduce_axes": [_i, _u32, _szp, _p, _sz, _sz, _szp, _u32, _u32p, _i, _i, _sz, _p, _p],
    "tc_arg_reduce": [_i, _u32, _szp, _p, _sz, _sz, _szp, _u32, _i, _u32p, _p],
    "tc_matmul": [_i, _i, _sz, _sz, _sz, _p, _p, _p, _i, _p],
    "tc_matvec": [_i, _sz, _sz, _p, _p, _p, _i, _p],
    "tc_vecmat": [_i, _sz, _sz, _p, _p, _p, _p],
    "tc_fused": [_i, _sz, _sz, _p, _u32, _p, _u32, _p, _p, _u32, _p],
    "tc_fused_with_statistics": [_i, _sz, _sz, _p, _u32, _p, _u32, _p, _u32, _p, _p, _u32, _p],
    "tc_fused_sum": [_i, _sz, _sz, _p, _u32, _p, _u32, _i, _p, _p],
    "tc_row_moments": [_i, _p, _sz, _sz, _p, _p, _p],
    "tc_matmul_program": [_i, _sz, _sz, _sz, _p, _p, _p, _u32, _p, _u32, _p, _p, _u32, _p],
    "tc_matmul_epilogue": [_i, _i, _sz, _sz, _sz, _p, _p, _p, _p, _p, _p, _p],
    "tc_vecmat_noalloc": [_i, _sz, _sz, _p, _p, _p, _p],
    "tc_adam": [_i, _sz, _p, _p, _p, _p, _i, _d, _d, _d, _d, _d, _d, _p],
    "tc_adam_multi": [_i, _p, _sz, _i, _d, _d, _d, _d, _d, _d, _p],
    "tc_sgd": [_i, _sz, _p, _p, _d, _p],
    "tc_momentum": [_i, _sz, _p, _p, _p, _d, _d, _i, _p],
    "tc_adagrad": [_i, _sz, _p, _p, _p, _d, _d, _p],
    "tc_rmsprop": [_i, _sz, _p, _p, _p, _d, _d, _d, _p],
    "tc_coalesce": [_u32, _szp, _u32, _szp, _u32p, _szp, _szp],
    "tc_device_status": [C.POINTER(_i)],
    "tc_device_status_reset": [],
    "tc_set_wait_limit": [C.c_ulonglong],
    "tc_set_peer_wait_limit": [C.c_ulonglong],
    "tc_mlp_create": [_i, _u32, _u32p, _u32, _u32, _d, _d, _d, _d, C.POINTER(_p)],
    "tc_mlp_destroy": [_p],
    "tc_mlp_params": [_p, _u32, _p, _p, _i],
    "tc_mlp_grads": [_p, _u32, _p, _p],
    "tc_mlp_block": [_p, _u32, C.POINTER(_sz), C.POINTER(_sz)],
    "tc_mlp_prune_leaves": [_p, _i],
    "tc_mlp_step": [_p, _p, _p, _p, _p, _p],
    "tc_mlp_attach": [_p, _p],
    "tc_tape_create": [_i, _p, C.POINTER(_p)],
    "tc_tape_destroy": [_p],
    "tc_tape_leaf": [_p, _p, _u32, _szp, _u32p],
    "tc_tape_binary": [_p, _i, _u32, _u32, _u32p],
    "tc_tape_relu": [_p, _u32, _u32p],
    "tc_tape_scale": [_p, _u32, _d, _u32p],
    "tc_tape_sum_axes": [_p, _u32, _u32, _u32p, _i, _i, _d, _u32p],
    "tc_tape_matmul": [_p, _u32, _u32, _u32p],
    "tc_tape_sum": [_p, _u32, _u32p],
    "tc_tape_value": [_p, _u32, C.POINTER(_p), _u32p, _szp],
    "tc_tape_backward": [_p, _u32],
    "tc_tape_adjoint": [_p, _u32, C.POINTER(_p)],
    "tc_comm_unique_id": [C.POINTER(C.c_uint8)],
    "tc_comm_init": [_i, _i, C.POINTER(C.c_uint8), C.POINTER(_p)],
    "tc_comm_destroy": [_p],
    "tc_allgather": [_p, _i, _p, _p, _sz, _p],
    "tc_allreduce": [_p, _i, _p, _sz, _i, _p],
    "tc_reducescatter": [_p, _i, _p, _p, _sz, _i, _p],
    "tc_comm_rank": [_p, _p, _p],
    "tc_peer_buffer_create": [_p, _sz, _p],
    "tc_peer_buffer_pointer": [_p, _p],
    "tc_peer_buffer_destroy": [_p],
    "tc_matmul_allgather": [_p, _i, _sz, _sz, _sz, _p, _p, _p, _p],
}


class TcError(RuntimeError):
    """A non-zero status from the library; `.status` is the tc_status code."""

    def __init__(self, op: str, status: int, message: str):
        super().__init__(f"{op} could not execute on the GPU (status {status}): {message}")
        self.status = status


_lib: C.CDLL | None = None


def lib() -> C.CDLL:
    """The loaded library; raises if it is missing (no fallback exists)."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise ImportError(
                f"{LIB_PATH} is missing: build it with `python -m tensorcrate_b200.build`; "
                "the CUDA backend has no CPU fallback"
            )
        handle = C.CDLL(str(LIB_PATH))
        for name, args in SIGNATURES.items():
            fn = getattr(handle, name)
            fn.argtypes = args
            fn.restype = C.c_int
        handle.tc_build_info.argtypes = []
        handle.tc_build_info.restype = C.c_char_p
        _lib = handle
    return _lib


def last_error() -> str:
    buf = C.create_string_buffer(512)
    lib().tc_last_error(buf, 512)
    return buf.value.decode(errors="replace")


def check(op: str, status: int) -> None:
    """Map a status to an exception naming the operation (require_metal's
    panic, src/tensors/backend.rs:418-426)."""
    if status != OK:
        raise TcError(op, status, last_error())


def call(name: str, *args) -> None:
    check(name, getattr(lib(), name)(*args))


def sizes(values) -> C.Array:
    values = [int(v) for v in values]
    arr = (_sz * max(1, len(values)))(*values)
    return arr


def u32s(values) -> C.Array:
    values = [int(v) for v in values]
    return (_u32 * max(1, len(values)))(*values)
