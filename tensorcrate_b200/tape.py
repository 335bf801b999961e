"""A reverse-mode tape over device tensors, run natively by libtccuda
(tc_tape_*): the tensor-level rules of tensorcrate's tape
(src/tensors/tape/tensor.rs, MatrixVar in src/tensors/tape/mod.rs) behind a
small Python handle."""
from __future__ import annotations

import ctypes as C

import numpy as np

from . import _native as N
from .cuda import ELEM, CudaStorage, _stream


class Tape:
    def __init__(self, dtype: str = "f32", stream=None):
        self.dtype = dtype
        out = C.c_void_p()
        N.call("tc_tape_create", N.DTYPES[dtype], _stream(stream), C.byref(out))
        self.handle = out
        self._keep = []  # leaves' storages outlive the tape's reads

    def _out(self, name, *args) -> int:
        v = C.c_uint32()
        N.call(name, self.handle, *args, C.byref(v))
        return v.value

    def leaf(self, storage: CudaStorage, shape) -> int:
        self._keep.append(storage)
        return self._out("tc_tape_leaf", storage.ptr, len(shape), N.sizes(shape))

    def add(self, a: int, b: int) -> int:
        return self._out("tc_tape_binary", N.ADD, a, b)

    def sub(self, a: int, b: int) -> int:
        return self._out("tc_tape_binary", N.SUB, a, b)

    def mul(self, a: int, b: int) -> int:
        return self._out("tc_tape_binary", N.MUL, a, b)

    def div(self, a: int, b: int) -> int:
        return self._out("tc_tape_binary", N.DIV, a, b)

    def relu(self, a: int) -> int:
        return self._out("tc_tape_relu", a)

    def scale(self, a: int, factor: float) -> int:
        return self._out("tc_tape_scale", a, float(factor))

    def sum_axes(self, a: int, axes, keep_dims=False, mean=False) -> int:
        shape = self.shape(a)
        count = int(np.prod([shape[i] for i in axes]))
        share = float(np.float32(1.0 / count)) if mean else 0.0
        return self._out("tc_tape_sum_axes", a, len(axes), N.u32s(axes), int(mean), int(keep_dims), share)

    def mean_axes(self, a: int, axes, keep_dims=False) -> int:
        return self.sum_axes(a, axes, keep_dims, mean=True)

    def matmul(self, a: int, b: int) -> int:
        return self._out("tc_tape_matmul", a, b)

    def sum(self, a: int) -> int:
        return self._out("tc_tape_sum", a)

    def shape(self, v: int) -> list[int]:
        rank = C.c_uint32()
        shape = (C.c_size_t * N.MAX_RANK)()
        N.call("tc_tape_value", self.handle, v, None, C.byref(rank), shape)
        return [int(shape[i]) for i in range(rank.value)]

    def _read(self, ptr: int | None, v: int):
        if not ptr:
            return None
        n = int(np.prod(self.shape(v))) if self.shape(v) else 1
        out = np.empty(n, ELEM[self.dtype][0])
        N.call("tc_stream_sync", None)
        N.call("tc_memcpy_d2h", out.ctypes.data, ptr, out.nbytes, None)
        return out.reshape(self.shape(v)) if self.shape(v) else out

    def value(self, v: int):
        p = C.c_void_p()
        N.call("tc_tape_value", self.handle, v, C.byref(p), None, None)
        return self._read(p.value, v)

    def backward(self, v: int) -> None:
        N.call("tc_tape_backward", self.handle, v)

    def grad(self, v: int):
        """The adjoint after backward, or None when nothing reached v."""
        p = C.c_void_p()
        N.call("tc_tape_adjoint", self.handle, v, C.byref(p))
        return self._read(p.value, v)

    def close(self) -> None:
        if self.handle:
            N.call("tc_stream_sync", None)
            N.call("tc_tape_destroy", self.handle)
            self.handle = None

    def __del__(self):
        try:
            if self.handle and N._lib is not None:
                N._lib.tc_tape_destroy(self.handle)
        except Exception:
            pass
