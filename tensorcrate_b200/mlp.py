"""Config 4's training step (the reference's tape + Adam, run natively by
libtccuda's tc_mlp_*) behind a small Python handle."""
from __future__ import annotations

import ctypes as C

import numpy as np

from . import _native as N
from .cuda import ELEM, CudaStorage, _stream, f32_to_bits


def xavier(fan_out: int, fan_in: int, rng: np.random.Generator) -> np.ndarray:
    """Xavier-uniform: U(-a, a), a = sqrt(6 / (fan_in + fan_out))."""
    a = np.sqrt(6.0 / (fan_in + fan_out))
    return rng.uniform(-a, a, (fan_out, fan_in)).astype(np.float32)


class Mlp:
    def __init__(self, dtype: str, dims, batch: int, global_batch: int | None = None, rate=1e-3, beta1=0.9,
                 beta2=0.999, eps=1e-8):
        self.dtype, self.dims, self.batch = dtype, [int(d) for d in dims], int(batch)
        out = C.c_void_p()
        N.call("tc_mlp_create", N.DTYPES[dtype], len(dims) - 1, N.u32s(dims), batch, global_batch or batch,
               rate, beta1, beta2, eps, C.byref(out))
        self.handle = out

    def load(self, weights, biases) -> None:
        for l, (w, b) in enumerate(zip(weights, biases)):
            w = np.ascontiguousarray(w if w.dtype == ELEM[self.dtype][0] else f32_to_bits(w, self.dtype))
            b = np.ascontiguousarray(b if b.dtype == ELEM[self.dtype][0] else f32_to_bits(b, self.dtype))
            N.call("tc_mlp_params", self.handle, l, w.ctypes.data, b.ctypes.data, 0)

    def params(self, l: int):
        w = np.empty(self.dims[l + 1] * self.dims[l], ELEM[self.dtype][0])
        b = np.empty(self.dims[l + 1], ELEM[self.dtype][0])
        N.call("tc_mlp_params", self.handle, l, w.ctypes.data, b.ctypes.data, 1)
        return w, b

    def grads(self, l: int):
        w = np.empty(self.dims[l + 1] * self.dims[l], ELEM[self.dtype][0])
        b = np.empty(self.dims[l + 1], ELEM[self.dtype][0])
        N.call("tc_mlp_grads", self.handle, l, w.ctypes.data, b.ctypes.data)
        return w, b

    def block(self, l: int) -> tuple[int, int]:
        """(length, bias offset) of layer l's block of the flat buffers."""
        n, at = C.c_size_t(), C.c_size_t()
        N.call("tc_mlp_block", self.handle, l, C.byref(n), C.byref(at))
        return n.value, at.value

    def prune_leaves(self, prune: bool) -> None:
        N.call("tc_mlp_prune_leaves", self.handle, int(prune))

    def step(self, x: CudaStorage, y: CudaStorage, comm=None, loss: CudaStorage | None = None, stream=None):
        N.call("tc_mlp_step", self.handle, x.ptr, y.ptr, comm, loss.ptr if loss is not None else None,
               _stream(stream))

    def attach(self, comm) -> None:
        """Exchange over NVLink peer memory in steps over `comm`
        (collective; close() is then collective too)."""
        N.call("tc_mlp_attach", self.handle, comm)
        self.attached = True

    def close(self) -> None:
        """Free the handle now (collective when attached: every rank closes
        its handle at the same point)."""
        if self.handle:
            N.call("tc_mlp_destroy", self.handle)
            self.handle = None

    def __del__(self):
        # An attached handle is freed collectively by close(); a handle left
        # attached at exit is left to the process's end.
        try:
            if self.handle and N._lib is not None and not getattr(self, "attached", False):
                N._lib.tc_mlp_destroy(self.handle)
        except Exception:
            pass
