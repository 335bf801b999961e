"""The `Cuda` backend as the reference's traits present it, over the C ABI.

This mirrors the parts of tensorcrate that sit on the hot path, with the
reference's names, argument meanings and panics (raised as exceptions):

- `CudaStorage` is `Backend::Storage<T>` (src/tensors/backend.rs:84): a
  device buffer; `store`/`as_slice`/`duplicate` are the Backend methods of
  the same names (backend.rs:88-111).
- `Cuda` holds the `Backend` copies (strided_copy, assemble, strided_write,
  backend.rs:141-173) and the `Kernels<T>` methods (kernels.rs:829-1188)
  that the hot path calls.
- `TensorView`/`Tensor` carry the view arithmetic of src/tensors/view.rs,
  tensor.rs, tensor_ops.rs and reduction.rs: shape checks, broadcasting and
  strides on the host, every element touched by a CUDA kernel.

Element types are "f32", "f16" and "bf16"; f16/bf16 values cross the host
boundary as their uint16 bit patterns (numpy has no bf16).
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass
from typing import Iterable, Sequence

import numpy as np

from . import _native as N

ELEM = {"f32": (np.float32, 4), "f16": (np.uint16, 2), "bf16": (np.uint16, 2), "u32": (np.uint32, 4)}
MAX_RANK = N.MAX_RANK


# ---------------------------------------------------------------------------
# host-side element conversions (round to nearest even, NaN kept quiet), the
# rounding crate `half` applies (src/compact.rs:5-22)
# ---------------------------------------------------------------------------
def f32_to_bits(values, dtype: str) -> np.ndarray:
    """f32 values rounded once to `dtype`, as its storage (bits for f16/bf16)."""
    x = np.ascontiguousarray(values, dtype=np.float32)
    if dtype == "f32":
        return x
    if dtype == "f16":
        return x.astype(np.float16).view(np.uint16)
    if dtype == "bf16":
        u = x.view(np.uint32).astype(np.uint64)
        nan = (u & 0x7FFFFFFF) > 0x7F800000
        r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
        q = ((u >> 16) | 0x0040).astype(np.uint16)
        return np.where(nan, q, r).astype(np.uint16)
    raise ValueError(dtype)


def bits_to_f32(bits, dtype: str) -> np.ndarray:
    b = np.asarray(bits)
    if dtype == "f32":
        return b.astype(np.float32)
    if dtype == "f16":
        return b.astype(np.uint16).view(np.float16).astype(np.float32)
    if dtype == "bf16":
        return (b.astype(np.uint32) << 16).view(np.float32)
    if dtype == "u32":
        return b.astype(np.float32)
    raise ValueError(dtype)


def _stream(stream) -> C.c_void_p:
    if stream is None:
        return None
    if isinstance(stream, int):
        return C.c_void_p(stream)
    return C.c_void_p(int(getattr(stream, "cuda_stream", stream)))


# ---------------------------------------------------------------------------
# storage
# ---------------------------------------------------------------------------
class CudaStorage:
    """A flat run of `len` elements of `dtype` in device memory.  Its block
    comes from the library's pool in the default stream's order and goes
    back in that order when the storage is dropped (tc_free_async), so a
    storage dropped while kernels that use it are queued is not handed out
    before they ran."""

    __slots__ = ("ptr", "len", "dtype", "_owned", "__weakref__")

    def __init__(self, dtype: str, length: int, ptr: int | None = None):
        if dtype not in ELEM:
            raise ValueError(f"unknown element type {dtype!r}")
        self.dtype, self.len = dtype, int(length)
        if ptr is None:
            out = C.c_void_p()
            N.call("tc_malloc_async", C.byref(out), max(1, self.len * ELEM[dtype][1]), None)
            self.ptr, self._owned = out.value, True
        else:
            self.ptr, self._owned = int(ptr), False

    @property
    def elem_bytes(self) -> int:
        return ELEM[self.dtype][1]

    @property
    def nbytes(self) -> int:
        return self.len * self.elem_bytes

    @classmethod
    def store(cls, values, dtype: str, stream=None) -> "CudaStorage":
        """Backend::store: upload `values` (already in `dtype`'s storage form)."""
        host = np.ascontiguousarray(values, dtype=ELEM[dtype][0]).reshape(-1)
        s = cls(dtype, host.size)
        if host.size:
            N.call("tc_memcpy_h2d", s.ptr, host.ctypes.data, host.nbytes, _stream(stream))
            if stream is None:
                N.call("tc_stream_sync", None)
        return s

    @classmethod
    def zeros(cls, dtype: str, length: int) -> "CudaStorage":
        s = cls(dtype, length)
        if length:
            N.call("tc_memset", s.ptr, 0, s.nbytes, None)
        return s

    def as_slice(self, stream=None) -> np.ndarray:
        """Backend::as_slice: the elements on the host (waits for the device)."""
        out = np.empty(self.len, dtype=ELEM[self.dtype][0])
        if self.len:
            N.call("tc_stream_sync", _stream(stream))
            N.call("tc_memcpy_d2h", out.ctypes.data, self.ptr, self.nbytes, None)
        return out

    def to_f32(self) -> np.ndarray:
        return bits_to_f32(self.as_slice(), self.dtype)

    def duplicate(self, stream=None) -> "CudaStorage":
        s = CudaStorage(self.dtype, self.len)
        if self.len:
            N.call("tc_memcpy_d2d", s.ptr, self.ptr, self.nbytes, _stream(stream))
        return s

    def __del__(self):
        try:
            if self._owned and self.ptr and N._lib is not None:
                N._lib.tc_free_async(self.ptr, None)
        except Exception:  # interpreter shutdown
            pass

    def __repr__(self) -> str:
        return f"CudaStorage({self.dtype}, len={self.len})"


# ---------------------------------------------------------------------------
# layout arithmetic (src/tensors/layout.rs)
# ---------------------------------------------------------------------------
def contiguous_strides(shape: Sequence[int]) -> list[int]:
    strides, step = [0] * len(shape), 1
    for axis in range(len(shape) - 1, -1, -1):
        strides[axis] = step
        step *= shape[axis]
    return strides


def broadcast_shape(left: Sequence[int], right: Sequence[int]) -> list[int] | None:
    rank = max(len(left), len(right))
    out = []
    for axis in range(rank):
        from_end = rank - axis
        l = left[len(left) - from_end] if len(left) >= from_end else 1
        r = right[len(right) - from_end] if len(right) >= from_end else 1
        if l == r or r == 1:
            out.append(l)
        elif l == 1:
            out.append(r)
        else:
            return None
    return out


def broadcast_strides(shape, strides, target) -> list[int] | None:
    added = len(target) - len(shape)
    if added < 0:
        return None
    out = [0] * len(target)
    for axis in range(len(shape)):
        wanted = target[added + axis]
        if shape[axis] == wanted:
            out[added + axis] = strides[axis]
        elif shape[axis] == 1:
            out[added + axis] = 0
        else:
            return None
    return out


def coalesce(shape, *strides) -> tuple[list[int], list[list[int]]]:
    """layout.rs:419-446, through the library's own descriptor builder."""
    rank, n = len(shape), len(strides)
    out_rank = C.c_uint32()
    out_shape = (C.c_size_t * MAX_RANK)()
    out_strides = (C.c_size_t * (MAX_RANK * 3))()
    flat = [s for op in strides for s in op]
    N.call("tc_coalesce", rank, N.sizes(shape), n, N.sizes(flat), C.byref(out_rank), out_shape, out_strides)
    r = out_rank.value
    return list(out_shape[:r]), [list(out_strides[o * r:(o + 1) * r]) for o in range(n)]


# ---------------------------------------------------------------------------
# views and tensors
# ---------------------------------------------------------------------------
@dataclass
class TensorView:
    """A strided window on a storage: element [i...] is
    storage[offset + sum(i_k * strides[k])] (view.rs)."""

    storage: CudaStorage
    shape: list[int]
    strides: list[int]
    offset: int = 0

    @property
    def dtype(self) -> str:
        return self.storage.dtype

    @property
    def rank(self) -> int:
        return len(self.shape)

    def numel(self) -> int:
        return int(np.prod(self.shape, dtype=np.int64)) if self.shape else 1

    def is_contiguous(self) -> bool:
        if 0 in self.shape:
            return True
        step = 1
        for e, s in zip(reversed(self.shape), reversed(self.strides)):
            if e != 1 and s != step:
                return False
            step *= e
        return True

    def is_whole(self) -> bool:
        return self.offset == 0 and self.is_contiguous() and self.numel() == self.storage.len

    # --- stride rewrites (view.rs:146-292) ---
    def permute(self, axes: Sequence[int]) -> "TensorView":
        if sorted(axes) != list(range(self.rank)):
            raise ValueError(f"permute: {list(axes)} is not a permutation of {self.rank} axes")
        return TensorView(self.storage, [self.shape[a] for a in axes], [self.strides[a] for a in axes], self.offset)

    def slice(self, axis: int, start: int, end: int) -> "TensorView":
        if not (0 <= start <= end <= self.shape[axis]):
            raise ValueError(f"slice: {start}..{end} reaches past axis {axis}'s extent of {self.shape[axis]}")
        shape = list(self.shape)
        shape[axis] = end - start
        return TensorView(self.storage, shape, list(self.strides), self.offset + start * self.strides[axis])

    def split(self, axis: int, sizes: Sequence[int]) -> list["TensorView"]:
        if sum(sizes) != self.shape[axis]:
            raise ValueError("split: sizes do not add up to the axis extent")
        out, at = [], 0
        for s in sizes:
            out.append(self.slice(axis, at, at + s))
            at += s
        return out

    def chunk(self, axis: int, pieces: int) -> list["TensorView"]:
        extent = self.shape[axis]
        step = -(-extent // pieces)
        return self.split(axis, [min(step, extent - k) for k in range(0, extent, step)])

    def broadcast_to(self, shape: Sequence[int]) -> "TensorView":
        st = broadcast_strides(self.shape, self.strides, shape)
        if st is None:
            raise ValueError(f"broadcast: {self.shape} does not broadcast to {list(shape)}")
        return TensorView(self.storage, list(shape), st, self.offset)

    def unsqueeze(self, axis: int) -> "TensorView":
        shape, strides = list(self.shape), list(self.strides)
        step = strides[axis] * shape[axis] if axis < self.rank else 1
        shape.insert(axis, 1)
        strides.insert(axis, step)
        return TensorView(self.storage, shape, strides, self.offset)

    # --- copies ---
    def contiguous(self, stream=None) -> "Tensor":
        """view.rs:407-421: Backend::strided_copy into a new row-major tensor."""
        return Tensor(Cuda.strided_copy(self.storage, self.shape, self.offset, self.strides, stream), self.shape)

    def to_numpy(self) -> np.ndarray:
        return self.contiguous().to_numpy()

    # --- elementwise and reductions ---
    def elementwise(self, other: "TensorView", kind: int, op: int, stream=None) -> "Tensor":
        return elementwise(self, other, kind, op, stream)

    def reduce_axes(self, op: int, axes, keep_dims: bool = False, stream=None) -> "Tensor":
        return reduction(self, axes, keep_dims, N.AXIS_FOLD, op, None, stream)

    def sum_axes(self, axes, keep_dims=False, stream=None):
        return self.reduce_axes(N.SUM, axes, keep_dims, stream)

    def max_axes(self, axes, keep_dims=False, stream=None):
        return self.reduce_axes(N.RMAX, axes, keep_dims, stream)

    def min_axes(self, axes, keep_dims=False, stream=None):
        return self.reduce_axes(N.RMIN, axes, keep_dims, stream)

    def mean_axes(self, axes, keep_dims=False, stream=None):
        return reduction(self, axes, keep_dims, N.AXIS_MEAN, 0, None, stream)

    def var_axes(self, axes, sample: bool, keep_dims=False, stream=None):
        return reduction(self, axes, keep_dims, N.AXIS_VARIANCE, 0, 1 if sample else 0, stream)

    def argmax(self, axis: int, keep_dims=False, stream=None):
        return arg_reduction(self, axis, keep_dims, N.RMAX, "argmax", stream)

    def argmin(self, axis: int, keep_dims=False, stream=None):
        return arg_reduction(self, axis, keep_dims, N.RMIN, "argmin", stream)


class Tensor:
    """An owned row-major tensor: a storage and a shape (tensor.rs)."""

    def __init__(self, storage: CudaStorage, shape: Sequence[int]):
        self.storage, self.shape = storage, [int(e) for e in shape]

    @classmethod
    def from_numpy(cls, values: np.ndarray, dtype: str) -> "Tensor":
        values = np.asarray(values)
        if values.dtype != ELEM[dtype][0]:
            values = f32_to_bits(values, dtype)
        return cls(CudaStorage.store(values, dtype), values.shape)

    @property
    def dtype(self) -> str:
        return self.storage.dtype

    def view(self) -> TensorView:
        return TensorView(self.storage, list(self.shape), contiguous_strides(self.shape), 0)

    def to_numpy(self) -> np.ndarray:
        return self.storage.as_slice().reshape(self.shape)

    def to_f32(self) -> np.ndarray:
        return bits_to_f32(self.to_numpy(), self.dtype)

    def __getattr__(self, name):
        # Every view operation reads a tensor as its whole view.
        return getattr(self.view(), name)

    @staticmethod
    def concat(pieces: Sequence, axis: int, stream=None) -> "Tensor":
        """tensor.rs:409-449: one assemble, one region per piece."""
        views = [p.view() if isinstance(p, Tensor) else p for p in pieces]
        if not views:
            raise ValueError("concat: no tensors")
        first = views[0]
        for v in views:
            if v.rank != first.rank or v.dtype != first.dtype or any(
                v.shape[a] != first.shape[a] for a in range(first.rank) if a != axis
            ):
                raise ValueError("concat: shapes differ off the concatenation axis")
        shape = list(first.shape)
        shape[axis] = sum(v.shape[axis] for v in views)
        to = contiguous_strides(shape)
        regions, at = [], 0
        for v in views:
            regions.append((v.storage, v.shape, v.offset, v.strides, at * to[axis], to))
            at += v.shape[axis]
        total = int(np.prod(shape, dtype=np.int64))
        return Tensor(Cuda.assemble(first.dtype, total, regions, stream), shape)

    @staticmethod
    def stack(pieces: Sequence, axis: int, stream=None) -> "Tensor":
        """tensor.rs:459-482: unsqueeze each, then concat."""
        views = [(p.view() if isinstance(p, Tensor) else p).unsqueeze(axis) for p in pieces]
        return Tensor.concat(views, axis, stream)

    def write_slice(self, axis: int, start: int, piece, stream=None) -> None:
        """tensor.rs:504-529: one strided write into this tensor in place."""
        v = piece.view() if isinstance(piece, Tensor) else piece
        to = contiguous_strides(self.shape)
        Cuda.strided_write(self.storage, (v.storage, v.shape, v.offset, v.strides, start * to[axis], to), stream)


def _as_view(x) -> TensorView:
    return x.view() if isinstance(x, Tensor) else x


# tensor_ops.rs:71-91 `zip`: whole same-shape operands take the vector
# kernel; anything else is broadcast and read through its strides.
def elementwise(a, b, kind: int, op: int, stream=None) -> Tensor:
    a, b = _as_view(a), _as_view(b)
    if a.dtype != b.dtype:
        raise ValueError("elementwise: element types differ")
    if a.shape == b.shape and a.is_whole() and b.is_whole():
        out = CudaStorage(a.dtype, a.numel())
        fn = {N.PAIR_ARITHMETIC: "tc_elementwise", N.PAIR_COMPARE: "tc_compare"}.get(kind)
        if fn is not None:
            N.call(fn, N.DTYPES[a.dtype], op, a.storage.ptr, b.storage.ptr, out.ptr, out.len, _stream(stream))
            return Tensor(out, a.shape)
    shape = broadcast_shape(a.shape, b.shape)
    if shape is None:
        raise ValueError(f"shapes {a.shape} and {b.shape} do not broadcast")
    av, bv = a.broadcast_to(shape), b.broadcast_to(shape)
    return Tensor(Cuda.strided_binary(av, bv, kind, op, stream), shape)


def _resolve_axes(axes, rank: int) -> list[int]:
    if axes is None or axes is Ellipsis:
        return list(range(rank))
    if isinstance(axes, int):
        axes = [axes]
    out = sorted({a + rank if a < 0 else a for a in axes})
    if len(out) != len(list(axes)) or any(a < 0 or a >= rank for a in out):
        raise ValueError(f"axes {axes} are not distinct axes of a rank-{rank} shape")
    return out


def _fill(shape, value: float, dtype: str) -> Tensor:
    n = int(np.prod(shape, dtype=np.int64)) if shape else 1
    host = f32_to_bits(np.full(n, value, dtype=np.float32), dtype)
    return Tensor(CudaStorage.store(host, dtype), shape)


# reduction.rs:126-143: resolve axes, fill empty results, else reduce_axes.
def reduction(view, axes, keep_dims, kind, op, correction, stream=None) -> Tensor:
    view = _as_view(view)
    axes = _resolve_axes(axes, view.rank)
    shape = [1 if a in axes else e for a, e in enumerate(view.shape) if keep_dims or a not in axes]
    depth = int(np.prod([view.shape[a] for a in axes], dtype=np.int64)) if axes else 1
    divisor = depth
    empty = {N.SUM: 0.0, N.RMIN: np.inf, N.RMAX: -np.inf}.get(op, 0.0) if kind == N.AXIS_FOLD else np.nan
    if kind == N.AXIS_VARIANCE:
        # Correction::divisor: n for Population, n - 1 for Sample; none -> NaN.
        divisor = depth - correction
    if depth == 0 or 0 in shape or (kind == N.AXIS_VARIANCE and divisor <= 0):
        return _fill(shape, empty, view.dtype)
    return Tensor(Cuda.reduce_axes(view, axes, kind, op, divisor, stream), shape)


# reduction.rs:288-312.
def arg_reduction(view, axis, keep_dims, op, name, stream=None) -> Tensor:
    view = _as_view(view)
    axis = axis + view.rank if axis < 0 else axis
    if not 0 <= axis < view.rank:
        raise ValueError(f"{name}: axis {axis} is out of range for shape {view.shape}")
    if view.shape[axis] == 0:
        raise ValueError(f"{name}: axis {axis} of shape {view.shape} is empty")
    shape = [1 if a == axis else e for a, e in enumerate(view.shape) if keep_dims or a != axis]
    if 0 in shape:
        return Tensor(CudaStorage.zeros("u32", 0), shape)
    return Tensor(Cuda.arg_reduce(view, axis, op, stream), shape)


# ---------------------------------------------------------------------------
# the backend
# ---------------------------------------------------------------------------
class Cuda:
    """`Backend` + `Kernels<T>` for the CUDA backend (the hot-path methods)."""

    # --- Backend (backend.rs:141-173) ---
    @staticmethod
    def strided_copy(storage: CudaStorage, shape, offset: int, strides, stream=None) -> CudaStorage:
        n = int(np.prod(shape, dtype=np.int64)) if shape else 1
        out = CudaStorage(storage.dtype, n)
        N.call("tc_strided_copy", storage.elem_bytes, len(shape), N.sizes(shape), storage.ptr, storage.len,
               offset, N.sizes(strides), out.ptr, _stream(stream))
        return out

    @staticmethod
    def _region(r) -> N.Region:
        source, shape, from_offset, from_strides, to_offset, to_strides = r
        reg = N.Region()
        reg.source, reg.source_len, reg.rank = source.ptr, source.len, len(shape)
        for k in range(len(shape)):
            reg.shape[k], reg.from_strides[k], reg.to_strides[k] = shape[k], from_strides[k], to_strides[k]
        reg.from_offset, reg.to_offset = from_offset, to_offset
        return reg

    @staticmethod
    def assemble(dtype: str, length: int, regions, stream=None) -> CudaStorage:
        """regions: (source, shape, from_offset, from_strides, to_offset, to_strides)."""
        out = CudaStorage(dtype, length)
        arr = (N.Region * max(1, len(regions)))(*[Cuda._region(r) for r in regions])
        N.call("tc_assemble", ELEM[dtype][1], out.ptr, length, arr, len(regions), _stream(stream))
        return out

    @staticmethod
    def strided_write(target: CudaStorage, region, stream=None) -> None:
        reg = Cuda._region(region)
        N.call("tc_strided_write", target.elem_bytes, target.ptr, target.len, C.byref(reg), _stream(stream))

    # --- Kernels<T>: vectors (kernels.rs:832-897) ---
    @staticmethod
    def vector_elementwise(a: CudaStorage, b: CudaStorage, op: int, stream=None) -> CudaStorage:
        if a.len != b.len:
            raise ValueError(f"elementwise: lengths {a.len} and {b.len} differ")
        out = CudaStorage(a.dtype, a.len)
        N.call("tc_elementwise", N.DTYPES[a.dtype], op, a.ptr, b.ptr, out.ptr, a.len, _stream(stream))
        return out

    @staticmethod
    def vector_broadcast(a: CudaStorage, scalar: float, op: int, scalar_left: bool, stream=None) -> CudaStorage:
        out = CudaStorage(a.dtype, a.len)
        N.call("tc_broadcast_scalar", N.DTYPES[a.dtype], op, a.ptr, float(scalar), int(scalar_left), out.ptr,
               a.len, _stream(stream))
        return out

    @staticmethod
    def vector_compare(a: CudaStorage, b: CudaStorage, op: int, stream=None) -> CudaStorage:
        if a.len != b.len:
            raise ValueError(f"compare: lengths {a.len} and {b.len} differ")
        out = CudaStorage(a.dtype, a.len)
        N.call("tc_compare", N.DTYPES[a.dtype], op, a.ptr, b.ptr, out.ptr, a.len, _stream(stream))
        return out

    @staticmethod
    def vector_compare_scalar(a: CudaStorage, scalar: float, op: int, scalar_left: bool, stream=None):
        out = CudaStorage(a.dtype, a.len)
        N.call("tc_compare_scalar", N.DTYPES[a.dtype], op, a.ptr, float(scalar), int(scalar_left), out.ptr,
               a.len, _stream(stream))
        return out

    @staticmethod
    def vector_clamp(a: CudaStorage, low: float, high: float, stream=None) -> CudaStorage:
        out = CudaStorage(a.dtype, a.len)
        N.call("tc_clamp", N.DTYPES[a.dtype], a.ptr, float(low), float(high), out.ptr, a.len, _stream(stream))
        return out

    @staticmethod
    def vector_reduce(a: CudaStorage, op: int, stream=None) -> CudaStorage:
        out = CudaStorage(a.dtype, 1)
        N.call("tc_vector_reduce", N.DTYPES[a.dtype], op, a.ptr, a.len, out.ptr, _stream(stream))
        return out

    @staticmethod
    def dot(a: CudaStorage, b: CudaStorage, stream=None) -> CudaStorage:
        out = CudaStorage(a.dtype, 1)
        N.call("tc_dot", N.DTYPES[a.dtype], a.ptr, b.ptr, a.len, out.ptr, _stream(stream))
        return out

    @staticmethod
    def vector_prefix_sum(a: CudaStorage, stream=None) -> CudaStorage:
        out = CudaStorage(a.dtype, a.len)
        N.call("tc_prefix_sum", N.DTYPES[a.dtype], a.ptr, out.ptr, a.len, _stream(stream))
        return out

    @staticmethod
    def vector_sort(a: CudaStorage, order: int, stream=None) -> CudaStorage:
        out = CudaStorage(a.dtype, a.len)
        N.call("tc_sort", N.DTYPES[a.dtype], order, a.ptr, out.ptr, a.len, _stream(stream))
        return out

    @staticmethod
    def vector_unary(a: CudaStorage, f: int, stream=None) -> CudaStorage:
        """vector_unary / matrix_unary: f an Analytic."""
        out = CudaStorage(a.dtype, a.len)
        N.call("tc_unary", N.DTYPES[a.dtype], f, a.ptr, out.ptr, a.len, _stream(stream))
        return out

    @staticmethod
    def vector_unary_dual(value: CudaStorage, tangent: CudaStorage, f: int,
                          stream=None) -> tuple[CudaStorage, CudaStorage]:
        if value.len != tangent.len:
            raise ValueError("unary_dual: value and tangent lengths differ")
        out_v, out_t = CudaStorage(value.dtype, value.len), CudaStorage(value.dtype, value.len)
        N.call("tc_unary_dual", N.DTYPES[value.dtype], f, value.ptr, tangent.ptr, out_v.ptr, out_t.ptr, value.len,
               _stream(stream))
        return out_v, out_t

    @staticmethod
    def vector_power(a: CudaStorage, b: CudaStorage, stream=None) -> CudaStorage:
        if a.len != b.len:
            raise ValueError(f"pow: lengths {a.len} and {b.len} differ")
        out = CudaStorage(a.dtype, a.len)
        N.call("tc_power", N.DTYPES[a.dtype], a.ptr, b.ptr, out.ptr, a.len, _stream(stream))
        return out

    @staticmethod
    def vector_power_scalar(a: CudaStorage, scalar: float, scalar_left: bool, stream=None) -> CudaStorage:
        out = CudaStorage(a.dtype, a.len)
        N.call("tc_power_scalar", N.DTYPES[a.dtype], a.ptr, float(scalar), int(scalar_left), out.ptr, a.len,
               _stream(stream))
        return out

    # --- windowed matrices (kernels.rs:998-1028) ---
    @staticmethod
    def correlate(input: CudaStorage, shape, window: CudaStorage, window_shape, flip: bool,
                  stream=None) -> CudaStorage:
        (r, c), (wr, wc) = shape, window_shape
        if wr > r or wc > c:
            raise ValueError(f"correlate: a {wr}x{wc} window does not fit in a {r}x{c} input")
        out = CudaStorage(input.dtype, (r - wr + 1) * (c - wc + 1))
        N.call("tc_correlate", N.DTYPES[input.dtype], r, c, wr, wc, int(flip), input.ptr, window.ptr, out.ptr,
               _stream(stream))
        return out

    @staticmethod
    def correlate_window_gradient(input: CudaStorage, shape, adjoint: CudaStorage, adjoint_shape,
                                  stream=None) -> CudaStorage:
        return Cuda.correlate(input, shape, adjoint, adjoint_shape, False, stream)

    @staticmethod
    def correlate_input_gradient(adjoint: CudaStorage, adjoint_shape, window: CudaStorage, window_shape,
                                 forward_flip: bool, stream=None) -> CudaStorage:
        (ar, ac), (wr, wc) = adjoint_shape, window_shape
        out = CudaStorage(adjoint.dtype, (ar + wr - 1) * (ac + wc - 1))
        N.call("tc_correlate_input_gradient", N.DTYPES[adjoint.dtype], ar, ac, wr, wc, int(forward_flip),
               adjoint.ptr, window.ptr, out.ptr, _stream(stream))
        return out

    @staticmethod
    def pad(input: CudaStorage, shape, pad_rows: int, pad_cols: int, stream=None) -> CudaStorage:
        r, c = shape
        out = CudaStorage(input.dtype, (r + 2 * pad_rows) * (c + 2 * pad_cols))
        N.call("tc_pad", N.DTYPES[input.dtype], r, c, pad_rows, pad_cols, input.ptr, out.ptr, _stream(stream))
        return out

    @staticmethod
    def flip(input: CudaStorage, shape, stream=None) -> CudaStorage:
        r, c = shape
        out = CudaStorage(input.dtype, r * c)
        N.call("tc_flip", N.DTYPES[input.dtype], r, c, input.ptr, out.ptr, _stream(stream))
        return out

    # --- moments and distributions (kernels.rs:1035-1070) ---
    @staticmethod
    def vector_moments(a: CudaStorage, stream=None) -> CudaStorage:
        """(mean, deviations) as a 2-element device vector."""
        out = CudaStorage(a.dtype, 2)
        N.call("tc_moments", N.DTYPES[a.dtype], a.ptr, a.len, out.ptr, _stream(stream))
        return out

    @staticmethod
    def matrix_axis_moments(a: CudaStorage, shape, axis: int, stream=None) -> tuple[CudaStorage, CudaStorage]:
        r, c = shape
        extent = r if axis == N.ROWS else c
        means, devs = CudaStorage(a.dtype, extent), CudaStorage(a.dtype, extent)
        N.call("tc_axis_moments", N.DTYPES[a.dtype], r, c, axis, a.ptr, means.ptr, devs.ptr, _stream(stream))
        return means, devs

    @staticmethod
    def vector_distribution(a: CudaStorage, family: int, statistic: int, parameters, stream=None) -> CudaStorage:
        out = CudaStorage(a.dtype, a.len)
        N.call("tc_distribution", N.DTYPES[a.dtype], family, statistic, a.ptr, a.len, float(parameters[0]),
               float(parameters[1]), out.ptr, _stream(stream))
        return out

    @staticmethod
    def matrix_axis_distribution(a: CudaStorage, shape, axis: int, family: int, statistic: int,
                                 first: CudaStorage, second: CudaStorage, stream=None) -> CudaStorage:
        r, c = shape
        out = CudaStorage(a.dtype, r * c)
        N.call("tc_axis_distribution", N.DTYPES[a.dtype], r, c, axis, family, statistic, a.ptr, first.ptr,
               second.ptr, out.ptr, _stream(stream))
        return out

    # --- products (kernels.rs:899-985) ---
    @staticmethod
    def matmul(a: CudaStorage, b: CudaStorage, rows: int, inner: int, cols: int, transposed: int = N.TRANS_NONE,
               addend: CudaStorage | None = None, stream=None) -> CudaStorage:
        """matmul / matmul_add / matmul_transposed_add: `addend` is consumed as
        the accumulator (kernels.rs:958-985)."""
        out = addend if addend is not None else CudaStorage(a.dtype, rows * cols)
        N.call("tc_matmul", N.DTYPES[a.dtype], transposed, rows, inner, cols, a.ptr, b.ptr, out.ptr,
               int(addend is not None), _stream(stream))
        return out

    @staticmethod
    def matvec(m: CudaStorage, v: CudaStorage, rows: int, cols: int, addend: CudaStorage | None = None,
               stream=None) -> CudaStorage:
        out = addend if addend is not None else CudaStorage(m.dtype, rows)
        N.call("tc_matvec", N.DTYPES[m.dtype], rows, cols, m.ptr, v.ptr, out.ptr, int(addend is not None),
               _stream(stream))
        return out

    @staticmethod
    def vecmat(v: CudaStorage, m: CudaStorage, rows: int, cols: int, stream=None) -> CudaStorage:
        out = CudaStorage(m.dtype, cols)
        N.call("tc_vecmat", N.DTYPES[m.dtype], rows, cols, v.ptr, m.ptr, out.ptr, _stream(stream))
        return out

    @staticmethod
    def transpose(m: CudaStorage, rows: int, cols: int, stream=None) -> CudaStorage:
        return Cuda.strided_copy(m, [cols, rows], 0, [1, cols], stream)

    # --- strided kernels (kernels.rs:1162-1187) ---
    @staticmethod
    def strided_binary(a: TensorView, b: TensorView, kind: int, op: int, stream=None) -> CudaStorage:
        if list(a.shape) != list(b.shape):
            raise ValueError("strided binary: the operands' shapes differ")
        out = CudaStorage(a.dtype, a.numel())
        N.call("tc_strided_binary", N.DTYPES[a.dtype], kind, op, a.rank, N.sizes(a.shape), a.storage.ptr,
               a.storage.len, a.offset, N.sizes(a.strides), b.storage.ptr, b.storage.len, b.offset,
               N.sizes(b.strides), out.ptr, _stream(stream))
        return out

    @staticmethod
    def reduce_axes(view: TensorView, axes: Sequence[int], kind: int, op: int, divisor: int,
                    stream=None) -> CudaStorage:
        results = int(np.prod([e for a, e in enumerate(view.shape) if a not in axes], dtype=np.int64))
        out = CudaStorage(view.dtype, results)
        N.call("tc_reduce_axes", N.DTYPES[view.dtype], view.rank, N.sizes(view.shape), view.storage.ptr,
               view.storage.len, view.offset, N.sizes(view.strides), len(axes), N.u32s(axes), kind, op,
               divisor, out.ptr, _stream(stream))
        return out

    @staticmethod
    def arg_reduce(view: TensorView, axis: int, op: int, stream=None) -> CudaStorage:
        results = int(np.prod([e for a, e in enumerate(view.shape) if a != axis], dtype=np.int64))
        out = CudaStorage("u32", results)
        N.call("tc_arg_reduce", N.DTYPES[view.dtype], view.rank, N.sizes(view.shape), view.storage.ptr,
               view.storage.len, view.offset, N.sizes(view.strides), axis, op,
               C.cast(C.c_void_p(out.ptr), C.POINTER(C.c_uint32)), _stream(stream))
        return out


def synchronize(stream=None) -> None:
    N.call("tc_stream_sync", _stream(stream))
