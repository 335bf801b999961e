"""tc_vecmat_noalloc: the vecmat for callers that cannot allocate device
memory -- those whose GPU memory another allocator has already claimed (a
framework's caching allocator, a fixed arena), where a cudaMalloc from the
library would fail or break that allocator's budget, and those under a hard
latency budget, where cudaMalloc may block and synchronise the device.  Its
row-split partial sums live in a static device array instead.  It must give
the same bits as tc_vecmat on the same inputs, on two calls in a row (the
second with other inputs, so stale partials would show), make no allocation
and ask for no scratch while it runs (the library's own counters), and
refuse a shape whose partials do not fit the array.  This file is named to
be collected last, so that the suite also runs it after every other test has
used the library; run alone, it is the first user of the library in its
process."""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

from tensorcrate_b200 import _native as N
from util import normal

pytestmark = pytest.mark.gpu

SCRATCH_BYTES = 1 << 20
CODES = {"f32": 0, "f16": 1, "bf16": 2}


def _bits(values: np.ndarray, dtype: str) -> np.ndarray:
    """Element bits of `values` in `dtype` (bf16 by truncation: any bits do)."""
    if dtype == "f32":
        return values.astype(np.float32)
    if dtype == "f16":
        return values.astype(np.float16).view(np.uint16)
    return (values.astype(np.float32).view(np.uint32) >> 16).astype(np.uint16)


class Buffer:
    """A device buffer from the library's own allocator."""

    def __init__(self, nbytes: int):
        self.nbytes = nbytes
        self.ptr = C.c_void_p()
        N.call("tc_malloc", C.byref(self.ptr), nbytes)

    def upload(self, host: np.ndarray) -> "Buffer":
        host = np.ascontiguousarray(host)
        assert host.nbytes <= self.nbytes
        N.call("tc_memcpy_h2d", self.ptr, host.ctypes.data_as(C.c_void_p), host.nbytes, None)
        return self

    def download(self, like: np.ndarray) -> np.ndarray:
        out = np.empty_like(like)
        N.call("tc_stream_sync", None)
        N.call("tc_memcpy_d2h", out.ctypes.data_as(C.c_void_p), self.ptr, out.nbytes, None)
        return out

    def free(self) -> None:
        N.call("tc_free", self.ptr)


def _sm_count() -> int:
    n = C.c_int(0)
    N.call("tc_sm_count", C.byref(n))
    return n.value


def _alloc_counts() -> tuple[int, int]:
    """(cudaMalloc calls the library made, scratch requests) so far."""
    a, s = C.c_uint64(0), C.c_uint64(0)
    N.call("tc_alloc_counts", C.byref(a), C.byref(s))
    return a.value, s.value


def _shares(rows: int, cols: int, dtype: str, sms: int | None = None) -> int:
    """The row split tc_vecmat picks for a 16-byte-aligned matrix on a GPU
    with `sms` SMs (the current device's when not given)."""
    sms = _sm_count() if sms is None else sms
    cpt = 16 // (4 if dtype == "f32" else 2)
    if cols % cpt:
        cpt = 1
    col_blocks = (cols + 32 * cpt - 1) // (32 * cpt)
    shares = 1
    while col_blocks * shares < 4 * sms and rows // (shares * 2) >= 64:
        shares *= 2
    return shares


CASES = [
    ("f32", 4096, 1024),   # 32 row shares, 16-byte packs
    ("f32", 3000, 1001),   # 16 shares, one column per thread
    ("bf16", 8192, 1536),  # 128 shares, 768 KiB of partials
    ("f16", 2048, 512),
    ("f32", 100, 4096),    # no split: the array is not used
]


@pytest.mark.parametrize("dtype,rows,cols", CASES, ids=lambda v: str(v))
def test_matches_vecmat_on_two_calls_in_a_row(device, dtype, rows, cols):
    assert _shares(rows, cols, dtype) * cols * 4 <= SCRATCH_BYTES
    code = CODES[dtype]
    m = _bits(normal((rows, cols), seed=rows + cols), dtype)
    xs = [_bits(normal(rows, seed=s), dtype) for s in (11, 12)]
    y_like = np.zeros(cols, dtype=m.dtype)
    dm = Buffer(m.nbytes).upload(m)
    dx = [Buffer(x.nbytes).upload(x) for x in xs]
    got = [Buffer(y_like.nbytes) for _ in xs]
    want = [Buffer(y_like.nbytes) for _ in xs]
    try:
        # Two calls in a row on one stream, then the allocating entry point.
        # The library allocates nothing and asks for no scratch meanwhile
        # (its first call on a device only looks the array's address up).
        before = _alloc_counts()
        for x, y in zip(dx, got):
            N.call("tc_vecmat_noalloc", code, rows, cols, x.ptr, dm.ptr, y.ptr, None)
        N.call("tc_stream_sync", None)
        assert _alloc_counts() == before
        for x, y in zip(dx, want):
            N.call("tc_vecmat", code, rows, cols, x.ptr, dm.ptr, y.ptr, None)
        for g, w in zip(got, want):
            a, b = g.download(y_like), w.download(y_like)
            assert np.array_equal(a.view(np.uint8), b.view(np.uint8))
        # The two inputs give different sums: the second call did its own work.
        assert not np.array_equal(got[0].download(y_like), got[1].download(y_like))
    finally:
        for b in [dm, *dx, *got, *want]:
            b.free()


def test_refuses_a_split_larger_than_the_array(device):
    dtype, rows, cols = "bf16", 16384, 2304  # 128 shares x 2304 columns x 4 bytes
    assert _shares(rows, cols, dtype) * cols * 4 > SCRATCH_BYTES
    m = Buffer(rows * cols * 2)
    x = Buffer(rows * 2)
    y = Buffer(cols * 2).upload(np.full(cols, 0x3F80, dtype=np.uint16))
    try:
        status = N.lib().tc_vecmat_noalloc(CODES[dtype], rows, cols, x.ptr, m.ptr, y.ptr, None)
        assert status == N.ERANGE
        assert "static scratch" in N.last_error()
        # Refused before any launch: the output is untouched.
        assert (y.download(np.zeros(cols, dtype=np.uint16)) == 0x3F80).all()
    finally:
        for b in (m, x, y):
            b.free()
