"""Threads and streams at the boundary.  The reference's Metal objects are
thread-affine (src/tensors/backend.rs:410-412): each thread has its own
device and queue.  Here each thread gets a context (tc_ctx_create) whose
stream keys its own scratch, ticket counters and pool frees, so two threads
running the split reductions and the split vecmat at the same time, each on
its own stream, get the bits they get alone.  Also: the pool's stream-ordered
frees hand a block back in the freeing stream's order."""
from __future__ import annotations

import ctypes as C
import threading

import numpy as np
import pytest

from tensorcrate_b200 import _native as N
from tensorcrate_b200 import cuda
from util import normal

pytestmark = pytest.mark.gpu

ITERATIONS = 100


class Context:
    def __init__(self):
        self.handle = C.c_void_p()
        N.call("tc_ctx_create", 0, C.byref(self.handle))
        s = C.c_void_p()
        N.call("tc_ctx_stream", self.handle, C.byref(s))
        self.stream = s

    def close(self):
        N.call("tc_ctx_destroy", self.handle)


def _work(seed: int):
    """One thread's inputs and the calls it makes: a row sum whose few long
    rows are split over many warps (partials merged by ticket), a column max
    whose tall tiles are split over blocks (ticketed merge), and a vecmat
    whose rows are split (partials in scratch, then a finish kernel)."""
    rows_x = normal((8, 1 << 20), seed)
    cols_x = normal((1 << 16, 256), seed + 1)
    vx, vm = normal(8192, seed + 2), normal((8192, 512), seed + 3)
    d = {k: cuda.CudaStorage.store(v.ravel(), "f32") for k, v in
         (("rows", rows_x), ("cols", cols_x), ("vx", vx), ("vm", vm))}

    def calls(outs, sp):
        lib = N.lib()
        N.check("sum", lib.tc_reduce_axes(N.F32, 2, N.sizes([8, 1 << 20]), d["rows"].ptr, 8 << 20, 0,
                                          N.sizes([1 << 20, 1]), 1, N.u32s([1]), N.AXIS_FOLD, N.SUM, 0,
                                          outs[0].ptr, sp))
        N.check("max", lib.tc_reduce_axes(N.F32, 2, N.sizes([1 << 16, 256]), d["cols"].ptr, 1 << 24, 0,
                                          N.sizes([256, 1]), 1, N.u32s([0]), N.AXIS_FOLD, N.RMAX, 0,
                                          outs[1].ptr, sp))
        N.check("vecmat", lib.tc_vecmat(N.F32, 8192, 512, d["vx"].ptr, d["vm"].ptr, outs[2].ptr, sp))
    return d, calls


def _outs():
    return [cuda.CudaStorage("f32", 8), cuda.CudaStorage("f32", 256), cuda.CudaStorage("f32", 512)]


def test_two_threads_on_their_own_streams_get_the_serial_bits(device):
    ctxs = [Context(), Context()]
    work = [_work(100), _work(200)]
    try:
        # Alone, one after the other: the reference bits.
        want = []
        for (d, calls), ctx in zip(work, ctxs):
            outs = _outs()
            calls(outs, ctx.stream)
            N.call("tc_stream_sync", ctx.stream)
            want.append([o.as_slice() for o in outs])
        assert not np.array_equal(want[0][0], want[1][0])
        # Both threads at once, each on its own stream, many times.
        results = [[_outs() for _ in range(ITERATIONS)] for _ in ctxs]
        errors = []
        start = threading.Barrier(2)

        def run(t):
            try:
                start.wait()
                d, calls = work[t]
                for outs in results[t]:
                    calls(outs, ctxs[t].stream)
                N.call("tc_stream_sync", ctxs[t].stream)
            except Exception as e:  # reported below
                errors.append(e)

        threads = [threading.Thread(target=run, args=(t,)) for t in range(2)]
        for t in threads:
            t.start()
        for t in threads:
            t.join()
        assert not errors, errors
        for t in range(2):
            for i, outs in enumerate(results[t]):
                for k, o in enumerate(outs):
                    assert np.array_equal(o.as_slice().view(np.uint32), want[t][k].view(np.uint32)), (t, i, k)
    finally:
        for c in ctxs:
            c.close()


def test_stream_ordered_frees(device):
    ctx = Context()
    size = (6 << 20) - 4096  # a size class of its own here (6 MiB)
    try:
        p = C.c_void_p()
        N.call("tc_malloc_async", C.byref(p), size, ctx.stream)
        first = p.value
        x = cuda.CudaStorage.store(normal(1 << 18, 3), "f32")
        # A copy still queued on the context's stream reads the block when it
        # is freed there: a request on the same stream may take it at once.
        N.call("tc_memcpy_d2d", first, x.ptr, 1 << 20, ctx.stream)
        N.call("tc_free_async", first, ctx.stream)
        q = C.c_void_p()
        N.call("tc_malloc_async", C.byref(q), size, ctx.stream)
        assert q.value == first
        N.call("tc_free_async", q.value, ctx.stream)
        N.call("tc_stream_sync", ctx.stream)
        # Once the stream has drained, a request without a stream takes it.
        r = C.c_void_p()
        N.call("tc_malloc", C.byref(r), size)
        assert r.value == first
        N.call("tc_free", r.value)
    finally:
        ctx.close()
