"""Failure detection on the device without a fault: the tensor-core GEMM's
pipeline waits are bounded, and a wait that runs out makes the kernel record
the fault, drain what it has in flight, free its tensor memory and return.
The reference reports GPU errors at the next sync and panics
(src/metal/mod.rs:17-21, src/tensors/backend.rs:418-426); here the status
is read with tc_device_status.  The test shortens the limit to 1 ns so that
waits give up, then checks that the context stays usable: with the default
limit the same product is right again."""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

import oracle as O
from tensorcrate_b200 import _native as N
from tensorcrate_b200 import cuda
from util import uniform

pytestmark = pytest.mark.gpu


def _status():
    fault = C.c_int(0)
    st = N.lib().tc_device_status(C.byref(fault))
    return st, fault.value


def test_a_gemm_wait_that_runs_out_returns_and_is_reported(device):
    m = k = n = 4096  # long enough that a wait cannot complete within its first retry
    a = O.narrow(uniform((m, k), 1), "bf16")
    b = O.narrow(uniform((k, n), 2), "bf16")
    da, db = cuda.CudaStorage.store(a, "bf16"), cuda.CudaStorage.store(b, "bf16")
    band = 8  # the oracle checks the first rows of the product
    want = O.widen(O.matmul("bf16", 0, band, k, n, a[:band], b), "bf16")
    assert _status() == (N.OK, 0)
    try:
        N.call("tc_set_wait_limit", 1)
        c = cuda.CudaStorage("bf16", m * n)
        N.call("tc_matmul", N.BF16, 0, m, k, n, da.ptr, db.ptr, c.ptr, 0, None)
        N.call("tc_stream_sync", None)  # the kernel returned: the context is alive
        st, fault = _status()
        assert st == N.ETIMEOUT and fault == 1
        assert "gave up" in N.last_error()
    finally:
        N.call("tc_set_wait_limit", 0)
        N.call("tc_device_status_reset")
    assert _status() == (N.OK, 0)
    got = O.widen(cuda.Cuda.matmul(da, db, m, k, n).as_slice()[: band * n], "bf16")
    assert np.max(np.abs(got - want)) <= 2.0 ** -7 * 2 * max(1.0, float(np.max(np.abs(want))))
    assert _status() == (N.OK, 0)
