"""The C ABI without a GPU: the library loads, exports every entry point
include/tccuda.h declares, builds layout descriptors as layout.rs does, and
refuses bad arguments before touching the device (the reference's shape
checks panic before the backend is called, backend.rs:225-252)."""
from __future__ import annotations

import ctypes as C
import itertools
import re
from pathlib import Path

import numpy as np
import pytest

import oracle as O
from tensorcrate_b200 import _native as N
from tensorcrate_b200 import cuda
from util import kats

HEADER = Path(__file__).resolve().parents[1] / "include" / "tccuda.h"


def declared() -> list[str]:
    text = HEADER.read_text()
    return sorted(set(re.findall(r"^\s*(?:int|const char \*)\s*(tc_\w+)\(", text, re.M)))


def test_header_declares_the_hot_path():
    names = declared()
    for required in ["tc_strided_copy", "tc_assemble", "tc_strided_write", "tc_elementwise", "tc_strided_binary",
                     "tc_reduce_axes", "tc_arg_reduce", "tc_matmul", "tc_matvec", "tc_vecmat", "tc_adam", "tc_sgd"]:
        assert required in names


def test_library_exports_every_declared_symbol():
    lib = N.lib()
    missing = [n for n in declared() if not hasattr(lib, n)]
    assert not missing, missing
    assert b"sm_100a" in lib.tc_build_info()


@pytest.mark.parametrize("k", kats("coalesce"), ids=lambda k: k["id"])
def test_coalesce_kats(k):
    shape, strides = cuda.coalesce(k["shape"], *k["strides"])
    assert shape == k["expect_shape"] and strides == k["expect_strides"]


def test_coalesce_agrees_with_the_oracle():
    rng = np.random.default_rng(5)
    for _ in range(300):
        rank = int(rng.integers(0, 7))
        shape = [int(rng.integers(1, 5)) for _ in range(rank)]
        ops = []
        for _ in range(int(rng.integers(1, 4))):
            perm = rng.permutation(rank)
            st = cuda.contiguous_strides([shape[p] for p in perm])
            s = [0] * rank
            for i, p in enumerate(perm):
                s[p] = st[i] if rng.random() > 0.2 else 0
            ops.append(s)
        got = cuda.coalesce(shape, *ops)
        r = C.c_uint32()
        osh = (C.c_size_t * 6)()
        ost = (C.c_size_t * 18)()
        O.call("orc_coalesce", rank, O.sizes(shape), len(ops), O.sizes([x for s in ops for x in s]), C.byref(r), osh,
               ost)
        want = (list(osh[: r.value]), [list(ost[o * r.value:(o + 1) * r.value]) for o in range(len(ops))])
        assert got == want


@pytest.mark.parametrize("k", kats("broadcast_shape"), ids=lambda k: k["id"])
def test_broadcast_shape_kats(k):
    assert cuda.broadcast_shape(k["left"], k["right"]) == k["expect"]


@pytest.mark.parametrize("k", kats("broadcast_strides"), ids=lambda k: k["id"])
def test_broadcast_strides_kats(k):
    assert cuda.broadcast_strides(k["shape"], k["strides"], k["target"]) == k["expect"]


@pytest.mark.parametrize("k", kats("permute"), ids=lambda k: k["id"])
def test_permute_is_a_stride_rewrite(k):
    v = cuda.TensorView(storage=None, shape=k["shape"], strides=cuda.contiguous_strides(k["shape"]))
    p = v.permute(k["axes"])
    assert p.shape == k["expect_shape"] and p.strides == k["expect_strides"]
    assert not p.is_contiguous()


def _status(name, *args):
    st = getattr(N.lib(), name)(*args)
    return st, N.last_error()


def test_out_of_range_layouts_are_refused_on_the_host():
    fake = C.c_void_p(0x1000)
    st, msg = _status("tc_strided_copy", 4, 2, N.sizes([2, 3]), fake, 5, 0, N.sizes([3, 1]), fake, None)
    assert st == N.ERANGE and "reaches" in msg
    st, _ = _status("tc_strided_copy", 3, 1, N.sizes([2]), fake, 5, 0, N.sizes([1]), fake, None)
    assert st == N.EINVAL
    st, _ = _status("tc_strided_copy", 4, 7, N.sizes([1] * 7), fake, 5, 0, N.sizes([1] * 7), fake, None)
    assert st == N.EINVAL


def test_bad_operations_are_refused_on_the_host():
    fake = C.c_void_p(0x1000)
    u32 = C.cast(fake, C.POINTER(C.c_uint32))
    shape, strides = N.sizes([2, 3]), N.sizes([3, 1])
    assert _status("tc_reduce_axes", 0, 2, shape, fake, 6, 0, strides, 2, N.u32s([1, 0]), 0, 0, 0, fake, None)[0] == N.EINVAL
    assert _status("tc_reduce_axes", 0, 2, shape, fake, 6, 0, strides, 1, N.u32s([1]), 5, 0, 0, fake, None)[0] == N.EINVAL
    assert _status("tc_arg_reduce", 0, 2, N.sizes([2, 0]), fake, 6, 0, strides, 1, 2, u32, None)[0] == N.EINVAL
    assert _status("tc_arg_reduce", 0, 2, shape, fake, 6, 0, strides, 1, 0, u32, None)[0] == N.EINVAL
    assert _status("tc_clamp", 0, fake, 2.0, 1.0, fake, 4, None)[0] == N.EINVAL
    assert _status("tc_matmul", 0, 7, 2, 2, 2, fake, fake, fake, 0, None)[0] == N.EINVAL
    assert _status("tc_elementwise", 0, 9, fake, fake, fake, 4, None)[0] == N.EINVAL
    assert _status("tc_strided_binary", 0, 1, 11, 2, shape, fake, 6, 0, strides, fake, 6, 0, strides, fake, None)[0] == N.EINVAL
    assert _status("tc_elementwise", 9, 0, fake, fake, fake, 4, None)[0] == N.EINVAL


def test_empty_work_touches_nothing():
    # Zero elements: every call returns at once, before any device call.
    assert _status("tc_elementwise", 0, 0, None, None, None, 0, None)[0] == N.OK
    assert _status("tc_strided_copy", 4, 2, N.sizes([0, 3]), None, 0, 0, N.sizes([3, 1]), None, None)[0] == N.OK
    assert _status("tc_matmul", 0, 0, 0, 4, 4, None, None, None, 0, None)[0] == N.OK


def test_no_host_code_calls_a_device_only_function():
    """nvcc compiles a __device__-only function called from host code into a
    stand-in that exits the process; no object of the library may contain
    one (it would end the caller without an error)."""
    import subprocess
    objs = sorted((Path(__file__).resolve().parents[1] / "tensorcrate_b200" / "_build").glob("*.o"))
    if not objs:
        pytest.skip("library objects not built here")
    for o in objs:
        out = subprocess.run(["nm", "-u", str(o)], capture_output=True, text=True).stdout.split()
        assert "exit" not in out, f"{o.name} references exit"


def test_other_methods_refuse_bad_arguments_on_the_host():
    """The trait methods beyond the configs check their enums and shapes
    before any device call: a bad Analytic, SortOrder, Axis, Family or
    Statistic, a window larger than its input, a place missing."""
    fake = C.c_void_p(0x1000)
    assert _status("tc_unary", N.F32, 14, fake, fake, 4, None)[0] == N.EINVAL
    assert _status("tc_unary_dual", N.F32, 99, fake, fake, fake, fake, 4, None)[0] == N.EINVAL
    assert _status("tc_sort", N.F32, 2, fake, fake, 4, None)[0] == N.EINVAL
    assert _status("tc_sort", 9, N.ASCENDING, fake, fake, 4, None)[0] == N.EINVAL
    assert _status("tc_correlate", N.F32, 2, 3, 3, 1, 0, fake, fake, fake, None)[0] == N.EINVAL
    assert _status("tc_correlate", N.F32, 2, 3, 0, 1, 0, fake, fake, fake, None)[0] == N.EINVAL
    assert _status("tc_correlate_input_gradient", N.F32, 0, 3, 1, 1, 0, fake, fake, fake, None)[0] == N.EINVAL
    assert _status("tc_axis_moments", N.F32, 2, 3, 2, fake, fake, fake, None)[0] == N.EINVAL
    assert _status("tc_distribution", N.F32, 2, N.PDF, fake, 4, 0.0, 1.0, fake, None)[0] == N.EINVAL
    assert _status("tc_distribution", N.F32, N.NORMAL, 3, fake, 4, 0.0, 1.0, fake, None)[0] == N.EINVAL
    assert _status("tc_axis_distribution", N.F32, 2, 2, 5, N.NORMAL, N.CDF, fake, fake, fake, fake, None)[0] == N.EINVAL
    assert _status("tc_row_moments", N.F32, None, 4, 4, fake, fake, None)[0] == N.EINVAL
    assert _status("tc_fused_sum", N.F32, 2, 2, None, 0, None, 0, 7, fake, None)[0] == N.EINVAL
    assert _status("tc_matmul_program", N.F32, 2, 2, 2, fake, fake, None, 0, None, 0, None, None, 0, None)[0] == N.EINVAL


def test_empty_inputs_of_the_other_methods_touch_nothing():
    assert _status("tc_prefix_sum", N.F32, None, None, 0, None)[0] == N.OK
    assert _status("tc_sort", N.F32, N.DESCENDING, None, None, 0, None)[0] == N.OK
    assert _status("tc_unary", N.BF16, N.EXP, None, None, 0, None)[0] == N.OK
    assert _status("tc_power", N.F16, None, None, None, 0, None)[0] == N.OK
    assert _status("tc_flip", N.F32, 0, 5, None, None, None)[0] == N.OK
    assert _status("tc_distribution", N.F32, N.NORMAL, N.PPF, None, 0, 0.0, 1.0, None, None)[0] == N.OK
    assert _status("tc_axis_moments", N.F32, 0, 4, N.ROWS, None, None, None, None)[0] == N.OK
