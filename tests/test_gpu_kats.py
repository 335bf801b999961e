"""The reference's known answers (tests/golden/reference_kats.json) through
the CUDA kernels."""
from __future__ import annotations

import numpy as np
import pytest

import oracle as O
from tensorcrate_b200 import cuda
from tensorcrate_b200 import _native as N
from util import expand, kats, same_floats

pytestmark = pytest.mark.gpu


def _tensor(k):
    vals = np.array(expand(k["input"]), dtype=np.float32)
    return cuda.Tensor(cuda.CudaStorage.store(O.narrow(vals, k["dtype"]), k["dtype"]), k["shape"])


@pytest.mark.parametrize("k", kats("reduce"), ids=lambda k: k["id"])
def test_reduce_kats(device, k):
    t = _tensor(k)
    out = cuda.Cuda.reduce_axes(t.view(), k["axes"], k["reduction"], k["op"], k["divisor"])
    assert same_floats(O.widen(out.as_slice(), k["dtype"]), expand(k["expect"])), k["source"]


@pytest.mark.parametrize("k", kats("arg"), ids=lambda k: k["id"])
def test_arg_kats(device, k):
    t = _tensor(k)
    out = cuda.Cuda.arg_reduce(t.view(), k["axis"], k["op"])
    assert list(out.as_slice()) == k["expect"], k["source"]


@pytest.mark.parametrize("k", kats("strided_copy"), ids=lambda k: k["id"])
def test_strided_copy_kats(device, k):
    s = cuda.CudaStorage.store(np.array(k["input"], np.uint32), "u32")
    out = cuda.Cuda.strided_copy(s, k["shape"], k["offset"], k["strides"])
    assert list(out.as_slice()) == k["expect"]


@pytest.mark.parametrize("k", kats("assemble"), ids=lambda k: k["id"])
def test_assemble_kats(device, k):
    s = cuda.CudaStorage.store(np.array(k["input"], np.uint32), "u32")
    regions = [(s, d["shape"], d["from_offset"], d["from_strides"], d["to_offset"], d["to_strides"])
               for d in k["regions"]]
    out = cuda.Cuda.assemble("u32", k["length"], regions)
    assert list(out.as_slice()) == k["expect"]


@pytest.mark.parametrize("k", kats("elementwise"), ids=lambda k: k["id"])
def test_elementwise_kats(device, k):
    a = cuda.CudaStorage.store(O.narrow(expand(k["a"]), k["dtype"]), k["dtype"])
    b = cuda.CudaStorage.store(O.narrow(expand(k["b"]), k["dtype"]), k["dtype"])
    out = cuda.Cuda.vector_elementwise(a, b, k["op"])
    assert same_floats(O.widen(out.as_slice(), k["dtype"]), expand(k["expect"]))


def test_sgd_kat(device):
    (k,) = kats("sgd")
    p = cuda.CudaStorage.store(np.array(k["p"], np.float32), "f32")
    g = cuda.CudaStorage.store(np.array(k["g"], np.float32), "f32")
    N.call("tc_sgd", 0, 2, p.ptr, g.ptr, k["rate"], None)
    assert list(p.as_slice()) == [np.float32(1.0) - np.float32(0.05), np.float32(-2.0) - np.float32(0.4)]


@pytest.mark.parametrize("k", kats("adam_first"), ids=lambda k: k["id"])
def test_adam_first_step_kat(device, k):
    coef = O.adam_coefficients("f32", k["rate"], 0.9, 0.999, 1e-8, 1)
    p = cuda.CudaStorage.store(np.array(k["p"], np.float32), "f32")
    g = cuda.CudaStorage.store(np.array(k["g"], np.float32), "f32")
    m, v = cuda.CudaStorage.zeros("f32", 1), cuda.CudaStorage.zeros("f32", 1)
    N.call("tc_adam", 0, 1, p.ptr, g.ptr, m.ptr, v.ptr, 0, *coef, None)
    assert abs(p.as_slice()[0] - k["expect"][0]) <= k["tol"]
