"""The strided layout copy (Backend::strided_copy / assemble / strided_write,
backend.rs:141-173) against the oracle: bit-exact for every element width,
layout and the permute/slice/split/concat/stack/write_slice uses of
tests/nd_tensor.rs, and config 3's pattern at full size through a
size-independent round trip."""
from __future__ import annotations

import itertools

import numpy as np
import pytest

import oracle as O
from tensorcrate_b200 import cuda
from util import integral, normal

pytestmark = pytest.mark.gpu

WIDTHS = {1: np.uint8, 2: np.uint16, 4: np.uint32, 8: np.uint64}


def _store_bits(values: np.ndarray) -> cuda.CudaStorage:
    # A storage of the right element width; the copy moves bits only.
    width = values.dtype.itemsize
    dtype = {2: "f16", 4: "u32"}.get(width)
    if dtype is None:
        raise ValueError(width)
    return cuda.CudaStorage.store(values.view({2: np.uint16, 4: np.uint32}[width]), dtype)


def _copy_bits(values, shape, offset, strides, elem):
    """strided copy of raw elements of `elem` bytes through the C ABI."""
    import ctypes as C
    from tensorcrate_b200 import _native as N
    raw = np.ascontiguousarray(values)
    n_src = raw.nbytes // elem
    src = cuda.CudaStorage("u32", (raw.nbytes + 3) // 4)
    N.call("tc_memcpy_h2d", src.ptr, raw.ctypes.data, raw.nbytes, None)
    n = int(np.prod(shape, dtype=np.int64)) if shape else 1
    dst = cuda.CudaStorage("u32", (n * elem + 3) // 4 + 1)
    N.call("tc_strided_copy", elem, len(shape), N.sizes(shape), src.ptr, n_src, offset, N.sizes(strides), dst.ptr,
           None)
    out = np.empty(n * elem, np.uint8)
    N.call("tc_stream_sync", None)
    N.call("tc_memcpy_d2h", out.ctypes.data, dst.ptr, n * elem, None)
    return out


@pytest.mark.parametrize("elem", [1, 2, 4, 8, 16])
def test_every_element_width_copies_exactly(device, elem):
    """tests/nd_tensor.rs:712: the copy is defined for every width."""
    rng = np.random.default_rng(elem)
    shape = [3, 5, 7, 4]
    n = int(np.prod(shape))
    src = rng.integers(0, 256, (n + 8) * elem, dtype=np.uint8).view(np.dtype((np.void, elem)))
    base = cuda.contiguous_strides(shape)
    for perm in [(0, 1, 2, 3), (3, 2, 1, 0), (1, 3, 0, 2), (2, 0, 3, 1)]:
        pshape = [shape[p] for p in perm]
        pstr = [base[p] for p in perm]
        for offset in (0, 3):
            got = _copy_bits(src, pshape, offset, pstr, elem)
            want = O.strided_copy(src, pshape, offset, pstr)
            assert got.tobytes() == want.tobytes(), (perm, offset)


@pytest.mark.parametrize("dtype", ["f32", "f16", "bf16"])
def test_permutations_slices_and_broadcasts(device, dtype):
    rng = np.random.default_rng(11)
    shape = [4, 6, 5, 8, 3]
    x = O.narrow(normal(shape, 1), dtype)
    s = cuda.CudaStorage.store(x, dtype)
    base = cuda.contiguous_strides(shape)
    for _ in range(40):
        perm = list(rng.permutation(5))
        pshape, pstr = [shape[p] for p in perm], [base[p] for p in perm]
        # a random slice of each axis
        offset = 0
        sl = []
        for a in range(5):
            lo = int(rng.integers(0, pshape[a]))
            hi = int(rng.integers(lo + 1, pshape[a] + 1))
            offset += lo * pstr[a]
            sl.append(hi - lo)
        got = cuda.Cuda.strided_copy(s, sl, offset, pstr).as_slice()
        want = O.strided_copy(x, sl, offset, pstr)
        assert np.array_equal(got, want), (perm, sl)
    # zero strides (a broadcast view made contiguous, tests/broadcast_reduce.rs:206-215)
    bias = O.narrow(normal([4], 2), dtype)
    b = cuda.CudaStorage.store(bias, dtype)
    got = cuda.Cuda.strided_copy(b, [2, 3, 4], 0, [0, 0, 1]).as_slice()
    assert np.array_equal(got, np.tile(bias, 6))


def test_concat_stack_and_write_slice(device):
    """tests/nd_tensor.rs:143-176, 229-292: views, splits, concat, stack and
    write_slice reproduce the index arithmetic exactly."""
    shape = [4, 5, 6]
    t = cuda.Tensor.from_numpy(integral(120).reshape(shape), "f32")
    host = integral(120).reshape(shape)
    narrow = t.view().slice(1, 1, 4)
    assert narrow.offset == 6 and narrow.shape == [4, 3, 6]
    assert np.array_equal(narrow.contiguous().to_numpy(), host[:, 1:4, :])
    pieces = t.view().split(2, [1, 2, 3])
    assert np.array_equal(cuda.Tensor.concat(pieces, 2).to_numpy(), host)
    for axis in range(3):
        b = host * 10
        stored = cuda.Tensor.from_numpy(np.ascontiguousarray(np.transpose(b, (2, 1, 0))), "f32")
        b_view = stored.view().permute([2, 1, 0])
        joined = cuda.Tensor.concat([t.view(), b_view], axis).to_numpy()
        assert np.array_equal(joined, np.concatenate([host, b], axis))
    for axis in range(4):
        stacked = cuda.Tensor.stack([t, cuda.Tensor.from_numpy(-host, "f32")], axis).to_numpy()
        assert np.array_equal(stacked, np.stack([host, -host], axis))
    cache = cuda.Tensor.from_numpy(np.zeros([2, 2, 5, 3], np.float32), "f32")
    step = integral(12).reshape(2, 3, 2)
    source = cuda.Tensor.from_numpy(step, "f32").view().permute([0, 2, 1]).unsqueeze(2)
    cache.write_slice(2, 3, source)
    want = np.zeros([2, 2, 5, 3], np.float32)
    want[:, :, 3, :] = np.transpose(step, (0, 2, 1))
    assert np.array_equal(cache.to_numpy(), want)


def test_attention_heads_round_trip_exactly(device):
    """tests/nd_tensor.rs:337-354."""
    batch, time, model, heads = 2, 5, 12, 3
    qkv_host = integral(batch * time * 3 * model).reshape(batch, time, 3 * model)
    qkv = cuda.Tensor.from_numpy(qkv_host, "f32")
    parts = []
    for k, part in enumerate(qkv.view().chunk(2, 3)):
        # [B, T, D] -> [B, T, H, Dh] (a stride split) -> [B, H, T, Dh]
        v = cuda.TensorView(part.storage, [batch, time, heads, model // heads],
                            [part.strides[0], part.strides[1], model // heads, 1], part.offset)
        parts.append(v.permute([0, 2, 1, 3]).contiguous())
        want = qkv_host[:, :, k * model:(k + 1) * model].reshape(batch, time, heads, -1).transpose(0, 2, 1, 3)
        assert np.array_equal(parts[-1].to_numpy(), want)
    merged = [cuda.Tensor(p.view().permute([0, 2, 1, 3]).contiguous().storage, [batch, time, model]) for p in parts]
    assert np.array_equal(cuda.Tensor.concat(merged, 2).to_numpy(), qkv_host)


def _config3(dtype_shape=(8, 16, 128, 64, 32), scale=1):
    shape = [s // scale if i in (0, 2) else s for i, s in enumerate(dtype_shape)]
    return shape


@pytest.mark.parametrize("scale", [8, 1])
def test_config3_permute_slice_split_concat(device, scale):
    """Config 3: f16 [8,16,128,64,32] permuted (0,3,1,4,2), made contiguous,
    sliced [:, 8:, :, :32, :], split in 4 along axis 1 and concatenated back.
    At 1/8 size against the oracle bit for bit; at full size through the
    round trip (the inverse permutation restores the input exactly, and the
    concatenation equals the slice made contiguous)."""
    shape = _config3(scale=scale)
    n = int(np.prod(shape))
    x = O.narrow(normal(n, 3), "f16")
    t = cuda.Tensor(cuda.CudaStorage.store(x, "f16"), shape)
    perm = [0, 3, 1, 4, 2]
    p = t.view().permute(perm).contiguous()
    sl = p.view().slice(1, 8, p.shape[1]).slice(3, 0, 32)
    pieces = sl.chunk(1, 4)
    joined = cuda.Tensor.concat(pieces, 1)
    whole = sl.contiguous()
    assert np.array_equal(joined.to_numpy(), whole.to_numpy())
    inverse = list(np.argsort(perm))
    back = p.view().permute(inverse).contiguous()
    assert np.array_equal(back.storage.as_slice(), x)
    if scale > 1:
        want = O.strided_copy(x, p.shape, 0, [cuda.contiguous_strides(shape)[a] for a in perm])
        assert np.array_equal(p.storage.as_slice(), want)
        sl_host = want.reshape(p.shape)[:, 8:, :, :32, :]
        assert np.array_equal(joined.to_numpy(), sl_host)


def _oracle_assemble(elem, length, regions_host):
    """The Host's assemble (backend.rs:303-323): regions written in order."""
    import ctypes as C
    from tensorcrate_b200 import _native as N
    arr = (N.Region * len(regions_host))()
    keep = []
    for reg, (src, shape, fo, fs, to, ts) in zip(arr, regions_host):
        keep.append(src)
        reg.source, reg.source_len, reg.rank = src.ctypes.data, src.size, len(shape)
        for k in range(len(shape)):
            reg.shape[k], reg.from_strides[k], reg.to_strides[k] = shape[k], fs[k], ts[k]
        reg.from_offset, reg.to_offset = fo, to
    out = np.empty(length, keep[0].dtype)
    O.call("orc_assemble", elem, O.ptr(out), length, C.cast(arr, C.c_void_p), len(regions_host))
    return out


def test_assemble_overlapping_regions_keeps_the_last_write(device):
    """Regions that overlap in the target are written in order, as the
    Host's sequential strided writes leave them: the later region wins."""
    a, b, c = integral(64), integral(64, 100), integral(48, 300)
    host = [(a, [64], 0, [1], 0, [1]), (b, [8, 8], 0, [8, 1], 16, [8, 1]), (c, [48], 0, [1], 40, [1])]
    dev = [(cuda.CudaStorage.store(s, "f32"), sh, fo, fs, to, ts) for s, sh, fo, fs, to, ts in host]
    got = cuda.Cuda.assemble("f32", 96, dev).as_slice()
    assert np.array_equal(got[:88], _oracle_assemble(4, 96, host)[:88])


@pytest.mark.parametrize("dtype", ["f32", "f16"])
def test_concat_of_many_pieces_in_one_launch(device, dtype):
    """A concatenation of up to 11 pieces of differing widths (16-byte
    units, odd lengths that copy element by element, a transposed view):
    the batched plain copies and the transposes together give the Host's
    result."""
    rng = np.random.default_rng(4)
    widths = [8, 16, 3, 32, 5, 64, 8, 1, 24, 40, 7]
    pieces, host = [], []
    for i, w in enumerate(widths):
        x = O.narrow(integral(6 * w, 50 * i), dtype).reshape(6, w)
        if i == 3:  # a transposed piece: stored [w, 6], viewed [6, w]
            stored = np.ascontiguousarray(x.T)
            pieces.append(cuda.Tensor(cuda.CudaStorage.store(stored.reshape(-1), dtype), [w, 6]).view().permute([1, 0]))
        else:
            pieces.append(cuda.Tensor(cuda.CudaStorage.store(x.reshape(-1), dtype), [6, w]).view())
        host.append(x)
    got = cuda.Tensor.concat(pieces, 1).to_numpy()
    want = np.concatenate(host, 1)
    assert np.array_equal(got.view(np.uint8), want.view(np.uint8))
    del rng


@pytest.mark.parametrize("shape,perm", [([4, 6, 40, 32], [0, 2, 1, 3]), ([3, 130, 32], [1, 2, 0]),
                                        ([5, 96, 70], [0, 2, 1]), ([2, 64, 128], [0, 2, 1]),
                                        ([7, 30, 66], [2, 1, 0]), ([9, 2, 14, 22], [3, 0, 2, 1])])
def test_two_byte_transposes_with_short_and_long_tiles(device, shape, perm):
    """Permutations whose innermost target axis comes from a strided source
    axis: 2-byte elements move as pairs through 64 x 32 or 64 x 64 tiles,
    ragged at the edges and in the last batch of tiles."""
    n = int(np.prod(shape))
    x = O.narrow(normal(n, 7), "f16")
    t = cuda.Tensor(cuda.CudaStorage.store(x, "f16"), shape)
    got = t.view().permute(perm).contiguous().storage.as_slice()
    want = np.ascontiguousarray(x.reshape(shape).transpose(perm)).reshape(-1)
    assert np.array_equal(got, want)


@pytest.mark.parametrize("shape,perm", [([3, 8, 200, 12], [0, 3, 1, 2]), ([2, 5, 4, 132, 32], [0, 4, 2, 1, 3]),
                                        ([8, 16, 128, 64, 32], [0, 3, 1, 4, 2])])
def test_two_byte_transposes_with_short_source_runs(device, shape, perm):
    """Permutations whose source-contiguous axis is short (at most 32) and
    whose other axes step in multiples of 4, ragged along the inner axis."""
    n = int(np.prod(shape))
    x = O.narrow(normal(n, 8), "f16")
    t = cuda.Tensor(cuda.CudaStorage.store(x, "f16"), shape)
    got = t.view().permute(perm).contiguous().storage.as_slice()
    want = np.ascontiguousarray(x.reshape(shape).transpose(perm)).reshape(-1)
    assert np.array_equal(got, want)
