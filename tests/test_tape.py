"""The native reverse-mode tape (tc_tape_*) against the reference's rules:
config 4's network built from its tensor-level ops gives the gradients the
oracle's replay of the reference tape gives; broadcast arithmetic, mean and
sum over axes give the f64 gradients of the same expression; the tape's
bookkeeping (unreached nodes have no adjoint, an operand used twice gets
both contributions, a new backward pass clears the old adjoints) follows
tape/mod.rs:316-322, 507-521."""
from __future__ import annotations

import numpy as np
import pytest

import oracle as O
from tensorcrate_b200 import cuda
from tensorcrate_b200.tape import Tape
from util import normal

pytestmark = pytest.mark.gpu


def _leaf(tape, values, dtype="f32"):
    values = np.asarray(values, np.float32)
    return tape.leaf(cuda.CudaStorage.store(O.narrow(values.ravel(), dtype), dtype), list(values.shape))


def test_mlp_built_on_the_tape_matches_the_oracles_tape(device):
    """W·IN + b (broadcast), ReLU, ..., (P - Y)², summed and scaled: the
    reference's rules for each op (matmul's transposed products, the
    broadcast add's sum over the batch, MaxShare) through the kernels."""
    from tensorcrate_b200.mlp import xavier
    dims, batch = [64, 128, 96, 48], 80
    rng = np.random.default_rng(5)
    ws = [xavier(dims[l + 1], dims[l], rng) for l in range(3)]
    bs = [rng.uniform(-0.1, 0.1, dims[l + 1]).astype(np.float32) for l in range(3)]
    x, y = normal((dims[0], batch), 15), normal((dims[-1], batch), 16)
    t = Tape("f32")
    h = _leaf(t, x)
    W = [_leaf(t, w) for w in ws]
    B = [_leaf(t, b.reshape(-1, 1)) for b in bs]
    for l in range(3):
        a = t.add(t.matmul(W[l], h), B[l])
        h = t.relu(a) if l < 2 else a
    r = t.sub(h, _leaf(t, y))
    loss = t.scale(t.sum(t.mul(r, r)), float(np.float32(1.0 / (dims[-1] * batch))))
    t.backward(loss)
    o = O.lib().orc_mlp_create(O.DTYPES["f32"], 3, O.u32s(dims), batch, batch, 1e-3, 0.9, 0.99, 1e-8)
    for l in range(3):
        O.call("orc_mlp_params", o, l, O.ptr(ws[l]), O.ptr(bs[l]), 0)
    want_loss = np.empty(1, np.float32)
    O.call("orc_mlp_step", o, O.ptr(x), O.ptr(y), O.ptr(want_loss), 1)
    # the loss sums 3840 squares: rel 1e-5*sqrt(K), the sums' contract
    assert abs(t.value(loss)[0] - want_loss[0]) <= 1e-5 * np.sqrt(dims[-1] * batch) * abs(want_loss[0])
    for l in range(3):
        gw = np.empty(dims[l + 1] * dims[l], np.float32)
        gb = np.empty(dims[l + 1], np.float32)
        O.call("orc_mlp_grads", o, l, O.ptr(gw), O.ptr(gb))
        got_w, got_b = t.grad(W[l]).ravel(), t.grad(B[l]).ravel()
        assert np.max(np.abs(got_w - gw)) <= 1e-4 * np.max(np.abs(gw)), l
        assert np.max(np.abs(got_b - gb)) <= 1e-4 * np.max(np.abs(gb)), l
    O.lib().orc_mlp_destroy(o)
    t.close()


def test_broadcast_rules_give_the_f64_gradients(device):
    """L = sum over j of mean over (i, k) of (x·w/z − y)², with w [4, 1] and
    z [5] broadcast against x, y [3, 4, 5]."""
    rng = np.random.default_rng(3)
    x, y = rng.uniform(-1, 1, (3, 4, 5)), rng.uniform(-1, 1, (3, 4, 5))
    w, z = rng.uniform(0.5, 1.5, (4, 1)), rng.uniform(0.5, 1.5, 5)
    x, y, w, z = (v.astype(np.float32) for v in (x, y, w, z))
    t = Tape("f32")
    X, Y, Wv, Z = _leaf(t, x), _leaf(t, y), _leaf(t, w), _leaf(t, z)
    d = t.sub(t.div(t.mul(X, Wv), Z), Y)
    m = t.mean_axes(t.mul(d, d), [0, 2])
    assert t.shape(m) == [4]
    loss = t.sum_axes(m, [0])
    t.backward(loss)
    x64, y64, w64, z64 = (v.astype(np.float64) for v in (x, y, w, z))
    dd = x64 * w64 / z64 - y64
    gd = 2.0 * dd / 15.0
    want = {X: gd * w64 / z64, Wv: (gd * x64 / z64).sum(axis=(0, 2)).reshape(4, 1),
            Z: (gd * -(x64 * w64) / z64 ** 2).sum(axis=(0, 1)), Y: -gd}
    assert abs(float(t.value(loss).ravel()[0]) - float((dd ** 2).mean(axis=(0, 2)).sum())) <= 1e-5
    for v, g in want.items():
        got = t.grad(v).astype(np.float64)
        assert got.shape == g.shape
        assert np.max(np.abs(got - g)) <= 1e-5 * max(1.0, float(np.max(np.abs(g)))), v
    t.close()


def test_bookkeeping_follows_the_reference_tape(device):
    t = Tape("f32")
    a = _leaf(t, np.array([1.5, -2.0, 0.0], np.float32))
    unused = _leaf(t, np.array([3.0], np.float32))
    sq = t.mul(a, a)  # a meets itself twice: both contributions land
    s = t.sum(t.relu(sq))
    t.backward(s)
    assert np.array_equal(t.grad(a), np.array([3.0, -4.0, 0.0], np.float32))
    assert t.grad(unused) is None
    # relu at exactly zero passes half: MaxShare(0, 0) = 1/2
    r = t.sum(t.relu(a))
    t.backward(r)
    assert np.array_equal(t.grad(a), np.array([1.0, 0.0, 0.5], np.float32))
    assert t.grad(sq) is None  # cleared: not reachable from r
    t.close()


@pytest.mark.parametrize("dtype", ["bf16", "f16"])
def test_half_types_round_each_rule(device, dtype):
    """The same broadcast expression in f16/bf16 stays within the element
    type's rounding of the f64 gradients."""
    rng = np.random.default_rng(8)
    x, w = rng.uniform(-1, 1, (16, 32)).astype(np.float32), rng.uniform(0.5, 1.5, (1, 32)).astype(np.float32)
    xq, wq = O.widen(O.narrow(x, dtype), dtype).reshape(x.shape), O.widen(O.narrow(w, dtype), dtype).reshape(w.shape)
    t = Tape(dtype)
    X, Wv = _leaf(t, xq, dtype), _leaf(t, wq, dtype)
    loss = t.sum(t.mul(t.mul(X, Wv), X))
    t.backward(loss)
    gx = O.widen(t.grad(X).ravel(), dtype).reshape(x.shape)
    gw = O.widen(t.grad(Wv).ravel(), dtype).reshape(w.shape)
    step = 2.0 ** -7 if dtype == "bf16" else 2.0 ** -10
    want_x = 2 * xq.astype(np.float64) * wq
    want_w = (xq.astype(np.float64) ** 2).sum(axis=0, keepdims=True)
    assert np.max(np.abs(gx - want_x)) <= 4 * step * np.max(np.abs(want_x))
    assert np.max(np.abs(gw - want_w)) <= 4 * step * np.max(np.abs(want_w))
    t.close()
