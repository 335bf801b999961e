"""Config 4's training step: the reference tape's rules and Adam, run by
libtccuda (tc_mlp_step), against the oracle's restatement of the same tape
on the same seeded inputs; and the oracle's gradients against f64
backpropagation."""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

import oracle as O
from util import normal

DIMS = [64, 128, 96, 48]
BATCH = 80


def _setup(dtype, seed=0, dims=DIMS, batch=BATCH):
    from tensorcrate_b200.mlp import xavier
    rng = np.random.default_rng(seed)
    ws = [xavier(dims[l + 1], dims[l], rng) for l in range(len(dims) - 1)]
    bs = [rng.uniform(-0.1, 0.1, dims[l + 1]).astype(np.float32) for l in range(len(dims) - 1)]
    x = normal((dims[0], batch), seed + 10)
    y = normal((dims[-1], batch), seed + 11)
    return ws, bs, x, y


def _oracle(dtype, ws, bs, beta2=0.999, dims=DIMS, batch=BATCH, eps=1e-8):
    h = O.lib().orc_mlp_create(O.DTYPES[dtype], len(dims) - 1, O.u32s(dims), batch, batch, 1e-3, 0.9, beta2, eps)
    for l, (w, b) in enumerate(zip(ws, bs)):
        wn, bn = O.narrow(w, dtype), O.narrow(b, dtype)
        O.call("orc_mlp_params", h, l, O.ptr(wn), O.ptr(bn), 0)
    return h


def _grads(h, l, dtype, dims=DIMS):
    gw = np.empty(dims[l + 1] * dims[l], O.STORE[dtype])
    gb = np.empty(dims[l + 1], O.STORE[dtype])
    O.call("orc_mlp_grads", h, l, O.ptr(gw), O.ptr(gb))
    return O.widen(gw, dtype).reshape(dims[l + 1], dims[l]), O.widen(gb, dtype)


def test_oracle_gradients_match_f64_backprop():
    ws, bs, x, y = _setup("f32")
    h = _oracle("f32", ws, bs)
    loss = np.empty(1, np.float32)
    O.call("orc_mlp_step", h, O.ptr(x), O.ptr(y), O.ptr(loss), 1)
    # f64 reference of the same network
    acts, pre = [x.astype(np.float64)], []
    for l, (w, b) in enumerate(zip(ws, bs)):
        a = w.astype(np.float64) @ acts[-1] + b.astype(np.float64)[:, None]
        pre.append(a)
        acts.append(np.maximum(a, 0) if l + 1 < len(ws) else a)
    n = y.size
    r = acts[-1] - y
    assert abs(loss[0] - (r * r).sum() / n) <= 1e-5 * max(1.0, (r * r).sum() / n)
    g = 2 * r / n
    for l in range(len(ws) - 1, -1, -1):
        gw_want, gb_want = g @ acts[l].T, g.sum(axis=1)
        gw, gb = _grads(h, l, "f32")
        assert np.max(np.abs(gw - gw_want)) <= 1e-4 * max(1e-3, np.max(np.abs(gw_want)))
        assert np.max(np.abs(gb - gb_want)) <= 1e-4 * max(1e-3, np.max(np.abs(gb_want)))
        if l:
            g = (ws[l].astype(np.float64).T @ g) * np.where(pre[l - 1] > 0, 1.0, np.where(pre[l - 1] < 0, 0.0, 0.5))
    O.lib().orc_mlp_destroy(h)


def test_oracle_training_reduces_the_loss():
    ws, bs, x, y = _setup("f32", seed=3)
    h = _oracle("f32", ws, bs)
    losses = []
    for _ in range(20):
        loss = np.empty(1, np.float32)
        O.call("orc_mlp_step", h, O.ptr(x), O.ptr(y), O.ptr(loss), 0)
        losses.append(float(loss[0]))
    assert losses[-1] < 0.9 * losses[0]
    O.lib().orc_mlp_destroy(h)


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", ["f32", "bf16", "f16"])
def test_mlp_step_matches_the_oracle(device, dtype):
    from tensorcrate_b200 import cuda
    from tensorcrate_b200.mlp import Mlp
    # beta2 = 0.999 rounds to 1.0 in bf16, and eps = 1e-8 to 0 in f16 (a
    # dead unit's zero gradient is then 0/0): the reference's updates are NaN
    # there.  beta2 = 0.99 and, for f16, eps = 1e-4 keep every run finite.
    beta2 = 0.99
    eps = 1e-4 if dtype == "f16" else 1e-8
    ws, bs, x, y = _setup(dtype, seed=5)
    h = _oracle(dtype, ws, bs, beta2, eps=eps)
    m = Mlp(dtype, DIMS, BATCH, beta2=beta2, eps=eps)
    m.load(ws, bs)
    xd = cuda.CudaStorage.store(O.narrow(x, dtype), dtype)
    yd = cuda.CudaStorage.store(O.narrow(y, dtype), dtype)
    tol = {"f32": 1e-4, "bf16": 4e-2, "f16": 8e-3}[dtype]
    for step in range(3):
        loss_d = cuda.CudaStorage(dtype, 1)
        m.step(xd, yd, loss=loss_d)
        loss_o = np.empty(1, O.STORE[dtype])
        O.call("orc_mlp_step", h, O.ptr(O.narrow(x, dtype)), O.ptr(O.narrow(y, dtype)), O.ptr(loss_o), 0)
        lg, lo = O.widen(loss_d.as_slice(), dtype)[0], O.widen(loss_o, dtype)[0]
        # The first step starts from identical parameters: every gradient
        # element agrees to the products' rounding.  Adam's normalised update
        # then moves each parameter by about the rate whatever the gradient's
        # size, so a near-zero gradient that rounds differently moves its
        # parameter differently; later steps are compared in norm.
        loose = 1 if step == 0 else 10
        assert abs(lg - lo) <= loose * tol * abs(lo), (step, lg, lo)
        for l in range(len(DIMS) - 1):
            gw, gb = m.grads(l)
            ow, ob = _grads(h, l, dtype)
            gw, gb = O.widen(gw, dtype).reshape(ow.shape), O.widen(gb, dtype)
            if step == 0:
                assert np.max(np.abs(gw - ow)) <= tol * np.max(np.abs(ow)), (step, l)
                assert np.max(np.abs(gb - ob)) <= tol * np.max(np.abs(ob)), (step, l)
            else:
                assert np.linalg.norm(gw - ow) <= loose * tol * np.linalg.norm(ow), (step, l)
                assert np.linalg.norm(gb - ob) <= loose * tol * np.linalg.norm(ob), (step, l)
    # parameters after three Adam steps: each step moves by about the rate
    for l in range(len(DIMS) - 1):
        w, _ = m.params(l)
        ow = np.empty(DIMS[l + 1] * DIMS[l], O.STORE[dtype])
        ob = np.empty(DIMS[l + 1], O.STORE[dtype])
        O.call("orc_mlp_params", h, l, O.ptr(ow), O.ptr(ob), 1)
        diff = np.abs(O.widen(w, dtype) - O.widen(ow, dtype))
        # At most two full steps apart per update (Adam moves a parameter by
        # about the rate either way), and typically equal to rounding.
        # In f16, v = g^2*(1-beta2) underflows to zero for |g| below ~2.4e-3,
        # and the step is then m*c1/eps (up to ~30x the rate): whether an
        # element underflows depends on its gradient's last bit, so f16 is
        # held to the median only.
        ulp = {"f32": 1e-6, "bf16": 8e-3, "f16": 1e-3}[dtype]
        if dtype != "f16":
            assert np.max(diff) <= 2 * 1e-3 * 3 + ulp, l
        assert np.median(diff) <= {"f32": 1e-6, "bf16": 4e-3, "f16": 2e-4}[dtype], l
    O.lib().orc_mlp_destroy(h)


@pytest.mark.gpu
def test_bf16_mlp_with_default_adam_is_nan_like_the_reference(device):
    from tensorcrate_b200 import cuda
    from tensorcrate_b200.mlp import Mlp
    ws, bs, x, y = _setup("bf16", seed=6)
    m = Mlp("bf16", DIMS, BATCH)
    m.load(ws, bs)
    xd = cuda.CudaStorage.store(O.narrow(x, "bf16"), "bf16")
    yd = cuda.CudaStorage.store(O.narrow(y, "bf16"), "bf16")
    m.step(xd, yd)
    w, _ = m.params(0)
    assert np.all(np.isnan(O.widen(w, "bf16")))


CONFIG4 = [1024, 4096, 4096, 1024]
CONFIG4_BATCH = 2048


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", ["bf16", "f32"])
def test_mlp_step_matches_the_oracle_at_config_4(device, dtype):
    """One training step at config 4's own size (1024-4096-4096-1024, batch
    2048), which takes the tile plans, split-K products and row splits the
    small network never reaches.  beta2 = 0.99: the configured 0.999 rounds
    to 1.0 in bf16 and turns the reference's update into NaN.  The oracle's
    products run on all host threads (same bits as its single thread)."""
    import os

    from tensorcrate_b200 import cuda
    from tensorcrate_b200.mlp import Mlp, xavier
    dims, batch, beta2 = CONFIG4, CONFIG4_BATCH, 0.99
    rng = np.random.default_rng(6)
    ws = [xavier(dims[l + 1], dims[l], rng) for l in range(3)]
    bs = [rng.uniform(-0.05, 0.05, dims[l + 1]).astype(np.float32) for l in range(3)]
    x = normal((dims[0], batch), 4)
    y = normal((dims[-1], batch), 5)
    O.set_matmul_threads(os.cpu_count() or 1)
    try:
        h = _oracle(dtype, ws, bs, beta2, dims=dims, batch=batch)
        loss_o = np.empty(1, O.STORE[dtype])
        O.call("orc_mlp_step", h, O.ptr(O.narrow(x, dtype)), O.ptr(O.narrow(y, dtype)), O.ptr(loss_o), 0)
    finally:
        O.set_matmul_threads(1)
    m = Mlp(dtype, dims, batch, beta2=beta2)
    m.load(ws, bs)
    loss_d = cuda.CudaStorage(dtype, 1)
    m.step(cuda.CudaStorage.store(O.narrow(x, dtype), dtype), cuda.CudaStorage.store(O.narrow(y, dtype), dtype),
           loss=loss_d)
    tol = {"f32": 1e-4, "bf16": 4e-2}[dtype]
    lg, lo = O.widen(loss_d.as_slice(), dtype)[0], O.widen(loss_o, dtype)[0]
    # The loss sums 2M squares: the Host's running f32 sum drifts by about
    # 1e-3 over that many terms, the device's tree by far less; the sums'
    # contract is rel 1e-5*sqrt(K).
    assert abs(lg - lo) <= max(tol, 1e-5 * np.sqrt(dims[-1] * batch)) * abs(lo), (lg, lo)
    report = {}
    for l in range(3):
        gw, gb = m.grads(l)
        ow, ob = _grads(h, l, dtype, dims=dims)
        gw, gb = O.widen(gw, dtype).reshape(ow.shape), O.widen(gb, dtype)
        w, b = m.params(l)
        pw = np.empty(dims[l + 1] * dims[l], O.STORE[dtype])
        pb = np.empty(dims[l + 1], O.STORE[dtype])
        O.call("orc_mlp_params", h, l, O.ptr(pw), O.ptr(pb), 1)
        diff = np.abs(O.widen(w, dtype) - O.widen(pw, dtype))
        report[l] = {"max_rel": float(np.max(np.abs(gw - ow)) / np.max(np.abs(ow))),
                     "norm_rel": float(np.linalg.norm(gw - ow) / np.linalg.norm(ow)),
                     "bias_max_rel": float(np.max(np.abs(gb - ob)) / np.max(np.abs(ob))),
                     "param_max": float(np.max(diff)), "param_median": float(np.median(diff)),
                     # Adam's first step moves a parameter by about the rate either
                     # way: parameters more than one rate apart moved opposite ways
                     "opposite_moves": float(np.mean(diff > 1e-3))}
    # A ReLU whose input sits within rounding of zero takes the other branch
    # on one side (MaxShare is 1, 0.5 or 0): that sample's whole contribution
    # to the gradients below it differs, about 1/sqrt(batch) of a gradient
    # element.  The top layer's gradients see such flips only through the
    # forward activations and are held element by element; the lower layers
    # are held in norm.  After Adam's first step every
    # parameter is within two rates (a gradient of the other sign moves it
    # the other way), and few move opposite ways.
    # (Measured on B200, f32: top layer 1.4e-4 of the largest element, the
    # lower layers 2e-3 and 3e-4 in norm; bf16: 4e-3, 4e-3 and 1e-3.)
    top = report[2]
    top_tol = {"f32": 1e-3, "bf16": 4e-2}[dtype]
    assert top["max_rel"] <= top_tol and top["bias_max_rel"] <= top_tol, report
    for l in range(2):
        assert report[l]["norm_rel"] <= 2e-2, report
    ulp = {"f32": 1e-6, "bf16": 8e-3}[dtype]
    for l in range(3):
        assert report[l]["param_max"] <= 2 * 1e-3 + ulp, report
        assert report[l]["param_median"] <= {"f32": 1e-6, "bf16": 4e-3}[dtype], report
        assert report[l]["opposite_moves"] <= 1e-2, report
    O.lib().orc_mlp_destroy(h)
