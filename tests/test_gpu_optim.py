"""The fused optimizer updates (Adam, SGD, Momentum, AdaGrad, RmsProp)
against the oracle's restatement of their programs (optim.rs:1048-1099,
773-787, 826-846, 892-904, 948-964): every operation rounds to the element
type in the program's order, so the updates agree bit for bit."""
from __future__ import annotations

import numpy as np
import pytest

import oracle as O
from tensorcrate_b200 import cuda
from tensorcrate_b200 import _native as N
from util import DTYPES, normal

pytestmark = pytest.mark.gpu


def same_bits(got, want, dtype):
    """Bit for bit, except that a NaN matches any NaN: an invalid operation
    gives x86's negative default NaN on the host and CUDA's positive
    canonical NaN on the device, and the reference pins neither."""
    g, w = O.widen(got, dtype), O.widen(want, dtype)
    return bool(np.all((got == want) | (np.isnan(g) & np.isnan(w))))


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("n", [1, 13, 4096 + 3, 250000])
def test_adam_steps_match_bit_for_bit(device, dtype, n):
    # beta2 = 0.99 keeps the bf16 run finite (0.999 rounds to 1.0 in bf16).
    beta2 = 0.99 if dtype == "bf16" else 0.999
    p = O.narrow(normal(n, 1), dtype)
    dp = cuda.CudaStorage.store(p, dtype)
    dm, dv = cuda.CudaStorage.zeros(dtype, n), cuda.CudaStorage.zeros(dtype, n)
    m, v = np.zeros_like(p), np.zeros_like(p)
    for step in range(1, 4):
        g = O.narrow(normal(n, 10 + step) * 0.1, dtype)
        dg = cuda.CudaStorage.store(g, dtype)
        coef = O.adam_coefficients(dtype, 1e-3, 0.9, beta2, 1e-8, step)
        resumed = int(step > 1)
        N.call("tc_adam", N.DTYPES[dtype], n, dp.ptr, dg.ptr, dm.ptr, dv.ptr, resumed, *coef, None)
        O.call("orc_adam", O.DTYPES[dtype], n, O.ptr(p), O.ptr(g), O.ptr(m), O.ptr(v), resumed, *coef)
        assert same_bits(dp.as_slice(), p, dtype), f"p at step {step}"
        assert same_bits(dm.as_slice(), m, dtype), f"m at step {step}"
        assert same_bits(dv.as_slice(), v, dtype), f"v at step {step}"


def test_bf16_adam_with_default_betas_is_nan_like_the_reference(device):
    coef = O.adam_coefficients("bf16", 1e-3, 0.9, 0.999, 1e-8, 1)
    p = O.narrow(normal(64, 1), "bf16")
    g = O.narrow(normal(64, 2), "bf16")
    dp, dg = cuda.CudaStorage.store(p, "bf16"), cuda.CudaStorage.store(g, "bf16")
    dm, dv = cuda.CudaStorage.zeros("bf16", 64), cuda.CudaStorage.zeros("bf16", 64)
    N.call("tc_adam", N.BF16, 64, dp.ptr, dg.ptr, dm.ptr, dv.ptr, 0, *coef, None)
    assert np.all(np.isnan(O.widen(dp.as_slice(), "bf16")))


@pytest.mark.parametrize("dtype", DTYPES)
def test_sgd_matches_bit_for_bit(device, dtype):
    n = 10007
    p = O.narrow(normal(n, 3), dtype)
    g = O.narrow(normal(n, 4), dtype)
    dp, dg = cuda.CudaStorage.store(p, dtype), cuda.CudaStorage.store(g, dtype)
    N.call("tc_sgd", N.DTYPES[dtype], n, dp.ptr, dg.ptr, 0.01, None)
    O.call("orc_sgd", O.DTYPES[dtype], n, O.ptr(p), O.ptr(g), 0.01)
    assert same_bits(dp.as_slice(), p, dtype)


@pytest.mark.parametrize("dtype", DTYPES)
def test_adam_over_many_tensors_in_one_launch(device, dtype):
    """tc_adam_multi gives every tensor the bits tc_adam gives it alone:
    18 tensors (two launches), lengths with and without whole 16-byte packs,
    one tensor not 16-byte aligned, an empty one; a first and a resumed step."""
    import ctypes as C
    beta2 = 0.99 if dtype == "bf16" else 0.999
    lengths = [1, 7, 8, 13, 4096, 4099, 0, 250000, 31, 64, 65, 1000, 3, 16, 17, 8191, 2, 9]
    code = N.DTYPES[dtype]
    singles, multi = [], []
    for i, n in enumerate(lengths):
        p = O.narrow(normal(max(n, 1) + 1, 100 + i), dtype)
        shift = 1 if i == 5 else 0  # an operand off the 16-byte grid
        for group in (singles, multi):
            d = {k: cuda.CudaStorage.store(p, dtype) for k in ("p",)}
            d["m"], d["v"] = cuda.CudaStorage.zeros(dtype, n + 1), cuda.CudaStorage.zeros(dtype, n + 1)
            d["shift"], d["n"] = shift, n
            group.append(d)
    eb = 4 if dtype == "f32" else 2
    for step in (1, 2):
        coef = O.adam_coefficients(dtype, 1e-3, 0.9, beta2, 1e-8, step)
        grads = [cuda.CudaStorage.store(O.narrow(normal(max(n, 1) + 1, 300 + 10 * step + i) * 0.1, dtype), dtype)
                 for i, n in enumerate(lengths)]
        arr = (N.AdamTensor * len(lengths))()
        for i, (d, g) in enumerate(zip(multi, grads)):
            o = d["shift"] * eb
            arr[i].p, arr[i].g, arr[i].m, arr[i].v, arr[i].n = (d["p"].ptr + o, g.ptr + o, d["m"].ptr + o,
                                                               d["v"].ptr + o, d["n"])
        N.call("tc_adam_multi", code, arr, len(lengths), int(step > 1), *coef, None)
        for d, g in zip(singles, grads):
            o = d["shift"] * eb
            N.call("tc_adam", code, d["n"], d["p"].ptr + o, g.ptr + o, d["m"].ptr + o, d["v"].ptr + o,
                   int(step > 1), *coef, None)
        for s, mu in zip(singles, multi):
            for k in ("p", "m", "v"):
                assert np.array_equal(s[k].as_slice(), mu[k].as_slice()), (s["n"], k)
    del C


def _in(dtype, x):
    """x as a value of the element type (the rules' coefficients are)."""
    return float(O.widen(O.narrow(np.array([x], np.float32), dtype), dtype)[0])


def _rule_program(rule, dtype, rate, coef, nesterov=False):
    """The rule's program as its builder makes it (optim.rs:826-846, 892-904,
    948-964; descend 1146-1159): places g, p, state; outputs p, state."""
    from test_fused import binary, const, load, store, unary
    code = [load(0, 0), load(1, 1)]
    if rule == "momentum":
        code += [load(2, 2), const(3, coef), binary(4, N.MUL, 2, 3), binary(5, N.ADD, 4, 0)]
        step, state = 5, 5
        if nesterov:
            code += [binary(6, N.MUL, 5, 3), binary(7, N.ADD, 0, 6)]
            step = 7
        code += [const(8, rate), binary(9, N.MUL, step, 8), binary(10, N.SUB, 1, 9)]
        return code + [store(10, 0), store(state, 1)]
    code += [binary(2, N.MUL, 0, 0)]
    if rule == "adagrad":
        eps = coef
        code += [load(3, 2), binary(4, N.ADD, 3, 2)]
        state = 4
    else:  # rmsprop: coef = decay
        eps = _in(dtype, 1e-8)
        code += [const(3, _in(dtype, 1.0 - coef)), binary(4, N.MUL, 2, 3), load(5, 2), const(6, coef),
                 binary(7, N.MUL, 5, 6), binary(8, N.ADD, 7, 4)]
        state = 8
    code += [unary(9, N.SQRT, state), const(10, eps), binary(11, N.ADD, 9, 10), binary(12, N.DIV, 0, 11),
             const(13, rate), binary(14, N.MUL, 12, 13), binary(15, N.SUB, 1, 14)]
    return code + [store(15, 0), store(state, 1)]


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("rule", ["momentum", "nesterov", "adagrad", "rmsprop"])
@pytest.mark.parametrize("n,shift", [(10007, 0), (4099, 1)])
def test_state_rules_match_their_programs_bit_for_bit(device, dtype, rule, n, shift):
    """tc_momentum, tc_adagrad and tc_rmsprop against the oracle's
    interpreter running the rule's program, twice in a row (the state carried
    over); `shift` starts every buffer one element past a 16-byte boundary
    (no 16-byte packs)."""
    from test_fused import run_oracle
    rate = _in(dtype, 0.01)
    coef = {"momentum": _in(dtype, 0.9), "nesterov": _in(dtype, 0.9), "adagrad": _in(dtype, 1e-8),
            "rmsprop": _in(dtype, 0.9)}[rule]
    p = O.narrow(normal(n, 31), dtype)
    s = O.narrow(normal(n, 33) * np.float32(0.01) if rule in ("momentum", "nesterov") else
                 np.abs(normal(n, 33)) * np.float32(0.01), dtype)
    dev = {k: cuda.CudaStorage.store(np.concatenate([np.zeros(shift, v.dtype), v]), dtype) for k, v in (("p", p), ("s", s))}
    code = _rule_program("momentum" if rule == "nesterov" else rule, dtype, rate, coef, nesterov=rule == "nesterov")
    esz = 4 if dtype == "f32" else 2
    for step in range(2):
        g = O.narrow(normal(n, 40 + step) * np.float32(0.1), dtype)
        dg = cuda.CudaStorage.store(np.concatenate([np.zeros(shift, g.dtype), g]), dtype)
        at = lambda d: d.ptr + shift * esz
        if rule in ("momentum", "nesterov"):
            N.call("tc_momentum", N.DTYPES[dtype], n, at(dev["p"]), at(dg), at(dev["s"]), rate, coef,
                   int(rule == "nesterov"), None)
        elif rule == "adagrad":
            N.call("tc_adagrad", N.DTYPES[dtype], n, at(dev["p"]), at(dg), at(dev["s"]), rate, coef, None)
        else:
            N.call("tc_rmsprop", N.DTYPES[dtype], n, at(dev["p"]), at(dg), at(dev["s"]), rate, coef,
                   _in(dtype, 1e-8), None)
        new_p, new_s = np.empty_like(p), np.empty_like(s)
        run_oracle(dtype, 1, n, code, [(g, dtype, 0, 1, n), (p, dtype, 0, 1, n), (s, dtype, 0, 1, n)],
                   [new_p, new_s], [dtype, dtype])
        p, s = new_p, new_s
        assert same_bits(dev["p"].as_slice()[shift:], p, dtype), step
        assert same_bits(dev["s"].as_slice()[shift:], s, dtype), step


def _adam_first_step_program(dtype, coef):
    """Adam's first-step program (optim.rs:1048-1099 with `resumed` false):
    the moments go to fresh outputs; places p, g."""
    from test_fused import binary, const, load, store, unary
    rate, b1, b2, eps, c1, c2 = coef
    one = lambda x: _in(dtype, x)
    s1, s2 = one(1.0 - np.float32(b1)), one(1.0 - np.float32(b2))
    return [load(0, 0), load(1, 1), const(2, s1), binary(3, N.MUL, 1, 2), binary(4, N.MUL, 1, 1), const(5, s2),
            binary(6, N.MUL, 4, 5), const(7, c1), binary(8, N.MUL, 3, 7), const(7, c2), binary(9, N.MUL, 6, 7),
            unary(9, N.SQRT, 9), const(7, eps), binary(9, N.ADD, 9, 7), binary(8, N.DIV, 8, 9), const(7, rate),
            binary(8, N.MUL, 8, 7), binary(0, N.SUB, 0, 8), store(0, 0), store(3, 1), store(6, 2)]


def _rule_case(rule, dtype):
    """(program, place names in load order, output names in store order,
    names updated in place) for each rule the reference's optimizers build."""
    from test_fused import adam_program, binary, const, load, store
    rate = _in(dtype, 0.01)
    if rule == "sgd":
        code = [load(0, 0), load(1, 1), const(2, rate), binary(3, N.MUL, 0, 2), binary(4, N.SUB, 1, 3), store(4, 0)]
        return code, ["g", "p"], ["p"], {"p"}
    if rule in ("momentum", "nesterov", "adagrad", "rmsprop"):
        coef = _in(dtype, 1e-8) if rule == "adagrad" else _in(dtype, 0.9)
        code = _rule_program("momentum" if rule == "nesterov" else rule, dtype, rate, coef, rule == "nesterov")
        return code, ["g", "p", "s"], ["p", "s"], {"p", "s"}
    beta2 = 0.99 if dtype == "bf16" else 0.999
    coef = O.adam_coefficients(dtype, 1e-3, 0.9, beta2, 1e-8, 3)
    if rule == "adam":
        return adam_program(dtype, coef), ["p", "g", "m", "v"], ["p", "m", "v"], {"p", "m", "v"}
    return _adam_first_step_program(dtype, coef), ["p", "g"], ["p", "m", "v"], {"p"}


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("rule", ["sgd", "momentum", "nesterov", "adagrad", "rmsprop", "adam", "adam_first"])
def test_rule_programs_through_tc_fused(device, dtype, rule):
    """The reference's optimizers hand their programs to Kernels::fused.
    tc_fused runs a program that is a rule's update, written in place, as
    the rule's kernel, and any other program (here the same one into fresh
    outputs) by the interpreter: both give the bits of the oracle's
    interpreter."""
    from test_fused import run_gpu, run_oracle
    n = 20011
    code, loads, stores, updated = _rule_case(rule, dtype)
    host = {"p": O.narrow(normal(n, 51), dtype), "g": O.narrow(normal(n, 52) * np.float32(0.1), dtype),
            "m": O.narrow(normal(n, 53) * np.float32(0.01), dtype),
            "v": O.narrow(np.abs(normal(n, 54)) * np.float32(1e-4), dtype),
            "s": O.narrow(np.abs(normal(n, 55)) * np.float32(0.01), dtype)}
    want = {k: np.empty_like(host["p"]) for k in stores}
    run_oracle(dtype, 1, n, code, [(host[k], dtype, 0, 1, n) for k in loads], [want[k] for k in stores],
               [dtype] * len(stores))
    for in_place in (True, False):
        dev = {k: cuda.CudaStorage.store(host[k], dtype) for k in loads}
        outs = {k: dev[k] if in_place and k in updated else cuda.CudaStorage(dtype, n) for k in stores}
        run_gpu(dtype, 1, n, code, [(dev[k], dtype, 0, 1, n) for k in loads], [outs[k] for k in stores],
                [dtype] * len(stores))
        for k in stores:
            assert same_bits(outs[k].as_slice(), want[k], dtype), (in_place, k)
