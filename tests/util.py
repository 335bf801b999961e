"""Shared test helpers: the reference tests' fillers, seeded inputs, KATs."""
from __future__ import annotations

import json
import math
from pathlib import Path

import numpy as np

GOLDEN = Path(__file__).resolve().parent / "golden"
DTYPES = ["f32", "f16", "bf16"]


def integral(n: int, offset: int = 0) -> np.ndarray:
    """((7i+3) mod 23) - 11 (tests/broadcast_reduce.rs:12-14): integral,
    mixed sign, so every sum of it is exact in f32."""
    i = np.arange(offset, offset + n, dtype=np.int64)
    return (((i * 7 + 3) % 23) - 11).astype(np.float32)


def normal(shape, seed: int) -> np.ndarray:
    return np.random.default_rng(seed).standard_normal(shape).astype(np.float32)


def uniform(shape, seed: int) -> np.ndarray:
    return np.random.default_rng(seed).uniform(-1.0, 1.0, shape).astype(np.float32)


def _value(v):
    if isinstance(v, str):
        return {"nan": math.nan, "inf": math.inf, "-inf": -math.inf}[v]
    return v


def expand(values):
    if isinstance(values, dict) and "fill" in values:
        return [values["fill"]] * values["n"]
    return [_value(v) for v in values]


def kats(kind: str | None = None) -> list[dict]:
    data = json.loads((GOLDEN / "reference_kats.json").read_text())["kats"]
    return [k for k in data if kind is None or k["kind"] == kind]


def same_floats(got: np.ndarray, want: np.ndarray) -> bool:
    """Equal, with NaN equal to NaN (positions must agree)."""
    got, want = np.asarray(got, np.float64), np.asarray(want, np.float64)
    return got.shape == want.shape and bool(np.all((got == want) | (np.isnan(got) & np.isnan(want))))


def bits_of(values, dtype):
    return np.asarray(values).view(np.uint32 if dtype == "f32" else np.uint16).astype(np.int64)


def steps(got, want, dtype):
    """How many representable values of `dtype` lie between got and want
    (0 = same bits; NaNs compare equal to NaNs)."""
    width = 32 if dtype == "f32" else 16
    sign = 1 << (width - 1)

    def ordered(b):
        return np.where(b & sign, -(b & (sign - 1)), b)

    g, w = bits_of(got, dtype), bits_of(want, dtype)
    d = np.abs(ordered(g) - ordered(w))
    import oracle as O

    gf, wf = O.widen(np.asarray(got), dtype), O.widen(np.asarray(want), dtype)
    return np.where(np.isnan(gf) & np.isnan(wf), 0, d)
