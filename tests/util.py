"""Shared helpers for the tests."""
from __future__ import annotations

import numpy as np

NP_DTYPES = [np.bool_, np.int16, np.int32, np.int64, np.float32, np.float64]
DT = {np.dtype(t): i for i, t in enumerate(NP_DTYPES)}


def rel_err(got, ref) -> float:
    """max|got - ref| / max|ref| — the reference tests' parity metric
    (tests/stress/testutils.py:43-50 of the reference)."""
    got = np.asarray(got, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    denom = np.max(np.abs(ref)) if ref.size else 1.0
    if denom == 0:
        denom = 1.0
    return float(np.max(np.abs(got - ref)) / denom) if ref.size else 0.0


def assert_bitexact(got, ref, what=""):
    got, ref = np.asarray(got), np.asarray(ref)
    assert got.shape == ref.shape, f"{what}: shape {got.shape} vs {ref.shape}"
    assert got.dtype == ref.dtype, f"{what}: dtype {got.dtype} vs {ref.dtype}"
    if got.dtype.kind == "f":
        same = (got.view(np.uint8 if got.itemsize == 1 else f"u{got.itemsize}") ==
                ref.view(f"u{ref.itemsize}")) | (np.isnan(got) & np.isnan(ref))
        bad = np.flatnonzero(~same.ravel())
    else:
        bad = np.flatnonzero((got != ref).ravel())
    assert bad.size == 0, (f"{what}: {bad.size} mismatches, first at {bad[0]}: "
                           f"{got.ravel()[bad[0]]!r} vs {ref.ravel()[bad[0]]!r}")


def rand(rng, shape, dtype, lo=-3.0, hi=3.0):
    dtype = np.dtype(dtype)
    if dtype == np.bool_:
        return rng.random(shape) < 0.5
    if dtype.kind == "i":
        return rng.integers(int(lo), int(hi) + 1, size=shape).astype(dtype)
    return rng.uniform(lo, hi, size=shape).astype(dtype)
