"""Pins the CPU restatement (oracle/lamp3_oracle.c) against (1) the known
answers of the reference's C++ tests and (2) the reference's own CPU core
compiled from its sources (oracle/_ref), on seeded inputs.  CPU only."""
from __future__ import annotations

import json
import os

import numpy as np
import pytest

from oracle import port, ref
from tests.util import DT, NP_DTYPES, assert_bitexact, rand, rel_err

HERE = os.path.dirname(os.path.abspath(__file__))
KA = json.load(open(os.path.join(HERE, "golden", "known_answers.json")))
BIN = {"add": 0, "sub": 1, "mul": 2, "div": 3, "pow": 4, "eq": 5, "ne": 6, "ge": 7, "le": 8,
       "gt": 9, "lt": 10, "abs_backward": 11, "clamp_backward": 12}
RED = {"sum": 0, "max": 1, "min": 2, "prod": 3}
needs_ref = pytest.mark.skipif(not ref.available(), reason="reference CPU build (oracle/_ref) absent")


def _arr(spec):
    vals, shape, dt = spec
    return np.array(vals, dtype=np.float64).astype(dt).reshape(shape)


@pytest.mark.parametrize("case", KA["tensor"], ids=lambda c: c["src"].split("/")[-1] + ":" + c["op"])
def test_known_answers_oracle(case):
    op = case["op"]
    a = _arr(case["a"])
    if op in BIN:
        b = _arr(case["b"])
        p = case.get("p", [0.0, 0.0])
        got = port.binary(BIN[op], a, b, p0=p[0], p1=p[1])
    elif op in RED:
        got = port.reduce(RED[op], a, case["axis"])
    elif op == "matmul":
        got = port.matmul(a, _arr(case["b"]))
    elif op == "transpose":
        got = port.transpose(a)
    exp = np.array(case["expect"], dtype=np.float64)
    if "out_dtype" in case:
        assert got.dtype == np.dtype(case["out_dtype"])
    assert rel_err(got.ravel(), exp) <= case.get("rtol", 1e-6) or np.allclose(got.ravel(), exp, atol=1e-5)


def _f(v):
    return {"inf": np.inf, "-inf": -np.inf}.get(v, v) if isinstance(v, str) else v


@needs_ref
@pytest.mark.parametrize("case", KA["autograd"], ids=lambda c: c["expr"])
def test_known_answers_reference_autograd(case):
    """The transcribed autograd answers hold on the reference build itself."""
    a = np.array([1, 2, 3, 4, 5, 2], np.float32).reshape(3, 2)
    b = np.array([-1, 4, -2, 0, 3, 0.5], np.float32).reshape(3, 2)
    A, B = ref.Var.of(a, True), ref.Var.of(b, True)
    expr = case["expr"]
    M = None
    if expr in ("a + b", "a - b", "a * b", "a / b"):
        out = ref.binary({"+": 0, "-": 1, "*": 2, "/": 3}[expr[2]], A, B)
    elif expr.startswith("sum"):
        out = ref.reduce(0, A, 1)
    elif expr.startswith("max"):
        out = ref.reduce(1, A, 1)
    else:
        M = ref.Var.of(np.array([[-1], [4]], np.float32), True)
        out = ref.matmul(A, M)
    np.testing.assert_allclose(out.numpy().ravel(), [_f(v) for v in case["out"]], atol=1e-5)
    out.backward()
    np.testing.assert_allclose(A.grad().ravel(), [_f(v) for v in case["grad_a"]], atol=1e-5)
    if "grad_b" in case:
        np.testing.assert_allclose(B.grad().ravel(), [_f(v) for v in case["grad_b"]], atol=1e-5)
    if M is not None:
        np.testing.assert_allclose(M.grad().ravel(), case["grad_m"], atol=1e-5)


SHAPES = [((5, 7), (5, 7)), ((4, 6), (1, 6)), ((4, 6), (4, 1)), ((3, 1, 5), (4, 1)), ((7,), (1,)),
          ((2, 3, 4), (3, 4))]


@needs_ref
@pytest.mark.parametrize("op", list(range(11)))
@pytest.mark.parametrize("dt", NP_DTYPES[1:])
def test_binary_oracle_matches_reference(op, dt):
    rng = np.random.default_rng(100 + op)
    for sa, sb in SHAPES:
        lo, hi = (0.5, 3.0) if op in (3, 4) else (-4, 4)
        a, b = rand(rng, sa, dt, lo, hi), rand(rng, sb, dt, lo, hi)
        if op == 4 and np.dtype(dt).kind == "i":
            b = rng.integers(0, 4, size=sb).astype(dt)
        if op == 3 and np.dtype(dt).kind == "i":  # x/0 traps (SIGFPE) in the reference
            b = rng.integers(1, 5, size=sb).astype(dt) * np.where(rng.random(sb) < 0.5, 1, -1).astype(dt)
        got = port.binary(op, a, b)
        want = ref.binary(op, ref.Var.of(a), ref.Var.of(b)).numpy()
        if op in (3, 4) and np.dtype(dt).kind == "f":
            # the reference's Release build uses -ffast-math (reciprocal-multiply
            # division, fast pow): not correctly rounded, compared in tolerance
            assert rel_err(got, want) <= 1e-6, (op, dt, sa, sb)
        else:
            assert_bitexact(got, want, f"op{op} {dt} {sa}x{sb}")


@needs_ref
@pytest.mark.parametrize("op", list(range(9)))
@pytest.mark.parametrize("dt", [np.int32, np.float32, np.float64])
def test_unary_oracle_matches_reference(op, dt):
    rng = np.random.default_rng(200 + op)
    lo, hi = (0.1, 5.0) if op in (2, 3) else (-1.2, 1.2) if op == 7 else (-4, 4)
    a = rand(rng, (37, 5), dt, lo, hi)
    got = port.unary(op, a, -1.0, 2.0)
    want = ref.unary(op, ref.Var.of(a), -1.0, 2.0).numpy()
    if np.dtype(dt).kind == "f" and op not in (0, 4, 8):
        assert rel_err(got, want) <= 1e-6
    else:
        assert_bitexact(got, want, f"unary{op} {dt}")


@needs_ref
@pytest.mark.parametrize("op", [0, 1, 2, 3])
@pytest.mark.parametrize("dt", [np.int32, np.int64, np.float32, np.float64])
@pytest.mark.parametrize("shape_axis", [((33, 17), 0), ((33, 17), 1), ((4, 5, 6), 1), ((9,), 0)])
def test_reduce_oracle_matches_reference(op, dt, shape_axis):
    shape, axis = shape_axis
    rng = np.random.default_rng(300 + op)
    a = rand(rng, shape, dt, -3, 3) if op != 3 else rand(rng, shape, dt, 0.5, 1.5)
    if op == 3 and np.dtype(dt).kind == "i":
        a = rng.integers(1, 3, size=shape).astype(dt)
    got = port.reduce(op, a, axis)
    want = ref.reduce(op, ref.Var.of(a), axis).numpy()
    if np.dtype(dt).kind == "f" and op in (0, 3):
        assert rel_err(got, want) <= 1e-6
    else:
        assert_bitexact(got, want, f"reduce{op}")


@needs_ref
@pytest.mark.parametrize("dts", [(np.float32, np.float32), (np.int32, np.int32), (np.int32, np.float32),
                                 (np.float64, np.float32)])
def test_matmul_oracle_matches_reference(dts):
    rng = np.random.default_rng(7)
    a = rand(rng, (13, 9), dts[0], -3, 3)
    b = rand(rng, (9, 11), dts[1], -3, 3)
    got = port.matmul(a, b)
    want = ref.matmul(ref.Var.of(a), ref.Var.of(b)).numpy()
    assert got.dtype == want.dtype
    if got.dtype.kind == "f":
        assert rel_err(got, want) <= 1e-6
    else:
        assert_bitexact(got, want)
    assert_bitexact(port.transpose(a), ref.transpose(ref.Var.of(a)).numpy())


@needs_ref
def test_c2_chain_oracle_matches_reference_small():
    """The headline chain d = exp(a*a + b)*a - log(b+1), op by op."""
    rng = np.random.default_rng(2)
    a = rng.random((64, 128), dtype=np.float32)
    b = rng.random((64, 1), dtype=np.float32)
    one = np.ones((1,), np.float32)
    d = port.binary(1, port.binary(2, port.unary(1, port.binary(0, port.binary(2, a, a), b)), a),
                    port.unary(2, port.binary(0, b, one)))
    A, B, O = ref.Var.of(a, True), ref.Var.of(b, True), ref.Var.of(one)
    D = ref.binary(1, ref.binary(2, ref.unary(1, ref.binary(0, ref.binary(2, A, A), B)), A),
                   ref.unary(2, ref.binary(0, B, O)))
    assert rel_err(d, D.numpy()) <= 1e-6
