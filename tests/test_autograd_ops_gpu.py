"""Forward and backward of every differentiable op against the reference's
own CPU build (oracle/_ref), eager and under capture, with broadcasting
operands (the gradient sums over broadcast axes run as fused reduce
epilogues here).  Bars: max|d|/max|ref| <= 1e-5 (1e-4 for pow's log term)."""
from __future__ import annotations

import numpy as np
import pytest

from oracle import ref
from tests.util import rel_err

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not ref.available(), reason="reference CPU build absent")]

SHAPES = [((24, 40), (24, 40)), ((24, 40), (1, 40)), ((24, 40), (24, 1)), ((24, 40), (40,)),
          ((2, 12, 40), (12, 1)), ((24, 1), (1, 40))]


@pytest.fixture(scope="module")
def rsl(cuda):
    import rushlite_b200

    return rushlite_b200


def _inputs(rng, op, sa, sb):
    if op in (3, 4):  # div, pow: keep away from 0 and keep pow's base positive
        return rng.uniform(0.5, 2.0, sa).astype(np.float32), rng.uniform(0.5, 2.0, sb).astype(np.float32)
    return rng.uniform(-2, 2, sa).astype(np.float32), rng.uniform(-2, 2, sb).astype(np.float32)


@pytest.mark.parametrize("op", [0, 1, 2, 3, 4], ids=["add", "sub", "mul", "div", "pow"])
@pytest.mark.parametrize("capture", [False, True])
def test_binary_backward(rsl, op, capture):
    fns = [rsl.add, rsl.sub, rsl.mul, rsl.div, rsl.pow]
    rng = np.random.default_rng(op)
    for sa, sb in SHAPES:
        a, b = _inputs(rng, op, sa, sb)
        g = rng.uniform(-1, 1, np.broadcast_shapes(sa, sb)).astype(np.float32)
        RA, RB, RG = ref.Var.of(a, True), ref.Var.of(b, True), ref.Var.of(g)
        ro = ref.binary(2, ref.binary(op, RA, RB), RG)  # * g so the output gradient is not all ones
        ro.backward()
        A = rsl.Variable(a, requires_grad=True)
        B = rsl.Variable(b, requires_grad=True)
        with rsl.capture_on(capture):
            mo = fns[op](A, B) * rsl.Variable(g)
        mo.backward()
        tol = 1e-4 if op == 4 else 1e-5
        assert rel_err(mo.numpy(), ro.numpy()) <= tol, (op, sa, sb)
        assert rel_err(A.grad.numpy(), RA.grad()) <= tol, (op, sa, sb, "grad a")
        assert rel_err(B.grad.numpy(), RB.grad()) <= tol, (op, sa, sb, "grad b")


@pytest.mark.parametrize("op", list(range(9)), ids=["neg", "exp", "log", "sqrt", "abs", "sin", "cos", "tan", "clamp"])
@pytest.mark.parametrize("capture", [False, True])
def test_unary_backward(rsl, op, capture):
    fns = [rsl.neg, rsl.exp, rsl.log, rsl.sqrt, rsl.abs, rsl.sin, rsl.cos, rsl.tan]
    rng = np.random.default_rng(10 + op)
    lo, hi = (0.2, 3.0) if op in (2, 3) else (-1.2, 1.2)
    x = rng.uniform(lo, hi, (37, 53)).astype(np.float32)
    x.ravel()[:4] = [0.0, -1.0, 1.0, 0.5] if op in (4, 8) else x.ravel()[:4]  # abs at 0, clamp at its bounds
    g = rng.uniform(-1, 1, (37, 53)).astype(np.float32)
    RX, RG = ref.Var.of(x, True), ref.Var.of(g)
    ro = ref.binary(2, ref.unary(op, RX, -1.0, 1.0), RG)
    ro.backward()
    X = rsl.Variable(x, requires_grad=True)
    with rsl.capture_on(capture):
        y = fns[op](X) if op < 8 else rsl.clamp(X, -1.0, 1.0)
        mo = y * rsl.Variable(g)
    mo.backward()
    assert rel_err(mo.numpy(), ro.numpy()) <= 1e-5
    assert rel_err(X.grad.numpy(), RX.grad()) <= 1e-5


@pytest.mark.parametrize("op", [0, 1, 2, 3], ids=["sum", "max", "min", "prod"])
@pytest.mark.parametrize("axis", [0, 1])
def test_reduction_backward(rsl, op, axis):
    rng = np.random.default_rng(20 + op)
    x = rng.uniform(0.9, 1.1, (33, 47)).astype(np.float32) if op == 3 else rng.standard_normal((33, 47)).astype(np.float32)
    x[3, :] = x[3, 0]  # ties: every tied max/min element gets the gradient
    RX = ref.Var.of(x, True)
    ro = ref.reduce(op, RX, axis)
    ref.binary(2, ro, ro).backward()
    fn = [rsl.sum, rsl.max, rsl.min, rsl.prod][op]
    X = rsl.Variable(x, requires_grad=True)
    mo = fn(X, axis)
    (mo * mo).backward()
    assert rel_err(mo.numpy(), ro.numpy()) <= 1e-5
    assert rel_err(X.grad.numpy(), RX.grad()) <= 1e-5


def test_transpose_and_views_backward(rsl):
    rng = np.random.default_rng(7)
    x = rng.standard_normal((6, 10)).astype(np.float32)
    w = rng.standard_normal((6, 10)).astype(np.float32)
    RX = ref.Var.of(x, True)
    ro = ref.matmul(ref.transpose(RX), ref.Var.of(w))
    ro.backward()
    X = rsl.Variable(x, requires_grad=True)
    mo = rsl.matmul(rsl.transpose(X), rsl.Variable(w))
    mo.backward()
    assert rel_err(mo.numpy(), ro.numpy()) <= 1e-5
    assert rel_err(X.grad.numpy(), RX.grad()) <= 1e-5
    Y = rsl.Variable(x, requires_grad=True)
    z = rsl.sum(rsl.reshape(Y, [60]) * 2.0, 0)
    z.backward()
    np.testing.assert_array_equal(Y.grad.numpy(), np.full((6, 10), 2.0, np.float32))
