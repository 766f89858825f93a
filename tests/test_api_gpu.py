"""Parity of the public API (rushlite_b200: Variable, ops, capture, backward)
on the GPU against the reference's own CPU build (oracle/_ref) on the same
seeded inputs, plus the reference's known answers (tests/golden)."""
from __future__ import annotations

import json
import os

import numpy as np
import pytest

from oracle import port, ref
from tests.util import assert_bitexact, rel_err

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))
KA = json.load(open(os.path.join(HERE, "golden", "known_answers.json")))
needs_ref = pytest.mark.skipif(not ref.available(), reason="reference CPU build (oracle/_ref) absent")


@pytest.fixture(scope="module")
def rsl(cuda):
    import rushlite_b200

    return rushlite_b200


def V(rsl, a, rg=False):
    a = np.asarray(a)
    dt = {np.dtype(np.float32): rsl.dtype.float32, np.dtype(np.float64): rsl.dtype.float64,
          np.dtype(np.int32): rsl.dtype.int32, np.dtype(np.int64): rsl.dtype.int64,
          np.dtype(np.int16): rsl.dtype.int16, np.dtype(np.bool_): rsl.dtype.bool}[a.dtype]
    return rsl.Variable(a, requires_grad=rg, device=rsl.device.cuda, dtype=dt)


class RslOps:
    def __init__(self, rsl):
        self.r = rsl

    def var(self, a, rg=False):
        return V(self.r, a, rg)

    def bin(self, op, a, b):
        return [self.r.add, self.r.sub, self.r.mul, self.r.div, self.r.pow][op](a, b)

    def un(self, op, a, p0=0.0, p1=0.0):
        r = self.r
        return [r.neg, r.exp, r.log, r.sqrt, r.abs, r.sin, r.cos, r.tan][op](a) if op < 8 else r.clamp(a, p0, p1)

    def red(self, op, a, axis):
        return [self.r.sum, self.r.max, self.r.min, self.r.prod][op](a, axis)

    def mm(self, a, b):
        return self.r.matmul(a, b)

    def val(self, v):
        return v.numpy()

    def grad(self, v):
        return v.grad.numpy()


class RefOps:
    def var(self, a, rg=False):
        return ref.Var.of(np.asarray(a), rg)

    def bin(self, op, a, b):
        return ref.binary(op, a, b)

    def un(self, op, a, p0=0.0, p1=0.0):
        return ref.unary(op, a, p0, p1)

    def red(self, op, a, axis):
        return ref.reduce(op, a, axis)

    def mm(self, a, b):
        return ref.matmul(a, b)

    def val(self, v):
        return v.numpy()

    def grad(self, v):
        return v.grad()


def _f(v):
    return {"inf": np.inf, "-inf": -np.inf}.get(v, v) if isinstance(v, str) else v


def test_known_answers_autograd(rsl):
    a = np.array([1, 2, 3, 4, 5, 2], np.float32).reshape(3, 2)
    b = np.array([-1, 4, -2, 0, 3, 0.5], np.float32).reshape(3, 2)
    for case in KA["autograd"]:
        A, B = V(rsl, a, True), V(rsl, b, True)
        e = case["expr"]
        M = None
        if e == "a + b":
            out = A + B
        elif e == "a - b":
            out = A - B
        elif e == "a * b":
            out = A * B
        elif e == "a / b":
            out = A / B
        elif e.startswith("sum"):
            out = rsl.sum(A, 1)
        elif e.startswith("max"):
            out = rsl.max(A, 1)
        else:
            M = V(rsl, np.array([[-1], [4]], np.float32), True)
            out = rsl.matmul(A, M)
        np.testing.assert_allclose(out.numpy().ravel(), [_f(x) for x in case["out"]], atol=1e-5, err_msg=e)
        out.backward()
        np.testing.assert_allclose(A.grad.numpy().ravel(), [_f(x) for x in case["grad_a"]], atol=1e-5, err_msg=e)
        if "grad_b" in case:
            np.testing.assert_allclose(B.grad.numpy().ravel(), [_f(x) for x in case["grad_b"]], atol=1e-5, err_msg=e)
        if M is not None:
            np.testing.assert_allclose(M.grad.numpy().ravel(), case["grad_m"], atol=1e-5)


def test_known_answers_tensor_ops(rsl):
    BIN = {"add": rsl.add, "sub": rsl.sub, "mul": rsl.mul, "div": rsl.div, "pow": rsl.pow, "eq": rsl.eq,
           "ne": rsl.ne, "ge": rsl.ge, "le": rsl.le, "gt": rsl.gt, "lt": rsl.lt}
    for case in KA["tensor"]:
        op = case["op"]
        arr = lambda s: np.array(s[0], dtype=np.float64).astype(s[2]).reshape(s[1])  # noqa: E731
        a = V(rsl, arr(case["a"]))
        if op in BIN:
            out = BIN[op](a, V(rsl, arr(case["b"])))
        elif op in ("sum", "max", "min"):
            out = getattr(rsl, op)(a, case["axis"])
        elif op == "matmul":
            out = rsl.matmul(a, V(rsl, arr(case["b"])))
        elif op == "transpose":
            out = rsl.transpose(a)
        elif op == "clamp_backward":
            out = rsl.Variable(rsl.clamp_backward(a.data, V(rsl, arr(case["b"])).data, *case["p"]))
        else:
            out = rsl.Variable(rsl.abs_backward(a.data, V(rsl, arr(case["b"])).data))
        got = out.numpy().ravel().astype(np.float64)
        np.testing.assert_allclose(got, case["expect"], rtol=case.get("rtol", 1e-6), atol=1e-5, err_msg=case["src"])
        if "out_dtype" in case:
            assert out.numpy().dtype == np.dtype(case["out_dtype"])


def c2_chain(ops, a, b):
    """d = exp(a*a + b) * a - log(b + 1)  (BASELINE config C2)."""
    one = ops.var(np.ones((1,), np.float32))
    return ops.bin(1, ops.bin(2, ops.un(1, ops.bin(0, ops.bin(2, a, a), b)), a), ops.un(2, ops.bin(0, b, one)))


@needs_ref
@pytest.mark.parametrize("capture", [False, True])
def test_c2_chain_vs_reference_small(rsl, capture):
    rng = np.random.default_rng(21)
    a = rng.random((128, 256), dtype=np.float32)
    b = rng.random((128, 1), dtype=np.float32)
    R, M = RefOps(), RslOps(rsl)
    ra, rb = R.var(a, True), R.var(b, True)
    rd = c2_chain(R, ra, rb)
    rd.backward()
    ma, mb = M.var(a, True), M.var(b, True)
    with rsl.capture_on(capture):
        md = c2_chain(M, ma, mb)
    md.backward()
    assert rel_err(md.numpy(), rd.numpy()) <= 1e-5
    assert rel_err(ma.grad.numpy(), ra.grad()) <= 1e-5
    assert rel_err(mb.grad.numpy(), rb.grad()) <= 1e-5


def test_capture_matches_eager_bitexact(rsl):
    """Fusion on/off equivalence (tests/graphs/runner.py of the reference):
    the fused kernel rounds every op like the op-by-op kernels."""
    rng = np.random.default_rng(5)
    a = rng.random((300, 1000), dtype=np.float32)
    b = rng.random((300, 1), dtype=np.float32)
    M = RslOps(rsl)
    eager = c2_chain(M, M.var(a), M.var(b)).numpy()
    with rsl.capture_on():
        fused = c2_chain(M, M.var(a), M.var(b))
    assert_bitexact(fused.numpy(), eager)


def test_c2_full_size_forward_backward(rsl):
    """C2 at its BASELINE size against the CPU restatement (forward) and the
    closed-form gradient in fp64."""
    rng = np.random.default_rng(0)
    a = rng.random((8192, 8192), dtype=np.float32)
    b = rng.random((8192, 1), dtype=np.float32)
    M = RslOps(rsl)
    ma, mb = M.var(a, True), M.var(b, True)
    with rsl.capture_on():
        d = c2_chain(M, ma, mb)
    d.backward()
    one = np.ones((1,), np.float32)
    c = port.binary(0, port.binary(2, a, a), b)
    x = port.unary(1, c)
    want = port.binary(1, port.binary(2, x, a), port.unary(2, port.binary(0, b, one)))
    assert rel_err(d.numpy(), want) <= 1e-5
    x64, a64 = x.astype(np.float64), a.astype(np.float64)
    assert rel_err(ma.grad.numpy(), x64 * (2 * a64 * a64 + 1)) <= 1e-5
    gb = (x64 * a64).sum(1, keepdims=True) - 8192.0 / (b.astype(np.float64) + 1)
    assert rel_err(mb.grad.numpy(), gb) <= 1e-5


def test_repeated_backward_accumulates_in_place(rsl):
    """csrc/tests/autograd_tests.cpp:487-499: gradients accumulate into the
    same buffer across backward calls."""
    a = V(rsl, np.array([1, 2, 3, 4, 5, 2], np.float32).reshape(3, 2), True)
    b = V(rsl, np.array([-1, 4, -2, 0, 3, 0.5], np.float32).reshape(3, 2), True)
    out = a * b
    out.backward()
    p0 = a.grad.data_ptr()
    out.backward()
    assert a.grad.data_ptr() == p0
    np.testing.assert_allclose(a.grad.numpy().ravel(), 2 * np.array([-1, 4, -2, 0, 3, 0.5]))


@needs_ref
@pytest.mark.parametrize("op", [0, 1, 2, 3])
@pytest.mark.parametrize("axis", [0, 1])
def test_reductions_with_backward_vs_reference(rsl, op, axis):
    rng = np.random.default_rng(op * 3 + axis)
    a = rng.standard_normal((64, 96)).astype(np.float32)
    if op == 3:
        a = rng.uniform(0.9, 1.1, (64, 96)).astype(np.float32)
    R, M = RefOps(), RslOps(rsl)
    ra, ma = R.var(a, True), M.var(a, True)
    ro, mo = R.red(op, ra, axis), M.red(op, ma, axis)
    ro2 = R.bin(2, ro, ro)
    mo2 = M.bin(2, mo, mo)
    ro2.backward()
    mo2.backward()
    assert rel_err(mo.numpy(), ro.numpy()) <= 1e-5
    assert rel_err(ma.grad.numpy(), ra.grad()) <= 1e-5


@needs_ref
@pytest.mark.parametrize("mkn", [(32, 256, 64), (32, 64, 10), (128, 96, 130)])
def test_matmul_with_backward_vs_reference(rsl, mkn):
    m, k, n = mkn
    rng = np.random.default_rng(m + n)
    a = (rng.standard_normal((m, k)) / np.sqrt(k)).astype(np.float32)
    b = rng.standard_normal((k, n)).astype(np.float32)
    R, M = RefOps(), RslOps(rsl)
    ra, rb, ma, mb = R.var(a, True), R.var(b, True), M.var(a, True), M.var(b, True)
    ro, mo = R.mm(ra, rb), M.mm(ma, mb)
    R.un(5, ro).backward()  # sin() so the output gradient is not all ones
    M.un(5, mo).backward()
    assert rel_err(mo.numpy(), ro.numpy()) <= 1e-5
    assert rel_err(ma.grad.numpy(), ra.grad()) <= 1e-5
    assert rel_err(mb.grad.numpy(), rb.grad()) <= 1e-5


@needs_ref
@pytest.mark.parametrize("seed", range(8))
def test_random_graph_chains_vs_reference(rsl, seed):
    """tests/graphs of the reference: random chains of binary/unary ops with
    broadcasting leaves, a matmul barrier and a reduction, forward + backward,
    with and without capture."""
    rng = np.random.default_rng(seed)
    S, Mx = (16, 16), (16, 8)
    shapes = [S, (1, 16), (16, 1), Mx, Mx, (8,), Mx]
    leaves = [(rng.uniform(-1, 1, s)).astype(np.float32) for s in shapes]
    bins = rng.integers(0, 3, size=5)
    un = int(rng.integers(0, 8))
    red = int(rng.integers(0, 3))

    def build(ops, xs):
        t = ops.bin(int(bins[0]), xs[0], xs[1])
        t = ops.bin(int(bins[1]), t, xs[2])
        t = ops.un(8, t, -1.0, 1.0)                       # clamp guard
        t = ops.un(un, t) if un not in (2, 3) else ops.un(un, ops.un(8, t, 1e-3, 1e3))
        t = ops.mm(t, xs[3])
        t = ops.bin(int(bins[2]), t, xs[4])
        t = ops.bin(int(bins[3]), t, xs[5])
        t = ops.bin(int(bins[4]), t, xs[6])
        return ops.red(red, t, 0)

    R, M = RefOps(), RslOps(rsl)
    rx = [R.var(x, True) for x in leaves]
    ro = build(R, rx)
    ro.backward()
    for cap in (False, True):
        mx = [M.var(x, True) for x in leaves]
        with rsl.capture_on(cap):
            mo = build(M, mx)
        mo.backward()
        assert rel_err(mo.numpy(), ro.numpy()) <= 1e-4
        for r_, m_ in zip(rx, mx):
            assert rel_err(m_.grad.numpy(), r_.grad()) <= 2e-4


def test_errors_are_runtime_errors(rsl):
    a = V(rsl, np.ones((3, 2), np.float32))
    b = V(rsl, np.ones((4, 2), np.float32))
    with pytest.raises(RuntimeError, match="Broadcast"):
        rsl.add(a, b)
    with pytest.raises(RuntimeError):
        rsl.matmul(a, a)
    with pytest.raises(RuntimeError):
        rsl.sum(a, 5)
