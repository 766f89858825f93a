"""The drop-in boundary, end to end: the reference's own, unchanged front-end
(lmp::tensor::Tensor, lmp::autograd::Variable, its capture flag and its
pybind11 module csrc/bindings/core.cpp) compiled with its CUDA device served
by lmpb (rushlite_b200/lamp3_cuda/lmpb_dispatch.cpp registers lmpb in every
CUDA DispatchStub slot and as the CUDA LazyBackend).

Each case runs the same calls twice through the reference's API: on
DeviceType::CUDA (this backend) and on DeviceType::CPU (the reference's own
CPU kernels, the oracle).  The CUDA runs must launch lmpb kernels (the
library's launch counter moves) and agree with the CPU runs: bit-exact for
integer sums, max/min and comparisons, max|d|/max|ref| <= 1e-5 for float
arithmetic and reductions, <= 1e-4 for matmul chains with K >= 4096.
"""
from __future__ import annotations

import os
import sys

import numpy as np
import pytest

from oracle import ref
from rushlite_b200 import capi
from tests.util import assert_bitexact, rel_err

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PY_FRONT = os.path.join(ROOT, "rushlite_b200", "lamp3_cuda", "_build", "py")
DMAX = sys.float_info.max


@pytest.fixture(scope="module")
def front(cuda):
    """(CUDA harness, CPU harness) over the reference's C++ API."""
    if not (os.path.exists(ref.CUDA_LIB) and ref.available()):
        pytest.fail("the reference front-end on lmpb (oracle/_ref/liblamp3_cuda_harness.so) is not built")
    return ref.cuda_front(), ref.lib()


class Ops:
    """The reference's autograd ops on one harness library."""

    def __init__(self, L, capture=False):
        self.L, self.capture = L, capture

    def var(self, a, rg=False):
        return ref.Var.of(np.asarray(a), rg, self.L)

    def __enter__(self):
        self.L.lref_set_capture(int(self.capture))
        return self

    def __exit__(self, *exc):
        self.L.lref_set_capture(0)


def c2(o, a, b):
    one = o.var(np.ones((1,), np.float32))
    s = ref.binary(0, ref.binary(2, a, a), b)
    return ref.binary(1, ref.binary(2, ref.unary(1, s), a), ref.unary(2, ref.binary(0, b, one)))


def launches():
    return capi.kernel_launches()


@pytest.mark.parametrize("capture", [False, True])
def test_c2_chain_through_reference_api(front, capture):
    """BASELINE C2 at full size: the reference's Variable ops on CUDA, forward
    (fused by lmpb's lazy backend under capture) and backward."""
    Lc, Lh = front
    rng = np.random.default_rng(1234)
    a = rng.random((8192, 8192), dtype=np.float32)
    b = rng.random((8192, 1), dtype=np.float32)
    cpu = Ops(Lh)
    ha, hb = cpu.var(a, True), cpu.var(b, True)
    hd = c2(cpu, ha, hb)
    hd.backward()
    want = hd.numpy(), ha.grad(), hb.grad()
    del hd, ha, hb
    n0 = launches()
    with Ops(Lc, capture) as g:
        da, db = g.var(a, True), g.var(b, True)
        assert da.device == "cuda"
        dd = c2(g, da, db)
    dd.backward()
    got = dd.numpy(), da.grad(), db.grad()
    assert launches() > n0, "no lmpb kernel ran"
    for x, y in zip(got, want):
        assert rel_err(x, y) <= 1e-5


def test_capture_fuses_into_few_kernels(front):
    """Under capture the forward chain is recorded and realized by lmpb's
    lazy backend: the broadcast operand log(b + 1) and the full-size chain
    are two generated kernels instead of seven op-by-op launches."""
    Lc, _ = front
    rng = np.random.default_rng(2)
    a = rng.random((512, 256), dtype=np.float32)
    b = rng.random((512, 1), dtype=np.float32)
    eager = Ops(Lc)
    ea, eb = eager.var(a), eager.var(b)
    n0 = launches()
    e = c2(eager, ea, eb).numpy()
    n_eager = launches() - n0
    with Ops(Lc, True) as g:
        fa, fb = g.var(a), g.var(b)
        fd = c2(g, fa, fb)
    n0 = launches()
    f = fd.numpy()
    n_fused = launches() - n0
    assert_bitexact(f, e, "fused vs eager")
    assert n_fused <= 3 < n_eager, (n_fused, n_eager)


@pytest.mark.parametrize("axis", [0, 1])
def test_c3_reductions_through_reference_api(front, axis):
    Lc, Lh = front
    rng = np.random.default_rng(3)
    x = rng.standard_normal((16384, 4096), dtype=np.float32)
    xi = rng.integers(-1000, 1001, (16384, 4096)).astype(np.int32)
    for arr in (x, xi):
        hx, dx = ref.Var.of(arr, False, Lh), ref.Var.of(arr, False, Lc)
        for op in (0, 1, 2):
            got, want = ref.reduce(op, dx, axis).numpy(), ref.reduce(op, hx, axis).numpy()
            if op == 0 and arr.dtype == np.float32:
                assert rel_err(got, want) <= 1e-5
            else:
                assert_bitexact(got, want, f"op {op} axis {axis} {arr.dtype}")
    # sum backward: loss = s*s, grad_x = broadcast(2 s)
    hx, dx = ref.Var.of(x, True, Lh), ref.Var.of(x, True, Lc)
    for v in (hx, dx):
        s = ref.reduce(0, v, axis)
        ref.binary(2, s, s).backward()
    assert rel_err(dx.grad(), hx.grad()) <= 1e-5


@pytest.mark.parametrize("mkn", [(128, 96, 130), (1024, 1024, 1024)])
def test_matmul_backward_through_reference_api(front, mkn):
    Lc, Lh = front
    m, k, n = mkn
    rng = np.random.default_rng(m)
    a = (rng.standard_normal((m, k)) / np.sqrt(k)).astype(np.float32)
    b = rng.standard_normal((k, n)).astype(np.float32)
    res = []
    for L in (Lc, Lh):
        A, B = ref.Var.of(a, True, L), ref.Var.of(b, True, L)
        C = ref.matmul(A, B)
        ref.unary(5, C).backward()
        res.append((C.numpy(), A.grad(), B.grad()))
    for x, y in zip(*res):
        assert rel_err(x, y) <= 1e-5


def test_elementwise_ops_and_dtypes_through_reference_api(front):
    """Every binary/unary op of the dispatch table, with broadcasting and
    mixed dtypes, against the reference's CPU kernels."""
    Lc, Lh = front
    rng = np.random.default_rng(7)
    xs = {np.float32: rng.uniform(0.5, 2.0, (33, 40)).astype(np.float32),
          np.int32: rng.integers(-5, 6, (33, 40)).astype(np.int32),
          np.float64: rng.uniform(0.5, 2.0, (1, 40))}
    for op in range(11):
        for da, db in ((np.float32, np.float32), (np.int32, np.float32), (np.float32, np.float64),
                       (np.int32, np.int32)):
            a = xs[da]
            b = xs[db][:1] if db is np.float64 else xs[db][:, :1] if da is np.int32 else xs[db]
            if op == 3 and db is np.int32:
                b = np.where(b == 0, 1, b).astype(np.int32)  # integer division by zero traps on the CPU
            if op == 4 and da is np.int32 and db is np.int32:
                b = np.abs(b).astype(np.int32)
            got = ref.binary(op, ref.Var.of(a, False, Lc), ref.Var.of(b, False, Lc)).numpy()
            want = ref.binary(op, ref.Var.of(a, False, Lh), ref.Var.of(b, False, Lh)).numpy()
            # the reference's CPU build uses -ffast-math: its float division and
            # pow are not correctly rounded
            if op in (3, 4) and got.dtype.kind == "f":
                nan = np.isnan(want)  # a negative base to a fractional power
                assert np.array_equal(np.isnan(got), nan), (op, da, db)
                assert rel_err(got[~nan], want[~nan]) <= 1e-5, (op, da, db)
            else:
                assert_bitexact(got, want, f"binary {op} {da} {db}")
    x = xs[np.float32]
    for op in range(9):
        got = ref.unary(op, ref.Var.of(x, False, Lc), -1.0, 1.5).numpy()
        want = ref.unary(op, ref.Var.of(x, False, Lh), -1.0, 1.5).numpy()
        if op in (1, 2, 3, 5, 6, 7):  # transcendentals, and sqrt under -ffast-math
            assert rel_err(got, want) <= 1e-5, op
        else:
            assert_bitexact(got, want, f"unary {op}")


def test_readme_mlp_through_reference_pybind_module(cuda):
    """The reference's own Python extension (csrc/bindings/core.cpp, built on
    the lmpb-served core) trains the README MLP on device=cuda; the same
    module on device=cpu runs the reference's CPU kernels as the oracle.

    It runs in a fresh interpreter: the reference's module and this
    package's own extension bind C++ types of the same names, and pybind11
    keeps one registry per process."""
    import json
    import subprocess

    worker = os.path.join(ROOT, "tests", "lamp3_front_worker.py")
    r = subprocess.run([sys.executable, worker], capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-4000:]
    res = json.loads(r.stdout.strip().splitlines()[-1])
    assert res["cuda_available"]
    assert res["lmpb_launches"] > 0
    for step in res["steps"]:
        assert abs(step["loss_cuda"] - step["loss_cpu"]) <= 1e-5 * abs(step["loss_cpu"]), step
    assert max(res["param_rel_err"]) <= 1e-5, res["param_rel_err"]
