"""Edge cases through the public API on the GPU: empty tensors, zero-size
reductions and matmul, high-rank broadcasting, mixed dtypes under capture,
scalar operands taking the tensor's dtype, and sizes that do not fill a
vector packet.  Checked against the CPU restatement (oracle/port)."""
from __future__ import annotations

import numpy as np
import pytest

from oracle import port
from tests.util import assert_bitexact, rel_err

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def rsl(cuda):
    import rushlite_b200

    return rushlite_b200


DT = {np.dtype(np.float32): "float32", np.dtype(np.float64): "float64", np.dtype(np.int32): "int32",
      np.dtype(np.int64): "int64", np.dtype(np.int16): "int16", np.dtype(np.bool_): "bool"}


def V(rsl, a, rg=False):
    a = np.asarray(a)
    return rsl.Variable(a, requires_grad=rg, dtype=getattr(rsl.dtype, DT[a.dtype]))


def test_empty_tensors(rsl):
    a = V(rsl, np.zeros((0, 4), np.float32), True)
    b = V(rsl, np.ones((1, 4), np.float32))
    for cap in (False, True):
        with rsl.capture_on(cap):
            c = rsl.exp(a * b + 1.0)
        assert c.numpy().shape == (0, 4)
    s0 = rsl.sum(a, 0)  # reduce an empty axis: the identity
    assert_bitexact(s0.numpy(), np.zeros((1, 4), np.float32))
    assert rsl.sum(a, 1).numpy().shape == (0, 1)
    assert_bitexact(rsl.max(a, 0).numpy(), np.full((1, 4), np.finfo(np.float32).min, np.float32))
    m = rsl.matmul(V(rsl, np.zeros((3, 0), np.float32)), V(rsl, np.zeros((0, 5), np.float32)))
    assert_bitexact(m.numpy(), np.zeros((3, 5), np.float32))


def test_high_rank_broadcast(rsl):
    rng = np.random.default_rng(1)
    sa = (2, 1, 3, 1, 2, 1, 2, 3)
    sb = (1, 4, 1, 2, 1, 3, 2, 1)
    a = rng.standard_normal(sa).astype(np.float32)
    b = rng.standard_normal(sb).astype(np.float32)
    want = port.binary(2, port.binary(0, a, b), a)
    for cap in (False, True):
        with rsl.capture_on(cap):
            got = (V(rsl, a) + V(rsl, b)) * V(rsl, a)
        assert_bitexact(got.numpy(), want)


def test_mixed_dtypes_under_capture(rsl):
    rng = np.random.default_rng(2)
    i = rng.integers(-50, 50, (33, 17)).astype(np.int32)
    f = rng.standard_normal((1, 17)).astype(np.float64)
    h = rng.integers(-3, 3, (33, 1)).astype(np.int16)
    want = port.binary(1, port.binary(2, i, f), h)  # int32*float64 -> f64, minus int16
    with rsl.capture_on():
        got = V(rsl, i) * V(rsl, f) - V(rsl, h)
    assert got.numpy().dtype == np.float64
    assert_bitexact(got.numpy(), want)


def test_scalar_takes_tensor_dtype(rsl):
    """csrc/include/lamp3/autograd/functions/overloads.hpp:16-29: the scalar
    becomes a {1} tensor of the Variable's dtype, so int * 0.5 multiplies by 0."""
    x = np.arange(1, 7, dtype=np.int32).reshape(3, 2)
    for cap in (False, True):
        with rsl.capture_on(cap):
            y = V(rsl, x) * 0.5
            z = 2.7 + V(rsl, x)
        assert_bitexact(y.numpy(), np.zeros_like(x))
        assert_bitexact(z.numpy(), x + 2)


@pytest.mark.parametrize("n", [1, 3, 5, 7, 9, 15, 17, 4097, 65537])
def test_odd_sizes_fused_and_eager(rsl, n):
    rng = np.random.default_rng(n)
    a = rng.random((n,), dtype=np.float32)
    b = rng.random((n,), dtype=np.float32)
    want = port.binary(3, port.binary(2, a, b), port.binary(0, a, np.ones((1,), np.float32)))
    for cap in (False, True):
        with rsl.capture_on(cap):
            got = (V(rsl, a) * V(rsl, b)) / (V(rsl, a) + 1.0)
        assert_bitexact(got.numpy(), want)
    # backward with a row-reduce epilogue over an odd width
    A = V(rsl, a.reshape(1, n), True)
    B = V(rsl, np.float32([[0.5]]), True)
    with rsl.capture_on():
        d = rsl.exp(A * B) * A
    d.backward()
    x = np.exp(a.astype(np.float64) * 0.5)
    assert rel_err(B.grad.numpy(), [[np.sum(a.astype(np.float64) ** 2 * x)]]) <= 1e-5
    assert rel_err(A.grad.numpy().ravel(), x * (1 + 0.5 * a)) <= 1e-5


def test_bias_grad_column_reduce(rsl):
    """Linear-layer bias gradient: the broadcast sum over the batch axis is a
    column-reduce epilogue (split rows, combined in order)."""
    rng = np.random.default_rng(3)
    x = rng.standard_normal((4096, 1000)).astype(np.float32)
    bias = rng.standard_normal((1000,)).astype(np.float32)
    X, Bv = V(rsl, x), V(rsl, bias, True)
    with rsl.capture_on():
        h = rsl.clamp(X + Bv, 0, 3.0e38)
    h.backward()
    want = ((x + bias) > 0).sum(0).astype(np.float64)
    assert rel_err(Bv.grad.numpy(), want) <= 1e-6


def test_async_upload_download(rsl, cuda):
    """rsl.upload / download_async on the copy streams: results equal the
    synchronous path, across back-to-back steps that overlap."""
    torch = cuda
    rng = np.random.default_rng(11)
    a = torch.empty((512, 1024), dtype=torch.float32, pin_memory=True).numpy()
    b = torch.empty((512, 1), dtype=torch.float32, pin_memory=True).numpy()
    a[...] = rng.random((512, 1024), dtype=np.float32)
    b[...] = rng.random((512, 1), dtype=np.float32)
    outs = [torch.empty((512, 1024), dtype=torch.float32, pin_memory=True).numpy() for _ in range(3)]
    handles = []
    for i in range(3):
        A = rsl.upload(a, True)
        B = rsl.upload(b)
        with rsl.capture_on():
            d = rsl.exp(A * B) - A
        handles.append(d.data.download_async(outs[i]))
        d.backward()
        handles.append(None)
    for h in handles:
        if h is not None:
            h.wait()
    want = V(rsl, a) * V(rsl, b)
    want = (rsl.exp(want) - V(rsl, a)).numpy()
    for o in outs:
        assert_bitexact(o, want)
    g = np.zeros((512, 1024), np.float32)
    A.grad.download_async(g).wait()
    assert rel_err(g, np.exp(a.astype(np.float64) * b) * b - 1) <= 1e-5
