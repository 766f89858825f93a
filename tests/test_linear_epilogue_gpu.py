"""Linear(+ReLU) through one tensor-core GEMM: the bias row and the clamp run
in the GEMM epilogue (lmpb_gemm_f32_bias_act), and under capture the host
layer recognises clamp(matmul + bias) / matmul + bias and realizes it that
way.  Both must equal the three eager ops (matmul, broadcast add, clamp)
bit for bit, forward and backward."""
from __future__ import annotations

import sys

import numpy as np
import pytest

from rushlite_b200 import capi
from tests.util import assert_bitexact, rel_err

pytestmark = pytest.mark.gpu
FMAX = sys.float_info.max


def _dev(torch, a):
    return torch.as_tensor(np.ascontiguousarray(a), device="cuda")


# shapes for the CTA-pair kernel (m >= 256), the single-CTA kernel (64 <= m < 256),
# the SIMT fallback (small), odd n (not a multiple of 4) and padded k
@pytest.mark.parametrize("mkn", [(512, 384, 1000), (128, 256, 512), (300, 200, 260), (300, 200, 257), (32, 64, 10),
                                 (8192, 512, 256)])
@pytest.mark.parametrize("trans", [(0, 0), (1, 0), (0, 1)])
@pytest.mark.parametrize("act", ["bias", "bias_relu", "relu_only", "clamp_range"])
def test_gemm_bias_act_matches_eager_ops(cuda, mkn, trans, act):
    torch = cuda
    m, k, n = mkn
    rng = np.random.default_rng(m * 7 + n)
    A = (rng.standard_normal((k, m) if trans[0] else (m, k)) / np.sqrt(k)).astype(np.float32)
    B = rng.standard_normal((n, k) if trans[1] else (k, n)).astype(np.float32)
    bias = rng.standard_normal(n).astype(np.float32)
    use_bias = act != "relu_only"
    clamp, lo, hi = {"bias": (0, 0.0, 0.0), "bias_relu": (1, 0.0, FMAX), "relu_only": (1, 0.0, FMAX),
                     "clamp_range": (1, -0.25, 0.5)}[act]
    dA, dB, dbias = _dev(torch, A), _dev(torch, B), _dev(torch, bias)
    fused = torch.empty(m, n, device="cuda")
    capi.gemm_f32_bias_act(trans[0], trans[1], dA.data_ptr(), dB.data_ptr(), fused.data_ptr(), m, n, k,
                           dbias.data_ptr() if use_bias else None, clamp, lo, hi)
    ref = torch.empty(m, n, device="cuda")
    capi.gemm_f32(trans[0], trans[1], dA.data_ptr(), dB.data_ptr(), ref.data_ptr(), m, n, k, 0.0)
    if use_bias:
        capi.binary(capi.ADD, capi.FLOAT32, ref.data_ptr(), capi.FLOAT32, (m, n), dbias.data_ptr(), capi.FLOAT32,
                    (n,), ref.data_ptr())
    if clamp:
        capi.unary(capi.CLAMP, capi.FLOAT32, ref.data_ptr(), ref.data_ptr(), m * n, lo, hi)
    capi.device_error()
    assert_bitexact(fused.cpu().numpy(), ref.cpu().numpy(), f"{mkn} {trans} {act}")


@pytest.fixture(scope="module")
def rsl(cuda):
    import rushlite_b200

    return rushlite_b200


def _layer(rsl, x, W, b, relu):
    h = rsl.matmul(x, W) + b
    return rsl.clamp(h, 0.0, FMAX) if relu else h


@pytest.mark.parametrize("relu", [True, False])
@pytest.mark.parametrize("m", [512, 96])
def test_captured_linear_relu_matches_eager(rsl, relu, m):
    """Forward bit-exact; gradients of x, W and b against the uncaptured
    ops (the bias gradient's row sum may be ordered differently)."""
    rng = np.random.default_rng(3)
    k, n = 384, 320
    xs = rng.standard_normal((m, k)).astype(np.float32)
    Ws = (rng.standard_normal((k, n)) / np.sqrt(k)).astype(np.float32)
    bs = rng.standard_normal((n,)).astype(np.float32)
    outs = []
    for captured in (False, True):
        x = rsl.Variable(xs, requires_grad=True)
        W = rsl.Variable(Ws, requires_grad=True)
        b = rsl.Variable(bs, requires_grad=True)
        if captured:
            with rsl.capture_on():
                y = _layer(rsl, x, W, b, relu)
                loss = rsl.sum(rsl.sum(y * y, 1), 0)
        else:
            y = _layer(rsl, x, W, b, relu)
            loss = rsl.sum(rsl.sum(y * y, 1), 0)
        loss.backward()
        outs.append((y.numpy(), x.grad.numpy(), W.grad.numpy(), b.grad.numpy()))
    (y0, gx0, gW0, gb0), (y1, gx1, gW1, gb1) = outs
    assert_bitexact(y1, y0, "forward")
    assert rel_err(gx1, gx0) <= 1e-6
    assert rel_err(gW1, gW0) <= 1e-6
    assert rel_err(gb1, gb0) <= 1e-6


def test_pending_matmul_realizes_when_read(rsl):
    """The product inside a fused Linear is never written; reading it later
    realizes it as a plain GEMM with the same values."""
    rng = np.random.default_rng(4)
    xs = rng.standard_normal((256, 128)).astype(np.float32)
    Ws = rng.standard_normal((128, 192)).astype(np.float32)
    bs = rng.standard_normal((192,)).astype(np.float32)
    x, W, b = rsl.Variable(xs), rsl.Variable(Ws), rsl.Variable(bs)
    with rsl.capture_on():
        mm = rsl.matmul(x, W)
        y = rsl.clamp(mm + b, 0.0, FMAX)
    yv = y.numpy()
    mv = mm.numpy()
    eager = rsl.matmul(x, W).numpy()
    assert_bitexact(mv, eager, "pending product")
    assert_bitexact(yv, np.maximum(mv + bs, 0.0).astype(np.float32), "fused layer")


def test_copy_of_linear_into_its_own_input(rsl):
    """h.copy(relu(h @ W + b)): the pending value reads h through a matmul, at
    other indices than the one written, so it must not be realized straight
    into h's storage; the result equals the out-of-place layer."""
    rng = np.random.default_rng(8)
    hs = rng.standard_normal((256, 256)).astype(np.float32)
    Ws = (rng.standard_normal((256, 256)) / 16).astype(np.float32)
    bs = rng.standard_normal((256,)).astype(np.float32)
    W, b = rsl.Variable(Ws), rsl.Variable(bs)
    want = rsl.clamp(rsl.matmul(rsl.Variable(hs), W) + b, 0.0, FMAX).numpy()
    h = rsl.Variable(hs)
    p0 = h.data.data_ptr()
    with rsl.no_grad(), rsl.capture_on():
        h.data.copy(rsl.clamp(rsl.matmul(h, W) + b, 0.0, FMAX).data)
    assert h.data.data_ptr() == p0
    assert_bitexact(h.numpy(), want, "in-place copy of a Linear of its own input")
