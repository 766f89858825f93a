"""Row softmax and its loss fused into one kernel (the remaining part of the
GEMM-epilogue/softmax fusion row), against the unfused ops.

The reference's softmax is max, subtract, exp, sum, divide
(src/rushlite/nets/layers/activation.py:26-40), four launches and a
materialised intermediate per op.  Under capture the max and the sum over the
last axis stay pending, and the kernel that reads them computes them per row
(LMPB_FN_ROWRED nodes: one walk along the row per reduction, the same thread
order and warp/CTA tree as the eager reduction kernel).  So:

* an in-kernel row sum / max equals lmpb_reduce over the last axis bit for
  bit (C ABI, several row lengths, warp and CTA rows, packet widths 8/4/2/1);
* softmax + cross-entropy forward and backward under capture equal the same
  calls issued op by op without capture, bit for bit;
* the forward softmax + loss row sums run as one kernel.
"""
from __future__ import annotations

import numpy as np
import pytest

from rushlite_b200 import capi
from tests.util import assert_bitexact

pytestmark = pytest.mark.gpu

F32 = capi.FLOAT32
LEAF, CONST, BIN, UN, ROWRED = 0, 1, 2, 3, 4


def _dev(torch, a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


@pytest.mark.parametrize("shape", [(64, 1000), (37, 4096), (5, 24), (7, 6), (3, 7), (1, 2048), (300, 130)])
@pytest.mark.parametrize("op", [capi.SUM, capi.MAX])
def test_rowred_node_equals_eager_reduction(cuda, shape, op):
    torch = cuda
    rng = np.random.default_rng(shape[0] * 31 + shape[1])
    x = rng.standard_normal(shape).astype(np.float32)
    dx = _dev(torch, x)
    R = shape[0]
    want = torch.empty((R, 1), device="cuda")
    capi.reduce(op, F32, dx.data_ptr(), list(shape), 1, want.data_ptr())
    # program: r = ROWRED(x); out = x - r (full) ; and r itself via x*0 + r summed?  Store x - r.
    nodes = [(LEAF, 0, F32, 0, 0), (ROWRED, op, F32, 0, 0), (BIN, capi.SUB, F32, 0, 1)]
    f = capi.Fused(nodes, [(F32, list(shape))], [(2, 0, F32, list(shape))], list(shape))
    out = torch.empty(shape, device="cuda")
    f.launch([dx.data_ptr()], [out.data_ptr()])
    torch.cuda.synchronize()
    # x - r rounds once per element: recover r exactly from an element where x == max (op MAX)
    # or compare x - r against x - want computed the same way
    ref_out = (dx - want).cpu().numpy()
    assert_bitexact(out.cpu().numpy(), ref_out, f"ROWRED {op} {shape}")


def test_fused_reduce_output_equals_eager_row_sum(cuda):
    """A fused REDUCE_SUM output over the last axis and lmpb_reduce agree bit for bit."""
    torch = cuda
    rng = np.random.default_rng(3)
    for shape in [(64, 1000), (37, 4096), (9, 30)]:
        x = rng.standard_normal(shape).astype(np.float32)
        dx = _dev(torch, x)
        want = torch.empty((shape[0], 1), device="cuda")
        capi.reduce(capi.SUM, F32, dx.data_ptr(), list(shape), 1, want.data_ptr())
        f = capi.Fused([(LEAF, 0, F32, 0, 0)], [(F32, list(shape))], [(0, 2, F32, [shape[0], 1])], list(shape))
        got = torch.empty((shape[0], 1), device="cuda")
        f.launch([dx.data_ptr()], [got.data_ptr()])
        torch.cuda.synchronize()
        assert_bitexact(got.cpu().numpy(), want.cpu().numpy(), f"row sum {shape}")


def _softmax_loss(rsl, h, y):
    m = rsl.max(h, 1)
    e = rsl.exp(h - m)
    p = e / rsl.sum(e, 1)
    return p, rsl.sum(rsl.sum(-y * rsl.log(p + 1e-3), 1), 0)


@pytest.mark.parametrize("shape", [(512, 1000), (64, 4096), (32, 10)])
def test_softmax_loss_capture_equals_eager(cuda, shape):
    import rushlite_b200 as rsl

    rng = np.random.default_rng(11)
    hs = (3 * rng.standard_normal(shape)).astype(np.float32)
    ys = np.zeros(shape, np.float32)
    ys[np.arange(shape[0]), rng.integers(0, shape[1], shape[0])] = 1
    res = []
    for cap in (False, True):
        h = rsl.Variable(hs, requires_grad=True)
        y = rsl.Variable(ys)
        with rsl.capture_on(cap):
            p, loss = _softmax_loss(rsl, h, y)
        loss.backward()
        res.append((p.numpy(), loss.numpy(), h.grad.numpy()))
    for a, b, what in zip(res[0], res[1], ("softmax", "loss", "grad")):
        assert_bitexact(b, a, f"{what} {shape}")


def test_softmax_loss_forward_is_one_kernel(cuda):
    import rushlite_b200 as rsl

    rng = np.random.default_rng(12)
    h = rsl.Variable(rng.standard_normal((256, 1000)).astype(np.float32))
    y = rsl.Variable(rng.random((256, 1000), dtype=np.float32))
    h.realize()
    y.realize()
    with rsl.capture_on():
        m = rsl.max(h, 1)
        e = rsl.exp(h - m)
        p = e / rsl.sum(e, 1)
        t = rsl.sum(-y * rsl.log(p + 1e-3), 1)
    n0 = rsl.cuda.kernel_launches()
    t.realize()
    assert rsl.cuda.kernel_launches() - n0 == 1
