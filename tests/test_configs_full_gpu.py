"""Parity at the BASELINE configs' full sizes.

* C2: d = exp(a*a + b)*a - log(b+1), a [8192, 8192], b [8192, 1], forward
  under capture plus backward w.r.t. a and b, against the reference's own CPU
  build (oracle/_ref) on the same seeded inputs.
* C3: sum / max / min along both axes of fp32 N(0,1) [16384, 4096] and the
  int32 U{-1000..1000} sum, plus the backward of sum, against oracle/_ref;
  max, min and int32 bit-exact.
* C4: the tcgen05 fp32 GEMM at 8192^3 and (32768, 4096, 4096) forward, and the
  two gradient products dA = G·Bᵀ and dB = Aᵀ·G through the transposed-operand
  flags at 4096^3 and 8192^3, against float64 (<= 1e-4 at K >= 4096).
* C5: one full-width training step (4 x Linear(4096, 4096) + ReLU,
  Linear(4096, 1000) + softmax, batch 8192, one-hot labels), loss and every
  parameter gradient against the same step in float64.

The float64 references of C4 and C5 run on the GPU in torch (float64 GEMMs);
the reference's CPU build would need hours for them.
"""
from __future__ import annotations

import sys

import numpy as np
import pytest

from oracle import ref
from rushlite_b200 import capi
from tests.test_api_gpu import RefOps, RslOps, c2_chain
from tests.util import assert_bitexact, rel_err

pytestmark = pytest.mark.gpu
needs_ref = pytest.mark.skipif(not ref.available(), reason="reference CPU build (oracle/_ref) absent")
DMAX = sys.float_info.max


@pytest.fixture(scope="module")
def rsl(cuda):
    import rushlite_b200

    return rushlite_b200


@needs_ref
def test_c2_full_size_vs_reference(rsl):
    rng = np.random.default_rng(1234)
    a = rng.random((8192, 8192), dtype=np.float32)
    b = rng.random((8192, 1), dtype=np.float32)
    R, M = RefOps(), RslOps(rsl)
    ra, rb = R.var(a, True), R.var(b, True)
    rd = c2_chain(R, ra, rb)
    rd.backward()
    want_d, want_ga, want_gb = rd.numpy(), ra.grad(), rb.grad()
    del rd, ra, rb
    ma, mb = M.var(a, True), M.var(b, True)
    with rsl.capture_on():
        md = c2_chain(M, ma, mb)
    md.backward()
    assert rel_err(md.numpy(), want_d) <= 1e-5
    assert rel_err(ma.grad.numpy(), want_ga) <= 1e-5
    assert rel_err(mb.grad.numpy(), want_gb) <= 1e-5
    # A second backward over the same graph (the reference's timed loop):
    # every Variable's gradient, intermediates included, accumulates in place,
    # so the leaves receive more than twice the first gradient; the result
    # must still match the reference's second backward.
    del md, ma, mb
    ra, rb = R.var(a, True), R.var(b, True)
    rd = c2_chain(R, ra, rb)
    rd.backward()
    rd.backward()
    want_ga, want_gb = ra.grad(), rb.grad()
    del rd, ra, rb
    ma, mb = M.var(a, True), M.var(b, True)
    with rsl.capture_on():
        md = c2_chain(M, ma, mb)
    md.backward()
    md.backward()
    assert rel_err(ma.grad.numpy(), want_ga) <= 1e-5
    assert rel_err(mb.grad.numpy(), want_gb) <= 1e-5


@needs_ref
@pytest.mark.parametrize("axis", [0, 1])
def test_c3_full_size_vs_reference(rsl, axis):
    rng = np.random.default_rng(3)
    x = rng.standard_normal((16384, 4096), dtype=np.float32)
    xi = rng.integers(-1000, 1001, size=(16384, 4096)).astype(np.int32)
    R, M = RefOps(), RslOps(rsl)
    rx, mx = R.var(x), M.var(x)
    for op in (0, 1, 2):
        got, want = M.red(op, mx, axis).numpy(), R.red(op, rx, axis).numpy()
        if op == 0:
            assert rel_err(got, want) <= 1e-5
        else:
            assert_bitexact(got, want, f"C3 op{op} axis{axis}")
    assert_bitexact(M.red(0, M.var(xi), axis).numpy(), R.red(0, R.var(xi), axis).numpy(), "C3 int32 sum")
    # backward of sum: loss = s*s elementwise, so grad_x = broadcast(2*s)
    rx, mx = R.var(x, True), M.var(x, True)
    rs, ms = R.red(0, rx, axis), M.red(0, mx, axis)
    R.bin(2, rs, rs).backward()
    M.bin(2, ms, ms).backward()
    assert rel_err(mx.grad.numpy(), rx.grad()) <= 1e-5


def _gemm(torch, ta, tb, A, B, m, n, k):
    C = torch.empty(m, n, device="cuda")
    capi.gemm_f32(ta, tb, A.data_ptr(), B.data_ptr(), C.data_ptr(), m, n, k, 0.0)
    capi.device_error()
    return C


def _rel(torch, got, want64):
    return ((got.double() - want64).abs().max() / want64.abs().max()).item()


@pytest.mark.parametrize("mkn", [(8192, 8192, 8192), (32768, 4096, 4096)])
def test_c4_forward_full_size(cuda, mkn):
    torch = cuda
    m, k, n = mkn
    g = torch.Generator(device="cuda").manual_seed(m + k + n)
    A = torch.randn(m, k, device="cuda", generator=g) / k ** 0.5
    B = torch.randn(k, n, device="cuda", generator=g) / k ** 0.5
    C = _gemm(torch, 0, 0, A, B, m, n, k)
    assert _rel(torch, C, A.double() @ B.double()) <= 1e-4


@pytest.mark.parametrize("mkn", [(4096, 4096, 4096), (8192, 8192, 8192)])
def test_c4_backward_full_size(cuda, mkn):
    """dA = G·Bᵀ (trans_b) and dB = Aᵀ·G (trans_a), G an upstream gradient."""
    torch = cuda
    m, k, n = mkn
    g = torch.Generator(device="cuda").manual_seed(m + 7)
    A = torch.randn(m, k, device="cuda", generator=g) / k ** 0.5
    B = torch.randn(k, n, device="cuda", generator=g) / k ** 0.5
    G = torch.randn(m, n, device="cuda", generator=g)
    dA = _gemm(torch, 0, 1, G, B, m, k, n)
    assert _rel(torch, dA, G.double() @ B.double().T) <= 1e-4
    dB = _gemm(torch, 1, 0, A, G, k, n, m)
    assert _rel(torch, dB, A.double().T @ G.double()) <= 1e-4


def test_c4_through_public_api(rsl, cuda):
    """matmul + backward through Variable at 4096^3 with a non-uniform upstream
    gradient (sin of the product), against float64."""
    torch = cuda
    m = k = n = 4096
    rng = np.random.default_rng(44)
    a = (rng.standard_normal((m, k)) / np.sqrt(k)).astype(np.float32)
    b = (rng.standard_normal((k, n)) / np.sqrt(k)).astype(np.float32)
    A, B = rsl.Variable(a, requires_grad=True), rsl.Variable(b, requires_grad=True)
    c = rsl.matmul(A, B)
    rsl.sin(c).backward()
    A64, B64 = torch.from_numpy(a).cuda().double(), torch.from_numpy(b).cuda().double()
    C64 = A64 @ B64
    G64 = torch.cos(torch.from_numpy(c.numpy()).cuda().double())
    assert _rel(torch, torch.from_numpy(c.numpy()).cuda(), C64) <= 1e-4
    assert _rel(torch, torch.from_numpy(A.grad.numpy()).cuda(), G64 @ B64.T) <= 1e-4
    assert _rel(torch, torch.from_numpy(B.grad.numpy()).cuda(), A64.T @ G64) <= 1e-4


def _c5_params(dims, seed):
    rng = np.random.default_rng(seed)
    ps = []
    for i in range(len(dims) - 1):
        ps.append((rng.standard_normal((dims[i], dims[i + 1])) / np.sqrt(dims[i])).astype(np.float32))
        ps.append((rng.standard_normal((dims[i + 1],)) / np.sqrt(dims[i])).astype(np.float32))
    return ps


def c5_f64_grads(torch, params, x, y, masks):
    """Loss and parameter gradients of the C5 step in float64 on the GPU:
    relu MLP, softmax with the max subtracted, loss (-y*log(p+1e-3)).sum().

    The ReLU masks are the ones the fp32 step under test produced.  A ReLU is
    a step function: wherever a pre-activation lies within fp32 rounding of
    zero (29-54 of the 33.5 M per layer at this size), fp32 and float64 take
    different branches, and one flipped mask entry moves a whole column of a
    weight gradient by ~1 % of its maximum.  With the masks shared, the
    comparison measures rounding error only."""
    P = [torch.from_numpy(p).cuda().double() for p in params]
    h = torch.from_numpy(x).cuda().double()
    Y = torch.from_numpy(y).cuda().double()
    hs = [h]
    n = len(P) // 2
    for i in range(n):
        z = h @ P[2 * i] + P[2 * i + 1]
        h = z * masks[i] if i < n - 1 else z
        hs.append(h)
    e = torch.exp(h - h.max(1, keepdim=True).values)
    p = e / e.sum(1, keepdim=True)
    loss = float((-Y * torch.log(p + 1e-3)).sum())
    gp = -Y / (p + 1e-3)
    g = p * (gp - (gp * p).sum(1, keepdim=True))
    grads = [None] * len(P)
    for i in reversed(range(n)):
        grads[2 * i], grads[2 * i + 1] = hs[i].T @ g, g.sum(0)
        if i > 0:
            g = (g @ P[2 * i].T) * masks[i - 1]
    return loss, grads


def c5_ours_grads(rsl, torch, params, x, y):
    """Loss, parameter gradients and the ReLU masks of our fp32 step."""
    P = [rsl.Variable(p, requires_grad=True) for p in params]
    X, Y = rsl.Variable(x), rsl.Variable(y)
    hs = []
    with rsl.capture_on():
        h = X
        n = len(P) // 2
        for i in range(n):
            h = rsl.matmul(h, P[2 * i]) + P[2 * i + 1]
            if i < n - 1:
                h = rsl.clamp(h, 0, DMAX)
                hs.append(h)
        m = rsl.max(h, 1)
        e = rsl.exp(h - m)
        p = e / rsl.sum(e, 1)
    loss = rsl.sum(rsl.sum(-Y * rsl.log(p + 1e-3), 1), 0)
    loss.backward()
    masks = [torch.from_numpy(q.numpy()).cuda() > 0 for q in hs]
    return float(loss.numpy().ravel()[0]), [q.grad.numpy() for q in P], masks


def test_c5_full_width_step_vs_float64(rsl, cuda):
    """BASELINE C5 at its real width and batch against float64 with the same
    ReLU masks: the loss within 1e-5, every gradient within 2e-4.

    The gradient bar is twice the single-GEMM bar for K >= 4096 because each
    gradient is the end of a chain of five K >= 4096 GEMMs plus the softmax:
    the fp16 hi/lo GEMM accumulates in fp32 inside the tensor core's TMEM
    accumulator, whose additions do not round to nearest, so one GEMM lands at
    ~1e-5 of float64 where an FMA GEMM lands near 1e-6, and the last layer's
    weight gradient (logit error through softmax, then a K = 8192 GEMM)
    measures 1.05e-4 here."""
    torch = cuda
    dims = [4096] * 5 + [1000]
    rng = np.random.default_rng(100)
    x = rng.standard_normal((8192, 4096), dtype=np.float32)
    y = np.zeros((8192, 1000), np.float32)
    y[np.arange(8192), rng.integers(0, 1000, 8192)] = 1
    params = _c5_params(dims, 5)
    loss, grads, masks = c5_ours_grads(rsl, torch, params, x, y)
    loss64, grads64 = c5_f64_grads(torch, params, x, y, masks)
    assert abs(loss - loss64) / abs(loss64) <= 1e-5, (loss, loss64)
    errs = [_rel(torch, torch.from_numpy(g).cuda(), g64) for g, g64 in zip(grads, grads64)]
    assert max(errs) <= 2e-4, errs
