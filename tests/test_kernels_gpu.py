"""Parity of every lmpb kernel, called through the C ABI, against the CPU
restatement (oracle/) on the same seeded inputs.  Bit-exact for integer,
comparison, clamp, indexing/broadcast and IEEE-rounded + - * / sqrt; the
reference parity metric max|d|/max|ref| <= 1e-5 for float transcendentals,
float reductions and matmul (<= 1e-4 at K >= 4096)."""
from __future__ import annotations

import numpy as np
import pytest

from oracle import port
from rushlite_b200 import capi
from tests.util import NP_DTYPES, assert_bitexact, rand, rel_err

pytestmark = pytest.mark.gpu

TORCH_DT = None


def dev(torch, a: np.ndarray):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def host(t) -> np.ndarray:
    import torch

    torch.cuda.synchronize()
    return t.cpu().numpy()


def empty(torch, shape, dtype):
    return dev(torch, np.zeros(shape, dtype=dtype))


EXACT_BIN = {capi.ADD, capi.SUB, capi.MUL, capi.DIV, capi.EQ, capi.NE, capi.GE, capi.LE, capi.GT, capi.LT}

BCAST = [((1000,), (1000,)), ((37, 53), (37, 53)), ((64, 256), (1, 256)), ((64, 256), (64, 1)),
         ((3, 1, 5), (4, 1)), ((2, 3, 4, 5), (3, 1, 5)), ((7, 9), (1,)), ((1,), (5, 3)),
         ((4097,), (4097,)), ((8, 1, 16), (1, 4, 1))]


@pytest.mark.parametrize("op", sorted(capi.BINARY_OPS.values()))
@pytest.mark.parametrize("dt", NP_DTYPES)
def test_binary_all_ops_dtypes(cuda, op, dt):
    rng = np.random.default_rng(op * 10 + NP_DTYPES.index(dt))
    for sa, sb in BCAST:
        lo, hi = (0.5, 3.0) if op in (capi.DIV, capi.POW) else (-4, 4)
        a, b = rand(rng, sa, dt, lo, hi), rand(rng, sb, dt, lo, hi)
        if np.dtype(dt).kind == "i" and op == capi.POW:
            b = rng.integers(0, 4, size=sb).astype(dt)
        if np.dtype(dt).kind == "i" and op == capi.DIV:
            b = rng.integers(1, 5, size=sb).astype(dt)
        want = port.binary(op, a, b)
        out = empty(cuda, want.shape, want.dtype)
        da, db = dev(cuda, a), dev(cuda, b)
        capi.binary(op, capi.FLOAT32 if False else port.DT[want.dtype], da.data_ptr(), port.DT[a.dtype], sa,
                    db.data_ptr(), port.DT[b.dtype], sb, out.data_ptr())
        got = host(out)
        if op in EXACT_BIN or np.dtype(dt).kind != "f":
            assert_bitexact(got, want, f"op{op} {dt} {sa}x{sb}")
        else:
            assert rel_err(got, want) <= 1e-5, (op, dt, sa, sb)


@pytest.mark.parametrize("dts", [(np.int32, np.float32), (np.float32, np.int32), (np.int16, np.float64),
                                 (np.bool_, np.int64), (np.float64, np.float32), (np.int64, np.int16)])
@pytest.mark.parametrize("op", [capi.ADD, capi.MUL, capi.SUB, capi.LT, capi.EQ])
def test_binary_mixed_dtypes(cuda, dts, op):
    rng = np.random.default_rng(11)
    for sa, sb in [((33, 17), (33, 17)), ((33, 17), (1, 17)), ((6, 1), (6, 8))]:
        a, b = rand(rng, sa, dts[0]), rand(rng, sb, dts[1])
        want = port.binary(op, a, b)
        out = empty(cuda, want.shape, want.dtype)
        da, db = dev(cuda, a), dev(cuda, b)
        capi.binary(op, port.DT[want.dtype], da.data_ptr(), port.DT[a.dtype], sa, db.data_ptr(),
                    port.DT[b.dtype], sb, out.data_ptr())
        assert_bitexact(host(out), want, f"{dts} op{op}")


@pytest.mark.parametrize("op", [capi.ABS_BACKWARD, capi.CLAMP_BACKWARD])
@pytest.mark.parametrize("dt", [np.float32, np.float64, np.int32])
def test_backward_kernels(cuda, op, dt):
    rng = np.random.default_rng(5)
    x = rand(rng, (1001,), dt, -3, 3)
    x[:5] = [-1, 0, 1, 2, -2]
    g = rand(rng, (1001,), dt, -3, 3)
    want = port.binary(op, x, g, p0=-1.0, p1=2.0)
    out = empty(cuda, want.shape, want.dtype)
    dx, dg = dev(cuda, x), dev(cuda, g)
    capi.binary(op, port.DT[want.dtype], dx.data_ptr(), port.DT[x.dtype], x.shape, dg.data_ptr(),
                port.DT[g.dtype], g.shape, out.data_ptr(), -1.0, 2.0)
    assert_bitexact(host(out), want)


@pytest.mark.parametrize("op", sorted(capi.UNARY_OPS.values()))
@pytest.mark.parametrize("dt", [np.int16, np.int32, np.int64, np.float32, np.float64])
def test_unary_all_ops(cuda, op, dt):
    rng = np.random.default_rng(op)
    lo, hi = (0.1, 5.0) if op in (capi.LOG, capi.SQRT) else (-1.2, 1.2) if op == capi.TAN else (-4, 4)
    if np.dtype(dt).kind == "i" and op in (capi.LOG, capi.SQRT):
        lo, hi = 1, 50
    for n in (1, 3, 4097, 100003):
        a = rand(rng, (n,), dt, lo, hi)
        want = port.unary(op, a, -1.5, 2.5)
        da = dev(cuda, a)
        out = empty(cuda, a.shape, a.dtype)
        capi.unary(op, port.DT[a.dtype], da.data_ptr(), out.data_ptr(), n, -1.5, 2.5)
        got = host(out)
        if np.dtype(dt).kind == "f" and op not in (capi.NEG, capi.ABS, capi.CLAMP, capi.SQRT):
            assert rel_err(got, want) <= 1e-5, (op, dt, n)
        else:
            assert_bitexact(got, want, f"unary{op} {dt} n={n}")


RED_CASES = [((33, 17), 0), ((33, 17), 1), ((4, 5, 6), 1), ((9,), 0), ((1, 4096), 1), ((5000, 3), 0),
             ((3, 20000), 1), ((2, 3000, 8), 1), ((1024, 1024), 0), ((100, 1030), 1), ((17, 1, 5), 1)]


@pytest.mark.parametrize("op", [capi.SUM, capi.MAX, capi.MIN, capi.PROD])
@pytest.mark.parametrize("dt", [np.int16, np.int32, np.int64, np.float32, np.float64])
def test_reduce(cuda, op, dt):
    rng = np.random.default_rng(op * 7 + 1)
    for shape, axis in RED_CASES:
        if op == capi.PROD:
            a = rng.integers(1, 3, size=shape).astype(dt) if np.dtype(dt).kind == "i" else \
                rng.uniform(0.999, 1.001, size=shape).astype(dt)
        else:
            a = rand(rng, shape, dt, -1000, 1000)
        want = port.reduce(op, a, axis)
        da = dev(cuda, a)
        out = empty(cuda, want.shape, dt)
        capi.reduce(op, port.DT[a.dtype], da.data_ptr(), shape, axis, out.data_ptr())
        got = host(out)
        if np.dtype(dt).kind == "f" and op == capi.SUM:
            assert rel_err(got, want) <= 1e-5, (op, dt, shape, axis)
        elif np.dtype(dt).kind == "f" and op == capi.PROD:
            # a long fp32 product random-walks by ~sqrt(n) ulp in ANY order; the
            # sequential oracle carries that error too, so both are held to the
            # fp64 product instead
            exact = np.prod(a.astype(np.float64), axis=axis, keepdims=True)
            # n roundings of relative size <= 2^-24 each: a random walk of
            # ~sqrt(n) ulp; 4 sqrt(n) ulp bounds it (>= 1e-5 only past n ~ 1700)
            n = a.shape[axis]
            tol = max(1e-5, 4 * np.sqrt(n) * 2.0 ** -24) if dt == np.float32 else 1e-12
            assert rel_err(got, exact) <= tol and rel_err(want, exact) <= tol, (dt, shape, axis)
        else:
            assert_bitexact(got, want, f"reduce{op} {dt} {shape} ax{axis}")


@pytest.mark.parametrize("axis", [0, 1])
def test_reduce_c3_full_size(cuda, axis):
    """fp32 N(0,1) and int32 U{-1000..1000} [16384, 4096]."""
    rng = np.random.default_rng(3)
    x = rng.standard_normal((16384, 4096), dtype=np.float32)
    xi = rng.integers(-1000, 1001, size=(16384, 4096)).astype(np.int32)
    dx, dxi = dev(cuda, x), dev(cuda, xi)
    for op in (capi.SUM, capi.MAX, capi.MIN):
        want = port.reduce(op, x, axis)
        out = empty(cuda, want.shape, np.float32)
        capi.reduce(op, capi.FLOAT32, dx.data_ptr(), x.shape, axis, out.data_ptr())
        if op == capi.SUM:
            assert rel_err(host(out), want) <= 1e-5
        else:
            assert_bitexact(host(out), want)
    want = port.reduce(capi.SUM, xi, axis)
    out = empty(cuda, want.shape, np.int32)
    capi.reduce(capi.SUM, capi.INT32, dxi.data_ptr(), xi.shape, axis, out.data_ptr())
    assert_bitexact(host(out), want)
    # deterministic run to run
    out2 = empty(cuda, want.shape, np.float32)
    out3 = empty(cuda, want.shape, np.float32)
    capi.reduce(capi.SUM, capi.FLOAT32, dx.data_ptr(), x.shape, axis, out2.data_ptr())
    capi.reduce(capi.SUM, capi.FLOAT32, dx.data_ptr(), x.shape, axis, out3.data_ptr())
    assert_bitexact(host(out2), host(out3))


@pytest.mark.parametrize("dts", [(np.int32, np.int32), (np.int32, np.float32), (np.float64, np.float64),
                                 (np.int16, np.int64), (np.float32, np.float64)])
def test_matmul_simt_dtypes(cuda, dts):
    rng = np.random.default_rng(9)
    for m, k, n in [(13, 9, 11), (32, 256, 64), (1, 1, 1), (70, 33, 5)]:
        a, b = rand(rng, (m, k), dts[0], -3, 3), rand(rng, (k, n), dts[1], -3, 3)
        want = port.matmul(a, b)
        out = empty(cuda, want.shape, want.dtype)
        da, db = dev(cuda, a), dev(cuda, b)
        capi.matmul(port.DT[want.dtype], da.data_ptr(), port.DT[a.dtype], db.data_ptr(),
                    port.DT[b.dtype], out.data_ptr(), m, k, n)
        got = host(out)
        if want.dtype.kind == "f":
            assert rel_err(got, want) <= 1e-12 if want.dtype == np.float64 else 1e-6
        else:
            assert_bitexact(got, want)


@pytest.mark.parametrize("mkn", [(32, 256, 64), (32, 64, 10), (128, 128, 128), (257, 129, 383),
                                 (1024, 1024, 1024)])
@pytest.mark.parametrize("trans", [(0, 0), (1, 0), (0, 1)])
def test_gemm_f32(cuda, mkn, trans):
    m, k, n = mkn
    rng = np.random.default_rng(m + k + n)
    A = (rng.standard_normal((k, m) if trans[0] else (m, k)) / np.sqrt(k)).astype(np.float32)
    B = rng.standard_normal((n, k) if trans[1] else (k, n)).astype(np.float32)
    Am = A.T if trans[0] else A
    Bm = B.T if trans[1] else B
    want = Am.astype(np.float64) @ Bm.astype(np.float64)
    C0 = rng.standard_normal((m, n)).astype(np.float32)
    dA, dB, dC = dev(cuda, A), dev(cuda, B), dev(cuda, C0)
    capi.gemm_f32(trans[0], trans[1], dA.data_ptr(), dB.data_ptr(), dC.data_ptr(), m, n, k, 1.0)
    assert rel_err(host(dC), want + C0) <= 1e-5
    capi.gemm_f32(trans[0], trans[1], dA.data_ptr(), dB.data_ptr(), dC.data_ptr(), m, n, k, 0.0)
    assert rel_err(host(dC), want) <= 1e-5


@pytest.mark.parametrize("trans", [(0, 0), (1, 0), (0, 1), (1, 1)])
def test_gemm_f32_wide_range(cuda, trans):
    """Rows of A and columns of B spread over 2^-100 .. 2^50 (the tensor-core
    path scales every row into fp16 range): each element within 1e-5 of
    |A|·|B|, underflowing products to fp32's subnormal resolution."""
    m, k, n = 256, 200, 384  # k pads to the k-block
    rng = np.random.default_rng(7)
    Am = rng.standard_normal((m, k)) * np.exp2(rng.integers(-100, 50, (m, 1)))
    Bm = rng.standard_normal((k, n)) * np.exp2(rng.integers(-60, 60, (1, n)))
    Am, Bm = Am.astype(np.float32), Bm.astype(np.float32)
    A = np.ascontiguousarray(Am.T) if trans[0] else Am
    B = np.ascontiguousarray(Bm.T) if trans[1] else Bm
    want = Am.astype(np.float64) @ Bm.astype(np.float64)
    bound = np.abs(Am.astype(np.float64)) @ np.abs(Bm.astype(np.float64))
    dA, dB, dC = dev(cuda, A), dev(cuda, B), dev(cuda, np.zeros((m, n), np.float32))
    capi.gemm_f32(trans[0], trans[1], dA.data_ptr(), dB.data_ptr(), dC.data_ptr(), m, n, k, 0.0)
    capi.device_error()
    err = np.abs(host(dC).astype(np.float64) - want)
    assert np.all(err <= 1e-5 * bound + 3e-45), float(np.max(err / (bound + 1e-300)))


def test_gemm_f32_nonfinite(cuda):
    """Inf and NaN in A propagate as in an fp32 dot product; the other
    elements of those rows keep full accuracy (B is integer-valued, so its
    low parts are exactly zero)."""
    m, k, n = 256, 256, 256
    rng = np.random.default_rng(8)
    A = rng.standard_normal((m, k)).astype(np.float32)
    A[3, 5] = np.inf
    A[9, 0] = -np.inf
    A[9, 1] = np.inf  # inf - inf = NaN wherever both B entries are non-zero
    A[17, 100] = np.nan
    A[40, :] = 0.0
    B = rng.integers(1, 9, (k, n)).astype(np.float32)
    B[5, 7] = 0.0  # inf * 0 = NaN in row 3, column 7
    with np.errstate(invalid="ignore"):
        want = A.astype(np.float64) @ B.astype(np.float64)
    dA, dB, dC = dev(cuda, A), dev(cuda, B), dev(cuda, np.zeros((m, n), np.float32))
    capi.gemm_f32(0, 0, dA.data_ptr(), dB.data_ptr(), dC.data_ptr(), m, n, k, 0.0)
    got = host(dC).astype(np.float64)
    np.testing.assert_array_equal(np.isnan(got), np.isnan(want))
    np.testing.assert_array_equal(np.isposinf(got), np.isposinf(want))
    np.testing.assert_array_equal(np.isneginf(got), np.isneginf(want))
    fin = np.isfinite(want)
    assert rel_err(got[fin], want[fin]) <= 1e-5


def test_memory_ops(cuda):
    rng = np.random.default_rng(1)
    for dt in NP_DTYPES:
        for n in (1, 7, 4099):
            buf = empty(cuda, (n,), dt)
            capi.fill(port.DT[np.dtype(dt)], buf.data_ptr(), n, 3.0)
            assert_bitexact(host(buf), np.full((n,), 3.0).astype(dt))
            x, y = rand(rng, (n,), dt), rand(rng, (n,), dt)
            dx, dy = dev(cuda, x), dev(cuda, y)
            capi.add_inplace(port.DT[np.dtype(dt)], dx.data_ptr(), dy.data_ptr(), n)
            assert_bitexact(host(dx), (x + y).astype(dt) if dt != np.bool_ else (x | y))
    # casting copies
    x = rng.uniform(-100, 100, size=(1000,)).astype(np.float64)
    d = empty(cuda, (1000,), np.int32)
    capi.copy(capi.H2D, x.ctypes.data, capi.FLOAT64, d.data_ptr(), capi.INT32, 1000)
    assert_bitexact(host(d), x.astype(np.int32))
    back = np.zeros(1000, np.float32)
    capi.copy(capi.D2H, d.data_ptr(), capi.INT32, back.ctypes.data, capi.FLOAT32, 1000)
    cuda.cuda.synchronize()
    assert_bitexact(back, x.astype(np.int32).astype(np.float32))
    # transpose
    for dt in (np.float32, np.int64, np.int16):
        a = rand(rng, (67, 131), dt)
        da = dev(cuda, a)
        out = empty(cuda, (131, 67), dt)
        capi.transpose(port.DT[np.dtype(dt)], da.data_ptr(), out.data_ptr(), 67, 131)
        assert_bitexact(host(out), port.transpose(a))


def _c2_inputs(rows, cols, seed=0):
    rng = np.random.default_rng(seed)
    return rng.random((rows, cols), dtype=np.float32), rng.random((rows, 1), dtype=np.float32)


def _c2_oracle(a, b):
    one = np.ones((1,), np.float32)
    s = port.binary(capi.MUL, a, a)
    c = port.binary(capi.ADD, s, b)
    x = port.unary(capi.EXP, c)
    e = port.binary(capi.MUL, x, a)
    lg = port.unary(capi.LOG, port.binary(capi.ADD, b, one))
    return port.binary(capi.SUB, e, lg), x


F32 = capi.FLOAT32
CHAIN = [(capi.FN_LEAF, 0, F32, 0), (capi.FN_LEAF, 0, F32, 1), (capi.FN_BINARY, capi.MUL, F32, 0, 0),
         (capi.FN_BINARY, capi.ADD, F32, 2, 1), (capi.FN_UNARY, capi.EXP, F32, 3),
         (capi.FN_BINARY, capi.MUL, F32, 4, 0), (capi.FN_CONST, 0, F32, 0, 0, 1.0),
         (capi.FN_BINARY, capi.ADD, F32, 1, 6), (capi.FN_UNARY, capi.LOG, F32, 7),
         (capi.FN_BINARY, capi.SUB, F32, 5, 8)]


@pytest.mark.parametrize("shape", [(64, 128), (8192, 8192), (33, 7), (5, 4100)])
def test_fused_chain_forward(cuda, shape):
    a, b = _c2_inputs(*shape)
    want, _ = _c2_oracle(a, b)
    f = capi.Fused(CHAIN, [(F32, a.shape), (F32, b.shape)], [(9, capi.OUT_STORE, F32, a.shape)], a.shape)
    da, db = dev(cuda, a), dev(cuda, b)
    out = empty(cuda, a.shape, np.float32)
    f.launch([da.data_ptr(), db.data_ptr()], [out.data_ptr()])
    got = host(out)
    assert rel_err(got, want) <= 1e-5
    # everything but exp/log rounds like the op-by-op path: compare the parts
    # that do not involve a transcendental bit-exactly
    g = capi.Fused(CHAIN[:4], [(F32, a.shape), (F32, b.shape)], [(3, capi.OUT_STORE, F32, a.shape)], a.shape)
    g.launch([da.data_ptr(), db.data_ptr()], [out.data_ptr()])
    assert_bitexact(host(out), port.binary(capi.ADD, port.binary(capi.MUL, a, a), b))


@pytest.mark.parametrize("shape", [(64, 128), (8192, 8192), (300, 1000)])
def test_fused_row_reduce_accumulate(cuda, shape):
    """grad_a += exp(c)-chain and grad_b += rowsum(exp(c)) in one pass."""
    a, b = _c2_inputs(*shape, seed=4)
    d, x = _c2_oracle(a, b)
    rng = np.random.default_rng(8)
    ga0 = rng.random(a.shape, dtype=np.float32)
    gb0 = rng.random(b.shape, dtype=np.float32)
    f = capi.Fused(CHAIN, [(F32, a.shape), (F32, b.shape)],
                   [(9, capi.OUT_ACCUM, F32, a.shape), (4, capi.OUT_REDUCE_SUM_ACCUM, F32, b.shape)], a.shape)
    da, db, dga, dgb = dev(cuda, a), dev(cuda, b), dev(cuda, ga0), dev(cuda, gb0)
    f.launch([da.data_ptr(), db.data_ptr()], [dga.data_ptr(), dgb.data_ptr()])
    assert rel_err(host(dga), port.binary(capi.ADD, ga0, d)) <= 1e-5
    want_b = gb0.astype(np.float64) + x.astype(np.float64).sum(1, keepdims=True)
    assert rel_err(host(dgb), want_b) <= 1e-5


@pytest.mark.parametrize("shape", [(512, 4096), (8192, 1000), (8192, 4096), (3, 5)])
def test_fused_column_reduce(cuda, shape):
    """ReLU backward feeding a bias grad: store g*[x>0] and bias += colsum."""
    rng = np.random.default_rng(12)
    x = rng.standard_normal(shape).astype(np.float32)
    g = rng.standard_normal(shape).astype(np.float32)
    bias0 = rng.standard_normal((shape[1],)).astype(np.float32)
    f = capi.Fused([(capi.FN_LEAF, 0, F32, 0), (capi.FN_LEAF, 0, F32, 1),
                    (capi.FN_BINARY, capi.CLAMP_BACKWARD, F32, 0, 1, 0.0, 1.7976931348623157e308)],
                   [(F32, shape), (F32, shape)],
                   [(2, capi.OUT_STORE, F32, shape), (2, capi.OUT_REDUCE_SUM_ACCUM, F32, (shape[1],))], shape)
    dx, dg, dbias = dev(cuda, x), dev(cuda, g), dev(cuda, bias0)
    out = empty(cuda, shape, np.float32)
    f.launch([dx.data_ptr(), dg.data_ptr()], [out.data_ptr(), dbias.data_ptr()])
    want = port.binary(capi.CLAMP_BACKWARD, x, g, p0=0.0, p1=1.7976931348623157e308)
    assert_bitexact(host(out), want)
    assert rel_err(host(dbias), bias0.astype(np.float64) + want.astype(np.float64).sum(0)) <= 1e-5


@pytest.mark.parametrize("mkn,tol", [((2048, 2048, 2048), 1e-5), ((4096, 4096, 4096), 1e-4),
                                     ((32768, 4096, 512), 1e-4), ((4096, 1024, 4096), 1e-5)])
def test_gemm_f32_c4_sizes(cuda, mkn, tol):
    """BASELINE C4 tolerances: rel <= 1e-5, and <= 1e-4 at K >= 4096, against fp64."""
    torch = cuda
    m, k, n = mkn
    g = torch.Generator(device="cuda").manual_seed(m + k)
    A = torch.randn(m, k, device="cuda", generator=g) / k ** 0.5
    B = torch.randn(k, n, device="cuda", generator=g) / k ** 0.5
    C = torch.empty(m, n, device="cuda")
    capi.gemm_f32(0, 0, A.data_ptr(), B.data_ptr(), C.data_ptr(), m, n, k, 0.0)
    capi.device_error()
    ref = A.double() @ B.double()
    assert ((C.double() - ref).abs().max() / ref.abs().max()).item() <= tol


@pytest.mark.parametrize("mkn,splits", [((4096, 8192, 4096), None), ((4096, 1024, 4096), "2"),
                                        ((8192, 4096, 1000), "3"), ((2048, 4096, 1000), "4"),
                                        ((1024, 4096, 1001), "2")])
def test_gemm_f32_split_k_deterministic(cuda, mkn, splits, monkeypatch):
    """Split K (chosen by the heuristic when splits is None, else forced with
    the tuning override): the last-arriving unit sums the partials in split
    order, so repeated runs are bit-identical, and they match the unsplit
    kernel within the GEMM tolerance, with accumulation into C (beta = 1)."""
    torch = cuda
    m, k, n = mkn
    g = torch.Generator(device="cuda").manual_seed(m + n)
    A = torch.randn(m, k, device="cuda", generator=g) / k ** 0.5
    B = torch.randn(k, n, device="cuda", generator=g)
    C0 = torch.randn(m, n, device="cuda", generator=g)
    outs = []
    for unsplit in (False, False, True):
        if unsplit:
            monkeypatch.setenv("LMPB_GEMM_SPLITK", "1")
        elif splits:
            monkeypatch.setenv("LMPB_GEMM_SPLITK", splits)
        C = C0.clone()
        capi.gemm_f32(0, 0, A.data_ptr(), B.data_ptr(), C.data_ptr(), m, n, k, 1.0)
        capi.device_error()
        outs.append(C)
    assert torch.equal(outs[0], outs[1])
    ref = A.double() @ B.double() + C0.double()
    for C in outs:
        assert ((C.double() - ref).abs().max() / ref.abs().max()).item() <= 1e-5
