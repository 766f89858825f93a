"""CUDA-graph capture and replay of a training step (rsl.cuda.Graph): the
replayed step must give bit-identical parameters and losses to running the
same step eagerly, step after step."""
from __future__ import annotations

import sys

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
FMAX = sys.float_info.max


@pytest.fixture(scope="module")
def rsl(cuda):
    import rushlite_b200

    return rushlite_b200


def _params(rsl, dims, seed=5):
    rng = np.random.default_rng(seed)
    ps = []
    for i in range(len(dims) - 1):
        w = (rng.standard_normal((dims[i], dims[i + 1])) / np.sqrt(dims[i])).astype(np.float32)
        b = (rng.standard_normal((dims[i + 1],)) / np.sqrt(dims[i])).astype(np.float32)
        ps += [rsl.Variable(w, requires_grad=True), rsl.Variable(b, requires_grad=True)]
    return ps


def _step_inplace(rsl, ps, x, y, lr):
    """README MLP step with the SGD update written into the parameters."""
    with rsl.capture_on():
        h = x
        n = len(ps) // 2
        for i in range(n):
            h = rsl.matmul(h, ps[2 * i]) + ps[2 * i + 1]
            if i < n - 1:
                h = rsl.clamp(h, 0.0, FMAX)
        m = rsl.max(h, 1)
        e = rsl.exp(h - m)
        p = e / rsl.sum(e, 1)
    loss = rsl.sum(rsl.sum(-y * rsl.log(p + 1e-3), 1), 0)
    loss.backward()
    with rsl.no_grad(), rsl.capture_on():
        for q in ps:
            q.data.copy(q.data - lr * q.grad)  # one fused kernel, written in place
            q.zero_grad()
    return loss


@pytest.mark.parametrize("dims,batch", [([256, 64, 10], 32), ([512, 384, 256, 100], 300)])
def test_graph_replay_matches_eager_steps(rsl, dims, batch):
    rng = np.random.default_rng(1)
    xs = rng.random((batch, dims[0]), dtype=np.float32)
    ys = rng.random((batch, dims[-1]), dtype=np.float32)
    runs = []
    for graphed in (False, True):
        x, y = rsl.Variable(xs), rsl.Variable(ys)
        ps = _params(rsl, dims)
        _step_inplace(rsl, ps, x, y, 1e-3)  # builds every fused program
        losses = []
        if graphed:
            g = rsl.cuda.Graph()
            with g:
                loss = _step_inplace(rsl, ps, x, y, 1e-3)
            assert g.kernels > 0
            for _ in range(6):
                g.replay()
                losses.append(float(loss.numpy().ravel()[0]))  # the latest replay's value
        else:
            for _ in range(6):
                losses.append(float(_step_inplace(rsl, ps, x, y, 1e-3).numpy().ravel()[0]))
        runs.append((losses, [q.numpy() for q in ps]))
        if graphed:
            del g
    (l0, p0), (l1, p1) = runs
    assert l0 == l1
    for a, b in zip(p0, p1):
        np.testing.assert_array_equal(a, b)


def test_host_read_inside_capture_fails_cleanly(rsl):
    x = rsl.Variable(np.ones((64, 64), np.float32))
    (x * 2.0).numpy()
    g = rsl.cuda.Graph()
    with pytest.raises(RuntimeError):
        with g:
            (x * 2.0).numpy()  # a synchronising read cannot be recorded
    # the library keeps working on its own stream afterwards
    np.testing.assert_array_equal((x * 3.0).numpy(), np.full((64, 64), 3.0, np.float32))


def test_copy_of_pending_value_writes_in_place(rsl):
    """Tensor.copy of a pending elementwise value realizes it straight into
    the destination (reading the destination's own old values at the same
    index), with the same values as the unfused path."""
    rng = np.random.default_rng(2)
    a0 = rng.standard_normal((300, 257)).astype(np.float32)
    g0 = rng.standard_normal((300, 257)).astype(np.float32)
    r0 = rng.standard_normal((257,)).astype(np.float32)
    got = []
    for captured in (False, True):
        a, g, r = rsl.Variable(a0), rsl.Variable(g0), rsl.Variable(r0)
        with rsl.no_grad(), rsl.capture_on(captured):
            a.data.copy(a.data - 1e-3 * g.data + r.data)  # broadcast of another tensor
            a.data.copy(a.data * a.data + a.data)
        got.append(a.numpy())
    np.testing.assert_array_equal(got[0], got[1])
