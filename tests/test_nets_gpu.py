"""The README's training loop, verbatim through rushlite_b200.nets
(README.md:102-125 of the reference): layers.Sequential of Linear, ReLU,
Linear, Softmax(dim=-1), the forward under @rsl.capture(), the cross-entropy
loss, backward, and the update rebound through model.params[name].  The
weights are injected (Linear draws unseeded randn) and the same steps run
on the reference's own CPU build: losses and parameters agree within 1e-5."""
from __future__ import annotations

import numpy as np
import pytest

from oracle import ref
from tests.test_mlp_gpu import _ref_step
from tests.util import rel_err

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not ref.available(), reason="reference CPU build absent")]


def test_readme_mlp_through_nets(cuda):
    import rushlite_b200 as rsl
    from rushlite_b200.nets import layers

    model = layers.Sequential([
        layers.Linear(256, 64),
        layers.ReLU(),
        layers.Linear(64, 10),
        layers.Softmax(dim=-1),
    ])

    @rsl.capture()
    def forward(x):
        return model(x)

    names = [n for n, _ in model.named_parameters()]
    assert names == ["0.weights", "0.bias", "2.weights", "2.bias"]
    rng = np.random.default_rng(4)
    init = []
    for i, o in ((256, 64), (64, 10)):
        init += [(rng.standard_normal((i, o)) / np.sqrt(i)).astype(np.float32),
                 (rng.standard_normal((o,)) / np.sqrt(i)).astype(np.float32)]
    for name, w in zip(names, init):
        model.params[name] = rsl.Variable(w, requires_grad=True)
    drng = np.random.default_rng(9)
    xs = drng.random((32, 256), dtype=np.float32)
    ys = drng.random((32, 10), dtype=np.float32)
    x, y = rsl.Variable(xs), rsl.Variable(ys)
    pr = init
    for step in range(5):
        probs = forward(x)
        loss = (-y * rsl.log(probs + 1e-3)).sum(1).sum(0)
        loss.backward()
        for name, p in model.named_parameters():
            model.params[name] = rsl.Variable(p.data - 1e-3 * p.grad, requires_grad=True)
        pr, lref = _ref_step(pr, xs, ys, 1e-3)
        lo = loss.tolist()[0]
        assert abs(lo - lref) <= 1e-5 * abs(lref), (step, lo, lref)
    for (name, p), want in zip(model.named_parameters(), pr):
        assert rel_err(p.numpy(), want) <= 1e-5, name
