"""rushlite_b200.nets bookkeeping without a GPU: parameter registration and
dotted names, the params view (rebinding, KeyError on unknown names),
zero_grad, Softmax's dim check and Flatten's shape rule, on CPU Variables
(constructors and shape ops only; no kernels)."""
from __future__ import annotations

import pytest

import rushlite_b200 as rsl
from rushlite_b200.nets import Module, layers


def _linear(i, o, bias=True):
    return layers.Linear(i, o, bias=bias, device=rsl.device.cpu)


def test_named_parameters_and_params_view():
    model = layers.Sequential([_linear(8, 4), layers.ReLU(), _linear(4, 2, bias=False)])
    names = [n for n, _ in model.named_parameters()]
    assert names == ["0.weights", "0.bias", "2.weights"]
    assert list(model.params) == names and len(model.params) == 3
    w = model.params["0.weights"]
    assert tuple(w.shape) == (8, 4) and w.requires_grad
    new = rsl.Variable([[1.0] * 4] * 8, requires_grad=True, device=rsl.device.cpu)
    model.params["0.weights"] = new
    assert model.params["0.weights"] is new
    assert model.layers[0].weights is new
    with pytest.raises(KeyError):
        model.params["0.nope"] = new
    assert len(list(model.parameters())) == 3


def test_module_attribute_rules():
    class Net(Module):
        def __init__(self):
            super().__init__()
            self.fc = _linear(3, 3)
            self.scale = 2.0

        def forward(self, x):
            return self.fc(x)

    n = Net()
    assert [k for k, _ in n.named_parameters()] == ["fc.weights", "fc.bias"]
    assert n.scale == 2.0
    del n.fc
    assert list(n.named_parameters()) == []
    with pytest.raises(AttributeError):
        n.missing
    with pytest.raises(NotImplementedError):
        Module()(1)


def test_softmax_dim_and_flatten_checks():
    x = rsl.Variable([[1.0, 2.0], [3.0, 4.0]], device=rsl.device.cpu)
    with pytest.raises(ValueError):
        layers.Softmax(dim=2)(x)
    with pytest.raises(ValueError):
        layers.Flatten(start_dim=-1)
    with pytest.raises(ValueError):
        layers.Sequential([])(x)
    y = rsl.Variable([[[1.0, 2.0], [3.0, 4.0]]], device=rsl.device.cpu)  # [1, 2, 2]
    assert list(layers.Flatten()(y).shape) == [1, 4]
