import sys

from ... import _C
from ..Module import Module


class ReLU(Module):
    def forward(self, x):
        return _C.clamp(x, 0, sys.float_info.max)


class Sigmoid(Module):
    def forward(self, x):
        return 1 / (1 + _C.exp(-x))


class Tanh(Module):
    def forward(self, x):
        e, ne = _C.exp(x), _C.exp(-x)
        return (e - ne) / (e + ne)


class Softmax(Module):
    def __init__(self, dim: int) -> None:
        super().__init__()
        object.__setattr__(self, "dim", dim)

    def forward(self, x):
        d = x.ndim + self.dim if self.dim < 0 else self.dim
        if not 0 <= d < x.ndim:
            raise ValueError("Dim not in bounds")
        shifted = x - _C.max(x, d)
        e = _C.exp(shifted)
        return e / _C.sum(e, d)
