from ... import _C
from ..Module import Module


class Linear(Module):
    """y = x @ W + b with W [in, out] ~ randn(0, 1) and b [out] ~ randn(0, 1),
    like the reference's layers/linear.py."""

    def __init__(self, in_features: int, out_features: int, bias: bool = True, device=None, dtype=None) -> None:
        super().__init__()
        kw = {}
        if device is not None:
            kw["device"] = device
        if dtype is not None:
            kw["dtype"] = dtype
        object.__setattr__(self, "requires_bias", bias)
        self.weights = _C.randn(0, 1, [in_features, out_features], requires_grad=True, **kw)
        if bias:
            self.bias = _C.randn(0, 1, [out_features], requires_grad=True, **kw)

    def forward(self, x):
        if not self.requires_bias:
            return _C.matmul(x, self.weights)
        return _C.matmul(x, self.weights) + self.bias


class Flatten(Module):
    def __init__(self, start_dim: int = 1, end_dim: int = -1) -> None:
        super().__init__()
        if start_dim < 0:
            raise ValueError("Start dim must be non-negative")
        object.__setattr__(self, "start_dim", start_dim)
        object.__setattr__(self, "end_dim", end_dim)

    def forward(self, x):
        end = x.ndim + self.end_dim if self.end_dim < 0 else self.end_dim
        if not self.start_dim < end:
            raise ValueError("Start and end dims not valid")
        shape = list(x.shape)
        new = shape[: self.start_dim]
        flat = 1
        for s in shape[self.start_dim : end + 1]:
            flat *= s
        new.append(flat)
        new += shape[end + 1 :]
        return _C.reshape(x, new)
