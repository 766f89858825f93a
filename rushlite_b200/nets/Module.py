"""Module base class with a functional parameter view, following the
behaviour of the reference's src/rushlite/nets/Module.py: parameters and
submodules live in ``_params_dict``; ``params[path] = Variable(...)`` rebinds
a parameter in place for SGD-style updates."""
from __future__ import annotations

from typing import Any, Iterator

from .._C import Variable


class Module:
    def __init__(self) -> None:
        object.__setattr__(self, "_params_dict", {})

    def forward(self, *args: Any, **kwds: Any) -> Any:
        raise NotImplementedError

    def __setattr__(self, name: str, value: Any) -> None:
        params = self.__dict__.get("_params_dict")
        if isinstance(value, (Module, Variable)):
            if params is None:
                raise AttributeError(f"cannot assign parameter {name!r}: call super().__init__() first")
            params[name] = value
        else:
            if params is not None:
                params.pop(name, None)
            object.__setattr__(self, name, value)

    def __getattr__(self, name: str) -> Any:
        params = self.__dict__.get("_params_dict")
        if params is not None and name in params:
            return params[name]
        raise AttributeError(f"{type(self).__name__!r} object has no attribute {name!r}")

    def __delattr__(self, name: str) -> None:
        params = self.__dict__.get("_params_dict")
        if params is not None and name in params:
            del params[name]
        else:
            object.__delattr__(self, name)

    def __call__(self, *args: Any, **kwds: Any) -> Any:
        return self.forward(*args, **kwds)

    @property
    def params(self) -> "_ParamsView":
        return _ParamsView(self)

    def parameters(self) -> Iterator[Variable]:
        for _, p in self.named_parameters():
            yield p

    def named_parameters(self, _prefix: str = "") -> Iterator[tuple[str, Variable]]:
        for key, val in self._params_dict.items():
            path = f"{_prefix}{key}"
            if isinstance(val, Variable):
                yield path, val
            else:
                yield from val.named_parameters(path + ".")

    def zero_grad(self) -> None:
        for p in self.parameters():
            if p.requires_grad:
                p.zero_grad()


class _ParamsView:
    """Dict-like view keyed by the dotted paths of named_parameters()."""

    def __init__(self, module: Module) -> None:
        self._m = module

    def _owner(self, key: str) -> tuple[Module, str]:
        parts = key.split(".")
        mod = self._m
        for p in parts[:-1]:
            mod = mod._params_dict[p]
        return mod, parts[-1]

    def __getitem__(self, key: str) -> Variable:
        mod, leaf = self._owner(key)
        return mod._params_dict[leaf]

    def __setitem__(self, key: str, value: Variable) -> None:
        mod, leaf = self._owner(key)
        if leaf not in mod._params_dict or not isinstance(mod._params_dict[leaf], Variable):
            raise KeyError(key)
        mod._params_dict[leaf] = value

    def __iter__(self):
        return (k for k, _ in self._m.named_parameters())

    def __len__(self) -> int:
        return sum(1 for _ in self._m.named_parameters())

    def keys(self):
        return list(iter(self))

    def items(self):
        return list(self._m.named_parameters())
