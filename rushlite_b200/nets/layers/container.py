from typing import Any, Sequence

from ..Module import Module


class Sequential(Module):
    def __init__(self, layers: "Sequence[Module]") -> None:
        super().__init__()
        object.__setattr__(self, "layers", list(layers))
        for i, layer in enumerate(self.layers):
            self._params_dict[str(i)] = layer

    def forward(self, *args: Any) -> Any:
        if not self.layers:
            raise ValueError("Must have at least one layer")
        out = self.layers[0](*args)
        for layer in self.layers[1:]:
            out = layer(out)
        return out
