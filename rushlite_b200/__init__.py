"""rushlite_b200 — the rushlite / Lamp3 Python API on a B200-native backend.

Same names as the reference's ``rushlite`` package (src/rushlite/__init__.py):
``Variable``, the op functions, ``capture_on`` / ``capture``, ``no_grad`` and
``nets``.  Every op on a CUDA Variable runs on the sm_100a kernels of
``liblmpb.so``; importing fails loudly if the native module is missing.
"""
from __future__ import annotations

try:
    from ._C import *  # noqa: F401,F403
    from ._C import Variable, cuda, device, dtype  # noqa: F401
except ImportError as e:  # pragma: no cover - surfaced to the user
    raise ImportError(
        "rushlite_b200 native module is not built; run `python -c 'import __graft_entry__ as g; g.build()'` "
        f"({e})") from e

from .capture_mode import capture, capture_on
from .grad_mode import no_grad
from .nets.Module import Module

__all__ = ["Variable", "Module", "capture_on", "capture", "no_grad"]
