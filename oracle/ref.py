"""The reference's own CPU core (built from its sources by oracle/Makefile)
behind a numpy API.  TEST ONLY.  Values are lmp::autograd::Variable handles."""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

from .port import DT, NP

HERE = os.path.dirname(os.path.abspath(__file__))
LIB = os.path.join(HERE, "_ref", "liblamp3_ref.so")

_lib = None


def available() -> bool:
    return os.path.exists(LIB)


def lib():
    global _lib
    if _lib is None:
        L = C.CDLL(LIB)
        vp, i, d, P = C.c_void_p, C.c_int, C.c_double, C.POINTER(C.c_int64)
        L.lref_tensor.argtypes = [i, vp, P, i, i]
        L.lref_tensor.restype = vp
        for f in ("lref_free", "lref_backward"):
            getattr(L, f).argtypes = [vp]
        L.lref_ndim.argtypes = [vp]
        L.lref_dtype.argtypes = [vp]
        L.lref_shape.argtypes = [vp, P]
        L.lref_data.argtypes = [vp, vp]
        L.lref_grad.argtypes = [vp, vp]
        L.lref_binary.argtypes = [i, vp, vp]
        L.lref_binary.restype = vp
        L.lref_binary_backward.argtypes = [i, vp, vp, d, d]
        L.lref_binary_backward.restype = vp
        L.lref_unary.argtypes = [i, vp, d, d]
        L.lref_unary.restype = vp
        L.lref_reduce.argtypes = [i, vp, i]
        L.lref_reduce.restype = vp
        L.lref_matmul.argtypes = [vp, vp]
        L.lref_matmul.restype = vp
        L.lref_transpose.argtypes = [vp]
        L.lref_transpose.restype = vp
        L.lref_set_threads.argtypes = [i]
        L.lref_get_threads.restype = i
        _lib = L
    return _lib


class Var:
    """An lmp::autograd::Variable of the reference build."""

    def __init__(self, h):
        self.h = h

    @classmethod
    def of(cls, a: np.ndarray, requires_grad: bool = False) -> "Var":
        a = np.ascontiguousarray(a)
        shp = (C.c_int64 * max(1, a.ndim))(*a.shape)
        return cls(lib().lref_tensor(DT[a.dtype], a.ctypes.data_as(C.c_void_p), shp, a.ndim,
                                     int(requires_grad)))

    @property
    def shape(self):
        nd = lib().lref_ndim(self.h)
        s = (C.c_int64 * max(1, nd))()
        lib().lref_shape(self.h, s)
        return tuple(s[:nd])

    @property
    def dtype(self):
        return NP[lib().lref_dtype(self.h)]

    def numpy(self) -> np.ndarray:
        out = np.empty(self.shape, dtype=self.dtype)
        lib().lref_data(self.h, out.ctypes.data_as(C.c_void_p))
        return out

    def grad(self) -> np.ndarray:
        out = np.empty(self.shape, dtype=self.dtype)
        lib().lref_grad(self.h, out.ctypes.data_as(C.c_void_p))
        return out

    def backward(self):
        lib().lref_backward(self.h)

    def __del__(self):
        if self.h and _lib is not None:
            _lib.lref_free(self.h)
            self.h = None


def binary(op, a: Var, b: Var) -> Var:
    return Var(lib().lref_binary(op, a.h, b.h))


def binary_backward(op, x: Var, g: Var, p0=0.0, p1=0.0) -> Var:
    return Var(lib().lref_binary_backward(op, x.h, g.h, p0, p1))


def unary(op, a: Var, p0=0.0, p1=0.0) -> Var:
    return Var(lib().lref_unary(op, a.h, p0, p1))


def reduce(op, a: Var, axis: int) -> Var:
    return Var(lib().lref_reduce(op, a.h, axis))


def matmul(a: Var, b: Var) -> Var:
    return Var(lib().lref_matmul(a.h, b.h))


def transpose(a: Var) -> Var:
    return Var(lib().lref_transpose(a.h))


def host_cores() -> int:
    """Cores this process may run on (its CPU affinity), whatever
    OMP_NUM_THREADS a launcher exported."""
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:  # pragma: no cover - non-Linux
        return os.cpu_count() or 1


def set_threads(n: int | None = None) -> int:
    """Sets the reference build's OpenMP thread count (default: every core of
    the affinity mask) and returns the count now in effect."""
    n = n or host_cores()
    lib().lref_set_threads(int(n))
    return int(lib().lref_get_threads())
