"""The reference's own CPU core (built from its sources by oracle/Makefile)
behind a numpy API.  TEST ONLY.  Values are lmp::autograd::Variable handles."""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

from .port import DT, NP

HERE = os.path.dirname(os.path.abspath(__file__))
LIB = os.path.join(HERE, "_ref", "liblamp3_ref.so")
# The same harness linked with the reference's core built with its CUDA
# device served by lmpb (rushlite_b200/lamp3_cuda): the reference's own
# front-end (lmp::tensor::Tensor, lmp::autograd::Variable) on this backend.
CUDA_LIB = os.path.join(HERE, "_ref", "liblamp3_cuda_harness.so")

_lib = None


def available() -> bool:
    return os.path.exists(LIB)


def _bind(L):
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
    L.lref_set_device.argtypes = [i]
    L.lref_device.argtypes = [vp]
    L.lref_set_capture.argtypes = [i]
    return L


def cuda_front():
    """ctypes handle of the reference front-end on lmpb's CUDA device, with
    lref_set_device(1) already applied.  Raises if it was not built."""
    L = _bind(C.CDLL(CUDA_LIB))
    L.lref_set_device(1)
    return L


def lib():
    global _lib
    if _lib is None:
        L = _bind(C.CDLL(LIB))
        _lib = L
    return _lib


class Var:
    """An lmp::autograd::Variable of a reference build (the CPU build by
    default; `L` selects another harness library, e.g. cuda_front())."""

    def __init__(self, h, L=None):
        self.h = h
        self.L = L or lib()

    @classmethod
    def of(cls, a: np.ndarray, requires_grad: bool = False, L=None) -> "Var":
        L = L or lib()
        a = np.ascontiguousarray(a)
        shp = (C.c_int64 * max(1, a.ndim))(*a.shape)
        return cls(L.lref_tensor(DT[a.dtype], a.ctypes.data_as(C.c_void_p), shp, a.ndim, int(requires_grad)), L)

    @property
    def shape(self):
        nd = self.L.lref_ndim(self.h)
        s = (C.c_int64 * max(1, nd))()
        self.L.lref_shape(self.h, s)
        return tuple(s[:nd])

    @property
    def dtype(self):
        return NP[self.L.lref_dtype(self.h)]

    @property
    def device(self) -> str:
        return "cuda" if self.L.lref_device(self.h) == 1 else "cpu"

    def numpy(self) -> np.ndarray:
        out = np.empty(self.shape, dtype=self.dtype)
        self.L.lref_data(self.h, out.ctypes.data_as(C.c_void_p))
        return out

    def grad(self) -> np.ndarray:
        out = np.empty(self.shape, dtype=self.dtype)
        self.L.lref_grad(self.h, out.ctypes.data_as(C.c_void_p))
        return out

    def backward(self):
        self.L.lref_backward(self.h)

    def __del__(self):
        if self.h:
            self.L.lref_free(self.h)
            self.h = None


def binary(op, a: Var, b: Var) -> Var:
    return Var(a.L.lref_binary(op, a.h, b.h), a.L)


def binary_backward(op, x: Var, g: Var, p0=0.0, p1=0.0) -> Var:
    return Var(x.L.lref_binary_backward(op, x.h, g.h, p0, p1), x.L)


def unary(op, a: Var, p0=0.0, p1=0.0) -> Var:
    return Var(a.L.lref_unary(op, a.h, p0, p1), a.L)


def reduce(op, a: Var, axis: int) -> Var:
    return Var(a.L.lref_reduce(op, a.h, axis), a.L)


def matmul(a: Var, b: Var) -> Var:
    return Var(a.L.lref_matmul(a.h, b.h), a.L)


def transpose(a: Var) -> Var:
    return Var(a.L.lref_transpose(a.h), a.L)


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
