"""numpy front-end of the plain-C restatement (lamp3_oracle.c).  TEST ONLY."""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB = os.path.join(HERE, "liblamp3_oracle.so")

DT = {np.dtype(np.bool_): 0, np.dtype(np.int16): 1, np.dtype(np.int32): 2,
      np.dtype(np.int64): 3, np.dtype(np.float32): 4, np.dtype(np.float64): 5}
NP = {v: k for k, v in DT.items()}
NAMES = {"bool": 0, "int16": 1, "int32": 2, "int64": 3, "float32": 4, "float64": 5}

_lib = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB):
            raise ImportError(f"{LIB} missing: run `make -C oracle`")
        L = C.CDLL(LIB)
        P, vp, i, d, i64 = C.POINTER(C.c_int64), C.c_void_p, C.c_int, C.c_double, C.c_int64
        L.lo_binary.argtypes = [i, i, vp, i, P, i, vp, i, P, i, vp, d, d]
        L.lo_unary.argtypes = [i, i, vp, vp, i64, d, d]
        L.lo_reduce.argtypes = [i, i, vp, P, i, i, vp]
        L.lo_matmul.argtypes = [i, vp, i, vp, i, vp, i64, i64, i64]
        L.lo_transpose.argtypes = [i, vp, vp, i64, i64]
        _lib = L
    return _lib


def _shape(s):
    s = list(s)
    return (C.c_int64 * max(1, len(s)))(*s)


def _ptr(a: np.ndarray):
    return a.ctypes.data_as(C.c_void_p)


def broadcast_shape(a, b):
    return list(np.broadcast_shapes(tuple(a), tuple(b)))


def binary(op: int, a: np.ndarray, b: np.ndarray, out_dtype=None, p0=0.0, p1=0.0) -> np.ndarray:
    a, b = np.ascontiguousarray(a), np.ascontiguousarray(b)
    odt = NP[max(DT[a.dtype], DT[b.dtype])] if out_dtype is None else np.dtype(out_dtype)
    out = np.empty(broadcast_shape(a.shape, b.shape), dtype=odt)
    r = lib().lo_binary(op, DT[odt], _ptr(a), DT[a.dtype], _shape(a.shape), a.ndim, _ptr(b),
                        DT[b.dtype], _shape(b.shape), b.ndim, _ptr(out), p0, p1)
    assert r == 0
    return out


def unary(op: int, a: np.ndarray, p0=0.0, p1=0.0) -> np.ndarray:
    a = np.ascontiguousarray(a)
    out = np.empty_like(a)
    assert lib().lo_unary(op, DT[a.dtype], _ptr(a), _ptr(out), a.size, p0, p1) == 0
    return out


def reduce(op: int, a: np.ndarray, axis: int) -> np.ndarray:
    a = np.ascontiguousarray(a)
    shp = list(a.shape)
    shp[axis] = 1
    out = np.empty(shp, dtype=a.dtype)
    assert lib().lo_reduce(op, DT[a.dtype], _ptr(a), _shape(a.shape), a.ndim, axis, _ptr(out)) == 0
    return out


def matmul(a: np.ndarray, b: np.ndarray, out_dtype=None) -> np.ndarray:
    a, b = np.ascontiguousarray(a), np.ascontiguousarray(b)
    odt = NP[max(DT[a.dtype], DT[b.dtype])] if out_dtype is None else np.dtype(out_dtype)
    m, k = a.shape
    k2, n = b.shape
    assert k == k2
    out = np.empty((m, n), dtype=odt)
    assert lib().lo_matmul(DT[odt], _ptr(a), DT[a.dtype], _ptr(b), DT[b.dtype], _ptr(out), m, k, n) == 0
    return out


def transpose(a: np.ndarray) -> np.ndarray:
    a = np.ascontiguousarray(a)
    m, n = a.shape
    out = np.empty((n, m), dtype=a.dtype)
    assert lib().lo_transpose(DT[a.dtype], _ptr(a), _ptr(out), m, n) == 0
    return out
