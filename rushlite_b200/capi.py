"""ctypes binding of the lmpb C ABI (include/lmpb.h).

This is the binding a Python caller of the kernel layer uses; the tests call
every kernel through it.  Device buffers are passed as raw addresses, e.g.
``tensor.data_ptr()`` of a CUDA torch tensor; streams as ``cudaStream_t``
integers (0 = legacy default stream).
"""
from __future__ import annotations

import ctypes as C
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "liblmpb.so")

MAX_DIMS = 16

# lmpb_dtype
BOOL, INT16, INT32, INT64, FLOAT32, FLOAT64 = range(6)
# lmpb_binary_op
ADD, SUB, MUL, DIV, POW, EQ, NE, GE, LE, GT, LT, ABS_BACKWARD, CLAMP_BACKWARD = range(13)
BINARY_OPS = {"add": ADD, "sub": SUB, "mul": MUL, "div": DIV, "pow": POW, "eq": EQ, "ne": NE,
              "ge": GE, "le": LE, "gt": GT, "lt": LT}
# lmpb_unary_op
NEG, EXP, LOG, SQRT, ABS, SIN, COS, TAN, CLAMP = range(9)
UNARY_OPS = {"neg": NEG, "exp": EXP, "log": LOG, "sqrt": SQRT, "abs": ABS, "sin": SIN,
             "cos": COS, "tan": TAN, "clamp": CLAMP}
# lmpb_reduce_op
SUM, MAX, MIN, PROD = range(4)
REDUCE_OPS = {"sum": SUM, "max": MAX, "min": MIN, "prod": PROD}
# lmpb_copy_kind
H2D, D2H, D2D, H2H = range(4)
# fused program
FN_LEAF, FN_CONST, FN_BINARY, FN_UNARY = range(4)
OUT_STORE, OUT_ACCUM, OUT_REDUCE_SUM, OUT_REDUCE_SUM_ACCUM = range(4)

STATUS = {0: "OK", 1: "INVALID", 2: "CUDA", 3: "UNSUPPORTED", 4: "COMPILE", 5: "TIMEOUT"}

# every symbol include/lmpb.h declares
EXPORTS = [
    "lmpb_last_error", "lmpb_version", "lmpb_kernel_launches", "lmpb_broadcast_shape", "lmpb_binary", "lmpb_unary",
    "lmpb_reduce", "lmpb_matmul", "lmpb_gemm_f32", "lmpb_transpose", "lmpb_malloc", "lmpb_free",
    "lmpb_fill", "lmpb_copy", "lmpb_add_inplace", "lmpb_fused_build", "lmpb_fused_launch",
    "lmpb_fused_release", "lmpb_fused_source", "lmpb_device_error", "lmpb_reduce_noalloc",
    "lmpb_gemm_f32_bias_act", "lmpb_comm_unique_id", "lmpb_comm_init", "lmpb_comm_destroy", "lmpb_comm_size",
    "lmpb_allreduce", "lmpb_comm_join", "lmpb_peer_export", "lmpb_peer_import", "lmpb_peer_close",
    "lmpb_peer_size", "lmpb_reduce_allreduce", "lmpb_gemm_sched_tile", "lmpb_gemm_sched_unit", "lmpb_gemm_sched_splits",
]
COMM_ID_BYTES = 128


class LmpbError(RuntimeError):
    def __init__(self, status: int, msg: str):
        super().__init__(f"lmpb {STATUS.get(status, status)}: {msg}")
        self.status = status


class FNode(C.Structure):
    _fields_ = [("kind", C.c_int32), ("sub", C.c_int32), ("dtype", C.c_int32), ("a", C.c_int32),
                ("b", C.c_int32), ("p0", C.c_double), ("p1", C.c_double)]


class FLeaf(C.Structure):
    _fields_ = [("dtype", C.c_int32), ("ndim", C.c_int32), ("shape", C.c_int64 * MAX_DIMS)]


class FOut(C.Structure):
    _fields_ = [("node", C.c_int32), ("mode", C.c_int32), ("dtype", C.c_int32), ("addend", C.c_int32),
                ("ndim", C.c_int32), ("reserved", C.c_int32), ("shape", C.c_int64 * MAX_DIMS)]


_lib = None


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"{LIB_PATH} is missing: run __graft_entry__.build() first")
        L = C.CDLL(LIB_PATH)
        vp, i64, i32, d, P64 = C.c_void_p, C.c_int64, C.c_int, C.c_double, C.POINTER(C.c_int64)
        L.lmpb_last_error.restype = C.c_char_p
        L.lmpb_version.restype = C.c_char_p
        L.lmpb_kernel_launches.restype = C.c_uint64
        L.lmpb_broadcast_shape.argtypes = [P64, i32, P64, i32, P64, C.POINTER(C.c_int)]
        L.lmpb_binary.argtypes = [i32, i32, vp, i32, P64, i32, vp, i32, P64, i32, vp, d, d, vp]
        L.lmpb_unary.argtypes = [i32, i32, vp, vp, i64, d, d, vp]
        L.lmpb_reduce.argtypes = [i32, i32, vp, P64, i32, i32, vp, vp]
        L.lmpb_reduce_noalloc.argtypes = [i32, i32, vp, P64, i32, i32, vp, vp]
        L.lmpb_matmul.argtypes = [i32, vp, i32, vp, i32, vp, i64, i64, i64, vp]
        L.lmpb_gemm_f32.argtypes = [i32, i32, vp, vp, vp, i64, i64, i64, C.c_float, vp]
        L.lmpb_gemm_f32_bias_act.argtypes = [i32, i32, vp, vp, vp, i64, i64, i64, vp, i32, d, d, vp]
        L.lmpb_transpose.argtypes = [i32, vp, vp, i64, i64, vp]
        L.lmpb_device_error.argtypes = []
        L.lmpb_malloc.argtypes = [C.POINTER(vp), C.c_size_t, vp]
        L.lmpb_free.argtypes = [vp, vp]
        L.lmpb_fill.argtypes = [i32, vp, i64, d, vp]
        L.lmpb_copy.argtypes = [i32, vp, i32, vp, i32, i64, vp]
        L.lmpb_add_inplace.argtypes = [i32, vp, vp, i64, vp]
        L.lmpb_fused_build.argtypes = [C.POINTER(FNode), i32, C.POINTER(FLeaf), i32, C.POINTER(FOut),
                                       i32, P64, i32, C.POINTER(vp)]
        L.lmpb_fused_launch.argtypes = [vp, C.POINTER(vp), C.POINTER(vp), vp]
        L.lmpb_fused_release.argtypes = [vp]
        L.lmpb_fused_source.argtypes = [vp]
        L.lmpb_fused_source.restype = C.c_char_p
        L.lmpb_comm_unique_id.argtypes = [vp, C.c_size_t]
        L.lmpb_comm_init.argtypes = [vp, i32, i32]
        L.lmpb_comm_destroy.argtypes = []
        L.lmpb_comm_size.argtypes = []
        L.lmpb_allreduce.argtypes = [i32, C.POINTER(vp), P64, i32, i32, i32, vp]
        L.lmpb_comm_join.argtypes = [vp]
        L.lmpb_peer_export.argtypes = [vp, C.c_size_t]
        L.lmpb_peer_import.argtypes = [vp, i32, i32]
        L.lmpb_peer_close.argtypes = []
        L.lmpb_peer_size.argtypes = []
        L.lmpb_reduce_allreduce.argtypes = [i32, i32, vp, P64, i32, i32, vp, vp]
        PI = C.POINTER(C.c_int)
        L.lmpb_gemm_sched_tile.argtypes = [i32, i32, i32, i32, i32, PI, PI]
        L.lmpb_gemm_sched_tile.restype = None
        L.lmpb_gemm_sched_unit.argtypes = [i32, i32, i32, PI, PI, PI]
        L.lmpb_gemm_sched_unit.restype = None
        L.lmpb_gemm_sched_splits.argtypes = [i64, i32, i32, i32]
        for name in EXPORTS:
            if name in ("lmpb_gemm_sched_tile", "lmpb_gemm_sched_unit"):
                continue
            if name not in ("lmpb_last_error", "lmpb_version", "lmpb_kernel_launches", "lmpb_fused_source"):
                getattr(L, name).restype = C.c_int
        _lib = L
    return _lib


def check(status: int) -> None:
    if status != 0:
        raise LmpbError(status, lib().lmpb_last_error().decode())


def shape_arr(shape) -> C.Array:
    shape = list(shape)
    return (C.c_int64 * max(1, len(shape)))(*shape)


def broadcast_shape(a, b) -> list[int]:
    out = (C.c_int64 * MAX_DIMS)()
    nd = C.c_int(0)
    check(lib().lmpb_broadcast_shape(shape_arr(a), len(a), shape_arr(b), len(b), out, C.byref(nd)))
    return list(out[: nd.value])


def binary(op, out_dt, a_ptr, a_dt, a_shape, b_ptr, b_dt, b_shape, out_ptr, p0=0.0, p1=0.0, stream=0):
    check(lib().lmpb_binary(op, out_dt, a_ptr, a_dt, shape_arr(a_shape), len(a_shape), b_ptr, b_dt,
                            shape_arr(b_shape), len(b_shape), out_ptr, p0, p1, stream))


def unary(op, dt, in_ptr, out_ptr, n, p0=0.0, p1=0.0, stream=0):
    check(lib().lmpb_unary(op, dt, in_ptr, out_ptr, n, p0, p1, stream))


def reduce(op, dt, in_ptr, shape, axis, out_ptr, stream=0):
    check(lib().lmpb_reduce(op, dt, in_ptr, shape_arr(shape), len(shape), axis, out_ptr, stream))


def matmul(out_dt, a_ptr, a_dt, b_ptr, b_dt, c_ptr, m, k, n, stream=0):
    check(lib().lmpb_matmul(out_dt, a_ptr, a_dt, b_ptr, b_dt, c_ptr, m, k, n, stream))


def gemm_f32(ta, tb, a_ptr, b_ptr, c_ptr, m, n, k, beta=0.0, stream=0):
    check(lib().lmpb_gemm_f32(ta, tb, a_ptr, b_ptr, c_ptr, m, n, k, beta, stream))


def gemm_f32_bias_act(ta, tb, a_ptr, b_ptr, c_ptr, m, n, k, bias_ptr=None, clamp=0, lo=0.0, hi=0.0, stream=0):
    check(lib().lmpb_gemm_f32_bias_act(ta, tb, a_ptr, b_ptr, c_ptr, m, n, k, bias_ptr, clamp, lo, hi, stream))


def transpose(dt, in_ptr, out_ptr, m, n, stream=0):
    check(lib().lmpb_transpose(dt, in_ptr, out_ptr, m, n, stream))


def fill(dt, ptr, n, value, stream=0):
    check(lib().lmpb_fill(dt, ptr, n, value, stream))


def copy(kind, src, src_dt, dst, dst_dt, n, stream=0):
    check(lib().lmpb_copy(kind, src, src_dt, dst, dst_dt, n, stream))


def add_inplace(dt, dst, src, n, stream=0):
    check(lib().lmpb_add_inplace(dt, dst, src, n, stream))


class Fused:
    """A compiled fused program (lmpb_fused handle)."""

    def __init__(self, nodes, leaves, outs, iter_shape):
        L = lib()
        self.n_leaves, self.n_outs = len(leaves), len(outs)
        na = (FNode * len(nodes))()
        for i, nd in enumerate(nodes):
            kind, sub, dt, a, b, p0, p1 = (list(nd) + [0, 0, 0.0, 0.0])[:7]
            na[i] = FNode(kind, sub, dt, a, b, p0, p1)
        la = (FLeaf * max(1, len(leaves)))()
        for i, (dt, shape) in enumerate(leaves):
            la[i].dtype, la[i].ndim = dt, len(shape)
            for k, s in enumerate(shape):
                la[i].shape[k] = s
        oa = (FOut * len(outs))()
        for j, out in enumerate(outs):
            node, mode, dt, shape = out[:4]
            oa[j].node, oa[j].mode, oa[j].dtype, oa[j].ndim = node, mode, dt, len(shape)
            oa[j].addend = out[4] if len(out) > 4 else -1
            for k, s in enumerate(shape):
                oa[j].shape[k] = s
        h = C.c_void_p()
        check(L.lmpb_fused_build(na, len(nodes), la, len(leaves), oa, len(outs),
                                 shape_arr(iter_shape), len(iter_shape), C.byref(h)))
        self.h = h

    @property
    def source(self) -> str:
        return lib().lmpb_fused_source(self.h).decode()

    def launch(self, leaf_ptrs, out_ptrs, stream=0):
        lp = (C.c_void_p * max(1, len(leaf_ptrs)))(*leaf_ptrs)
        op = (C.c_void_p * max(1, len(out_ptrs)))(*out_ptrs)
        check(lib().lmpb_fused_launch(self.h, lp, op, stream))

    def __del__(self):
        if getattr(self, "h", None) and _lib is not None:
            _lib.lmpb_fused_release(self.h)
            self.h = None


def kernel_launches() -> int:
    return int(lib().lmpb_kernel_launches())


def device_error() -> None:
    """Raises if a bounded device wait expired since the last call."""
    check(lib().lmpb_device_error())


# ------------------------------------------------------------ collectives

def comm_unique_id() -> bytes:
    buf = C.create_string_buffer(COMM_ID_BYTES)
    check(lib().lmpb_comm_unique_id(buf, COMM_ID_BYTES))
    return buf.raw


def comm_init(uid: bytes, nranks: int, rank: int) -> None:
    buf = C.create_string_buffer(uid, COMM_ID_BYTES)
    check(lib().lmpb_comm_init(buf, nranks, rank))


def comm_destroy() -> None:
    check(lib().lmpb_comm_destroy())


def comm_size() -> int:
    return int(lib().lmpb_comm_size())


def allreduce(dtype, ptrs, counts, op=SUM, overlap=False, stream=0) -> None:
    """In-place all-reduce of device buffers in one grouped launch (lmpb_allreduce)."""
    n = len(ptrs)
    pa = (C.c_void_p * max(1, n))(*ptrs)
    ca = (C.c_int64 * max(1, n))(*counts)
    check(lib().lmpb_allreduce(dtype, pa, ca, n, op, int(overlap), stream))


def comm_join(stream=0) -> None:
    check(lib().lmpb_comm_join(stream))


# ------------------------------------------------- peer-memory collectives

PEER_HANDLE_BYTES = 64


def peer_export() -> bytes:
    buf = C.create_string_buffer(PEER_HANDLE_BYTES)
    check(lib().lmpb_peer_export(buf, PEER_HANDLE_BYTES))
    return buf.raw


def peer_import(handles: list[bytes], rank: int) -> None:
    blob = b"".join(handles)
    buf = C.create_string_buffer(blob, len(blob))
    check(lib().lmpb_peer_import(buf, len(handles), rank))


def peer_close() -> None:
    check(lib().lmpb_peer_close())


def peer_size() -> int:
    return int(lib().lmpb_peer_size())


def reduce_allreduce(op, dt, in_ptr, shape, axis, out_ptr, stream=0) -> int:
    """lmpb_reduce_allreduce; returns the status (UNSUPPORTED lets the caller fall back)."""
    st = lib().lmpb_reduce_allreduce(op, dt, in_ptr, shape_arr(shape), len(shape), axis, out_ptr, stream)
    if st not in (0, 3):
        check(st)
    return st
