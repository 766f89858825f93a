"""lmpb_reduce_noalloc: the reduction entry point for callers that may not
allocate device memory while it runs (their own memory planner owns all
allocations, or a pool miss must never turn into a cudaMalloc).  It must give
the same results as lmpb_reduce, call after call, while keeping its split
workspace in the library's fixed scratch array.

This file is named so that pytest collects it last."""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

from rushlite_b200 import capi
from tests.util import assert_bitexact, rel_err

pytestmark = pytest.mark.gpu


def _noalloc(op, dt, in_ptr, shape, axis, out_ptr):
    capi.check(capi.lib().lmpb_reduce_noalloc(op, dt, in_ptr, capi.shape_arr(shape), len(shape), axis,
                                              out_ptr, None))


# Narrow leading-axis reductions split their rows over many chunks whose
# partials live in the scratch array ([65536, 256] axis 0: 296 chunks, 0.3 MB;
# [100000, 100] axis 0: 592 chunks).  The C3 column case [16384, 4096] axis 0
# folds its chunks inside a thread-block cluster and needs no scratch at all;
# the last axis never does.
CASES = [((65536, 256), 0, np.float32), ((65536, 256), 0, np.int32), ((100000, 100), 0, np.float32),
         ((16384, 4096), 0, np.float32), ((2048, 1024), 1, np.float32)]


def _pool_used():
    """(current, high-water) bytes in use of the current device's default
    stream-ordered pool, the pool lmpb_reduce takes its workspace from."""
    rt = C.CDLL("libcudart.so.12")
    dev, pool = C.c_int(), C.c_void_p()
    assert rt.cudaGetDevice(C.byref(dev)) == 0
    assert rt.cudaDeviceGetDefaultMemPool(C.byref(pool), dev) == 0
    cur, high = C.c_uint64(), C.c_uint64()
    # cudaMemPoolAttrUsedMemCurrent = 7, cudaMemPoolAttrUsedMemHigh = 8
    assert rt.cudaMemPoolGetAttribute(pool, 7, C.byref(cur)) == 0
    assert rt.cudaMemPoolGetAttribute(pool, 8, C.byref(high)) == 0
    return cur.value, high.value, rt, pool


def _reset_high(rt, pool):
    zero = C.c_uint64(0)  # resets the high-water mark to the current use
    assert rt.cudaMemPoolSetAttribute(pool, 8, C.byref(zero)) == 0


def test_noalloc_allocates_nothing(cuda):
    """The property the entry point exists for: its calls leave the device's
    pool untouched, where lmpb_reduce on the same shape draws its workspace
    from it (the control shows the check can see an allocation)."""
    torch = cuda
    shape = (65536, 256)
    x = torch.randn(shape, device="cuda")
    out = torch.empty((1, 256), device="cuda")
    _noalloc(capi.SUM, capi.FLOAT32, x.data_ptr(), shape, 0, out.data_ptr())  # first call: symbol lookup
    torch.cuda.synchronize()
    cur, _, rt, pool = _pool_used()
    _reset_high(rt, pool)
    for _ in range(2):
        _noalloc(capi.SUM, capi.FLOAT32, x.data_ptr(), shape, 0, out.data_ptr())
    torch.cuda.synchronize()
    cur2, high, _, _ = _pool_used()
    assert high == cur and cur2 == cur, (cur, cur2, high)
    capi.reduce(capi.SUM, capi.FLOAT32, x.data_ptr(), shape, 0, out.data_ptr())
    torch.cuda.synchronize()
    _, high2, _, _ = _pool_used()
    assert high2 > cur, "the control allocation did not show in the pool's high-water mark"


@pytest.mark.parametrize("shape,axis,dt", CASES)
def test_noalloc_matches_lmpb_reduce_twice(cuda, shape, axis, dt):
    torch = cuda
    rng = np.random.default_rng(17)
    dtc = {np.float32: capi.FLOAT32, np.int32: capi.INT32}[dt]
    for call in range(2):  # two calls in a row: the shared scratch keeps the last call's contents
        x = (rng.standard_normal(shape) if dt == np.float32 else rng.integers(-1000, 1001, shape)).astype(dt)
        dx = torch.from_numpy(x).cuda()
        oshape = list(shape)
        oshape[axis] = 1
        for op in (capi.SUM, capi.MAX, capi.MIN):
            ref_out = torch.zeros(oshape, dtype=dx.dtype, device="cuda")
            got_out = torch.full(oshape, 7, dtype=dx.dtype, device="cuda")
            capi.reduce(op, dtc, dx.data_ptr(), shape, axis, ref_out.data_ptr())
            _noalloc(op, dtc, dx.data_ptr(), shape, axis, got_out.data_ptr())
            torch.cuda.synchronize()
            want, got = ref_out.cpu().numpy(), got_out.cpu().numpy()
            # same plan and summation order as lmpb_reduce: identical results
            assert_bitexact(got, want, f"call {call} op {op} {shape} ax{axis}")
            assert rel_err(got, want) <= 1e-5

