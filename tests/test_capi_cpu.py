"""C-ABI checks that need no GPU: the library loads and exports every symbol
include/lmpb.h declares, host-side shape logic, and the fused compiler's
generated programs compile for sm_100a under NVRTC."""
from __future__ import annotations

import ctypes as C
import os
import re

import pytest

from rushlite_b200 import capi

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    text = open(os.path.join(ROOT, "include", "lmpb.h")).read()
    return sorted(set(re.findall(r"\b(lmpb_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    lib = capi.lib()
    decl = declared_symbols()
    assert len(decl) >= 18
    missing = [s for s in decl if not hasattr(lib, s)]
    assert not missing, missing
    assert sorted(capi.EXPORTS) == decl


def test_version_and_error_string():
    assert b"sm_100a" in capi.lib().lmpb_version()
    with pytest.raises(capi.LmpbError) as e:
        capi.broadcast_shape([3, 2], [4, 2])
    assert "Broadcast rule violation" in str(e.value)


@pytest.mark.parametrize("a,b,out", [([3, 2], [1, 2], [3, 2]), ([3, 2], [3, 1], [3, 2]),
                                      ([3, 2], [1], [3, 2]), ([3, 1, 5], [4, 1], [3, 4, 5]),
                                      ([], [2], [2]), ([2, 1, 3], [1, 4, 1], [2, 4, 3])])
def test_broadcast_shape(a, b, out):
    assert capi.broadcast_shape(a, b) == out


def test_invalid_arguments_are_reported_without_a_gpu():
    L = capi.lib()
    # unknown dtype / op never reach a kernel
    assert L.lmpb_unary(0, 17, None, None, 4, 0.0, 0.0, None) == 1
    assert L.lmpb_reduce(0, 4, None, capi.shape_arr([3]), 1, 2, None, None) == 1
    assert L.lmpb_gemm_f32(0, 0, None, None, None, 2, 2, 2, C.c_float(0.5), None) == 1
    # the fused Linear entry: negative sizes and missing pointers are user errors
    assert L.lmpb_gemm_f32_bias_act(0, 0, None, None, None, -1, 2, 2, None, 0, 0.0, 0.0, None) == 1
    assert L.lmpb_gemm_f32_bias_act(0, 0, None, None, None, 2, 2, 2, None, 1, 0.0, 1.0, None) == 1
    assert b"lmpb_gemm_f32_bias_act" in L.lmpb_last_error()
    # zero-size work is a no-op
    assert L.lmpb_unary(0, 4, None, None, 0, 0.0, 0.0, None) == 0
    assert L.lmpb_gemm_f32_bias_act(0, 0, None, None, None, 0, 8, 8, None, 1, 0.0, 1.0, None) == 0


def _nvrtc():
    for p in ("/usr/local/cuda/lib64/libnvrtc.so", "/usr/local/cuda/lib64/libnvrtc.so.12"):
        if os.path.exists(p):
            return C.CDLL(p)
    pytest.skip("libnvrtc not found")


def _compile(src: str) -> str:
    nv = _nvrtc()
    prog = C.c_void_p()
    assert nv.nvrtcCreateProgram(C.byref(prog), src.encode(), b"t.cu", 0, None, None) == 0
    opts = [b"--gpu-architecture=sm_100a", b"-std=c++17", b"--fmad=false", b"-default-device"]
    r = nv.nvrtcCompileProgram(prog, len(opts), (C.c_char_p * len(opts))(*opts))
    n = C.c_size_t()
    nv.nvrtcGetProgramLogSize(prog, C.byref(n))
    log = C.create_string_buffer(max(1, n.value))
    nv.nvrtcGetProgramLog(prog, log)
    assert r == 0, log.value.decode()[:4000]
    return log.value.decode()


F32 = capi.FLOAT32
A, B = (64, 128), (64, 1)
CHAIN = [(capi.FN_LEAF, 0, F32, 0), (capi.FN_LEAF, 0, F32, 1), (capi.FN_BINARY, capi.MUL, F32, 0, 0),
         (capi.FN_BINARY, capi.ADD, F32, 2, 1), (capi.FN_UNARY, capi.EXP, F32, 3),
         (capi.FN_BINARY, capi.MUL, F32, 4, 0), (capi.FN_CONST, 0, F32, 0, 0, 1.0),
         (capi.FN_BINARY, capi.ADD, F32, 1, 6), (capi.FN_UNARY, capi.LOG, F32, 7),
         (capi.FN_BINARY, capi.SUB, F32, 5, 8)]


@pytest.mark.parametrize("outs,pattern", [
    ([(9, capi.OUT_STORE, F32, A)], "elementwise"),
    ([(9, capi.OUT_ACCUM, F32, A), (4, capi.OUT_REDUCE_SUM_ACCUM, F32, B)], "row"),
])
def test_fused_chain_compiles(outs, pattern):
    f = capi.Fused(CHAIN, [(F32, A), (F32, B)], outs, A)
    src = f.source
    assert "lmpb_fused_v" in src and "lmpb_fused_s" in src
    if pattern == "row":
        assert "warp_sum" in src
    _compile(src)


def test_fused_column_reduce_and_mixed_dtypes_compile():
    f = capi.Fused([(capi.FN_LEAF, 0, F32, 0), (capi.FN_LEAF, 0, F32, 1),
                    (capi.FN_BINARY, capi.CLAMP_BACKWARD, F32, 0, 1, 0.0, 1e308)],
                   [(F32, (512, 4096)), (F32, (512, 4096))],
                   [(2, capi.OUT_STORE, F32, (512, 4096)), (2, capi.OUT_REDUCE_SUM_ACCUM, F32, (4096,))],
                   (512, 4096))
    assert "lmpb_fused_c" in f.source  # split-row combine kernel
    _compile(f.source)
    g = capi.Fused([(capi.FN_LEAF, 0, capi.INT32, 0), (capi.FN_LEAF, 0, capi.FLOAT64, 1),
                    (capi.FN_BINARY, capi.POW, capi.FLOAT64, 0, 1),
                    (capi.FN_UNARY, capi.CLAMP, capi.FLOAT64, 2, 0, -1.0, 3.0)],
                   [(capi.INT32, (3, 1, 5)), (capi.FLOAT64, (4, 1))],
                   [(3, capi.OUT_STORE, capi.FLOAT64, (3, 4, 5))], (3, 4, 5))
    _compile(g.source)


def test_fused_rejects_bad_programs():
    with pytest.raises(capi.LmpbError):  # leaf does not broadcast
        capi.Fused([(capi.FN_LEAF, 0, F32, 0)], [(F32, (3, 5))], [(0, capi.OUT_STORE, F32, (3, 4))], (3, 4))
    with pytest.raises(capi.LmpbError):  # forward reference
        capi.Fused([(capi.FN_BINARY, capi.ADD, F32, 0, 1), (capi.FN_LEAF, 0, F32, 0)],
                   [(F32, (4,))], [(0, capi.OUT_STORE, F32, (4,))], (4,))
    with pytest.raises(capi.LmpbError) as e:  # reduce over a middle axis of 3 groups
        capi.Fused([(capi.FN_LEAF, 0, F32, 0)], [(F32, (2, 3, 4))],
                   [(0, capi.OUT_REDUCE_SUM, F32, (2, 1, 4))], (2, 3, 4))
    assert e.value.status == 3


def test_fastdiv_emulation():
    """Host model of the 32-bit multiply-shift division used by the kernels."""
    import random

    def make(d):
        s = 0
        while (1 << s) < d:
            s += 1
        m = ((1 << (32 + s)) + d - 1) // d
        return (m - (1 << 32)) & 0xFFFFFFFF, s

    rnd = random.Random(0)
    for d in [1, 2, 3, 7, 10, 1000, 4096, 8191, 65535, 1 << 20, (1 << 31) - 1] + [rnd.randint(1, 1 << 31) for _ in range(200)]:
        mul, s = make(d)
        for n in [0, 1, d - 1, d, d + 1, (1 << 31) - 1] + [rnd.randint(0, (1 << 31) - 1) for _ in range(200)]:
            t = (n * mul) >> 32
            assert ((t + n) >> s) == n // d, (n, d)


@pytest.mark.parametrize("env,expect", [({"LMPB_FUSED_ROW_UNROLL": "4"}, "#pragma unroll 4"),
                                        ({"LMPB_FUSED_WARP_ROWS": "100000"}, "wid; row <"),
                                        ({"LMPB_FUSED_VEC_RED": "4"}, "Pack<float, 4>")])
def test_fused_tuning_overrides_generate_and_compile(monkeypatch, env, expect):
    """The tuning switches of the generated row-reduce kernel (unroll, warp
    per row, packet width) change the source as documented and still compile."""
    for k, v in env.items():
        monkeypatch.setenv(k, v)
    big = (64, 4096)  # rows of 4096: a CTA per row by default
    f = capi.Fused(CHAIN, [(F32, big), (F32, (64, 1))],
                   [(9, capi.OUT_STORE, F32, big), (5, capi.OUT_REDUCE_SUM, F32, (64, 1))], big)
    assert expect in f.source
    _compile(f.source)
