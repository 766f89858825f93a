"""Builds the native parts of rushlite_b200 in-tree.

* ``liblmpb.so``  — the C-ABI kernel library (include/lmpb.h): sm_100a CUDA
  kernels, the NVRTC fused-kernel compiler and its host glue.
* ``_C*.so``      — the pybind11 module with the Lamp3 host API (Tensor,
  Variable, ops, lazy capture) layered on liblmpb.so.

Everything is compiled with nvcc / g++ directly (no CMake); objects are rebuilt
only when a source or header is newer than the object.
"""
from __future__ import annotations

import concurrent.futures as cf
import glob
import os
import subprocess
import sys
import sysconfig

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
OBJ = os.path.join(PKG, "_build")
INC = os.path.join(ROOT, "include")
CUDA = os.environ.get("CUDA_HOME", "/usr/local/cuda")
NVCC = os.path.join(CUDA, "bin", "nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]

LIB = os.path.join(PKG, "liblmpb.so")
EXT = os.path.join(PKG, "_C" + sysconfig.get_config_var("EXT_SUFFIX"))


def _newer(target: str, deps: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _run(cmd: list[str]) -> None:
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError("build failed:\n" + " ".join(cmd) + "\n" + r.stdout + r.stderr)


def _headers(d: str) -> list[str]:
    return glob.glob(os.path.join(d, "**", "*.h*"), recursive=True) + glob.glob(
        os.path.join(d, "**", "*.cuh"), recursive=True)


def _gen_ops_inc() -> None:
    """Embeds ops_device.cuh as a C++ string for the NVRTC programs."""
    src = os.path.join(CSRC, "ops_device.cuh")
    dst = os.path.join(OBJ, "ops_device_inc.h")
    if not _newer(dst, [src]):
        return
    text = open(src).read()
    with open(dst, "w") as f:
        f.write('static const char* const kOpsDeviceSource = R"LMPBSRC(' + text + ')LMPBSRC";\n')


def _compile_lib(jobs: int) -> None:
    os.makedirs(OBJ, exist_ok=True)
    _gen_ops_inc()
    hdrs = _headers(CSRC) + _headers(INC) + [os.path.join(OBJ, "ops_device_inc.h")]
    srcs = sorted(glob.glob(os.path.join(CSRC, "*.cu")) + glob.glob(os.path.join(CSRC, "*.cpp")))
    os.makedirs(OBJ, exist_ok=True)
    tasks = []
    objs = []
    for s in srcs:
        o = os.path.join(OBJ, os.path.basename(s) + ".o")
        objs.append(o)
        if not _newer(o, [s] + hdrs):
            continue
        if s.endswith(".cu"):
            cmd = [NVCC, *ARCH, "-lineinfo", "-O3", "-std=c++17", "-Xcompiler", "-fPIC",
                   "--expt-relaxed-constexpr", "-I", INC, "-I", CSRC, "-c", s, "-o", o]
        else:
            cmd = ["g++", "-O2", "-std=c++17", "-fPIC", "-I", INC, "-I", CSRC, "-I", OBJ,
                   "-I", os.path.join(CUDA, "include"), "-c", s, "-o", o]
        tasks.append(cmd)
    with cf.ThreadPoolExecutor(max_workers=jobs) as ex:
        list(ex.map(_run, tasks))
    if tasks or _newer(LIB, objs):
        _run([NVCC, *ARCH, "-shared", "-o", LIB, *objs,
              "-L" + os.path.join(CUDA, "lib64"), "-L" + os.path.join(CUDA, "lib64", "stubs"),
              "-lnvrtc", "-Xlinker", "-rpath," + os.path.join(CUDA, "lib64")])


def _compile_ext(jobs: int) -> None:
    bdir = os.path.join(PKG, "host")
    if not os.path.isdir(bdir):
        return
    import pybind11

    hdrs = _headers(bdir) + _headers(INC)
    srcs = sorted(glob.glob(os.path.join(bdir, "*.cpp")))
    objs, tasks = [], []
    pyinc = sysconfig.get_paths()["include"]
    for s in srcs:
        o = os.path.join(OBJ, "host_" + os.path.basename(s) + ".o")
        objs.append(o)
        if not _newer(o, [s] + hdrs):
            continue
        tasks.append(["g++", "-O2", "-std=c++20", "-fPIC", "-fvisibility=hidden", "-I", INC,
                      "-I", bdir, "-I", pybind11.get_include(), "-I", pyinc,
                      "-I", os.path.join(CUDA, "include"), "-c", s, "-o", o])
    with cf.ThreadPoolExecutor(max_workers=jobs) as ex:
        list(ex.map(_run, tasks))
    if tasks or _newer(EXT, objs + [LIB]):
        _run(["g++", "-shared", "-o", EXT, *objs, "-L" + PKG, "-llmpb",
              "-L" + os.path.join(CUDA, "lib64"), "-lcudart",
              "-Wl,-rpath,$ORIGIN", "-Wl,-rpath," + os.path.join(CUDA, "lib64")])


def build(jobs: int | None = None) -> None:
    jobs = jobs or max(2, os.cpu_count() or 2)
    _compile_lib(jobs)
    _compile_ext(jobs)


if __name__ == "__main__":
    build()
    print("built", LIB, file=sys.stderr)
