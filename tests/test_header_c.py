"""The boundary header is plain C: a C99 program (no C++ compiler, no CUDA
headers) includes include/lmpb.h, links rushlite_b200/liblmpb.so and calls
the host-only entry points — what a cgo / FFI consumer would do."""
from __future__ import annotations

import os
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIBDIR = os.path.join(ROOT, "rushlite_b200")

PROGRAM = r"""
#include <stdio.h>
#include <string.h>
#include "lmpb.h"

int main(void) {
  int64_t a[2] = {8192, 8192}, b[2] = {8192, 1}, out[LMPB_MAX_DIMS];
  int nd = 0;
  if (lmpb_broadcast_shape(a, 2, b, 2, out, &nd) != LMPB_OK) return 1;
  int64_t c[2] = {3, 2}, d[2] = {4, 2};
  lmpb_status bad = lmpb_broadcast_shape(c, 2, d, 2, out + 2, &nd);
  printf("%s|%d|%lld|%lld|%d|%s\n", strstr(lmpb_version(), "sm_100a") ? "ver" : "nover", nd,
         (long long)out[0], (long long)out[1], (int)bad, lmpb_last_error());
  return 0;
}
"""


@pytest.mark.skipif(shutil.which("gcc") is None, reason="gcc absent")
def test_header_compiles_and_links_as_c99(tmp_path):
    src = tmp_path / "consumer.c"
    src.write_text(PROGRAM)
    exe = tmp_path / "consumer"
    subprocess.run(["gcc", "-std=c99", "-Wall", "-Werror", "-I", os.path.join(ROOT, "include"), str(src),
                    "-o", str(exe), "-L", LIBDIR, "-llmpb", f"-Wl,-rpath,{LIBDIR}"], check=True)
    r = subprocess.run([str(exe)], capture_output=True, text=True, check=True)
    ver, nd, d0, d1, bad, msg = r.stdout.strip().split("|", 5)
    assert (ver, nd, d0, d1) == ("ver", "2", "8192", "8192")
    assert int(bad) == 1 and "Broadcast" in msg


@pytest.mark.skipif(shutil.which("g++") is None, reason="g++ absent")
def test_header_compiles_as_cpp(tmp_path):
    src = tmp_path / "consumer.cpp"
    src.write_text(PROGRAM)
    subprocess.run(["g++", "-std=c++17", "-Wall", "-Werror", "-fsyntax-only", "-I", os.path.join(ROOT, "include"),
                    str(src)], check=True)


@pytest.mark.skipif(shutil.which("g++") is None, reason="g++ absent")
def test_host_api_header_is_self_contained(tmp_path):
    """The C++ Lamp3 API of this backend (lmp::tensor, lmp::autograd) compiles
    from its one header plus the C ABI."""
    src = tmp_path / "user.cpp"
    src.write_text('#include "lamp.hpp"\n'
                   "int main() {\n"
                   "  using namespace lmp;\n"
                   "  autograd::Variable (*mm)(const autograd::Variable&, const autograd::Variable&) =\n"
                   "      &autograd::ops::matmul;\n"
                   "  tensor::Graph* g = tensor::capturing_graph();\n"
                   "  return (mm != nullptr && g == nullptr) ? 0 : 1;\n"
                   "}\n")
    cuda_inc = "/usr/local/cuda/include"
    subprocess.run(["g++", "-std=c++17", "-Wall", "-Werror", "-fsyntax-only", "-I", os.path.join(ROOT, "include"),
                    "-I", os.path.join(ROOT, "rushlite_b200", "host"), "-I", cuda_inc, str(src)], check=True)
