"""Resource budgets of the tensor-core GEMM kernels, checked at build time
from `nvcc -Xptxas -v` (no GPU): the CTA-pair kernel must fit one 320-thread
CTA per SM (at most 168 registers a thread: 10 warps share the SM's four
16K-register sub-partitions, three on some), and no GEMM kernel may spill."""
from __future__ import annotations

import os
import re
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
NVCC = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"


@pytest.mark.skipif(not os.path.exists(NVCC), reason="nvcc absent")
def test_gemm_kernels_register_budget_and_no_spills(tmp_path):
    src = os.path.join(ROOT, "rushlite_b200", "csrc", "gemm_sm100.cu")
    r = subprocess.run([NVCC, "-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-std=c++17", "-Xptxas", "-v",
                        "-I", os.path.join(ROOT, "rushlite_b200", "csrc"), "-I", os.path.join(ROOT, "include"),
                        "-c", src, "-o", str(tmp_path / "g.o")], capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    kernels = {}
    current = None
    for line in r.stderr.splitlines():
        m = re.search(r"Compiling entry function '(\S+)'", line)
        if m:
            current = m.group(1)
            continue
        if current is None:
            continue
        m = re.search(r"(\d+) bytes spill stores, (\d+) bytes spill loads", line)
        if m:
            kernels.setdefault(current, {})["spill"] = int(m.group(1)) + int(m.group(2))
        m = re.search(r"Used (\d+) registers", line)
        if m:
            kernels.setdefault(current, {})["regs"] = int(m.group(1))
    pair = [k for k in kernels if "gemm_f16x3_pair_kernel" in k]
    single = [k for k in kernels if "gemm_f16x3_kernel" in k]
    assert pair and single, sorted(kernels)
    assert kernels[pair[0]]["regs"] <= 168, kernels[pair[0]]
    for k in pair + single + [k for k in kernels if "split" in k or "colmax" in k]:
        assert kernels[k].get("spill", 0) == 0, (k, kernels[k])
