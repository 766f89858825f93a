"""No silent fallback: without its native libraries the package refuses to
import and the C-ABI binding refuses to load (there is no CPU path to fall
back to)."""
from __future__ import annotations

import os
import shutil
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _copy_without_native(dst):
    src = os.path.join(ROOT, "rushlite_b200")
    shutil.copytree(src, os.path.join(dst, "rushlite_b200"),
                    ignore=shutil.ignore_patterns("*.so", "_build", "__pycache__", "csrc", "host"))


def test_package_import_fails_without_native_module(tmp_path):
    _copy_without_native(str(tmp_path))
    r = subprocess.run([sys.executable, "-c", "import rushlite_b200"], cwd=str(tmp_path), capture_output=True,
                       text=True, env={**os.environ, "PYTHONPATH": str(tmp_path)})
    assert r.returncode != 0
    assert "native module is not built" in r.stderr


def test_capi_refuses_to_load_without_library(tmp_path):
    _copy_without_native(str(tmp_path))
    code = ("import importlib.util, sys\n"
            "spec = importlib.util.spec_from_file_location('capi', 'rushlite_b200/capi.py')\n"
            "m = importlib.util.module_from_spec(spec); spec.loader.exec_module(m)\n"
            "try:\n    m.lib()\nexcept ImportError as e:\n    print('refused:', e); sys.exit(0)\n"
            "sys.exit(1)\n")
    r = subprocess.run([sys.executable, "-c", code], cwd=str(tmp_path), capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    assert "liblmpb.so is missing" in r.stdout
