"""The in-tree extensions import in a fresh interpreter that has not imported
torch first (the way the build entry point loads them): the loader brings in
torch's shared libraries, which both extensions link against."""
import glob
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = "3080_mod_p2p_sglang_patch_b200"


@pytest.mark.parametrize("name,getter", [("_cpu", "cpu_ext"), ("_C", "cuda_ext")])
def test_extension_imports_without_a_prior_torch_import(name, getter):
    if not glob.glob(os.path.join(ROOT, PKG, f"{name}.*.so")):
        pytest.skip(f"{name} not built in this tree")
    code = ("import importlib, sys; assert 'torch' not in sys.modules; "
            f"ext = importlib.import_module('{PKG}._ext'); m = ext.{getter}(); print(m.__name__)")
    r = subprocess.run([sys.executable, "-c", code], cwd=ROOT, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    assert r.stdout.strip().endswith(name)
