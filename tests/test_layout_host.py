"""Index functions of the device layouts, checked on the host (no GPU): the
64-byte swizzle of the 3xBF16 tile images and the lane-block item layout of
the staged SpMV kernel (tests/layout_check.cu, built with nvcc's host compiler)."""
import os
import shutil
import subprocess
import tempfile

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")


@pytest.mark.skipif(not (os.path.exists(NVCC) or shutil.which("nvcc")), reason="nvcc not available")
def test_layout_index_functions():
    nvcc = NVCC if os.path.exists(NVCC) else shutil.which("nvcc")
    with tempfile.TemporaryDirectory() as d:
        exe = os.path.join(d, "layout_check")
        subprocess.run([nvcc, "-std=c++17", "-O1", "-gencode", "arch=compute_100a,code=sm_100a", "-I", os.path.join(ROOT, "sparse_computation_b200", "csrc"),
                        "-I", os.path.join(ROOT, "include"), os.path.join(ROOT, "tests", "layout_check.cu"),
                        "-o", exe], check=True, capture_output=True, text=True)
        r = subprocess.run([exe], capture_output=True, text=True)
        assert r.returncode == 0 and r.stdout.strip() == "ok", r.stdout + r.stderr
