"""Reference-facing callers: the .mtx -> .cfmtx converter command line and
the three demo executables (reference flags and CSV report)."""
import csv
import io
import os
import shutil
import subprocess
import sys

import pytest

from sparse_computation_b200 import build as b

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def exe(name):
    path = os.path.join(b.BIN, name)
    if not os.path.exists(path):
        b.build_apps()
    return path


@pytest.mark.parametrize("m,n", [(4, 1), (3, 2), (6, 8)])
def test_format_generator_cli(tmp_path, m, n):
    shutil.copy(os.path.join(GOLDEN, "ragged.mtx"), tmp_path / "ragged.mtx")
    subprocess.run([sys.executable, "-m", "sparse_computation_b200.format_generator", str(tmp_path / "ragged.mtx"),
                    str(m), str(n), "--save_collection", "true"], check=True, cwd=ROOT, capture_output=True)
    want = open(os.path.join(GOLDEN, f"ragged-{m}-{n}.cfmtx")).read()
    assert open(tmp_path / f"ragged-{m}-{n}.cfmtx").read() == want
    assert open(tmp_path / "ragged.cfmtx").read() == want


def test_format_generator_custom_dictionary(tmp_path):
    shutil.copy(os.path.join(GOLDEN, "ragged_dict.mtx"), tmp_path / "ragged_dict.mtx")
    subprocess.run([sys.executable, "-m", "sparse_computation_b200.format_generator",
                    str(tmp_path / "ragged_dict.mtx"), "3", "2", "--pattern_dictionary",
                    os.path.join(GOLDEN, "dict3.txt")], check=True, cwd=ROOT, capture_output=True)
    assert open(tmp_path / "ragged_dict-3-2.cfmtx").read() == open(os.path.join(GOLDEN, "ragged_dict-3-2.cfmtx")).read()


@pytest.mark.parametrize("args,msg", [
    ([], "'matrix' is manditory argument"),
    (["-m", "a.cfmtx"], "'numerical_operation' is manditory argument"),
    (["-m", "a.cfmtx", "-n", "SPMM"], "'storage_format' is manditory argument"),
    (["-m", "a.cfmtx", "-n", "FOO", "-s", "CSR"], "'numerical_operation' must be passed in as one of"),
    (["-m", "a.cfmtx", "-n", "SPMM", "-s", "COO"], "'storage_format' must be passed in as one of"),
])
def test_demo_argument_errors(args, msg):
    # src/InputParser.cpp:74-93: message on stdout, exit status 0
    r = subprocess.run([exe("spmm_demo_gpu"), *args], capture_output=True, text=True)
    assert r.returncode == 0 and msg in r.stdout


@pytest.mark.gpu
@pytest.mark.parametrize("name,n,cf", [("spmm_demo_gpu", 32, "cfg1small-4-1.cfmtx"),
                                       ("spmm_demo_gpu", 128, "cfg1small-6-3.cfmtx"),
                                       ("spmm_small_b_col_demo_gpu", 4, "ragged-4-1.cfmtx"),
                                       ("spmm_small_b_col_demo_gpu", 1, "cfg1small-2-4.cfmtx"),
                                       ("spmv_demo_gpu", 1, "widevals-3-4.cfmtx")])
def test_demo_executables_report_correct(name, n, cf):
    r = subprocess.run([exe(name), "-m", os.path.join(GOLDEN, cf), "--header", "--baseline=true", "-n",
                        "SPMV" if "spmv" in name else "SPMM", "-s", "CSR", "-t", str(n),
                        f"--b_matrix_columns={n}", "--number_of_warps=1"], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    rows = list(csv.reader(io.StringIO(r.stdout)))
    head, body = rows[0], rows[1:]
    assert len(body) == 3  # cuBLAS, cuSPARSE, ours
    ours = dict(zip(head, body[-1]))
    assert "Pattern B200" in ours["Implementation Name"]
    for i in range(7):
        assert ours[f"Correct{i}"] == "1", ours
    assert float(ours["GFLOPs"]) > 0
