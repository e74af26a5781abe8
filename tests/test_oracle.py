"""Pins the oracle: the C restatement of the reference's host CSR SpMM/SpMV
against the reference's own functions (built into oracle/_ref from the
reference sources), and the Python coarsening restatement against the
reference's shipped .cfmtx fixtures and the committed golden fixtures
(written by the reference's own converter)."""
import glob
import os

import numpy as np
import pytest

from conftest import REFERENCE, has_reference
from oracle import coarsen_ref, cpu
from sparse_computation_b200 import workloads as wl

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def read_mtx_scipy(path):
    from scipy.io import mmread
    a = mmread(path).tocsr()
    a.sort_indices()
    return a.shape[0], a.shape[1], a.indptr, a.indices, a.data


def golden_cfmtx():
    out = []
    for f in sorted(glob.glob(os.path.join(GOLDEN, "*.cfmtx"))):
        stem, m, n = os.path.basename(f)[:-6].rsplit("-", 2)
        out.append((f, os.path.join(GOLDEN, stem + ".mtx"), int(m), int(n)))
    return out


@pytest.mark.parametrize("f,mtx,m,n", golden_cfmtx(), ids=lambda x: os.path.basename(str(x)))
def test_coarsen_oracle_matches_golden(f, mtx, m, n):
    if "dict" in os.path.basename(f):
        pytest.skip("custom dictionary case is covered in test_formats")
    M, K, ip, ix, dx = read_mtx_scipy(mtx)
    cf = coarsen_ref.coarsen(M, K, ip, ix, dx, m, n)
    assert coarsen_ref.cfmtx_text(cf) == open(f).read()


def test_coarsen_oracle_matches_shipped_fixtures():
    if not has_reference():
        pytest.skip("reference tree not present")
    d = os.path.join(REFERENCE, "matrices")
    stem = "body_decoder_layer_1_encdec_attention_multihead_attention_k_fully_connected"
    M, K, ip, ix, dx = read_mtx_scipy(os.path.join(d, stem + ".mtx"))
    for m, n in [(1, 2), (2, 3), (4, 2), (6, 8)]:
        cf = coarsen_ref.coarsen(M, K, ip, ix, dx, m, n)
        assert coarsen_ref.cfmtx_text(cf) == open(os.path.join(d, f"{stem}-{m}-{n}.cfmtx")).read()


def test_dense_from_cf_roundtrip():
    m, n, ip, ix, dx = wl.config1()[0]
    cf = coarsen_ref.coarsen(m, n, ip, ix, dx, 3, 2)
    A = np.zeros((m, n))
    for r in range(m):
        A[r, ix[ip[r]:ip[r + 1]]] = dx[ip[r]:ip[r + 1]]
    assert np.array_equal(coarsen_ref.dense_from_cf(cf), A)


@pytest.mark.parametrize("case", ["cfg1small", "ragged", "widevals"])
@pytest.mark.parametrize("N", [1, 4, 32])
def test_spmm_oracle_matches_golden(case, N):
    """Golden C = A*B computed by the reference's own spmm_csr_float."""
    g = np.load(os.path.join(GOLDEN, f"spmm_{case}_n{N}.npz"))
    M, K, ip, ix, dx = read_mtx_scipy(os.path.join(GOLDEN, case + ".mtx"))
    C = cpu.spmm_csr_float(ip, ix, dx, g["B"])
    assert np.array_equal(C, g["C"])  # same loop order, same float rounding: bit-exact


def test_spmm_oracle_matches_reference_function():
    if not cpu.ref_available("libref_spmm.so"):
        pytest.skip("oracle/_ref not built (reference tree absent)")
    (m, n, ip, ix, dx), B = wl.config1()
    C0 = cpu.spmm_csr_float(ip, ix, dx, B)
    C1 = cpu.ref_spmm_csr_float(ip, ix, dx, B)
    assert np.array_equal(C0, C1)
    C2 = cpu.spmm_csr_float(ip, ix, dx, B, nthreads=7)
    assert np.array_equal(C0, C2)
    # accumulate semantics (C += A*B)
    Cs = np.full_like(C0, 0.5)
    assert np.array_equal(cpu.spmm_csr_float(ip, ix, dx, B, Cs.copy()),
                          cpu.ref_spmm_csr_float(ip, ix, dx, B, Cs.copy()))
    # row-slice call used by the threaded reference baseline
    Cr = np.zeros_like(C0)
    cpu.ref_spmm_csr_float(ip, ix, dx, B, Cr, 0, 200)
    cpu.ref_spmm_csr_float(ip, ix, dx, B, Cr, 200, m)
    assert np.array_equal(Cr, C0)


def test_spmv_oracle_matches_reference_function():
    if not cpu.ref_available("libref_spmv.so"):
        pytest.skip("oracle/_ref not built (reference tree absent)")
    (m, n, ip, ix, dx), _ = wl.config2(0.9, 1)
    x = wl.dense_b(n, 1, 5)[:, 0]
    assert np.array_equal(cpu.spmv_csr_float(ip, ix, dx, x), cpu.ref_spmv_csr_float(ip, ix, dx, x))


def test_double_and_abs_helpers():
    (m, n, ip, ix, dx), B = wl.config1()
    A = np.zeros((m, n))
    for r in range(m):
        A[r, ix[ip[r]:ip[r + 1]]] = dx[ip[r]:ip[r + 1]]
    Bd = B.astype(np.float64)
    assert np.allclose(cpu.spmm_csr_double(ip, ix, dx, B), A @ Bd, rtol=1e-12, atol=1e-12)
    assert np.allclose(cpu.spmm_csr_abs(ip, ix, dx, B), np.abs(A) @ np.abs(Bd), rtol=1e-12, atol=1e-12)
