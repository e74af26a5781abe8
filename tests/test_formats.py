"""Host formats and the native enumerate + coarsen (no GPU): bit-exact with
the reference converter's output and with the reference's loaders."""
import glob
import os
import random
import struct

import numpy as np
import pytest

import sparse_computation_b200 as sc
from conftest import REFERENCE, has_reference
from oracle import coarsen_ref, cpu
from sparse_computation_b200 import workloads as wl

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
SHIPPED_STEM = "body_decoder_layer_1_encdec_attention_multihead_attention_k_fully_connected"


def golden_cases():
    out = []
    for f in sorted(glob.glob(os.path.join(GOLDEN, "*.cfmtx"))):
        stem, m, n = os.path.basename(f)[:-6].rsplit("-", 2)
        out.append((f, os.path.join(GOLDEN, stem + ".mtx"), int(m), int(n)))
    return out


@pytest.mark.parametrize("f,mtx,m,n", golden_cases(), ids=lambda x: os.path.basename(str(x)))
def test_native_coarsen_matches_reference_converter(f, mtx, m, n, tmp_path):
    a = sc.read_csr_from_mtx(mtx)
    d = os.path.join(GOLDEN, "dict3.txt") if "dict" in os.path.basename(f) else None
    cf = sc.csr_to_compressed_format_converter(a, m, n, d)
    out = tmp_path / "o.cfmtx"
    sc.format_writer(out, cf)
    assert open(out).read() == open(f).read()
    # round trip through the reader keeps every token
    cf2 = sc.read_cfmtx(f)
    cf2.write(tmp_path / "rt.cfmtx")
    assert open(tmp_path / "rt.cfmtx").read() == open(f).read()


def test_native_coarsen_matches_all_shipped_fixtures(tmp_path):
    if not has_reference():
        pytest.skip("reference tree not present")
    d = os.path.join(REFERENCE, "matrices")
    a = sc.read_csr_from_mtx(os.path.join(d, SHIPPED_STEM + ".mtx"))
    checked = 0
    for f in sorted(glob.glob(os.path.join(d, SHIPPED_STEM + "-*.cfmtx"))):
        m, n = map(int, os.path.basename(f)[len(SHIPPED_STEM) + 1:-6].split("-"))
        cf = sc.csr_to_compressed_format_converter(a, m, n)
        cf.write(tmp_path / "o.cfmtx")
        assert open(tmp_path / "o.cfmtx", "rb").read() == open(f, "rb").read(), f
        checked += 1
    assert checked == 46


def test_reader_matches_reference_loader():
    """sc_cf_load vs readCFMTXFile (built from the reference's Sparse_io.cpp)."""
    if not cpu.ref_available("libref_io.so"):
        pytest.skip("oracle/_ref not built")
    files = [f for f, *_ in golden_cases()]
    if has_reference():
        files += sorted(glob.glob(os.path.join(REFERENCE, "matrices", SHIPPED_STEM + "-[246]-*.cfmtx")))
    for f in files:
        mine = sc.read_cfmtx(f)
        ref = cpu.ref_read_cfmtx(f)
        assert len(ref) == mine.num_patterns
        for pid, (km, kn, rpp, npp, cb, vals) in enumerate(ref):
            pc, r, c, v = mine.pattern(pid)
            assert km == mine.kernel_rows
            assert kn == max(1, mine.vector_length)
            assert np.array_equal(r, rpp[: len(r)])
            assert np.array_equal(npp[: len(r)], r * pc)
            assert np.array_equal(c, cb)
            assert np.array_equal(v.view(np.uint32), vals.view(np.uint32)), f


def test_mtx_reader_matches_scipy_and_reference(tmp_path):
    from scipy.io import mmread
    for mtx in sorted(glob.glob(os.path.join(GOLDEN, "*.mtx"))):
        a = sc.read_csr_from_mtx(mtx)
        ip, ix, dx = a.arrays()
        s = mmread(mtx).tocsr()
        s.sort_indices()
        assert np.array_equal(ip, s.indptr) and np.array_equal(ix, s.indices)
        assert np.array_equal(dx, s.data)
        if cpu.ref_available("libref_io.so"):
            cfm = glob.glob(mtx[:-4] + "-*.cfmtx")[0]
            m, n, rp, ri, rx = cpu.ref_read_csr(cfm)
            assert np.array_equal(rp, ip) and np.array_equal(ri, ix) and np.array_equal(rx, dx)


def test_mtx_variants(tmp_path):
    p = tmp_path / "s.mtx"
    p.write_text("%%MatrixMarket matrix coordinate pattern symmetric\n% c\n\n4 4 3\n1 1\n3 2\n4 1\n")
    ip, ix, dx = sc.read_csr_from_mtx(p).arrays()
    assert list(ip) == [0, 2, 3, 4, 5] and list(ix) == [0, 3, 2, 1, 0] and list(dx) == [1.0] * 5
    p.write_text("%%MatrixMarket matrix coordinate integer general\n2 3 3\n1 3 4\n1 3 5\n2 1 -2\n")
    ip, ix, dx = sc.read_csr_from_mtx(p).arrays()  # duplicates summed (scipy tocsr)
    assert list(ip) == [0, 1, 2] and list(ix) == [2, 0] and list(dx) == [9.0, -2.0]
    for bad in ["%%MatrixMarket matrix array real general\n1 1\n1\n",
                "%%MatrixMarket matrix coordinate complex general\n1 1 1\n1 1 1 0\n",
                "%%MatrixMarket matrix coordinate real general\n2 2 2\n1 1 1\n",
                "%%MatrixMarket matrix coordinate real general\n2 2 1\n3 1 1\n"]:
        p.write_text(bad)
        with pytest.raises(sc.ScError) as e:
            sc.read_csr_from_mtx(p)
        assert e.value.code in (sc.SC_ERR_FORMAT, sc.SC_ERR_UNSUPPORTED)


def _py_csr(a):
    m, n, ip, ix, dx = a
    return sc.CSR.from_arrays(m, n, ip, ix, dx)


@pytest.mark.parametrize("m,n", [(1, 1), (2, 4), (3, 0), (4, 1), (5, 7), (6, 2)])
def test_native_vs_oracle_synthetic(m, n):
    for a in [wl.config1()[0], wl.config2(0.5, 1)[0], wl.config3((512, 2048), 32)[0]]:
        cf = sc.csr_to_compressed_format_converter(_py_csr(a), m, n, nthreads=3)
        ref = coarsen_ref.coarsen(*a, m, n) if a[0] <= 512 else None
        if ref is None:
            continue
        assert cf.header == ref["header"]
        for pid, (rpp, cb, vals) in enumerate(ref["blocks"]):
            pc, r, c, v = cf.pattern(pid)
            assert list(r) == rpp and list(c) == cb
            assert np.array_equal(v, np.array([0.0 if x is None else x for x in vals], np.float32))


def test_thread_count_does_not_change_output(tmp_path):
    a = _py_csr(wl.config3((2048, 512), 32)[0])
    outs = []
    for t in (1, 2, 5, 16):
        cf = sc.csr_to_compressed_format_converter(a, 4, 2, nthreads=t)
        cf.write(tmp_path / f"t{t}.cfmtx")
        outs.append(open(tmp_path / f"t{t}.cfmtx", "rb").read())
    assert all(o == outs[0] for o in outs)


def test_edge_matrices(tmp_path):
    # empty matrix, all-empty rows, single row, M not a multiple of m
    cases = [wl.csr_from_dense(np.zeros((0, 5), np.float32)),
             wl.csr_from_dense(np.zeros((7, 5), np.float32)),
             wl.csr_from_dense(np.array([[0, 1.5, 0, 2]], np.float32)),
             wl.csr_from_dense(np.eye(9, dtype=np.float32))]
    for a in cases:
        for m, n in [(4, 1), (3, 2), (1, 3), (2, 0)]:
            cf = sc.csr_to_compressed_format_converter(_py_csr(a), m, n)
            cf.write(tmp_path / "e.cfmtx")
            ref = coarsen_ref.coarsen(*a, m, n)
            assert open(tmp_path / "e.cfmtx").read() == coarsen_ref.cfmtx_text(ref)
            assert cf.real_nnz == len(a[3])


def test_custom_dictionary_rules(tmp_path):
    d = tmp_path / "d.txt"
    d.write_text("2 1 2\n10 1\n01 0\n")  # "11" missing: those columns are dropped
    a = wl.csr_from_dense(np.array([[1, 2, 0], [0, 3, 4]], np.float32))
    cf = sc.csr_to_compressed_format_converter(_py_csr(a), 2, 1, str(d))
    assert cf.header == [("10", 1), ("01", 0)]
    assert cf.real_nnz == 2  # column 1 (both rows) dropped
    d.write_text("2 1 1\n11 3\n")  # id outside [0, number of patterns)
    with pytest.raises(sc.ScError):
        sc.csr_to_compressed_format_converter(_py_csr(a), 2, 1, str(d))
    d.write_text("2 1 2\n00 0\n11 1\n")  # popcount-0 pattern cannot be packed
    with pytest.raises(sc.ScError):
        sc.csr_to_compressed_format_converter(_py_csr(a), 2, 1, str(d))


def test_float_repr_matches_python(tmp_path):
    """Values are written as Python's float repr (numpy float64 str)."""
    rng = random.Random(5)
    vals = [0.1, 1.0, -2.5, 1e-5, 1.5e16, 1e16, 9999999999999998.0, 123456789012345.6, 5e-324,
            1.7976931348623157e308, 0.0001, 0.00001234, -0.0, 3.0000000000000004]
    vals += [struct.unpack("<d", struct.pack("<Q", rng.getrandbits(64)))[0] for _ in range(3000)]
    vals += [float(np.float32(rng.gauss(0, 1) * 10 ** rng.randint(-30, 30))) for _ in range(3000)]
    vals = [v for v in vals if np.isfinite(v)]
    m = len(vals)
    ip = np.arange(m + 1, dtype=np.int32)
    ix = np.zeros(m, np.int32)
    cf = sc.csr_to_compressed_format_converter(sc.CSR.from_arrays(m, 1, ip, ix, np.array(vals)), 1, 1)
    cf.write(tmp_path / "v.cfmtx")
    line = open(tmp_path / "v.cfmtx").read().split("\n")[4]
    assert line.split(" ") == [str(np.float64(v)) for v in vals]


def test_binary_sidecar_roundtrip(tmp_path):
    for f, *_ in golden_cases():
        cf = sc.read_cfmtx(f)
        cf.write_binary(tmp_path / "x.cfbin")
        cb = sc.read_cfbin(tmp_path / "x.cfbin")
        assert cb.header == cf.header and cb.num_patterns == cf.num_patterns and cb.real_nnz == cf.real_nnz
        for pid in range(cf.num_patterns):
            a, b = cf.pattern(pid), cb.pattern(pid)
            assert a[0] == b[0] and all(np.array_equal(x, y) for x, y in zip(a[1:], b[1:]))
        cb.write(tmp_path / "back.cfmtx")
        assert open(tmp_path / "back.cfmtx").read() == open(f).read()
    # from a CF built in memory
    a = wl.config3((512, 2048), 32)[0]
    cf = sc.csr_to_compressed_format_converter(_py_csr(a), 5, 3)
    cf.write(tmp_path / "m.cfmtx")
    cf.write_binary(tmp_path / "m.cfbin")
    sc.read_cfbin(tmp_path / "m.cfbin").write(tmp_path / "m2.cfmtx")
    assert open(tmp_path / "m2.cfmtx").read() == open(tmp_path / "m.cfmtx").read()
    # corrupt / truncated
    data = open(tmp_path / "m.cfbin", "rb").read()
    open(tmp_path / "t.cfbin", "wb").write(data[: len(data) // 2])
    with pytest.raises(sc.ScError) as e:
        sc.read_cfbin(tmp_path / "t.cfbin")
    assert e.value.code == sc.SC_ERR_FORMAT
    with pytest.raises(sc.ScError):
        sc.read_cfbin(tmp_path / "m.cfmtx")
