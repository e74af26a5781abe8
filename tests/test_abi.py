"""The C ABI library loads, exports exactly what include/sc_b200.h declares,
and reports errors as status codes (no GPU needed)."""
import ctypes
import os
import re

import pytest

import sparse_computation_b200 as sc

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    text = open(os.path.join(ROOT, "include", "sc_b200.h")).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(sc_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    L = ctypes.CDLL(sc.LIB_PATH)
    decl = declared_symbols()
    assert decl, "no declarations parsed"
    missing = [s for s in decl if not hasattr(L, s)]
    assert not missing, missing
    assert sorted(decl) == sorted(sc.EXPORTED_SYMBOLS)


def test_only_c_abi_is_exported():
    out = os.popen(f"nm -D --defined-only {sc.LIB_PATH}").read().split("\n")
    names = [l.split()[-1] for l in out if l.strip() and l.split()[1] in "TtWw"]
    ours = [n for n in names if n.startswith("sc_")]
    assert sorted(ours) == sorted(declared_symbols())


def test_version_and_errors(tmp_path):
    L = sc.lib()
    assert L.sc_version() >= 100
    with pytest.raises(sc.ScError) as e:
        sc.read_cfmtx(tmp_path / "missing.cfmtx")
    assert e.value.code == sc.SC_ERR_IO
    assert "unable to open" in str(e.value)
    bad = tmp_path / "bad.cfmtx"
    bad.write_text("1 2 3\n")
    with pytest.raises(sc.ScError) as e:
        sc.read_cfmtx(bad)
    assert e.value.code == sc.SC_ERR_FORMAT
    trunc = tmp_path / "t.cfmtx"
    trunc.write_text("4 4 2 3 1\n11 0 \n10 1 \n01 2 \n0 1 1\n")
    with pytest.raises(sc.ScError) as e:
        sc.read_cfmtx(trunc)
    assert e.value.code == sc.SC_ERR_FORMAT


def test_plan_fails_loudly_without_gpu():
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    a = sc.CSR.from_arrays(4, 4, [0, 1, 1, 1, 1], [2], [1.0])
    cf = sc.csr_to_compressed_format_converter(a, 2, 1)
    with pytest.raises(sc.ScError) as e:
        sc.SpMMPlan(cf, 32)
    assert e.value.code == sc.SC_ERR_CUDA


def test_plan_rejects_bad_cf_before_device():
    """Validation happens on the host, before any CUDA call."""
    a = sc.CSR.from_arrays(4, 4, [0, 1, 1, 1, 1], [2], [1.0])
    cf = sc.csr_to_compressed_format_converter(a, 8, 1)  # kernel_m 8 > 6
    with pytest.raises(sc.ScError) as e:
        sc.SpMMPlan(cf, 32)
    assert e.value.code == sc.SC_ERR_UNSUPPORTED


def test_plan_flags_validated_on_host():
    """sc_plan_create_ex rejects unknown or contradictory flags and bad panel
    ranges before any CUDA call."""
    a = sc.CSR.from_arrays(4, 4, [0, 1, 1, 1, 1], [2], [1.0])
    cf = sc.csr_to_compressed_format_converter(a, 2, 1)
    for flags, rng in ((32, None), (sc.SC_PLAN_DENSE_OFF | sc.SC_PLAN_DENSE_BF16, None),
                       (sc.SC_PLAN_DENSE_OFF | sc.SC_PLAN_DENSE_ON, None), (sc.SC_PLAN_DENSE_ON, (2, 1)),
                       (sc.SC_PLAN_DENSE_ON, (-1, 3)), (sc.SC_PLAN_VALUES_F16 | sc.SC_PLAN_VALUES_BF16, None)):
        with pytest.raises(sc.ScError) as e:
            sc.SpMMPlan(cf, 128, panel_range=rng, flags=flags)
        assert e.value.code == sc.SC_ERR_ARG


def test_csr_create_validates():
    with pytest.raises(sc.ScError):
        sc.CSR.from_arrays(2, 2, [0, 2, 1], [0, 1], [1.0, 2.0])
    with pytest.raises(sc.ScError):
        sc.CSR.from_arrays(1, 2, [0, 2], [1, 0], [1.0, 2.0])  # unsorted
    with pytest.raises(sc.ScError):
        sc.CSR.from_arrays(1, 2, [0, 1], [5], [1.0])  # out of range


def test_companion_path():
    # utils/Sparse_io.cpp:28-46
    assert sc.companion_mtx_path("dir/mat-4-8.cfmtx") == "dir/mat.mtx"
    assert sc.companion_mtx_path("dir/my-mat-64-128.cfmtx") == "dir/my-mat.mtx"
    assert sc.companion_mtx_path("mat.cfmtx") == "mat.mtx"
    assert sc.companion_mtx_path("mat-4.cfmtx") == "mat-4.mtx"
    assert sc.companion_mtx_path("-4.cfmtx") == "-4.mtx"
    assert sc.companion_mtx_path(".cfmtx") == ".cfmtx"


def _cf_text(rpp_line="0 1 1", cb_line="2", vals_line="1.5"):
    # 4x4 matrix, kernel_m 2, one pattern "11"... plus the other two patterns empty
    return ("4 4 2 3 1\n11 0 \n10 1 \n01 2 \n"
            f"{rpp_line}\n{cb_line}\n{' '.join([vals_line, vals_line])}\n"
            "0 0 0\n\n\n0 0 0\n\n\n")


@pytest.mark.parametrize("text,what", [
    (_cf_text(cb_line="9"), "column index out of range"),
    (_cf_text(rpp_line="0 1"), "row-panel pointer length"),
    (_cf_text(rpp_line="1 1 1"), "must start at 0"),
    (_cf_text(rpp_line="0 2 1", cb_line="1 2"), "non-decreasing"),
    (_cf_text(rpp_line="0 1 3", cb_line="1 2"), "exceeds column list"),
    (_cf_text(vals_line="1.5").replace("1.5 1.5", "1.5"), "shorter than columns"),
])
def test_plan_validates_cf_on_host(tmp_path, text, what):
    """Corrupt .cfmtx content is rejected before anything reaches a GPU
    (SC_ERR_FORMAT), whether or not a GPU is present."""
    f = tmp_path / "bad-2-1.cfmtx"
    f.write_text(text)
    cf = sc.read_cfmtx(f)  # the loader is as lenient as the reference's
    with pytest.raises(sc.ScError) as e:
        sc.SpMMPlan(cf, 32)
    assert e.value.code == sc.SC_ERR_FORMAT and what in str(e.value)


def test_valid_small_cf_reaches_device_step(tmp_path):
    f = tmp_path / "ok-2-1.cfmtx"
    f.write_text(_cf_text())
    cf = sc.read_cfmtx(f)
    import torch
    if torch.cuda.is_available():
        pytest.skip("GPU present: covered by the GPU tests")
    with pytest.raises(sc.ScError) as e:
        sc.SpMMPlan(cf, 32)
    assert e.value.code == sc.SC_ERR_CUDA
