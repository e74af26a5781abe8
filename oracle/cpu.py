"""TEST INFRASTRUCTURE ONLY -- ctypes access to the CPU oracle (liboracle.so,
built from oracle/spmm_ref.c) and to the reference's own CPU code built into
oracle/_ref/ (when present).  Used by tests/, __graft_entry__.smoke() and
bench.py's CPU-baseline leg only."""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIBORACLE = os.path.join(HERE, "liboracle.so")
REF_DIR = os.path.join(HERE, "_ref")

_P = ctypes.c_void_p


REF_SOURCE_FILE = os.path.join(REF_DIR, "source_dir.txt")


def reference_dir() -> str:
    """The reference checkout: SC_REFERENCE_DIR, else the one the last build
    compiled oracle/_ref from ("" when neither exists)."""
    d = os.environ.get("SC_REFERENCE_DIR", "")
    if not d and os.path.exists(REF_SOURCE_FILE):
        d = open(REF_SOURCE_FILE).read().strip()
    return d if d and os.path.isdir(d) else ""


def build(ref_dir: str = "") -> None:
    """Runs the oracle Makefile; the _ref targets only when a reference
    checkout is given (argument or SC_REFERENCE_DIR), whose location is then
    recorded for the tests that read the reference's fixtures."""
    ref = ref_dir or os.environ.get("SC_REFERENCE_DIR", "")
    cmd = ["make", "-s", "-j4", "-C", HERE]
    if ref and os.path.isdir(ref):
        cmd.append(f"REF={ref}")
    subprocess.run(cmd, check=True)
    if ref and os.path.isdir(ref):
        os.makedirs(REF_DIR, exist_ok=True)
        with open(REF_SOURCE_FILE, "w") as f:
            f.write(os.path.abspath(ref) + "\n")


def _load(path, sigs):
    L = ctypes.CDLL(path)
    for name, (args, res) in sigs.items():
        f = getattr(L, name)
        f.argtypes = args
        f.restype = res
    return L


_oracle = None


def oracle():
    global _oracle
    if _oracle is None:
        if not os.path.exists(LIBORACLE):
            build()
        i = ctypes.c_int
        _oracle = _load(LIBORACLE, {
            "oracle_spmm_csr_float": ([i, i, _P, _P, _P, _P, _P], None),
            "oracle_spmv_csr_float": ([i, _P, _P, _P, _P, _P], None),
            "oracle_spmm_csr_abs": ([i, i, _P, _P, _P, _P, _P], None),
            "oracle_spmm_csr_double": ([i, i, _P, _P, _P, _P, _P], None),
            "oracle_spmm_csr_float_threads": ([i, i, i, _P, _P, _P, _P, _P], ctypes.c_int),
        })
    return _oracle


def _ptr(a):
    return ctypes.c_void_p(a.ctypes.data)


def _csr32(indptr, indices, data):
    return (np.ascontiguousarray(indptr, np.int32), np.ascontiguousarray(indices, np.int32),
            np.ascontiguousarray(data, np.float32))


def spmm_csr_float(indptr, indices, data, B, C=None, nthreads=1):
    """C += A*B with the reference's float accumulation (restatement)."""
    ip, ix, dx = _csr32(indptr, indices, data)
    B = np.ascontiguousarray(B, np.float32)
    m = len(ip) - 1
    n = B.shape[1]
    if C is None:
        C = np.zeros((m, n), np.float32)
    if nthreads > 1:
        oracle().oracle_spmm_csr_float_threads(nthreads, m, n, _ptr(ip), _ptr(ix), _ptr(dx), _ptr(B), _ptr(C))
    else:
        oracle().oracle_spmm_csr_float(m, n, _ptr(ip), _ptr(ix), _ptr(dx), _ptr(B), _ptr(C))
    return C


def spmv_csr_float(indptr, indices, data, x, y=None):
    ip, ix, dx = _csr32(indptr, indices, data)
    x = np.ascontiguousarray(x, np.float32)
    m = len(ip) - 1
    if y is None:
        y = np.zeros(m, np.float32)
    oracle().oracle_spmv_csr_float(m, _ptr(ip), _ptr(ix), _ptr(dx), _ptr(x), _ptr(y))
    return y


def spmm_csr_abs(indptr, indices, data, B):
    """sum_k |A_ik * B_kj| in float64: the scale of the parity tolerance."""
    ip, ix, dx = _csr32(indptr, indices, data)
    B = np.ascontiguousarray(B, np.float32)
    C = np.zeros((len(ip) - 1, B.shape[1]), np.float64)
    oracle().oracle_spmm_csr_abs(len(ip) - 1, B.shape[1], _ptr(ip), _ptr(ix), _ptr(dx), _ptr(B), _ptr(C))
    return C


def spmm_csr_double(indptr, indices, data, B):
    ip, ix, dx = _csr32(indptr, indices, data)
    B = np.ascontiguousarray(B, np.float32)
    C = np.zeros((len(ip) - 1, B.shape[1]), np.float64)
    oracle().oracle_spmm_csr_double(len(ip) - 1, B.shape[1], _ptr(ip), _ptr(ix), _ptr(dx), _ptr(B), _ptr(C))
    return C


def round_values_f16(data):
    """float32 values rounded to IEEE binary16 (round to nearest even, subnormals
    kept) and back: what a 16-bit value record stores.  Models the reference's
    half-precision value arrays (example_cuda/spmm_small_b_col_demo_gpu_utils.h:2987-5168)."""
    return np.asarray(data, np.float32).astype(np.float16).astype(np.float32)


def round_values_bf16(data):
    """float32 values rounded to bfloat16 (round to nearest even on the 16 dropped
    mantissa bits; finite inputs) and back."""
    u = np.ascontiguousarray(data, np.float32).view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000
    return u.astype(np.uint32).view(np.float32)


# ---------------------------------------------- the reference's own code --

def ref_available(name="libref_spmm.so") -> bool:
    return os.path.exists(os.path.join(REF_DIR, name))


_refs = {}


def ref_lib(name):
    if name not in _refs:
        i = ctypes.c_int
        path = os.path.join(REF_DIR, name)
        if name == "libref_spmm.so":
            sigs = {"ref_spmm_csr_float": ([i, i, _P, _P, _P, _P, _P], None)}
        elif name == "libref_spmv.so":
            sigs = {"ref_spmv_csr_float": ([i, _P, _P, _P, _P, _P], None)}
        elif name == "libref_gpu_spmm.so":
            sigs = {"ref_gpu_spmm_create": ([ctypes.c_char_p, _P, i], _P), "ref_gpu_spmm_zero": ([_P, _P], i),
                    "ref_gpu_spmm_run": ([_P, _P], i), "ref_gpu_spmm_result": ([_P, _P], i),
                    "ref_gpu_spmm_free": ([_P], None)}
        elif name == "libref_gpu_spmv.so":
            sigs = {"ref_gpu_spmv_create": ([ctypes.c_char_p, _P], _P), "ref_gpu_spmv_zero": ([_P, _P], i),
                    "ref_gpu_spmv_run": ([_P, _P], i), "ref_gpu_spmv_result": ([_P, _P], i),
                    "ref_gpu_spmv_free": ([_P], None)}
        else:
            P64 = ctypes.POINTER(ctypes.c_int64)
            PP = ctypes.POINTER(ctypes.c_void_p)
            sigs = {
                "ref_cf_load": ([ctypes.c_char_p], _P),
                "ref_cf_num_patterns": ([_P], i),
                "ref_cf_pattern": ([_P, i, P64, P64, P64, P64, P64, PP, PP, PP, PP], None),
                "ref_csr_load_mtx": ([ctypes.c_char_p], _P),
                "ref_csr_arrays": ([_P, P64, P64, P64, PP, PP, PP], None),
            }
        _refs[name] = _load(path, sigs)
    return _refs[name]


def ref_spmm_csr_float(indptr, indices, data, B, C=None, row_begin=0, row_end=None):
    """The reference's spmm_csr_float on rows [row_begin, row_end) (C += A*B)."""
    ip, ix, dx = _csr32(indptr, indices, data)
    B = np.ascontiguousarray(B, np.float32)
    m = len(ip) - 1
    n = B.shape[1]
    if C is None:
        C = np.zeros((m, n), np.float32)
    row_end = m if row_end is None else row_end
    L = ref_lib("libref_spmm.so")
    L.ref_spmm_csr_float(row_end - row_begin, n, ctypes.c_void_p(ip.ctypes.data + 4 * row_begin),
                         _ptr(ix), _ptr(dx), _ptr(B), ctypes.c_void_p(C.ctypes.data + 4 * n * row_begin))
    return C


def ref_spmv_csr_float(indptr, indices, data, x, y=None):
    ip, ix, dx = _csr32(indptr, indices, data)
    x = np.ascontiguousarray(x, np.float32)
    if y is None:
        y = np.zeros(len(ip) - 1, np.float32)
    ref_lib("libref_spmv.so").ref_spmv_csr_float(len(ip) - 1, _ptr(ip), _ptr(ix), _ptr(dx), _ptr(x), _ptr(y))
    return y


def ref_read_cfmtx(path):
    """The reference loader's view of a .cfmtx: per pattern (km, kn, RPP, NPP, CB, NNZ)."""
    L = ref_lib("libref_io.so")
    h = L.ref_cf_load(os.fsencode(path))
    if not h:
        raise RuntimeError("reference loader returned nullptr")
    out = []
    for i in range(L.ref_cf_num_patterns(h)):
        km, kn, nrpp, ncb, nnz = (ctypes.c_int64() for _ in range(5))
        rpp, npp, cb, vals = (ctypes.c_void_p() for _ in range(4))
        L.ref_cf_pattern(h, i, *(ctypes.byref(x) for x in (km, kn, nrpp, ncb, nnz, rpp, npp, cb, vals)))

        def arr(p, ct, n, dt):
            if n == 0 or not p.value:
                return np.zeros(0, dt)
            return np.ctypeslib.as_array(ctypes.cast(p, ctypes.POINTER(ct)), (n,)).copy()

        out.append((km.value, kn.value, arr(rpp, ctypes.c_int, nrpp.value, np.int32),
                    arr(npp, ctypes.c_int, nrpp.value, np.int32), arr(cb, ctypes.c_int, ncb.value, np.int32),
                    arr(vals, ctypes.c_float, nnz.value, np.float32)))
    return out


def ref_read_csr(cfmtx_path):
    """The reference's CSR of the companion .mtx: (m, n, indptr, indices, data float64)."""
    L = ref_lib("libref_io.so")
    h = L.ref_csr_load_mtx(os.fsencode(cfmtx_path))
    m, n, z = ctypes.c_int64(), ctypes.c_int64(), ctypes.c_int64()
    p, i, x = ctypes.c_void_p(), ctypes.c_void_p(), ctypes.c_void_p()
    L.ref_csr_arrays(h, *(ctypes.byref(a) for a in (m, n, z, p, i, x)))
    ip = np.ctypeslib.as_array(ctypes.cast(p, ctypes.POINTER(ctypes.c_int)), (m.value + 1,)).copy()
    ix = np.ctypeslib.as_array(ctypes.cast(i, ctypes.POINTER(ctypes.c_int)), (z.value,)).copy()
    vx = np.ctypeslib.as_array(ctypes.cast(x, ctypes.POINTER(ctypes.c_double)), (z.value,)).copy()
    return m.value, n.value, ip, ix, vx
