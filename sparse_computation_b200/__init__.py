"""B200-native enumerate + sparse-coarsen SpMM/SpMV.

Python mirror of the reference's host interface for this path, over the C ABI
of ``libsc_b200.so`` (declared in ``include/sc_b200.h``):

=============================================  =====================================================
this module                                    reference (hosseinal/sparse-computation)
=============================================  =====================================================
``build_patterns_map(m, n)``                   code_gen/pattern_utiles/pattern_dictionary.py:29-37
``read_csr_from_mtx(path)``                    utils/Sparse_io.cpp:48-82 (readCSRMatrixFromMTX)
``csr_to_compressed_format_converter(...)``    code_gen/ss_format/format_generator.py:68-129
``format_writer(name, cf)``                    code_gen/ss_format/format_generator.py:132-160
``read_cfmtx(path)``                           utils/Sparse_io.cpp:84-181 (readCFMTXFile)
``load_cfmtx_matrices(path)``                  utils/Sparse_io.cpp:186-196 (loadCfmtxMatrices)
``companion_mtx_path(path)``                   utils/Sparse_io.cpp:28-46
``SpMMPlan(cf, n).spmm(B, C)``                 example_cuda/spmm_demo_gpu_utils.h:1357-1712 and
                                               spmm_small_b_col_demo_gpu_utils.h:4911-5064
``SpMMPlan(cf, 1).spmv(x, y)``                 example_cuda/spmv_demo_gpu_utils.h:632-952
=============================================  =====================================================

All numerical work runs in the CUDA kernels of ``libsc_b200.so``; there is no
CPU fallback.  Importing this module does not need a GPU (the host formats
and the coarsener are native C++ and run anywhere); creating a plan does.
"""
from __future__ import annotations

import ctypes
import os
from typing import Dict, Optional, Tuple

import numpy as np

_PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.environ.get("SC_LIB", os.path.join(_PKG, "libsc_b200.so"))

SC_OK = 0
SC_ERR_ARG = 1
SC_ERR_IO = 2
SC_ERR_FORMAT = 3
SC_ERR_CUDA = 4
SC_ERR_UNSUPPORTED = 5
SC_ERR_NOMEM = 6
SC_ERR_DEVICE = 7

# sc_plan_create_ex flags
SC_PLAN_DENSE_OFF = 1
SC_PLAN_DENSE_ON = 2
SC_PLAN_DENSE_BF16 = 4
SC_PLAN_VALUES_F16 = 8
SC_PLAN_VALUES_BF16 = 16
SC_PLAN_TEST_STARVE = 1 << 30  # test hook: dense-tile and staged small-B waits expire (error path tests)

# Every symbol include/sc_b200.h declares (checked by the CPU tests).
EXPORTED_SYMBOLS = (
    "sc_version", "sc_last_error_string",
    "sc_mtx_load_csr", "sc_csr_create", "sc_csr_dims", "sc_csr_arrays", "sc_csr_free",
    "sc_cf_load", "sc_cf_from_csr", "sc_cf_write", "sc_cf_dims", "sc_cf_header_line",
    "sc_cf_pattern_sizes", "sc_cf_pattern_arrays", "sc_cf_real_nnz", "sc_cf_free",
    "sc_companion_mtx_path", "sc_cf_write_binary", "sc_cf_load_binary",
    "sc_plan_create", "sc_plan_create_panels", "sc_plan_create_ex", "sc_plan_get_info", "sc_spmm", "sc_spmv",
    "sc_spmm_host", "sc_plan_free", "sc_spmm_peers", "sc_wait_flags",
    "sc_batch_create", "sc_batch_bind", "sc_batch_spmm", "sc_batch_free",
    "sc_spmm_dense_noalloc", "sc_noalloc_status", "sc_plan_status", "sc_batch_status",
    "sc_graph_capture_plan", "sc_graph_capture_batch", "sc_graph_launch", "sc_graph_free",
)


class ScError(RuntimeError):
    """A failed libsc_b200 call: ``code`` is the SC_ERR_* status."""

    def __init__(self, code: int, msg: str):
        super().__init__(f"[sc error {code}] {msg}")
        self.code = code


class _PlanInfo(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int64) for n in (
        "rows", "cols", "n_cols_b", "panels", "kernel_m", "nnz", "entries", "items",
        "device_bytes")] + [("kernel", ctypes.c_int32), ("warps_per_panel", ctypes.c_int32),
                        ("dense_bf16", ctypes.c_int32), ("value_type", ctypes.c_int32)]


_lib = None


def lib() -> ctypes.CDLL:
    """Loads libsc_b200.so, building it in-tree first (about a minute with
    nvcc, ``sparse_computation_b200.build``) when it is missing.  There is no
    fallback: without nvcc and without a built library this raises."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        from . import build as _build
        try:
            _build.build()
        except Exception as ex:
            raise ImportError(f"{LIB_PATH} is missing and could not be built: {ex}") from ex
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"{LIB_PATH} is missing after the build")
    L = ctypes.CDLL(LIB_PATH)
    P = ctypes.POINTER
    vp = ctypes.c_void_p
    i32, i64, cp = ctypes.c_int32, ctypes.c_int64, ctypes.c_char_p
    sig = {
        "sc_version": ([], ctypes.c_int),
        "sc_last_error_string": ([], cp),
        "sc_mtx_load_csr": ([cp, P(vp)], ctypes.c_int),
        "sc_csr_create": ([i32, i32, i64, vp, vp, vp, P(vp)], ctypes.c_int),
        "sc_csr_dims": ([vp, P(i32), P(i32), P(i64)], ctypes.c_int),
        "sc_csr_arrays": ([vp, P(vp), P(vp), P(vp)], ctypes.c_int),
        "sc_csr_free": ([vp], None),
        "sc_cf_load": ([cp, P(vp)], ctypes.c_int),
        "sc_cf_from_csr": ([vp, i32, i32, cp, i32, P(vp)], ctypes.c_int),
        "sc_cf_write": ([vp, cp], ctypes.c_int),
        "sc_cf_dims": ([vp, P(i32), P(i32), P(i32), P(i32), P(i32)], ctypes.c_int),
        "sc_cf_header_line": ([vp, i32, ctypes.c_char_p, i32, P(i32)], ctypes.c_int),
        "sc_cf_pattern_sizes": ([vp, i32, P(i32), P(i64), P(i64), P(i64)], ctypes.c_int),
        "sc_cf_pattern_arrays": ([vp, i32, P(vp), P(vp), P(vp)], ctypes.c_int),
        "sc_cf_real_nnz": ([vp, P(i64)], ctypes.c_int),
        "sc_cf_free": ([vp], None),
        "sc_companion_mtx_path": ([cp, ctypes.c_char_p, i32], ctypes.c_int),
        "sc_cf_write_binary": ([vp, cp], ctypes.c_int),
        "sc_cf_load_binary": ([cp, P(vp)], ctypes.c_int),
        "sc_plan_create": ([vp, i32, i32, P(vp)], ctypes.c_int),
        "sc_plan_create_panels": ([vp, i32, i32, i64, i64, P(vp)], ctypes.c_int),
        "sc_plan_create_ex": ([vp, i32, i32, i64, i64, ctypes.c_uint32, P(vp)], ctypes.c_int),
        "sc_plan_get_info": ([vp, P(_PlanInfo)], ctypes.c_int),
        "sc_spmm": ([vp, vp, i64, vp, i64, i32, vp], ctypes.c_int),
        "sc_spmv": ([vp, vp, vp, i32, vp], ctypes.c_int),
        "sc_spmm_peers": ([vp, vp, i64, vp, i64, vp, i32, vp, i32, i32, i32, vp], ctypes.c_int),
        "sc_wait_flags": ([vp, i32, i32, vp, vp], ctypes.c_int),
        "sc_spmm_host": ([vp, vp, vp, vp], ctypes.c_int),
        "sc_plan_free": ([vp], None),
        "sc_batch_create": ([vp, i32, P(vp)], ctypes.c_int),
        "sc_batch_bind": ([vp, vp, vp, vp, vp], ctypes.c_int),
        "sc_batch_spmm": ([vp, i32, vp], ctypes.c_int),
        "sc_batch_free": ([vp], None),
        "sc_graph_capture_plan": ([vp, vp, i64, vp, i64, i32, i32, P(vp)], ctypes.c_int),
        "sc_graph_capture_batch": ([vp, i32, i32, P(vp)], ctypes.c_int),
        "sc_graph_launch": ([vp, vp], ctypes.c_int),
        "sc_graph_free": ([vp], None),
        "sc_spmm_dense_noalloc": ([vp, i64, i64, i64, vp, i64, i64, vp, i64, i32, vp], ctypes.c_int),
        "sc_noalloc_status": ([P(i32)], ctypes.c_int),
        "sc_plan_status": ([vp, P(i32)], ctypes.c_int),
        "sc_batch_status": ([vp, P(i32)], ctypes.c_int),
    }
    for name, (args, res) in sig.items():
        f = getattr(L, name)
        f.argtypes = args
        f.restype = res
    _lib = L
    return L


def _check(status: int) -> None:
    if status != SC_OK:
        raise ScError(status, lib().sc_last_error_string().decode(errors="replace"))


def _enc(path) -> bytes:
    return os.fsencode(os.fspath(path))


# ------------------------------------------------------------ dictionary --

def build_patterns_map(kernel_m: int, kernel_n: int = 1) -> Dict[Tuple[bool, ...], int]:
    """All non-zero kernel masks: id ``i-1`` <-> the binary string of
    ``2**bits - i`` (bits = kernel_m*kernel_n), most significant bit = panel
    row 0.  Same mapping as pattern_dictionary.py:29-37."""
    bits = kernel_m * kernel_n
    out = {}
    for i in range(1, 2 ** bits):
        x = 2 ** bits - i
        out[tuple(c == "1" for c in format(x, f"0{bits}b"))] = i - 1
    return out


# ------------------------------------------------------------------- CSR --

class CSR:
    """Owned CSR matrix (int32 indices, float64 values)."""

    def __init__(self, handle: int):
        self._h = ctypes.c_void_p(handle)

    @classmethod
    def from_arrays(cls, m: int, n: int, indptr, indices, data) -> "CSR":
        indptr = np.ascontiguousarray(indptr, dtype=np.int32)
        indices = np.ascontiguousarray(indices, dtype=np.int32)
        data = np.ascontiguousarray(data, dtype=np.float64)
        h = ctypes.c_void_p()
        _check(lib().sc_csr_create(m, n, len(indices), indptr.ctypes.data, indices.ctypes.data,
                                   data.ctypes.data, ctypes.byref(h)))
        return cls(h.value)

    @classmethod
    def from_scipy(cls, a) -> "CSR":
        a = a.tocsr()
        a.sort_indices()
        return cls.from_arrays(a.shape[0], a.shape[1], a.indptr, a.indices, a.data)

    @property
    def shape(self) -> Tuple[int, int]:
        m, n, z = ctypes.c_int32(), ctypes.c_int32(), ctypes.c_int64()
        _check(lib().sc_csr_dims(self._h, ctypes.byref(m), ctypes.byref(n), ctypes.byref(z)))
        return m.value, n.value

    @property
    def nnz(self) -> int:
        z = ctypes.c_int64()
        _check(lib().sc_csr_dims(self._h, None, None, ctypes.byref(z)))
        return z.value

    def arrays(self) -> Tuple[np.ndarray, np.ndarray, np.ndarray]:
        """Copies of (indptr, indices, data)."""
        m, _ = self.shape
        z = self.nnz
        rp, ci, vx = ctypes.c_void_p(), ctypes.c_void_p(), ctypes.c_void_p()
        _check(lib().sc_csr_arrays(self._h, ctypes.byref(rp), ctypes.byref(ci), ctypes.byref(vx)))
        indptr = np.ctypeslib.as_array(ctypes.cast(rp, ctypes.POINTER(ctypes.c_int32)), (m + 1,)).copy()
        if z == 0:
            return indptr, np.zeros(0, np.int32), np.zeros(0, np.float64)
        indices = np.ctypeslib.as_array(ctypes.cast(ci, ctypes.POINTER(ctypes.c_int32)), (z,)).copy()
        data = np.ctypeslib.as_array(ctypes.cast(vx, ctypes.POINTER(ctypes.c_double)), (z,)).copy()
        return indptr, indices, data

    def __del__(self):
        if getattr(self, "_h", None) and self._h.value and _lib is not None:
            _lib.sc_csr_free(self._h)
            self._h = ctypes.c_void_p()


def read_csr_from_mtx(path) -> CSR:
    """Matrix-Market -> CSR (readCSRMatrixFromMTX, utils/Sparse_io.cpp:48-82)."""
    h = ctypes.c_void_p()
    _check(lib().sc_mtx_load_csr(_enc(path), ctypes.byref(h)))
    return CSR(h.value)


# -------------------------------------------------------------------- CF --

class CompressedFormat:
    """Pattern-compressed matrix: one (RPP, CB, values) block per pattern id
    (CompressedFormat<T> / MixedFormat<T>,
    include/compressed_format/CompressedFormat.h:88-279)."""

    def __init__(self, handle: int):
        self._h = ctypes.c_void_p(handle)
        r, c, km, np_, vl = (ctypes.c_int32() for _ in range(5))
        _check(lib().sc_cf_dims(self._h, ctypes.byref(r), ctypes.byref(c), ctypes.byref(km),
                                ctypes.byref(np_), ctypes.byref(vl)))
        self.num_row, self.num_col = r.value, c.value
        self.kernel_rows = km.value
        self.num_patterns = np_.value
        self.vector_length = vl.value

    @property
    def header(self):
        """[(mask string, id)] in file order."""
        out = []
        buf = ctypes.create_string_buffer(1024)
        pid = ctypes.c_int32()
        for i in range(self.num_patterns):
            _check(lib().sc_cf_header_line(self._h, i, buf, 1024, ctypes.byref(pid)))
            out.append((buf.value.decode(), pid.value))
        return out

    def pattern(self, pid: int):
        """(popcount, RPP, CB, values float32) of body block ``pid`` (copies)."""
        pc, nr, nc, nv = ctypes.c_int32(), ctypes.c_int64(), ctypes.c_int64(), ctypes.c_int64()
        _check(lib().sc_cf_pattern_sizes(self._h, pid, ctypes.byref(pc), ctypes.byref(nr),
                                         ctypes.byref(nc), ctypes.byref(nv)))
        a, b, c = ctypes.c_void_p(), ctypes.c_void_p(), ctypes.c_void_p()
        _check(lib().sc_cf_pattern_arrays(self._h, pid, ctypes.byref(a), ctypes.byref(b), ctypes.byref(c)))

        def arr(ptr, ctype, n, dt):
            if n == 0:
                return np.zeros(0, dt)
            return np.ctypeslib.as_array(ctypes.cast(ptr, ctypes.POINTER(ctype)), (n,)).copy()

        return (pc.value, arr(a, ctypes.c_int32, nr.value, np.int32), arr(b, ctypes.c_int32, nc.value, np.int32),
                arr(c, ctypes.c_float, nv.value, np.float32))

    @property
    def real_nnz(self) -> int:
        z = ctypes.c_int64()
        _check(lib().sc_cf_real_nnz(self._h, ctypes.byref(z)))
        return z.value

    def write(self, path) -> None:
        _check(lib().sc_cf_write(self._h, _enc(path)))

    def write_binary(self, path) -> None:
        """Binary sidecar (.cfbin): fast to load, same content."""
        _check(lib().sc_cf_write_binary(self._h, _enc(path)))

    def __del__(self):
        if getattr(self, "_h", None) and self._h.value and _lib is not None:
            _lib.sc_cf_free(self._h)
            self._h = ctypes.c_void_p()


def csr_to_compressed_format_converter(csr: CSR, kernel_m: int = 4, kernel_n: int = 4,
                                       pattern_dictionary: Optional[str] = None,
                                       nthreads: int = 0) -> CompressedFormat:
    """Enumerate + coarsen on the host, bit-exact with
    format_generator.py:68-129 (``row_panel_size`` = kernel_m,
    ``p_col_size`` = kernel_n; ``pattern_dictionary`` = a dictionary file as
    read by read_pattern_dictionary, or None for the default map)."""
    h = ctypes.c_void_p()
    d = None if pattern_dictionary in (None, "false") else _enc(pattern_dictionary)
    _check(lib().sc_cf_from_csr(csr._h, kernel_m, kernel_n, d, nthreads, ctypes.byref(h)))
    return CompressedFormat(h.value)


def format_writer(name, cf: CompressedFormat) -> None:
    """Writes ``cf`` as text .cfmtx (format_generator.py:132-160)."""
    cf.write(name)


def read_cfmtx(path) -> CompressedFormat:
    """Parses a .cfmtx (readCFMTXFile, utils/Sparse_io.cpp:84-181)."""
    h = ctypes.c_void_p()
    _check(lib().sc_cf_load(_enc(path), ctypes.byref(h)))
    return CompressedFormat(h.value)


def read_cfbin(path) -> CompressedFormat:
    """Loads a binary sidecar written by CompressedFormat.write_binary."""
    h = ctypes.c_void_p()
    _check(lib().sc_cf_load_binary(_enc(path), ctypes.byref(h)))
    return CompressedFormat(h.value)


def companion_mtx_path(cfmtx_path) -> str:
    buf = ctypes.create_string_buffer(4096)
    _check(lib().sc_companion_mtx_path(_enc(cfmtx_path), buf, 4096))
    return os.fsdecode(buf.value)


def load_cfmtx_matrices(cfmtx_path) -> Tuple[CSR, CompressedFormat]:
    """(companion CSR, CF) like loadCfmtxMatrices (utils/Sparse_io.cpp:186-196);
    raises instead of returning nullptr."""
    if not os.fspath(cfmtx_path).endswith(".cfmtx"):
        raise ScError(SC_ERR_ARG, f"load_cfmtx_matrices expects a .cfmtx path: {cfmtx_path}")
    cf = read_cfmtx(cfmtx_path)
    return read_csr_from_mtx(companion_mtx_path(cfmtx_path)), cf


# ------------------------------------------------------------------ plan --

def wait_flags(flags_ptr: int, n: int, epoch: int, status_ptr: int, stream) -> None:
    """Stream-ordered bounded wait until the n ints at device address
    flags_ptr have all reached `epoch` (sc_wait_flags)."""
    _check(lib().sc_wait_flags(ctypes.c_void_p(flags_ptr), n, int(epoch), ctypes.c_void_p(status_ptr),
                               ctypes.c_void_p(stream.cuda_stream)))


def noalloc_status() -> int:
    """sc_noalloc_status: error status of the last sc_spmm_dense_noalloc on
    the current device (waits for the device, then clears it)."""
    v = ctypes.c_int32()
    _check(lib().sc_noalloc_status(ctypes.byref(v)))
    return v.value


def _torch():
    import torch
    return torch


class SpMMPlan:
    """Device-resident CF matrix plus schedule for products with an N-column B.

    ``spmm(B, C=None, accumulate=False)`` computes C = A @ B (or C += A @ B)
    for float32 CUDA tensors B (K x N) and C (rows x N), row-major with unit
    column stride, on torch's current stream of the plan's device.
    ``flags`` (SC_PLAN_DENSE_OFF / _ON / _BF16) select the dense-tile kernel and
    its precision; SC_PLAN_VALUES_F16 / _BF16 store A's values in 16 bits for
    small-B / SpMV plans.  The 16-bit modes are opt-in, with looser error bounds.
    """

    def __init__(self, cf: CompressedFormat, n_cols_b: int, device: int = 0,
                 panel_range: Optional[Tuple[int, int]] = None, flags: int = 0):
        self.cf = cf
        h = ctypes.c_void_p()
        if flags:
            pb, pe = panel_range if panel_range is not None else (-1, -1)
            _check(lib().sc_plan_create_ex(cf._h, n_cols_b, device, pb, pe, flags, ctypes.byref(h)))
        elif panel_range is None:
            _check(lib().sc_plan_create(cf._h, n_cols_b, device, ctypes.byref(h)))
        else:
            _check(lib().sc_plan_create_panels(cf._h, n_cols_b, device, panel_range[0], panel_range[1],
                                               ctypes.byref(h)))
        self._h = h
        self.device = device
        info = _PlanInfo()
        _check(lib().sc_plan_get_info(self._h, ctypes.byref(info)))
        self.info = {f: getattr(info, f) for f, _ in _PlanInfo._fields_}
        self.rows = info.rows
        self.cols = info.cols
        self.n = info.n_cols_b

    def _stream(self, stream):
        torch = _torch()
        s = stream if stream is not None else torch.cuda.current_stream(self.device)
        return ctypes.c_void_p(s.cuda_stream)

    def spmm(self, B, C=None, accumulate: bool = False, stream=None):
        torch = _torch()
        if B.dtype != torch.float32 or not B.is_cuda or B.dim() != 2 or B.stride(1) != 1:
            raise ScError(SC_ERR_ARG, "B must be a 2-D float32 CUDA tensor with unit column stride")
        if B.shape[0] != self.cols or B.shape[1] != self.n:
            raise ScError(SC_ERR_ARG, f"B must be {self.cols} x {self.n}, got {tuple(B.shape)}")
        if C is None:
            if accumulate:
                raise ScError(SC_ERR_ARG, "accumulate needs an output tensor")
            C = torch.empty((self.rows, self.n), dtype=torch.float32, device=B.device)
        if C.dtype != torch.float32 or not C.is_cuda or C.dim() != 2 or C.stride(1) != 1 or \
                tuple(C.shape) != (self.rows, self.n):
            raise ScError(SC_ERR_ARG, f"C must be a {self.rows} x {self.n} float32 CUDA tensor")
        _check(lib().sc_spmm(self._h, ctypes.c_void_p(B.data_ptr()), B.stride(0),
                             ctypes.c_void_p(C.data_ptr()), C.stride(0), 1 if accumulate else 0,
                             self._stream(stream)))
        return C

    def spmm_peers(self, B, C, peer_ptrs, accumulate: bool = False, stream=None, flag_ptrs=(), epoch=0):
        """spmm() that also stores C into peer GPUs' buffers (device addresses
        `peer_ptrs`, each pointing at the same first row as C); with
        `flag_ptrs`, the last CTA then stores `epoch` into each flag address
        (see wait_flags)."""
        torch = _torch()
        if B.dtype != torch.float32 or C.dtype != torch.float32 or B.stride(1) != 1 or C.stride(1) != 1:
            raise ScError(SC_ERR_ARG, "B and C must be float32 with unit column stride")
        if tuple(B.shape) != (self.cols, self.n) or tuple(C.shape) != (self.rows, self.n):
            raise ScError(SC_ERR_ARG, "operand shapes do not match the plan")
        arr = (ctypes.c_void_p * max(1, len(peer_ptrs)))(*peer_ptrs)
        fl = (ctypes.c_void_p * max(1, len(flag_ptrs)))(*flag_ptrs)
        _check(lib().sc_spmm_peers(self._h, ctypes.c_void_p(B.data_ptr()), B.stride(0),
                                   ctypes.c_void_p(C.data_ptr()), C.stride(0), arr, len(peer_ptrs), fl,
                                   len(flag_ptrs), int(epoch), 1 if accumulate else 0, self._stream(stream)))
        return C

    def capture(self, B, C, repeat: int = 1, accumulate: bool = False) -> "Graph":
        """CUDA graph of `repeat` products C = A @ B with these fixed tensors."""
        h = ctypes.c_void_p()
        _check(lib().sc_graph_capture_plan(self._h, ctypes.c_void_p(B.data_ptr()), B.stride(0),
                                           ctypes.c_void_p(C.data_ptr()), C.stride(0), 1 if accumulate else 0,
                                           repeat, ctypes.byref(h)))
        return Graph(h.value, self.device, keep=(self, B, C))

    def spmv(self, x, y=None, accumulate: bool = False, stream=None):
        torch = _torch()
        if x.dtype != torch.float32 or not x.is_cuda or x.numel() != self.cols or not x.is_contiguous():
            raise ScError(SC_ERR_ARG, f"x must be a contiguous float32 CUDA vector of length {self.cols}")
        if y is None:
            if accumulate:
                raise ScError(SC_ERR_ARG, "accumulate needs an output tensor")
            y = torch.empty(self.rows, dtype=torch.float32, device=x.device)
        if y.dtype != torch.float32 or not y.is_cuda or y.numel() != self.rows or not y.is_contiguous():
            raise ScError(SC_ERR_ARG, f"y must be a contiguous float32 CUDA vector of length {self.rows}")
        _check(lib().sc_spmv(self._h, ctypes.c_void_p(x.data_ptr()), ctypes.c_void_p(y.data_ptr()),
                             1 if accumulate else 0, self._stream(stream)))
        return y

    def spmm_host(self, B: np.ndarray, C: Optional[np.ndarray] = None, stream=None) -> np.ndarray:
        """C = A @ B from host arrays (copies in, kernel, copy out, synchronize)."""
        B = np.ascontiguousarray(B, dtype=np.float32)
        if B.shape != (self.cols, self.n):
            raise ScError(SC_ERR_ARG, f"B must be {self.cols} x {self.n}")
        if C is None:
            C = np.empty((self.rows, self.n), np.float32)
        s = self._stream(stream) if stream is not None else ctypes.c_void_p()
        _check(lib().sc_spmm_host(self._h, ctypes.c_void_p(B.ctypes.data), ctypes.c_void_p(C.ctypes.data), s))
        return C

    def status(self) -> int:
        """Device-side error status of this plan's kernels since the last
        call (waits for the device, then clears it): 0 = none; 1-3 = a
        bounded wait of the dense-tile kernel expired and C is incomplete."""
        v = ctypes.c_int32()
        _check(lib().sc_plan_status(self._h, ctypes.byref(v)))
        return v.value

    def check(self) -> None:
        """Raises ScError(SC_ERR_DEVICE) when status() is non-zero."""
        v = self.status()
        if v:
            raise ScError(SC_ERR_DEVICE, f"a bounded device wait expired (status {v}); C is incomplete")

    def __del__(self):
        if getattr(self, "_h", None) and self._h.value and _lib is not None:
            _lib.sc_plan_free(self._h)
            self._h = ctypes.c_void_p()


class SpMMBatch:
    """Several plans (same device, kernel_m and B width) computed by ONE
    kernel launch: ``bind(Bs, Cs)`` once, then ``spmm()`` per step."""

    def __init__(self, plans):
        self.plans = list(plans)
        arr = (ctypes.c_void_p * len(self.plans))(*[p._h.value for p in self.plans])
        h = ctypes.c_void_p()
        _check(lib().sc_batch_create(arr, len(self.plans), ctypes.byref(h)))
        self._h = h
        self._bound = None

    def bind(self, Bs, Cs):
        torch = _torch()
        n = len(self.plans)
        if len(Bs) != n or len(Cs) != n:
            raise ScError(SC_ERR_ARG, f"need {n} B and {n} C tensors")
        for p, B, C in zip(self.plans, Bs, Cs):
            if B.dtype != torch.float32 or C.dtype != torch.float32 or B.stride(1) != 1 or C.stride(1) != 1:
                raise ScError(SC_ERR_ARG, "B and C must be float32 with unit column stride")
            if tuple(B.shape) != (p.cols, p.n) or tuple(C.shape) != (p.rows, p.n):
                raise ScError(SC_ERR_ARG, "operand shapes do not match the plans")
        bp = (ctypes.c_void_p * n)(*[B.data_ptr() for B in Bs])
        cp = (ctypes.c_void_p * n)(*[C.data_ptr() for C in Cs])
        lb = (ctypes.c_int64 * n)(*[B.stride(0) for B in Bs])
        lc = (ctypes.c_int64 * n)(*[C.stride(0) for C in Cs])
        _check(lib().sc_batch_bind(self._h, bp, lb, cp, lc))
        self._bound = (list(Bs), list(Cs))  # keep the buffers alive

    def spmm(self, accumulate: bool = False, stream=None):
        torch = _torch()
        dev = self.plans[0].device
        s = stream if stream is not None else torch.cuda.current_stream(dev)
        _check(lib().sc_batch_spmm(self._h, 1 if accumulate else 0, ctypes.c_void_p(s.cuda_stream)))
        return self._bound[1] if self._bound else None

    def capture(self, repeat: int = 1, accumulate: bool = False) -> "Graph":
        """CUDA graph of `repeat` batch products with the bound operands."""
        h = ctypes.c_void_p()
        _check(lib().sc_graph_capture_batch(self._h, 1 if accumulate else 0, repeat, ctypes.byref(h)))
        return Graph(h.value, self.plans[0].device, keep=(self,))

    def status(self) -> int:
        """sc_batch_status: the dense-tile launch's error status (see SpMMPlan.status)."""
        v = ctypes.c_int32()
        _check(lib().sc_batch_status(self._h, ctypes.byref(v)))
        return v.value

    def __del__(self):
        if getattr(self, "_h", None) and self._h.value and _lib is not None:
            _lib.sc_batch_free(self._h)
            self._h = ctypes.c_void_p()


class Graph:
    """A captured CUDA graph of products (sc_graph); launch() replays it on a stream."""

    def __init__(self, handle: int, device: int, keep=()):
        self._h = ctypes.c_void_p(handle)
        self.device = device
        self._keep = keep  # the plan/batch and tensors the graph reads and writes

    def launch(self, stream=None):
        torch = _torch()
        s = stream if stream is not None else torch.cuda.current_stream(self.device)
        _check(lib().sc_graph_launch(self._h, ctypes.c_void_p(s.cuda_stream)))

    def __del__(self):
        if getattr(self, "_h", None) and self._h.value and _lib is not None:
            _lib.sc_graph_free(self._h)
            self._h = ctypes.c_void_p()
