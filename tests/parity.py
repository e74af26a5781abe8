"""Shared parity helpers: run the CUDA path through the library and compare
with the CPU oracle under the stated fp32 tolerance."""
import numpy as np

import sparse_computation_b200 as sc
from oracle import cpu

# |C_gpu - C_ref| <= RTOL * sum_k |A_ik * B_kj|   (fp32 path; stated in BASELINE.json)
RTOL = 1e-5


def to_csr_handle(a):
    m, n, ip, ix, dx = a
    return sc.CSR.from_arrays(m, n, ip, ix, dx)


def assert_parity(C, a, B, C0=None, rows=None):
    """C: GPU result (numpy); a: CSR arrays; B: dense; C0: initial C for
    accumulate; rows: optional row subset (indices) that C holds."""
    m, n, ip, ix, dx = a
    if rows is not None:
        sub_ip = np.concatenate([[0], np.cumsum(ip[rows + 1] - ip[rows])]).astype(np.int32)
        sel = np.concatenate([np.arange(ip[r], ip[r + 1]) for r in rows]) if len(rows) else np.zeros(0, int)
        ip, ix, dx = sub_ip, ix[sel], dx[sel]
    B2 = B if B.ndim == 2 else B[:, None]
    ref = cpu.spmm_csr_float(ip, ix, dx, B2, None if C0 is None else np.array(C0, np.float32).reshape(-1, B2.shape[1]).copy())
    scale = cpu.spmm_csr_abs(ip, ix, dx, B2)
    if C0 is not None:
        scale = scale + np.abs(np.asarray(C0, np.float64)).reshape(scale.shape)
    C = np.asarray(C).reshape(ref.shape)
    err = np.abs(C.astype(np.float64) - ref.astype(np.float64))
    bad = err > RTOL * scale
    assert not np.isnan(C).any()
    assert not bad.any(), (f"{bad.sum()} of {bad.size} entries outside tolerance; "
                           f"max err {err.max():.3e}, at scale {scale[np.unravel_index(err.argmax(), err.shape)]:.3e}")
