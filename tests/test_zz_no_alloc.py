"""The allocation-free entry point sc_spmm_dense_noalloc, called through the C
ABI.  It exists for callers that cannot allocate device memory on their hot
path (their memory belongs to their own pool or budget); it keeps all its
scratch in one fixed array inside the library.  Two calls in a row must match
the existing plan-based entry point (sc_spmm) on the same matrix.

This file is named to be collected last, so that a run stopping at its first
failure has already run every other test; it also passes on its own in a
fresh process.
"""
import ctypes

import numpy as np
import pytest

import sparse_computation_b200 as sc
from oracle import cpu
from parity import RTOL, to_csr_handle
from sparse_computation_b200 import workloads as wl

pytestmark = pytest.mark.gpu


def _call_noalloc(A, B, C, accumulate=0):
    import torch
    m, k = A.shape
    n = B.shape[1]
    st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    return sc.lib().sc_spmm_dense_noalloc(
        ctypes.c_void_p(A.data_ptr()), A.stride(0), m, k, ctypes.c_void_p(B.data_ptr()), B.stride(0), n,
        ctypes.c_void_p(C.data_ptr()), C.stride(0), accumulate, st)


def test_noalloc_matches_plan_entry_point_twice(cuda):
    import torch
    name, a, B1 = wl.config4(128)[4]  # a 2048 x 512 FFN weight, 80% pruned
    m, k, ip, ix, dx = a
    Ad = np.zeros((m, k), np.float32)
    for r in range(m):
        Ad[r, ix[ip[r]:ip[r + 1]]] = dx[ip[r]:ip[r + 1]]
    A = torch.from_numpy(Ad).to(cuda)
    plan = sc.SpMMPlan(sc.csr_to_compressed_format_converter(to_csr_handle(a), 4, 1), 128)
    for B_np in (B1, wl.dense_b(k, 128, 77)):  # two calls in a row, different B
        B = torch.from_numpy(B_np).to(cuda)
        C_new = torch.full((m, 128), float("nan"), device=cuda)
        assert _call_noalloc(A, B, C_new) == sc.SC_OK, sc.lib().sc_last_error_string()
        C_old = plan.spmm(B)
        torch.cuda.synchronize()
        new, old = C_new.cpu().numpy().astype(np.float64), C_old.cpu().numpy().astype(np.float64)
        scale = cpu.spmm_csr_abs(ip, ix, dx, B_np)
        ref = cpu.spmm_csr_float(ip, ix, dx, B_np)
        # each within the fp32 tolerance of the CPU oracle, hence within twice it of each other
        assert np.all(np.abs(new - ref) <= RTOL * scale)
        assert np.all(np.abs(new - old) <= 2 * RTOL * scale)


def test_noalloc_rejects_oversized_inputs(cuda):
    import torch
    A = torch.zeros((4096, 4096), device=cuda)  # 128 MiB of tile images > the 16 MiB scratch
    B = torch.zeros((4096, 128), device=cuda)
    C = torch.zeros((4096, 128), device=cuda)
    assert _call_noalloc(A, B, C) == sc.SC_ERR_ARG
    assert b"scratch" in sc.lib().sc_last_error_string()
    B2 = torch.zeros((4096, 100), device=cuda)
    C2 = torch.zeros((4096, 100), device=cuda)
    assert _call_noalloc(A[:128, :64], B2[:64], C2[:128]) == sc.SC_ERR_UNSUPPORTED


def test_noalloc_ragged_strided_and_accumulate(cuda):
    """Shapes that are not multiples of the tiles (m % 128, k % 32), a leading
    dimension wider than k, then C += A*B on the same C: each call checked
    against the CPU oracle at the fp32 bound, and the status word stays 0."""
    import torch
    rng = np.random.default_rng(11)
    m, k, lda, n = 200, 100, 104, 128
    Ad = np.where(rng.random((m, k)) < 0.3, rng.normal(0, 0.05, (m, k)), 0).astype(np.float32)
    a = wl.csr_from_dense(Ad)
    _, _, ip, ix, dx = a
    Apad = np.full((m, lda), np.nan, np.float32)  # the columns past k must never be read
    Apad[:, :k] = Ad
    A = torch.from_numpy(Apad).to(cuda)[:, :k]
    assert A.stride(0) == lda
    B_np = wl.dense_b(k, n, 12)
    B = torch.from_numpy(B_np).to(cuda)
    C = torch.full((m, n), float("nan"), device=cuda)
    assert _call_noalloc(A, B, C, 0) == sc.SC_OK, sc.lib().sc_last_error_string()
    first = C.cpu().numpy()
    assert sc.noalloc_status() == 0
    ref = cpu.spmm_csr_float(ip, ix, dx, B_np)
    scale = cpu.spmm_csr_abs(ip, ix, dx, B_np)
    assert np.all(np.abs(first.astype(np.float64) - ref) <= RTOL * scale)
    assert _call_noalloc(A, B, C, 1) == sc.SC_OK, sc.lib().sc_last_error_string()
    second = C.cpu().numpy()
    assert sc.noalloc_status() == 0
    ref2 = cpu.spmm_csr_float(ip, ix, dx, B_np, first.copy())
    scale2 = scale + np.abs(first.astype(np.float64))
    assert np.all(np.abs(second.astype(np.float64) - ref2) <= RTOL * scale2)
