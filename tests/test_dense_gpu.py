"""Dense-tile tensor-core path (tcgen05, 3xTF32 split, fp32 accumulation in
tensor memory) against the CPU oracle under the same fp32 tolerance as the
sparse kernels."""
import numpy as np
import pytest

import sparse_computation_b200 as sc
from parity import assert_parity, to_csr_handle
from sparse_computation_b200 import workloads as wl

pytestmark = pytest.mark.gpu


def run_dense(a, B, km=4, accumulate=False, C0=None):
    import torch
    cf = sc.csr_to_compressed_format_converter(to_csr_handle(a), km, 1)
    plan = sc.SpMMPlan(cf, B.shape[1])
    assert plan.info["kernel"] == 3, plan.info
    Bt = torch.from_numpy(B).cuda()
    C = None if C0 is None else torch.from_numpy(np.array(C0, np.float32)).cuda()
    out = plan.spmm(Bt, C, accumulate=accumulate)
    torch.cuda.synchronize()
    return out.cpu().numpy(), plan


@pytest.fixture
def force_dense(monkeypatch):
    monkeypatch.setenv("SC_DENSE", "1")


def test_dense_small(cuda, force_dense):
    a, _ = wl.config1()
    B = wl.dense_b(512, 128, 3)
    C, plan = run_dense(a, B)
    assert_parity(C, a, B)


@pytest.mark.parametrize("shape", [(2048, 512), (512, 2048)])
def test_dense_config3(cuda, force_dense, shape):
    a, B = wl.config3(shape, 128)
    C, _ = run_dense(a, B)
    assert_parity(C, a, B)


def test_dense_ragged_and_zero_blocks(cuda, force_dense):
    rng = np.random.default_rng(3)
    A = np.where(rng.random((300, 77)) < 0.2, rng.normal(0, 1, (300, 77)), 0).astype(np.float32)
    A[128:256] = 0  # an all-zero row block
    A[:, 32:64] = 0  # an all-zero K chunk
    a = wl.csr_from_dense(A)
    for N in (128, 256):
        B = wl.dense_b(77, N, 4)
        for km in (1, 3, 4):
            C, plan = run_dense(a, B, km=km)
            assert_parity(C, a, B)
            assert np.all(C[128:256] == 0)


def test_dense_accumulate(cuda, force_dense):
    a, B = wl.config3((2048, 512), 128)
    C0 = wl.dense_b(2048, 128, 9)
    C, _ = run_dense(a, B, accumulate=True, C0=C0)
    assert_parity(C, a, B, C0=C0)


def test_dense_repeat_and_default_selection(cuda, monkeypatch):
    monkeypatch.delenv("SC_DENSE", raising=False)
    a, B = wl.config4(128)[4][1:]  # an FFN weight, 80% sparse: chosen by default
    for _ in range(2):
        C, plan = run_dense(a, B)
        assert_parity(C, a, B)
    a5, _ = wl.config1()
    cf = sc.csr_to_compressed_format_converter(to_csr_handle(a5), 4, 1)
    assert sc.SpMMPlan(cf, 32).info["kernel"] == 2  # N not a multiple of 128
