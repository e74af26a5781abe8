"""Device-side failure detection, exercised without faulting the GPU: every
wait inside a kernel here is bounded, and on expiry the kernel writes an error
status that the host reads back.  The tests make a wait run out on purpose (a
flag that nothing publishes; a dense-tile producer that issues no copies) and
check that the status arrives, that the synchronous entry point reports
SC_ERR_DEVICE instead of SC_OK, and that the context stays usable afterwards.
The reference checks launch errors only (example_cuda/spmm_demo_gpu_utils.h:16-23)."""
import time

import numpy as np
import pytest

import sparse_computation_b200 as sc
from parity import assert_parity, to_csr_handle
from sparse_computation_b200 import workloads as wl

pytestmark = pytest.mark.gpu


def _small_product_ok(cuda):
    import torch
    a, B = wl.config1()
    plan = sc.SpMMPlan(sc.csr_to_compressed_format_converter(to_csr_handle(a), 2, 4), 32)
    C = plan.spmm(torch.from_numpy(B).to(cuda))
    torch.cuda.synchronize()
    assert_parity(C.cpu().numpy(), a, B)


def test_flag_wait_expires_with_status_5(cuda):
    """sc_wait_flags on an epoch no rank publishes: the bounded acquire loop
    gives up and writes 5 into the status word."""
    import torch
    flags = torch.zeros(2, dtype=torch.int32, device=cuda)
    flags[0] = 7  # one flag already at the epoch, the other never reaches it
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    stream = torch.cuda.current_stream(cuda)
    t0 = time.perf_counter()
    sc.wait_flags(flags.data_ptr(), 2, 7, status.data_ptr(), stream)
    torch.cuda.synchronize()
    waited = time.perf_counter() - t0
    assert int(status.item()) == 5
    assert waited < 30.0
    # a published epoch passes without touching the status
    status.zero_()
    flags.fill_(8)
    sc.wait_flags(flags.data_ptr(), 2, 8, status.data_ptr(), stream)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    _small_product_ok(cuda)


def _dense_plan(flags):
    a, B = wl.config3((512, 2048), 128)
    cf = sc.csr_to_compressed_format_converter(to_csr_handle(a), 4, 1)
    plan = sc.SpMMPlan(cf, 128, flags=sc.SC_PLAN_DENSE_ON | flags)
    assert plan.info["kernel"] == 3
    return a, B, plan


def test_dense_status_clean_after_a_normal_product(cuda):
    import torch
    a, B, plan = _dense_plan(0)
    C = plan.spmm(torch.from_numpy(B).to(cuda))
    assert plan.status() == 0
    assert_parity(C.cpu().numpy(), a, B)
    Ch = plan.spmm_host(B)  # checks the status itself
    assert_parity(Ch, a, B)


def test_dense_wait_expiry_is_reported(cuda):
    """With the producer starved, the MMA issuer's bounded mbarrier wait
    expires: C stays untouched, the plan's status is non-zero once, and the
    host entry point returns SC_ERR_DEVICE rather than SC_OK."""
    import torch
    a, B, plan = _dense_plan(sc.SC_PLAN_TEST_STARVE)
    C = torch.full((plan.rows, 128), 123.0, device=cuda)
    plan.spmm(torch.from_numpy(B).to(cuda), C)
    st = plan.status()
    assert st in (2, 3), st
    assert plan.status() == 0  # read and cleared
    assert bool(torch.all(C == 123.0))  # no CTA stored a partial C
    with pytest.raises(sc.ScError) as ei:
        plan.spmm_host(B)
    assert ei.value.code == sc.SC_ERR_DEVICE
    assert plan.status() == 0
    # the context is still usable: a normal dense plan and a sparse product
    a2, B2, ok = _dense_plan(0)
    C2 = ok.spmm(torch.from_numpy(B2).to(cuda))
    assert ok.status() == 0
    assert_parity(C2.cpu().numpy(), a2, B2)
    _small_product_ok(cuda)


def test_staged_small_b_wait_expiry_is_reported(cuda):
    """Staged small-B kernel (SpMV of a large matrix) with its record copies
    starved: every warp's bounded mbarrier wait expires, C stays untouched,
    the status is 7 once, and the host entry point returns SC_ERR_DEVICE."""
    import torch
    from sparse_computation_b200.partition import row_slice
    a, B = wl.config5(n_cols_b=1)
    a = row_slice(a, 0, 4096)
    cf = sc.csr_to_compressed_format_converter(to_csr_handle(a), 4, 1)
    plan = sc.SpMMPlan(cf, 1, flags=sc.SC_PLAN_TEST_STARVE)
    C = torch.full((a[0], 1), 123.0, device=cuda)
    t0 = time.perf_counter()
    plan.spmm(torch.from_numpy(B).to(cuda), C)
    assert plan.status() == 7
    assert time.perf_counter() - t0 < 60.0
    assert plan.status() == 0
    assert bool(torch.all(C == 123.0))
    with pytest.raises(sc.ScError) as ei:
        plan.spmm_host(B)
    assert ei.value.code == sc.SC_ERR_DEVICE
    ok = sc.SpMMPlan(cf, 1)
    y = ok.spmm(torch.from_numpy(B).to(cuda))
    assert ok.status() == 0
    assert_parity(y.cpu().numpy(), a, B)
    _small_product_ok(cuda)


def test_batch_status_clean(cuda):
    import torch
    mats = wl.config4(128)[:4]
    plans, Bs, Cs = [], [], []
    for _, a, B in mats:
        cf = sc.csr_to_compressed_format_converter(to_csr_handle(a), 4, 1)
        p = sc.SpMMPlan(cf, 128, flags=sc.SC_PLAN_DENSE_ON)
        plans.append(p)
        Bs.append(torch.from_numpy(B).to(cuda))
        Cs.append(torch.empty((a[0], 128), device=cuda))
    bt = sc.SpMMBatch(plans)
    bt.bind(Bs, Cs)
    bt.spmm()
    assert bt.status() == 0
    for (_, a, B), C in zip(mats, Cs):
        assert_parity(C.cpu().numpy(), a, B)
