"""Opt-in bf16 mode of the dense-tile tensor-core kernel (SC_PLAN_DENSE_BF16).

A and B are rounded to bf16 (round to nearest even, 8-bit significand) and the
products accumulate in fp32 in tensor memory, so the stated bound is

    |C_gpu - C_ref| <= (2^-7 + RTOL) * sum_k |A_ik * B_kj|

(each operand carries a relative rounding error of at most 2^-8; their product
at most 2^-7 + 2^-16).  The reference computes in fp32 only; this mode is not
its default and never chosen without the flag.  Inputs whose values are exact
in bf16 must come out within the fp32 bound: that checks the tile layout
independently of the rounding.
"""
import numpy as np
import pytest

import sparse_computation_b200 as sc
from oracle import cpu
from parity import RTOL, assert_parity, to_csr_handle
from sparse_computation_b200 import workloads as wl

pytestmark = pytest.mark.gpu

BF16_RTOL = 2.0 ** -7 + RTOL
BF16 = sc.SC_PLAN_DENSE_BF16 | sc.SC_PLAN_DENSE_ON


def bf16_plan(a, n, km=4, flags=BF16):
    cf = sc.csr_to_compressed_format_converter(to_csr_handle(a), km, 1)
    plan = sc.SpMMPlan(cf, n, flags=flags)
    assert plan.info["kernel"] == 3 and plan.info["dense_bf16"] == 1, plan.info
    return plan


def check_bf16(C, a, B, C0=None):
    m, n, ip, ix, dx = a
    ref = cpu.spmm_csr_float(ip, ix, dx, B, None if C0 is None else np.array(C0, np.float32))
    scale = cpu.spmm_csr_abs(ip, ix, dx, B)
    if C0 is not None:
        scale = scale + np.abs(np.asarray(C0, np.float64))
    err = np.abs(C.astype(np.float64) - ref.astype(np.float64))
    assert not np.isnan(C).any()
    bad = err > BF16_RTOL * scale
    assert not bad.any(), f"{bad.sum()} entries outside the bf16 bound; max err {err.max():.3e}"
    return err, scale


def run(plan, B, C0=None, accumulate=False):
    import torch
    C = None if C0 is None else torch.from_numpy(np.array(C0, np.float32)).cuda()
    out = plan.spmm(torch.from_numpy(B).cuda(), C, accumulate=accumulate)
    torch.cuda.synchronize()
    return out.cpu().numpy()


def to_bf16_exact(x):
    """Rounds float32 values to ones that bf16 holds exactly (truncation)."""
    u = np.ascontiguousarray(x, np.float32).view(np.uint32) & np.uint32(0xFFFF0000)
    return u.view(np.float32)


@pytest.mark.parametrize("shape", [(2048, 512), (512, 2048)])
def test_bf16_config3_within_bound(cuda, shape):
    a, B = wl.config3(shape, 128)
    err, scale = check_bf16(run(bf16_plan(a, 128), B), a, B)
    # the rounding is really there (not an fp32 kernel under another name)
    assert (err > RTOL * scale).any()


def test_bf16_exact_operands_meet_fp32_bound(cuda):
    rng = np.random.default_rng(11)
    A = np.where(rng.random((384, 200)) < 0.3, to_bf16_exact(rng.normal(0, 1, (384, 200))), 0).astype(np.float32)
    a = wl.csr_from_dense(A)
    B = to_bf16_exact(wl.dense_b(200, 256, 12))
    assert_parity(run(bf16_plan(a, 256), B), a, B)


def test_bf16_ragged_zero_blocks_accumulate(cuda):
    rng = np.random.default_rng(5)
    A = np.where(rng.random((300, 77)) < 0.25, rng.normal(0, 1, (300, 77)), 0).astype(np.float32)
    A[128:256] = 0   # an all-zero row block
    A[:, 0:64] = 0   # an all-zero 64-wide K chunk
    a = wl.csr_from_dense(A)
    for km in (1, 3):
        B = wl.dense_b(77, 128, 6)
        C = run(bf16_plan(a, 128, km=km), B)
        check_bf16(C, a, B)
        assert np.all(C[128:256] == 0)
    C0 = wl.dense_b(300, 128, 7)
    check_bf16(run(bf16_plan(a, 128), B, C0=C0, accumulate=True), a, B, C0=C0)


def test_bf16_batch_and_mixed_precision_rejected(cuda):
    import torch
    mats = wl.config4(128)[:6]
    plans = [bf16_plan(a, 128) for _, a, _ in mats]
    batch = sc.SpMMBatch(plans)
    Bs = [torch.from_numpy(B).cuda() for _, _, B in mats]
    Cs = [torch.empty((p.rows, 128), device="cuda") for p in plans]
    batch.bind(Bs, Cs)
    batch.spmm()
    torch.cuda.synchronize()
    for (_, a, B), C in zip(mats, Cs):
        check_bf16(C.cpu().numpy(), a, B)
    tf32 = sc.SpMMPlan(sc.csr_to_compressed_format_converter(to_csr_handle(mats[0][1]), 4, 1), 128,
                       flags=sc.SC_PLAN_DENSE_ON)
    assert tf32.info["kernel"] == 3 and tf32.info["dense_bf16"] == 0
    with pytest.raises(sc.ScError):
        sc.SpMMBatch([plans[0], tf32])


def test_dense_off_flag_overrides_env(cuda, monkeypatch):
    monkeypatch.setenv("SC_DENSE", "1")
    a, B = wl.config3((2048, 512), 128)
    cf = sc.csr_to_compressed_format_converter(to_csr_handle(a), 4, 1)
    plan = sc.SpMMPlan(cf, 128, flags=sc.SC_PLAN_DENSE_OFF)
    assert plan.info["kernel"] == 2
    assert_parity(run(plan, B), a, B)
