"""16-bit value records for the small-B / SpMV kernel (SC_PLAN_VALUES_F16 and
SC_PLAN_VALUES_BF16): A's values stored as fp16 or bf16 with 16-bit column
indices, products and sums in fp32.

Two checks per case:
* against the CPU oracle run on A's values rounded the same way (numpy's
  IEEE binary16 conversion; a round-to-nearest-even bf16 restatement): the
  fp32 bound |dC| <= 1e-5 * sum|A||B| -- this pins the record layout exactly;
* against the oracle on the unrounded values: the stated looser bound,
  relative 2^-11 (fp16, plus 2^-25 absolute per value below 2^-14) or 2^-8
  (bf16) on top of the fp32 one.
"""
import numpy as np
import pytest

import sparse_computation_b200 as sc
from oracle import cpu
from parity import RTOL, assert_parity, to_csr_handle
from sparse_computation_b200 import workloads as wl

pytestmark = pytest.mark.gpu

MODES = {
    "f16": (sc.SC_PLAN_VALUES_F16, 1, cpu.round_values_f16, 2.0 ** -11, 2.0 ** -25),
    "bf16": (sc.SC_PLAN_VALUES_BF16, 2, cpu.round_values_bf16, 2.0 ** -8, 0.0),
}


def run16(a, B, km, kn, mode, C0=None):
    import torch
    flag, vt, _, _, _ = MODES[mode]
    cf = sc.csr_to_compressed_format_converter(to_csr_handle(a), km, kn)
    plan = sc.SpMMPlan(cf, B.shape[1], flags=flag)
    assert plan.info["kernel"] == 1 and plan.info["value_type"] == vt, plan.info
    C = None if C0 is None else torch.from_numpy(np.array(C0, np.float32)).cuda()
    out = plan.spmm(torch.from_numpy(B).cuda(), C, accumulate=C0 is not None)
    torch.cuda.synchronize()
    return out.cpu().numpy(), plan


def check16(C, a, B, mode, C0=None):
    m, n, ip, ix, dx = a
    _, _, rnd, rel, absv = MODES[mode]
    # exact layout: fp32 bound against the oracle on the rounded values
    assert_parity(C, (m, n, ip, ix, rnd(dx)), B, C0=C0)
    # stated bound against the unrounded values
    ref = cpu.spmm_csr_float(ip, ix, dx, B, None if C0 is None else np.array(C0, np.float32))
    scale = cpu.spmm_csr_abs(ip, ix, dx, B)
    bsum = cpu.spmm_csr_abs(ip, ix, np.ones_like(dx), B)
    if C0 is not None:
        scale = scale + np.abs(np.asarray(C0, np.float64))
    err = np.abs(C.astype(np.float64) - ref)
    assert np.all(err <= (rel + 2 * RTOL) * scale + absv * bsum)


@pytest.mark.parametrize("mode", ["f16", "bf16"])
@pytest.mark.parametrize("N", [1, 2, 4])
def test_config2_16bit_values(cuda, mode, N):
    for sparsity in (0.5, 0.9, 0.98):
        a, B = wl.config2(sparsity, N)
        for km, kn in ((1, 1), (2, 4), (3, 0), (4, 1), (5, 2), (6, 8)):
            C, plan = run16(a, B, km, kn, mode)
            check16(C, a, B, mode)


@pytest.mark.parametrize("mode", ["f16", "bf16"])
def test_16bit_spmv_accumulate_and_edges(cuda, mode):
    import torch
    a, _ = wl.config2(0.9, 1)
    m, n, ip, ix, dx = a
    x = wl.dense_b(512, 1, 6)
    y0 = wl.dense_b(512, 1, 8)
    C, _ = run16(a, x, 4, 1, mode, C0=y0)
    check16(C, a, x, mode, C0=y0)
    flag = MODES[mode][0]
    plan = sc.SpMMPlan(sc.csr_to_compressed_format_converter(to_csr_handle(a), 6, 1), 1, flags=flag)
    y = plan.spmv(torch.from_numpy(x[:, 0].copy()).cuda()).cpu().numpy()
    check16(y[:, None], a, x, mode)
    # ragged rows, empty rows, one column, zero-row matrix; columns up to K-1
    rng = np.random.default_rng(4)
    A = np.where(rng.random((301, 77)) < 0.2, rng.normal(0, 1, (301, 77)), 0).astype(np.float32)
    A[100:140] = 0
    A[:, 76] = 3.0
    for Ad in (A, np.zeros((7, 5), np.float32), np.eye(9, dtype=np.float32)):
        ae = wl.csr_from_dense(Ad)
        for km in (1, 3, 6):
            for N in (1, 4):
                B = wl.dense_b(Ad.shape[1], N, 3)
                C, _ = run16(ae, B, km, 1, mode)
                check16(C, ae, B, mode)


def test_16bit_values_smaller_records(cuda):
    a, B = wl.config2(0.5, 4)
    cf = sc.csr_to_compressed_format_converter(to_csr_handle(a), 4, 1)
    p32 = sc.SpMMPlan(cf, 4)
    p16 = sc.SpMMPlan(cf, 4, flags=sc.SC_PLAN_VALUES_F16)
    assert p16.info["entries"] == p32.info["entries"] and p16.info["nnz"] == p32.info["nnz"]
    # fp32 small-B plans use split item blocks (2 + 4P bytes per entry, below
    # the interleaved 8 bytes per nonzero); 16-bit records are smaller still
    assert p32.info["device_bytes"] < 8 * p32.info["nnz"]
    assert p16.info["device_bytes"] < 0.8 * p32.info["device_bytes"]


def test_16bit_values_rejections(cuda):
    a, _ = wl.config2(0.9, 4)
    cf = sc.csr_to_compressed_format_converter(to_csr_handle(a), 4, 1)
    with pytest.raises(sc.ScError) as e:   # wide B
        sc.SpMMPlan(cf, 32, flags=sc.SC_PLAN_VALUES_F16)
    assert e.value.code == sc.SC_ERR_UNSUPPORTED
    big = wl.csr_from_dense(np.array([[0, 70000.0, 0, 1]], np.float32))
    cfb = sc.csr_to_compressed_format_converter(to_csr_handle(big), 1, 1)
    with pytest.raises(sc.ScError) as e:   # beyond fp16 range
        sc.SpMMPlan(cfb, 1, flags=sc.SC_PLAN_VALUES_F16)
    assert e.value.code == sc.SC_ERR_UNSUPPORTED
    sc.SpMMPlan(cfb, 1, flags=sc.SC_PLAN_VALUES_BF16)  # bf16 has the range
    wide = sc.CSR.from_arrays(1, 70000, [0, 1], [69999], [1.0])
    cfw = sc.csr_to_compressed_format_converter(wide, 1, 1)
    with pytest.raises(sc.ScError) as e:   # columns beyond 16 bits
        sc.SpMMPlan(cfw, 1, flags=sc.SC_PLAN_VALUES_BF16)
    assert e.value.code == sc.SC_ERR_UNSUPPORTED
