"""Parity of the CUDA path (through the C ABI) with the CPU oracle
(restated spmm_csr_float / spmv_csr_float), under
|dC_ij| <= 1e-5 * sum_k |A_ik * B_kj|, on the benchmark configurations at
full size and on the golden fixtures written by the reference's converter."""
import glob
import os

import numpy as np
import pytest

import sparse_computation_b200 as sc
from oracle import cpu
from parity import RTOL, assert_parity, to_csr_handle
from sparse_computation_b200 import workloads as wl

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def run(cf, B, device, accumulate=False, C0=None):
    import torch
    plan = sc.SpMMPlan(cf, B.shape[1])
    Bt = torch.from_numpy(B).to(device)
    C = None if C0 is None else torch.from_numpy(np.array(C0, np.float32)).to(device)
    out = plan.spmm(Bt, C, accumulate=accumulate)
    torch.cuda.synchronize()
    return out.cpu().numpy(), plan


@pytest.mark.parametrize("case", ["cfg1small", "ragged", "widevals"])
@pytest.mark.parametrize("N", [1, 4, 32])
def test_golden_cfmtx_files(cuda, case, N):
    """.cfmtx written by the reference converter -> our kernels == C from the
    reference's own spmm_csr_float."""
    g = np.load(os.path.join(GOLDEN, f"spmm_{case}_n{N}.npz"))
    a_h = sc.read_csr_from_mtx(os.path.join(GOLDEN, case + ".mtx"))
    ip, ix, dx = a_h.arrays()
    a = (*a_h.shape, ip, ix, dx)
    for f in sorted(glob.glob(os.path.join(GOLDEN, f"{case}-*.cfmtx"))):
        cf = sc.read_cfmtx(f)
        if cf.kernel_rows > 6:
            continue
        C, _ = run(cf, g["B"], cuda)
        scale = cpu.spmm_csr_abs(ip, ix, dx, g["B"])
        assert np.all(np.abs(C.astype(np.float64) - g["C"]) <= RTOL * scale), f
        assert_parity(C, a, g["B"])


def test_config1(cuda):
    a, B = wl.config1()
    cf = sc.csr_to_compressed_format_converter(to_csr_handle(a), 2, 4)
    C, plan = run(cf, B, cuda)
    assert plan.info["nnz"] == len(a[3])
    assert_parity(C, a, B)


@pytest.mark.parametrize("sparsity", wl.CONFIG2_SPARSITIES)
@pytest.mark.parametrize("N", [1, 2, 4])
def test_config2_small_b(cuda, sparsity, N):
    a, B = wl.config2(sparsity, N)
    h = to_csr_handle(a)
    grid = [(m, n) for m in range(1, 7) for n in range(1, 9)] if sparsity == 0.9 else \
        [(1, 1), (2, 4), (4, 1), (6, 8), (3, 0)]
    for m, n in grid:
        cf = sc.csr_to_compressed_format_converter(h, m, n)
        C, plan = run(cf, B, cuda)
        assert plan.info["kernel"] == 1
        assert_parity(C, a, B)


@pytest.mark.parametrize("shape", [(2048, 512), (512, 2048)])
@pytest.mark.parametrize("N", [32, 64, 128])
def test_config3_large_b(cuda, shape, N):
    a, B = wl.config3(shape, N)
    h = to_csr_handle(a)
    for m in range(1, 7):
        cf = sc.csr_to_compressed_format_converter(h, m, 1)
        C, plan = run(cf, B, cuda)
        assert plan.info["kernel"] in (2, 3)  # 3: dense-tile tensor-core path (N = 128)
        assert_parity(C, a, B)


def test_config4_layer_stack(cuda):
    for name, a, B in wl.config4(128):
        cf = sc.csr_to_compressed_format_converter(to_csr_handle(a), 4, 1)
        C, _ = run(cf, B, cuda)
        assert_parity(C, a, B)


@pytest.mark.parametrize("N", [3, 5, 8, 16, 33, 96, 200, 256])
def test_odd_widths_and_strides(cuda, N):
    import torch
    a, _ = wl.config3((2048, 512), 32)
    B = wl.dense_b(512, N, 9)
    cf = sc.csr_to_compressed_format_converter(to_csr_handle(a), 4, 2)
    C, _ = run(cf, B, cuda)
    assert_parity(C, a, B)
    # leading dimensions larger than N (column slices of wider buffers)
    plan = sc.SpMMPlan(cf, N)
    Bw = torch.zeros((512, N + 7), device=cuda)
    Bw[:, :N] = torch.from_numpy(B).to(cuda)
    Cw = torch.full((2048, N + 3), 7.0, device=cuda)
    plan.spmm(Bw[:, :N], Cw[:, :N])
    torch.cuda.synchronize()
    assert_parity(Cw[:, :N].cpu().numpy(), a, B)
    assert torch.all(Cw[:, N:] == 7.0)


@pytest.mark.parametrize("N", [1, 4, 32, 128])
def test_accumulate(cuda, N):
    a, _ = wl.config2(0.8, 1)
    B = wl.dense_b(512, N, 4)
    C0 = wl.dense_b(512, N, 5)
    cf = sc.csr_to_compressed_format_converter(to_csr_handle(a), 4, 1)
    C, _ = run(cf, B, cuda, accumulate=True, C0=C0)
    assert_parity(C, a, B, C0=C0)


def test_spmv(cuda):
    import torch
    a, _ = wl.config2(0.9, 1)
    x = wl.dense_b(512, 1, 6)[:, 0].copy()
    m, n, ip, ix, dx = a
    for km in (1, 4, 6):
        cf = sc.csr_to_compressed_format_converter(to_csr_handle(a), km, 1)
        plan = sc.SpMMPlan(cf, 1)
        y = plan.spmv(torch.from_numpy(x).to(cuda)).cpu().numpy()
        ref = cpu.spmv_csr_float(ip, ix, dx, x)  # double accumulation (spmv_csr_float)
        scale = cpu.spmm_csr_abs(ip, ix, dx, x[:, None])[:, 0]
        assert np.all(np.abs(y.astype(np.float64) - ref) <= RTOL * scale)
        y0 = wl.dense_b(512, 1, 8)[:, 0]
        yt = torch.from_numpy(y0.copy()).to(cuda)
        plan.spmv(torch.from_numpy(x).to(cuda), yt, accumulate=True)
        assert np.all(np.abs(yt.cpu().numpy().astype(np.float64) - (ref + y0)) <= RTOL * (scale + np.abs(y0)))


def test_panel_range_plans_tile_the_matrix(cuda):
    import torch
    a, B = wl.config3((2048, 512), 64)
    cf = sc.csr_to_compressed_format_converter(to_csr_handle(a), 4, 1)
    panels = (2048 + 3) // 4
    cuts = [0, 100, 101, 333, panels]
    Bt = torch.from_numpy(B).to(cuda)
    C = torch.empty((2048, 64), device=cuda)
    for p0, p1 in zip(cuts[:-1], cuts[1:]):
        plan = sc.SpMMPlan(cf, 64, panel_range=(p0, p1))
        assert plan.rows == min(2048, p1 * 4) - p0 * 4
        plan.spmm(Bt, C[p0 * 4: p1 * 4])
    torch.cuda.synchronize()
    assert_parity(C.cpu().numpy(), a, B)


def test_host_entry_point(cuda):
    a, B = wl.config1()
    cf = sc.csr_to_compressed_format_converter(to_csr_handle(a), 2, 4)
    plan = sc.SpMMPlan(cf, 32)
    for _ in range(2):
        C = plan.spmm_host(B)
        assert_parity(C, a, B)


def test_host_entry_point_pinned_buffers(cuda):
    """Page-locked host buffers take the direct path (the kernel stores C into
    host memory; B copied as two concurrent halves); pageable ones the staged,
    row-chunked path.  Both match the oracle, and each other."""
    import torch
    a, B = wl.config3((2048, 512), 128)
    for km in (4, 1):
        cf = sc.csr_to_compressed_format_converter(to_csr_handle(a), km, 1)
        plan = sc.SpMMPlan(cf, 128)
        hB = torch.from_numpy(B).pin_memory()
        hC = torch.full((2048, 128), float("nan")).pin_memory()
        for _ in range(2):
            plan.spmm_host(hB.numpy(), hC.numpy())
            assert_parity(hC.numpy(), a, B)
        assert np.array_equal(plan.spmm_host(B), hC.numpy())
    # K >= 4096: the wide plan's K-split pipeline (half the columns per launch,
    # second launch stores C to the host); odd item cuts included
    a2 = wl.magnitude_pruned(1000, 6000, 0.95, 0.05, 77)
    B2 = wl.dense_b(6000, 64, 78)
    for km in (4, 3):
        plan = sc.SpMMPlan(sc.csr_to_compressed_format_converter(to_csr_handle(a2), km, 1), 64)
        hB = torch.from_numpy(B2).pin_memory()
        hC = torch.full((1000, 64), float("nan")).pin_memory()
        for _ in range(2):
            plan.spmm_host(hB.numpy(), hC.numpy())
            assert_parity(hC.numpy(), a2, B2)
        assert_parity(plan.spmm_host(B2), a2, B2)
    # a page-locked C that is only 4-byte aligned (narrower stores)
    buf = torch.empty(1000 * 64 + 1).pin_memory()
    hC = buf[1:].view(1000, 64)
    plan.spmm_host(torch.from_numpy(B2).pin_memory().numpy(), hC.numpy())
    assert_parity(hC.numpy(), a2, B2)
    a1, B1 = wl.config2(0.9, 4)  # small-B plan through the direct path
    plan = sc.SpMMPlan(sc.csr_to_compressed_format_converter(to_csr_handle(a1), 4, 1), 4)
    hC = torch.empty((512, 4)).pin_memory()
    plan.spmm_host(torch.from_numpy(B1).pin_memory().numpy(), hC.numpy())
    assert_parity(hC.numpy(), a1, B1)


def test_edge_matrices(cuda):
    import torch
    cases = [np.zeros((7, 5), np.float32), np.array([[0, 1.5, 0, 2]], np.float32), np.eye(9, dtype=np.float32),
             np.ones((13, 3), np.float32)]
    for A in cases:
        a = wl.csr_from_dense(A)
        for m, n in [(4, 1), (3, 2), (1, 3), (6, 0)]:
            cf = sc.csr_to_compressed_format_converter(to_csr_handle(a), m, n)
            for N in (1, 2, 4, 32, 40):
                B = wl.dense_b(A.shape[1], N, 3)
                C, _ = run(cf, B, cuda)
                assert_parity(C, a, B)
    # a matrix with zero rows gives an empty plan
    cf = sc.csr_to_compressed_format_converter(to_csr_handle(wl.csr_from_dense(np.zeros((0, 4), np.float32))), 4, 1)
    plan = sc.SpMMPlan(cf, 32)
    assert plan.rows == 0
    plan.spmm(torch.zeros((4, 32), device=cuda), torch.zeros((0, 32), device=cuda))


def test_deterministic(cuda):
    a, B = wl.config3((512, 2048), 128)
    cf = sc.csr_to_compressed_format_converter(to_csr_handle(a), 4, 1)
    C1, _ = run(cf, B, cuda)
    C2, _ = run(cf, B, cuda)
    assert np.array_equal(C1, C2)


def test_config5_full_size_parity(cuda):
    """16384^2 at 95% (the bench workload), every row against the oracle at
    the fp32 bound; then a 2-way panel split into one C must agree with it, and
    the product must be linear in B (within the bound of both terms)."""
    import os

    import torch
    a, B = wl.config5()
    m, _, ip, ix, dx = a
    cf = sc.csr_to_compressed_format_converter(to_csr_handle(a), 4, 1)
    plan = sc.SpMMPlan(cf, 128)
    Bt = torch.from_numpy(B).to(cuda)
    C = plan.spmm(Bt)
    ref = cpu.spmm_csr_float(ip, ix, dx, B, nthreads=os.cpu_count() or 1)
    scale = cpu.spmm_csr_abs(ip, ix, dx, B)
    got = C.cpu().numpy().astype(np.float64)
    assert np.all(np.abs(got - ref) <= RTOL * scale)
    half = (m // 4) // 2
    Cs = torch.full_like(C, float("nan"))
    for r in [(0, half), (half, m // 4)]:
        p = sc.SpMMPlan(cf, 128, panel_range=r)
        p.spmm(Bt, Cs[r[0] * 4: r[1] * 4])
    assert np.all(np.abs(Cs.cpu().numpy().astype(np.float64) - ref) <= RTOL * scale)
    B2_np = wl.dense_b(m, 128, 99)
    B2 = torch.from_numpy(B2_np).to(cuda)
    lhs = plan.spmm(Bt + B2).cpu().numpy().astype(np.float64)
    rhs = got + plan.spmm(B2).cpu().numpy().astype(np.float64)
    scale2 = scale + cpu.spmm_csr_abs(ip, ix, dx, B2_np)
    assert np.all(np.abs(lhs - rhs) <= 3 * RTOL * scale2)


@pytest.mark.parametrize("N", [1, 2, 4])
def test_config5_small_b_full_size_parity(cuda, N):
    """The config-5 matrix on the small-B kernel (SpMV and N = 4): every row
    against the oracle at the fp32 bound."""
    import torch
    a, B = wl.config5(n_cols_b=N)
    _, _, ip, ix, dx = a
    plan = sc.SpMMPlan(sc.csr_to_compressed_format_converter(to_csr_handle(a), 4, 1), N)
    assert plan.info["kernel"] == 1
    if N == 1:
        y = plan.spmv(torch.from_numpy(B[:, 0].copy()).to(cuda)).cpu().numpy()[:, None]
    else:
        y = plan.spmm(torch.from_numpy(B).to(cuda)).cpu().numpy()
    ref = cpu.spmm_csr_float(ip, ix, dx, B)
    scale = cpu.spmm_csr_abs(ip, ix, dx, B)
    assert np.all(np.abs(y.astype(np.float64) - ref) <= RTOL * scale)


def test_staged_small_b_kernel_m_sweep(cuda):
    """The kernel that stages B in shared memory (SpMV of large matrices) at
    every kernel_m, with a strided B and C and in accumulate mode, against
    the oracle at the fp32 bound.  6144 rows give >= 1024 panels at every
    kernel_m, so every plan here takes the staged kernel."""
    import torch
    from sparse_computation_b200.partition import row_slice
    N = 1
    a, B = wl.config5(n_cols_b=N)
    a = row_slice(a, 0, 6144)
    _, _, ip, ix, dx = a
    ref = cpu.spmm_csr_float(ip, ix, dx, B)
    scale = cpu.spmm_csr_abs(ip, ix, dx, B)
    C0 = wl.dense_b(a[0], N, 11)
    for km in range(1, 7):
        plan = sc.SpMMPlan(sc.csr_to_compressed_format_converter(to_csr_handle(a), km, 1), N)
        Bw = torch.zeros((B.shape[0], N + 3), device=cuda)
        Bw[:, :N] = torch.from_numpy(B).to(cuda)
        Cw = torch.full((a[0], N + 5), 7.0, device=cuda)
        Cw[:, :N] = torch.from_numpy(C0).to(cuda)
        plan.spmm(Bw[:, :N], Cw[:, :N], accumulate=True)
        y = Cw[:, :N].cpu().numpy().astype(np.float64)
        assert np.all(np.abs(y - (ref + C0)) <= RTOL * (scale + np.abs(C0))), km
        assert torch.all(Cw[:, N:] == 7.0)
        assert plan.status() == 0
        y2 = plan.spmm(torch.from_numpy(B).to(cuda)).cpu().numpy().astype(np.float64)
        assert np.all(np.abs(y2 - ref) <= RTOL * scale), km


def test_staged_spmv_host_entry_point(cuda):
    """The host entry point on a plan that takes the staged SpMV kernel:
    pageable buffers (row chunks, each a subset of the panel order) and
    page-locked ones (C stored straight into host memory) both match the
    oracle at the fp32 bound, twice in a row."""
    import torch
    from sparse_computation_b200.partition import row_slice
    a, B = wl.config5(n_cols_b=1)
    a = row_slice(a, 0, 6144)
    _, _, ip, ix, dx = a
    ref = cpu.spmm_csr_float(ip, ix, dx, B)
    scale = cpu.spmm_csr_abs(ip, ix, dx, B)
    plan = sc.SpMMPlan(sc.csr_to_compressed_format_converter(to_csr_handle(a), 4, 1), 1)
    hB = torch.from_numpy(B).pin_memory()
    hC = torch.full((a[0], 1), float("nan")).pin_memory()
    for _ in range(2):
        y = plan.spmm_host(B).astype(np.float64)
        assert np.all(np.abs(y - ref) <= RTOL * scale)
        plan.spmm_host(hB.numpy(), hC.numpy())
        assert np.all(np.abs(hC.numpy().astype(np.float64) - ref) <= RTOL * scale)
    assert plan.status() == 0


def test_batch_layer_stack_one_launch(cuda):
    """All 96 weights of config 4 in one launch == the oracle for each."""
    import torch
    mats = wl.config4(128)
    plans, Bs, Cs = [], [], []
    for name, a, B in mats:
        cf = sc.csr_to_compressed_format_converter(to_csr_handle(a), 4, 1)
        plans.append(sc.SpMMPlan(cf, 128))
        Bs.append(torch.from_numpy(B).to(cuda))
        Cs.append(torch.full((a[0], 128), float("nan"), device=cuda))
    batch = sc.SpMMBatch(plans)
    batch.bind(Bs, Cs)
    for _ in range(2):
        batch.spmm()
    torch.cuda.synchronize()
    for (name, a, B), C in zip(mats, Cs):
        assert_parity(C.cpu().numpy(), a, B)
    # accumulate doubles the product
    batch.spmm(accumulate=True)
    torch.cuda.synchronize()
    for (name, a, B), C in zip(mats[:5], Cs[:5]):
        assert_parity(C.cpu().numpy() / 2, a, B)


def test_batch_rejects_mixed_plans(cuda, monkeypatch):
    monkeypatch.setenv("SC_DENSE", "0")
    a, _ = wl.config1()
    h = to_csr_handle(a)
    p1 = sc.SpMMPlan(sc.csr_to_compressed_format_converter(h, 4, 1), 128)
    p2 = sc.SpMMPlan(sc.csr_to_compressed_format_converter(h, 2, 1), 128)
    p3 = sc.SpMMPlan(sc.csr_to_compressed_format_converter(h, 4, 1), 4)
    for bad in ([p1, p2], [p3]):
        with pytest.raises(sc.ScError):
            sc.SpMMBatch(bad)


def test_peer_store_epilogue_single_gpu(cuda):
    """sc_spmm_peers with 'peers' that are other buffers on the same GPU: each
    receives exactly the tile written to C."""
    import torch
    a, B = wl.config3((2048, 512), 128)
    cf = sc.csr_to_compressed_format_converter(to_csr_handle(a), 4, 1)
    plan = sc.SpMMPlan(cf, 128, panel_range=(100, 300))
    Bt = torch.from_numpy(B).to(cuda)
    full = [torch.full((2048, 128), -1.0, device=cuda) for _ in range(4)]
    C = full[0][400:1200]
    peers = [f.data_ptr() + 400 * 128 * 4 for f in full[1:]]
    plan.spmm_peers(Bt, C, peers)
    torch.cuda.synchronize()
    for f in full[1:]:
        assert torch.equal(f, full[0])
    assert torch.all(full[0][:400] == -1) and torch.all(full[0][1200:] == -1)
    rows = np.arange(400, 1200)
    assert_parity(C.cpu().numpy(), a, B, rows=rows)
    with pytest.raises(sc.ScError):
        sc.SpMMPlan(cf, 4).spmm_peers(torch.zeros((512, 4), device=cuda), torch.zeros((2048, 4), device=cuda), peers)


def test_autotune_kernel_m(cuda):
    from sparse_computation_b200 import tuning
    a, B = wl.config3((2048, 512), 128)
    best, times = tuning.autotune_kernel_m(to_csr_handle(a), 128, candidates=(1, 4), reps=3)
    assert best in (1, 4) and set(times) == {1, 4} and all(t > 0 for t in times.values())


@pytest.mark.parametrize("dense", ["0", "1"])
def test_config4_per_plan_paths(cuda, monkeypatch, dense):
    """A few stack matrices through each path explicitly (wide FFMA / dense tiles)."""
    import torch
    monkeypatch.setenv("SC_DENSE", dense)
    for name, a, B in wl.config4(128)[:6]:
        cf = sc.csr_to_compressed_format_converter(to_csr_handle(a), 4, 1)
        plan = sc.SpMMPlan(cf, 128)
        assert plan.info["kernel"] == (3 if dense == "1" else 2)
        C = plan.spmm(torch.from_numpy(B).to(cuda))
        torch.cuda.synchronize()
        assert_parity(C.cpu().numpy(), a, B)


def test_batch_mixed_dense_and_wide(cuda, monkeypatch):
    """One batch holding dense-tile and wide-B plans (two groups, one launch each)."""
    import torch
    mats = wl.config4(128)[:8]
    plans, Bs, Cs = [], [], []
    for i, (name, a, B) in enumerate(mats):
        monkeypatch.setenv("SC_DENSE", "1" if i % 2 else "0")
        cf = sc.csr_to_compressed_format_converter(to_csr_handle(a), 4, 1)
        plans.append(sc.SpMMPlan(cf, 128))
        Bs.append(torch.from_numpy(B).to(cuda))
        Cs.append(torch.full((a[0], 128), float("nan"), device=cuda))
    assert {p.info["kernel"] for p in plans} == {2, 3}
    batch = sc.SpMMBatch(plans)
    batch.bind(Bs, Cs)
    batch.spmm()
    torch.cuda.synchronize()
    for (name, a, B), C in zip(mats, Cs):
        assert_parity(C.cpu().numpy(), a, B)


@pytest.mark.parametrize("cfg", ["narrow", "wide", "dense"])
def test_graph_capture_plan(cuda, monkeypatch, cfg):
    import torch
    if cfg == "narrow":
        a, B = wl.config2(0.9, 4)
    else:
        monkeypatch.setenv("SC_DENSE", "1" if cfg == "dense" else "0")
        a, B = wl.config3((2048, 512), 128)
    cf = sc.csr_to_compressed_format_converter(to_csr_handle(a), 4, 1)
    plan = sc.SpMMPlan(cf, B.shape[1])
    Bt = torch.from_numpy(B).to(cuda)
    C = torch.zeros((a[0], B.shape[1]), device=cuda)
    g = plan.capture(Bt, C, repeat=3, accumulate=True)  # three C += A*B per replay
    for _ in range(2):
        g.launch()
    torch.cuda.synchronize()
    assert_parity(C.cpu().numpy() / 6.0, a, B)


def test_graph_capture_batch(cuda):
    import torch
    mats = wl.config4(128)[:10]
    plans, Bs, Cs = [], [], []
    for name, a, B in mats:
        plans.append(sc.SpMMPlan(sc.csr_to_compressed_format_converter(to_csr_handle(a), 4, 1), 128))
        Bs.append(torch.from_numpy(B).to(cuda))
        Cs.append(torch.full((a[0], 128), float("nan"), device=cuda))
    batch = sc.SpMMBatch(plans)
    batch.bind(Bs, Cs)
    g = batch.capture(repeat=4)
    g.launch()
    torch.cuda.synchronize()
    for (name, a, B), C in zip(mats, Cs):
        assert_parity(C.cpu().numpy(), a, B)
