"""Host logic of the multi-GPU paths, on CPU: the nonzero-balanced row-panel
partition, its agreement with the whole matrix's CF, the padded all-gather of
C row blocks (world_size 2, gloo), and the LPT layer assignment."""
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

import sparse_computation_b200 as sc
from oracle import cpu
from sparse_computation_b200 import partition as pt
from sparse_computation_b200 import workloads as wl


def test_cuts_cover_and_balance():
    a, _ = wl.config3((2048, 512), 32)
    m, n, ip, ix, dx = a
    for world in (1, 2, 3, 4, 8):
        cuts = pt.balanced_panel_cuts(ip, m, 4, world)
        assert cuts[0] == 0 and cuts[-1] == (m + 3) // 4 and all(x <= y for x, y in zip(cuts, cuts[1:]))
        shares = [ip[pt.panel_rows(cuts, r, 4, m)[1]] - ip[pt.panel_rows(cuts, r, 4, m)[0]] for r in range(world)]
        assert sum(shares) == len(ix)
        assert max(shares) - min(shares) <= 2 * 4 * max(np.diff(ip))  # within ~one panel of balance
    assert pt.balanced_panel_cuts(np.zeros(1, np.int32), 0, 4, 3) == [0, 0, 0, 0]
    # ragged: rows not a multiple of kernel_m, more ranks than panels
    cuts = pt.balanced_panel_cuts(np.arange(8, dtype=np.int32), 7, 4, 4)
    assert cuts[-1] == 2 and cuts[0] == 0


def test_row_slices_coarsen_to_the_panel_range_of_the_whole_cf(tmp_path):
    """Each rank may coarsen only its rows: the slice's CF equals the whole
    CF restricted to that panel range (panels are independent)."""
    a, _ = wl.config3((512, 2048), 32)
    m = a[0]
    whole = sc.csr_to_compressed_format_converter(sc.CSR.from_arrays(*a), 4, 2)
    cuts = pt.balanced_panel_cuts(a[2], m, 4, 3)
    for r in range(3):
        r0, r1 = pt.panel_rows(cuts, r, 4, m)
        part = sc.csr_to_compressed_format_converter(sc.CSR.from_arrays(*pt.row_slice(a, r0, r1)), 4, 2)
        for pid in range(whole.num_patterns):
            pc, rpp, cb, v = whole.pattern(pid)
            pc2, rpp2, cb2, v2 = part.pattern(pid)
            s, e = rpp[cuts[r]], rpp[cuts[r + 1]]
            assert np.array_equal(rpp2, rpp[cuts[r]:cuts[r + 1] + 1] - s)
            assert np.array_equal(cb2, cb[s:e]) and np.array_equal(v2, v[s * pc:e * pc])


def test_lpt_assign():
    owner = pt.lpt_assign([10, 9, 8, 1, 1, 1], 2)
    loads = [sum(w for w, o in zip([10, 9, 8, 1, 1, 1], owner) if o == r) for r in range(2)]
    assert sorted(loads) == [13, 17]  # greedy LPT (within 4/3 of the optimum 15)
    assert pt.lpt_assign([5], 4) == [0]


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, result):
    import torch
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        a, B = wl.config3((2048, 512), 16)
        m = a[0]
        cuts = pt.balanced_panel_cuts(a[2], m, 4, world)
        r0, r1 = pt.panel_rows(cuts, rank, 4, m)
        blk = pt.row_slice(a, r0, r1)
        Cb = cpu.spmm_csr_float(blk[2], blk[3], blk[4], B)  # stands in for the GPU block product
        C = pt.gather_row_blocks(torch.from_numpy(Cb), cuts, rank, world, 4, m)
        full = cpu.spmm_csr_float(a[2], a[3], a[4], B)
        result[rank] = bool(np.array_equal(C.numpy(), full))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2])
def test_gather_row_blocks_gloo(world):
    ctx = mp.get_context("spawn")
    mgr = ctx.Manager()
    result = mgr.dict()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, result)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
        assert p.exitcode == 0
    assert all(result[r] for r in range(world))


def _dead_rank_worker(rank, world, port, result):
    import datetime

    import torch
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
    a, B = wl.config3((2048, 512), 16)
    m = a[0]
    cuts = pt.balanced_panel_cuts(a[2], m, 4, world)
    if rank == 1:
        os._exit(3)  # this rank dies between steps, before the exchange
    r0, r1 = pt.panel_rows(cuts, rank, 4, m)
    blk = pt.row_slice(a, r0, r1)
    Cb = cpu.spmm_csr_float(blk[2], blk[3], blk[4], B)
    try:
        pt.gather_row_blocks(torch.from_numpy(Cb), cuts, rank, world, 4, m)
        result[rank] = "completed"
    except Exception as ex:  # the collective must fail, not hang
        result[rank] = "raised: " + type(ex).__name__


def test_dead_rank_is_detected_gloo():
    """A rank that exits before the C exchange: the survivor's collective
    ends with an error within the process-group timeout instead of hanging."""
    import time
    ctx = mp.get_context("spawn")
    mgr = ctx.Manager()
    result = mgr.dict()
    port = _free_port()
    procs = [ctx.Process(target=_dead_rank_worker, args=(r, 2, port, result)) for r in range(2)]
    t0 = time.time()
    for p in procs:
        p.start()
    for p in procs:
        p.join(90)
    assert all(p.exitcode is not None for p in procs), "a rank hung"
    assert procs[1].exitcode == 3
    assert result.get(0, "").startswith("raised"), result.get(0)
    assert time.time() - t0 < 90
