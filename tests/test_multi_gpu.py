"""Row-partitioned SpMM over 2 GPUs (one process per GPU): C row blocks
exchanged (a) by the SpMM kernel's own peer stores into symmetric memory and
(b) by NCCL all-gather; every rank must end with the full C matching the
oracle.  Needs >= 2 GPUs (skipped otherwise)."""
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, mode, result):
    import sys
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    import torch
    import torch.distributed as dist

    import sparse_computation_b200 as sc
    from oracle import cpu
    from sparse_computation_b200 import partition as pt
    from sparse_computation_b200 import workloads as wl

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev)
    try:
        a, B = wl.config3((2048, 512), 128)
        m = a[0]
        cuts = pt.balanced_panel_cuts(a[2], m, 4, world)
        r0, r1 = pt.panel_rows(cuts, rank, 4, m)
        cf = sc.csr_to_compressed_format_converter(sc.CSR.from_arrays(*pt.row_slice(a, r0, r1)), 4, 1)
        plan = sc.SpMMPlan(cf, 128, device=rank)
        Bt = torch.from_numpy(B).to(dev)
        if mode in ("peer", "signal"):
            import torch.distributed._symmetric_memory as symm_mem
            g = dist.group.WORLD
            try:
                symm_mem.enable_symm_mem_for_group(g.group_name)
            except Exception:
                pass
            full = symm_mem.empty((m, 128), dtype=torch.float32, device=dev)
            hdl = symm_mem.rendezvous(full, g.group_name)
            peers = [int(hdl.buffer_ptrs[q]) + r0 * 128 * 4 for q in range(world) if q != rank]
            if mode == "peer":
                for _ in range(2):
                    plan.spmm_peers(Bt, full[r0:r1], peers)
                    hdl.barrier(channel=0)
            else:
                flags = symm_mem.empty((world,), dtype=torch.int32, device=dev)
                fh = symm_mem.rendezvous(flags, g.group_name)
                flags.zero_()
                status = torch.zeros(1, dtype=torch.int32, device=dev)
                fh.barrier(channel=0)
                fptrs = [int(fh.buffer_ptrs[q]) + rank * 4 for q in range(world)]
                stream = torch.cuda.current_stream()
                for epoch in (1, 2, 3):
                    full.zero_() if epoch == 3 else None
                    if epoch == 3:
                        fh.barrier(channel=0)  # every rank cleared its C before new stores arrive
                    plan.spmm_peers(Bt, full[r0:r1], peers, flag_ptrs=fptrs, epoch=epoch)
                    sc.wait_flags(flags.data_ptr(), world, epoch, status.data_ptr(), stream)
                torch.cuda.synchronize()
                assert int(status.item()) == 0
            C = full
        else:
            C = pt.gather_row_blocks(plan.spmm(Bt), cuts, rank, world, 4, m)
        torch.cuda.synchronize()
        got = C.cpu().numpy()
        ref = cpu.spmm_csr_float(a[2], a[3], a[4], B)
        scale = cpu.spmm_csr_abs(a[2], a[3], a[4], B)
        result[rank] = bool(np.all(np.abs(got.astype(np.float64) - ref) <= 1e-5 * scale))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("mode", ["peer", "signal", "nccl"])
def test_row_partition_two_gpus(mode):
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    world = 2
    ctx = mp.get_context("spawn")
    mgr = ctx.Manager()
    result = mgr.dict()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, mode, result)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(300)
        assert p.exitcode == 0
    assert all(result[r] for r in range(world))
