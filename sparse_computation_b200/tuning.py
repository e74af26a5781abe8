"""Per-matrix choice of the coarsening (the "best coarsening per pattern
enumeration" of the benchmark configurations; the reference hard-codes (4, 1)
in its run scripts and ships a sweep of (1..6) x (1..8) files).

On this build kernel_n only decides the padding that the device layout drops,
so the device work depends on kernel_m alone; kernel_n is kept for the
`.cfmtx` file the caller may write.  `autotune_kernel_m` measures every
candidate kernel_m with the real kernel (CUDA events, warm L2) and returns
the fastest.  (A cost model on entry/item counts picked badly -- the 512-row
layers prefer kernel_m = 1 for parallelism while the scale-out matrix prefers
4 -- so the choice is measured.)
"""
from __future__ import annotations

from typing import Dict, Sequence, Tuple

import sparse_computation_b200 as sc


def autotune_kernel_m(csr: sc.CSR, n_cols_b: int, device: int = 0,
                      candidates: Sequence[int] = (1, 2, 3, 4, 5, 6), reps: int = 20) -> Tuple[int, Dict[int, float]]:
    """Times one SpMM per candidate kernel_m on `device`; returns (best m, {m: microseconds})."""
    import torch
    m_rows, k = csr.shape
    dev = torch.device("cuda", device)
    B = torch.rand((k, n_cols_b), device=dev)
    times = {}
    for m in candidates:
        cf = sc.csr_to_compressed_format_converter(csr, m, 1)
        plan = sc.SpMMPlan(cf, n_cols_b, device=device)
        C = torch.empty((plan.rows, n_cols_b), device=dev)
        plan.spmm(B, C)
        torch.cuda.synchronize(dev)
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        for _ in range(reps):
            plan.spmm(B, C)
        e.record()
        e.synchronize()
        times[m] = s.elapsed_time(e) / reps * 1e3
    best = min(times, key=times.get)
    return best, times
