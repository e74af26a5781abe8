"""Multi-GPU work division for the two configurations that shard naturally.

* Row partition of one large A (scale-out): A is cut at row-panel boundaries
  (multiples of kernel_m, so every rank's slice coarsens to exactly its panel
  range of the whole matrix's CF), balanced by nonzeros.  Each rank computes
  its C row block; blocks are padded to the largest one and gathered with one
  all-gather (NCCL over NVLink on GPUs).  B is replicated.
* Layer stacks: whole matrices are assigned to ranks by greedy
  longest-processing-time on nonzeros; no collective is needed.

The reference has no multi-GPU code; this module is the B200 build's own.
"""
from __future__ import annotations

from typing import List, Sequence, Tuple

import numpy as np


def balanced_panel_cuts(indptr, m_rows: int, kernel_m: int, world: int) -> List[int]:
    """Panel indices [c_0=0, c_1, ..., c_world=panels] splitting the nonzeros
    of A (CSR row pointer `indptr`) into `world` near-equal contiguous shares."""
    panels = (m_rows + kernel_m - 1) // kernel_m
    if panels == 0:
        return [0] * (world + 1)
    ends = np.minimum(np.arange(1, panels + 1) * kernel_m, m_rows)
    cum = np.asarray(indptr)[ends].astype(np.int64)
    total = int(cum[-1])
    cuts = [0]
    for r in range(1, world):
        if total:
            c = int(np.searchsorted(cum, total * r / world, side="left")) + 1
        else:
            c = panels * r // world
        cuts.append(c)
    cuts.append(panels)
    cuts = [min(max(c, 0), panels) for c in cuts]
    for i in range(1, len(cuts)):
        cuts[i] = max(cuts[i], cuts[i - 1])
    return cuts


def panel_rows(cuts: Sequence[int], r: int, kernel_m: int, m_rows: int) -> Tuple[int, int]:
    """Row range [r0, r1) of rank r's panels."""
    return min(cuts[r] * kernel_m, m_rows), min(cuts[r + 1] * kernel_m, m_rows)


def row_slice(a, r0: int, r1: int):
    """CSR arrays (m, n, indptr, indices, data) restricted to rows [r0, r1)."""
    m, n, ip, ix, dx = a
    s, e = int(ip[r0]), int(ip[r1])
    return r1 - r0, n, (np.asarray(ip[r0:r1 + 1]) - s).astype(np.int32), ix[s:e], dx[s:e]


def lpt_assign(weights: Sequence[int], world: int) -> List[int]:
    """Owner rank of every item: heaviest first, each to the least-loaded rank."""
    load = [0] * world
    owner = [0] * len(weights)
    for i in sorted(range(len(weights)), key=lambda i: (-weights[i], i)):
        r = min(range(world), key=lambda r: (load[r], r))
        load[r] += weights[i]
        owner[i] = r
    return owner


def gather_row_blocks(local_block, cuts, rank: int, world: int, kernel_m: int, m_rows: int, group=None):
    """All-gathers equal-padded C row blocks and returns the full C (rows x N)
    as a view-concatenation.  `local_block` is this rank's rows; works with
    any torch.distributed backend (NCCL on GPUs, gloo on CPU)."""
    import torch
    import torch.distributed as dist
    max_rows = max(panel_rows(cuts, r, kernel_m, m_rows)[1] - panel_rows(cuts, r, kernel_m, m_rows)[0]
                   for r in range(world))
    n = local_block.shape[1]
    buf = torch.zeros((world, max_rows, n), dtype=local_block.dtype, device=local_block.device)
    buf[rank, : local_block.shape[0]] = local_block
    if hasattr(dist, "all_gather_into_tensor") and local_block.is_cuda:
        dist.all_gather_into_tensor(buf, buf[rank], group=group)
    else:
        parts = list(buf.unbind(0))
        dist.all_gather(parts, buf[rank].clone(), group=group)
        buf = torch.stack(parts)
    pieces = []
    for r in range(world):
        r0, r1 = panel_rows(cuts, r, kernel_m, m_rows)
        pieces.append(buf[r, : r1 - r0])
    return torch.cat(pieces, 0)
