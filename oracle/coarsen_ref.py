"""TEST INFRASTRUCTURE ONLY -- oracle for enumerate + coarsen and the .cfmtx text.

Only tests/ use this module, as the checker of libsc_b200's native coarsener
and writer.  It restates, in plain Python over CSR arrays:

  default_patterns(m)       build_patterns_map(m, 1)
                            (code_gen/pattern_utiles/pattern_dictionary.py:29-37)
  coarsen(...)              csr_to_compressed_format_converter + transform_row_panel
                            (code_gen/ss_format/format_generator.py:36-129)
  cfmtx_text(...)           format_writer (format_generator.py:132-160)

Pinned by tests/test_oracle.py against the reference's shipped .cfmtx
fixtures (matrices/, byte-identical) and against format_generator.py run
here, and by the committed golden fixtures under tests/golden/.
"""
from __future__ import annotations

from typing import Dict, List, Tuple

import numpy as np


PAD = None  # marker of a coarsening pad value (written as "0")


def default_patterns(m: int) -> Dict[Tuple[bool, ...], int]:
    out = {}
    for i in range(1, 2 ** m):
        x = 2 ** m - i
        out[tuple(c == "1" for c in format(x, f"0{m}b"))] = i - 1
    return out


def coarsen(num_rows: int, num_cols: int, indptr, indices, data, kernel_m: int, kernel_n: int,
            patterns=None):
    """Returns {"header": [(mask, id)], "blocks": [(rpp, cb, vals)], ...}.

    vals entries are Python floats, or PAD for padding.  Rows are visited in
    panels of kernel_m; inside a panel the rows' next nonzeros are merged by
    column (the k-way merge of format_generator.py:102-124).
    """
    if patterns is None:
        patterns = default_patterns(kernel_m)
    npat = len(patterns)
    rpp = [[0] for _ in range(npat)]
    cbs = [[] for _ in range(npat)]
    vals = [[] for _ in range(npat)]
    indptr = [int(x) for x in indptr]
    indices = [int(x) for x in indices]
    data = [float(x) for x in data]
    for start in range(0, num_rows, kernel_m):
        ptr, end = [], []
        for r in range(start, start + kernel_m):
            if r < num_rows:
                ptr.append(indptr[r]); end.append(indptr[r + 1])
            else:
                ptr.append(0); end.append(0)
        pc = [[] for _ in range(npat)]
        pv = [[] for _ in range(npat)]
        while any(p < e for p, e in zip(ptr, end)):
            mn = min(indices[p] for p, e in zip(ptr, end) if p < e)
            match = tuple(p < e and indices[p] == mn for p, e in zip(ptr, end))
            pid = patterns.get(match, -1)
            if pid != -1:
                pc[pid].append(mn)
                pv[pid].extend(data[ptr[r]] for r in range(kernel_m) if match[r])
            for r in range(kernel_m):
                if match[r]:
                    ptr[r] += 1
        for key, pid in patterns.items():
            P = sum(key)
            pack = kernel_n if kernel_n != 0 else 32 // P
            v = pv[pid]
            rem = len(v) % (pack * P)
            vals[pid].extend(v)
            if v and rem:
                vals[pid].extend([PAD] * (pack * P - rem))
            c = pc[pid]
            cbs[pid].extend(c)
            remc = len(c) % pack
            if c and remc:
                cbs[pid].extend([max(c)] * (pack - remc))
            rpp[pid].append(len(cbs[pid]))
    header = [("".join("1" if b else "0" for b in key), pid) for key, pid in patterns.items()]
    return {"num_rows": num_rows, "num_cols": num_cols, "kernel_m": kernel_m, "kernel_n": kernel_n,
            "header": header, "blocks": [(rpp[i], cbs[i], vals[i]) for i in range(npat)]}


def cfmtx_text(cf) -> str:
    """format_writer's text: values as Python float repr, padding as "0"."""
    lines = [f"{cf['num_rows']} {cf['num_cols']} {cf['kernel_m']} {len(cf['header'])} {cf['kernel_n']}\n"]
    for mask, pid in cf["header"]:
        lines.append(f"{mask} {pid} \n")
    for rpp, cb, vals in cf["blocks"]:
        lines.append(" ".join(str(x) for x in rpp) + "\n")
        lines.append(" ".join(str(x) for x in cb) + "\n")
        lines.append(" ".join("0" if x is PAD else repr(float(x)) for x in vals) + "\n")
    return "".join(lines)


def dense_from_cf(cf) -> np.ndarray:
    """Rebuilds the dense matrix the CF encodes (float64), for small checks."""
    m = cf["kernel_m"]
    A = np.zeros((((cf["num_rows"] + m - 1) // m) * m, cf["num_cols"]))
    masks = {pid: mask for mask, pid in cf["header"]}
    for pid, (rpp, cb, vals) in enumerate(cf["blocks"]):
        rows = [j for j, c in enumerate(masks[pid]) if c == "1"]
        P = len(rows)
        for panel in range(len(rpp) - 1):
            for j in range(rpp[panel], rpp[panel + 1]):
                for p in range(P):
                    v = vals[j * P + p]
                    if v is not PAD:
                        A[panel * m + rows[p], cb[j]] += v
    return A[: cf["num_rows"]]
