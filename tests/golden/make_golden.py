"""Regenerates the golden fixtures in this folder by running the REFERENCE's
own code in a container where the reference tree is available:

  * <case>.mtx                     seeded small matrices (inputs)
  * <case>-<m>-<n>.cfmtx           written by the reference's converter
                                   code_gen/ss_format/format_generator.py
  * spmm_<case>_n<N>.npz           B and C = A*B from the reference's own
                                   spmm_csr_float (oracle/_ref/libref_spmm.so)

    python tests/golden/make_golden.py [/path/to/reference]

The fixtures are committed; tests only read them (no reference at run time).
"""
import os
import subprocess
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from sparse_computation_b200 import workloads as wl  # noqa: E402
from oracle import cpu  # noqa: E402

REF = sys.argv[1] if len(sys.argv) > 1 else cpu.reference_dir()
if not REF:
    sys.exit("usage: make_golden.py <reference checkout> (or set SC_REFERENCE_DIR)")
CONVERTER = os.path.join(REF, "code_gen", "ss_format", "format_generator.py")


def ragged():
    """37x23 with empty rows, an empty last row block and explicit zeros."""
    rng = np.random.default_rng(7)
    A = np.where(rng.random((37, 23)) < 0.3, rng.normal(0, 1, (37, 23)), 0).astype(np.float32)
    A[[3, 4, 5, 6, 20, 36]] = 0
    m, n, ip, ix, dx = wl.csr_from_dense(A)
    # two explicit zeros
    r, c = 10, int(np.nonzero(A[10] == 0)[0][0])
    rows = np.repeat(np.arange(m), np.diff(ip))
    rows = np.concatenate([rows, [r, 12]])
    cols = np.concatenate([ix, [c, int(np.nonzero(A[12] == 0)[0][0])]])
    vals = np.concatenate([dx, [0.0, 0.0]])
    return wl.csr_from_coords(m, n, rows, cols, vals)


def small_cfg1():
    """128x96 Bernoulli(0.10) N(0, 0.05^2): config 1's law at fixture size."""
    mask = np.random.default_rng(1).random((128, 96)) < 0.10
    vals = np.random.default_rng(2).normal(0.0, 0.05, size=(128, 96)).astype(np.float32)
    return wl.csr_from_dense(np.where(mask, vals, 0).astype(np.float32))


def wide_values():
    """64x64, values spanning many decades (exercises the float repr)."""
    rng = np.random.default_rng(11)
    A = np.where(rng.random((64, 64)) < 0.2, rng.normal(0, 1, (64, 64)) * 10.0 ** rng.integers(-12, 18, (64, 64)),
                 0).astype(np.float32)
    return wl.csr_from_dense(A)


CASES = {
    "ragged": (ragged, [(3, 2), (4, 1), (4, 0), (5, 3), (1, 1), (6, 8)]),
    "cfg1small": (small_cfg1, [(2, 4), (4, 1), (4, 2), (6, 3)]),
    "widevals": (wide_values, [(2, 1), (3, 4)]),
}

# A custom dictionary in read_pattern_dictionary's format, ids not in mask
# order and one mask left out (its columns are dropped by the converter).
CUSTOM_DICT = "3 1 6\n111 0\n001 1\n100 2\n010 3\n110 4\n011 5\n"


def run_converter(mtx, m, n, extra=()):
    subprocess.run([sys.executable, CONVERTER, mtx, str(m), str(n), *extra], check=True,
                   stdout=subprocess.DEVNULL, stderr=subprocess.DEVNULL)


def main():
    for case, (fn, params) in CASES.items():
        a = fn()
        mtx = os.path.join(HERE, f"{case}.mtx")
        wl.write_mtx(mtx, a)
        for m, n in params:
            run_converter(mtx, m, n)
    # custom dictionary case (written to a separate stem so names do not clash)
    a = ragged()
    mtx = os.path.join(HERE, "ragged_dict.mtx")
    wl.write_mtx(mtx, a)
    with open(os.path.join(HERE, "dict3.txt"), "w") as f:
        f.write(CUSTOM_DICT)
    run_converter(mtx, 3, 2, ["--pattern_dictionary", os.path.join(HERE, "dict3.txt")])
    # SpMM goldens from the reference's own spmm_csr_float
    cpu.build()
    for case, (fn, _) in CASES.items():
        m, n, ip, ix, dx = fn()
        for N in (1, 4, 32):
            B = wl.dense_b(n, N, 77 + N)
            C = cpu.ref_spmm_csr_float(ip, ix, dx, B)
            np.savez_compressed(os.path.join(HERE, f"spmm_{case}_n{N}.npz"), B=B, C=C)


if __name__ == "__main__":
    main()
