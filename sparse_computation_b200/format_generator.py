"""Command-line converter .mtx -> .cfmtx with the reference converter's
interface (code_gen/ss_format/format_generator.py:175-225):

    python -m sparse_computation_b200.format_generator <path.mtx> <kernel_m> <kernel_n>
           [--pattern_dictionary <file>|false] [--save_collection true|false]
           [--threads T]

writes <stem>-<kernel_m>-<kernel_n>.cfmtx next to the input (and <stem>.cfmtx
with --save_collection true), byte-identical to the reference converter.
Enumeration and coarsening run in native code on all host cores.
"""
import argparse
import sys
import time

import sparse_computation_b200 as sc


def main(argv=None) -> int:
    p = argparse.ArgumentParser(description="Enumerate + coarsen a Matrix-Market file into .cfmtx")
    p.add_argument("path", type=str, default="")
    p.add_argument("kernel_m", type=int, default=4)
    p.add_argument("kernel_n", type=int, default=4)
    p.add_argument("--pattern_dictionary", type=str, default="false")
    p.add_argument("--save_collection", type=str, default="false")
    p.add_argument("--threads", type=int, default=0)
    a = p.parse_args(argv)
    if a.path == "":
        raise ValueError("Please provide the path to the matrix file")
    if not a.path.endswith(".mtx"):
        return 0  # the reference converter silently ignores other inputs
    t0 = time.time()
    csr = sc.read_csr_from_mtx(a.path)
    d = None if a.pattern_dictionary == "false" else a.pattern_dictionary
    cf = sc.csr_to_compressed_format_converter(csr, a.kernel_m, a.kernel_n, d, nthreads=a.threads)
    out = a.path[:-4] + f"-{a.kernel_m}-{a.kernel_n}.cfmtx"
    sc.format_writer(out, cf)
    if a.save_collection == "true":
        sc.format_writer(a.path[:-4] + ".cfmtx", cf)
    print(f"{out}: {cf.num_patterns} patterns, {cf.real_nnz} nonzeros, {time.time() - t0:.3f} s",
          file=sys.stderr)
    return 0


if __name__ == "__main__":
    sys.exit(main())
