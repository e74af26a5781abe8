#!/bin/bash
# Large-B SpMM run with the reference script's arguments and steps
# (run_local_spmm_large_b_col.sh of hosseinal/sparse-computation):
#   ./run_local_spmm_large_b_col.sh <path.mtx> <b_col>
# convert (native enumerate + coarsen, kernel_m=4 kernel_n=1) -> build -> run.
# There is no code-generation step: the kernels are template-specialised per
# pattern at build time.
set -e
cd "$(dirname "$0")"
matrix_path=$1
b_col=$2
kernel_m=4
kernel_n=1
b_unroll_factor=1
if [ "$b_col" -gt 32 ]; then warp_num=2; else warp_num=1; fi
matrix_dir=$(dirname "$matrix_path")
matrix_name=$(basename "$matrix_path" .mtx)
compressed_matrix_path="${matrix_dir}/${matrix_name}-${kernel_m}-${kernel_n}.cfmtx"

python3 -m sparse_computation_b200.format_generator "$matrix_path" "$kernel_m" "$kernel_n" --pattern_dictionary false
python3 -m sparse_computation_b200.build > /dev/null

sparse_computation_b200/bin/spmm_demo_gpu \
  -m "$compressed_matrix_path" \
  --header --baseline=true \
  -n SPMM -s CSR -t "$b_col" \
  --b_matrix_columns="$b_col" \
  --number_of_warps="$warp_num" \
  --b_unroll_factor="$b_unroll_factor"
