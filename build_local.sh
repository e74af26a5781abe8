#!/bin/bash
# Builds the library, the demo executables and the CPU oracle
# (build_local.sh of hosseinal/sparse-computation; its kernel_m / b_col
# arguments selected code generation, which this build does not need).
set -e
cd "$(dirname "$0")"
python3 -m sparse_computation_b200.build
make -s -C oracle
