// TEST INFRASTRUCTURE ONLY.  Exports the reference's own spmm_csr_float
// (example_cuda/spmm_demo_gpu_utils.h:25-36), compiled from the reference
// header where it lies, so the oracle restatement can be checked against it
// and so bench.py --impl reference can time the reference's CPU path.
#include "spmm_demo_gpu_utils.h"

extern "C" void ref_spmm_csr_float(int m, int n, const int *Ap, const int *Ai, const float *Ax,
                                   const float *B, float *C) {
  spmm_csr_float(m, n, Ap, Ai, Ax, B, C);
}
