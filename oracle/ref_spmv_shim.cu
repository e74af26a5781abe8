// TEST INFRASTRUCTURE ONLY.  Exports the reference's own spmv_csr_float
// (example_cuda/spmv_demo_gpu_utils.h:86-98), compiled from the reference
// header where it lies.
#include "spmv_demo_gpu_utils.h"

extern "C" void ref_spmv_csr_float(int m, const int *Ap, const int *Ai, const float *Ax, const float *x,
                                   float *y) {
  spmv_csr_float(m, Ap, Ai, Ax, x, y);
}
