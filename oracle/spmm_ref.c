/*
 * TEST INFRASTRUCTURE ONLY -- the CPU oracle for the SpMM/SpMV hot path.
 * Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg load
 * this library, and only as the checker or the timed CPU baseline; the
 * product (sparse_computation_b200/libsc_b200.so) never calls it.
 *
 * Plain-C restatement of the reference's host CSR references:
 *   oracle_spmm_csr_float  <- spmm_csr_float, example_cuda/spmm_demo_gpu_utils.h:25-36
 *                             (rows in order, CSR order inside a row, float
 *                             accumulation straight into C: C += A*B)
 *   oracle_spmv_csr_float  <- spmv_csr_float, example_cuda/spmv_demo_gpu_utils.h:86-98
 *                             (double accumulation per row, then y += sum)
 * plus helpers the parity tests use:
 *   oracle_spmm_csr_abs    C_abs += |A|*|B| in double: the scale of the
 *                          tolerance |dC_ij| <= 1e-5 * sum_k |A_ik * B_kj|
 *   oracle_spmm_csr_double C += A*B accumulated in double
 *   oracle_spmm_csr_float_threads  oracle_spmm_csr_float over row blocks on
 *                          `nthreads` POSIX threads (same per-row arithmetic,
 *                          so bit-identical to the serial call)
 * Pinned against the reference's own spmm_csr_float / spmv_csr_float, built
 * from the reference sources into oracle/_ref/ (see Makefile), by
 * tests/test_oracle.py.
 */
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <math.h>

void oracle_spmm_csr_float(int m, int n, const int *Ap, const int *Ai, const float *Ax,
                           const float *B, float *C) {
  for (int i = 0; i < m; i++) {
    for (int j = Ap[i]; j < Ap[i + 1]; j++) {
      int col_index = Ai[j];
      float value = Ax[j];
      for (int k = 0; k < n; k++) C[(int64_t)i * n + k] += value * B[(int64_t)col_index * n + k];
    }
  }
}

void oracle_spmv_csr_float(int m, const int *Ap, const int *Ai, const float *Ax, const float *x,
                           float *y) {
  for (int i = 0; i < m; i++) {
    double sum = 0.0;
    for (int j = Ap[i]; j < Ap[i + 1]; j++) {
      double value = Ax[j];
      sum += value * x[Ai[j]];
    }
    y[i] += sum;
  }
}

void oracle_spmm_csr_abs(int m, int n, const int *Ap, const int *Ai, const float *Ax, const float *B,
                         double *Cabs) {
  for (int i = 0; i < m; i++)
    for (int j = Ap[i]; j < Ap[i + 1]; j++) {
      double a = fabs((double)Ax[j]);
      for (int k = 0; k < n; k++) Cabs[(int64_t)i * n + k] += a * fabs((double)B[(int64_t)Ai[j] * n + k]);
    }
}

void oracle_spmm_csr_double(int m, int n, const int *Ap, const int *Ai, const float *Ax, const float *B,
                            double *C) {
  for (int i = 0; i < m; i++)
    for (int j = Ap[i]; j < Ap[i + 1]; j++) {
      double a = (double)Ax[j];
      for (int k = 0; k < n; k++) C[(int64_t)i * n + k] += a * (double)B[(int64_t)Ai[j] * n + k];
    }
}

typedef struct {
  int r0, r1, n;
  const int *Ap, *Ai;
  const float *Ax, *B;
  float *C;
} slice_t;

static void *run_slice(void *arg) {
  slice_t *s = (slice_t *)arg;
  /* Ap values are absolute offsets, so a row block is Ap + r0 with C shifted. */
  oracle_spmm_csr_float(s->r1 - s->r0, s->n, s->Ap + s->r0, s->Ai, s->Ax, s->B,
                        s->C + (int64_t)s->r0 * s->n);
  return NULL;
}

int oracle_spmm_csr_float_threads(int nthreads, int m, int n, const int *Ap, const int *Ai,
                                  const float *Ax, const float *B, float *C) {
  if (nthreads < 1) nthreads = 1;
  if (nthreads > 1024) nthreads = 1024;
  pthread_t th[1024];
  slice_t sl[1024];
  for (int t = 0; t < nthreads; t++) {
    sl[t].r0 = (int)((int64_t)m * t / nthreads);
    sl[t].r1 = (int)((int64_t)m * (t + 1) / nthreads);
    sl[t].n = n; sl[t].Ap = Ap; sl[t].Ai = Ai; sl[t].Ax = Ax; sl[t].B = B; sl[t].C = C;
    if (pthread_create(&th[t], NULL, run_slice, &sl[t]) != 0) return -1;
  }
  for (int t = 0; t < nthreads; t++) pthread_join(th[t], NULL);
  return 0;
}
