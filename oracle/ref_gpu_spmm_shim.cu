// BENCH/TEST INFRASTRUCTURE ONLY.  The reference's own large-B GPU kernel,
// SpMMFullRowPanelGeneralKernel4With2BlockCacheLess
// (example_cuda/spmm_demo_gpu_utils.h:1583-1665), compiled from the reference
// header where it lies for sm_100a, run the way its benchmark class runs it
// (SpMMMixePatternGeneralCacheLess::execute, spmm_demo_gpu_utils.h:1697-1721):
// the .cfmtx is read by the reference's readCFMTXFile
// (utils/Sparse_io.cpp:84-181, through readCompressedFormatMatrix :208-215), uploaded by allocateAndCopyMixedFormat
// (spmm_demo_gpu_utils.h:207-245), one 32-thread block per (row panel,
// pattern), C accumulated with atomicAdd into a zeroed buffer.  The kernel was
// generated for kernel_m = 4 and two-column packs: the .cfmtx must be
// coarsened with (4, 2).  bench.py times it beside the product kernels as a
// reported baseline; nothing in the product links it.
#include "spmm_demo_gpu_utils.h"
#include "Sparse_io.h"

namespace {
struct RefSpmm {
  swiftware::compression::MixedFormat<float> *host = nullptr;
  swiftware::compression::MixedFormatGPU<float> *mf = nullptr;
  float *dX = nullptr, *dY = nullptr;
  int rows = 0, cols = 0, n = 0, nrpp = 0;
};
}  // namespace

extern "C" void *ref_gpu_spmm_create(const char *cfmtx_path, const float *hB, int n_cols_b) {
  auto *h = new RefSpmm();
  h->host = swiftware::compression::readCompressedFormatMatrix(cfmtx_path);
  if (!h->host || h->host->cf.size() != 15) {
    delete h;
    return nullptr;
  }
  h->rows = (int)h->host->cf[0]->m;
  h->cols = (int)h->host->cf[0]->n;
  h->nrpp = (int)h->host->cf[0]->nrpp;
  h->n = n_cols_b;
  cudaMalloc((void **)&h->dX, (size_t)h->cols * n_cols_b * sizeof(float));
  cudaMalloc((void **)&h->dY, (size_t)h->rows * n_cols_b * sizeof(float));
  cudaMemset(h->dY, 0, (size_t)h->rows * n_cols_b * sizeof(float));
  cudaMemcpy(h->dX, hB, (size_t)h->cols * n_cols_b * sizeof(float), cudaMemcpyHostToDevice);
  h->mf = allocateAndCopyMixedFormat(h->host);
  // the upload's zero-byte copies (patterns without entries) leave a
  // non-sticky error behind; clear it so that the launch check sees its own
  cudaGetLastError();
  return cudaDeviceSynchronize() == cudaSuccess ? h : nullptr;
}

// C = 0 (outside the reference's timed region).
extern "C" int ref_gpu_spmm_zero(void *p, void *stream) {
  auto *h = static_cast<RefSpmm *>(p);
  return (int)cudaMemsetAsync(h->dY, 0, (size_t)h->rows * h->n * sizeof(float), (cudaStream_t)stream);
}

// One launch of the reference kernel (its timed region).
extern "C" int ref_gpu_spmm_run(void *p, void *stream) {
  auto *h = static_cast<RefSpmm *>(p);
  dim3 grid((h->nrpp - 1) * 15, 1);
  SpMMFullRowPanelGeneralKernel4With2BlockCacheLess<<<grid, 32, 0, (cudaStream_t)stream>>>(h->mf, h->dX, h->dY,
                                                                                           h->n);
  return (int)cudaGetLastError();
}

extern "C" int ref_gpu_spmm_result(void *p, float *hC) {
  auto *h = static_cast<RefSpmm *>(p);
  return (int)cudaMemcpy(hC, h->dY, (size_t)h->rows * h->n * sizeof(float), cudaMemcpyDeviceToHost);
}

// Device buffers only (the reference never frees its device copy either).
extern "C" void ref_gpu_spmm_free(void *p) {
  auto *h = static_cast<RefSpmm *>(p);
  cudaFree(h->dX);
  cudaFree(h->dY);
  delete h;
}
