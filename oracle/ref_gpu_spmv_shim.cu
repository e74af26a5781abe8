// BENCH/TEST INFRASTRUCTURE ONLY.  The reference's own SpMV GPU kernel,
// SpmvComplexPatternDecomposeByRowSeperated
// (example_cuda/spmv_demo_gpu_utils.h:852-904), compiled from the reference
// header where it lies for sm_100a and run as its benchmark class runs it
// (SpMVMixePatternDecomposeByRowSeperated::execute, spmv_demo_gpu_utils.h:925-940):
// one 32-thread block per (row panel, pattern), y accumulated with atomicAdd
// into a zeroed buffer.  Generated for kernel_m = 4: the .cfmtx must be
// coarsened with (4, 1).  A reported baseline for bench.py; nothing in the
// product links it.
#include "spmv_demo_gpu_utils.h"
#include "Sparse_io.h"

namespace {
struct RefSpmv {
  swiftware::compression::MixedFormat<float> *host = nullptr;
  swiftware::compression::MixedFormatGPU<float> *mf = nullptr;
  float *dX = nullptr, *dY = nullptr;
  int rows = 0, cols = 0, nrpp = 0;
};
}  // namespace

extern "C" void *ref_gpu_spmv_create(const char *cfmtx_path, const float *hx) {
  auto *h = new RefSpmv();
  h->host = swiftware::compression::readCompressedFormatMatrix(cfmtx_path);
  if (!h->host || h->host->cf.size() != 15) {
    delete h;
    return nullptr;
  }
  h->rows = (int)h->host->cf[0]->m;
  h->cols = (int)h->host->cf[0]->n;
  h->nrpp = (int)h->host->cf[0]->nrpp;
  cudaMalloc((void **)&h->dX, (size_t)h->cols * sizeof(float));
  cudaMalloc((void **)&h->dY, (size_t)h->rows * sizeof(float));
  cudaMemset(h->dY, 0, (size_t)h->rows * sizeof(float));
  cudaMemcpy(h->dX, hx, (size_t)h->cols * sizeof(float), cudaMemcpyHostToDevice);
  h->mf = allocateAndCopyMixedFormat(h->host);
  // the upload's zero-byte copies (patterns without entries) leave a
  // non-sticky error behind; clear it so that the launch check sees its own
  cudaGetLastError();
  return cudaDeviceSynchronize() == cudaSuccess ? h : nullptr;
}

extern "C" int ref_gpu_spmv_zero(void *p, void *stream) {
  auto *h = static_cast<RefSpmv *>(p);
  return (int)cudaMemsetAsync(h->dY, 0, (size_t)h->rows * sizeof(float), (cudaStream_t)stream);
}

extern "C" int ref_gpu_spmv_run(void *p, void *stream) {
  auto *h = static_cast<RefSpmv *>(p);
  SpmvComplexPatternDecomposeByRowSeperated<<<(h->nrpp - 1) * 15, 32, 0, (cudaStream_t)stream>>>(h->mf, h->dX,
                                                                                                 h->dY);
  return (int)cudaGetLastError();
}

extern "C" int ref_gpu_spmv_result(void *p, float *hy) {
  auto *h = static_cast<RefSpmv *>(p);
  return (int)cudaMemcpy(hy, h->dY, (size_t)h->rows * sizeof(float), cudaMemcpyDeviceToHost);
}

extern "C" void ref_gpu_spmv_free(void *p) {
  auto *h = static_cast<RefSpmv *>(p);
  cudaFree(h->dX);
  cudaFree(h->dY);
  delete h;
}
