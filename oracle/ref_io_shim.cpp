// TEST INFRASTRUCTURE ONLY.  Exposes the reference's own loaders
// (utils/Sparse_io.cpp: readCompressedFormatMatrix, readCSRMatrix) through a
// C interface so tests can compare libsc_b200's readers with them.
#include <cstdint>
#include <cstring>
#include "Sparse_io.h"

using swiftware::compression::MixedFormat;

extern "C" void *ref_cf_load(const char *path) {
  return swiftware::compression::readCompressedFormatMatrix(path);
}

extern "C" int ref_cf_num_patterns(void *h) {
  return (int)static_cast<MixedFormat<float> *>(h)->cf.size();
}

// Sizes and borrowed arrays of pattern i: RPP/NPP have nrpp entries, CB ncb,
// NNZ nnz.
extern "C" void ref_cf_pattern(void *h, int i, int64_t *km, int64_t *kn, int64_t *nrpp, int64_t *ncb,
                               int64_t *nnz, const int **rpp, const int **npp, const int **cb,
                               const float **vals) {
  auto *c = static_cast<MixedFormat<float> *>(h)->cf[i];
  *km = (int64_t)c->km;
  *kn = (int64_t)c->kn;
  *nrpp = (int64_t)c->nrpp;
  *ncb = (int64_t)c->CB.size();
  *nnz = (int64_t)c->nnz;
  *rpp = c->RPP;
  *npp = c->NPP;
  *cb = c->CB.data();
  *vals = c->NNZ;
}

extern "C" void *ref_csr_load_mtx(const char *cfmtx_path) {
  return swiftware::compression::readCSRMatrix(cfmtx_path);
}

extern "C" void ref_csr_arrays(void *h, int64_t *m, int64_t *n, int64_t *nnz, const int **p, const int **i,
                               const double **x) {
  auto *a = static_cast<sym_lib::CSR *>(h);
  *m = (int64_t)a->m;
  *n = (int64_t)a->n;
  *nnz = (int64_t)a->nnz;
  *p = a->p;
  *i = a->i;
  *x = a->x;
}
