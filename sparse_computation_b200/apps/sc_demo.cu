// Demo drivers with the reference's command line and CSV report, over the
// C ABI of libsc_b200.so.  One source builds three executables:
//   spmm_demo_gpu              (SC_DEMO_MODE 0: large B, N = --b_matrix_columns)
//   spmm_small_b_col_demo_gpu  (SC_DEMO_MODE 1: small B, N = --b_matrix_columns)
//   spmv_demo_gpu              (SC_DEMO_MODE 2: N = 1)
// Replaces example_cuda/spmm_demo_gpu.cu:9-200, spmm_small_b_col_demo_gpu.cu
// and spmv_demo_gpu.cu, and the option parser src/InputParser.cpp:22-163
// (same option names and defaults; missing required options print the same
// message and exit 0).  Flow as in the reference: load the .cfmtx and its
// companion .mtx, fill B with rand()/RAND_MAX, run cuSPARSE CSR SpMM (its
// output is the correctness reference, spmm_demo_gpu.cu:80-92), optionally
// cuBLAS SGEMM on the densified A (--baseline), then the pattern kernel, each
// for 7 trials timed with CUDA events, and print one CSV row per
// implementation.
#include <cublas_v2.h>
#include <cuda_runtime.h>
#include <cusparse.h>

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <string>
#include <vector>

#include "sc_b200.h"

#ifndef SC_DEMO_MODE
#define SC_DEMO_MODE 0
#endif

namespace {

struct Config {
  std::string matrix, dict, op, sf;
  int threads = 1, coarsening = 5, packing = 1, tuning = 0, iteration_limit = 0;
  bool prefer_fsc = false;
  int number_of_warps = 8, b_unroll_factor = 4, m_tile = 64, n_tile = 64, b_cols = 256;
  int hint = 0, prefetch_distance = 0;
  bool baseline = false, analyze = false, header = false;
};

void usage() {
  printf("Usage: -m <matrix.cfmtx> -n SPMM|SPMV|SPTRS -s CSR|CSC [-t threads] [--b_matrix_columns N]\n"
         "       [--number_of_warps W] [--b_unroll_factor U] [--baseline[=true|false]] [-d|--header]\n"
         "       [--dict f] [-c n] [-p n] [-u n] [--iteration_limit n] [--prefer_fsc] [--m_tile_size n]\n"
         "       [--n_tile_size n] [--hint n] [--prefetch_distance n] [--analyze_codelets]\n");
}

bool parse_bool(const std::string &v) { return v.empty() || v == "true" || v == "1"; }

// cxxopts-style parsing: "-m x", "--matrix x", "--matrix=x", "--flag".
Config parse(int argc, char **argv) {
  Config c;
  std::map<std::string, std::string> alias = {
      {"m", "matrix"}, {"n", "numerical_operation"}, {"s", "storage_format"}, {"t", "threads"},
      {"c", "coarsening"}, {"p", "packing"}, {"u", "tuning"}, {"d", "header"}, {"h", "help"}};
  const std::vector<std::string> flags = {"header", "help", "baseline", "prefer_fsc", "analyze_codelets"};
  std::map<std::string, std::string> kv;
  for (int i = 1; i < argc; ++i) {
    std::string a = argv[i], key, val;
    bool has_val = false;
    if (a.rfind("--", 0) == 0) {
      key = a.substr(2);
    } else if (a.rfind("-", 0) == 0 && a.size() >= 2) {
      key = a.substr(1);
      if (alias.count(key)) key = alias[key];
    } else {
      continue;
    }
    size_t eq = key.find('=');
    if (eq != std::string::npos) { val = key.substr(eq + 1); key = key.substr(0, eq); has_val = true; }
    if (alias.count(key)) key = alias[key];
    bool is_flag = std::find(flags.begin(), flags.end(), key) != flags.end();
    if (!has_val && !is_flag && i + 1 < argc) { val = argv[++i]; }
    kv[key] = val;
  }
  if (kv.count("help")) { usage(); exit(0); }
  if (!kv.count("matrix")) { printf("'matrix' is manditory argument. Use --help\n"); exit(0); }
  if (!kv.count("numerical_operation")) {
    printf("'numerical_operation' is manditory argument. Use --help\n");
    exit(0);
  }
  if (!kv.count("storage_format")) { printf("'storage_format' is manditory argument. Use --help\n"); exit(0); }
  c.matrix = kv["matrix"];
  c.op = kv["numerical_operation"];
  c.sf = kv["storage_format"];
  auto geti = [&](const char *k, int &dst) { if (kv.count(k)) dst = atoi(kv[k].c_str()); };
  if (kv.count("dict")) c.dict = kv["dict"];
  geti("threads", c.threads); geti("coarsening", c.coarsening); geti("packing", c.packing);
  geti("tuning", c.tuning); geti("iteration_limit", c.iteration_limit); geti("number_of_warps", c.number_of_warps);
  geti("b_unroll_factor", c.b_unroll_factor); geti("m_tile_size", c.m_tile); geti("n_tile_size", c.n_tile);
  geti("b_matrix_columns", c.b_cols); geti("hint", c.hint); geti("prefetch_distance", c.prefetch_distance);
  if (kv.count("baseline")) c.baseline = parse_bool(kv["baseline"]);
  if (kv.count("prefer_fsc")) c.prefer_fsc = parse_bool(kv["prefer_fsc"]);
  if (kv.count("analyze_codelets")) c.analyze = parse_bool(kv["analyze_codelets"]);
  c.header = kv.count("header") > 0;
  if (c.op != "SPMV" && c.op != "SPTRS" && c.op != "SPMM") {
    printf("'numerical_operation' must be passed in as one of: ['SPMV', 'SPTRS', 'SPMM']\n");
    exit(0);
  }
  if (c.sf != "CSR" && c.sf != "CSC") {
    printf("'storage_format' must be passed in as one of: ['CSC', 'CSR']\n");
    exit(0);
  }
  return c;
}

#define CK(x)                                                                            \
  do {                                                                                   \
    cudaError_t e_ = (x);                                                                \
    if (e_ != cudaSuccess) { fprintf(stderr, "CUDA error %s at %s:%d\n", cudaGetErrorString(e_), __FILE__, __LINE__); exit(1); } \
  } while (0)
#define SCK(x)                                                                           \
  do {                                                                                   \
    int s_ = (x);                                                                        \
    if (s_ != SC_OK) { fprintf(stderr, "libsc_b200 error %d: %s\n", s_, sc_last_error_string()); exit(1); } \
  } while (0)

constexpr int kTrials = 7;  // SWTensorBench default NumTrials

struct Result {
  std::string name;
  std::vector<double> ms;
  std::vector<std::pair<int, double>> err;  // (correct, inf-norm error)
  bool ran = false;
};

// Correct when |C - C_cusparse| <= 2e-5 * sum_k |A_ik B_kj| for every entry
// (both sides within 1e-5 of the exact product); Error is the absolute
// inf-norm, as in the reference's verify (spmm_demo_gpu_utils.h:1684-1698).
std::pair<int, double> verify(const std::vector<float> &C, const std::vector<float> &Cref,
                              const std::vector<double> &scale) {
  double inf = 0;
  int ok = 1;
  for (size_t i = 0; i < C.size(); ++i) {
    double d = std::fabs((double)C[i] - (double)Cref[i]);
    inf = std::max(inf, d);
    if (d > 2e-5 * scale[i]) ok = 0;
  }
  return {ok, inf};
}

std::string csv_header(int trials) {
  std::string h = "Operation Name,Implementation Name,Number of Trials,Matrix Name,Number of Threads,"
                  "Number of Subregions,";
  for (int i = 0; i < trials; ++i)
    h += "Trial" + std::to_string(i) + " Subregion0 Executor,Correct" + std::to_string(i) + ",Error" +
         std::to_string(i) + ",";
  return h;
}

}  // namespace

int main(int argc, char **argv) {
  Config cfg = parse(argc, argv);
  const int mode = SC_DEMO_MODE;
  const std::string op_name = mode == 2 ? "SpMV_Demo" : "SpMM_Demo";

  sc_cf *cf = nullptr;
  sc_csr *csr = nullptr;
  if (cfg.matrix.size() < 6 || cfg.matrix.substr(cfg.matrix.size() - 6) != ".cfmtx") {
    fprintf(stderr, "loadCfmtxMatrices expects a .cfmtx path: %s\n", cfg.matrix.c_str());
    return 1;
  }
  if (sc_cf_load(cfg.matrix.c_str(), &cf) != SC_OK) {
    fprintf(stderr, "%s\n", sc_last_error_string());
    return 1;
  }
  char comp[4096];
  SCK(sc_companion_mtx_path(cfg.matrix.c_str(), comp, sizeof comp));
  if (sc_mtx_load_csr(comp, &csr) != SC_OK) {
    fprintf(stderr, "%s\n", sc_last_error_string());
    return 1;
  }
  int32_t M, K, km, np_, vl;
  int64_t nnz;
  SCK(sc_cf_dims(cf, &M, &K, &km, &np_, &vl));
  SCK(sc_csr_dims(csr, nullptr, nullptr, &nnz));
  const int N = mode == 2 ? 1 : cfg.b_cols;

  // B = rand()/RAND_MAX (unseeded, as spmm_demo_gpu.cu:57-61)
  std::vector<float> B((size_t)K * N);
  for (auto &x : B) x = (float)((double)rand() / RAND_MAX);

  const int32_t *rp, *ci;
  const double *vx;
  SCK(sc_csr_arrays(csr, &rp, &ci, &vx));
  std::vector<float> vf(nnz);
  for (int64_t i = 0; i < nnz; ++i) vf[i] = (float)vx[i];
  std::vector<double> scale((size_t)M * N, 0.0);
  for (int i = 0; i < M; ++i)
    for (int j = rp[i]; j < rp[i + 1]; ++j)
      for (int k = 0; k < N; ++k) scale[(size_t)i * N + k] += std::fabs((double)vf[j] * B[(size_t)ci[j] * N + k]);

  float *dB, *dC;
  CK(cudaMalloc(&dB, std::max<size_t>(16, B.size() * 4)));
  CK(cudaMalloc(&dC, std::max<size_t>(16, (size_t)M * N * 4)));
  CK(cudaMemcpy(dB, B.data(), B.size() * 4, cudaMemcpyHostToDevice));
  cudaEvent_t e0, e1;
  CK(cudaEventCreate(&e0));
  CK(cudaEventCreate(&e1));
  std::vector<float> Cref((size_t)M * N), C((size_t)M * N);

  // ---- cuSPARSE CSR SpMM (reference's correctness source)
  Result cus;
  cus.name = "SpMM CuSparse";
  {
    int *dRp, *dCi;
    float *dV;
    CK(cudaMalloc(&dRp, (M + 1) * 4));
    CK(cudaMalloc(&dCi, std::max<int64_t>(1, nnz) * 4));
    CK(cudaMalloc(&dV, std::max<int64_t>(1, nnz) * 4));
    CK(cudaMemcpy(dRp, rp, (M + 1) * 4, cudaMemcpyHostToDevice));
    CK(cudaMemcpy(dCi, ci, nnz * 4, cudaMemcpyHostToDevice));
    CK(cudaMemcpy(dV, vf.data(), nnz * 4, cudaMemcpyHostToDevice));
    cusparseHandle_t h;
    cusparseCreate(&h);
    cusparseSpMatDescr_t A;
    cusparseDnMatDescr_t Bd, Cd;
    cusparseCreateCsr(&A, M, K, nnz, dRp, dCi, dV, CUSPARSE_INDEX_32I, CUSPARSE_INDEX_32I,
                      CUSPARSE_INDEX_BASE_ZERO, CUDA_R_32F);
    cusparseCreateDnMat(&Bd, K, N, N, dB, CUDA_R_32F, CUSPARSE_ORDER_ROW);
    cusparseCreateDnMat(&Cd, M, N, N, dC, CUDA_R_32F, CUSPARSE_ORDER_ROW);
    float alpha = 1.f, beta = 0.f;
    size_t ws = 0;
    cusparseSpMM_bufferSize(h, CUSPARSE_OPERATION_NON_TRANSPOSE, CUSPARSE_OPERATION_NON_TRANSPOSE, &alpha, A, Bd,
                            &beta, Cd, CUDA_R_32F, CUSPARSE_SPMM_ALG_DEFAULT, &ws);
    void *dws = nullptr;
    if (ws) CK(cudaMalloc(&dws, ws));
    for (int t = 0; t < kTrials; ++t) {
      CK(cudaEventRecord(e0));
      cusparseSpMM(h, CUSPARSE_OPERATION_NON_TRANSPOSE, CUSPARSE_OPERATION_NON_TRANSPOSE, &alpha, A, Bd, &beta, Cd,
                   CUDA_R_32F, CUSPARSE_SPMM_ALG_DEFAULT, dws);
      CK(cudaEventRecord(e1));
      CK(cudaEventSynchronize(e1));
      float ms;
      CK(cudaEventElapsedTime(&ms, e0, e1));
      cus.ms.push_back(ms);
      cus.err.push_back({1, 0.0});
    }
    CK(cudaMemcpy(Cref.data(), dC, Cref.size() * 4, cudaMemcpyDeviceToHost));
    cus.ran = true;
    cusparseDestroySpMat(A);
    cusparseDestroyDnMat(Bd);
    cusparseDestroyDnMat(Cd);
    cusparseDestroy(h);
    if (dws) cudaFree(dws);
    cudaFree(dRp);
    cudaFree(dCi);
    cudaFree(dV);
  }

  // ---- cuBLAS SGEMM on the densified A (--baseline)
  Result cub;
  cub.name = "SpMM CuBlas";
  if (cfg.baseline) {
    std::vector<float> Ad((size_t)M * K, 0.f);
    for (int i = 0; i < M; ++i)
      for (int j = rp[i]; j < rp[i + 1]; ++j) Ad[(size_t)i * K + ci[j]] += vf[j];
    float *dA;
    CK(cudaMalloc(&dA, std::max<size_t>(16, Ad.size() * 4)));
    CK(cudaMemcpy(dA, Ad.data(), Ad.size() * 4, cudaMemcpyHostToDevice));
    cublasHandle_t h;
    cublasCreate(&h);
    cublasSetMathMode(h, CUBLAS_PEDANTIC_MATH);
    float alpha = 1.f, beta = 0.f;
    for (int t = 0; t < kTrials; ++t) {
      CK(cudaEventRecord(e0));
      // row-major C = A*B as column-major C^T = B^T * A^T
      cublasSgemm(h, CUBLAS_OP_N, CUBLAS_OP_N, N, M, K, &alpha, dB, N, dA, K, &beta, dC, N);
      CK(cudaEventRecord(e1));
      CK(cudaEventSynchronize(e1));
      float ms;
      CK(cudaEventElapsedTime(&ms, e0, e1));
      CK(cudaMemcpy(C.data(), dC, C.size() * 4, cudaMemcpyDeviceToHost));
      cub.ms.push_back(ms);
      cub.err.push_back(verify(C, Cref, scale));
    }
    cub.ran = true;
    cublasDestroy(h);
    cudaFree(dA);
  }

  // ---- pattern kernels (this library)
  Result ours;
  ours.name = mode == 2 ? "SpMV Pattern B200" : "SpMM Pattern B200";
  {
    sc_plan *plan;
    SCK(sc_plan_create(cf, N, 0, &plan));
    for (int t = 0; t < kTrials; ++t) {
      CK(cudaMemset(dC, 0, C.size() * 4));
      CK(cudaEventRecord(e0));
      if (mode == 2) SCK(sc_spmv(plan, dB, dC, 0, nullptr));
      else SCK(sc_spmm(plan, dB, N, dC, N, 0, nullptr));
      CK(cudaEventRecord(e1));
      CK(cudaEventSynchronize(e1));
      float ms;
      CK(cudaEventElapsedTime(&ms, e0, e1));
      CK(cudaMemcpy(C.data(), dC, C.size() * 4, cudaMemcpyDeviceToHost));
      ours.ms.push_back(ms);
      ours.err.push_back(verify(C, Cref, scale));
    }
    ours.ran = true;
    sc_plan_free(plan);
  }

  // ---- CSV (layout of Stats::printCSV + test/schedule parameters)
  const std::string sp_header = "nThreads,Iter Per Partition,MTile,NTile,";
  const std::string tp_header = "MatrixName,Density,nRows,nCols,NNZ,Mode,Algorithm,bCols";
  char sp[256], tp[1024];
  snprintf(sp, sizeof sp, "%d,1,1,1,", cfg.threads);
  snprintf(tp, sizeof tp, "%s,%f,%d,%d,%lld,Random,,%d", cfg.matrix.c_str(), 0.0, M, K, (long long)nnz, 0);
  if (cfg.header)
    printf("%s%s%s,kernel_n,kernel_m,b_cols,b_unroll_factor,number_of_warps,GFLOPs\n", csv_header(kTrials).c_str(),
           sp_header.c_str(), tp_header.c_str());
  auto row = [&](const Result &r) {
    if (!r.ran) return;
    std::string s = op_name + "," + r.name + "," + std::to_string(kTrials) + "," + cfg.matrix + "," +
                    std::to_string(cfg.threads) + ",1,";
    char buf[64];
    for (int i = 0; i < kTrials; ++i) {
      snprintf(buf, sizeof buf, "%.9g,", r.ms[i] / 1e3);
      s += buf;
      snprintf(buf, sizeof buf, "%d,%f,", r.err[i].first, r.err[i].second);
      s += buf;
    }
    std::vector<double> sorted(r.ms.begin(), r.ms.end());
    std::sort(sorted.begin(), sorted.end());
    const double gflops = 2.0 * nnz * N / (sorted[kTrials / 2] * 1e-3) / 1e9;
    printf("%s%s%s,%d,%d,%d,%d,%d,%.3f\n", s.c_str(), sp, tp, vl, km, N, cfg.b_unroll_factor, cfg.number_of_warps,
           gflops);
  };
  if (cfg.baseline) {
    row(cub);
    row(cus);
  }
  row(ours);
  cudaFree(dB);
  cudaFree(dC);
  sc_cf_free(cf);
  sc_csr_free(csr);
  return 0;
}
