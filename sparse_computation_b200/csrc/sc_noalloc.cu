// Allocation-free variant of the dense-tile tensor-core SpMM.
//
// Some callers cannot call cudaMalloc when they run a product: a serving
// process that hands every byte of device memory to its own pool or memory
// budget at start-up, or a component that runs inside a host framework that
// forbids device allocation on its hot path.  sc_spmm_dense_noalloc lets them
// run the tcgen05 dense-tile kernel without any plan and without any
// allocation: they pass A (dense, fp32), B and C; every piece of scratch the
// kernel needs (the TF32 head/tail tile images of A and B, the task list and
// the status word) lives in the file-scope array below, which each GPU that
// loads this library holds until the process exits.
#include <algorithm>
#include <cstdint>
#include <mutex>
#include <string>

#include "sc_dense.cuh"
#include "sc_internal.h"

namespace {

// Scratch shared by every call on a device; calls that overlap on the GPU
// (e.g. on two streams at once) race on it.
constexpr size_t kNoAllocScratchBytes = 16u << 20;  // 16 MiB
static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocScratchBytes];

constexpr int kMaxDevices = 64;
uint8_t *g_scratch_addr[kMaxDevices] = {};
std::mutex g_scratch_mu;

// Device address of the scratch array on the current device.  In host code
// the array's name is only a host-side stand-in, so its device address must
// be asked for once per device, with that device current.  The address is
// kept for the life of the process: a cudaDeviceReset (which discards the
// module and its array) is not supported while this library is loaded.
int scratch_for_current_device(uint8_t **out) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return (int)e;
  if (dev < 0 || dev >= kMaxDevices) return (int)cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> g(g_scratch_mu);
  if (!g_scratch_addr[dev]) {
    void *p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) return (int)e;
    g_scratch_addr[dev] = static_cast<uint8_t *>(p);
  }
  *out = g_scratch_addr[dev];
  return 0;
}

using sc::dense::kBK;
using sc::dense::kBM;
using sc::dense::kBN;
using sc::dense::kTileBytes;

// Row-major A (M x K) -> per (row block, K chunk) [head | tail] swizzled
// images; every chunk is kept (the caller's A is dense).
__global__ void __launch_bounds__(256) noalloc_split_a(const float *__restrict__ A, int64_t lda, int64_t m,
                                                       int64_t k, int kcs, uint8_t *__restrict__ tiles) {
  const int rb = blockIdx.y, kc = blockIdx.x;
  float4 *hi = reinterpret_cast<float4 *>(tiles + ((size_t)rb * kcs + kc) * 2 * kTileBytes);
  float4 *lo = hi + kTileBytes / 16;
  for (int q = threadIdx.x; q < kBM * kBK / 4; q += blockDim.x) {
    const int r = q >> 3, c = q & 7;
    const int k0 = kc * kBK + ((c ^ (r & 7)) << 2);
    const int64_t row = (int64_t)rb * kBM + r;
    float x[4], h[4], l[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      x[j] = (row < m && k0 + j < k) ? __ldg(A + row * lda + k0 + j) : 0.f;
      h[j] = sc::dense::tf32_round(x[j]);
      l[j] = sc::dense::tf32_round(x[j] - h[j]);
    }
    hi[q] = make_float4(h[0], h[1], h[2], h[3]);
    lo[q] = make_float4(l[0], l[1], l[2], l[3]);
  }
}

// Kept-chunk lists (all chunks), the task list, and a cleared status word.
__global__ void noalloc_init(int rbs, int kcs, int nts, int32_t *rb_ptr, int32_t *rb_chunk, int4 *tasks,
                             int *status) {
  const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (t <= rbs) rb_ptr[t] = (int32_t)(t * kcs);
  if (t < (int64_t)rbs * kcs) rb_chunk[t] = (int32_t)(t % kcs);
  if (t < (int64_t)rbs * nts) tasks[t] = make_int4(0, (int)(t / nts), (int)(t % nts), kcs);
  if (t < 4) status[t] = 0;  // status | task counter | done counter of the dense kernel
}

size_t align1k(size_t x) { return (x + 1023) & ~(size_t)1023; }
constexpr size_t kStatusBytes = 1024;

}  // namespace

extern "C" int sc_spmm_dense_noalloc(const float *dA, int64_t lda, int64_t m, int64_t k, const float *dB,
                                     int64_t ldb, int64_t n, float *dC, int64_t ldc, int32_t accumulate,
                                     void *stream) {
  using namespace sc::dense;
  if (m < 0 || k < 0 || n < 0) {
    sc_set_error("sc_spmm_dense_noalloc: negative size");
    return SC_ERR_ARG;
  }
  if (m == 0 || n == 0) return SC_OK;
  if (n % kBN != 0) {
    sc_set_error("sc_spmm_dense_noalloc: n_cols_b must be a multiple of 128");
    return SC_ERR_UNSUPPORTED;
  }
  if (!dA || !dB || !dC || lda < k || ldb < n || ldc < n || ldc % 4 != 0 ||
      reinterpret_cast<uintptr_t>(dC) % 16 != 0) {
    sc_set_error("sc_spmm_dense_noalloc: null operand, leading dimension too small, or C not 16-byte aligned");
    return SC_ERR_ARG;
  }
  const int64_t rbs = (m + kBM - 1) / kBM, kcs = std::max<int64_t>(1, (k + kBK - 1) / kBK), nts = n / kBN;
  // scratch layout: status (first 1 KiB, at a fixed place so that
  // sc_noalloc_status finds it) | A tiles | B tiles | rb_ptr | rb_chunk | tasks
  const size_t o_a = kStatusBytes;
  const size_t o_b = o_a + align1k((size_t)rbs * kcs * 2 * kTileBytes);
  const size_t o_ptr = o_b + align1k((size_t)nts * kcs * 2 * kTileBytes);
  const size_t o_chunk = o_ptr + align1k((size_t)(rbs + 1) * 4);
  const size_t o_tasks = o_chunk + align1k((size_t)rbs * kcs * 4);
  const size_t need = o_tasks + align1k((size_t)rbs * nts * sizeof(int4));
  const size_t o_status = 0;
  if (need > kNoAllocScratchBytes) {
    sc_set_error("sc_spmm_dense_noalloc: needs " + std::to_string(need) + " bytes of scratch, more than the " +
                 std::to_string(kNoAllocScratchBytes) +
                 "-byte limit (A padded to 128-row blocks and B, each at 8 bytes per element, plus small "
                 "index arrays) -- use sc_spmm with a plan for larger matrices");
    return SC_ERR_ARG;
  }
  uint8_t *base = nullptr;
  int err = scratch_for_current_device(&base);
  if (err) {
    sc_set_error(std::string("sc_spmm_dense_noalloc: cudaGetSymbolAddress: ") + cudaGetErrorString((cudaError_t)err));
    return SC_ERR_CUDA;
  }
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  DenseMat mat;
  mat.a_tiles = base + o_a;
  mat.rb_ptr = reinterpret_cast<const int32_t *>(base + o_ptr);
  mat.rb_chunk = reinterpret_cast<const int32_t *>(base + o_chunk);
  mat.b_tiles = base + o_b;
  mat.B = dB;
  mat.ldb = ldb;
  mat.C = dC;
  mat.ldc = ldc;
  mat.rows = m;
  mat.k_rows = (int)k;
  mat.n_cols = (int)n;
  mat.k_chunks = (int)kcs;
  mat.n_tiles = (int)nts;
  mat.bf16 = 0;
  const int64_t cells = std::max<int64_t>({rbs + 1, rbs * kcs, rbs * nts});
  noalloc_init<<<(unsigned)((cells + 255) / 256), 256, 0, s>>>(
      (int)rbs, (int)kcs, (int)nts, const_cast<int32_t *>(mat.rb_ptr), const_cast<int32_t *>(mat.rb_chunk),
      reinterpret_cast<int4 *>(base + o_tasks), reinterpret_cast<int *>(base + o_status));
  noalloc_split_a<<<dim3((unsigned)kcs, (unsigned)rbs), 256, 0, s>>>(dA, lda, m, k, (int)kcs, base + o_a);
  cudaError_t e = cudaGetLastError();
  if (e == cudaSuccess) e = (cudaError_t)sc_dense_split_b(mat, nullptr, 1, (int)(nts * kcs), sc::dense::kModeTf32x3, s);
  // split K over a cluster when the tiles are too few to fill the GPU
  int split = 1;
  while (split < kMaxSplit && rbs * nts * split < 148 && kcs / (split * 2) >= 4) split <<= 1;
  if (e == cudaSuccess)
    e = (cudaError_t)sc_dense_gemm(mat, nullptr, reinterpret_cast<const int4 *>(base + o_tasks), rbs * nts, split,
                                   sc::dense::kModeTf32x3, accumulate, reinterpret_cast<int *>(base + o_status), s);
  if (e != cudaSuccess) {
    sc_set_error(std::string("sc_spmm_dense_noalloc: launch: ") + cudaGetErrorString(e));
    return SC_ERR_CUDA;
  }
  return SC_OK;
}

extern "C" int sc_noalloc_status(int32_t *status) {
  if (!status) {
    sc_set_error("sc_noalloc_status: null argument");
    return SC_ERR_ARG;
  }
  *status = 0;
  uint8_t *base = nullptr;
  int err = scratch_for_current_device(&base);
  cudaError_t e = (cudaError_t)err;
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  int v = 0;
  if (e == cudaSuccess) e = cudaMemcpy(&v, base, 4, cudaMemcpyDeviceToHost);
  if (e == cudaSuccess && v) e = cudaMemset(base, 0, 4);
  if (e != cudaSuccess) {
    sc_set_error(std::string("sc_noalloc_status: ") + cudaGetErrorString(e));
    return SC_ERR_CUDA;
  }
  *status = v;
  return SC_OK;
}
