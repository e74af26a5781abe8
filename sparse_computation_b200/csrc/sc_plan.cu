// Device half of libsc_b200.so: builds the plan (device layout + schedule)
// from a CF matrix and launches the pattern-specialised kernels.
//
// Replaces the reference's device deep copy (allocateAndCopyMixedFormat,
// example_cuda/spmm_demo_gpu_utils.h:207-245: one cudaMalloc/cudaMemcpy per
// array and per pattern, pointer-of-pointers on the device) with one
// contiguous allocation holding a flat record stream and a work list.

#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <memory>
#include <mutex>
#include <string>
#include <vector>

#include "sc_internal.h"
#include "sc_dense.cuh"
#include "sc_kernels.cuh"

#ifndef SC_DEFAULT_DENSE_MODE
#define SC_DEFAULT_DENSE_MODE 2
#endif

namespace {

void require(bool cond, int code, const std::string &msg) {
  if (!cond) throw sc_error(code, msg);
}

void cuda_check(cudaError_t e, const char *what) {
  if (e != cudaSuccess)
    throw sc_error(SC_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

struct DeviceGuard {
  int prev = -1;
  explicit DeviceGuard(int dev) {
    cuda_check(cudaGetDevice(&prev), "cudaGetDevice");
    if (prev != dev) cuda_check(cudaSetDevice(dev), "cudaSetDevice");
  }
  ~DeviceGuard() {
    int cur;
    if (cudaGetDevice(&cur) == cudaSuccess && cur != prev && prev >= 0) cudaSetDevice(prev);
  }
};

}  // namespace

struct sc_plan {
  int device = 0;
  int64_t rows = 0, cols = 0, n = 0, panels = 0, km = 0;
  int64_t nnz = 0, entries = 0, items = 0;
  int kernel = 0;   // 1 narrow, 2 wide
  int warps = 1;
  int vec = 1;      // wide kernel column vector width
  void *dev = nullptr;
  size_t dev_bytes = 0;
  const uint32_t *recs = nullptr;
  const int2 *item_list = nullptr;
  const int32_t *item_ptr = nullptr;
  const int32_t *order = nullptr;
  float *stage_b = nullptr, *stage_c = nullptr;
  // Row-chunked panel orders for the host entry point, so that the copy of a
  // finished chunk of C overlaps the kernels of the next chunks.
  static constexpr int kHostChunks = 4;
  int32_t *chunk_order = nullptr;
  std::vector<int64_t> chunk_off;  // kHostChunks + 1 offsets into chunk_order (= panel ranges)
  cudaStream_t side = nullptr;
  cudaEvent_t chunk_ev[kHostChunks] = {};
  // K-split item lists (wide plans): half 0 holds the entries whose column is
  // below ksplit, half 1 the rest, so the host entry point can start on the
  // first rows of B while the second ones are still being copied.
  int64_t ksplit = 0;                         // 0: no split lists
  int2 *khalf_items[2] = {nullptr, nullptr};  // one allocation
  int32_t *khalf_ptr[2] = {nullptr, nullptr};
  cudaStream_t side2 = nullptr;
  cudaEvent_t host_ev[5] = {};
  std::vector<int64_t> work;  // per local panel, for batch scheduling
  // Dense-tile tensor-core path (kernel == 3): swizzled A_hi/A_lo tiles of
  // the kept (row block, K-chunk) pairs, per-call B tile images, error word.
  uint8_t *a_tiles = nullptr;
  int32_t *rb_ptr = nullptr, *rb_chunk = nullptr;
  uint8_t *b_tiles = nullptr;
  int *status = nullptr;
  int64_t row_blocks = 0, kept_chunks = 0;
  int4 *dense_tasks = nullptr;  // {0, row block, n tile, kept chunks}, heaviest first
  int64_t dense_ntasks = 0;
  int dense_split = 1;          // CTAs (cluster) per task
  bool dense_bf16 = false;      // bf16 tiles (SC_PLAN_DENSE_BF16) instead of the fp32-exact splits
  int dense_mode = 0;           // sc::dense::kModeTf32x3 / kModeBf16 / kModeBf16x3
  int value_type = 0;           // stored values: 0 fp32, 1 fp16, 2 bf16 (compact small-B records)
  int record_vt = 0;            // record layout the narrow kernel reads: value_type, 3 split blocks, 4 lane blocks
  bool xstage = false;          // lane blocks read by the kernel that stages B in shared memory
  int4 *panel_meta = nullptr;   // xstage: per panel {first item, end item, first word, end word} | status
  uint32_t flags = 0;           // SC_PLAN_* given at creation
  ~sc_plan() {
    if (dev || stage_b || stage_c || a_tiles || chunk_order || panel_meta || side || khalf_items[0] || side2) {
      int prev;
      bool ok = cudaGetDevice(&prev) == cudaSuccess;
      if (ok && prev != device) cudaSetDevice(device);
      if (dev) cudaFree(dev);
      if (a_tiles) cudaFree(a_tiles);  // one allocation: tiles | rb_ptr | rb_chunk | b_tiles | status
      if (chunk_order) cudaFree(chunk_order);
      if (panel_meta) cudaFree(panel_meta);
      if (khalf_items[0]) cudaFree(khalf_items[0]);
      for (auto &e : host_ev)
        if (e) cudaEventDestroy(e);
      if (side2) cudaStreamDestroy(side2);
      for (auto &e : chunk_ev)
        if (e) cudaEventDestroy(e);
      if (side) cudaStreamDestroy(side);
      if (stage_b) cudaFree(stage_b);
      if (stage_c) cudaFree(stage_c);
      if (ok && prev != device) cudaSetDevice(prev);
    }
  }
};

namespace {

using sc::WideFn;
using sc::NarrowFn;
using sc::LaneXFn;

// Shared-memory carveout preference (percent) applied once per kernel;
// SC_CARVEOUT overrides for tuning experiments (-1 = driver default).
int carveout_percent() {
  static const int v = [] {
    const char *e = getenv("SC_CARVEOUT");
    return e ? atoi(e) : -1;
  }();
  return v;
}

template <typename F>
F with_carveout(F fn) {
  static std::mutex mu;
  static std::vector<const void *> done;
  const int pct = carveout_percent();
  if (pct < 0) return fn;
  std::lock_guard<std::mutex> g(mu);
  const void *key = reinterpret_cast<const void *>(fn);
  if (std::find(done.begin(), done.end(), key) == done.end()) {
    cudaFuncSetAttribute(key, cudaFuncAttributePreferredSharedMemoryCarveout, pct);
    done.push_back(key);
  }
  return fn;
}

WideFn wide_kernel_raw(int km, int vec, bool batch) {
  switch (km) {
    case 1: return sc_wide_kernel_km1(vec, batch);
    case 2: return sc_wide_kernel_km2(vec, batch);
    case 3: return sc_wide_kernel_km3(vec, batch);
    case 4: return sc_wide_kernel_km4(vec, batch);
    case 5: return sc_wide_kernel_km5(vec, batch);
    default: return sc_wide_kernel_km6(vec, batch);
  }
}
WideFn wide_kernel(int km, int vec, bool batch) { return with_carveout(wide_kernel_raw(km, vec, batch)); }

LaneXFn lane_x_kernel(int km, int nb) {
  switch (km) {
    case 1: return sc_lane_x_kernel_km1(nb);
    case 2: return sc_lane_x_kernel_km2(nb);
    case 3: return sc_lane_x_kernel_km3(nb);
    case 4: return sc_lane_x_kernel_km4(nb);
    case 5: return sc_lane_x_kernel_km5(nb);
    default: return sc_lane_x_kernel_km6(nb);
  }
}

NarrowFn narrow_kernel(int km, int nb, int vt) {
  switch (km) {
    case 1: return sc_narrow_kernel_km1(nb, vt);
    case 2: return sc_narrow_kernel_km2(nb, vt);
    case 3: return sc_narrow_kernel_km3(nb, vt);
    case 4: return sc_narrow_kernel_km4(nb, vt);
    case 5: return sc_narrow_kernel_km5(nb, vt);
    default: return sc_narrow_kernel_km6(nb, vt);
  }
}

// Record layout of fp32 small-B plans with K <= 65536: lane blocks where the
// kernel that stages B in shared memory applies (SpMV, K fp32 within
// kXStageMaxBytes, at least xstage_min_panels() panels), split item blocks
// otherwise (N = 2 staged measured no faster than split blocks: 35.0 vs
// 34.8 us on the config-5 matrix).  SC_NARROW_LAYOUT=lane / split / rec (interleaved records; also
// SC_SPLIT_RECORDS=0) forces one (measurement switch).
constexpr int64_t kXStageMaxBytes = 160 * 1024;
int narrow_layout_override() {
  static const int v = [] {
    const char *r = getenv("SC_SPLIT_RECORDS");
    if (r && r[0] == '0') return 0;
    const char *e = getenv("SC_NARROW_LAYOUT");
    if (e && strcmp(e, "rec") == 0) return 0;
    if (e && strcmp(e, "split") == 0) return 3;
    if (e && strcmp(e, "lane") == 0) return 4;
    return -1;
  }();
  return v;
}
// Panels from which the staged kernel is used (small matrices keep one CTA
// per panel: a warp per panel leaves too few warps busy); SC_XSTAGE_MIN_PANELS.
int64_t xstage_min_panels() {
  static const int64_t v = [] {
    const char *e = getenv("SC_XSTAGE_MIN_PANELS");
    return (int64_t)(e ? atoll(e) : 1024);
  }();
  return v;
}
// Threads per CTA of the staged kernel (at most its launch bound);
// SC_XSTAGE_THREADS overrides it for tuning experiments.
int xstage_threads() {
  static const int v = [] {
    const char *e = getenv("SC_XSTAGE_THREADS");
    const int x = e ? atoi(e) : sc::kXMaxThreads;
    return (x >= 32 && x <= sc::kXMaxThreads && x % 32 == 0) ? x : sc::kXMaxThreads;
  }();
  return v;
}

int pow2_at_least(int64_t x) {
  int p = 1;
  while (p < x && p < (1 << 30)) p <<= 1;
  return p;
}

// Warps the schedule aims to put in flight (B200: 148 SMs); SC_TARGET_WARPS
// overrides it for tuning experiments.
int64_t target_warps() {
  static const int64_t v = [] {
    const char *e = getenv("SC_TARGET_WARPS");
    long long x = e ? atoll(e) : 0;
    return (int64_t)(x > 0 ? x : 148 * 64);
  }();
  return v;
}

// ---- dense-tile tensor-core path selection and tile building

// SC_DENSE=0 disables, =1 forces (when N is a multiple of 128); by default
// the path is used where the dense tiles cost less than the sparse gather:
// density >= 15% (measured: the 20%-dense layer stack runs 2x faster dense,
// the 10%-dense config-3 layers 1.7x slower) and a densified A that fits
// comfortably in host memory.
// CTAs per dense task (split K over a cluster) so that small matrices still
// spread over the SMs, keeping >= 4 kept chunks per CTA.
int dense_split_for(const std::vector<int4> &tasks) {
  int64_t chunks = 0;
  for (auto &t : tasks) chunks += t.w;
  const int64_t nt = (int64_t)tasks.size();
  if (nt == 0) return 1;
  int sp = 1;
  while (sp < sc::dense::kMaxSplit && nt * sp < 148 && chunks / (nt * sp * 2) >= 4) sp <<= 1;
  return sp;
}

sc::dense::DenseMat dense_mat(const sc_plan *p, const float *B, int64_t ldb, float *C, int64_t ldc) {
  sc::dense::DenseMat m;
  m.a_tiles = p->a_tiles;
  m.rb_ptr = p->rb_ptr;
  m.rb_chunk = p->rb_chunk;
  m.b_tiles = p->b_tiles;
  m.B = B;
  m.ldb = ldb;
  m.C = C;
  m.ldc = ldc;
  m.rows = p->rows;
  m.k_rows = (int)p->cols;
  m.n_cols = (int)p->n;
  const int bk = sc::dense::mode_bk(p->dense_mode);
  m.k_chunks = (int)((p->cols + bk - 1) / bk);
  m.n_tiles = (int)(p->n / sc::dense::kBN);
  m.bf16 = p->dense_mode;
  m.starve = (p->flags & SC_PLAN_TEST_STARVE) ? 1 : 0;
  return m;
}

// Exact-fp32 tile mode of dense plans: SC_DENSE_MODE=0 3xTF32, =2 3xBF16
// (measurement switch; the default is the one measured faster).
int default_dense_mode() {
  static const int v = [] {
    const char *e = getenv("SC_DENSE_MODE");
    if (e && e[0] == '0') return sc::dense::kModeTf32x3;
    if (e && e[0] == '2') return sc::dense::kModeBf16x3;
    return SC_DEFAULT_DENSE_MODE;
  }();
  return v;
}

bool use_dense(const sc_plan &p, const sc_cf &cf) {
  const char *e = getenv("SC_DENSE");
  if (p.flags & SC_PLAN_DENSE_OFF) return false;
  if (!(p.flags & SC_PLAN_DENSE_ON) && e && e[0] == '0') return false;
  if (p.n % sc::dense::kBN != 0) return false;
  const double cells = (double)p.rows * (double)p.cols;
  if (cells <= 0 || (double)p.rows * p.cols * 4.0 > 2e9) return false;
  if (p.flags & SC_PLAN_DENSE_ON) return true;
  if (e && e[0] == '1') return true;
  return (double)p.nnz / cells >= 0.15;
}

void build_dense(sc_plan &p, const sc_cf &cf, int64_t pb, const std::vector<int> &rowbits) {
  using namespace sc::dense;
  const int km = (int)p.km;
  const int64_t rows = p.rows, K = p.cols;
  const int64_t rbs = (rows + kBM - 1) / kBM;
  const int mode = p.dense_mode;
  const int bk = mode_bk(mode);             // K per chunk (one 128-byte tile row)
  const int images = mode_images(mode);     // tf32: head + tail; bf16: one; bf16 x3: three parts
  const int kcs = (int)((K + bk - 1) / bk);
  // densify this plan's rows
  std::vector<float> A((size_t)rbs * kBM * K, 0.f);
  for (int64_t lp = 0; lp < p.panels; ++lp) {
    const int64_t gp = pb + lp;
    for (size_t g = 0; g < cf.pats.size(); ++g) {
      const sc_pattern &pt = cf.pats[g];
      const int P = pt.popcount;
      int rowsof[32];
      int n = 0;
      for (int j = 0; j < km && n < 32; ++j)
        if (rowbits[g] >> j & 1) rowsof[n++] = j;
      for (int32_t j = pt.rpp[gp]; j < pt.rpp[gp + 1]; ++j)
        for (int q = 0; q < P; ++q) {
          if (pt.pad[(size_t)j * P + q]) continue;
          const int64_t r = lp * km + rowsof[q];
          if (r < rows) A[(size_t)r * K + pt.cb[j]] += pt.vals[(size_t)j * P + q];
        }
    }
  }
  // kept (row block, chunk) pairs and their swizzled images: [hi | lo] fp32
  // TF32 pairs, or one bf16 image
  std::vector<int32_t> rb_ptr(rbs + 1, 0), rb_chunk;
  std::vector<uint8_t> tiles;
  for (int64_t b = 0; b < rbs; ++b) {
    for (int kc = 0; kc < kcs; ++kc) {
      bool any = false;
      for (int r = 0; r < kBM && !any; ++r)
        for (int k = 0; k < bk; ++k) {
          const int64_t gk = (int64_t)kc * bk + k;
          if (gk < K && A[(size_t)(b * kBM + r) * K + gk] != 0.f) { any = true; break; }
        }
      if (!any) continue;
      rb_chunk.push_back(kc);
      const size_t off = tiles.size();
      const size_t tb = (size_t)mode_tile_bytes(mode);
      tiles.resize(off + (size_t)images * tb, 0);
      for (int r = 0; r < kBM; ++r)
        for (int k = 0; k < bk; ++k) {
          const int64_t gk = (int64_t)kc * bk + k;
          const float x = gk < K ? A[(size_t)(b * kBM + r) * K + gk] : 0.f;
          if (mode == kModeBf16x3) {
            uint16_t h[3];
            bf16x3_split(x, h);
            for (int j = 0; j < 3; ++j) memcpy(&tiles[off + j * tb + swz_offset_bf16_64(r, k)], &h[j], 2);
          } else if (mode == kModeBf16) {
            const uint16_t h = bf16_bits(x);
            memcpy(&tiles[off + swz_offset_bf16(r, k)], &h, 2);
          } else {
            const float h = tf32_round(x), l = tf32_round(x - h);
            memcpy(&tiles[off + swz_offset(r, k)], &h, 4);
            memcpy(&tiles[off + kTileBytes + swz_offset(r, k)], &l, 4);
          }
        }
    }
    rb_ptr[b + 1] = (int32_t)rb_chunk.size();
  }
  const int nts = (int)(p.n / kBN);
  const size_t b_bytes = (size_t)nts * kcs * images * mode_tile_bytes(mode);
  std::vector<int4> tasks;
  for (int64_t b = 0; b < rbs; ++b)
    for (int t = 0; t < nts; ++t) tasks.push_back(make_int4(0, (int)b, t, rb_ptr[b + 1] - rb_ptr[b]));
  std::stable_sort(tasks.begin(), tasks.end(), [](const int4 &x, const int4 &y) { return x.w > y.w; });
  p.dense_split = dense_split_for(tasks);
  auto al = [](size_t x) { return (x + 1023) & ~(size_t)1023; };
  const size_t o_ptr = al(std::max<size_t>(tiles.size(), 1024));
  const size_t o_chunk = o_ptr + al((rbs + 1) * 4);
  const size_t o_b = o_chunk + al(std::max<size_t>(rb_chunk.size(), 1) * 4);
  const size_t o_tasks = o_b + al(std::max<size_t>(b_bytes, 1024));
  const size_t o_status = o_tasks + al(std::max<size_t>(tasks.size(), 1) * sizeof(int4));
  uint8_t *base = nullptr;
  cuda_check(cudaMalloc(&base, o_status + 1024), "cudaMalloc(dense tiles)");
  p.a_tiles = base;
  p.rb_ptr = reinterpret_cast<int32_t *>(base + o_ptr);
  p.rb_chunk = reinterpret_cast<int32_t *>(base + o_chunk);
  p.b_tiles = base + o_b;
  p.status = reinterpret_cast<int *>(base + o_status);
  p.dense_tasks = reinterpret_cast<int4 *>(base + o_tasks);
  p.dense_ntasks = (int64_t)tasks.size();
  if (!tasks.empty())
    cuda_check(cudaMemcpy(p.dense_tasks, tasks.data(), tasks.size() * sizeof(int4), cudaMemcpyHostToDevice),
               "upload tasks");
  if (!tiles.empty()) cuda_check(cudaMemcpy(base, tiles.data(), tiles.size(), cudaMemcpyHostToDevice), "upload tiles");
  cuda_check(cudaMemcpy(p.rb_ptr, rb_ptr.data(), rb_ptr.size() * 4, cudaMemcpyHostToDevice), "upload tiles");
  if (!rb_chunk.empty())
    cuda_check(cudaMemcpy(p.rb_chunk, rb_chunk.data(), rb_chunk.size() * 4, cudaMemcpyHostToDevice), "upload tiles");
  cuda_check(cudaMemset(p.status, 0, 16), "clear status");  // status | task counter | done counter
  p.row_blocks = rbs;
  p.kept_chunks = (int64_t)rb_chunk.size();
  p.dev_bytes += o_status + 1024;
  p.kernel = 3;
}

// K-split item lists for the host entry point.  Each item's entries are
// split at the first column >= ksplit; the cut is moved down to keep the
// second part's records 16-byte aligned (the wide kernel stages records in
// 16-byte pieces), which only moves a few low-column entries into half 1 --
// half 1 runs after all of B has arrived, so that is still correct.  Entries
// of an item must be in increasing column order (the coarsener's merge order);
// otherwise no split lists are built.
void build_ksplit(sc_plan &p, const std::vector<uint32_t> &recs, const std::vector<int2> &items,
                  const std::vector<int32_t> &item_ptr) {
  const int64_t kc = (p.cols / 2) & ~(int64_t)63;
  std::vector<int2> half[2];
  std::vector<int32_t> hptr[2];
  hptr[0].push_back(0);
  hptr[1].push_back(0);
  for (int64_t lp = 0; lp < p.panels; ++lp) {
    for (int32_t it = item_ptr[lp]; it < item_ptr[lp + 1]; ++it) {
      const int2 item = items[it];
      const int mask = item.y & 0xffff, len = item.y >> 16;
      const int S = sc::rec_stride(__builtin_popcount(mask));
      int j = 0;
      int64_t prev = -1;
      for (int e = 0; e < len; ++e) {
        const int64_t col = recs[(size_t)item.x + (size_t)e * S];
        if (col < prev) return;  // not column-sorted: no split lists
        prev = col;
        if (col < kc) j = e + 1;
      }
      const int step = S == 2 ? 2 : 1;  // 16-byte aligned start of the second part
      const int j0 = j - j % step;
      if (j0 > 0) half[0].push_back(make_int2(item.x, mask | (j0 << 16)));
      if (len - j0 > 0) half[1].push_back(make_int2(item.x + j0 * S, mask | ((len - j0) << 16)));
    }
    hptr[0].push_back((int32_t)half[0].size());
    hptr[1].push_back((int32_t)half[1].size());
  }
  auto al = [](size_t x) { return (x + 255) & ~(size_t)255; };
  size_t off[4], tot = 0;
  for (int h = 0; h < 2; ++h) {
    off[2 * h] = tot;
    tot += al(std::max<size_t>(1, half[h].size()) * sizeof(int2));
    off[2 * h + 1] = tot;
    tot += al(hptr[h].size() * 4);
  }
  char *base = nullptr;
  cuda_check(cudaMalloc(&base, tot), "cudaMalloc(K-split items)");
  for (int h = 0; h < 2; ++h) {
    p.khalf_items[h] = reinterpret_cast<int2 *>(base + off[2 * h]);
    p.khalf_ptr[h] = reinterpret_cast<int32_t *>(base + off[2 * h + 1]);
    if (!half[h].empty())
      cuda_check(cudaMemcpy(p.khalf_items[h], half[h].data(), half[h].size() * sizeof(int2), cudaMemcpyHostToDevice),
                 "upload K-split items");
    cuda_check(cudaMemcpy(p.khalf_ptr[h], hptr[h].data(), hptr[h].size() * 4, cudaMemcpyHostToDevice),
               "upload K-split items");
  }
  p.ksplit = kc;
  p.dev_bytes += tot;
}

// Warps per CTA (<= max_w, powers of two) minimising waves(W) * (2 + items/W)
// for `units` CTAs averaging `avg_items` work items each; the device must be
// current.
int wave_model_warps(int km, int vec, bool batch, int64_t units, double avg_items, int max_w) {
  int dev = 0, sms = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  WideFn fn = wide_kernel(km, vec, batch);
  double best = 0;
  int best_w = 1;
  for (int w = 1; w <= max_w; w <<= 1) {
    int per_sm = 0;
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, 32 * w, sc::wide_smem_bytes(w, km, vec));
    const int64_t resident = std::max<int64_t>(1, (int64_t)per_sm * sms);
    const double t = (double)((units + resident - 1) / resident) * (2.0 + avg_items / w);
    if (w == 1 || t < best) {
      best = t;
      best_w = w;
    }
  }
  return best_w;
}

sc_plan *build_plan(const sc_cf &cf, int32_t n, int32_t device, int64_t pb, int64_t pe, uint32_t flags) {
  const int km = cf.kernel_m;
  require(km >= 1 && km <= 6, SC_ERR_UNSUPPORTED, "plans support kernel_m 1..6");
  require(n >= 1, SC_ERR_ARG, "n_cols_b must be >= 1");
  const int64_t total_panels = ((int64_t)cf.num_rows + km - 1) / km;
  if (pb < 0) pb = 0;
  if (pe < 0 || pe > total_panels) pe = total_panels;
  require(pb <= pe, SC_ERR_ARG, "panel range is empty or reversed");
  const int np = (int)cf.pats.size();

  // Validate every block before anything reaches the device.
  std::vector<int> rowbits(np, 0);
  for (int g = 0; g < np; ++g) {
    const sc_pattern &pt = cf.pats[g];
    require((int)pt.mask.size() == km, SC_ERR_UNSUPPORTED,
            "pattern mask length differs from kernel_m (custom dictionary)");
    for (int j = 0; j < km; ++j)
      if (pt.mask[j] == '1') rowbits[g] |= 1 << j;
    require(pt.popcount >= 1 && pt.popcount == __builtin_popcount(rowbits[g]), SC_ERR_FORMAT,
            "pattern mask must have at least one row");
    require((int64_t)pt.rpp.size() == total_panels + 1, SC_ERR_FORMAT,
            "row-panel pointer length differs from ceil(rows/kernel_m)+1");
    require(pt.rpp[0] == 0, SC_ERR_FORMAT, "row-panel pointer must start at 0");
    for (size_t i = 0; i + 1 < pt.rpp.size(); ++i)
      require(pt.rpp[i] <= pt.rpp[i + 1], SC_ERR_FORMAT, "row-panel pointer must be non-decreasing");
    require((size_t)pt.rpp.back() <= pt.cb.size(), SC_ERR_FORMAT, "row-panel pointer exceeds column list");
    require((size_t)pt.rpp.back() * pt.popcount <= pt.vals.size(), SC_ERR_FORMAT,
            "value list shorter than columns x popcount");
    require(pt.pad.size() == pt.vals.size(), SC_ERR_FORMAT, "internal: pad flags missing");
  }

  auto plan = std::make_unique<sc_plan>();
  plan->device = device;
  plan->flags = flags;
  plan->dense_bf16 = (flags & SC_PLAN_DENSE_BF16) != 0;
  plan->dense_mode = plan->dense_bf16 ? sc::dense::kModeBf16 : default_dense_mode();
  plan->value_type = (flags & SC_PLAN_VALUES_F16) ? 1 : ((flags & SC_PLAN_VALUES_BF16) ? 2 : 0);
  const bool compact = plan->value_type != 0;
  // fp32 small-B plans with K <= 65536: split item blocks (16-bit columns,
  // then exactly P values per entry); SC_SPLIT_RECORDS=0 keeps the
  // interleaved records (measurement switch).
  int layout = 0;
  bool xstage = false;
  if (!compact && (n == 1 || n == 2 || n == 4) && cf.num_cols <= 65536) {
    xstage = n == 1 && (int64_t)cf.num_cols * 4 <= kXStageMaxBytes && (pe - pb) >= xstage_min_panels();
    layout = narrow_layout_override();
    if (layout < 0) layout = xstage ? 4 : 3;
    xstage = xstage && layout == 4;
  }
  plan->xstage = xstage;
  const bool split = layout == 3;
  const bool lanes = layout == 4;
  plan->record_vt = layout != 0 ? layout : plan->value_type;
  if (compact) {
    require(n == 1 || n == 2 || n == 4, SC_ERR_UNSUPPORTED,
            "16-bit value records are for the small-B / SpMV kernel (n_cols_b 1, 2 or 4)");
    require(cf.num_cols <= 65536, SC_ERR_UNSUPPORTED, "16-bit value records need K <= 65536 (16-bit columns)");
  }
  plan->km = km;
  plan->n = n;
  plan->cols = cf.num_cols;
  plan->panels = pe - pb;
  plan->rows = std::max<int64_t>(0, std::min<int64_t>(cf.num_rows, pe * km) - pb * km);

  // entries per item: 32 for the wide kernel (one cp.async stage), 128 for the
  // narrow kernel (four entries per lane)
  const int64_t item_cap = (n == 1 || n == 2 || n == 4) ? sc::kNarrowItemEntries : sc::kItemEntries;
  std::vector<uint32_t> recs;
  std::vector<uint16_t> recs16;  // compact form: recs16[i] encodes recs[i] (same indexing, halfwords)
  std::vector<int2> items;
  std::vector<int32_t> item_ptr(plan->panels + 1, 0);
  std::vector<int64_t> work(plan->panels, 0);
  struct LaneGroup {
    std::vector<uint8_t> masks;  // per block
    std::vector<uint32_t> cols;  // 16 per block
    std::vector<uint32_t> vals;  // kLaneSlots per block
  };
  std::vector<LaneGroup> lane_groups(km + 1);
  for (int64_t lp = 0; lp < plan->panels; ++lp) {
    const int64_t gp = pb + lp;
    for (int g = 0; g < np; ++g) {
      const sc_pattern &pt = cf.pats[g];
      const int P = pt.popcount;
      const int S = sc::rec_stride(P);
      int64_t seg_start = -1;
      int64_t seg_len = 0;
      std::vector<uint32_t> seg_cols, seg_vals;  // split mode: the segment's columns and value bits
      auto close_items = [&]() {
        if (lanes) {  // blocks of U entries of this mask, emitted per popcount at the panel's end
          const int U = sc::lane_entries(P);
          LaneGroup &lg = lane_groups[P];
          for (int64_t e = 0; e < seg_len; e += U) {
            const int len = (int)std::min<int64_t>(U, seg_len - e);
            lg.masks.push_back((uint8_t)rowbits[g]);
            const size_t c0 = lg.cols.size(), v0 = lg.vals.size();
            lg.cols.resize(c0 + 16, 0u);
            lg.vals.resize(v0 + sc::kLaneSlots, 0u);
            for (int i = 0; i < len; ++i) {
              lg.cols[c0 + i] = seg_cols[e + i];
              for (int q = 0; q < P; ++q) lg.vals[v0 + (size_t)i * P + q] = seg_vals[(e + i) * P + q];
            }
          }
          return;
        }
        if (split) {
          for (int64_t e = 0; e < seg_len; e += item_cap) {
            const int len = (int)std::min<int64_t>(item_cap, seg_len - e);
            while (recs.size() % 4) recs.push_back(0);
            const int64_t off = (int64_t)recs.size();
            require(off < (int64_t)INT32_MAX, SC_ERR_UNSUPPORTED, "record stream exceeds 8 GiB");
            for (int i = 0; i < len; i += 2)
              recs.push_back(seg_cols[e + i] | (i + 1 < len ? seg_cols[e + i + 1] << 16 : 0u));
            while (recs.size() % 4) recs.push_back(0);
            recs.insert(recs.end(), seg_vals.begin() + e * P, seg_vals.begin() + (e + len) * P);
            items.push_back(make_int2((int)off, rowbits[g] | (len << 16)));
          }
          return;
        }
        for (int64_t e = 0; e < seg_len; e += item_cap) {
          int len = (int)std::min<int64_t>(item_cap, seg_len - e);
          int64_t off = seg_start + e * S;
          require(off < (int64_t)UINT32_MAX / 2, SC_ERR_UNSUPPORTED, "record stream exceeds 8 GiB");
          items.push_back(make_int2((int)off, rowbits[g] | (len << 16)));
        }
      };
      for (int32_t j = pt.rpp[gp]; j < pt.rpp[gp + 1]; ++j) {
        bool all_pad = true;
        for (int p = 0; p < P; ++p) all_pad &= pt.pad[(size_t)j * P + p] != 0;
        if (all_pad) continue;
        const int32_t col = pt.cb[j];
        require(col >= 0 && col < cf.num_cols, SC_ERR_FORMAT, "column index out of range in CF");
        if (split || lanes) {
          seg_cols.push_back((uint32_t)col);
          for (int p = 0; p < P; ++p) {
            const float v = pt.vals[(size_t)j * P + p];
            uint32_t w;
            memcpy(&w, &v, 4);
            seg_vals.push_back(w);
            if (!pt.pad[(size_t)j * P + p]) plan->nnz++;
          }
          seg_len++;
          plan->entries++;
          work[lp] += P + 1;
          continue;
        }
        if (seg_start < 0) {
          // 16-byte aligned segment (8 words when compact: 16 bytes of halfwords)
          const size_t al = compact ? 8 : 4;
          while (recs.size() % al) recs.push_back(0);
          seg_start = (int64_t)recs.size();
        }
        recs.push_back((uint32_t)col);
        for (int p = 0; p < P; ++p) {
          float v = pt.vals[(size_t)j * P + p];
          uint32_t w;
          memcpy(&w, &v, 4);
          recs.push_back(w);
          if (!pt.pad[(size_t)j * P + p]) plan->nnz++;
        }
        for (int p = 1 + P; p < S; ++p) recs.push_back(0);
        if (compact) {
          recs16.resize(recs.size() - S, 0);  // alignment fill
          recs16.push_back((uint16_t)col);
          for (int p = 0; p < P; ++p) {
            const float v = pt.vals[(size_t)j * P + p];
            if (plan->value_type == 1) {
              require(std::fabs(v) <= 65504.f || v != v, SC_ERR_UNSUPPORTED,
                      "value outside the fp16 range; use SC_PLAN_VALUES_BF16");
              recs16.push_back(__half_as_ushort(__float2half_rn(v)));
            } else {
              recs16.push_back(__bfloat16_as_ushort(__float2bfloat16_rn(v)));
            }
          }
          for (int p = 1 + P; p < S; ++p) recs16.push_back(0);
        }
        seg_len++;
        plan->entries++;
        work[lp] += P + 2;
      }
      if (seg_len > 0) close_items();
    }
    if (lanes) {
      for (int P = 1; P <= km; ++P) {
        LaneGroup &lg = lane_groups[P];
        const int nblk = (int)lg.masks.size();
        for (int b0 = 0; b0 < nblk; b0 += 32) {
          const int nl = std::min(32, nblk - b0);
          while (recs.size() % 4) recs.push_back(0);
          const int64_t off = (int64_t)recs.size();
          require(off < (int64_t)INT32_MAX, SC_ERR_UNSUPPORTED, "record stream exceeds 8 GiB");
          recs.resize(recs.size() + sc::lane_item_words(nl, P), 0u);
          uint8_t *mk = reinterpret_cast<uint8_t *>(recs.data() + off);
          uint32_t *cw = recs.data() + off + 8;
          uint32_t *vw = cw + sc::lane_col_region(nl, P) / 4;
          for (int l = 0; l < nl; ++l) {
            const int blk = b0 + l;
            mk[l] = lg.masks[blk];
            for (int u = 0; u < sc::lane_entries(P); ++u)
              cw[sc::lane_col_word(nl, P, l, u)] |= lg.cols[(size_t)blk * 16 + u] << (16 * (u % 2));
            for (int q = 0; q < sc::kLaneSlots; ++q)  // chunk-major: chunk c of lane l at words (c * nl + l) * 4
              vw[((size_t)(q / 4) * nl + l) * 4 + q % 4] = lg.vals[(size_t)blk * sc::kLaneSlots + q];
          }
          items.push_back(make_int2((int)off, P | (nl << 8)));
        }
        lg.masks.clear();
        lg.cols.clear();
        lg.vals.clear();
      }
    }
    item_ptr[lp + 1] = (int32_t)items.size();
    work[lp] += 4 * (item_ptr[lp + 1] - item_ptr[lp]);
  }
  plan->items = (int64_t)items.size();
  while (recs.size() % 4) recs.push_back(0);
  if (recs.empty()) recs.assign(4, 0);
  if (compact) {
    recs16.resize(recs.size(), 0);
    // upload the halfword stream in place of the fp32 one
    recs.assign((recs16.size() + 1) / 2, 0);
    memcpy(recs.data(), recs16.data(), recs16.size() * 2);
    while (recs.size() % 4) recs.push_back(0);
    std::vector<uint16_t>().swap(recs16);
  }

  std::vector<int32_t> order(plan->panels);
  for (int64_t i = 0; i < plan->panels; ++i) order[i] = (int32_t)i;
  std::stable_sort(order.begin(), order.end(), [&](int32_t a, int32_t b) { return work[a] > work[b]; });
  plan->work = work;

  // Kernel family and CTA shape.
  int slices = 1;
  if (n == 1 || n == 2 || n == 4) {
    plan->kernel = 1;
  } else {
    plan->kernel = 2;
    plan->vec = n >= 128 ? 4 : (n >= 64 ? 2 : 1);
    slices = (int)((n + 32 * plan->vec - 1) / (32 * plan->vec));
  }
  {
    int64_t units = std::max<int64_t>(1, plan->panels * slices);
    int w = pow2_at_least((target_warps() + units - 1) / units);
    int64_t avg_items = plan->panels ? (plan->items + plan->panels - 1) / plan->panels : 1;
    w = std::min(w, pow2_at_least(std::max<int64_t>(1, avg_items)));
    plan->warps = std::max(1, std::min(w, 8));
  }

  // One device allocation: recs | items | item_ptr | order.
  DeviceGuard dg(device);
  // Warps per CTA from a wave model: time ~ waves(W) * (2 + items/W), where a
  // wave is the CTAs resident at once (occupancy at W warps) and "2" is the
  // per-CTA start-up chain (panel -> item range -> records -> B rows) in item
  // units.  Avoids e.g. a thin second wave for one rank's share of a
  // row-partitioned matrix.
  if (plan->kernel == 2 && plan->panels > 0)
    plan->warps = wave_model_warps(km, plan->vec, false, plan->panels * slices,
                                   (double)plan->items / (double)plan->panels, plan->warps);
  if (const char *e = getenv("SC_WIDE_WARPS"))  // tuning experiments: fixed warps per panel
    if (plan->kernel == 2 && atoi(e) >= 1 && atoi(e) <= 8) plan->warps = atoi(e);
  if (const char *e = getenv("SC_NARROW_WARPS"))  // tuning experiments: fixed warps per panel
    if (plan->kernel == 1 && atoi(e) >= 1 && atoi(e) <= 8) plan->warps = atoi(e);
  auto align = [](size_t x) { return (x + 255) & ~(size_t)255; };
  const size_t b_recs = align(recs.size() * 4);
  const size_t b_items = align(std::max<size_t>(1, items.size()) * sizeof(int2));
  const size_t b_ptr = align(item_ptr.size() * 4);
  const size_t b_order = align(std::max<size_t>(1, order.size()) * 4);
  plan->dev_bytes = b_recs + b_items + b_ptr + b_order;
  cuda_check(cudaMalloc(&plan->dev, plan->dev_bytes), "cudaMalloc(plan)");
  char *base = static_cast<char *>(plan->dev);
  plan->recs = reinterpret_cast<const uint32_t *>(base);
  plan->item_list = reinterpret_cast<const int2 *>(base + b_recs);
  plan->item_ptr = reinterpret_cast<const int32_t *>(base + b_recs + b_items);
  plan->order = reinterpret_cast<const int32_t *>(base + b_recs + b_items + b_ptr);
  cuda_check(cudaMemcpy(base, recs.data(), recs.size() * 4, cudaMemcpyHostToDevice), "upload records");
  if (!items.empty())
    cuda_check(cudaMemcpy(base + b_recs, items.data(), items.size() * sizeof(int2), cudaMemcpyHostToDevice),
               "upload items");
  cuda_check(cudaMemcpy(base + b_recs + b_items, item_ptr.data(), item_ptr.size() * 4, cudaMemcpyHostToDevice),
             "upload item pointers");
  if (!order.empty())
    cuda_check(cudaMemcpy(base + b_recs + b_items + b_ptr, order.data(), order.size() * 4,
                          cudaMemcpyHostToDevice),
               "upload panel order");
  if (plan->xstage) {
    std::vector<int4> pmh(std::max<int64_t>(1, plan->panels), make_int4(0, 0, 0, 0));
    for (int64_t i = 0; i < plan->panels; ++i) {
      const int a = item_ptr[i], b = item_ptr[i + 1];
      int w0 = 0, w1 = 0;
      if (b > a) {
        const int2 l = items[b - 1];
        w0 = items[a].x;
        w1 = l.x + (int)sc::lane_item_words(l.y >> 8, l.y & 0xff);
      }
      pmh[i] = make_int4(a, b, w0, w1);
    }
    // one allocation: panel table | status word of the staged kernel's bounded waits
    cuda_check(cudaMalloc(&plan->panel_meta, (pmh.size() + 1) * sizeof(int4)), "cudaMalloc(panel table)");
    cuda_check(cudaMemcpy(plan->panel_meta, pmh.data(), pmh.size() * sizeof(int4), cudaMemcpyHostToDevice),
               "upload panel table");
    plan->status = reinterpret_cast<int *>(plan->panel_meta + pmh.size());
    cuda_check(cudaMemset(plan->status, 0, sizeof(int4)), "clear status");
  }
  if (plan->kernel == 2 && plan->rows > 0 && use_dense(*plan, cf)) build_dense(*plan, cf, pb, rowbits);
  if (plan->kernel == 2 && plan->cols >= 4096 && plan->panels > 0) build_ksplit(*plan, recs, items, item_ptr);
  if (plan->kernel != 3 && plan->panels >= sc_plan::kHostChunks) {
    // panels split into kHostChunks contiguous row ranges, heaviest first inside each
    std::vector<int32_t> co;
    plan->chunk_off.push_back(0);
    for (int c = 0; c < sc_plan::kHostChunks; ++c) {
      const int64_t a0 = plan->panels * c / sc_plan::kHostChunks, a1 = plan->panels * (c + 1) / sc_plan::kHostChunks;
      std::vector<int32_t> part;
      for (int64_t q = a0; q < a1; ++q) part.push_back((int32_t)q);
      std::stable_sort(part.begin(), part.end(), [&](int32_t x, int32_t y) { return work[x] > work[y]; });
      co.insert(co.end(), part.begin(), part.end());
      plan->chunk_off.push_back((int64_t)co.size());
    }
    cuda_check(cudaMalloc(&plan->chunk_order, co.size() * 4), "cudaMalloc(chunk order)");
    cuda_check(cudaMemcpy(plan->chunk_order, co.data(), co.size() * 4, cudaMemcpyHostToDevice), "upload chunks");
  }
  return plan.release();
}

bool aligned(const void *p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

sc::WideArgs wide_args(const sc_plan *p, const float *B, int64_t ldb, float *C, int64_t ldc) {
  require(ldb <= (int64_t)(UINT32_MAX / 4), SC_ERR_UNSUPPORTED, "ldb too large (row pitch must be < 4 GiB)");
  sc::WideArgs a;
  a.recs = p->recs;
  a.items = p->item_list;
  a.item_ptr = p->item_ptr;
  a.B = B;
  a.C = C;
  a.ldc = ldc;
  a.rows = p->rows;
  a.ldb_bytes = (uint32_t)(ldb * 4);
  a.n_cols = (int)p->n;
  a.npeers = 0;
  for (int i = 0; i < sc::kMaxPeers; ++i) a.peers[i] = nullptr;
  return a;
}

void launch_panels(sc_plan *p, const float *B, int64_t ldb, float *C, int64_t ldc, int accumulate,
                   cudaStream_t stream, const int32_t *order, int64_t count);

void launch(sc_plan *p, const float *B, int64_t ldb, float *C, int64_t ldc, int accumulate,
            cudaStream_t stream) {
  launch_panels(p, B, ldb, C, ldc, accumulate, stream, p->order, p->panels);
}

// Runs the panels listed in order[0..count) (all panels: p->order).
void launch_panels(sc_plan *p, const float *B, int64_t ldb, float *C, int64_t ldc, int accumulate,
                   cudaStream_t stream, const int32_t *order, int64_t count) {
  require(ldb >= p->n && ldc >= p->n, SC_ERR_ARG, "leading dimension smaller than n_cols_b");
  if (count == 0) return;
  if (p->panels == 0 || p->rows == 0) return;  // nothing to write (C may be an empty buffer)
  require(B != nullptr && C != nullptr, SC_ERR_ARG, "null B or C");
  DeviceGuard dg(p->device);
  const int threads = 32 * p->warps;
  const int nb = (int)p->n;
  if (p->kernel == 3 && ldc % 4 == 0 && aligned(C, 16)) {
    const sc::dense::DenseMat m = dense_mat(p, B, ldb, C, ldc);
    int e = sc_dense_split_b(m, nullptr, 1, m.n_tiles * m.k_chunks, p->dense_mode, stream);
    cuda_check((cudaError_t)e, "B tile split launch");
    e = sc_dense_gemm(m, nullptr, p->dense_tasks, p->dense_ntasks, p->dense_split, p->dense_mode, accumulate,
                      p->status, stream);
    cuda_check((cudaError_t)e, "dense tile kernel launch");
    return;
  }
  if (p->kernel == 1 && p->xstage) {
    // B staged in shared memory; persistent CTAs whose warps stream whole panels
    LaneXFn fn = lane_x_kernel((int)p->km, nb);
    int dev = 0, sms = 0, smem_max = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    cudaDeviceGetAttribute(&smem_max, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    // warps per CTA: what shared memory allows, but no more than spreads the
    // panels over every SM (a warp takes whole panels)
    int warps = xstage_threads() / 32;
    while (warps > 1 && sc::lane_x_smem(p->cols, nb, warps) > (size_t)smem_max) --warps;
    warps = (int)std::max<int64_t>(1, std::min<int64_t>(warps, (count + sms - 1) / std::max(1, sms)));
    const size_t smem = sc::lane_x_smem(p->cols, nb, warps);
    require(smem <= (size_t)smem_max, SC_ERR_UNSUPPORTED, "B does not fit in shared memory");
    {
      // raise the kernel's dynamic shared memory limit once per (device, kernel, size)
      static std::mutex mu;
      static std::vector<std::pair<std::pair<int, const void *>, size_t>> done;
      std::lock_guard<std::mutex> lk(mu);
      size_t *have = nullptr;
      for (auto &d : done)
        if (d.first.first == dev && d.first.second == (const void *)fn) have = &d.second;
      if (!have || *have < smem) {
        cuda_check(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem),
                   "shared memory size of the staged kernel");
        if (have) *have = smem;
        else done.push_back({{dev, (const void *)fn}, smem});
      }
    }
    int per_sm = 0;
    cuda_check(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, 32 * warps, smem), "occupancy");
    const int64_t want = (count + warps - 1) / warps;
    const int64_t grid = std::max<int64_t>(1, std::min<int64_t>(want, (int64_t)std::max(1, per_sm) * sms));
    fn<<<dim3((unsigned)grid), 32 * warps, smem, stream>>>(p->recs, p->item_list, p->panel_meta, order, count, B,
                                                           ldb, p->cols, C, ldc, p->rows, accumulate, p->status,
                                                           (p->flags & SC_PLAN_TEST_STARVE) ? 1 : 0);
  } else if (p->kernel == 1) {
    if (ldb % nb == 0 && aligned(B, 4 * nb)) {
      NarrowFn fn = narrow_kernel((int)p->km, nb, p->record_vt);
      fn<<<dim3((unsigned)count), threads, 0, stream>>>(p->recs, p->item_list, p->item_ptr, order, B, ldb, C, ldc,
                                                         p->rows, accumulate);
    } else {
      // B rows not aligned for an nb-wide vector load: one single-column
      // launch per column of B (scalar loads at any alignment)
      NarrowFn fn = narrow_kernel((int)p->km, 1, p->record_vt);
      for (int q = 0; q < nb; ++q)
        fn<<<dim3((unsigned)count), threads, 0, stream>>>(p->recs, p->item_list, p->item_ptr, order, B + q, ldb,
                                                           C + q, ldc, p->rows, accumulate);
    }
  } else {
    int vec = p->kernel == 2 ? p->vec : 1;
    while (vec > 1 && !(p->n % vec == 0 && ldb % vec == 0 && ldc % vec == 0 && aligned(B, 4 * vec) &&
                        aligned(C, 4 * vec)))
      vec >>= 1;
    const int slices = (int)((p->n + 32 * vec - 1) / (32 * vec));
    WideFn fn = wide_kernel((int)p->km, vec, false);
    const size_t smem = sc::wide_smem_bytes(p->warps, (int)p->km, vec);
    fn<<<dim3((unsigned)count, slices), threads, smem, stream>>>(wide_args(p, B, ldb, C, ldc), nullptr, order,
                                                                 accumulate);
  }
  cuda_check(cudaGetLastError(), "kernel launch");
}

// SC_HOST_KSPLIT=0 turns the host entry point's K-split pipeline off.
bool host_ksplit_enabled() {
  static const bool v = [] {
    const char *e = getenv("SC_HOST_KSPLIT");
    return !(e && e[0] == '0');
  }();
  return v;
}

// One half of a K-split wide product over all panels: half 0 writes
// C = A[:, :ksplit] B[:ksplit]; half 1 adds A[:, ksplit:] B[ksplit:] to it and,
// when `host_c` is given, stores the finished tiles there as well.
void launch_khalf(sc_plan *p, int h, float *C, float *host_c, cudaStream_t stream, const int32_t *order,
                  int64_t count) {
  if (count <= 0) return;
  int vec = p->vec;
  while (vec > 1 && (p->n % vec != 0 || (host_c && !aligned(host_c, 4 * vec)))) vec >>= 1;
  const int slices = (int)((p->n + 32 * vec - 1) / (32 * vec));
  sc::WideArgs a = wide_args(p, p->stage_b, p->n, C, p->n);
  a.items = p->khalf_items[h];
  a.item_ptr = p->khalf_ptr[h];
  if (host_c) {
    a.npeers = 1;
    a.peers[0] = host_c;
  }
  WideFn fn = wide_kernel((int)p->km, vec, false);
  const size_t smem = sc::wide_smem_bytes(p->warps, (int)p->km, vec);
  fn<<<dim3((unsigned)count, slices), 32 * p->warps, smem, stream>>>(a, nullptr, order, h);
  cuda_check(cudaGetLastError(), "kernel launch");
}

// Waits for the current device, reads a device status word and clears it.
int take_status(int *dstatus) {
  cuda_check(cudaDeviceSynchronize(), "device synchronize");
  int v = 0;
  cuda_check(cudaMemcpy(&v, dstatus, 4, cudaMemcpyDeviceToHost), "read status");
  if (v) cuda_check(cudaMemset(dstatus, 0, 4), "clear status");
  return v;
}

// After a synchronous product: a dense-tile CTA whose bounded wait expired
// skipped its C stores, so the call must not report success.
void check_plan_status(sc_plan *p) {
  if (!p->status) return;
  const int v = take_status(p->status);
  if (v)
    throw sc_error(SC_ERR_DEVICE, "product kernel: a bounded device wait expired (status " + std::to_string(v) +
                                      "); C is incomplete");
}

}  // namespace

#define SC_API_BEGIN try {
#define SC_API_END                          \
  }                                         \
  catch (const sc_error &e) {               \
    sc_set_error(e.what());                 \
    return e.code;                          \
  }                                         \
  catch (const std::bad_alloc &) {          \
    sc_set_error("host allocation failed"); \
    return SC_ERR_NOMEM;                    \
  }                                         \
  catch (const std::exception &e) {         \
    sc_set_error(e.what());                 \
    return SC_ERR_ARG;                      \
  }                                         \
  return SC_OK;

extern "C" {

int sc_plan_create(const sc_cf *cf, int32_t n_cols_b, int32_t device, sc_plan **out) {
  SC_API_BEGIN
  require(cf != nullptr && out != nullptr, SC_ERR_ARG, "null argument");
  *out = build_plan(*cf, n_cols_b, device, 0, -1, 0);
  SC_API_END
}

int sc_plan_create_panels(const sc_cf *cf, int32_t n_cols_b, int32_t device, int64_t panel_begin,
                          int64_t panel_end, sc_plan **out) {
  SC_API_BEGIN
  require(cf != nullptr && out != nullptr, SC_ERR_ARG, "null argument");
  require(panel_begin >= 0 && panel_end >= panel_begin, SC_ERR_ARG, "bad panel range");
  *out = build_plan(*cf, n_cols_b, device, panel_begin, panel_end, 0);
  SC_API_END
}

int sc_plan_create_ex(const sc_cf *cf, int32_t n_cols_b, int32_t device, int64_t panel_begin, int64_t panel_end,
                      uint32_t flags, sc_plan **out) {
  SC_API_BEGIN
  require(cf != nullptr && out != nullptr, SC_ERR_ARG, "null argument");
  require(panel_begin == -1 ? panel_end == -1 : (panel_begin >= 0 && panel_end >= panel_begin), SC_ERR_ARG,
          "bad panel range (both -1 for the whole matrix)");
  require((flags & ~(uint32_t)(SC_PLAN_DENSE_OFF | SC_PLAN_DENSE_ON | SC_PLAN_DENSE_BF16 | SC_PLAN_VALUES_F16 |
                                SC_PLAN_VALUES_BF16 | SC_PLAN_TEST_STARVE)) == 0,
          SC_ERR_ARG, "unknown plan flag");
  require(!((flags & SC_PLAN_VALUES_F16) && (flags & SC_PLAN_VALUES_BF16)), SC_ERR_ARG,
          "SC_PLAN_VALUES_F16 and SC_PLAN_VALUES_BF16 exclude each other");
  require(!((flags & SC_PLAN_DENSE_OFF) && (flags & (SC_PLAN_DENSE_ON | SC_PLAN_DENSE_BF16))), SC_ERR_ARG,
          "SC_PLAN_DENSE_OFF excludes the other dense flags");
  *out = build_plan(*cf, n_cols_b, device, panel_begin == -1 ? 0 : panel_begin, panel_end, flags);
  SC_API_END
}

int sc_plan_get_info(const sc_plan *p, sc_plan_info *info) {
  SC_API_BEGIN
  require(p != nullptr && info != nullptr, SC_ERR_ARG, "null argument");
  info->rows = p->rows;
  info->cols = p->cols;
  info->n_cols_b = p->n;
  info->panels = p->panels;
  info->kernel_m = p->km;
  info->nnz = p->nnz;
  info->entries = p->entries;
  info->items = p->items;
  info->device_bytes = (int64_t)p->dev_bytes;
  info->kernel = p->kernel;
  info->warps_per_panel = p->warps;
  info->dense_bf16 = p->kernel == 3 && p->dense_bf16 ? 1 : 0;
  info->value_type = p->value_type;
  SC_API_END
}

int sc_spmm(sc_plan *p, const float *dB, int64_t ldb, float *dC, int64_t ldc, int32_t accumulate, void *stream) {
  SC_API_BEGIN
  require(p != nullptr, SC_ERR_ARG, "null plan");
  launch(p, dB, ldb, dC, ldc, accumulate, static_cast<cudaStream_t>(stream));
  SC_API_END
}

int sc_spmm_peers(sc_plan *p, const float *dB, int64_t ldb, float *dC, int64_t ldc, float *const *peer_C,
                  int32_t npeers, int *const *flag_dst, int32_t nflags, int32_t epoch, int32_t accumulate,
                  void *stream) {
  SC_API_BEGIN
  require(nflags >= 0 && nflags <= sc::kMaxPeers + 1 && (nflags == 0 || flag_dst != nullptr), SC_ERR_ARG,
          "nflags must be 0..8 with a flag pointer list");
  require(p != nullptr, SC_ERR_ARG, "null plan");
  require(npeers >= 0 && npeers <= sc::kMaxPeers, SC_ERR_ARG, "npeers must be 0..7");
  require(npeers == 0 || peer_C != nullptr, SC_ERR_ARG, "null peer list");
  require(p->kernel == 2, SC_ERR_UNSUPPORTED, "peer stores are implemented for the wide-B kernel (N not in {1,2,4})");
  require(ldb >= p->n && ldc >= p->n, SC_ERR_ARG, "leading dimension smaller than n_cols_b");
  if (p->panels == 0 || p->rows == 0) return SC_OK;
  require(dB != nullptr && dC != nullptr, SC_ERR_ARG, "null B or C");
  int vec = p->vec;
  bool al = true;
  for (int i = 0; i < npeers; ++i) al = al && peer_C[i] != nullptr && aligned(peer_C[i], 4 * vec);
  require(al, SC_ERR_ARG, "peer C pointers must be non-null and aligned like C");
  while (vec > 1 && !(p->n % vec == 0 && ldb % vec == 0 && ldc % vec == 0 && aligned(dB, 4 * vec) &&
                      aligned(dC, 4 * vec)))
    vec >>= 1;
  DeviceGuard dg(p->device);
  sc::WideArgs a = wide_args(p, dB, ldb, dC, ldc);
  a.npeers = npeers;
  for (int i = 0; i < npeers; ++i) a.peers[i] = peer_C[i];
  sc::FlagList fl;
  fl.n = nflags;
  for (int i = 0; i < nflags; ++i) {
    require(flag_dst[i] != nullptr && aligned(flag_dst[i], 4), SC_ERR_ARG, "bad flag pointer");
    fl.dst[i] = flag_dst[i];
  }
  const int slices = (int)((p->n + 32 * vec - 1) / (32 * vec));
  WideFn fn = wide_kernel((int)p->km, vec, false);
  fn<<<dim3((unsigned)p->panels, slices), 32 * p->warps, sc::wide_smem_bytes(p->warps, (int)p->km, vec),
       static_cast<cudaStream_t>(stream)>>>(a, nullptr, p->order, accumulate);
  cuda_check(cudaGetLastError(), "kernel launch");
  if (nflags > 0) {
    sc::signal_flags_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(fl, epoch);
    cuda_check(cudaGetLastError(), "kernel launch");
  }
  SC_API_END
}

int sc_wait_flags(const int *flags, int32_t n, int32_t epoch, int *status, void *stream) {
  SC_API_BEGIN
  require(flags != nullptr && status != nullptr && n >= 1 && n <= 1024, SC_ERR_ARG, "bad flag wait arguments");
  sc::wait_flags_kernel<<<1, 32 * ((n + 31) / 32), 0, static_cast<cudaStream_t>(stream)>>>(flags, n, epoch, status);
  cuda_check(cudaGetLastError(), "kernel launch");
  SC_API_END
}

int sc_spmv(sc_plan *p, const float *dx, float *dy, int32_t accumulate, void *stream) {
  SC_API_BEGIN
  require(p != nullptr, SC_ERR_ARG, "null plan");
  require(p->n == 1, SC_ERR_ARG, "sc_spmv needs a plan built with n_cols_b == 1");
  launch(p, dx, 1, dy, 1, accumulate, static_cast<cudaStream_t>(stream));
  SC_API_END
}

int sc_spmm_host(sc_plan *p, const float *hB, float *hC, void *stream) {
  SC_API_BEGIN
  require(p != nullptr && hB != nullptr && hC != nullptr, SC_ERR_ARG, "null argument");
  DeviceGuard dg(p->device);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const size_t bb = (size_t)p->cols * p->n * sizeof(float);
  const size_t cb = (size_t)p->rows * p->n * sizeof(float);
  if (!p->stage_b) cuda_check(cudaMalloc(&p->stage_b, std::max<size_t>(bb, 16)), "cudaMalloc(B staging)");
  if (!p->stage_c) cuda_check(cudaMalloc(&p->stage_c, std::max<size_t>(cb, 16)), "cudaMalloc(C staging)");
  if (!p->side) {
    cuda_check(cudaStreamCreateWithFlags(&p->side, cudaStreamNonBlocking), "create side stream");
    for (auto &e : p->chunk_ev) cuda_check(cudaEventCreateWithFlags(&e, cudaEventDisableTiming), "create event");
  }
  // C in page-locked host memory that this device can address: the kernel
  // stores C straight into it over the host link while it computes, so the
  // device-to-host transfer overlaps the whole product instead of following it.
  float *dC_host = nullptr;
  if (cb) {
    cudaPointerAttributes at{};
    if (cudaPointerGetAttributes(&at, hC) == cudaSuccess && at.type == cudaMemoryTypeHost && at.devicePointer)
      dC_host = static_cast<float *>(at.devicePointer);
    else
      cudaGetLastError();  // pageable memory: not an error, use the staged copy below
  }
  if (dC_host && p->kernel == 2 && p->ksplit > 0 && host_ksplit_enabled()) {
    // K-split pipeline: B rows [0, ksplit) arrive first (two concurrent
    // quarter copies), the half-0 product runs on them while rows
    // [ksplit, K) are still being copied, then the half-1 product adds the
    // rest and stores the finished C tiles into host memory as its second
    // (peer) destination.
    if (!p->side2) {
      cuda_check(cudaStreamCreateWithFlags(&p->side2, cudaStreamNonBlocking), "create side stream");
      for (auto &e : p->host_ev) cuda_check(cudaEventCreateWithFlags(&e, cudaEventDisableTiming), "create event");
    }
    const size_t row = (size_t)p->n * sizeof(float);
    const size_t k0 = (size_t)p->ksplit, K = (size_t)p->cols;
    const size_t cut[5] = {0, k0 / 2 * row, k0 * row, (k0 + (K - k0) / 2) * row, K * row};
    const char *hb = reinterpret_cast<const char *>(hB);
    char *db = reinterpret_cast<char *>(p->stage_b);
    auto copy = [&](int q, cudaStream_t st) {
      if (cut[q + 1] > cut[q])
        cuda_check(cudaMemcpyAsync(db + cut[q], hb + cut[q], cut[q + 1] - cut[q], cudaMemcpyHostToDevice, st),
                   "copy B to device");
    };
    cudaEvent_t *ev = p->host_ev;
    cuda_check(cudaEventRecord(ev[0], s), "record event");
    cuda_check(cudaStreamWaitEvent(p->side, ev[0], 0), "wait event");
    copy(0, s);
    cuda_check(cudaEventRecord(ev[1], s), "record event");
    copy(1, p->side);
    cuda_check(cudaEventRecord(ev[2], p->side), "record event");
    copy(2, p->side);
    cuda_check(cudaEventRecord(ev[3], p->side), "record event");
    cuda_check(cudaStreamWaitEvent(p->side2, ev[1], 0), "wait event");
    copy(3, p->side2);
    cuda_check(cudaEventRecord(ev[4], p->side2), "record event");
    cuda_check(cudaStreamWaitEvent(s, ev[2], 0), "wait event");
    launch_khalf(p, 0, p->stage_c, nullptr, s, p->order, p->panels);
    cuda_check(cudaStreamWaitEvent(s, ev[3], 0), "wait event");
    cuda_check(cudaStreamWaitEvent(s, ev[4], 0), "wait event");
    // One launch: the row-chunked alternative (C of one chunk crossing the
    // host link while the next computes) measured slower on config 5 --
    // 508 us whole, 583 / 734 / 1062 us in 2 / 4 / 8 chunks -- since each
    // chunk alone is a thin, latency-bound wave.
    launch_khalf(p, 1, p->stage_c, dC_host, s, p->order, p->panels);
    cuda_check(cudaStreamSynchronize(s), "stream synchronize");
    return SC_OK;  // wide plan: no device-side waits
  }
  if (bb >= (1u << 20)) {
    // two concurrent copies (this stream + the side stream): one DMA stream
    // alone does not fill the host link (measured 27-42 GB/s alone, 47 GB/s
    // as two halves)
    const size_t half = (bb / 2) & ~(size_t)4095;
    cuda_check(cudaEventRecord(p->chunk_ev[0], s), "record event");
    cuda_check(cudaStreamWaitEvent(p->side, p->chunk_ev[0], 0), "wait event");
    cuda_check(cudaMemcpyAsync(p->stage_b, hB, half, cudaMemcpyHostToDevice, s), "copy B to device");
    cuda_check(cudaMemcpyAsync(reinterpret_cast<char *>(p->stage_b) + half, reinterpret_cast<const char *>(hB) + half,
                               bb - half, cudaMemcpyHostToDevice, p->side),
               "copy B to device");
    cuda_check(cudaEventRecord(p->chunk_ev[1], p->side), "record event");
    cuda_check(cudaStreamWaitEvent(s, p->chunk_ev[1], 0), "wait event");
  } else if (bb) {
    cuda_check(cudaMemcpyAsync(p->stage_b, hB, bb, cudaMemcpyHostToDevice, s), "copy B to device");
  }
  if (dC_host) {
    launch(p, p->stage_b, p->n, dC_host, p->n, 0, s);
    cuda_check(cudaStreamSynchronize(s), "stream synchronize");
  } else if (!p->chunk_order || cb == 0) {
    launch(p, p->stage_b, p->n, p->stage_c, p->n, 0, s);
    if (cb) cuda_check(cudaMemcpyAsync(hC, p->stage_c, cb, cudaMemcpyDeviceToHost, s), "copy C to host");
    cuda_check(cudaStreamSynchronize(s), "stream synchronize");
  } else {
    // row chunks: kernel of chunk c on `s`, then its C rows to the host on a
    // side stream while the next chunks compute
    for (int c = 0; c < sc_plan::kHostChunks; ++c) {
      const int64_t a0 = p->chunk_off[c], a1 = p->chunk_off[c + 1];
      launch_panels(p, p->stage_b, p->n, p->stage_c, p->n, 0, s, p->chunk_order + a0, a1 - a0);
      cuda_check(cudaEventRecord(p->chunk_ev[c], s), "record event");
      cuda_check(cudaStreamWaitEvent(p->side, p->chunk_ev[c], 0), "wait event");
      const int64_t r0 = std::min<int64_t>(p->rows, a0 * p->km), r1 = std::min<int64_t>(p->rows, a1 * p->km);
      if (r1 > r0)
        cuda_check(cudaMemcpyAsync(hC + r0 * p->n, p->stage_c + r0 * p->n, (size_t)(r1 - r0) * p->n * sizeof(float),
                                   cudaMemcpyDeviceToHost, p->side),
                   "copy C to host");
    }
    cuda_check(cudaStreamSynchronize(p->side), "stream synchronize");
    cuda_check(cudaStreamSynchronize(s), "stream synchronize");
  }
  check_plan_status(p);
  SC_API_END
}

int sc_plan_status(sc_plan *p, int32_t *status) {
  SC_API_BEGIN
  require(p != nullptr && status != nullptr, SC_ERR_ARG, "null argument");
  *status = 0;
  if (!p->status) return SC_OK;
  DeviceGuard dg(p->device);
  *status = take_status(p->status);
  SC_API_END
}

void sc_plan_free(sc_plan *p) { delete p; }

}  // extern "C"

// A set of plans (same device, kernel_m and B width) run as one launch: one
// A batch splits its plans into two groups, each run by one launch:
//  * wide-B plans: one CTA per (matrix, panel), heaviest panels first;
//  * dense-tile plans: one B-split launch and one tensor-core launch over all
//    (matrix, row block, n tile) tasks, heaviest first.
struct sc_batch {
  int device = 0;
  int km = 0, vec = 1, warps = 1, slices = 1;
  int64_t n = 0;
  std::vector<sc_plan *> plans;
  std::vector<int> wide_ids, dense_ids;  // plan indices per group
  int64_t tasks = 0;                     // wide group: (matrix, panel) tasks
  int64_t dense_ntasks = 0;
  int dense_split = 1, dense_max_tiles = 0;
  int dense_mode = 0;  // all dense plans of a batch share one tile mode
  void *dev = nullptr;  // wide descs | wide order | dense mats | dense tasks | status
  sc::WideArgs *descs = nullptr;
  int2 *order = nullptr;
  sc::dense::DenseMat *dmats = nullptr;
  int4 *dtasks = nullptr;
  int *status = nullptr;
  bool bound = false;
  ~sc_batch() {
    if (dev) {
      int prev;
      bool ok = cudaGetDevice(&prev) == cudaSuccess;
      if (ok && prev != device) cudaSetDevice(device);
      cudaFree(dev);
      if (ok && prev != device) cudaSetDevice(prev);
    }
  }
};

extern "C" {

int sc_batch_create(sc_plan *const *plans, int32_t count, sc_batch **out) {
  SC_API_BEGIN
  require(plans != nullptr && out != nullptr && count >= 1, SC_ERR_ARG, "need at least one plan");
  auto b = std::make_unique<sc_batch>();
  const sc_plan *p0 = plans[0];
  require(p0 != nullptr, SC_ERR_ARG, "null plan");
  b->device = p0->device;
  b->n = p0->n;
  for (int32_t i = 0; i < count; ++i) {
    const sc_plan *p = plans[i];
    require(p != nullptr, SC_ERR_ARG, "null plan");
    require(p->kernel == 2 || p->kernel == 3, SC_ERR_UNSUPPORTED,
            "batches run wide-B plans (n_cols_b not in {1, 2, 4})");
    require(p->device == b->device && p->n == b->n, SC_ERR_UNSUPPORTED,
            "plans of a batch must share device and n_cols_b");
    if (p->kernel == 3) {
      if (b->dense_ids.empty()) b->dense_mode = p->dense_mode;
      require(p->dense_mode == b->dense_mode, SC_ERR_UNSUPPORTED,
              "dense-tile plans of a batch must share one precision (all bf16 or all 3xTF32)");
    }
    b->plans.push_back(plans[i]);
    (p->kernel == 3 ? b->dense_ids : b->wide_ids).push_back(i);
  }
  // wide group (one kernel_m, one vector width)
  std::vector<std::pair<int64_t, int2>> tasks;
  int64_t items = 0;
  if (!b->wide_ids.empty()) {
    const sc_plan *w0 = plans[b->wide_ids[0]];
    b->km = (int)w0->km;
    b->vec = w0->vec;
    b->slices = (int)((b->n + 32 * b->vec - 1) / (32 * b->vec));
    for (size_t gi = 0; gi < b->wide_ids.size(); ++gi) {
      const sc_plan *p = plans[b->wide_ids[gi]];
      require(p->km == b->km, SC_ERR_UNSUPPORTED, "wide-B plans of a batch must share kernel_m");
      items += p->items;
      for (int64_t lp = 0; lp < p->panels; ++lp) tasks.push_back({p->work[lp], make_int2((int)gi, (int)lp)});
    }
    std::stable_sort(tasks.begin(), tasks.end(), [](const std::pair<int64_t, int2> &x,
                                                    const std::pair<int64_t, int2> &y) { return x.first > y.first; });
  }
  b->tasks = (int64_t)tasks.size();
  {
    int64_t units = std::max<int64_t>(1, b->tasks * b->slices);
    int w = pow2_at_least((target_warps() + units - 1) / units);
    int64_t avg_items = b->tasks ? (items + b->tasks - 1) / b->tasks : 1;
    w = std::min(w, pow2_at_least(std::max<int64_t>(1, avg_items)));
    // (the single-plan wave model below mispredicted the mixed-size batches of
    // config 3: 25 -> 37 us; batches keep the warp-count rule)
    b->warps = std::max(1, std::min(w, 8));
  }
  // dense group
  std::vector<int4> dtasks;
  for (size_t gi = 0; gi < b->dense_ids.size(); ++gi) {
    const sc_plan *p = plans[b->dense_ids[gi]];
    const int nts = (int)(p->n / sc::dense::kBN);
    const int bk = sc::dense::mode_bk(p->dense_mode);
    const int kcs = (int)((p->cols + bk - 1) / bk);
    b->dense_max_tiles = std::max(b->dense_max_tiles, nts * kcs);
    std::vector<int32_t> rbp(p->row_blocks + 1);
    DeviceGuard dgp(p->device);
    cuda_check(cudaMemcpy(rbp.data(), p->rb_ptr, rbp.size() * 4, cudaMemcpyDeviceToHost), "read row blocks");
    for (int64_t r = 0; r < p->row_blocks; ++r)
      for (int t = 0; t < nts; ++t) dtasks.push_back(make_int4((int)gi, (int)r, t, rbp[r + 1] - rbp[r]));
  }
  std::stable_sort(dtasks.begin(), dtasks.end(), [](const int4 &x, const int4 &y) { return x.w > y.w; });
  b->dense_ntasks = (int64_t)dtasks.size();
  b->dense_split = dense_split_for(dtasks);

  DeviceGuard dg(b->device);
  auto align = [](size_t x) { return (x + 255) & ~(size_t)255; };
  const size_t bd = align(std::max<size_t>(1, b->wide_ids.size()) * sizeof(sc::WideArgs));
  const size_t bo = align(std::max<size_t>(1, tasks.size()) * sizeof(int2));
  const size_t bm = align(std::max<size_t>(1, b->dense_ids.size()) * sizeof(sc::dense::DenseMat));
  const size_t bt = align(std::max<size_t>(1, dtasks.size()) * sizeof(int4));
  cuda_check(cudaMalloc(&b->dev, bd + bo + bm + bt + 256), "cudaMalloc(batch)");
  char *base = static_cast<char *>(b->dev);
  b->descs = reinterpret_cast<sc::WideArgs *>(base);
  b->order = reinterpret_cast<int2 *>(base + bd);
  b->dmats = reinterpret_cast<sc::dense::DenseMat *>(base + bd + bo);
  b->dtasks = reinterpret_cast<int4 *>(base + bd + bo + bm);
  b->status = reinterpret_cast<int *>(base + bd + bo + bm + bt);
  cuda_check(cudaMemset(b->status, 0, 16), "clear status");  // status | task counter | done counter
  std::vector<int2> ord(tasks.size());
  for (size_t i = 0; i < tasks.size(); ++i) ord[i] = tasks[i].second;
  if (!ord.empty())
    cuda_check(cudaMemcpy(b->order, ord.data(), ord.size() * sizeof(int2), cudaMemcpyHostToDevice),
               "upload batch order");
  if (!dtasks.empty())
    cuda_check(cudaMemcpy(b->dtasks, dtasks.data(), dtasks.size() * sizeof(int4), cudaMemcpyHostToDevice),
               "upload dense tasks");
  *out = b.release();
  SC_API_END
}

int sc_batch_bind(sc_batch *b, const float *const *dB, const int64_t *ldb, float *const *dC,
                  const int64_t *ldc) {
  SC_API_BEGIN
  require(b != nullptr && dB != nullptr && dC != nullptr && ldb != nullptr && ldc != nullptr, SC_ERR_ARG,
          "null argument");
  std::vector<sc::WideArgs> d;
  std::vector<sc::dense::DenseMat> dm;
  for (size_t i = 0; i < b->plans.size(); ++i) {
    const sc_plan *p = b->plans[i];
    require(ldb[i] >= p->n && ldc[i] >= p->n, SC_ERR_ARG, "leading dimension smaller than n_cols_b");
    require(p->rows == 0 || (dB[i] != nullptr && dC[i] != nullptr), SC_ERR_ARG, "null B or C");
    if (p->kernel == 3) {
      require(ldc[i] % 4 == 0 && aligned(dC[i], 16), SC_ERR_ARG, "dense-tile plans need 16-byte aligned C rows");
      dm.push_back(dense_mat(p, dB[i], ldb[i], dC[i], ldc[i]));
    } else {
      require(ldb[i] % b->vec == 0 && ldc[i] % b->vec == 0 && aligned(dB[i], 4 * b->vec) &&
                  aligned(dC[i], 4 * b->vec),
              SC_ERR_ARG, "batch operands must be aligned to the vector width (16 bytes for n_cols_b >= 128)");
      d.push_back(wide_args(p, dB[i], ldb[i], dC[i], ldc[i]));
    }
  }
  DeviceGuard dg(b->device);
  if (!d.empty())
    cuda_check(cudaMemcpy(b->descs, d.data(), d.size() * sizeof(sc::WideArgs), cudaMemcpyHostToDevice),
               "upload batch operands");
  if (!dm.empty())
    cuda_check(cudaMemcpy(b->dmats, dm.data(), dm.size() * sizeof(sc::dense::DenseMat), cudaMemcpyHostToDevice),
               "upload batch operands");
  b->bound = true;
  SC_API_END
}

int sc_batch_status(sc_batch *b, int32_t *status) {
  SC_API_BEGIN
  require(b != nullptr && status != nullptr, SC_ERR_ARG, "null argument");
  *status = 0;
  if (!b->status) return SC_OK;
  DeviceGuard dg(b->device);
  *status = take_status(b->status);
  SC_API_END
}

int sc_batch_spmm(sc_batch *b, int32_t accumulate, void *stream) {
  SC_API_BEGIN
  require(b != nullptr, SC_ERR_ARG, "null batch");
  require(b->bound, SC_ERR_ARG, "sc_batch_bind must be called before sc_batch_spmm");
  DeviceGuard dg(b->device);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (b->dense_ntasks > 0) {
    sc::dense::DenseMat none{};
    int e = sc_dense_split_b(none, b->dmats, (int)b->dense_ids.size(), b->dense_max_tiles, b->dense_mode, s);
    cuda_check((cudaError_t)e, "B tile split launch");
    e = sc_dense_gemm(none, b->dmats, b->dtasks, b->dense_ntasks, b->dense_split, b->dense_mode, accumulate,
                      b->status, s);
    cuda_check((cudaError_t)e, "dense tile kernel launch");
  }
  if (b->tasks > 0) {
    WideFn fn = wide_kernel(b->km, b->vec, true);
    sc::WideArgs none{};
    fn<<<dim3((unsigned)b->tasks, b->slices), 32 * b->warps, sc::wide_smem_bytes(b->warps, b->km, b->vec), s>>>(
        none, b->descs, reinterpret_cast<const int32_t *>(b->order), accumulate);
    cuda_check(cudaGetLastError(), "kernel launch");
  }
  SC_API_END
}

void sc_batch_free(sc_batch *b) { delete b; }

}  // extern "C"

// A captured CUDA graph of `repeat` back-to-back products with fixed operands.
struct sc_graph {
  int device = 0;
  cudaGraph_t graph = nullptr;
  cudaGraphExec_t exec = nullptr;
  ~sc_graph() {
    int prev;
    bool ok = cudaGetDevice(&prev) == cudaSuccess;
    if (ok && prev != device) cudaSetDevice(device);
    if (exec) cudaGraphExecDestroy(exec);
    if (graph) cudaGraphDestroy(graph);
    if (ok && prev != device) cudaSetDevice(prev);
  }
};

namespace {

template <typename F>
sc_graph *capture(int device, int repeat, F issue) {
  require(repeat >= 1 && repeat <= 100000, SC_ERR_ARG, "repeat must be 1..100000");
  DeviceGuard dg(device);
  auto g = std::make_unique<sc_graph>();
  g->device = device;
  cudaStream_t s;
  cuda_check(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking), "create capture stream");
  cudaError_t e = cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal);
  if (e == cudaSuccess) {
    try {
      for (int r = 0; r < repeat; ++r) issue(s);
    } catch (...) {
      cudaGraph_t junk = nullptr;
      cudaStreamEndCapture(s, &junk);
      if (junk) cudaGraphDestroy(junk);
      cudaStreamDestroy(s);
      throw;
    }
    e = cudaStreamEndCapture(s, &g->graph);
  }
  cudaStreamDestroy(s);
  cuda_check(e, "stream capture");
  cuda_check(cudaGraphInstantiate(&g->exec, g->graph, 0), "graph instantiate");
  return g.release();
}

}  // namespace

extern "C" {

int sc_graph_capture_plan(sc_plan *p, const float *dB, int64_t ldb, float *dC, int64_t ldc, int32_t accumulate,
                          int32_t repeat, sc_graph **out) {
  SC_API_BEGIN
  require(p != nullptr && out != nullptr, SC_ERR_ARG, "null argument");
  *out = capture(p->device, repeat, [&](cudaStream_t s) { launch(p, dB, ldb, dC, ldc, accumulate, s); });
  SC_API_END
}

int sc_graph_capture_batch(sc_batch *b, int32_t accumulate, int32_t repeat, sc_graph **out) {
  SC_API_BEGIN
  require(b != nullptr && out != nullptr, SC_ERR_ARG, "null argument");
  *out = capture(b->device, repeat, [&](cudaStream_t s) {
    int st = sc_batch_spmm(b, accumulate, s);
    if (st != SC_OK) throw sc_error(st, sc_last_error_string());
  });
  SC_API_END
}

int sc_graph_launch(sc_graph *g, void *stream) {
  SC_API_BEGIN
  require(g != nullptr, SC_ERR_ARG, "null graph");
  DeviceGuard dg(g->device);
  cuda_check(cudaGraphLaunch(g->exec, static_cast<cudaStream_t>(stream)), "graph launch");
  SC_API_END
}

void sc_graph_free(sc_graph *g) { delete g; }

}  // extern "C"
