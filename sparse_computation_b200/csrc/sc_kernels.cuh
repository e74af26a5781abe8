// Pattern-specialised SpMM/SpMV kernels over the plan's device layout.
//
// Device layout (built by sc_plan.cu):
//   recs      uint32 words.  One record per (row panel, column) entry of a
//             pattern: [column, v_0 .. v_{P-1}, zero fill] with P the pattern
//             popcount and a stride of 2 words (P == 1), 4 words (P <= 3) or
//             8 words (P <= 7).  v_p is the value of the p-th set row of the
//             mask.  Coarsening padding (zero values, repeated column) is
//             dropped.  Every segment starts on a 16-byte boundary.
//   items     int2 {record offset in words, mask | len << 16}: up to 32
//             (wide kernel) or 128 (narrow kernel) consecutive entries of
//             one (panel, pattern) segment.
//   item_ptr  items of local panel i are [item_ptr[i], item_ptr[i+1]).
//   order     CTA -> panel map, heaviest panels first.
//
// One CTA owns one row panel (and, for wide B, one 32*VEC-column slice of C),
// so C is written once, without atomics and without pre-zeroing; the result
// does not depend on scheduling.  The reference instead launched one block
// per (panel, pattern) pair and combined them with atomicAdd
// (example_cuda/spmm_demo_gpu_utils.h:1411-1416).
//
// Specialisation: for kernel_m <= 4 the mask of each item is dispatched
// (binary search over compile-time masks) to a body instantiated for that
// exact mask, so the rows it feeds are compile-time register indices -- the
// role of the reference's generated PatternWith{m}NNZByRowPanel{P} functions
// (code_gen/spmm/spmm_format_code_generator.py:121-223).  For kernel_m 5 and
// 6 (31 and 63 masks) the body is specialised on the popcount, with the rows
// read from the mask once per item.
#pragma once

#include <cstdint>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

namespace sc {

// kernel_m up to which items dispatch to a body per pattern mask.
#ifndef SC_MASK_KM_MAX
#define SC_MASK_KM_MAX 4
#endif

#ifndef SC_NARROW_PREFETCH
#define SC_NARROW_PREFETCH 1
#endif

constexpr int kItemEntries = 32;        // wide kernel: entries per item
#ifndef SC_NARROW_UNROLL
#define SC_NARROW_UNROLL 4
#endif
constexpr int kNarrowUnroll = SC_NARROW_UNROLL;  // narrow kernel: entries per lane per pass
constexpr int kNarrowItemEntries = 32 * kNarrowUnroll;

__host__ __device__ constexpr int popc_c(int x) {
  int c = 0;
  for (; x; x >>= 1) c += x & 1;
  return c;
}
__host__ __device__ constexpr int rec_stride(int p) { return p == 1 ? 2 : (p <= 3 ? 4 : 8); }
// Row (panel-relative) of the p-th set bit of mask.  Loop-based so that it
// inlines and folds to a constant once the caller's loops are unrolled.
__host__ __device__ constexpr int nth_row(int mask, int p) {
  for (int r = 0; r < 32; ++r)
    if ((mask >> r) & 1) {
      if (p == 0) return r;
      --p;
    }
  return 0;
}

template <int VEC> struct VecT;
template <> struct VecT<1> { using T = float; };
template <> struct VecT<2> { using T = float2; };
template <> struct VecT<4> { using T = float4; };

template <int VEC>
__device__ __forceinline__ void load_vec(const float *p, float (&out)[VEC]) {
  if constexpr (VEC == 1) {
    out[0] = __ldg(p);
  } else if constexpr (VEC == 2) {
    float2 t = __ldg(reinterpret_cast<const float2 *>(p));
    out[0] = t.x; out[1] = t.y;
  } else {
    float4 t = __ldg(reinterpret_cast<const float4 *>(p));
    out[0] = t.x; out[1] = t.y; out[2] = t.z; out[3] = t.w;
  }
}

// B-row loads of the wide kernel: read-only, and (SC_B_NOALLOC) without
// allocating in L1 -- a B row is rarely re-read by the same SM before eviction.
template <int VEC>
__device__ __forceinline__ void load_b(const float *p, float (&out)[VEC]) {
#if SC_B_NOALLOC
  if constexpr (VEC == 1) {
    asm volatile("ld.global.nc.L1::no_allocate.f32 %0, [%1];" : "=f"(out[0]) : "l"(p));
  } else if constexpr (VEC == 2) {
    asm volatile("ld.global.nc.L1::no_allocate.v2.f32 {%0,%1}, [%2];" : "=f"(out[0]), "=f"(out[1]) : "l"(p));
  } else {
    asm volatile("ld.global.nc.L1::no_allocate.v4.f32 {%0,%1,%2,%3}, [%4];"
                 : "=f"(out[0]), "=f"(out[1]), "=f"(out[2]), "=f"(out[3]) : "l"(p));
  }
#else
  load_vec<VEC>(p, out);
#endif
}

// Read-only load: through the non-coherent global path, or a plain load
// when SM (the data was staged in shared memory).
template <bool SM, typename T>
__device__ __forceinline__ T ldro(const T *p) {
  if constexpr (SM) return *p;
  else return __ldg(p);
}

// Loads one record (column + P values) at `r`.
template <int P, bool SM = false>
__device__ __forceinline__ void load_rec(const uint32_t *__restrict__ r, int &col, float (&v)[P]) {
  constexpr int S = rec_stride(P);
  if constexpr (S == 2) {
    uint2 t = ldro<SM>(reinterpret_cast<const uint2 *>(r));
    col = (int)t.x; v[0] = __uint_as_float(t.y);
  } else if constexpr (S == 4) {
    uint4 t = ldro<SM>(reinterpret_cast<const uint4 *>(r));
    col = (int)t.x;
    uint32_t w[3] = {t.y, t.z, t.w};
#pragma unroll
    for (int p = 0; p < P; ++p) v[p] = __uint_as_float(w[p]);
  } else {
    uint4 a = ldro<SM>(reinterpret_cast<const uint4 *>(r));
    uint4 b = ldro<SM>(reinterpret_cast<const uint4 *>(r) + 1);
    col = (int)a.x;
    uint32_t w[7] = {a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
    for (int p = 0; p < P; ++p) v[p] = __uint_as_float(w[p]);
  }
}

// Compact 16-bit records (small-B plans created with SC_PLAN_VALUES_F16 or
// SC_PLAN_VALUES_BF16): the same record layout with 16-bit units --
// [column (uint16), v_0 .. v_{P-1} (fp16 or bf16), zero fill], stride S
// halfwords with the same S as above, so every record is half the bytes of
// its fp32 form and is read with one 4-, 8- or 16-byte load.  Offsets in the
// items count halfwords.  VT: 1 = fp16, 2 = bf16.
template <int VT>
__device__ __forceinline__ float half_bits_to_float(uint32_t h) {
  if constexpr (VT == 1) return __half2float(__ushort_as_half((unsigned short)h));
  else return __bfloat162float(__ushort_as_bfloat16((unsigned short)h));
}

// ------------------------------------------------------------ wide B ------
// One warp walks the entries of an item; lane l owns C columns
// [col0, col0+VEC) with col0 = slice*32*VEC + l*VEC.
//
// Per warp, the records of the next item are copied global -> shared with
// cp.async (16 B per lane, bypassing L1) while the current item is
// processed, so the record stream's DRAM latency overlaps the B loads.  Each
// entry's record is then read with one broadcast shared load, its B row
// address formed with one 32x32->64 multiply-add, and U entries' B rows are
// loaded (U independent 32*VEC-wide loads in flight) before the P*VEC FMAs.

constexpr int kMaxPeers = 7;

// Flag destinations of a completion signal: this rank's slot in each GPU's
// flag array (own GPU included).
struct FlagList {
  int n;
  int *dst[kMaxPeers + 1];
};

// Operands of one matrix for the wide kernel.
struct WideArgs {
  const uint32_t *recs;
  const int2 *items;
  const int32_t *item_ptr;
  const float *B;
  float *C;
  int64_t ldc;
  int64_t rows;
  uint32_t ldb_bytes;  // row pitch of B in bytes (< 4 GiB)
  int n_cols;
  // Peer copies of C (other GPUs' buffers mapped into this address space,
  // same layout and ldc): every C tile is also stored there, so the row
  // blocks of a row-partitioned product are exchanged by the kernel itself.
  int npeers;
  float *peers[kMaxPeers];
};

#ifndef SC_B_NOALLOC
#define SC_B_NOALLOC 0
#endif
// Entries whose B rows are loaded together (P <= 2), and the launch-bound
// CTA count (256-thread units: 4 -> at most 64 registers a thread).  Measured
// on config 5 (B200): U 8 / 3 CTAs 291 us, U 4 / 4 CTAs 251 us; more
// resident warps (5, 6, 8) were slower (292-420 us): the B rows they share
// through L1 are evicted sooner.  The batched kernel (many small matrices,
// one launch) keeps U 8 / 3 CTAs: config 3 measured 24.1 us there against
// 27.0 us with the single-matrix setting.
#ifndef SC_WIDE_U
#define SC_WIDE_U 4
#endif
#ifndef SC_WIDE_MINB
#define SC_WIDE_MINB 4
#endif
#ifndef SC_WIDE_BATCH_U
#define SC_WIDE_BATCH_U 8
#endif
#ifndef SC_WIDE_BATCH_MINB
#define SC_WIDE_BATCH_MINB 3
#endif
constexpr int kRecBufWords = kItemEntries * 8;  // one item of the widest stride

__device__ __forceinline__ void cp_async16(void *smem, const void *gmem) {
  const uint32_t s = (uint32_t)__cvta_generic_to_shared(smem);
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(s), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_1() { asm volatile("cp.async.wait_group 1;\n" ::: "memory"); }

// Warp-cooperative copy of an item's records (16-byte chunks) into `dst`.
__device__ __forceinline__ void copy_item_recs(uint32_t *dst, const uint32_t *__restrict__ recs, int2 item,
                                               int lane) {
  const int len = item.y >> 16;
  const int P = __popc(item.y & 0xffff);
  const int S = P == 1 ? 2 : (P <= 3 ? 4 : 8);
  const int chunks = (len * S + 3) >> 2;
  const uint4 *src = reinterpret_cast<const uint4 *>(recs + (uint32_t)item.x);
  for (int c = lane; c < chunks; c += 32) cp_async16(reinterpret_cast<uint4 *>(dst) + c, src + c);
}

template <int P>
__device__ __forceinline__ void lds_rec(const uint32_t *r, uint32_t &col, float (&v)[P]) {
  constexpr int S = rec_stride(P);
  if constexpr (S == 2) {
    const uint2 t = *reinterpret_cast<const uint2 *>(r);
    col = t.x; v[0] = __uint_as_float(t.y);
  } else if constexpr (S == 4) {
    const uint4 t = *reinterpret_cast<const uint4 *>(r);
    col = t.x;
    const uint32_t w[3] = {t.y, t.z, t.w};
#pragma unroll
    for (int p = 0; p < P; ++p) v[p] = __uint_as_float(w[p]);
  } else {
    const uint4 a = *reinterpret_cast<const uint4 *>(r);
    const uint4 b = *(reinterpret_cast<const uint4 *>(r) + 1);
    col = a.x;
    const uint32_t w[7] = {a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
    for (int p = 0; p < P; ++p) v[p] = __uint_as_float(w[p]);
  }
}

template <int KM, int MASK, int VEC, int UW>
__device__ __forceinline__ void seg_wide(const uint32_t *rbuf, int len, const char *__restrict__ Bcol,
                                         uint32_t ldb_bytes, bool active, float (&acc)[KM][VEC]) {
  constexpr int P = popc_c(MASK);
  constexpr int S = rec_stride(P);
  constexpr int U = P <= 2 ? UW : 4;
  for (int e0 = 0; e0 < len; e0 += U) {
    float v[U][P];
    float b[U][VEC];
    uint32_t col[U];
    if constexpr (S == 2 && U % 2 == 0) {
      // two 8-byte records per 16-byte broadcast load (one shared-memory
      // wavefront instead of two); the pair index is clamped into the item,
      // and a pair's second record past an odd length is the segment's zero
      // fill (copied with the item's last 16-byte chunk)
#pragma unroll
      for (int u = 0; u < U; u += 2) {
        const int e = min(e0 + u, (len - 1) & ~1);
        const uint4 t = *reinterpret_cast<const uint4 *>(rbuf + e * 2);
        col[u] = t.x;
        v[u][0] = __uint_as_float(t.y);
        col[u + 1] = t.z;
        v[u + 1][0] = __uint_as_float(t.w);
      }
    } else {
#pragma unroll
      for (int u = 0; u < U; ++u) lds_rec<P>(rbuf + min(e0 + u, len - 1) * S, col[u], v[u]);
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      if (active && e0 + u < len) {
        load_b<VEC>(reinterpret_cast<const float *>(Bcol + (uint64_t)col[u] * ldb_bytes), b[u]);
      } else {
#pragma unroll
        for (int q = 0; q < VEC; ++q) b[u][q] = 0.f;
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u)
#pragma unroll
      for (int p = 0; p < P; ++p)
#pragma unroll
        for (int q = 0; q < VEC; ++q)
          acc[nth_row(MASK, p)][q] = fmaf(v[u][p], b[u][q], acc[nth_row(MASK, p)][q]);
  }
}

// acc[row of the p-th set bit of mask] += t[p], for p < P (P == popc(mask)).
template <int KM, int P, int W>
__device__ __forceinline__ void add_rows(int mask, const float (&t)[P][W], float (&acc)[KM][W]) {
  int m = mask;
#pragma unroll
  for (int p = 0; p < P; ++p) {
    const int r = __ffs(m) - 1;
    m &= m - 1;
#pragma unroll
    for (int k = p; k <= KM - P + p; ++k)
      if (r == k) {
#pragma unroll
        for (int q = 0; q < W; ++q) acc[k][q] += t[p][q];
      }
  }
}

// Popcount-class body (kernel_m above SC_MASK_KM_MAX): specialised on the
// pattern's popcount P, with the rows of its P set bits taken from the mask
// at run time.  Sums go to item-local registers t[P][VEC] and are added to
// the panel's rows once per item; the p-th set bit lies in rows
// [p, KM-P+p], so the add is a short unrolled, predicated chain.
template <int KM, int P, int VEC, int UW>
__device__ __forceinline__ void seg_wide_pc(const uint32_t *rbuf, int len, const char *__restrict__ Bcol,
                                            uint32_t ldb_bytes, bool active, int mask, float (&acc)[KM][VEC]) {
  constexpr int S = rec_stride(P);
  constexpr int U = P <= 2 ? UW : 4;
  float t[P][VEC];
#pragma unroll
  for (int p = 0; p < P; ++p)
#pragma unroll
    for (int q = 0; q < VEC; ++q) t[p][q] = 0.f;
  for (int e0 = 0; e0 < len; e0 += U) {
    float v[U][P];
    float b[U][VEC];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      uint32_t col;
      lds_rec<P>(rbuf + min(e0 + u, len - 1) * S, col, v[u]);
      if (active && e0 + u < len) {
        load_b<VEC>(reinterpret_cast<const float *>(Bcol + (uint64_t)col * ldb_bytes), b[u]);
      } else {
#pragma unroll
        for (int q = 0; q < VEC; ++q) b[u][q] = 0.f;
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u)
#pragma unroll
      for (int p = 0; p < P; ++p)
#pragma unroll
        for (int q = 0; q < VEC; ++q) t[p][q] = fmaf(v[u][p], b[u][q], t[p][q]);
  }
  add_rows<KM, P, VEC>(mask, t, acc);
}

template <int KM, int VEC, int UW, int LO, int HI>
__device__ __forceinline__ void dispatch_wide_pc(int mask, const uint32_t *rbuf, int len,
                                                 const char *__restrict__ Bcol, uint32_t ldb_bytes, bool active,
                                                 float (&acc)[KM][VEC]) {
  if constexpr (HI - LO == 1) {
    seg_wide_pc<KM, LO, VEC, UW>(rbuf, len, Bcol, ldb_bytes, active, mask, acc);
  } else {
    constexpr int MID = (LO + HI) / 2;
    if (__popc(mask) < MID) dispatch_wide_pc<KM, VEC, UW, LO, MID>(mask, rbuf, len, Bcol, ldb_bytes, active, acc);
    else dispatch_wide_pc<KM, VEC, UW, MID, HI>(mask, rbuf, len, Bcol, ldb_bytes, active, acc);
  }
}

template <int KM, int VEC, int UW, int LO, int HI>
__device__ __forceinline__ void dispatch_wide_mask(int mask, const uint32_t *rbuf, int len,
                                                   const char *__restrict__ Bcol, uint32_t ldb_bytes, bool active,
                                                   float (&acc)[KM][VEC]) {
  if constexpr (HI - LO == 1) {
    seg_wide<KM, LO, VEC, UW>(rbuf, len, Bcol, ldb_bytes, active, acc);
  } else {
    constexpr int MID = (LO + HI) / 2;
    if (mask < MID) dispatch_wide_mask<KM, VEC, UW, LO, MID>(mask, rbuf, len, Bcol, ldb_bytes, active, acc);
    else dispatch_wide_mask<KM, VEC, UW, MID, HI>(mask, rbuf, len, Bcol, ldb_bytes, active, acc);
  }
}

// Item dispatch: a body per mask for kernel_m <= SC_MASK_KM_MAX (2^KM - 1
// bodies), a body per popcount above it (KM bodies: the mask-specialised
// kernel_m = 6 kernels alone took ~20 minutes of nvcc time).
template <int KM, int VEC, int UW>
__device__ __forceinline__ void dispatch_wide(int mask, const uint32_t *rbuf, int len, const char *__restrict__ Bcol,
                                              uint32_t ldb_bytes, bool active, float (&acc)[KM][VEC]) {
  if constexpr (KM <= SC_MASK_KM_MAX) dispatch_wide_mask<KM, VEC, UW, 1, (1 << KM)>(mask, rbuf, len, Bcol, ldb_bytes, active, acc);
  else dispatch_wide_pc<KM, VEC, UW, 1, KM + 1>(mask, rbuf, len, Bcol, ldb_bytes, active, acc);
}

// Dynamic shared memory: max(2 record buffers per warp, the cross-warp
// reduction area (warps-1) x KM x 32*VEC floats).
__host__ __device__ constexpr size_t wide_smem_bytes(int warps, int km, int vec) {
  return (size_t)4 * ((size_t)warps * 2 * kRecBufWords > (size_t)(warps - 1) * km * 32 * vec
                          ? (size_t)warps * 2 * kRecBufWords
                          : (size_t)(warps - 1) * km * 32 * vec);
}

// BATCH == false: CTA b computes panel order[b] of `one`.
// BATCH == true : CTA b computes panel order2[b].y of matrix many[order2[b].x]
//                 (a whole set of matrices -- e.g. a layer stack -- in one launch).
template <int KM, int VEC, bool BATCH>
__global__ void __launch_bounds__(256, BATCH ? SC_WIDE_BATCH_MINB : SC_WIDE_MINB)
spmm_wide_kernel(WideArgs one, const WideArgs *__restrict__ many, const int32_t *__restrict__ order,
                 int accumulate) {
  extern __shared__ __align__(16) uint32_t smem[];
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int nw = blockDim.x >> 5;
  int panel;
  if constexpr (BATCH) {
    const int2 o = reinterpret_cast<const int2 *>(order)[blockIdx.x];
    one = many[o.x];
    panel = o.y;
  } else {
    panel = order[blockIdx.x];
  }
  const int col0 = blockIdx.y * 32 * VEC + lane * VEC;
  const bool active = col0 < one.n_cols;
  const char *Bcol = reinterpret_cast<const char *>(one.B + col0);
  uint32_t *rbuf = smem + warp * 2 * kRecBufWords;

  float acc[KM][VEC];
#pragma unroll
  for (int k = 0; k < KM; ++k)
#pragma unroll
    for (int q = 0; q < VEC; ++q) acc[k][q] = 0.f;

  const int it0 = one.item_ptr[panel], it1 = one.item_ptr[panel + 1];
  int it = it0 + warp;
  int2 nitem = make_int2(0, 0);
  if (it < it1) {
    nitem = __ldg(one.items + it);
    copy_item_recs(rbuf, one.recs, nitem, lane);
  }
  cp_async_commit();
  int buf = 0;
  for (; it < it1; it += nw) {
    const int2 item = nitem;
    if (it + nw < it1) {  // next item's records into the other buffer
      nitem = __ldg(one.items + it + nw);
      copy_item_recs(rbuf + (buf ^ 1) * kRecBufWords, one.recs, nitem, lane);
    }
    cp_async_commit();
    cp_async_wait_1();
    __syncwarp();
    dispatch_wide<KM, VEC, BATCH ? SC_WIDE_BATCH_U : SC_WIDE_U>(item.y & 0xffff, rbuf + buf * kRecBufWords, item.y >> 16, Bcol,
                                         one.ldb_bytes, active, acc);
    __syncwarp();
    buf ^= 1;
  }

  if (nw > 1) {
    float *red = reinterpret_cast<float *>(smem);
    __syncthreads();  // record buffers are reused as the reduction area
    if (warp > 0) {
#pragma unroll
      for (int k = 0; k < KM; ++k)
#pragma unroll
        for (int q = 0; q < VEC; ++q) red[((warp - 1) * KM + k) * 32 * VEC + lane * VEC + q] = acc[k][q];
    }
    __syncthreads();
    if (warp != 0) return;
    for (int w = 1; w < nw; ++w)
#pragma unroll
      for (int k = 0; k < KM; ++k)
#pragma unroll
        for (int q = 0; q < VEC; ++q) acc[k][q] += red[((w - 1) * KM + k) * 32 * VEC + lane * VEC + q];
  }
#pragma unroll
  for (int k = 0; k < KM; ++k) {
    const int64_t row = (int64_t)panel * KM + k;
    if (!active || row >= one.rows) break;
    const int64_t off = row * one.ldc + col0;
    float *c = one.C + off;
    if constexpr (VEC == 1) {
      const float o = accumulate ? c[0] + acc[k][0] : acc[k][0];
      c[0] = o;
      for (int p = 0; p < one.npeers; ++p) one.peers[p][off] = o;
    } else if constexpr (VEC == 2) {
      float2 o = make_float2(acc[k][0], acc[k][1]);
      if (accumulate) { float2 x = *reinterpret_cast<float2 *>(c); o.x += x.x; o.y += x.y; }
      *reinterpret_cast<float2 *>(c) = o;
      for (int p = 0; p < one.npeers; ++p) *reinterpret_cast<float2 *>(one.peers[p] + off) = o;
    } else {
      float4 o = make_float4(acc[k][0], acc[k][1], acc[k][2], acc[k][3]);
      if (accumulate) {
        float4 x = *reinterpret_cast<float4 *>(c);
        o.x += x.x; o.y += x.y; o.z += x.z; o.w += x.w;
      }
      *reinterpret_cast<float4 *>(c) = o;
      for (int p = 0; p < one.npeers; ++p) *reinterpret_cast<float4 *>(one.peers[p] + off) = o;
    }
  }
  // Without a completion signal no fence is needed here: the peer stores are
  // complete when the kernel completes, and the caller's cross-GPU barrier
  // (stream-ordered after this kernel) publishes them.
}

// Publishes `epoch` into flag_dst[0..n) (release, system scope).  Launched on
// the stream right after a product kernel: that kernel's stores (local and
// peer) are complete when it completes, so the release orders all of them
// before the flags.  (Counting CTAs inside the product kernel and fencing each
// one measured +27 us on a 160 us product: every CTA waited for its remote
// stores to be acknowledged.)
static __global__ void signal_flags_kernel(FlagList fl, int epoch) {
  const int i = threadIdx.x;
  if (i < fl.n) asm volatile("st.release.sys.global.b32 [%0], %1;" ::"l"(fl.dst[i]), "r"(epoch) : "memory");
}

// Waits (bounded) until flags[0..n) have all reached `epoch` (wrap-safe
// compare), with acquire semantics at system scope; on expiry records 5 in
// *status and returns.
static __global__ void wait_flags_kernel(const int *flags, int n, int epoch, int *status) {
  const int i = threadIdx.x;
  if (i >= n) return;
  for (uint32_t it = 0; it < (1u << 22); ++it) {
    int v;
    asm volatile("ld.acquire.sys.global.b32 %0, [%1];" : "=r"(v) : "l"(flags + i) : "memory");
    if (v - epoch >= 0) return;
    __nanosleep(32);
  }
  atomicExch(status, 5);
}

// ------------------------------------------------------------ narrow B ----
// N in {1, 2, 4}: lane l takes entries l, l+32, ... of an item,
// multiplies their P values by the NB-wide B rows, and keeps KM*NB
// partial sums; a warp transpose-reduction then a cross-warp pass through
// shared memory produce the panel's KM x NB block.  This replaces the
// reference's lane-packed segmented shuffle reduction
// (code_gen/spmm_small_b_col/spmm_small_b_col_format_code_generator.py:212-323).
//
// Items of the narrow kernel hold up to 128 entries: lane l takes entries
// l, l+32, l+64, l+96 and issues all their record loads, then all their B
// loads, before the FMAs -- four independent DRAM requests per lane in
// flight, and the item's mask dispatch paid once per 128 entries.
template <int P, int VT, bool SM>
__device__ __forceinline__ void load_rec_any(const uint32_t *__restrict__ recs, uint32_t off, int &col,
                                             float (&v)[P]) {
  constexpr int S = rec_stride(P);
  if constexpr (VT == 0) {
    load_rec<P, SM>(recs + off, col, v);
  } else {
    const uint16_t *r = reinterpret_cast<const uint16_t *>(recs) + off;
    uint32_t w[4] = {0u, 0u, 0u, 0u};
    if constexpr (S == 2) {
      w[0] = ldro<SM>(reinterpret_cast<const uint32_t *>(r));
    } else if constexpr (S == 4) {
      const uint2 t = ldro<SM>(reinterpret_cast<const uint2 *>(r));
      w[0] = t.x; w[1] = t.y;
    } else {
      const uint4 t = ldro<SM>(reinterpret_cast<const uint4 *>(r));
      w[0] = t.x; w[1] = t.y; w[2] = t.z; w[3] = t.w;
    }
    col = (int)(w[0] & 0xffffu);
#pragma unroll
    for (int p = 0; p < P; ++p) {
      const int h = p + 1;  // halfword index within the record
      v[p] = half_bits_to_float<VT>((h & 1) ? (w[h >> 1] >> 16) : (w[h >> 1] & 0xffffu));
    }
  }
}

// Split item blocks (VT == 3, fp32 small-B plans with K <= 65536): an item of
// `len` entries is [len 16-bit columns, zero-filled to 16 bytes][len * P fp32
// values, zero-filled to 16 bytes], starting 16-byte aligned at word `off`.
// 2 + 4P bytes per entry -- the interleaved fp32 record costs 8 bytes per
// nonzero (column word and stride padding).
__host__ __device__ constexpr uint32_t split_col_words(int len) { return (uint32_t)((len * 2 + 15) / 16) * 4u; }
__host__ __device__ constexpr uint32_t split_val_words(int len, int p) { return (uint32_t)((len * p * 4 + 15) / 16) * 4u; }

// Entry e of the item at `off` (len entries, popcount P): its column and values.
template <int P, int VT, bool SM>
__device__ __forceinline__ void load_entry(const uint32_t *__restrict__ recs, uint32_t off, int len, int e, int &col,
                                           float (&v)[P]) {
  if constexpr (VT == 3) {
    col = (int)ldro<SM>(reinterpret_cast<const uint16_t *>(recs + off) + e);
    const float *vals = reinterpret_cast<const float *>(recs + off + split_col_words(len)) + e * P;
    if constexpr (P % 4 == 0) {
#pragma unroll
      for (int p = 0; p < P; p += 4) {
        const float4 t = ldro<SM>(reinterpret_cast<const float4 *>(vals + p));
        v[p] = t.x; v[p + 1] = t.y; v[p + 2] = t.z; v[p + 3] = t.w;
      }
    } else if constexpr (P % 2 == 0) {
#pragma unroll
      for (int p = 0; p < P; p += 2) {
        const float2 t = ldro<SM>(reinterpret_cast<const float2 *>(vals + p));
        v[p] = t.x; v[p + 1] = t.y;
      }
    } else {
#pragma unroll
      for (int p = 0; p < P; ++p) v[p] = ldro<SM>(vals + p);
    }
  } else {
    load_rec_any<P, VT, SM>(recs, off + (uint32_t)(e * rec_stride(P)), col, v);
  }
}

// Words of an item's records (from its first word), for the L2 prefetch.
template <int VT>
__device__ __forceinline__ uint32_t item_words(int2 item) {
  const int len = item.y >> 16, P = __popc(item.y & 0xffff);
  if constexpr (VT == 3) return split_col_words(len) + split_val_words(len, P);
  const uint32_t units = (uint32_t)len * (P == 1 ? 2u : (P <= 3 ? 4u : 8u));
  return VT == 0 ? units : (units + 1) / 2;
}

template <int KM, int MASK, int NB, int VT, bool SM>
__device__ __forceinline__ void seg_narrow(const uint32_t *__restrict__ recs, uint32_t off, int len,
                                           const float *__restrict__ B, int64_t ldb, int lane,
                                           float (&acc)[KM][NB]) {
  constexpr int P = popc_c(MASK);
  constexpr int U = kNarrowUnroll;
  for (int e0 = 0; e0 < len; e0 += 32 * U) {
    int col[U];
    float v[U][P];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int e = e0 + u * 32 + lane;
      if (e < len) {
        load_entry<P, VT, SM>(recs, off, len, e, col[u], v[u]);
      } else {
        col[u] = 0;  // row 0 of B, weight 0
#pragma unroll
        for (int p = 0; p < P; ++p) v[u][p] = 0.f;
      }
    }
    float b[U][NB];
#pragma unroll
    for (int u = 0; u < U; ++u) load_vec<NB>(B + (int64_t)col[u] * ldb, b[u]);
#pragma unroll
    for (int u = 0; u < U; ++u)
#pragma unroll
      for (int p = 0; p < P; ++p)
#pragma unroll
        for (int q = 0; q < NB; ++q)
          acc[nth_row(MASK, p)][q] = fmaf(v[u][p], b[u][q], acc[nth_row(MASK, p)][q]);
  }
}

// Popcount-class body of the narrow kernel (kernel_m above SC_MASK_KM_MAX);
// see seg_wide_pc.
template <int KM, int P, int NB, int VT, bool SM>
__device__ __forceinline__ void seg_narrow_pc(const uint32_t *__restrict__ recs, uint32_t off, int len,
                                              const float *__restrict__ B, int64_t ldb, int lane, int mask,
                                              float (&acc)[KM][NB]) {
  constexpr int U = kNarrowUnroll;
  float t[P][NB];
#pragma unroll
  for (int p = 0; p < P; ++p)
#pragma unroll
    for (int q = 0; q < NB; ++q) t[p][q] = 0.f;
  for (int e0 = 0; e0 < len; e0 += 32 * U) {
    int col[U];
    float v[U][P];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int e = e0 + u * 32 + lane;
      if (e < len) {
        load_entry<P, VT, SM>(recs, off, len, e, col[u], v[u]);
      } else {
        col[u] = 0;
#pragma unroll
        for (int p = 0; p < P; ++p) v[u][p] = 0.f;
      }
    }
    float b[U][NB];
#pragma unroll
    for (int u = 0; u < U; ++u) load_vec<NB>(B + (int64_t)col[u] * ldb, b[u]);
#pragma unroll
    for (int u = 0; u < U; ++u)
#pragma unroll
      for (int p = 0; p < P; ++p)
#pragma unroll
        for (int q = 0; q < NB; ++q) t[p][q] = fmaf(v[u][p], b[u][q], t[p][q]);
  }
  add_rows<KM, P, NB>(mask, t, acc);
}

template <int KM, int NB, int VT, bool SM, int LO, int HI>
__device__ __forceinline__ void dispatch_narrow_mask(int mask, const uint32_t *__restrict__ recs, uint32_t off,
                                                     int len, const float *__restrict__ B, int64_t ldb, int lane,
                                                     float (&acc)[KM][NB]) {
  if constexpr (HI - LO == 1) {
    seg_narrow<KM, LO, NB, VT, SM>(recs, off, len, B, ldb, lane, acc);
  } else {
    constexpr int MID = (LO + HI) / 2;
    if (mask < MID) dispatch_narrow_mask<KM, NB, VT, SM, LO, MID>(mask, recs, off, len, B, ldb, lane, acc);
    else dispatch_narrow_mask<KM, NB, VT, SM, MID, HI>(mask, recs, off, len, B, ldb, lane, acc);
  }
}

template <int KM, int NB, int VT, bool SM, int LO, int HI>
__device__ __forceinline__ void dispatch_narrow_pc(int mask, const uint32_t *__restrict__ recs, uint32_t off,
                                                   int len, const float *__restrict__ B, int64_t ldb, int lane,
                                                   float (&acc)[KM][NB]) {
  if constexpr (HI - LO == 1) {
    seg_narrow_pc<KM, LO, NB, VT, SM>(recs, off, len, B, ldb, lane, mask, acc);
  } else {
    constexpr int MID = (LO + HI) / 2;
    if (__popc(mask) < MID) dispatch_narrow_pc<KM, NB, VT, SM, LO, MID>(mask, recs, off, len, B, ldb, lane, acc);
    else dispatch_narrow_pc<KM, NB, VT, SM, MID, HI>(mask, recs, off, len, B, ldb, lane, acc);
  }
}

template <int KM, int NB, int VT, bool SM>
__device__ __forceinline__ void dispatch_narrow(int mask, const uint32_t *__restrict__ recs, uint32_t off, int len,
                                                const float *__restrict__ B, int64_t ldb, int lane,
                                                float (&acc)[KM][NB]) {
  if constexpr (KM <= SC_MASK_KM_MAX) dispatch_narrow_mask<KM, NB, VT, SM, 1, (1 << KM)>(mask, recs, off, len, B, ldb, lane, acc);
  else dispatch_narrow_pc<KM, NB, VT, SM, 1, KM + 1>(mask, recs, off, len, B, ldb, lane, acc);
}

__host__ __device__ constexpr int pow2_ceil(int x) {
  int p = 1;
  while (p < x) p <<= 1;
  return p;
}
__host__ __device__ constexpr int log2_c(int x) {
  int l = 0;
  while ((1 << l) < x) ++l;
  return l;
}

// Reduces V (power of two <= 32) values across the warp with V-1 + 5-log2(V)
// shuffles: at each halving step a lane keeps one half of its values and
// sends the other half to its partner.  Afterwards v[0] of lane l is the
// full sum of value index  sum_s bit(l, 4-s) * (V >> (s+1)).
template <int V>
__device__ __forceinline__ void warp_transpose_reduce(float (&v)[V], int lane) {
  constexpr int L = log2_c(V);
#pragma unroll
  for (int s = 0; s < L; ++s) {
    const int off = 16 >> s;
    const bool upper = (lane & off) != 0;
    const int half = V >> (s + 1);
#pragma unroll
    for (int i = 0; i < half; ++i) {
      float send = upper ? v[i] : v[i + half];
      float keep = upper ? v[i + half] : v[i];
      v[i] = keep + __shfl_xor_sync(0xffffffffu, send, off);
    }
  }
#pragma unroll
  for (int s = L; s < 5; ++s) v[0] += __shfl_xor_sync(0xffffffffu, v[0], 16 >> s);
}

template <int V>
__device__ __forceinline__ int transpose_reduce_index(int lane) {
  constexpr int L = log2_c(V);
  int idx = 0;
#pragma unroll
  for (int s = 0; s < L; ++s)
    if (lane & (16 >> s)) idx += V >> (s + 1);
  return idx;
}

template <int KM, int NB, int VT>
__global__ void __launch_bounds__(256)
spmm_narrow_kernel(const uint32_t *__restrict__ recs, const int2 *__restrict__ items,
                   const int32_t *__restrict__ item_ptr, const int32_t *__restrict__ order,
                   const float *__restrict__ B, int64_t ldb, float *__restrict__ C, int64_t ldc,
                   int64_t rows, int accumulate) {
  constexpr int V = pow2_ceil(KM * NB);
  static_assert(V <= 32, "KM*NB must not exceed 32");
  __shared__ float red[8][V];
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int nw = blockDim.x >> 5;
  const int panel = order[blockIdx.x];

  float acc[KM][NB];
#pragma unroll
  for (int k = 0; k < KM; ++k)
#pragma unroll
    for (int q = 0; q < NB; ++q) acc[k][q] = 0.f;

  const int it0 = item_ptr[panel], it1 = item_ptr[panel + 1];
#if SC_NARROW_PREFETCH
  // The panel's records are one contiguous range: ask the bulk-copy engine to
  // pull all of it into L2 at once, so the warps' record loads below meet L2
  // latency instead of a chain of DRAM round trips.
  if (threadIdx.x == 0 && it1 > it0) {
    const int2 f = __ldg(items + it0), l = __ldg(items + it1 - 1);
    // item offsets count words (VT 0, 3) or halfwords (VT 1, 2)
    constexpr uint32_t unit = (VT == 0 || VT == 3) ? 4u : 2u;
    const uint32_t end_bytes = ((uint32_t)l.x * unit + item_words<VT>(l) * 4u);
    const uint32_t b0 = ((uint32_t)f.x * unit) & ~15u, b1 = (end_bytes + 15u) & ~15u;
    const char *base = reinterpret_cast<const char *>(recs) + b0;
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(base), "r"(b1 - b0) : "memory");
  }
#endif
  const int mine_total = it1 > it0 + warp ? (it1 - it0 - warp + nw - 1) / nw : 0;  // items it0+warp+j*nw
  for (int base = 0; base < mine_total; base += 32) {
    const int cnt = min(32, mine_total - base);
    const int2 mine = lane < cnt ? __ldg(items + it0 + warp + (base + lane) * nw) : make_int2(0, 0);
    for (int j = 0; j < cnt; ++j) {
      const int2 item = make_int2(__shfl_sync(0xffffffffu, mine.x, j), __shfl_sync(0xffffffffu, mine.y, j));
      dispatch_narrow<KM, NB, VT, false>(item.y & 0xffff, recs, (uint32_t)item.x, item.y >> 16, B, ldb,
                                                lane, acc);
    }
  }

  float v[V];
#pragma unroll
  for (int i = 0; i < V; ++i) v[i] = (i < KM * NB) ? acc[i / NB][i % NB] : 0.f;
  warp_transpose_reduce<V>(v, lane);
  constexpr int kRep = 32 / V;  // lanes sharing one value index
  if ((lane % kRep) == 0) red[warp][transpose_reduce_index<V>(lane)] = v[0];
  __syncthreads();
  if (threadIdx.x < KM * NB) {
    float s = 0.f;
    for (int w = 0; w < nw; ++w) s += red[w][threadIdx.x];
    const int k = threadIdx.x / NB, q = threadIdx.x % NB;
    const int64_t row = (int64_t)panel * KM + k;
    if (row < rows) {
      float *c = C + row * ldc + q;
      *c = accumulate ? *c + s : s;
    }
  }
}

// ------------------------------------------------ narrow B, lane blocks ----
// Lane blocks (the layout of fp32 SpMV plans whose vector fits in shared
// memory).  A lane block holds U = kLaneSlots / P consecutive entries of one
// pattern (mask) of a row panel: U 16-bit columns and U*P fp32 values.  The
// blocks of one (panel, popcount) group are cut into items of up to 32
// blocks, one per lane, stored chunk-major (the k-th 16-byte chunk of every
// lane together, so that a warp-wide 16-byte load reads 512 contiguous bytes
// from global memory or conflict-free from shared memory):
//   [32 bytes: the mask of each block (uint8), zero-filled]
//   [column region: 16-byte column chunks chunk-major, or one 8-byte chunk
//    per lane when a block has at most 4 columns; padded to 16 bytes]
//   [kLaneSlots/4 value chunks x nl x 16 bytes: 4 values each, entry-major]
// with nl the blocks of the item; item header {word offset, P | nl << 8}.
// Fill entries have column 0 and value 0.  A lane's loads do not depend on
// P, so they can be issued before the item's pattern is dispatched.
#ifndef SC_LANE_SLOTS
#define SC_LANE_SLOTS 16
#endif
constexpr int kLaneSlots = SC_LANE_SLOTS;  // fp32 values per lane block (8 or 16)
__host__ __device__ constexpr int lane_entries(int p) { return kLaneSlots / p; }
// bytes of a lane's columns: 8, 16 or 32 (U <= 4, 8 or 16 columns)
__host__ __device__ constexpr int lane_col_bytes(int p) {
  return lane_entries(p) <= 4 ? 8 : (lane_entries(p) <= 8 ? 16 : 32);
}
__host__ __device__ constexpr uint32_t lane_col_region(int nl, int p) {
  return ((uint32_t)nl * (uint32_t)lane_col_bytes(p) + 15u) & ~15u;
}
__host__ __device__ constexpr uint32_t lane_item_words(int nl, int p) {
  return 8u + (lane_col_region(nl, p) + (uint32_t)nl * kLaneSlots * 4u) / 4u;
}
// Word of column u of lane l in an item's column region.
__host__ __device__ constexpr uint32_t lane_col_word(int nl, int p, int l, int u) {
  return lane_col_bytes(p) == 8 ? (uint32_t)(l * 2 + u / 2) : (uint32_t)(((u / 8) * nl + l) * 4 + (u % 8) / 2);
}

struct LaneBuf {
  uint32_t m;                  // block mask (0: no block for this lane)
  uint32_t c[kLaneSlots / 2];  // packed 16-bit columns
  float v[kLaneSlots];
};

// Chunk c of lane `lane` of an item with nl blocks, from a region base.
__device__ __forceinline__ const uint4 *lane_chunk(const char *region, int nl, int c, int lane) {
  return reinterpret_cast<const uint4 *>(region) + (c * nl + lane);
}

template <bool SM>
__device__ __forceinline__ void lane_load(const char *base, int2 item, int lane, LaneBuf &b) {
  const int P = item.y & 0xff, nl = item.y >> 8;
  if (lane < nl) {
    b.m = ldro<SM>(reinterpret_cast<const uint8_t *>(base) + lane);
    const int cb = P == 1 ? lane_col_bytes(1)
                   : P == 2 ? lane_col_bytes(2)
                   : P == 3 ? lane_col_bytes(3)
                   : P == 4 ? lane_col_bytes(4)
                   : P == 5 ? lane_col_bytes(5)
                            : lane_col_bytes(6);
    if (cb == 8) {
      const uint2 c0 = ldro<SM>(reinterpret_cast<const uint2 *>(base + 32) + lane);
      b.c[0] = c0.x; b.c[1] = c0.y;
    } else {
#pragma unroll
      for (int i = 0; i < kLaneSlots / 8; ++i) {
        if (i * 16 < cb) {
          const uint4 c0 = ldro<SM>(lane_chunk(base + 32, nl, i, lane));
          b.c[4 * i] = c0.x; b.c[4 * i + 1] = c0.y; b.c[4 * i + 2] = c0.z; b.c[4 * i + 3] = c0.w;
        }
      }
    }
    const char *vals = base + 32 + lane_col_region(nl, P);
#pragma unroll
    for (int i = 0; i < kLaneSlots / 4; ++i) {
      const uint4 f = ldro<SM>(lane_chunk(vals, nl, i, lane));
      b.v[4 * i] = __uint_as_float(f.x); b.v[4 * i + 1] = __uint_as_float(f.y);
      b.v[4 * i + 2] = __uint_as_float(f.z); b.v[4 * i + 3] = __uint_as_float(f.w);
    }
  } else {
    // no block: mask 0 adds nothing; columns 0 keep the gathers in range
    b.m = 0;
#pragma unroll
    for (int i = 0; i < kLaneSlots / 2; ++i) b.c[i] = 0;
#pragma unroll
    for (int i = 0; i < kLaneSlots; ++i) b.v[i] = 0.f;
  }
}

// One lane block against B in global memory (L1 gathers).
template <int KM, int P, int NB>
__device__ __forceinline__ void lane_compute(const LaneBuf &b, const float *__restrict__ B, int64_t ldb,
                                             float (&acc)[KM][NB]) {
  constexpr int U = lane_entries(P);
  constexpr int G = NB == 4 ? 4 : (NB == 2 ? 8 : 16);  // B rows in flight per group
  float t[P][NB];
#pragma unroll
  for (int p = 0; p < P; ++p)
#pragma unroll
    for (int q = 0; q < NB; ++q) t[p][q] = 0.f;
#pragma unroll
  for (int u0 = 0; u0 < U; u0 += G) {
    float x[G][NB];
#pragma unroll
    for (int g = 0; g < G; ++g) {
      const int u = u0 + g;
      if (u < U) {
        const uint32_t c = (b.c[u >> 1] >> ((u & 1) * 16)) & 0xffffu;
        load_vec<NB>(B + (int64_t)c * ldb, x[g]);
      }
    }
#pragma unroll
    for (int g = 0; g < G; ++g) {
      const int u = u0 + g;
      if (u < U) {
#pragma unroll
        for (int p = 0; p < P; ++p)
#pragma unroll
          for (int q = 0; q < NB; ++q) t[p][q] = fmaf(b.v[u * P + p], x[g][q], t[p][q]);
      }
    }
  }
  add_rows<KM, P, NB>((int)b.m, t, acc);
}

template <int KM, int NB, int LO, int HI>
__device__ __forceinline__ void dispatch_lane(int P, const LaneBuf &b, const float *__restrict__ B, int64_t ldb,
                                              float (&acc)[KM][NB]) {
  if constexpr (HI - LO == 1) {
    lane_compute<KM, LO, NB>(b, B, ldb, acc);
  } else {
    constexpr int MID = (LO + HI) / 2;
    if (P < MID) dispatch_lane<KM, NB, LO, MID>(P, b, B, ldb, acc);
    else dispatch_lane<KM, NB, MID, HI>(P, b, B, ldb, acc);
  }
}

// Lane blocks with B read through L1 (only when SC_NARROW_LAYOUT=lane forces
// the layout on a plan the staged kernel does not take; measured 31.7 us on
// the config-5 SpMV against 30.7 us for split blocks): same arguments, grid
// and result as
// spmm_narrow_kernel; each warp loads its next item before it gathers the B
// rows of the current one.
template <int KM, int NB>
__global__ void __launch_bounds__(256)
spmm_lane_kernel(const uint32_t *__restrict__ recs, const int2 *__restrict__ items,
                 const int32_t *__restrict__ item_ptr, const int32_t *__restrict__ order,
                 const float *__restrict__ B, int64_t ldb, float *__restrict__ C, int64_t ldc,
                 int64_t rows, int accumulate) {
  constexpr int V = pow2_ceil(KM * NB);
  static_assert(V <= 32, "KM*NB must not exceed 32");
  __shared__ float red[8][V];
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int nw = blockDim.x >> 5;
  const int panel = order[blockIdx.x];

  float acc[KM][NB];
#pragma unroll
  for (int k = 0; k < KM; ++k)
#pragma unroll
    for (int q = 0; q < NB; ++q) acc[k][q] = 0.f;

  const int it0 = item_ptr[panel], it1 = item_ptr[panel + 1];
  const int total = it1 > it0 + warp ? (it1 - it0 - warp + nw - 1) / nw : 0;  // items it0+warp+j*nw
  int2 hb = lane < total ? __ldg(items + it0 + warp + lane * nw) : make_int2(0, 0);
  LaneBuf cur, nxt;
  int2 hc = make_int2(__shfl_sync(0xffffffffu, hb.x, 0), __shfl_sync(0xffffffffu, hb.y, 0));
  if (total > 0) lane_load<false>(reinterpret_cast<const char *>(recs + (uint32_t)hc.x), hc, lane, cur);
  for (int j = 0; j < total; ++j) {
    int2 hn = make_int2(0, 0);
    if (j + 1 < total) {
      if (((j + 1) & 31) == 0) {  // next batch of 32 headers
        const int k = j + 1 + lane;
        hb = k < total ? __ldg(items + it0 + warp + k * nw) : make_int2(0, 0);
      }
      hn = make_int2(__shfl_sync(0xffffffffu, hb.x, (j + 1) & 31), __shfl_sync(0xffffffffu, hb.y, (j + 1) & 31));
      lane_load<false>(reinterpret_cast<const char *>(recs + (uint32_t)hn.x), hn, lane, nxt);
    }
    dispatch_lane<KM, NB, 1, KM + 1>(hc.y & 0xff, cur, B, ldb, acc);
    cur = nxt;
    hc = hn;
  }

  float v[V];
#pragma unroll
  for (int i = 0; i < V; ++i) v[i] = (i < KM * NB) ? acc[i / NB][i % NB] : 0.f;
  warp_transpose_reduce<V>(v, lane);
  constexpr int kRep = 32 / V;
  if ((lane % kRep) == 0) red[warp][transpose_reduce_index<V>(lane)] = v[0];
  __syncthreads();
  if (threadIdx.x < KM * NB) {
    float s = 0.f;
    for (int w = 0; w < nw; ++w) s += red[w][threadIdx.x];
    const int k = threadIdx.x / NB, q = threadIdx.x % NB;
    const int64_t row = (int64_t)panel * KM + k;
    if (row < rows) {
      float *c = C + row * ldc + q;
      *c = accumulate ? *c + s : s;
    }
  }
}

// ------------------------------------- narrow B, B staged in shared memory ----
// SpMV over lane blocks when the fp32 vector fits in shared memory.  The
// random B-row gathers bound the kernels above: a warp load whose 32 lanes
// touch 32 different 128-byte lines costs up to 32 L1 wavefronts, ~1 cycle
// per entry per SM (config-5 SpMV: 7.9 M gathers, ~27 us; records resident in
// L2 did not make it faster), while a random 4- or 8-byte shared-memory
// gather costs a few bank-conflict wavefronts per warp.  Each CTA copies B
// (K x N) into shared memory once; then every warp is an independent worker
// over whole panels in the plan's heaviest-first order (panel t, t + T, ...
// for T warps in the grid).  A warp's items stream through kXRing slots of
// its own in shared memory, one cp.async.bulk per item with completion on
// the slot's mbarrier, issued ahead across panel boundaries; the headers of
// the items are read 32 at a time, one per lane.  Panel sums stay in
// registers; one store per C element; no CTA barrier after the staging, no
// atomics.  Every mbarrier wait is bounded: on expiry the warp records 7 in
// *status, waits (bounded) for its copies still in flight, and stops.
// `starve` (test hook) issues no copies, so that the first wait expires.
constexpr int kLaneSlotBytes = 32 + 32 * (2 * kLaneSlots + 4 * kLaneSlots);  // largest item: 32 P=1 blocks
constexpr int kXRing = 3;                                                   // slots per warp
constexpr uint32_t kXWaitLimit = 1u << 20;                                 // polls of mbarrier.try_wait
// 16-value lane blocks leave shared memory for 16 warps beside a 64 KB B
constexpr int kXMaxThreads = kLaneSlots >= 16 ? 512 : 1024;

__device__ __forceinline__ uint32_t smem_addr(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }
__device__ __forceinline__ bool xb_try_wait(uint64_t *bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ bool xb_wait(uint64_t *bar, uint32_t parity) {
  for (uint32_t i = 0; i < kXWaitLimit; ++i)
    if (xb_try_wait(bar, parity)) return true;
  return false;
}

template <int KM, int P, int NB>
__device__ __forceinline__ void lane_compute_sp(const LaneBuf &b, const float *__restrict__ xs,
                                                float (&acc)[KM][NB]) {
  constexpr int U = lane_entries(P);
  float t[P][NB];
#pragma unroll
  for (int p = 0; p < P; ++p)
#pragma unroll
    for (int q = 0; q < NB; ++q) t[p][q] = 0.f;
  float x[U][NB];
#pragma unroll
  for (int u = 0; u < U; ++u) {
    const uint32_t c = (b.c[u >> 1] >> ((u & 1) * 16)) & 0xffffu;
    if constexpr (NB == 1) {
      x[u][0] = xs[c];
    } else {
      const float2 f = reinterpret_cast<const float2 *>(xs)[c];
      x[u][0] = f.x; x[u][1] = f.y;
    }
  }
#pragma unroll
  for (int u = 0; u < U; ++u)
#pragma unroll
    for (int p = 0; p < P; ++p)
#pragma unroll
      for (int q = 0; q < NB; ++q) t[p][q] = fmaf(b.v[u * P + p], x[u][q], t[p][q]);
  add_rows<KM, P, NB>((int)b.m, t, acc);
}

template <int KM, int NB, int LO, int HI>
__device__ __forceinline__ void dispatch_lane_s(int P, const LaneBuf &b, const float *__restrict__ xs,
                                                float (&acc)[KM][NB]) {
  if constexpr (HI - LO == 1) {
    lane_compute_sp<KM, LO, NB>(b, xs, acc);
  } else {
    constexpr int MID = (LO + HI) / 2;
    if (P < MID) dispatch_lane_s<KM, NB, LO, MID>(P, b, xs, acc);
    else dispatch_lane_s<KM, NB, MID, HI>(P, b, xs, acc);
  }
}

// Dynamic shared memory of the staged kernel: B, then each warp's slots,
// slot headers and mbarriers.
__host__ __device__ constexpr size_t lane_x_bytes(int64_t kcols, int nb) {
  return ((size_t)kcols * nb * 4 + 127) & ~(size_t)127;
}
__host__ __device__ constexpr size_t lane_x_smem(int64_t kcols, int nb, int warps) {
  return lane_x_bytes(kcols, nb) + (size_t)warps * kXRing * (kLaneSlotBytes + 8 + 8);
}

template <int KM, int NB>
__global__ void __launch_bounds__(kXMaxThreads)
spmm_lane_x_kernel(const uint32_t *__restrict__ recs, const int2 *__restrict__ items,
                   const int4 *__restrict__ pm, const int32_t *__restrict__ order, int64_t panels,
                   const float *__restrict__ B, int64_t ldb, int64_t kcols, float *__restrict__ C, int64_t ldc,
                   int64_t rows, int accumulate, int *status, int starve) {
  static_assert(NB == 1 || NB == 2, "B staging is for N = 1 and 2");
  constexpr int V = pow2_ceil(KM * NB);
  static_assert(V <= 32, "KM*NB must not exceed 32");
  extern __shared__ __align__(128) unsigned char smraw[];
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int nw = blockDim.x >> 5;
  const size_t xb = lane_x_bytes(kcols, NB);
  float *xs = reinterpret_cast<float *>(smraw);
  unsigned char *ring = smraw + xb + (size_t)warp * kXRing * kLaneSlotBytes;
  int2 *hdr = reinterpret_cast<int2 *>(smraw + xb + (size_t)nw * kXRing * kLaneSlotBytes) + warp * kXRing;
  uint64_t *bar = reinterpret_cast<uint64_t *>(smraw + xb + (size_t)nw * kXRing * (kLaneSlotBytes + 8)) +
                  warp * kXRing;
  if (lane == 0) {
#pragma unroll
    for (int r = 0; r < kXRing; ++r)
      asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_addr(bar + r)) : "memory");
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }

  // stage B (K x NB, row pitch ldb) as a dense K*NB array
  const int64_t total_x = kcols * NB;
  if (ldb == NB && (reinterpret_cast<uintptr_t>(B) & 15) == 0) {
    const int64_t n4 = total_x >> 2;
    for (int64_t i = threadIdx.x; i < n4; i += blockDim.x)
      reinterpret_cast<float4 *>(xs)[i] = __ldg(reinterpret_cast<const float4 *>(B) + i);
    for (int64_t i = (n4 << 2) + threadIdx.x; i < total_x; i += blockDim.x) xs[i] = __ldg(B + i);
  } else {
    for (int64_t i = threadIdx.x; i < total_x; i += blockDim.x) xs[i] = __ldg(B + (i / NB) * ldb + (i % NB));
  }
  __syncthreads();

  const int64_t T = (int64_t)gridDim.x * nw;
  // issue cursor (warp-uniform): panel position ti, its table entry mi, next
  // item ii; the headers of items [ib0, ib0 + 32) sit one per lane in ib
  int64_t ti = (int64_t)blockIdx.x * nw + warp;
  if (ti >= panels) return;
  int4 mi = __ldg(pm + order[ti]);
  int ii = mi.x, ib0 = mi.x;
  int2 ib = lane < mi.y - mi.x ? __ldg(items + mi.x + lane) : make_int2(0, 0);
  int pn_next = ti + T < panels ? order[ti + T] : -1;  // panel after the issue cursor's
  int in_flight = 0, slot_in = 0, slot_out = 0;
  uint32_t phase = 0;  // bit r: parity of slot r's next completion
  auto issue = [&]() {
    while (in_flight < kXRing) {
      while (ii >= mi.y) {  // next panel of this warp (empty panels have no items)
        ti += T;
        if (ti >= panels) return;
        mi = __ldg(pm + pn_next);
        pn_next = ti + T < panels ? order[ti + T] : -1;
        ii = ib0 = mi.x;
        ib = lane < mi.y - mi.x ? __ldg(items + mi.x + lane) : make_int2(0, 0);
      }
      if (ii - ib0 >= 32) {
        ib0 = ii;
        ib = lane < mi.y - ii ? __ldg(items + ii + lane) : make_int2(0, 0);
      }
      const int2 it = make_int2(__shfl_sync(0xffffffffu, ib.x, ii - ib0), __shfl_sync(0xffffffffu, ib.y, ii - ib0));
      if (lane == 0 && !starve) {
        const uint32_t bytes = lane_item_words(it.y >> 8, it.y & 0xff) * 4u;
        hdr[slot_in] = it;
        asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar + slot_in)),
                     "r"(bytes)
                     : "memory");
        asm volatile(
            "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                smem_addr(ring + slot_in * kLaneSlotBytes)),
            "l"(recs + (uint32_t)it.x), "r"(bytes), "r"(smem_addr(bar + slot_in))
            : "memory");
      }
      slot_in = slot_in + 1 == kXRing ? 0 : slot_in + 1;
      ++in_flight;
      ++ii;
    }
  };
  issue();

  for (int64_t t = (int64_t)blockIdx.x * nw + warp; t < panels; t += T) {
    const int panel = order[t];
    const int4 m = __ldg(pm + panel);
    float acc[KM][NB];
#pragma unroll
    for (int k = 0; k < KM; ++k)
#pragma unroll
      for (int q = 0; q < NB; ++q) acc[k][q] = 0.f;
    for (int j = m.x; j < m.y; ++j) {
      if (!xb_wait(bar + slot_out, (phase >> slot_out) & 1u)) {
        if (lane == 0) atomicExch(status, 7);
        if (!starve)  // let the copies still in flight land before the CTA may exit
          for (int k = 1; k < in_flight; ++k) {
            const int r = (slot_out + k) % kXRing;
            xb_wait(bar + r, (phase >> r) & 1u);
          }
        return;
      }
      __syncwarp();
      const int2 it = hdr[slot_out];
      LaneBuf b;
      lane_load<true>(reinterpret_cast<const char *>(ring + slot_out * kLaneSlotBytes), it, lane, b);
      __syncwarp();  // every lane has read the slot: it may be refilled
      phase ^= 1u << slot_out;
      slot_out = slot_out + 1 == kXRing ? 0 : slot_out + 1;
      --in_flight;
      issue();
      dispatch_lane_s<KM, NB, 1, KM + 1>(it.y & 0xff, b, xs, acc);
    }
    float v[V];
#pragma unroll
    for (int i = 0; i < V; ++i) v[i] = (i < KM * NB) ? acc[i / NB][i % NB] : 0.f;
    warp_transpose_reduce<V>(v, lane);
    constexpr int kRep = 32 / V;
    const int idx = transpose_reduce_index<V>(lane);
    if ((lane % kRep) == 0 && idx < KM * NB) {
      const int k = idx / NB, q = idx % NB;
      const int64_t row = (int64_t)panel * KM + k;
      if (row < rows) {
        float *c = C + row * ldc + q;
        *c = accumulate ? *c + v[0] : v[0];
      }
    }
  }
}

using LaneXFn = void (*)(const uint32_t *, const int2 *, const int4 *, const int32_t *, int64_t, const float *,
                         int64_t, int64_t, float *, int64_t, int64_t, int, int *, int);

using WideFn = void (*)(WideArgs, const WideArgs *, const int32_t *, int);
using NarrowFn = void (*)(const uint32_t *, const int2 *, const int32_t *, const int32_t *, const float *,
                          int64_t, float *, int64_t, int64_t, int);

}  // namespace sc

// Per-kernel_m kernel tables, defined in sc_inst.cu (one object per kernel_m).
sc::WideFn sc_wide_kernel_km1(int vec, bool batch);
sc::WideFn sc_wide_kernel_km2(int vec, bool batch);
sc::WideFn sc_wide_kernel_km3(int vec, bool batch);
sc::WideFn sc_wide_kernel_km4(int vec, bool batch);
sc::WideFn sc_wide_kernel_km5(int vec, bool batch);
sc::WideFn sc_wide_kernel_km6(int vec, bool batch);
sc::NarrowFn sc_narrow_kernel_km1(int nb, int vt);
sc::NarrowFn sc_narrow_kernel_km2(int nb, int vt);
sc::NarrowFn sc_narrow_kernel_km3(int nb, int vt);
sc::NarrowFn sc_narrow_kernel_km4(int nb, int vt);
sc::NarrowFn sc_narrow_kernel_km5(int nb, int vt);
sc::NarrowFn sc_narrow_kernel_km6(int nb, int vt);
sc::LaneXFn sc_lane_x_kernel_km1(int nb);
sc::LaneXFn sc_lane_x_kernel_km2(int nb);
sc::LaneXFn sc_lane_x_kernel_km3(int nb);
sc::LaneXFn sc_lane_x_kernel_km4(int nb);
sc::LaneXFn sc_lane_x_kernel_km5(int nb);
sc::LaneXFn sc_lane_x_kernel_km6(int nb);
