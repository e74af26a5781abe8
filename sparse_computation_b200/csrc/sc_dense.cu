// Dense-tile tcgen05 kernels (see sc_dense.cuh for the scheme).
//
// dense_gemm_persist_kernel (tasks not split over a cluster; described at
// its definition) and dense_gemm_kernel, one CTA per task:
//
// CTA = one 128-row block x one 128-column C tile, 4 warps:
//   thread 0   producer: per kept K-chunk, bulk-copies the A_hi, A_lo, B_hi,
//              B_lo tile images (4 x 16 KiB) into a 3-stage ring, completion
//              tracked by mbarrier transaction counts;
//   thread 32  MMA issuer: per stage 4 k-steps x 3 tcgen05.mma (kind::tf32,
//              M=128, N=128, K=8) into one 128x128 fp32 accumulator in tensor
//              memory; tcgen05.commit releases the stage back to the producer;
//   all warps  epilogue: tcgen05.ld of the accumulator (warp w owns TMEM lanes
//              32w..32w+31 = C rows), then row-contiguous stores of C.
// Every wait on an mbarrier is bounded; on expiry the CTA records an error in
// *status, stops issuing work, and still releases its tensor memory.
#include <algorithm>
#include <atomic>
#include <cstdlib>
#include <cstring>

#include <cooperative_groups.h>
#include <cuda_bf16.h>

#include "sc_dense.cuh"

namespace cg = cooperative_groups;

namespace sc {
namespace dense {
namespace {

constexpr uint32_t kWaitLimit = 1u << 18;  // polls of mbarrier.try_wait (each suspends briefly)

__device__ __forceinline__ uint32_t smem_u32(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait; false when the limit expired.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, volatile int *abort_flag) {
  for (uint32_t i = 0; i < kWaitLimit; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if (abort_flag && *abort_flag) return false;
  }
  return false;
}

__device__ __forceinline__ void bulk_copy(void *dst_smem, const void *src, uint32_t bytes, uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst_smem)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// tcgen05 shared-memory matrix descriptor: K-major, 128B swizzle, 8-row
// groups 1024 bytes apart (tile base 1024-byte aligned).
// SW64: 64-byte swizzle instead, 8-row groups 512 bytes apart (3xBF16 images).
template <bool SW64 = false>
__device__ __forceinline__ uint64_t sdesc(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr & 0x3FFFFu) >> 4);           // start address       [0,14)
  d |= (uint64_t)1 << 16;                              // leading byte offset [16,30) (unused for swizzled K-major)
  d |= (uint64_t)((SW64 ? 512 : 1024) >> 4) << 32;     // stride byte offset  [32,46)
  d |= (uint64_t)1 << 46;                              // descriptor version  [46,48)
  d |= (uint64_t)(SW64 ? 4 : 2) << 61;                 // SWIZZLE_64B / SWIZZLE_128B [61,64)
  return d;
}

// Instruction descriptor: D f32, A/B tf32, both K-major, N=128, M=128.
constexpr uint32_t kIdesc = (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)(kBN >> 3) << 17) |
                            ((uint32_t)(kBM >> 4) << 24);

__device__ __forceinline__ void mma_tf32(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t accum) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(kIdesc), "r"(accum)
      : "memory");
}

// Instruction descriptor: D f32, A/B bf16 (kind::f16), both K-major, N=128, M=128.
constexpr uint32_t kIdescBf16 = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(kBN >> 3) << 17) |
                                ((uint32_t)(kBM >> 4) << 24);

__device__ __forceinline__ void mma_bf16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t accum) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(kIdescBf16), "r"(accum)
      : "memory");
}

__device__ __forceinline__ void mma_commit(uint64_t *bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }

// 32 consecutive accumulator columns of this thread's TMEM lane.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// The MMAs of one stage (one kept K-chunk) into the accumulator at `acc`;
// `first`: the stage starts the accumulator.
template <int MODE>
__device__ __forceinline__ void mma_stage(uint32_t acc, uint32_t base, bool first) {
  if constexpr (MODE == kModeBf16x3) {
    constexpr int TB = mode_tile_bytes(kModeBf16x3);
    uint64_t a[3], b[3];
#pragma unroll
    for (int j = 0; j < 3; ++j) {
      a[j] = sdesc<true>(base + j * TB);
      b[j] = sdesc<true>(base + (3 + j) * TB);
    }
#pragma unroll
    for (int k = 0; k < kBKx3 / 16; ++k) {
      const uint64_t step = (uint64_t)((k * 32) >> 4);  // 16 bf16 = 32 bytes along K
      mma_bf16(acc, a[2] + step, b[0] + step, (!first || k > 0) ? 1u : 0u);
      mma_bf16(acc, a[0] + step, b[2] + step, 1u);
      mma_bf16(acc, a[1] + step, b[1] + step, 1u);
      mma_bf16(acc, a[1] + step, b[0] + step, 1u);
      mma_bf16(acc, a[0] + step, b[1] + step, 1u);
      mma_bf16(acc, a[0] + step, b[0] + step, 1u);
    }
  } else if constexpr (MODE == kModeBf16) {
    const uint64_t a = sdesc(base), b = sdesc(base + kTileBytes);
#pragma unroll
    for (int k = 0; k < kBKb / 16; ++k) {
      const uint64_t step = (uint64_t)((k * 32) >> 4);
      mma_bf16(acc, a + step, b + step, (!first || k > 0) ? 1u : 0u);
    }
  } else {
    const uint64_t a_hi = sdesc(base), a_lo = sdesc(base + kTileBytes);
    const uint64_t b_hi = sdesc(base + 2 * kTileBytes), b_lo = sdesc(base + 3 * kTileBytes);
#pragma unroll
    for (int k = 0; k < kBK / 8; ++k) {
      const uint64_t step = (uint64_t)((k * 32) >> 4);
      mma_tf32(acc, a_lo + step, b_hi + step, (!first || k > 0) ? 1u : 0u);
      mma_tf32(acc, a_hi + step, b_lo + step, 1u);
      mma_tf32(acc, a_hi + step, b_hi + step, 1u);
    }
  }
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// Sum of the partial accumulators of a cluster of S CTAs (split K): warp w's
// TMEM rows (C rows 32w..32w+31 of the tile) are owned by CTA w / (4/S); the
// other CTAs send theirs into the owner's shared memory (slots of 32 rows x
// 128 floats), then the owner adds them up and stores C.
template <bool BATCH, int MODE>
__global__ void __launch_bounds__(kThreads, 1)
dense_gemm_kernel(DenseMat one, const DenseMat *__restrict__ mats, const int4 *__restrict__ tasks, int accumulate,
                  int *status) {
  // tf32 x3: stage = A_hi, A_lo, B_hi, B_lo (64 KiB), 3 stages;
  // bf16:    stage = A, B (32 KiB), 6 stages;
  // bf16 x3: stage = A1, A2, A3, B1, B2, B3 (48 KiB, 32-wide K), 4 stages.
  constexpr int NST = mode_stages(MODE);
  constexpr int SB = 2 * mode_images(MODE) * mode_tile_bytes(MODE);
  extern __shared__ __align__(1024) uint8_t dsmem[];
  // 1024-byte aligned stage ring (the swizzle is applied on address bits).
  uint8_t *ring = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(dsmem) + 1023) & ~(uintptr_t)1023);
  __shared__ __align__(8) uint64_t full_bar[NST], empty_bar[NST], done_bar;
  __shared__ uint32_t tmem_base;
  __shared__ int abort_flag;

  cg::cluster_group cluster = cg::this_cluster();
  const int S = (int)cluster.num_blocks();
  const int crank = (int)cluster.block_rank();
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int4 task = tasks[blockIdx.x / S];
  DenseMat m;
  if constexpr (BATCH) m = mats[task.x];
  else m = one;
  const int rb = task.y, nt = task.z;
  const int c0 = m.rb_ptr[rb], c1 = m.rb_ptr[rb + 1];
  // this CTA's kept chunks: c0 + crank, c0 + crank + S, ...
  const int nk = (c1 - c0 > crank) ? (c1 - c0 - crank + S - 1) / S : 0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < NST; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    mbar_init(&done_bar, 1);
    abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 2) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_base)),
                 "r"(kBN));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_base;

  if (threadIdx.x == 0 && nk > 0 && !m.starve) {
    // producer
    constexpr int OP = mode_images(MODE) * mode_tile_bytes(MODE);  // bytes of one operand's images
    for (int i = 0; i < nk; ++i) {
      const int s = i % NST;
      if (i >= NST && !mbar_wait(&empty_bar[s], ((i / NST) - 1) & 1, &abort_flag)) {
        atomicExch(status, 1);
        abort_flag = 1;
        break;
      }
      const int ci = c0 + crank + i * S;
      uint8_t *st = ring + (size_t)s * SB;
      const uint8_t *at = m.a_tiles + (size_t)ci * OP;
      const int kc = m.rb_chunk[ci];
      const uint8_t *bt = m.b_tiles + ((size_t)nt * m.k_chunks + kc) * OP;
      mbar_expect_tx(&full_bar[s], SB);
      bulk_copy(st, at, OP, &full_bar[s]);
      bulk_copy(st + OP, bt, OP, &full_bar[s]);
    }
  } else if (threadIdx.x == 32 && nk > 0) {
    // MMA issuer
    bool ok = true;
    for (int i = 0; i < nk; ++i) {
      const int s = i % NST;
      if (!mbar_wait(&full_bar[s], (i / NST) & 1, &abort_flag)) {
        atomicExch(status, 2);
        abort_flag = 1;
        ok = false;
        break;
      }
      tc_fence_after();
      mma_stage<MODE>(tmem, smem_u32(ring + (size_t)s * SB), i == 0);
      mma_commit(&empty_bar[s]);  // stage free once these MMAs have read it
    }
    if (ok) mma_commit(&done_bar);
    else abort_flag = 1;
  }

  // ---- epilogue
  bool have = nk > 0;
  if (have && !mbar_wait(&done_bar, 0, &abort_flag)) {
    if (lane == 0) atomicExch(status, 3);
    abort_flag = 1;
    have = false;
  }
  __syncwarp();
  tc_fence_after();
  const int64_t row = (int64_t)rb * kBM + warp * 32 + lane;
  const int col_base = nt * kBN;
  const uint32_t trow = tmem + ((uint32_t)(warp * 32) << 16);
  const int wpc = 4 / S;           // warps (row groups) owned per CTA
  const int owner = warp / wpc;    // CTA that finalises this warp's rows
  constexpr int kSlotFloats = 32 * kBN;
  if (S > 1) {
    cluster.sync();  // every CTA's MMAs are done: stage rings are free
    if (owner != crank) {
      const int sidx = crank < owner ? crank : crank - 1;
      float *slot = reinterpret_cast<float *>(ring) + ((warp - owner * wpc) * (S - 1) + sidx) * kSlotFloats;
      float *dst = cluster.map_shared_rank(slot, owner) + lane * kBN;
#pragma unroll 1
      for (int cb = 0; cb < kBN / 32; ++cb) {
        float v[32];
        if (have) tmem_ld32(trow + (uint32_t)(cb * 32), v);
        else {
#pragma unroll
          for (int i = 0; i < 32; ++i) v[i] = 0.f;
        }
#pragma unroll
        for (int i = 0; i < 32; i += 4)
          *reinterpret_cast<float4 *>(dst + cb * 32 + i) = make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]);
      }
    }
    cluster.sync();  // partials delivered
  }
  if (owner == crank) {
#pragma unroll 1
    for (int cb = 0; cb < kBN / 32; ++cb) {
      float v[32];
      if (have) tmem_ld32(trow + (uint32_t)(cb * 32), v);
      else {
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] = 0.f;
      }
      for (int sidx = 0; sidx < S - 1; ++sidx) {
        const float *src = reinterpret_cast<const float *>(ring) +
                           ((warp - owner * wpc) * (S - 1) + sidx) * kSlotFloats + lane * kBN + cb * 32;
#pragma unroll
        for (int i = 0; i < 32; i += 4) {
          const float4 x = *reinterpret_cast<const float4 *>(src + i);
          v[i] += x.x; v[i + 1] += x.y; v[i + 2] += x.z; v[i + 3] += x.w;
        }
      }
      if (row < m.rows && !abort_flag) {
        float *c = m.C + row * m.ldc + col_base + cb * 32;
#pragma unroll
        for (int i = 0; i < 32; i += 4) {
          float4 o = make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]);
          if (accumulate) {
            const float4 x = *reinterpret_cast<const float4 *>(c + i);
            o.x += x.x; o.y += x.y; o.z += x.z; o.w += x.w;
          }
          *reinterpret_cast<float4 *>(c + i) = o;
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 2) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kBN));
  }
}

// Persistent form for tasks not split over a cluster: one CTA per SM.  Its
// producer thread takes task tickets from a counter in global memory
// (status[1]; heaviest tasks first, so SMs that finish early take more) and
// passes them to the MMA issuer and the epilogue warps through a four-entry
// queue in shared memory; the last CTA to finish resets the counter
// (status[2] counts finished CTAs).  Warp 0 (one thread) bulk-copies the
// stages of its tasks through the ring without a break between tasks;
// warp 1 (one thread) issues the MMAs into two 128-column accumulators in
// tensor memory, alternating per task; warps 2-5 drain the finished
// accumulator (warp w reads TMEM lanes 32*(w%4) ..) and store C while the
// next task's stages load and multiply.  Every wait is bounded; on expiry the
// CTA records 1 (producer), 2 (MMA issuer) or 3 (epilogue) in *status (the
// first error stays), stores nothing more, and still frees its tensor memory.
constexpr int kPersistThreads = 192;
constexpr int kTaskQ = 4;
template <bool BATCH, int MODE>
__global__ void __launch_bounds__(kPersistThreads, 1)
dense_gemm_persist_kernel(DenseMat one, const DenseMat *__restrict__ mats, const int4 *__restrict__ tasks,
                          int64_t ntasks, int accumulate, int *status) {
  constexpr int NST = mode_stages(MODE);
  constexpr int SB = 2 * mode_images(MODE) * mode_tile_bytes(MODE);
  constexpr int OP = mode_images(MODE) * mode_tile_bytes(MODE);  // bytes of one operand's images
  extern __shared__ __align__(1024) uint8_t dsmem[];
  uint8_t *ring = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(dsmem) + 1023) & ~(uintptr_t)1023);
  __shared__ __align__(8) uint64_t full_bar[NST], empty_bar[NST], acc_full[2], acc_empty[2], done_bar;
  __shared__ __align__(8) uint64_t tq_full[kTaskQ], tq_empty[kTaskQ];
  __shared__ int tq[kTaskQ];
  __shared__ uint32_t tmem_base;
  __shared__ int abort_flag;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  int *ctr = status + 1, *done = status + 2;

  if (threadIdx.x == 0) {
    for (int s = 0; s < NST; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&acc_full[a], 1);
      mbar_init(&acc_empty[a], 4);
    }
    for (int q = 0; q < kTaskQ; ++q) {
      mbar_init(&tq_full[q], 1);
      mbar_init(&tq_empty[q], 5);  // the MMA issuer and the four epilogue warps
    }
    mbar_init(&done_bar, 1);
    abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 2) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_base)),
                 "r"(2 * kBN));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_base;

  if (threadIdx.x == 0) {
    // producer: stage counter g runs over all kept chunks of all this CTA's tasks
    uint32_t g = 0;
    for (int j = 0;; ++j) {
      const int q = j & (kTaskQ - 1);
      if (j >= kTaskQ && !mbar_wait(&tq_empty[q], ((j / kTaskQ) - 1) & 1, &abort_flag)) {
        atomicCAS(status, 0, 1);
        abort_flag = 1;
        break;
      }
      const int t = atomicAdd(ctr, 1);
      tq[q] = t < ntasks ? t : -1;
      mbar_arrive(&tq_full[q]);
      if (t >= ntasks) break;
      const int4 task = tasks[t];
      DenseMat m;
      if constexpr (BATCH) m = mats[task.x];
      else m = one;
      if (m.starve) continue;  // test hook: no copies, the MMA issuer's wait expires
      const int c0 = m.rb_ptr[task.y], c1 = m.rb_ptr[task.y + 1];
      for (int ci = c0; ci < c1; ++ci, ++g) {
        const int s = (int)(g % NST);
        if (g >= (uint32_t)NST && !mbar_wait(&empty_bar[s], ((g / NST) - 1) & 1, &abort_flag)) {
          atomicCAS(status, 0, 1);
          abort_flag = 1;
          break;
        }
        uint8_t *st = ring + (size_t)s * SB;
        const uint8_t *at = m.a_tiles + (size_t)ci * OP;
        const uint8_t *bt = m.b_tiles + ((size_t)task.z * m.k_chunks + m.rb_chunk[ci]) * OP;
        mbar_expect_tx(&full_bar[s], SB);
        bulk_copy(st, at, OP, &full_bar[s]);
        bulk_copy(st + OP, bt, OP, &full_bar[s]);
      }
      if (abort_flag) break;
    }
    // every CTA has taken its last ticket once all have counted themselves here
    if (atomicAdd(done, 1) == (int)gridDim.x - 1) {
      atomicExch(ctr, 0);
      atomicExch(done, 0);
    }
  } else if (threadIdx.x == 32) {
    // MMA issuer
    uint32_t g = 0;
    for (int j = 0;; ++j) {
      const int q = j & (kTaskQ - 1);
      if (!mbar_wait(&tq_full[q], (j / kTaskQ) & 1, &abort_flag)) {
        atomicCAS(status, 0, 2);
        abort_flag = 1;
        break;
      }
      const int t = tq[q];
      mbar_arrive(&tq_empty[q]);
      if (t < 0) break;
      const int4 task = tasks[t];
      DenseMat m;
      if constexpr (BATCH) m = mats[task.x];
      else m = one;
      const int a = j & 1;
      if (j >= 2 && !mbar_wait(&acc_empty[a], ((j >> 1) - 1) & 1, &abort_flag)) {
        atomicCAS(status, 0, 2);
        abort_flag = 1;
        break;
      }
      tc_fence_after();
      const int nk = m.rb_ptr[task.y + 1] - m.rb_ptr[task.y];
      bool ok = true;
      for (int i = 0; i < nk; ++i, ++g) {
        const int s = (int)(g % NST);
        if (!mbar_wait(&full_bar[s], (g / NST) & 1, &abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        mma_stage<MODE>(tmem + (uint32_t)(a * kBN), smem_u32(ring + (size_t)s * SB), i == 0);
        mma_commit(&empty_bar[s]);  // stage free once these MMAs have read it
      }
      if (!ok) {
        atomicCAS(status, 0, 2);
        abort_flag = 1;
        break;
      }
      mma_commit(&acc_full[a]);  // accumulator a complete (arrives at once when nk == 0)
    }
    mma_commit(&done_bar);  // every MMA issued here has completed
  } else if (warp >= 2) {
    // epilogue
    const int qr = warp & 3;  // TMEM lanes 32qr .. 32qr + 31 = tile rows
    for (int j = 0;; ++j) {
      const int q = j & (kTaskQ - 1);
      if (!mbar_wait(&tq_full[q], (j / kTaskQ) & 1, &abort_flag)) {
        if (lane == 0) atomicCAS(status, 0, 3);
        abort_flag = 1;
        break;
      }
      const int t = tq[q];
      __syncwarp();
      if (lane == 0) mbar_arrive(&tq_empty[q]);
      if (t < 0) break;
      const int4 task = tasks[t];
      DenseMat m;
      if constexpr (BATCH) m = mats[task.x];
      else m = one;
      const int a = j & 1;
      if (!mbar_wait(&acc_full[a], (j >> 1) & 1, &abort_flag)) {
        if (lane == 0) atomicCAS(status, 0, 3);
        abort_flag = 1;
        break;
      }
      __syncwarp();
      tc_fence_after();
      const bool have = m.rb_ptr[task.y + 1] > m.rb_ptr[task.y];
      const int64_t row = (int64_t)task.y * kBM + qr * 32 + lane;
      const uint32_t trow = tmem + (uint32_t)(a * kBN) + ((uint32_t)(qr * 32) << 16);
#pragma unroll 1
      for (int cb = 0; cb < kBN / 32; ++cb) {
        float v[32];
        if (have) tmem_ld32(trow + (uint32_t)(cb * 32), v);
        else {
#pragma unroll
          for (int i = 0; i < 32; ++i) v[i] = 0.f;
        }
        if (row < m.rows && !abort_flag) {
          float *c = m.C + row * m.ldc + task.z * kBN + cb * 32;
#pragma unroll
          for (int i = 0; i < 32; i += 4) {
            float4 o = make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]);
            if (accumulate) {
              const float4 x = *reinterpret_cast<const float4 *>(c + i);
              o.x += x.x; o.y += x.y; o.z += x.z; o.w += x.w;
            }
            *reinterpret_cast<float4 *>(c + i) = o;
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[a]);
    }
  }
  // free tensor memory only after the MMAs issued here have completed
  if (threadIdx.x == 32) mbar_wait(&done_bar, 0, nullptr);
  tc_fence_before();
  __syncthreads();
  if (warp == 2) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(2 * kBN));
  }
}

// Rows [kc*BK, kc*BK + BK) x columns [nt*128, nt*128 + 128) of B into T (zero
// past K or N).  With 16-byte aligned rows every thread issues its BK/8
// float4 loads together (the scalar form left this kernel latency-bound);
// otherwise scalar loads.
template <int BK>
__device__ __forceinline__ void load_b_chunk(const DenseMat &m, int nt, int kc, float (&T)[BK][kBN + 1]) {
  const bool vec = (reinterpret_cast<uintptr_t>(m.B) % 16 == 0) && (m.ldb % 4 == 0);
  if (vec) {
    constexpr int kQuads = BK * kBN / 4;
    constexpr int kPer = kQuads / 256;  // launched with 256 threads
    float4 x[kPer];
#pragma unroll
    for (int i = 0; i < kPer; ++i) {
      const int q = threadIdx.x + i * 256;
      const int k = q / (kBN / 4), n4 = (q % (kBN / 4)) * 4;
      const int gk = kc * BK + k, gn = nt * kBN + n4;
      x[i] = (gk < m.k_rows && gn < m.n_cols) ? __ldg(reinterpret_cast<const float4 *>(m.B + (int64_t)gk * m.ldb + gn))
                                              : make_float4(0.f, 0.f, 0.f, 0.f);
    }
#pragma unroll
    for (int i = 0; i < kPer; ++i) {
      const int q = threadIdx.x + i * 256;
      const int k = q / (kBN / 4), n4 = (q % (kBN / 4)) * 4;
      T[k][n4] = x[i].x;
      T[k][n4 + 1] = x[i].y;
      T[k][n4 + 2] = x[i].z;
      T[k][n4 + 3] = x[i].w;
    }
  } else {
    for (int e = threadIdx.x; e < kBN * BK; e += blockDim.x) {
      const int n = e % kBN, k = e / kBN;
      const int gk = kc * BK + k, gn = nt * kBN + n;
      T[k][n] = (gk < m.k_rows && gn < m.n_cols) ? __ldg(m.B + (int64_t)gk * m.ldb + gn) : 0.f;
    }
  }
}

// B (K x N row-major fp32) -> per (n tile, K chunk) [hi | lo] K-major
// swizzled images; rows of a B image are C columns (n), K-chunk tail zeroed.
// Block (x, y): tile x of matrix y.  The 32 x 128 chunk is read coalesced
// (n fastest) into shared memory, then the images are written in order.
template <bool BATCH>
__global__ void __launch_bounds__(256) split_b_kernel(DenseMat one, const DenseMat *__restrict__ mats) {
  __shared__ float T[kBK][kBN + 1];
  DenseMat m;
  if constexpr (BATCH) m = mats[blockIdx.y];
  else m = one;
  const int tile = blockIdx.x;
  if (tile >= m.n_tiles * m.k_chunks) return;
  const int nt = tile / m.k_chunks, kc = tile % m.k_chunks;
  load_b_chunk<kBK>(m, nt, kc, T);
  __syncthreads();
  float4 *hi = reinterpret_cast<float4 *>(m.b_tiles + ((size_t)nt * m.k_chunks + kc) * 2 * kTileBytes);
  float4 *lo = hi + kTileBytes / 16;
  // 16-byte chunk q of the image: row n = q / 8, physical chunk c = q % 8,
  // holding logical k = 4 * (c ^ (n & 7)) .. +3
  for (int q = threadIdx.x; q < kBN * kBK / 4; q += blockDim.x) {
    const int n = q >> 3, c = q & 7;
    const int k0 = ((c ^ (n & 7)) << 2);
    float h[4], l[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float x = T[k0 + j][n];
      h[j] = tf32_round(x);
      l[j] = tf32_round(x - h[j]);
    }
    hi[q] = make_float4(h[0], h[1], h[2], h[3]);
    lo[q] = make_float4(l[0], l[1], l[2], l[3]);
  }
}

// bf16 mode: one image per (n tile, 64-wide K chunk).
template <bool BATCH>
__global__ void __launch_bounds__(256) split_b_bf16_kernel(DenseMat one, const DenseMat *__restrict__ mats) {
  __shared__ float T[kBKb][kBN + 1];
  DenseMat m;
  if constexpr (BATCH) m = mats[blockIdx.y];
  else m = one;
  const int tile = blockIdx.x;
  if (tile >= m.n_tiles * m.k_chunks) return;
  const int nt = tile / m.k_chunks, kc = tile % m.k_chunks;
  load_b_chunk<kBKb>(m, nt, kc, T);
  __syncthreads();
  uint4 *img = reinterpret_cast<uint4 *>(m.b_tiles + ((size_t)nt * m.k_chunks + kc) * kTileBytes);
  // 16-byte chunk q: row n = q / 8, physical chunk c = q % 8 holding logical
  // k = 8 * (c ^ (n & 7)) .. +7
  for (int q = threadIdx.x; q < kBN * 8; q += blockDim.x) {
    const int n = q >> 3, c = q & 7;
    const int k0 = (c ^ (n & 7)) << 3;
    uint32_t w[4];
#pragma unroll
    for (int j = 0; j < 4; ++j)
      w[j] = (uint32_t)bf16_bits(T[k0 + 2 * j][n]) | ((uint32_t)bf16_bits(T[k0 + 2 * j + 1][n]) << 16);
    img[q] = make_uint4(w[0], w[1], w[2], w[3]);
  }
}

// bf16 x3 mode: three images (x1, x2, x3 parts) per (n tile, 32-wide K chunk),
// 64-byte swizzled rows.
template <bool BATCH>
__global__ void __launch_bounds__(256) split_b_bf16x3_kernel(DenseMat one, const DenseMat *__restrict__ mats) {
  constexpr int TB = mode_tile_bytes(kModeBf16x3);
  __shared__ float T[kBKx3][kBN + 1];
  DenseMat m;
  if constexpr (BATCH) m = mats[blockIdx.y];
  else m = one;
  const int tile = blockIdx.x;
  if (tile >= m.n_tiles * m.k_chunks) return;
  const int nt = tile / m.k_chunks, kc = tile % m.k_chunks;
  load_b_chunk<kBKx3>(m, nt, kc, T);
  __syncthreads();
  uint4 *img = reinterpret_cast<uint4 *>(m.b_tiles + ((size_t)nt * m.k_chunks + kc) * 3 * TB);
  // 16-byte chunk q: row n = q / 4, physical chunk c = q % 4 holding logical
  // k = 8 * (c ^ ((n >> 1) & 3)) .. +7; the parts from the hardware bf16
  // conversion (round to nearest even at each step, as bf16x3_split)
  for (int q = threadIdx.x; q < kBN * 4; q += blockDim.x) {
    const int n = q >> 2, c = q & 3;
    const int k0 = (c ^ ((n >> 1) & 3)) << 3;
    uint32_t w[3][4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 x = make_float2(T[k0 + 2 * j][n], T[k0 + 2 * j + 1][n]);
      const __nv_bfloat162 p1 = __floats2bfloat162_rn(x.x, x.y);
      const float2 f1 = __bfloat1622float2(p1);
      // inf / nan (or rounded up to inf): no tail parts
      const bool okx = (__bfloat16_as_ushort(p1.x) & 0x7f80u) != 0x7f80u;
      const bool oky = (__bfloat16_as_ushort(p1.y) & 0x7f80u) != 0x7f80u;
      const float2 r1 = make_float2(okx ? x.x - f1.x : 0.f, oky ? x.y - f1.y : 0.f);
      const __nv_bfloat162 p2 = __floats2bfloat162_rn(r1.x, r1.y);
      const float2 f2 = __bfloat1622float2(p2);
      const __nv_bfloat162 p3 = __floats2bfloat162_rn(r1.x - f2.x, r1.y - f2.y);
      w[0][j] = *reinterpret_cast<const uint32_t *>(&p1);
      w[1][j] = *reinterpret_cast<const uint32_t *>(&p2);
      w[2][j] = *reinterpret_cast<const uint32_t *>(&p3);
    }
#pragma unroll
    for (int r = 0; r < 3; ++r) img[r * (TB / 16) + q] = make_uint4(w[r][0], w[r][1], w[r][2], w[r][3]);
  }
}

}  // namespace
}  // namespace dense
}  // namespace sc

int sc_dense_split_b(const sc::dense::DenseMat &one, const sc::dense::DenseMat *mats, int nmats, int max_tiles,
                     int mode, cudaStream_t s) {
  using namespace sc::dense;
  if (nmats <= 0 || max_tiles <= 0) return 0;
  if (mode == kModeBf16x3) {
    if (mats) split_b_bf16x3_kernel<true><<<dim3(max_tiles, nmats), 256, 0, s>>>(one, mats);
    else split_b_bf16x3_kernel<false><<<dim3(max_tiles, 1), 256, 0, s>>>(one, nullptr);
  } else if (mode == kModeBf16) {
    if (mats) split_b_bf16_kernel<true><<<dim3(max_tiles, nmats), 256, 0, s>>>(one, mats);
    else split_b_bf16_kernel<false><<<dim3(max_tiles, 1), 256, 0, s>>>(one, nullptr);
  } else {
    if (mats) split_b_kernel<true><<<dim3(max_tiles, nmats), 256, 0, s>>>(one, mats);
    else split_b_kernel<false><<<dim3(max_tiles, 1), 256, 0, s>>>(one, nullptr);
  }
  return (int)cudaGetLastError();
}

// SC_DENSE_PERSIST=0 keeps one CTA per task (measurement switch).
static bool persist_enabled() {
  static const bool v = [] {
    const char *e = getenv("SC_DENSE_PERSIST");
    return !(e && e[0] == '0');
  }();
  return v;
}

int sc_dense_gemm(const sc::dense::DenseMat &one, const sc::dense::DenseMat *mats, const int4 *tasks,
                  int64_t ntasks, int split, int mode, int accumulate, int *status, cudaStream_t s) {
  using namespace sc::dense;
  if (ntasks <= 0) return 0;
  if (mode < 0 || mode > 2) return (int)cudaErrorInvalidValue;
  const size_t smem = (size_t)kStages * kStageBytes + 1024;  // 192 KiB ring in every mode
  using Fn = void (*)(DenseMat, const DenseMat *, const int4 *, int, int *);
  const Fn table[2][3] = {{dense_gemm_kernel<false, kModeTf32x3>, dense_gemm_kernel<false, kModeBf16>,
                           dense_gemm_kernel<false, kModeBf16x3>},
                          {dense_gemm_kernel<true, kModeTf32x3>, dense_gemm_kernel<true, kModeBf16>,
                           dense_gemm_kernel<true, kModeBf16x3>}};
  const Fn fn = table[mats ? 1 : 0][mode];
  if (split == 1 && persist_enabled()) {
    // persistent kernel: one CTA per SM over the tasks, double-buffered accumulator
    using PFn = void (*)(DenseMat, const DenseMat *, const int4 *, int64_t, int, int *);
    const PFn ptable[2][3] = {
        {dense_gemm_persist_kernel<false, kModeTf32x3>, dense_gemm_persist_kernel<false, kModeBf16>,
         dense_gemm_persist_kernel<false, kModeBf16x3>},
        {dense_gemm_persist_kernel<true, kModeTf32x3>, dense_gemm_persist_kernel<true, kModeBf16>,
         dense_gemm_persist_kernel<true, kModeBf16x3>}};
    const PFn pfn = ptable[mats ? 1 : 0][mode];
    static std::atomic<unsigned> pattr_done[6];
    int dev = 0, sms = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    std::atomic<unsigned> &bits = pattr_done[(mats ? 1 : 0) + 2 * mode];
    if (dev >= 32 || !(bits.load() & (1u << dev))) {
      cudaError_t e = cudaFuncSetAttribute(pfn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      if (e != cudaSuccess) return (int)e;
      if (dev < 32) bits.fetch_or(1u << dev);
    }
    const int64_t grid = std::max<int64_t>(1, std::min<int64_t>(ntasks, sms));
    pfn<<<(unsigned)grid, kPersistThreads, smem, s>>>(one, mats, tasks, ntasks, accumulate, status);
    return (int)cudaGetLastError();
  }
  // one bit per device ordinal (< 32); concurrent callers may both set the
  // attribute, which is harmless, and the bit update is atomic
  static std::atomic<unsigned> attr_done[6];
  int dev = 0;
  cudaGetDevice(&dev);
  std::atomic<unsigned> &bits = attr_done[(mats ? 1 : 0) + 2 * mode];
  if (dev >= 32 || !(bits.load() & (1u << dev))) {
    cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return (int)e;
    if (dev < 32) bits.fetch_or(1u << dev);
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(ntasks * split), 1, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = (unsigned)split;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = split > 1 ? 1 : 0;
  cudaError_t e = cudaLaunchKernelEx(&cfg, fn, one, mats, tasks, accumulate, status);
  if (e != cudaSuccess) return (int)e;
  return (int)cudaGetLastError();
}
