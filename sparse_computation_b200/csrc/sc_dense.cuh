// Dense-tile tensor-core path (tcgen05, kind::tf32) for moderately sparse
// matrices: the row panels of a plan are densified into 128-row blocks,
// K-chunks of 32 columns that hold no nonzero are skipped, and each 128x128
// C tile is computed as A_hi*B_hi + A_hi*B_lo + A_lo*B_hi ("3xTF32": every
// fp32 operand split into a TF32 head and a TF32 tail), accumulated in fp32
// in tensor memory.  The dropped A_lo*B_lo term is ~2^-22 relative, so the
// result stays within the fp32 parity tolerance.
//
// Shared-memory tile image (both operands K-major, 128B swizzle): a tile is
// 128 rows x 32 fp32 (128 bytes per row); within each 1024-byte group of 8
// rows the 16-byte chunk c of row r sits at chunk c ^ (r & 7).  A tiles are
// written in this image on the host at plan time; B tiles by a small kernel
// per call, so every stage is loaded with plain bulk copies (cp.async.bulk,
// no tensor map; each copy lands in its own CTA only).
//
// Work: a task is (matrix, 128-row block, 128-column tile); a task's K-chunks
// are split over a thread-block cluster of S CTAs (S in {1, 2, 4}) whose
// partial accumulators are summed through distributed shared memory, so small
// matrices still fill the GPU.  A batch runs the tasks of many matrices (a
// transformer layer stack) in one launch.
#pragma once

#include <cstdint>
#include <cstring>
#include <cuda_runtime.h>

namespace sc {
namespace dense {

constexpr int kBM = 128;             // rows of a tile (MMA M)
constexpr int kBN = 128;             // columns of a C tile (MMA N)
constexpr int kBK = 32;              // K per stage (one 128-byte swizzle row)
constexpr int kTileBytes = kBM * kBK * 4;  // 16 KiB per operand image
constexpr int kStages = 3;
constexpr int kStageBytes = 4 * kTileBytes;  // A_hi, A_lo, B_hi, B_lo
constexpr int kThreads = 128;
constexpr int kMaxSplit = 4;

// Byte offset of element (r, k) of a tile in the swizzled image.
__host__ __device__ inline uint32_t swz_offset(int r, int k) {
  const uint32_t chunk = (uint32_t)(k >> 2) ^ (uint32_t)(r & 7);
  return (uint32_t)r * 128u + chunk * 16u + (uint32_t)(k & 3) * 4u;
}

// fp32 -> TF32 (round to nearest even on the 13 dropped mantissa bits).
__host__ __device__ inline float tf32_round(float x) {
  uint32_t u;
  memcpy(&u, &x, 4);
  if ((u & 0x7f800000u) != 0x7f800000u) {  // finite
    u += 0x0fffu + ((u >> 13) & 1u);
    u &= 0xffffe000u;
  }
  float y;
  memcpy(&y, &u, 4);
  return y;
}

// BF16 mode (opt-in, looser tolerance): A and B tiles hold bf16 (round to
// nearest even), one tcgen05.mma kind::f16 per 16-wide k-step, fp32
// accumulation.  A tile row is still 128 bytes (64 bf16), so the tile image,
// its swizzle and the per-k-step descriptor advance (32 bytes) are the same.
constexpr int kBKb = 64;  // bf16 K per stage

__host__ __device__ inline uint32_t swz_offset_bf16(int r, int k) {
  const uint32_t chunk = (uint32_t)(k >> 3) ^ (uint32_t)(r & 7);
  return (uint32_t)r * 128u + chunk * 16u + (uint32_t)(k & 7) * 2u;
}

__host__ __device__ inline uint16_t bf16_bits(float x) {
  uint32_t u;
  memcpy(&u, &x, 4);
  if ((u & 0x7f800000u) == 0x7f800000u) return (uint16_t)((u >> 16) | ((u & 0xffffu) ? 0x40u : 0u));  // inf/nan
  u += 0x7fffu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}

// One matrix of the dense path.
struct DenseMat {
  const uint8_t *a_tiles;   // per kept (row block, chunk): [hi image | lo image]
  const int32_t *rb_ptr;    // kept chunks of row block b: [rb_ptr[b], rb_ptr[b+1])
  const int32_t *rb_chunk;  // K-chunk index of each kept chunk
  uint8_t *b_tiles;         // per (n tile, K chunk): [hi image | lo image], written per call
  const float *B;
  int64_t ldb;
  float *C;
  int64_t ldc;
  int64_t rows;             // C rows
  int k_rows;               // K
  int n_cols;               // N (multiple of 128)
  int k_chunks;             // ceil(K / 32), or ceil(K / 64) in bf16 mode
  int n_tiles;              // N / 128
  int bf16;                 // 1: bf16 tiles (one image per operand)
  int starve = 0;           // test hook: the producer issues no copies, so the
                            // MMA issuer's bounded wait expires (status 2, then 3)
};

}  // namespace dense
}  // namespace sc

// Launch helpers (sc_dense.cu).  `mats` is a device array of `nmats`
// matrices (or nullptr with `one` used instead when nmats == 1); `tasks`
// holds int4 {matrix, row block, n tile, kept chunks}, heaviest first.
int sc_dense_split_b(const sc::dense::DenseMat &one, const sc::dense::DenseMat *mats, int nmats, int max_tiles,
                     bool bf16, cudaStream_t s);
int sc_dense_gemm(const sc::dense::DenseMat &one, const sc::dense::DenseMat *mats, const int4 *tasks,
                  int64_t ntasks, int split, bool bf16, int accumulate, int *status, cudaStream_t s);
