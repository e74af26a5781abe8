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

// 3xBF16 mode (the default for fp32 plans where it measures faster): every
// fp32 operand split into three bf16 parts, x = x1 + x2 + x3 (x1 = rn(x),
// x2 = rn(x - x1), x3 = rn(x - x1 - x2): 24 significant bits), and the
// products x1y1 + x1y2 + x2y1 + x2y2 + x1y3 + x3y1 accumulated in fp32; the
// dropped terms are ~2^-24 relative, inside the fp32 parity bound.  Six
// images of 2 bytes instead of two of 4 bytes per element at the same
// tensor-pipe time (kind::f16 runs at twice the kind::tf32 rate).
constexpr int kModeTf32x3 = 0;
constexpr int kModeBf16 = 1;
constexpr int kModeBf16x3 = 2;
__host__ __device__ constexpr int mode_images(int mode) { return mode == kModeBf16 ? 1 : (mode == kModeBf16x3 ? 3 : 2); }
// 3xBF16 stages hold 32-wide K chunks in 64-byte swizzled rows (six 8 KiB
// images, 48 KiB a stage, four stages); the other modes 128-byte rows.
constexpr int kBKx3 = 32;
__host__ __device__ constexpr int mode_bk(int mode) {
  return mode == kModeTf32x3 ? kBK : (mode == kModeBf16x3 ? kBKx3 : kBKb);
}
__host__ __device__ constexpr int mode_tile_bytes(int mode) { return mode == kModeBf16x3 ? kTileBytes / 2 : kTileBytes; }
__host__ __device__ constexpr int mode_stages(int mode) { return mode == kModeBf16 ? 6 : (mode == kModeBf16x3 ? 4 : kStages); }

// 64-byte swizzle (3xBF16 images): row r of 64 bytes, 16-byte chunk c stored
// at c ^ ((r >> 1) & 3) -- byte address bits [4,6) xor bits [7,9).
__host__ __device__ inline uint32_t swz_offset_bf16_64(int r, int k) {
  const uint32_t chunk = (uint32_t)(k >> 3) ^ (uint32_t)((r >> 1) & 3);
  return (uint32_t)r * 64u + chunk * 16u + (uint32_t)(k & 7) * 2u;
}

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

__host__ __device__ inline float bf16_float(uint16_t h) {
  const uint32_t u = (uint32_t)h << 16;
  float y;
  memcpy(&y, &u, 4);
  return y;
}

// The three bf16 parts of x (3xBF16 mode).
__host__ __device__ inline void bf16x3_split(float x, uint16_t (&h)[3]) {
  h[0] = bf16_bits(x);
  if ((h[0] & 0x7f80u) == 0x7f80u) {  // inf / nan (or rounded up to inf): no tail parts
    h[1] = h[2] = 0;
    return;
  }
  const float r1 = x - bf16_float(h[0]);
  h[1] = bf16_bits(r1);
  h[2] = bf16_bits(r1 - bf16_float(h[1]));
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
  int bf16;                 // tile mode: kModeTf32x3, kModeBf16 or kModeBf16x3
  int starve = 0;           // test hook: the producer issues no copies, so the
                            // MMA issuer's bounded wait expires (status 2, then 3)
};

}  // namespace dense
}  // namespace sc

// Launch helpers (sc_dense.cu).  `mats` is a device array of `nmats`
// matrices (or nullptr with `one` used instead when nmats == 1); `tasks`
// holds int4 {matrix, row block, n tile, kept chunks}, heaviest first.
// `mode`: sc::dense::kModeTf32x3, kModeBf16 or kModeBf16x3.
int sc_dense_split_b(const sc::dense::DenseMat &one, const sc::dense::DenseMat *mats, int nmats, int max_tiles,
                     int mode, cudaStream_t s);
int sc_dense_gemm(const sc::dense::DenseMat &one, const sc::dense::DenseMat *mats, const int4 *tasks,
                  int64_t ntasks, int split, int mode, int accumulate, int *status, cudaStream_t s);
