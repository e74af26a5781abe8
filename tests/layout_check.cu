// Host-side check of the device layouts' index functions (no GPU needed):
// the 64-byte swizzle of 3xBF16 tile images is a bijection onto the tile and
// follows address bits [4,6) ^= bits [7,9); the lane-block item layout puts
// every (lane, column) and (lane, value slot) in distinct words inside the
// item's size.  Prints "ok" or the first failure.
#include <cstdio>
#include <vector>

#include "sc_dense.cuh"
#include "sc_kernels.cuh"

int main() {
  using namespace sc;
  // 3xBF16 image: 128 rows x 32 bf16 = 8 KiB
  {
    std::vector<int> seen(dense::mode_tile_bytes(dense::kModeBf16x3) / 2, 0);
    for (int r = 0; r < dense::kBM; ++r)
      for (int k = 0; k < dense::kBKx3; ++k) {
        const uint32_t o = dense::swz_offset_bf16_64(r, k);
        const uint32_t plain = (uint32_t)r * 64u + (uint32_t)k * 2u;
        const uint32_t want = plain ^ (((plain >> 7) & 3u) << 4);
        if (o != want || o / 2 >= seen.size() || seen[o / 2]++) {
          printf("swizzle r=%d k=%d -> %u (want %u)\n", r, k, o, want);
          return 1;
        }
      }
  }
  // lane blocks: every popcount, every item width
  for (int p = 1; p <= 6; ++p)
    for (int nl = 1; nl <= 32; ++nl) {
      const uint32_t words = lane_item_words(nl, p);
      std::vector<int> used(words, 0);
      for (int l = 0; l < nl; ++l) used[l / 4] = 1;  // mask bytes: first 8 words
      for (int w = 0; w < 8; ++w) used[w] = 1;
      for (int l = 0; l < nl; ++l)
        for (int u = 0; u < lane_entries(p); u += 2) {  // two 16-bit columns per word
          const uint32_t w = 8 + lane_col_word(nl, p, l, u);
          if (w >= 8 + lane_col_region(nl, p) / 4 || used[w]++) {
            printf("columns p=%d nl=%d l=%d u=%d word %u\n", p, nl, l, u, w);
            return 1;
          }
        }
      const uint32_t v0 = 8 + lane_col_region(nl, p) / 4;
      for (int l = 0; l < nl; ++l)
        for (int q = 0; q < kLaneSlots; ++q) {
          const uint32_t w = v0 + (uint32_t)((q / 4) * nl + l) * 4 + q % 4;
          if (w >= words || used[w]++) {
            printf("values p=%d nl=%d l=%d q=%d word %u of %u\n", p, nl, l, q, w, words);
            return 1;
          }
        }
      if (words % 4) {
        printf("item p=%d nl=%d not a multiple of 16 bytes\n", p, nl);
        return 1;
      }
    }
  printf("ok\n");
  return 0;
}
