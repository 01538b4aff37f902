// 4-bit weight format: 32-element blocks along K, each with an fp16 scale d and an
// fp16 min m; element value = d * q + m with q in [0, 15].
//
// Two byte layouts carry the same numbers:
//
// * Row blocks ("q4_1 rows", the interchange layout stored in weight files): per output
//   row, K/32 blocks of 20 bytes {fp16 d, fp16 m, 16 bytes qs}; byte j of qs holds element
//   j in its low nibble and element j + 16 in its high nibble.  This is the GGUF Q4_1 block
//   (public ggml block definition, reference plan/rfcs/RFC-0042-quantization-and-numerical-
//   fidelity.md §2.1 table row Q4_1), kept byte-compatible so GGUF-style files load directly.
//
// * Tiled ("q4t", the device layout): nibbles pre-permuted so that one 128-bit load per
//   lane of a warp yields exactly that lane's mma.sync m16n8k16 A-operand fragments for a
//   16-row x 64-column tile, and scale/min pairs grouped per 16-row tile.  N % 16 == 0 and
//   K % 64 == 0 are required.
//
//   qw  : uint32 [N/16][K/64][32 lanes][4 words]
//         word w of lane l covers block (2*kg + w/2), k-step (w%2) (16 elements each);
//         with g = l/4, t = l%4 and kk the k offset inside that 16-element step:
//           nibble 0: row g,   kk = 2t      nibble 4: row g,   kk = 2t+1
//           nibble 1: row g+8, kk = 2t      nibble 5: row g+8, kk = 2t+1
//           nibble 2: row g,   kk = 2t+8    nibble 6: row g,   kk = 2t+9
//           nibble 3: row g+8, kk = 2t+8    nibble 7: row g+8, kk = 2t+9
//         so ((w >> 4j) & 0x000F000F) is fragment register j as two 16-bit lanes.
//   sm  : half2 (d, m) [N/16][K/64][16 rows][2 blocks]
#pragma once
#include <stdint.h>

#define SYN_Q4_BLOCK 32
#define SYN_Q4_ROW_BLOCK_BYTES 20

#ifdef __CUDACC__
#define SYN_HD __host__ __device__ __forceinline__
#else
#define SYN_HD inline
#endif

namespace syn {

// Position (word index inside qw, nibble index inside the word) of element (n, k).
SYN_HD void q4t_locate(int64_t N, int64_t K, int64_t n, int64_t k, int64_t* word, int* nib) {
  (void)N;
  const int64_t tile = n >> 4;
  const int r = (int)(n & 15);
  const int64_t kg = k >> 6;
  const int kin = (int)(k & 63);
  const int blk = kin >> 5;        // block inside the 64-column group
  const int step = (kin >> 4) & 1; // k16 step inside the block
  const int kk = kin & 15;
  const int g = r & 7;
  const int hi_row = r >> 3;           // 0: row g, 1: row g+8
  const int hi_col = (kk >> 3) & 1;    // 0: cols 2t..2t+1, 1: cols 2t+8..2t+9
  const int t = (kk & 7) >> 1;
  const int odd = kk & 1;
  const int lane = g * 4 + t;
  const int reg = hi_col * 2 + hi_row; // fragment register 0..3
  *nib = reg + 4 * odd;
  *word = (((tile * (K >> 6) + kg) * 32 + lane) * 4) + blk * 2 + step;
}

// Index (in half2 units) of the (d, m) pair of block (n, k/32).
SYN_HD int64_t q4t_scale_index(int64_t K, int64_t n, int64_t kb) {
  const int64_t tile = n >> 4;
  const int r = (int)(n & 15);
  const int64_t kg = kb >> 1;
  const int blk = (int)(kb & 1);
  return ((tile * (K >> 6) + kg) * 16 + r) * 2 + blk;
}

}  // namespace syn
