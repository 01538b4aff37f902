// Step descriptor: the packed per-step inputs of one decode step, written by the host into
// pinned memory and copied to the device as the first operation of every step (the CUDA
// graph of a batch bucket reads only the device copy).  Field order and types:
//   int32 tokens[R], pos[R], ctx_len[R], top_k[R];  f32 temperature[R], top_p[R];
//   int32 block_tables[R][MB];  (padding to 8 bytes)
//   int64 slot[R], seed[R], stream[R], counter[R]
// with R = row capacity and MB = block-table width.  Same semantics as the reference's step
// descriptor (one record per live row, padding rows inert: slot -1, null page, greedy).
#pragma once
#include <stddef.h>
#include <stdint.h>

namespace syn {

struct StepDescLayout {
  int64_t rows, max_blocks;
  size_t off_tokens, off_pos, off_ctx, off_topk, off_temp, off_topp, off_bt;
  size_t off_slot, off_seed, off_stream, off_counter, nbytes;

  StepDescLayout(int64_t r, int64_t mb) : rows(r), max_blocks(mb) {
    size_t o = 0;
    off_tokens = o; o += r * 4;
    off_pos = o; o += r * 4;
    off_ctx = o; o += r * 4;
    off_topk = o; o += r * 4;
    off_temp = o; o += r * 4;
    off_topp = o; o += r * 4;
    off_bt = o; o += r * mb * 4;
    o = (o + 7) & ~size_t(7);
    off_slot = o; o += r * 8;
    off_seed = o; o += r * 8;
    off_stream = o; o += r * 8;
    off_counter = o; o += r * 8;
    nbytes = o;
  }
};

}  // namespace syn
