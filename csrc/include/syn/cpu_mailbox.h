// Host-mapped mailbox between a decode step on the GPU and the CPU expert workers (the role of
// the MoE doorbell layer, reference crates/kernels/src/moe/doorbell.rs, and of the CPU expert
// misses, crates/kernels-cpu/src/moe.rs): the GPU publishes the routed rows of a layer, the
// host computes the cold experts it owns, the GPU waits for the answer before combining.
//
// One pinned buffer, shared by every MoE layer (layers hand off one after the other):
//   words [0..15]  : go line   -- [0] go sequence (GPU release-stores it last), [1] layer, [2] rows
//   words [16..31] : done line -- [16] done sequence (CPU release-stores it last), [17] n_out,
//                                 [18] CPU error bits
//   then tok_off [E+1] i32, tok_idx [R*k] i32, pair_w [R*k] f32, h [R][H] bf16,
//   out_pairs [R*k] i32 (pair index of each CPU output row), out [R*k][H] f32.
// The go and done words sit on separate 64-byte lines so neither side's polling shares a line
// with the other side's writes.
#pragma once
#include <stdint.h>

#ifdef __CUDACC__
#define SYN_MB_HD __host__ __device__ __forceinline__
#else
#define SYN_MB_HD inline
#endif

namespace syn {

constexpr int MB_GO = 0, MB_LAYER = 1, MB_ROWS = 2;
constexpr int MB_DONE = 16, MB_NOUT = 17, MB_ERR = 18;

struct CpuMailboxLayout {
  int64_t tok_off, tok_idx, pair_w, h, out_pairs, out, bytes;
};

SYN_MB_HD int64_t mb_align(int64_t x) { return (x + 255) & ~int64_t(255); }

SYN_MB_HD CpuMailboxLayout cpu_mailbox_layout(int64_t E, int64_t k, int64_t max_rows, int64_t H) {
  CpuMailboxLayout l;
  int64_t o = 256;
  l.tok_off = o;   o = mb_align(o + (E + 1) * 4);
  l.tok_idx = o;   o = mb_align(o + max_rows * k * 4);
  l.pair_w = o;    o = mb_align(o + max_rows * k * 4);
  l.h = o;         o = mb_align(o + max_rows * H * 2);
  l.out_pairs = o; o = mb_align(o + max_rows * k * 4);
  l.out = o;       o = mb_align(o + max_rows * k * H * 4);
  l.bytes = o;
  return l;
}

}  // namespace syn
