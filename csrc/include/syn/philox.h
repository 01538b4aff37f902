// Philox4x32-10 counter-based generator, written from its published description:
// J. K. Salmon, M. A. Moraes, R. O. Dror, D. E. Shaw, "Parallel random numbers: as easy as
// 1, 2, 3", SC'11 (multipliers 0xD2511F53 / 0xCD9E8D57, Weyl key increments
// 0x9E3779B9 / 0xBB67AE85, ten rounds).  Shared by the CPU oracle and the device sampler.
//
// Draw contract (reference: plan/decisions/ADR-0107-counter-based-sampling-rng.md):
//   key     = (seed_lo, seed_hi)
//   counter = (rng_counter_lo, rng_counter_hi, stream_lo, stream_hi)
//   draw    = first output word x0; uniform u = x0 / 2^32 in [0, 1).
#pragma once
#include <stdint.h>

#ifdef __CUDACC__
#define SYN_PHX_HD __host__ __device__ __forceinline__
#else
#define SYN_PHX_HD inline
#endif

namespace syn {

SYN_PHX_HD uint32_t phx_mulhi(uint32_t a, uint32_t b) {
  return (uint32_t)(((uint64_t)a * (uint64_t)b) >> 32);
}

SYN_PHX_HD void philox4x32_10(uint32_t c[4], uint32_t k0, uint32_t k1) {
  const uint32_t M0 = 0xD2511F53u, M1 = 0xCD9E8D57u;
  const uint32_t W0 = 0x9E3779B9u, W1 = 0xBB67AE85u;
  for (int r = 0; r < 10; ++r) {
    if (r > 0) {
      k0 += W0;
      k1 += W1;
    }
    const uint32_t hi0 = phx_mulhi(M0, c[0]), lo0 = M0 * c[0];
    const uint32_t hi1 = phx_mulhi(M1, c[2]), lo1 = M1 * c[2];
    const uint32_t n0 = hi1 ^ c[1] ^ k0;
    const uint32_t n2 = hi0 ^ c[3] ^ k1;
    c[0] = n0;
    c[1] = lo1;
    c[2] = n2;
    c[3] = lo0;
  }
}

// The 32-bit draw for (seed, stream, counter).
SYN_PHX_HD uint32_t philox_draw(uint64_t seed, uint64_t stream, uint64_t counter) {
  uint32_t c[4] = {(uint32_t)counter, (uint32_t)(counter >> 32), (uint32_t)stream, (uint32_t)(stream >> 32)};
  philox4x32_10(c, (uint32_t)seed, (uint32_t)(seed >> 32));
  return c[0];
}

}  // namespace syn
