// MoE split rule between the three sites of an expert-cache miss (reference semantics:
// crates/kernels/include/syntropy/moe_assign.h, RFC-0023 §6, RFC-0040 §3.4):
//   * HIT            when the routed expert has a VRAM cache slot;
//   * copy slot c    when it missed, is copy-eligible, and is the c-th eligible miss in the
//                    order (more tokens first, then lower expert id, then earlier entry),
//                    with c < copy_slots and (c + 1) * expert_bytes <= b_copy;
//   * CPU            otherwise (computed in place from host memory).
// This implementation sorts the eligible misses once (O(n log n)) instead of ranking each
// entry against all others; the assignment it produces is the same.  Usable from host code
// and device code (the sort is an insertion sort over at most n_route entries).
#pragma once
#include <stdint.h>

#ifdef __CUDACC__
#define SYN_MA_HD __host__ __device__
#else
#define SYN_MA_HD
#endif

// Codes shared with the reference's doorbell ABI (crates/kernels/include/syntropy/
// moe_doorbell.h): a route slot's cache_slot is SYN_MOE_MISS when the expert is not resident;
// an assignment is SYN_MOE_HIT, SYN_MOE_CPU or a copy-slot index.
#define SYN_MOE_MISS 0xFFFFFFFFu
#define SYN_MOE_HIT 0xFFFFFFFFu
#define SYN_MOE_CPU 0xFFFFFFFEu

struct syn_doorbell_header {
  uint32_t seq;      // step sequence the layer's routing belongs to
  uint16_t n_route;  // routed (union) experts that follow
  uint16_t n_pred;   // predicted next-layer experts after them
};

struct syn_route_slot {
  uint16_t expert;
  uint16_t tokens;
  uint32_t cache_slot;  // SYN_MOE_MISS when not resident
};

struct syn_pred_slot {
  uint8_t ahead;   // layers ahead (1 = next layer)
  uint8_t _pad;
  uint16_t expert;
};

SYN_MA_HD static inline int syn_moe_before(const struct syn_route_slot* r, uint32_t a, uint32_t b) {
  if (r[a].tokens != r[b].tokens) return r[a].tokens > r[b].tokens;
  if (r[a].expert != r[b].expert) return r[a].expert < r[b].expert;
  return a < b;
}

// `order` is scratch of n_route entries.
SYN_MA_HD static inline void syn_moe_assign(const struct syn_route_slot* route, uint32_t n_route,
                                            const uint32_t* eligible, uint32_t n_experts, uint32_t b_copy,
                                            uint64_t expert_bytes, uint32_t copy_slots, uint32_t* order,
                                            uint32_t* out) {
  uint32_t m = 0;
  for (uint32_t i = 0; i < n_route; ++i) {
    const uint32_t e = route[i].expert;
    if (route[i].cache_slot != SYN_MOE_MISS) {
      out[i] = SYN_MOE_HIT;
    } else {
      out[i] = SYN_MOE_CPU;
      if (e < n_experts && ((eligible[e >> 5] >> (e & 31u)) & 1u)) {
        // insertion into the sorted list of eligible misses
        uint32_t j = m++;
        while (j > 0 && syn_moe_before(route, i, order[j - 1])) {
          order[j] = order[j - 1];
          --j;
        }
        order[j] = i;
      }
    }
  }
  for (uint32_t c = 0; c < m; ++c) {
    if (c < copy_slots && expert_bytes <= (uint64_t)b_copy && ((uint64_t)c + 1u) * expert_bytes <= (uint64_t)b_copy)
      out[order[c]] = c;
  }
}
