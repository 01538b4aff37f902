// Shared epilogue of the decode GEMV kernels (4-bit and fp8): output modes and the
// per-(row, pair) store.
#pragma once
#include "common.cuh"
#include "syn/launch.h"

namespace syn {

enum GemvMode : int {
  GEMV_STORE_BF16 = 0,   // out_bf16[p][n]
  GEMV_SWIGLU = 1,       // rows interleaved in 8-row gate/up chunks -> out_bf16[p][n/2]
  GEMV_SCALED_F32 = 2,   // out_f32[p][n] = route_w[p] * y
  GEMV_ADD_F32 = 3,      // out_f32[p][n] += y (residual stream kept in f32)
  GEMV_SCALED_F32_PTR = 4,  // ((float*)out_ptrs[p])[n] = route_w[p] * y (peer memory allowed)
  GEMV_STORE_F32 = 5,    // out_f32[p][n] = y (logits)
  GEMV_PEERS_F32 = 6,    // y -> every TP peer's receive slot (one-shot all-reduce push)
};


__device__ __forceinline__ uint4 ld_stream_v4(const uint4* p) { return __ldcs(p); }
__device__ __forceinline__ uint2 ld_stream_v2(const uint2* p) { return __ldcs(p); }

// Epilogue for one (row n, token j) value.  `p` is the pair index.
__device__ __forceinline__ void gemv_store(const GemvArgs& a, int p, int n, float v) {
  switch (a.mode) {
    case GEMV_STORE_BF16:
      reinterpret_cast<__nv_bfloat16*>(a.out)[(int64_t)p * a.N + n] = f2bf(v);
      break;
    case GEMV_SCALED_F32:
      reinterpret_cast<float*>(a.out)[(int64_t)p * a.N + n] = a.route_w[p] * v;
      break;
    case GEMV_ADD_F32:
      reinterpret_cast<float*>(a.out)[(int64_t)p * a.N + n] += v;
      break;
    case GEMV_STORE_F32:
      reinterpret_cast<float*>(a.out)[(int64_t)p * a.N + n] = v;
      break;
    case GEMV_SCALED_F32_PTR:
      reinterpret_cast<float*>(a.out_ptrs[p])[n] = a.route_w[p] * v;
      break;
    case GEMV_PEERS_F32:
      for (int q = 0; q < a.sig_n; ++q)
        reinterpret_cast<float*>(a.sig_peers[q] + a.peer_off)[((int64_t)a.sig_rank * a.peer_cap + p) * a.N + n] = v;
      break;
    default:
      break;
  }
}

}  // namespace syn
