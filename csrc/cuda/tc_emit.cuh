// Epilogue of the dense tcgen05 GEMMs (bf16 weights: gemm_bf16_tc.cu; 4-bit weights in the
// decode orientation: gemm_q4_dec.cu): the argument block, the thread-block-cluster helpers of
// the split-K reduction, and the per-lane store of a 32-column group of the TMEM accumulator
// in both orientations (bf16 store, SwiGLU of interleaved 8-row gate/up chunks, f32 add / store,
// and the tensor-parallel peer push over NVLink).
#pragma once
#include "tc_common.cuh"

namespace syn {

struct DenseGemmArgs {
  int decode;               // 1: A = W, B = X; 0: A = X, B = W
  int T, N, K;              // tokens, outputs, reduction length
  int splits;               // K slices per row tile (decode)
  int mode;                 // 0 bf16, 1 SwiGLU bf16 [T, N/2], 3 f32 +=, 5 f32 =, 6 peer push f32
  void* out;
  int ldo;                  // output row stride (elements)
  // peer push (mode 6): row t of output column n -> peers[d] + off_recv + (rank * src_stride + t' * ldo + n) * 4
  // with d = every rank (owner_rows == 0; t' = t) or d = t / owner_rows (t' = t % owner_rows)
  const int64_t* peers;
  int n_peers, rank, cap, owner_rows;
  int64_t src_stride;
  int64_t off_recv, off_flag;
  unsigned* done_ctr;       // CTA arrivals of the launch (left zero)
  const uint32_t* step_ctr;
  int n_layers, layer;
  int* status;
  int vec_out;              // out and ldo allow 16-byte row-major epilogue stores (prefill orientation)
};


// Thread-block cluster helpers: every thread of every CTA of the cluster passes the barrier;
// a load from the same shared-memory offset of CTA `rank` of the cluster.
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\nbarrier.cluster.wait.acquire.aligned;\n" ::: "memory");
}
__device__ __forceinline__ float4 ld_dsmem_f4(const float* local, int rank) {
  uint32_t remote;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;\n" : "=r"(remote) : "r"(smem_u32(local)), "r"(rank));
  float4 v;
  asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];\n"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(remote)
               : "memory");
  return v;
}

// Epilogue of one 32-column group of one TMEM lane (row r of D).
template <int BN, int MODE, bool DEC>
__device__ __forceinline__ void bf16_emit(const DenseGemmArgs& a, int tile_a, int tile_b, int r, int c0,
                                          const float* v, int nc = 32) {
  if constexpr (DEC) {
    const int n = tile_a * 128 + r;  // output feature of this lane
    if constexpr (MODE == 1) {
      // interleaved gate/up: rows 16c..16c+7 gate, 16c+8..16c+15 up; the partner is lane ^ 8
      const bool gate = (n & 8) == 0;
      const int m = (n >> 4) * 8 + (n & 7);
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        const float other = __shfl_xor_sync(0xffffffffu, v[j], 8);
        const int t = c0 + j;
        if (gate && j < nc && t < a.T && n < a.N)
          reinterpret_cast<__nv_bfloat16*>(a.out)[(int64_t)t * a.ldo + m] = f2bf(silu(v[j]) * other);
      }
      return;
    }
    if (n >= a.N) return;  // rows past N of a partial tile (zero-filled by TMA)
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      const int t = c0 + j;
      if (j >= nc || t >= a.T) continue;
      const int64_t o = (int64_t)t * a.ldo + n;
      if constexpr (MODE == 0) {
        reinterpret_cast<__nv_bfloat16*>(a.out)[o] = f2bf(v[j]);
      } else if constexpr (MODE == 3) {
        reinterpret_cast<float*>(a.out)[o] += v[j];
      } else if constexpr (MODE == 5) {
        reinterpret_cast<float*>(a.out)[o] = v[j];
      } else {  // 6: peer push
        if (a.owner_rows > 0) {
          const int d = t / a.owner_rows, tt = t % a.owner_rows;
          float* dst = reinterpret_cast<float*>(a.peers[d] + a.off_recv);
          dst[(int64_t)a.rank * a.src_stride + (int64_t)tt * a.ldo + n] = v[j];
        } else {
          for (int d = 0; d < a.n_peers; ++d) {
            float* dst = reinterpret_cast<float*>(a.peers[d] + a.off_recv);
            dst[(int64_t)a.rank * a.src_stride + (int64_t)t * a.ldo + n] = v[j];
          }
        }
      }
    }
    return;
  }
  // prefill orientation: lane = token, 32 consecutive output columns
  const int t = tile_a * 128 + r;
  const int n0 = tile_b * BN + c0;
  if (t >= a.T || n0 >= a.N) return;  // N % 32 == 0: a 32-column group is all in or all out
  if constexpr (MODE == 1) {
    __nv_bfloat16* o = reinterpret_cast<__nv_bfloat16*>(a.out) + (int64_t)t * a.ldo + n0 / 2;
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const int gi = (j / 8) * 16 + (j % 8);
      o[j] = f2bf(silu(v[gi]) * v[gi + 8]);
    }
  } else if constexpr (MODE == 0) {
    uint4* o = reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(a.out) + (int64_t)t * a.ldo + n0);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      uint4 w;
      w.x = pack_bf16x2(v[8 * j + 0], v[8 * j + 1]);
      w.y = pack_bf16x2(v[8 * j + 2], v[8 * j + 3]);
      w.z = pack_bf16x2(v[8 * j + 4], v[8 * j + 5]);
      w.w = pack_bf16x2(v[8 * j + 6], v[8 * j + 7]);
      o[j] = w;
    }
  } else if constexpr (MODE == 3 || MODE == 5) {
    float4* o = reinterpret_cast<float4*>(reinterpret_cast<float*>(a.out) + (int64_t)t * a.ldo + n0);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      float4 w = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
      if constexpr (MODE == 3) {
        const float4 p = o[j];
        w.x += p.x;
        w.y += p.y;
        w.z += p.z;
        w.w += p.w;
      }
      o[j] = w;
    }
  } else {  // 6: peer push
    const int d0 = a.owner_rows > 0 ? t / a.owner_rows : 0;
    const int d1 = a.owner_rows > 0 ? d0 + 1 : a.n_peers;
    const int tt = a.owner_rows > 0 ? t % a.owner_rows : t;
    for (int d = d0; d < d1; ++d) {
      float4* o = reinterpret_cast<float4*>(reinterpret_cast<float*>(a.peers[d] + a.off_recv) +
                                            (int64_t)a.rank * a.src_stride + (int64_t)tt * a.ldo + n0);
#pragma unroll
      for (int j = 0; j < 8; ++j) o[j] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
    }
  }
}

}  // namespace syn
