// Causal prefill attention (GQA, head_dim 128) over the paged KV cache: FlashAttention-2
// style online softmax on mma.sync tiles.  Works for plain prefill and for chunked prefill
// after a cached prefix: query row i of sequence s sits at absolute position
// kv_len[s] - q_len[s] + i and attends to keys 0..that position, read through the
// sequence's block table.  Reference op: `AttnPrefill(Gqa)` (crates/kernels/src/op/kind.rs;
// f32 reference crates/kernels/src/reference/attention.rs).
//
// B200 mapping: CTA = 4 warps = 64 query rows of one head; K/V tiles of 64 keys (four
// 16-token pages) stream through a two-stage cp.async double buffer with an XOR swizzle on
// 16-byte chunks (conflict-free ldmatrix).  S = Q K^T (ldmatrix of K rows), P stays in
// registers as the A operand of O += P V (ldmatrix.trans of V rows), f32 statistics with
// exp2.  Tiles strictly above the causal diagonal are skipped; the diagonal tile is masked.
#include "common.cuh"

namespace syn {

constexpr int AP_D = 128;
constexpr int AP_BM = 64;   // query rows per CTA
constexpr int AP_BN = 64;   // keys per tile
constexpr int AP_TILE_BYTES = AP_BN * AP_D * 2;  // 16 KB

struct AttnPrefillArgs {
  const __nv_bfloat16* q;       // [Tq, Hq, D]
  const __nv_bfloat16* kc;      // [nblocks, Hkv, 16, D]
  const __nv_bfloat16* vc;
  const int32_t* block_tables;  // [nseq, max_blocks]
  const int32_t* cu_q;          // [nseq + 1] query row offsets
  const int32_t* kv_lens;       // [nseq] context length including the new rows
  __nv_bfloat16* out;           // [Tq, Hq, D]
  int Hq, Hkv, max_blocks;
  float scale_log2;
};

__device__ __forceinline__ uint32_t ap_swz(int r, int c) { return (uint32_t)(r * 256 + ((c ^ (r & 7)) << 4)); }

__device__ __forceinline__ void ap_cp16(uint32_t s, const void* g) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(s), "l"(g));
}

__global__ void __launch_bounds__(128) attn_prefill_kernel(AttnPrefillArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int s = blockIdx.z, h = blockIdx.y;
  const int q0 = a.cu_q[s], q_len = a.cu_q[s + 1] - q0;
  const int i0 = blockIdx.x * AP_BM;
  if (i0 >= q_len) return;
  const int kv_len = a.kv_lens[s];
  const int pos0 = kv_len - q_len;  // absolute position of query row 0
  const int hk = h / (a.Hq / a.Hkv);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int g = lane >> 2, t = lane & 3;
  uint8_t* sQ = smem;                              // 64 rows x 256 B, swizzled
  uint8_t* sK = smem + AP_TILE_BYTES;              // [2][64 x 256 B]
  uint8_t* sV = sK + 2 * AP_TILE_BYTES;            // [2][64 x 256 B]
  const uint32_t uQ = (uint32_t)__cvta_generic_to_shared(sQ);
  const uint32_t uK = (uint32_t)__cvta_generic_to_shared(sK);
  const uint32_t uV = (uint32_t)__cvta_generic_to_shared(sV);
  const int32_t* bt = a.block_tables + (int64_t)s * a.max_blocks;

  // ---- Q tile (rows past q_len repeat the last row; they are never stored) ----
  for (int idx = threadIdx.x; idx < AP_BM * 16; idx += 128) {
    const int r = idx >> 4, c = idx & 15;
    const int row = q0 + min(i0 + r, q_len - 1);
    ap_cp16(uQ + ap_swz(r, c), a.q + ((int64_t)row * a.Hq + h) * AP_D + c * 8);
  }
  asm volatile("cp.async.commit_group;\n" ::);

  const int p_last = pos0 + min(i0 + AP_BM, q_len) - 1;  // last query position of the CTA
  const int n_tiles = p_last / AP_BN + 1;

  auto load_kv = [&](int tile, int stage) {
    for (int idx = threadIdx.x; idx < AP_BN * 16; idx += 128) {
      const int r = idx >> 4, c = idx & 15;
      const int key = min(tile * AP_BN + r, kv_len - 1);
      const int page = bt[key >> 4];
      const int64_t off = (((int64_t)page * a.Hkv + hk) * 16 + (key & 15)) * AP_D + c * 8;
      ap_cp16(uK + stage * AP_TILE_BYTES + ap_swz(r, c), a.kc + off);
      ap_cp16(uV + stage * AP_TILE_BYTES + ap_swz(r, c), a.vc + off);
    }
    asm volatile("cp.async.commit_group;\n" ::);
  };
  load_kv(0, 0);

  // Q fragments of this warp's 16 rows (A operand, 8 k16 steps over D = 128)
  asm volatile("cp.async.wait_group 1;\n" ::);
  __syncthreads();
  uint32_t qf[8][4];
#pragma unroll
  for (int kk = 0; kk < 8; ++kk) {
    // matrices: (rows 0-7, d 0-7), (rows 8-15, d 0-7), (rows 0-7, d 8-15), (rows 8-15, d 8-15)
    const int r = warp * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
    const int c = kk * 2 + (lane >> 4);
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
                 : "=r"(qf[kk][0]), "=r"(qf[kk][1]), "=r"(qf[kk][2]), "=r"(qf[kk][3])
                 : "r"(uQ + ap_swz(r, c)));
  }

  float o[16][4];
#pragma unroll
  for (int n = 0; n < 16; ++n)
#pragma unroll
    for (int i = 0; i < 4; ++i) o[n][i] = 0.f;
  float m_run[2] = {-INFINITY, -INFINITY}, l_run[2] = {0.f, 0.f};
  const int prow[2] = {pos0 + i0 + warp * 16 + g, pos0 + i0 + warp * 16 + g + 8};

  for (int tile = 0; tile < n_tiles; ++tile) {
    const int st = tile & 1;
    if (tile + 1 < n_tiles) {
      load_kv(tile + 1, st ^ 1);
      asm volatile("cp.async.wait_group 1;\n" ::);
    } else {
      asm volatile("cp.async.wait_group 0;\n" ::);
    }
    __syncthreads();
    // ---- S = Q K^T : 16 rows x 64 keys per warp ----
    float sc[8][4];
#pragma unroll
    for (int n = 0; n < 8; ++n)
#pragma unroll
      for (int i = 0; i < 4; ++i) sc[n][i] = 0.f;
#pragma unroll
    for (int n = 0; n < 8; ++n) {
#pragma unroll
      for (int k2 = 0; k2 < 4; ++k2) {
        // matrices: keys n*8..+7 x d chunks (k2*4 + m), m = 0..3 -> b0,b1 of k-steps 2k2, 2k2+1
        uint32_t b[4];
        const int r = n * 8 + (lane & 7);
        const int c = k2 * 4 + (lane >> 3);
        asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
                     : "=r"(b[0]), "=r"(b[1]), "=r"(b[2]), "=r"(b[3])
                     : "r"(uK + st * AP_TILE_BYTES + ap_swz(r, c)));
        mma_bf16_16816(sc[n], qf[2 * k2], b, sc[n]);
        mma_bf16_16816(sc[n], qf[2 * k2 + 1], b + 2, sc[n]);
      }
    }
    // ---- causal / length mask and online softmax ----
    const int key0 = tile * AP_BN;
    const bool edge = key0 + AP_BN - 1 > pos0 + i0 + warp * 16 || key0 + AP_BN > kv_len;
    float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int n = 0; n < 8; ++n) {
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        float v = sc[n][i] * a.scale_log2;
        if (edge) {
          const int key = key0 + n * 8 + 2 * t + (i & 1);
          if (key > prow[i >> 1] || key >= kv_len) v = -INFINITY;
        }
        sc[n][i] = v;
        mx[i >> 1] = fmaxf(mx[i >> 1], v);
      }
    }
    float corr[2];
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 1));
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 2));
      const float m_new = fmaxf(m_run[r], mx[r]);
      corr[r] = exp2f(m_run[r] - m_new);  // 0 on the first tile (m_run = -inf)
      m_run[r] = m_new;
    }
    float rs[2] = {0.f, 0.f};
    uint32_t pf[4][4];  // P as A fragments (4 k16 steps over the 64 keys)
#pragma unroll
    for (int n = 0; n < 8; ++n) {
      const float p0 = exp2f(sc[n][0] - m_run[0]), p1 = exp2f(sc[n][1] - m_run[0]);
      const float p2 = exp2f(sc[n][2] - m_run[1]), p3 = exp2f(sc[n][3] - m_run[1]);
      rs[0] += p0 + p1;
      rs[1] += p2 + p3;
      const int kk = n >> 1, hi = n & 1;
      pf[kk][hi * 2 + 0] = pack_bf16x2(p0, p1);
      pf[kk][hi * 2 + 1] = pack_bf16x2(p2, p3);
    }
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      rs[r] += __shfl_xor_sync(0xffffffffu, rs[r], 1);
      rs[r] += __shfl_xor_sync(0xffffffffu, rs[r], 2);
      l_run[r] = l_run[r] * corr[r] + rs[r];
    }
#pragma unroll
    for (int n = 0; n < 16; ++n) {
      o[n][0] *= corr[0];
      o[n][1] *= corr[0];
      o[n][2] *= corr[1];
      o[n][3] *= corr[1];
    }
    // ---- O += P V ----
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
#pragma unroll
      for (int n2 = 0; n2 < 8; ++n2) {
        // matrices (trans): keys kk*16 + 0..7 / 8..15  x  d chunk 2*n2 / 2*n2+1
        uint32_t b[4];
        const int r = kk * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
        const int c = n2 * 2 + (lane >> 4);
        asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
                     : "=r"(b[0]), "=r"(b[1]), "=r"(b[2]), "=r"(b[3])
                     : "r"(uV + st * AP_TILE_BYTES + ap_swz(r, c)));
        // a-fragment order of pf: {row g k lo, row g+8 k lo, row g k hi, row g+8 k hi}
        const uint32_t af[4] = {pf[kk][0], pf[kk][1], pf[kk][2], pf[kk][3]};
        mma_bf16_16816(o[2 * n2], af, b, o[2 * n2]);
        mma_bf16_16816(o[2 * n2 + 1], af, b + 2, o[2 * n2 + 1]);
      }
    }
    __syncthreads();  // the stage is refilled two tiles later
  }
  // ---- epilogue ----
  const float inv[2] = {1.f / l_run[0], 1.f / l_run[1]};
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int i = i0 + warp * 16 + g + 8 * r;
    if (i >= q_len) continue;
    __nv_bfloat16* orow = a.out + ((int64_t)(q0 + i) * a.Hq + h) * AP_D;
#pragma unroll
    for (int n = 0; n < 16; ++n)
      *reinterpret_cast<uint32_t*>(orow + n * 8 + 2 * t) = pack_bf16x2(o[n][2 * r] * inv[r], o[n][2 * r + 1] * inv[r]);
  }
}

cudaError_t launch_attn_prefill(const void* q, const void* kc, const void* vc, const int32_t* block_tables,
                                const int32_t* cu_q, const int32_t* kv_lens, void* out, int nseq, int max_q_len,
                                int Hq, int Hkv, int D, int max_blocks, float scale, cudaStream_t s) {
  if (D != AP_D || Hq % Hkv || nseq <= 0 || max_q_len <= 0) return cudaErrorInvalidValue;
  AttnPrefillArgs a{reinterpret_cast<const __nv_bfloat16*>(q), reinterpret_cast<const __nv_bfloat16*>(kc),
                    reinterpret_cast<const __nv_bfloat16*>(vc), block_tables, cu_q, kv_lens,
                    reinterpret_cast<__nv_bfloat16*>(out), Hq, Hkv, max_blocks, scale * 1.4426950408889634f};
  constexpr int smem = 5 * AP_TILE_BYTES;  // Q + 2 x (K, V)
  static bool set = false;
  if (!set) {
    cudaError_t e = cudaFuncSetAttribute(attn_prefill_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    set = true;
  }
  dim3 grid((unsigned)((max_q_len + AP_BM - 1) / AP_BM), (unsigned)Hq, (unsigned)nseq);
  attn_prefill_kernel<<<grid, 128, smem, s>>>(a);
  return cudaGetLastError();
}

}  // namespace syn
