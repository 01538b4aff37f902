// MLA decode attention in the absorbed form over the paged latent cache (DeepSeek-V3
// shape: latent C = 512, rope part R = 64, one shared latent row per token for all heads).
//   s[h][j] = q_lat[h] . c_j + q_pe[h] . pe_j        (576-wide rows [c_j | pe_j])
//   o_lat[h] = sum_j softmax_j(s[h]) c_j              (512 wide; W_uv is applied afterwards)
// Reference op: `AttnDecode(Mla)` (crates/kernels/src/op/kind.rs; RFC-0040 :474-491).
//
// B200 mapping: CTA = 4 warps = 16 heads x one KV split; 32-key tiles (two 16-token pages)
// stream through a two-stage cp.async buffer (rows XOR-swizzled on 16-byte chunks).  The
// 4 warps split S = Q K^T by keys (one 8-key MMA n-tile each, 36 k16 steps over the 576-wide
// rows) and share the scores through shared memory; every warp keeps the same online-softmax
// statistics and accumulates its own 128-column quarter of o_lat with P in registers (the A
// operand) and the latent rows as B (ldmatrix.trans).  Splits merge in a second kernel in
// split order (deterministic).
#include "common.cuh"

namespace syn {

constexpr int MLA_C = 512;
constexpr int MLA_R = 64;
constexpr int MLA_W = MLA_C + MLA_R;     // 576 elements per latent row
constexpr int MLA_ROWB = MLA_W * 2;      // 1152 bytes
constexpr int MLA_CH = MLA_ROWB / 16;    // 72 chunks of 16 bytes
constexpr int MLA_BN = 32;               // keys per tile
constexpr int MLA_TILEB = MLA_BN * MLA_ROWB;
constexpr int MLA_SS = 20;  // score row stride (16 heads + pad): bank = 8t + g, conflict-free

struct MlaDecodeArgs {
  const __nv_bfloat16* q;       // [B, H, 576]: [q_lat | q_pe]
  const __nv_bfloat16* cache;   // [blocks, 16, 576]
  const int32_t* block_tables;  // [B, max_blocks]
  const int32_t* ctx_lens;      // [B]
  float* part_o;                // [B, H/16, S, 16, 512]
  float* part_ml;               // [B, H/16, S, 16, 2]
  int H, max_blocks, pages_per_split, n_splits;
  float scale_log2;
};

__device__ __forceinline__ uint32_t mla_swz(int r, int c) {
  return (uint32_t)(r * MLA_ROWB + (((c & ~7) | ((c ^ r) & 7)) << 4));
}

__global__ void __launch_bounds__(128) mla_decode_kernel(MlaDecodeArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int split = blockIdx.x, ht = blockIdx.y, b = blockIdx.z;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int g = lane >> 2, t = lane & 3;
  const int ctx = a.ctx_lens[b];
  const int key_begin = split * a.pages_per_split * 16;
  const int key_end = min(ctx, key_begin + a.pages_per_split * 16);
  const int64_t pbase = (((int64_t)b * (a.H / 16) + ht) * a.n_splits + split) * 16;
  float* po = a.part_o + pbase * MLA_C;
  float* pml = a.part_ml + pbase * 2;
  if (key_begin >= key_end) {  // empty split: contributes nothing to the merge
    for (int i = threadIdx.x; i < 16; i += 128) {
      pml[i * 2] = -INFINITY;
      pml[i * 2 + 1] = 0.f;
    }
    return;
  }
  uint8_t* sQ = smem;                               // 16 rows x 1152 B
  uint8_t* sKV = smem + 16 * MLA_ROWB;              // [2][32 x 1152 B]
  float* sS = reinterpret_cast<float*>(sKV + 2 * MLA_TILEB);  // [32 keys][MLA_SS] (heads; padded)
  const uint32_t uQ = (uint32_t)__cvta_generic_to_shared(sQ);
  const uint32_t uKV = (uint32_t)__cvta_generic_to_shared(sKV);
  const int32_t* bt = a.block_tables + (int64_t)b * a.max_blocks;

  for (int idx = threadIdx.x; idx < 16 * MLA_CH; idx += 128) {
    const int r = idx / MLA_CH, c = idx % MLA_CH;
    const __nv_bfloat16* src = a.q + ((int64_t)b * a.H + ht * 16 + r) * MLA_W + c * 8;
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(uQ + mla_swz(r, c)), "l"(src));
  }
  asm volatile("cp.async.commit_group;\n" ::);
  auto load_tile = [&](int k0, int stage) {
    for (int idx = threadIdx.x; idx < MLA_BN * MLA_CH; idx += 128) {
      const int r = idx / MLA_CH, c = idx % MLA_CH;
      const int key = min(k0 + r, key_end - 1);
      const __nv_bfloat16* src = a.cache + ((int64_t)bt[key >> 4] * 16 + (key & 15)) * MLA_W + c * 8;
      asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(uKV + stage * MLA_TILEB + mla_swz(r, c)),
                   "l"(src));
    }
    asm volatile("cp.async.commit_group;\n" ::);
  };
  const int n_tiles = (key_end - key_begin + MLA_BN - 1) / MLA_BN;
  load_tile(key_begin, 0);

  float o[16][4];
#pragma unroll
  for (int n = 0; n < 16; ++n)
#pragma unroll
    for (int i = 0; i < 4; ++i) o[n][i] = 0.f;
  float m_run[2] = {-INFINITY, -INFINITY}, l_run[2] = {0.f, 0.f};

  for (int tile = 0; tile < n_tiles; ++tile) {
    const int st = tile & 1;
    const int k0 = key_begin + tile * MLA_BN;
    if (tile + 1 < n_tiles) {
      load_tile(k0 + MLA_BN, st ^ 1);
      asm volatile("cp.async.wait_group 1;\n" ::);
    } else {
      asm volatile("cp.async.wait_group 0;\n" ::);
    }
    __syncthreads();
    const uint32_t uT = uKV + st * MLA_TILEB;
    // ---- scores of keys 8w..8w+7 for the 16 heads ----
    {
      float sc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 4
      for (int k2 = 0; k2 < MLA_W / 32; ++k2) {
        uint32_t kb[4];
        asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
                     : "=r"(kb[0]), "=r"(kb[1]), "=r"(kb[2]), "=r"(kb[3])
                     : "r"(uT + mla_swz(warp * 8 + (lane & 7), k2 * 4 + (lane >> 3))));
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          uint32_t qa[4];
          const int r = (lane & 7) + ((lane >> 3) & 1) * 8;
          const int c = (k2 * 2 + h) * 2 + (lane >> 4);
          asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
                       : "=r"(qa[0]), "=r"(qa[1]), "=r"(qa[2]), "=r"(qa[3])
                       : "r"(uQ + mla_swz(r, c)));
          mma_bf16_16816(sc, qa, kb + 2 * h, sc);
        }
      }
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int key = k0 + warp * 8 + 2 * t + (i & 1);
        sS[(warp * 8 + 2 * t + (i & 1)) * MLA_SS + g + 8 * (i >> 1)] =
            key < key_end ? sc[i] * a.scale_log2 : -INFINITY;
      }
    }
    __syncthreads();
    // ---- online softmax (identical in every warp) and P as A fragments ----
    float mx[2] = {-INFINITY, -INFINITY};
    float sv[2][2][4];  // [row half][k-step][value]
#pragma unroll
    for (int r = 0; r < 2; ++r)
#pragma unroll
      for (int kk = 0; kk < 2; ++kk) {
        const float* col = sS + (kk * 16 + 2 * t) * MLA_SS + g + 8 * r;
        sv[r][kk][0] = col[0];
        sv[r][kk][1] = col[MLA_SS];
        sv[r][kk][2] = col[8 * MLA_SS];
        sv[r][kk][3] = col[9 * MLA_SS];
#pragma unroll
        for (int i = 0; i < 4; ++i) mx[r] = fmaxf(mx[r], sv[r][kk][i]);
      }
    float corr[2], rs[2] = {0.f, 0.f};
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 1));
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 2));
      const float m_new = fmaxf(m_run[r], mx[r]);
      corr[r] = exp2f(m_run[r] - m_new);
      m_run[r] = m_new;
    }
    uint32_t pf[2][4];
#pragma unroll
    for (int kk = 0; kk < 2; ++kk) {
      float p[2][4];
#pragma unroll
      for (int r = 0; r < 2; ++r)
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          p[r][i] = exp2f(sv[r][kk][i] - m_run[r]);
          rs[r] += p[r][i];
        }
      pf[kk][0] = pack_bf16x2(p[0][0], p[0][1]);  // row g, keys 2t, 2t+1
      pf[kk][1] = pack_bf16x2(p[1][0], p[1][1]);  // row g+8
      pf[kk][2] = pack_bf16x2(p[0][2], p[0][3]);  // row g, keys 8+2t, 9+2t
      pf[kk][3] = pack_bf16x2(p[1][2], p[1][3]);
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
    // ---- o_lat[:, 128w .. 128w+127] += P V ----
#pragma unroll
    for (int kk = 0; kk < 2; ++kk) {
#pragma unroll
      for (int n2 = 0; n2 < 8; ++n2) {
        uint32_t vb[4];
        const int r = kk * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
        const int c = warp * 16 + n2 * 2 + (lane >> 4);
        asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
                     : "=r"(vb[0]), "=r"(vb[1]), "=r"(vb[2]), "=r"(vb[3])
                     : "r"(uT + mla_swz(r, c)));
        mma_bf16_16816(o[2 * n2], pf[kk], vb, o[2 * n2]);
        mma_bf16_16816(o[2 * n2 + 1], pf[kk], vb + 2, o[2 * n2 + 1]);
      }
    }
    __syncthreads();  // stage and scores are rewritten by the next tile
  }
  // ---- partial (normalised) output and statistics ----
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int row = g + 8 * r;
    const float inv = l_run[r] > 0.f ? 1.f / l_run[r] : 0.f;
#pragma unroll
    for (int n = 0; n < 16; ++n) {
      float2 v = make_float2(o[n][2 * r] * inv, o[n][2 * r + 1] * inv);
      *reinterpret_cast<float2*>(po + row * MLA_C + warp * 128 + n * 8 + 2 * t) = v;
    }
    if (warp == 0 && t == 0) {
      pml[row * 2] = m_run[r];
      pml[row * 2 + 1] = l_run[r];
    }
  }
}

// out[b][h][c] (f32) = sum over splits weighted by exp2(m_s - M) * l_s, normalised.
__global__ void mla_merge_kernel(const float* __restrict__ part_o, const float* __restrict__ part_ml,
                                 float* __restrict__ out, int H, int n_splits) {
  const int b = blockIdx.x, h = blockIdx.y;
  const int ht = h >> 4, row = h & 15;
  const int64_t base = ((int64_t)b * (H / 16) + ht) * n_splits;
  float M = -INFINITY;
  for (int s = 0; s < n_splits; ++s) M = fmaxf(M, part_ml[((base + s) * 16 + row) * 2]);
  for (int c = threadIdx.x; c < MLA_C; c += blockDim.x) {
    float L = 0.f, O = 0.f;
    for (int s = 0; s < n_splits; ++s) {
      const float ms = part_ml[((base + s) * 16 + row) * 2];
      if (ms == -INFINITY) continue;
      const float f = part_ml[((base + s) * 16 + row) * 2 + 1] * exp2f(ms - M);
      L += f;
      O += part_o[((base + s) * 16 + row) * MLA_C + c] * f;
    }
    out[((int64_t)b * H + h) * MLA_C + c] = L > 0.f ? O / L : 0.f;
  }
}

cudaError_t launch_mla_decode(const void* q, const void* cache, const int32_t* block_tables, const int32_t* ctx_lens,
                              float* part_o, float* part_ml, float* out, int B, int H, int max_blocks,
                              int pages_per_split, int n_splits, float scale, cudaStream_t s) {
  if (B == 0) return cudaSuccess;
  if (H % 16 || pages_per_split <= 0) return cudaErrorInvalidValue;
  constexpr int smem = 16 * MLA_ROWB + 2 * MLA_TILEB + MLA_BN * MLA_SS * 4;
  static bool set = false;
  if (!set) {
    cudaError_t e = cudaFuncSetAttribute(mla_decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    set = true;
  }
  MlaDecodeArgs a{reinterpret_cast<const __nv_bfloat16*>(q), reinterpret_cast<const __nv_bfloat16*>(cache),
                  block_tables, ctx_lens, part_o, part_ml, H, max_blocks, pages_per_split, n_splits,
                  scale * 1.4426950408889634f};
  mla_decode_kernel<<<dim3(n_splits, H / 16, B), 128, smem, s>>>(a);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  mla_merge_kernel<<<dim3(B, H), 128, 0, s>>>(part_o, part_ml, out, H, n_splits);
  return cudaGetLastError();
}

}  // namespace syn
