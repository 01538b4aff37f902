// Paged decode attention (GQA): up to 16 query heads sharing one KV head, against a
// paged cache of 16-token pages, split over the context with an exact log-sum-exp merge.
// Reference op: `AttnDecode(Gqa)` + `AttnPartial`/`AttnMerge` (plan/rfcs/RFC-0040-kernel-
// providers-and-backends.md:474-491; crates/kernels/src/op/kind.rs).
//
// B200 mapping (bandwidth-bound on KV bytes):
//  * grid (split, kv_head, token); each CTA streams its pages with cp.async into a
//    per-warp double buffer (XOR-swizzled 16-byte chunks: conflict-free ldmatrix);
//  * the query heads of one KV head form the M=16 side of mma.sync m16n8k16, so one page
//    costs 16 MMAs for S = Q K^T and 16 for O += P V, with P kept in registers;
//  * online softmax in f32 with exp2; warps merge in shared memory in a fixed order;
//    splits merge in a second kernel in split order (deterministic).
#include "common.cuh"

namespace syn {

constexpr int AD_WARPS = 4;
constexpr int AD_D = 128;
constexpr int AD_BS = 16;
constexpr int AD_PAGE_ELEMS = AD_BS * AD_D;  // 2048 bf16 = 4 KB

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
  const uint32_t s = (uint32_t)__cvta_generic_to_shared(smem);
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(s), "l"(gmem));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N)); }

__device__ __forceinline__ void ldmatrix_x4(uint32_t* r, const void* smem) {
  const uint32_t s = (uint32_t)__cvta_generic_to_shared(smem);
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(s));
}
__device__ __forceinline__ void ldmatrix_x4_trans(uint32_t* r, const void* smem) {
  const uint32_t s = (uint32_t)__cvta_generic_to_shared(smem);
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(s));
}

// Byte offset of 16-byte chunk `c` (0..15) of token row `r` in a swizzled 4 KB page.
__device__ __forceinline__ int swz(int r, int c) { return r * 256 + ((c ^ (r & 7)) << 4); }

struct AttnDecodeArgs {
  const __nv_bfloat16* q;      // [T, Hq, D]
  const __nv_bfloat16* kc;     // [nblocks, Hkv, 16, D]
  const __nv_bfloat16* vc;
  const int32_t* block_tables; // [T, max_blocks]
  const int32_t* ctx_lens;     // [T]
  float* part_o;               // [T, Hkv, S, 16, D]
  float* part_ml;              // [T, Hkv, S, 16, 2]
  int Hq, Hkv, max_blocks, pages_per_split, n_splits;
  float scale_log2;            // softmax scale * log2(e)
};

__global__ void __launch_bounds__(AD_WARPS * 32)
attn_decode_kernel(AttnDecodeArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int split = blockIdx.x, kvh = blockIdx.y, t = blockIdx.z;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int g = lane >> 2, tq = lane & 3;
  const int G = a.Hq / a.Hkv;
  const int ctx = a.ctx_lens[t];
  const int n_pages = (ctx + AD_BS - 1) / AD_BS;
  const int p_begin = split * a.pages_per_split;
  const int p_end = min(n_pages, p_begin + a.pages_per_split);

  float* po = a.part_o + ((((int64_t)t * a.Hkv + kvh) * a.n_splits + split) * 16) * AD_D;
  float* pml = a.part_ml + ((((int64_t)t * a.Hkv + kvh) * a.n_splits + split) * 16) * 2;
  if (p_begin >= p_end) {
    // empty split: m = -inf, l = 0
    if (threadIdx.x < 16) {
      pml[threadIdx.x * 2 + 0] = -INFINITY;
      pml[threadIdx.x * 2 + 1] = 0.f;
    }
    return;
  }

  // Q fragments (rows = heads of this KV group; rows >= G are zero).
  uint32_t qf[8][4];
  {
    const __nv_bfloat16* qb = a.q + ((int64_t)t * a.Hq + kvh * G) * AD_D;
#pragma unroll
    for (int ks = 0; ks < 8; ++ks) {
      const int d0 = ks * 16 + 2 * tq;
      qf[ks][0] = g < G ? *reinterpret_cast<const uint32_t*>(qb + g * AD_D + d0) : 0u;
      qf[ks][1] = g + 8 < G ? *reinterpret_cast<const uint32_t*>(qb + (g + 8) * AD_D + d0) : 0u;
      qf[ks][2] = g < G ? *reinterpret_cast<const uint32_t*>(qb + g * AD_D + d0 + 8) : 0u;
      qf[ks][3] = g + 8 < G ? *reinterpret_cast<const uint32_t*>(qb + (g + 8) * AD_D + d0 + 8) : 0u;
    }
  }

  float o[16][4];
#pragma unroll
  for (int i = 0; i < 16; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float m_lo = -INFINITY, m_hi = -INFINITY, l_lo = 0.f, l_hi = 0.f;

  uint8_t* wbuf = smem + warp * (2 * 2 * 4096);  // [stage][K,V][4 KB]
  const int32_t* bt = a.block_tables + (int64_t)t * a.max_blocks;

  auto issue = [&](int page, int stage) {
    const int64_t blk = bt[page];
    const __nv_bfloat16* ks = a.kc + (blk * a.Hkv + kvh) * AD_PAGE_ELEMS;
    const __nv_bfloat16* vs = a.vc + (blk * a.Hkv + kvh) * AD_PAGE_ELEMS;
    uint8_t* kd = wbuf + stage * 8192;
    uint8_t* vd = kd + 4096;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int idx = i * 32 + lane;  // 16-byte chunk index 0..255
      const int r = idx >> 4, c = idx & 15;
      cp_async16(kd + swz(r, c), ks + idx * 8);
      cp_async16(vd + swz(r, c), vs + idx * 8);
    }
    cp_async_commit();
  };

  int page = p_begin + warp;
  int stage = 0;
  if (page < p_end) issue(page, 0);
  for (; page < p_end; page += AD_WARPS) {
    const int next = page + AD_WARPS;
    if (next < p_end) {
      issue(next, stage ^ 1);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncwarp();
    const uint8_t* kd = wbuf + stage * 8192;
    const uint8_t* vd = kd + 4096;

    // S = Q K^T : two n-tiles of 8 tokens
    float s[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
    for (int ks = 0; ks < 8; ++ks) {
      uint32_t b[4];
      const int mi = lane >> 3, r = lane & 7;
      const int tok = (mi >> 1) * 8 + r;
      const int chunk = ks * 2 + (mi & 1);
      ldmatrix_x4(b, kd + swz(tok, chunk));
      mma_bf16_16816(s[0], qf[ks], b, s[0]);
      mma_bf16_16816(s[1], qf[ks], b + 2, s[1]);
    }
    // mask + scale
    const int tok0 = page * AD_BS;
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int tok = tok0 + nt * 8 + 2 * tq + (i & 1);
        s[nt][i] = tok < ctx ? s[nt][i] * a.scale_log2 : -INFINITY;
      }
    }
    float mx_lo = fmaxf(fmaxf(s[0][0], s[0][1]), fmaxf(s[1][0], s[1][1]));
    float mx_hi = fmaxf(fmaxf(s[0][2], s[0][3]), fmaxf(s[1][2], s[1][3]));
    mx_lo = fmaxf(mx_lo, __shfl_xor_sync(0xffffffffu, mx_lo, 1));
    mx_lo = fmaxf(mx_lo, __shfl_xor_sync(0xffffffffu, mx_lo, 2));
    mx_hi = fmaxf(mx_hi, __shfl_xor_sync(0xffffffffu, mx_hi, 1));
    mx_hi = fmaxf(mx_hi, __shfl_xor_sync(0xffffffffu, mx_hi, 2));
    const float mn_lo = fmaxf(m_lo, mx_lo), mn_hi = fmaxf(m_hi, mx_hi);
    const float al_lo = exp2f(m_lo - mn_lo), al_hi = exp2f(m_hi - mn_hi);
    m_lo = mn_lo;
    m_hi = mn_hi;
    float p[2][4];
    float rs_lo = 0.f, rs_hi = 0.f;
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
      p[nt][0] = exp2f(s[nt][0] - mn_lo);
      p[nt][1] = exp2f(s[nt][1] - mn_lo);
      p[nt][2] = exp2f(s[nt][2] - mn_hi);
      p[nt][3] = exp2f(s[nt][3] - mn_hi);
      rs_lo += p[nt][0] + p[nt][1];
      rs_hi += p[nt][2] + p[nt][3];
    }
    rs_lo += __shfl_xor_sync(0xffffffffu, rs_lo, 1);
    rs_lo += __shfl_xor_sync(0xffffffffu, rs_lo, 2);
    rs_hi += __shfl_xor_sync(0xffffffffu, rs_hi, 1);
    rs_hi += __shfl_xor_sync(0xffffffffu, rs_hi, 2);
    l_lo = l_lo * al_lo + rs_lo;
    l_hi = l_hi * al_hi + rs_hi;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      o[i][0] *= al_lo;
      o[i][1] *= al_lo;
      o[i][2] *= al_hi;
      o[i][3] *= al_hi;
    }
    uint32_t pa[4];
    pa[0] = pack_bf16x2(p[0][0], p[0][1]);
    pa[1] = pack_bf16x2(p[0][2], p[0][3]);
    pa[2] = pack_bf16x2(p[1][0], p[1][1]);
    pa[3] = pack_bf16x2(p[1][2], p[1][3]);
    // O += P V : 16 n-tiles of 8 dims, two per ldmatrix.x4.trans
#pragma unroll
    for (int c = 0; c < 16; c += 2) {
      uint32_t b[4];
      const int mi = lane >> 3, r = lane & 7;
      const int tok = (mi & 1) * 8 + r;
      const int chunk = c + (mi >> 1);
      ldmatrix_x4_trans(b, vd + swz(tok, chunk));
      mma_bf16_16816(o[c], pa, b, o[c]);
      mma_bf16_16816(o[c + 1], pa, b + 2, o[c + 1]);
    }
    __syncwarp();
    stage ^= 1;
  }

  // Merge the warps of this CTA in shared memory (fixed order).
  __syncthreads();
  float* so = reinterpret_cast<float*>(smem);            // [warps][16][128]
  float* sml = so + AD_WARPS * 16 * AD_D;                 // [warps][16][2]
#pragma unroll
  for (int nt = 0; nt < 16; ++nt) {
    const int d = nt * 8 + 2 * tq;
    so[(warp * 16 + g) * AD_D + d] = o[nt][0];
    so[(warp * 16 + g) * AD_D + d + 1] = o[nt][1];
    so[(warp * 16 + g + 8) * AD_D + d] = o[nt][2];
    so[(warp * 16 + g + 8) * AD_D + d + 1] = o[nt][3];
  }
  if (tq == 0) {
    sml[(warp * 16 + g) * 2 + 0] = m_lo;
    sml[(warp * 16 + g) * 2 + 1] = l_lo;
    sml[(warp * 16 + g + 8) * 2 + 0] = m_hi;
    sml[(warp * 16 + g + 8) * 2 + 1] = l_hi;
  }
  __syncthreads();
  for (int idx = threadIdx.x; idx < 16 * AD_D; idx += blockDim.x) {
    const int row = idx / AD_D, d = idx % AD_D;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < AD_WARPS; ++w) M = fmaxf(M, sml[(w * 16 + row) * 2]);
    float L = 0.f, O = 0.f;
    if (M != -INFINITY) {
#pragma unroll
      for (int w = 0; w < AD_WARPS; ++w) {
        const float mw = sml[(w * 16 + row) * 2];
        const float f = mw == -INFINITY ? 0.f : exp2f(mw - M);
        L += sml[(w * 16 + row) * 2 + 1] * f;
        O += so[(w * 16 + row) * AD_D + d] * f;
      }
    }
    po[row * AD_D + d] = O;
    if (d == 0) {
      pml[row * 2 + 0] = M;
      pml[row * 2 + 1] = L;
    }
  }
}

// out[t][h][:] = sum_s exp2(m_s - M) o_s / sum_s exp2(m_s - M) l_s
__global__ void attn_merge_kernel(const float* __restrict__ part_o, const float* __restrict__ part_ml,
                                  __nv_bfloat16* __restrict__ out, int Hq, int Hkv, int n_splits) {
  const int t = blockIdx.x;
  const int h = blockIdx.y;
  const int G = Hq / Hkv;
  const int kvh = h / G, row = h % G;
  const int64_t base = ((int64_t)t * Hkv + kvh) * n_splits;
  float M = -INFINITY;
  for (int s = 0; s < n_splits; ++s) M = fmaxf(M, part_ml[((base + s) * 16 + row) * 2]);
  for (int d = threadIdx.x; d < AD_D; d += blockDim.x) {
    float L = 0.f, O = 0.f;
    for (int s = 0; s < n_splits; ++s) {
      const float ms = part_ml[((base + s) * 16 + row) * 2];
      if (ms == -INFINITY) continue;
      const float f = exp2f(ms - M);
      L += part_ml[((base + s) * 16 + row) * 2 + 1] * f;
      O += part_o[((base + s) * 16 + row) * AD_D + d] * f;
    }
    out[((int64_t)t * Hq + h) * AD_D + d] = f2bf(L > 0.f ? O / L : 0.f);
  }
}

cudaError_t launch_attn_decode(const void* q, const void* kc, const void* vc, const int32_t* block_tables,
                               const int32_t* ctx_lens, float* part_o, float* part_ml, void* out, int T, int Hq,
                               int Hkv, int D, int max_blocks, int pages_per_split, int n_splits, float scale,
                               cudaStream_t s) {
  if (T == 0) return cudaSuccess;
  if (D != AD_D || Hq % Hkv != 0 || Hq / Hkv > 16) return cudaErrorInvalidValue;
  static bool attr_set = false;
  const int smem = AD_WARPS * 2 * 2 * 4096;  // 64 KB staging (reused for the merge: 33 KB)
  if (!attr_set) {
    cudaError_t e = cudaFuncSetAttribute(attn_decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    attr_set = true;
  }
  AttnDecodeArgs a;
  a.q = reinterpret_cast<const __nv_bfloat16*>(q);
  a.kc = reinterpret_cast<const __nv_bfloat16*>(kc);
  a.vc = reinterpret_cast<const __nv_bfloat16*>(vc);
  a.block_tables = block_tables;
  a.ctx_lens = ctx_lens;
  a.part_o = part_o;
  a.part_ml = part_ml;
  a.Hq = Hq;
  a.Hkv = Hkv;
  a.max_blocks = max_blocks;
  a.pages_per_split = pages_per_split;
  a.n_splits = n_splits;
  a.scale_log2 = scale * 1.4426950408889634f;
  dim3 grid(n_splits, Hkv, T);
  attn_decode_kernel<<<grid, AD_WARPS * 32, smem, s>>>(a);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  attn_merge_kernel<<<dim3(T, Hq), 128, 0, s>>>(part_o, part_ml, reinterpret_cast<__nv_bfloat16*>(out), Hq, Hkv,
                                                n_splits);
  return cudaGetLastError();
}

}  // namespace syn
