// MoE routing for decode-sized batches: router logits, top-k (softmax or sigmoid with
// group-limited selection), renormalisation, and the per-expert CSR lists the grouped
// GEMV consumes.  Reference op: `MoeRoute{Softmax,Sigmoid}` — f32, ties to the lower
// expert index, no atomics in any value path (plan/rfcs/RFC-0042-quantization-and-
// numerical-fidelity.md:222-234; crates/kernels/src/op/kind.rs).
//
// The logits kernel can take the next layer's router rows too (E_pred > 0): their top-k is
// the next-layer prediction that drives expert prefetch (RFC-0023 §9).
#include "common.cuh"

namespace syn {

// logits[t][e] = dot(h[t], W[e]).  One warp per (expert row, group of 8 tokens): the
// warp keeps its slice of the weight row in registers and reuses it for the 8 tokens.
// W: bf16 [E_rows, H]; h: bf16 [T, H]; H % 256 == 0 and H <= 8192.
template <int CH>  // 16-byte chunks per lane = H / 256
__global__ void router_logits_kernel(const __nv_bfloat16* __restrict__ h, const __nv_bfloat16* __restrict__ W,
                                     float* __restrict__ logits, int T, int H, int E_rows) {
  const int lane = threadIdx.x & 31;
  const int gw = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int tg_count = (T + 7) / 8;
  const int e = gw / tg_count, tg = gw % tg_count;
  if (e >= E_rows) return;
  const uint4* wr = reinterpret_cast<const uint4*>(W + (int64_t)e * H);
  float2 wf[CH][4];
#pragma unroll
  for (int i = 0; i < CH; ++i) {
    const uint4 v = __ldg(wr + i * 32 + lane);
    wf[i][0] = unpack_bf16x2(v.x);
    wf[i][1] = unpack_bf16x2(v.y);
    wf[i][2] = unpack_bf16x2(v.z);
    wf[i][3] = unpack_bf16x2(v.w);
  }
  const int t1 = min(T, tg * 8 + 8);
  for (int t = tg * 8; t < t1; ++t) {
    const uint4* hr = reinterpret_cast<const uint4*>(h + (int64_t)t * H);
    float acc = 0.f;
#pragma unroll
    for (int i = 0; i < CH; ++i) {
      const uint4 v = __ldg(hr + i * 32 + lane);
      const uint32_t hh[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 b = unpack_bf16x2(hh[j]);
        acc = fmaf(wf[i][j].x, b.x, acc);
        acc = fmaf(wf[i][j].y, b.y, acc);
      }
    }
    acc = warp_sum(acc);
    if (lane == 0) logits[(int64_t)t * E_rows + e] = acc;
  }
}

constexpr int TOPK_MAX_E = 512;
constexpr int TOPK_MAX_K = 16;

// Select k of E scores held 16 per lane (E <= 512): repeated warp argmax, ties to lower index.
__device__ void warp_topk(const float* sel, int E, int k, int* out_ids) {
  const int lane = threadIdx.x & 31;
  uint32_t taken = 0;  // bit i: lane's element i taken
  for (int j = 0; j < k; ++j) {
    float best = -INFINITY;
    int bi = 0x7fffffff;
    for (int i = 0; i < 16; ++i) {
      const int e = i * 32 + lane;
      if (e < E && !((taken >> i) & 1u)) {
        const float v = sel[i];
        if (v > best || (v == best && e < bi)) { best = v; bi = e; }
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ob = __shfl_xor_sync(0xffffffffu, best, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ob > best || (ob == best && oi < bi)) { best = ob; bi = oi; }
    }
    out_ids[j] = bi;
    if ((bi & 31) == lane) taken |= 1u << (bi >> 5);
  }
}

__global__ void __launch_bounds__(1024) moe_topk_kernel(TopkArgs a) {
  __shared__ int s_ids[256][TOPK_MAX_K];
  __shared__ int s_cnt[TOPK_MAX_E];
  __shared__ int s_pred[TOPK_MAX_E];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  for (int e = threadIdx.x; e < a.E; e += blockDim.x) { s_cnt[e] = 0; s_pred[e] = 0; }
  __syncthreads();
  for (int t = warp; t < a.T; t += nw) {
    for (int pass = 0; pass < (a.pred ? 2 : 1); ++pass) {
      const float* lg = a.logits + (int64_t)t * a.E_rows + pass * a.E;
      float score[16], sel[16];
      float mx = -INFINITY;
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const int e = i * 32 + lane;
        score[i] = e < a.E ? lg[e] : -INFINITY;
        mx = fmaxf(mx, score[i]);
      }
      if (a.scoring == 0) {
        mx = warp_max(mx);
        float sum = 0.f;
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const int e = i * 32 + lane;
          score[i] = e < a.E ? __expf(score[i] - mx) : 0.f;
          sum += score[i];
        }
        sum = warp_sum(sum);
#pragma unroll
        for (int i = 0; i < 16; ++i) { score[i] = score[i] / sum; sel[i] = score[i]; }
      } else {
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const int e = i * 32 + lane;
          score[i] = e < a.E ? 1.f / (1.f + __expf(-score[i])) : 0.f;
          sel[i] = e < a.E ? score[i] + (a.bias ? a.bias[e] : 0.f) : -INFINITY;
        }
      }
      if (a.n_groups > 1) {
        // group score: sum of top-2 (sigmoid) or max (softmax) inside each group
        const int gsz = a.E / a.n_groups;
        float gscore = -INFINITY;  // lane g < n_groups holds group g's score
        for (int grp = 0; grp < a.n_groups; ++grp) {
          float b1 = -INFINITY, b2 = -INFINITY;
          for (int i = 0; i < 16; ++i) {
            const int e = i * 32 + lane;
            if (e < a.E && e / gsz == grp) {
              const float v = sel[i];
              if (v > b1) { b2 = b1; b1 = v; } else if (v > b2) { b2 = v; }
            }
          }
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) {
            const float c1 = __shfl_xor_sync(0xffffffffu, b1, o), c2 = __shfl_xor_sync(0xffffffffu, b2, o);
            float n1, n2;
            if (c1 > b1) { n1 = c1; n2 = fmaxf(b1, c2); } else { n1 = b1; n2 = fmaxf(b2, c1); }
            b1 = n1; b2 = n2;
          }
          const float gs = a.scoring == 1 ? b1 + b2 : b1;
          if (lane == grp) gscore = gs;
        }
        // top groups (ties to lower group index)
        uint32_t keep = 0;
        for (int j = 0; j < a.topk_groups; ++j) {
          float best = (keep >> lane) & 1u ? -INFINITY : gscore;
          int bi = ((keep >> lane) & 1u) || lane >= a.n_groups ? 0x7fffffff : lane;
          if (lane >= a.n_groups) best = -INFINITY;
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) {
            const float ob = __shfl_xor_sync(0xffffffffu, best, o);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (ob > best || (ob == best && oi < bi)) { best = ob; bi = oi; }
          }
          keep |= 1u << bi;
        }
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const int e = i * 32 + lane;
          if (e < a.E && !((keep >> (e / gsz)) & 1u)) sel[i] = -INFINITY;
        }
      }
      int ids[TOPK_MAX_K];
      warp_topk(sel, a.E, a.k, ids);
      if (pass == 1) {
        if (lane == 0)
          for (int j = 0; j < a.k; ++j) s_pred[ids[j]] = 1;  // benign same-value writes
        continue;
      }
      // weights = scores of the chosen experts
      float w[TOPK_MAX_K];
      float wsum = 0.f;
      for (int j = 0; j < a.k; ++j) {
        const int e = ids[j];
        float v = 0.f;
        for (int i = 0; i < 16; ++i)
          if (i * 32 + lane == e) v = score[i];
        v = __shfl_sync(0xffffffffu, v, e & 31);
        w[j] = v;
        wsum += v;
      }
      if (lane == 0) {
        for (int j = 0; j < a.k; ++j) {
          float v = a.norm ? w[j] / wsum : w[j];
          v *= a.scaling;
          a.topk_ids[t * a.k + j] = ids[j];
          a.topk_w[t * a.k + j] = v;
          s_ids[t][j] = ids[j];
        }
        for (int j = 0; j < a.k; ++j) atomicAdd(&s_cnt[ids[j]], 1);  // counts only: order-free
      }
    }
  }
  __syncthreads();
  // exclusive scan over experts (single thread: E <= 512)
  if (threadIdx.x == 0) {
    int acc = 0;
    for (int e = 0; e < a.E; ++e) {
      a.tok_off[e] = acc;
      const int c = s_cnt[e];
      s_cnt[e] = acc;
      acc += c;
    }
    a.tok_off[a.E] = acc;
  }
  for (int e = threadIdx.x; e < a.E; e += blockDim.x)
    if (a.pred_mask) a.pred_mask[e] = a.pred ? s_pred[e] : 0;
  __syncthreads();
  // Pair position = offset[e] + number of earlier tokens that chose e (deterministic).
  for (int idx = threadIdx.x; idx < a.T * a.k; idx += blockDim.x) {
    const int t = idx / a.k, j = idx % a.k;
    const int e = s_ids[t][j];
    int rank = 0;
    for (int t2 = 0; t2 < t; ++t2)
      for (int j2 = 0; j2 < a.k; ++j2) rank += (s_ids[t2][j2] == e);
    const int p = s_cnt[e] + rank;
    a.tok_idx[p] = t;
    a.pair_w[p] = a.topk_w[t * a.k + j];
    // choice slot in ascending expert order
    int slot = 0;
    for (int j2 = 0; j2 < a.k; ++j2) slot += (s_ids[t][j2] < e);
    a.pair_of[t * a.k + slot] = p;
  }
}

cudaError_t launch_router_logits(const void* h, const void* W, float* logits, int T, int H, int E_rows,
                                 cudaStream_t s) {
  if (T == 0) return cudaSuccess;
  if (H % 256 != 0 || H > 8192) return cudaErrorInvalidValue;
  const int warps = 8;
  const long n_warps = (long)E_rows * ((T + 7) / 8);
  const unsigned grid = (unsigned)((n_warps + warps - 1) / warps);
  auto hp = reinterpret_cast<const __nv_bfloat16*>(h);
  auto wp = reinterpret_cast<const __nv_bfloat16*>(W);
  switch (H / 256) {
    case 1: router_logits_kernel<1><<<grid, warps * 32, 0, s>>>(hp, wp, logits, T, H, E_rows); break;
    case 2: router_logits_kernel<2><<<grid, warps * 32, 0, s>>>(hp, wp, logits, T, H, E_rows); break;
    case 4: router_logits_kernel<4><<<grid, warps * 32, 0, s>>>(hp, wp, logits, T, H, E_rows); break;
    case 8: router_logits_kernel<8><<<grid, warps * 32, 0, s>>>(hp, wp, logits, T, H, E_rows); break;
    case 16: router_logits_kernel<16><<<grid, warps * 32, 0, s>>>(hp, wp, logits, T, H, E_rows); break;
    case 28: router_logits_kernel<28><<<grid, warps * 32, 0, s>>>(hp, wp, logits, T, H, E_rows); break;
    case 32: router_logits_kernel<32><<<grid, warps * 32, 0, s>>>(hp, wp, logits, T, H, E_rows); break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

cudaError_t launch_moe_topk(const TopkArgs& a, cudaStream_t s) {
  if (a.T == 0) return cudaSuccess;
  if (a.T > 256 || a.E > TOPK_MAX_E || a.k > TOPK_MAX_K || a.n_groups > 32) return cudaErrorInvalidValue;
  moe_topk_kernel<<<1, 1024, 0, s>>>(a);
  return cudaGetLastError();
}

}  // namespace syn
