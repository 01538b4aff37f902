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
constexpr int TOPK_MAX_T = 256;

// Warp-per-token routing: lane l holds experts [l*EPL, l*EPL + EPL) (one or more float4
// loads of the logits row).  Selection is k rounds of a warp argmax over the not-yet-taken
// experts, ties to the lower expert index, carrying the routing score of the winner.  Lane j
// keeps choice j (my_id, my_w); wsum is the sum of the k chosen scores (same in every lane).
template <int EPL>
__device__ __forceinline__ void route_token(const TopkArgs& a, const float* lg, bool with_bias, int& my_id,
                                            float& my_w, float& wsum) {
  const int lane = threadIdx.x & 31;
  const int e0 = lane * EPL;
  float score[EPL], sel[EPL];
#pragma unroll
  for (int i = 0; i < EPL; i += 4) {
    float4 v = make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
    if (e0 + i < a.E) v = *reinterpret_cast<const float4*>(lg + e0 + i);
    score[i] = v.x; score[i + 1] = v.y; score[i + 2] = v.z; score[i + 3] = v.w;
  }
  if (a.scoring == 0) {
    float mx = -INFINITY;
#pragma unroll
    for (int i = 0; i < EPL; ++i) mx = fmaxf(mx, score[i]);
    mx = warp_max(mx);
    float sum = 0.f;
#pragma unroll
    for (int i = 0; i < EPL; ++i) {
      score[i] = e0 + i < a.E ? __expf(score[i] - mx) : 0.f;
      sum += score[i];
    }
    const float inv = 1.f / warp_sum(sum);
#pragma unroll
    for (int i = 0; i < EPL; ++i) {
      score[i] *= inv;
      sel[i] = e0 + i < a.E ? score[i] : -INFINITY;
    }
  } else {
#pragma unroll
    for (int i = 0; i < EPL; ++i) {
      const int e = e0 + i;
      score[i] = e < a.E ? 1.f / (1.f + __expf(-score[i])) : 0.f;
      sel[i] = e < a.E ? score[i] + (with_bias && a.bias ? a.bias[e] : 0.f) : -INFINITY;
    }
  }
  if (a.n_groups > 1) {
    // group score: sum of the top two (sigmoid) or the max (softmax) inside each group
    const int gsz = a.E / a.n_groups;
    float gscore = -INFINITY;  // lane g < n_groups holds group g's score
    for (int grp = 0; grp < a.n_groups; ++grp) {
      float b1 = -INFINITY, b2 = -INFINITY;
#pragma unroll
      for (int i = 0; i < EPL; ++i) {
        if ((e0 + i) / gsz == grp && e0 + i < a.E) {
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
    uint32_t keep = 0;  // top groups, ties to the lower group index
    for (int j = 0; j < a.topk_groups; ++j) {
      float best = ((keep >> lane) & 1u) || lane >= a.n_groups ? -INFINITY : gscore;
      int bi = ((keep >> lane) & 1u) || lane >= a.n_groups ? 0x7fffffff : lane;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float ob = __shfl_xor_sync(0xffffffffu, best, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (ob > best || (ob == best && oi < bi)) { best = ob; bi = oi; }
      }
      keep |= 1u << bi;
    }
#pragma unroll
    for (int i = 0; i < EPL; ++i)
      if (e0 + i < a.E && !((keep >> ((e0 + i) / gsz)) & 1u)) sel[i] = -INFINITY;
  }
  uint32_t taken = 0;
  my_id = -1;
  my_w = 0.f;
  wsum = 0.f;
  for (int j = 0; j < a.k; ++j) {
    float best = -INFINITY, bw = 0.f;
    int bi = 0x7fffffff;
#pragma unroll
    for (int i = 0; i < EPL; ++i) {
      // strictly greater keeps the lower index among equal values inside a lane
      if (!((taken >> i) & 1u) && e0 + i < a.E && (sel[i] > best || bi == 0x7fffffff)) {
        best = sel[i]; bi = e0 + i; bw = score[i];
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ob = __shfl_xor_sync(0xffffffffu, best, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      const float ow = __shfl_xor_sync(0xffffffffu, bw, o);
      if (ob > best || (ob == best && oi < bi)) { best = ob; bi = oi; bw = ow; }
    }
    if (lane == j) { my_id = bi; my_w = bw; }
    wsum += bw;
    if (bi / EPL == lane) taken |= 1u << (bi - e0);
  }
}

// Multi-CTA routing: each 4-warp CTA routes 4 tokens (warp per token) and marks its choices
// in a global token bitmask per expert; the last CTA to finish (arrival counter) builds the
// CSR from the masks, then clears the masks and the counter for the next call.
template <int EPL>
__global__ void __launch_bounds__(128) moe_topk_kernel(TopkArgs a) {
  __shared__ uint32_t s_mask[TOPK_MAX_E * (TOPK_MAX_T / 32)];
  __shared__ int s_ids[TOPK_MAX_T * TOPK_MAX_K];
  __shared__ int s_off[TOPK_MAX_E];
  __shared__ uint32_t s_valid[TOPK_MAX_T / 32];  // rows that count toward the usage statistics
  __shared__ int s_last;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int TW = (a.T + 31) >> 5;
  uint32_t* gmask = a.ws;                                  // [E][TW] token bits
  uint32_t* gpred = a.ws + TOPK_MAX_E * (TOPK_MAX_T / 32);  // [E/32] predicted-expert bits
  unsigned* gctr = a.ws + TOPK_MAX_E * (TOPK_MAX_T / 32) + TOPK_MAX_E / 32;
  const int t = blockIdx.x * 4 + warp;
  if (t < a.T) {
    int id;
    float w, wsum;
    route_token<EPL>(a, a.logits + (int64_t)t * a.E_rows, true, id, w, wsum);
    if (lane < a.k) {  // lane j publishes choice j
      a.topk_ids[t * a.k + lane] = id;
      a.topk_w[t * a.k + lane] = a.norm ? w / wsum * a.scaling : w * a.scaling;
      atomicOr(&gmask[id * TW + (t >> 5)], 1u << (t & 31));
    }
    if (a.pred) {
      route_token<EPL>(a, a.logits + (int64_t)t * a.E_rows + a.E, false, id, w, wsum);
      if (lane < a.k) atomicOr(&gpred[id >> 5], 1u << (id & 31));
    }
  }
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) s_last = atomicAdd(gctr, 1u) == gridDim.x - 1;
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  // ---- last CTA: CSR over experts ----
  for (int i = threadIdx.x; i < a.E * TW; i += blockDim.x) {
    s_mask[i] = __ldcg(gmask + i);
    gmask[i] = 0u;
  }
  for (int i = threadIdx.x; i < a.T * a.k; i += blockDim.x) s_ids[i] = __ldcg(a.topk_ids + i);
  if (a.counts)
    for (int q = threadIdx.x; q < TW; q += blockDim.x) {
      uint32_t v = 0u;
      for (int b = 0; b < 32; ++b) {
        const int tt = q * 32 + b;
        if (tt < a.T && (!a.count_rows || a.count_rows[tt] >= 0)) v |= 1u << b;
      }
      s_valid[q] = v;
    }
  if (a.pred_mask)
    for (int e = threadIdx.x; e < a.E; e += blockDim.x)
      a.pred_mask[e] = a.pred ? (int)((__ldcg(gpred + (e >> 5)) >> (e & 31)) & 1u) : 0;
  __syncthreads();
  for (int i = threadIdx.x; i < (a.E + 31) / 32; i += blockDim.x) gpred[i] = 0u;
  if (threadIdx.x == 0) *gctr = 0u;
  if (warp == 0) {  // exclusive scan of the per-expert counts
    constexpr int PER = TOPK_MAX_E / 32;
    int c[PER];
    int run = 0;
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      const int e = lane * PER + i;
      int n = 0;
      if (e < a.E)
        for (int q = 0; q < TW; ++q) n += __popc(s_mask[e * TW + q]);
      c[i] = run;
      run += n;
    }
    int incl = run;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int v = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += v;
    }
    const int base = incl - run;
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      const int e = lane * PER + i;
      if (e < a.E) {
        s_off[e] = base + c[i];
        a.tok_off[e] = base + c[i];
      }
    }
    if (lane == 31) a.tok_off[a.E] = incl;
    if (a.counts) {  // usage statistics for the expert cache (live rows only)
#pragma unroll
      for (int i = 0; i < PER; ++i) {
        const int e = lane * PER + i;
        if (e < a.E) {
          int n = 0;
          for (int q = 0; q < TW; ++q) n += __popc(s_mask[e * TW + q] & s_valid[q]);
          a.counts[e] += n;
        }
      }
    }
  }
  __syncthreads();
  // pair position = offset[e] + number of earlier tokens that chose e (deterministic)
  for (int idx = threadIdx.x; idx < a.T * a.k; idx += blockDim.x) {
    const int tt = idx / a.k;
    const int e = s_ids[idx];
    int rank = __popc(s_mask[e * TW + (tt >> 5)] & ((1u << (tt & 31)) - 1u));
    for (int q = 0; q < (tt >> 5); ++q) rank += __popc(s_mask[e * TW + q]);
    const int p = s_off[e] + rank;
    a.tok_idx[p] = tt;
    a.pair_w[p] = __ldcg(a.topk_w + idx);
    int slot = 0;  // choice slot in ascending expert order
    for (int j2 = 0; j2 < a.k; ++j2) slot += (s_ids[tt * a.k + j2] < e);
    a.pair_of[tt * a.k + slot] = p;
  }
}

// ---- routing of large token counts (prefill): two launches ----
// A: warp per token; choices go to topk_ids/topk_w, a token bitmask per expert and a count.
template <int EPL>
__global__ void __launch_bounds__(128) moe_route_tokens_kernel(TopkArgs a) {
  const int lane = threadIdx.x & 31;
  const int t = blockIdx.x * 4 + (threadIdx.x >> 5);
  if (t >= a.T) return;
  const int TW = (a.T + 31) >> 5;
  uint32_t* mask = a.ws;
  uint32_t* cnt = a.ws + (size_t)a.E * TW;
  int id;
  float w, wsum;
  route_token<EPL>(a, a.logits + (int64_t)t * a.E_rows, true, id, w, wsum);
  if (lane < a.k) {
    a.topk_ids[t * a.k + lane] = id;
    a.topk_w[t * a.k + lane] = a.norm ? w / wsum * a.scaling : w * a.scaling;
    atomicOr(&mask[(size_t)id * TW + (t >> 5)], 1u << (t & 31));
    atomicAdd(&cnt[id], 1u);
  }
}

// B: CTA per expert.  Offset = sum of the counts of lower experts; the expert's pairs are
// placed in token order by a block scan of the popcounts of its mask words.
__global__ void __launch_bounds__(256) moe_csr_kernel(TopkArgs a) {
  __shared__ int s_red[8];
  __shared__ int s_base;
  const int e = blockIdx.x;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int TW = (a.T + 31) >> 5;
  const uint32_t* mask = a.ws + (size_t)e * TW;
  const uint32_t* cnt = a.ws + (size_t)a.E * TW;
  int part = 0;
  for (int i = threadIdx.x; i < e; i += blockDim.x) part += (int)cnt[i];
  part = __reduce_add_sync(0xffffffffu, part);
  if (lane == 0) s_red[warp] = part;
  __syncthreads();
  if (threadIdx.x == 0) {
    int off = 0;
    for (int i = 0; i < 8; ++i) off += s_red[i];
    s_base = off;
    a.tok_off[e] = off;
    if (e == a.E - 1) a.tok_off[a.E] = off + (int)cnt[e];
    if (a.counts) a.counts[e] += (int)cnt[e];
  }
  __syncthreads();
  int base = s_base;
  for (int w0 = 0; w0 < TW; w0 += blockDim.x) {
    const int wi = w0 + threadIdx.x;
    uint32_t word = wi < TW ? mask[wi] : 0u;
    const int c = __popc(word);
    int incl = c;  // block-wide inclusive scan of the popcounts
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int v = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += v;
    }
    __syncthreads();
    if (lane == 31) s_red[warp] = incl;
    __syncthreads();
    int wpre = 0, total = 0;
    for (int i = 0; i < 8; ++i) {
      if (i < warp) wpre += s_red[i];
      total += s_red[i];
    }
    int p = base + wpre + incl - c;
    while (word) {
      const int bit = __ffs(word) - 1;
      word &= word - 1u;
      const int t = wi * 32 + bit;
      int j = 0, slot = 0;
      for (int j2 = 0; j2 < a.k; ++j2) {
        const int id = a.topk_ids[t * a.k + j2];
        if (id == e) j = j2;
        slot += id < e;
      }
      a.tok_idx[p] = t;
      a.pair_w[p] = a.topk_w[t * a.k + j];
      a.pair_of[t * a.k + slot] = p;
      ++p;
    }
    base += total;
  }
}

cudaError_t launch_moe_route_large(const TopkArgs& a, cudaStream_t s) {
  if (a.T == 0) return cudaSuccess;
  if (a.E > TOPK_MAX_E || a.k > TOPK_MAX_K || a.n_groups > 32 || a.E % 4 || a.E_rows % 4 || a.pred || !a.ws)
    return cudaErrorInvalidValue;
  const unsigned grid = (unsigned)((a.T + 3) / 4);
  if (a.E <= 128) moe_route_tokens_kernel<4><<<grid, 128, 0, s>>>(a);
  else if (a.E <= 256) moe_route_tokens_kernel<8><<<grid, 128, 0, s>>>(a);
  else moe_route_tokens_kernel<16><<<grid, 128, 0, s>>>(a);
  cudaError_t err = cudaGetLastError();
  if (err != cudaSuccess) return err;
  moe_csr_kernel<<<a.E, 256, 0, s>>>(a);
  return cudaGetLastError();
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
  if (a.T > TOPK_MAX_T || a.E > TOPK_MAX_E || a.k > TOPK_MAX_K || a.k > 32 || a.n_groups > 32 || a.E % 4 ||
      a.E_rows % 4)
    return cudaErrorInvalidValue;
  if (!a.ws) return cudaErrorInvalidValue;
  const unsigned grid = (unsigned)((a.T + 3) / 4);
  if (a.E <= 128) moe_topk_kernel<4><<<grid, 128, 0, s>>>(a);
  else if (a.E <= 256) moe_topk_kernel<8><<<grid, 128, 0, s>>>(a);
  else moe_topk_kernel<16><<<grid, 128, 0, s>>>(a);
  return cudaGetLastError();
}

}  // namespace syn
