// Normalisation, RoPE and KV-cache writes.
//
//  * rmsnorm: y = x * rsqrt(mean(x^2) + eps) * w, sum of squares in f32 in a fixed order
//    (reference: crates/kernels/src/reference/norm.rs:63).
//  * moe_combine_rmsnorm: x += sum of a token's expert outputs in ascending expert order
//    (reference rule: plan/rfcs/RFC-0040-kernel-providers-and-backends.md:419), then the
//    next layer's input norm, in one pass over the row.
//  * qk_rope_kv_write: per-head RMSNorm of q and k (Qwen3 QK-norm), rotate-half RoPE from
//    an f32 cos/sin table, q to a contiguous buffer and k/v into 16-token pages; the fused
//    RmsNorm + Rope + KvWrite of the reference's design (RFC-0040 `KvWrite`, rope fused).
#include <algorithm>

#include "common.cuh"

namespace syn {

// One CTA per row.  x: f32 or bf16 [T, H]; out bf16 [T, H].
template <typename TIn>
__global__ void rmsnorm_kernel(const TIn* __restrict__ x, const float* __restrict__ w, __nv_bfloat16* __restrict__ y,
                               int H, float eps) {
  __shared__ float red[32];
  const int64_t row = blockIdx.x;
  const TIn* xr = x + row * H;
  float ss = 0.f;
  for (int i = threadIdx.x; i < H; i += blockDim.x) {
    const float v = (float)xr[i];
    ss += v * v;
  }
  ss = block_sum(ss, red);
  const float r = rsqrtf(ss / (float)H + eps);
  for (int i = threadIdx.x; i < H; i += blockDim.x) y[row * H + i] = f2bf((float)xr[i] * r * w[i]);
}

cudaError_t launch_rmsnorm(const void* x, bool x_bf16, const float* w, void* y, int T, int H, float eps,
                           cudaStream_t s) {
  if (T == 0) return cudaSuccess;
  const int threads = std::min(1024, std::max(128, ((H / 4 + 31) / 32) * 32));
  if (x_bf16)
    rmsnorm_kernel<__nv_bfloat16><<<T, threads, 0, s>>>(reinterpret_cast<const __nv_bfloat16*>(x), w,
                                                      reinterpret_cast<__nv_bfloat16*>(y), H, eps);
  else
    rmsnorm_kernel<float><<<T, threads, 0, s>>>(reinterpret_cast<const float*>(x), w,
                                             reinterpret_cast<__nv_bfloat16*>(y), H, eps);
  return cudaGetLastError();
}

// x[t] += sum_j yp[pair_of[t][j]] (pair_of sorted by expert), then y = rmsnorm(x) * w.
// If `shared` is given it is added first (shared-expert output, f32 [T, H]).  One CTA of
// H/4 threads per token, float4 accesses: every thread keeps top_k row loads in flight.
// KT > 0: top_k == KT known at compile time (the pair rows are read once into registers and
// their KT row loads issued back to back; the same summation order as the generic loop).
template <int KT>
__global__ void moe_combine_rmsnorm_kernel(float* __restrict__ x, const float* __restrict__ yp,
                                           const int32_t* __restrict__ pair_of, int top_k,
                                           const float* __restrict__ shared, const float* __restrict__ w,
                                           __nv_bfloat16* __restrict__ y, int H, float eps) {
  __shared__ float red[32];
  const int64_t t = blockIdx.x;
  float* xr = x + t * H;
  float ss = 0.f;
  const bool vec = (H % 4) == 0;
  if (KT > 0 && vec) {
    const float4* rows[KT > 0 ? KT : 1];
#pragma unroll
    for (int j = 0; j < KT; ++j)
      rows[j] = reinterpret_cast<const float4*>(yp + (int64_t)__ldg(pair_of + t * KT + j) * H);
    for (int i4 = threadIdx.x; i4 < H / 4; i4 += blockDim.x) {
      float4 v[KT > 0 ? KT : 1];
#pragma unroll
      for (int j = 0; j < KT; ++j) v[j] = __ldg(rows[j] + i4);
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int j = 0; j < KT; ++j) {
        acc.x += v[j].x; acc.y += v[j].y; acc.z += v[j].z; acc.w += v[j].w;
      }
      if (shared) {
        const float4 u = reinterpret_cast<const float4*>(shared + t * H)[i4];
        acc.x += u.x; acc.y += u.y; acc.z += u.z; acc.w += u.w;
      }
      float4 xv = reinterpret_cast<float4*>(xr)[i4];
      xv.x += acc.x; xv.y += acc.y; xv.z += acc.z; xv.w += acc.w;
      reinterpret_cast<float4*>(xr)[i4] = xv;
      ss += xv.x * xv.x + xv.y * xv.y + xv.z * xv.z + xv.w * xv.w;
    }
  } else if (vec) {
    for (int i4 = threadIdx.x; i4 < H / 4; i4 += blockDim.x) {
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int j = 0; j < top_k; ++j) {
        const float4 v = __ldg(reinterpret_cast<const float4*>(yp + (int64_t)pair_of[t * top_k + j] * H) + i4);
        acc.x += v.x; acc.y += v.y; acc.z += v.z; acc.w += v.w;
      }
      if (shared) {
        const float4 v = reinterpret_cast<const float4*>(shared + t * H)[i4];
        acc.x += v.x; acc.y += v.y; acc.z += v.z; acc.w += v.w;
      }
      float4 xv = reinterpret_cast<float4*>(xr)[i4];
      xv.x += acc.x; xv.y += acc.y; xv.z += acc.z; xv.w += acc.w;
      reinterpret_cast<float4*>(xr)[i4] = xv;
      ss += xv.x * xv.x + xv.y * xv.y + xv.z * xv.z + xv.w * xv.w;
    }
  } else {
    for (int i = threadIdx.x; i < H; i += blockDim.x) {
      float acc = 0.f;
      for (int j = 0; j < top_k; ++j) acc += yp[(int64_t)pair_of[t * top_k + j] * H + i];
      if (shared) acc += shared[t * H + i];
      const float v = xr[i] + acc;
      xr[i] = v;
      ss += v * v;
    }
  }
  if (w == nullptr) return;
  ss = block_sum(ss, red);
  const float r = rsqrtf(ss / (float)H + eps);
  for (int i = threadIdx.x; i < H; i += blockDim.x) y[t * H + i] = f2bf(xr[i] * r * w[i]);
}

cudaError_t launch_moe_combine_rmsnorm(float* x, const float* yp, const int32_t* pair_of, int top_k,
                                       const float* shared, const float* w, void* y, int T, int H, float eps,
                                       cudaStream_t s) {
  if (T == 0) return cudaSuccess;
  const int threads = H % 4 == 0 ? std::min(1024, std::max(128, ((H / 4 + 31) / 32) * 32)) : 256;
  if (top_k == 8)
    moe_combine_rmsnorm_kernel<8><<<T, threads, 0, s>>>(x, yp, pair_of, top_k, shared, w,
                                                        reinterpret_cast<__nv_bfloat16*>(y), H, eps);
  else
    moe_combine_rmsnorm_kernel<0><<<T, threads, 0, s>>>(x, yp, pair_of, top_k, shared, w,
                                                        reinterpret_cast<__nv_bfloat16*>(y), H, eps);
  return cudaGetLastError();
}

// qkv: bf16 [T, (Hq + 2 Hkv) * D].  One CTA per token, one warp per head (q heads first,
// then k heads, then v heads).  D == 128 or 64 (lane owns D/32 consecutive elements
// from each half for rotate-half pairing).
template <int D>
__global__ void qk_rope_kv_write_kernel(const __nv_bfloat16* __restrict__ qkv, int Hq, int Hkv,
                                        const float* __restrict__ qn, const float* __restrict__ kn, float eps,
                                        const int32_t* __restrict__ pos, const float* __restrict__ cos_t,
                                        const float* __restrict__ sin_t, const int64_t* __restrict__ slot,
                                        __nv_bfloat16* __restrict__ q_out, __nv_bfloat16* __restrict__ k_cache,
                                        __nv_bfloat16* __restrict__ v_cache, int block_size) {
  constexpr int PER = D / 64;  // elements per lane per half (1 or 2: one 2- or 4-byte access)
  const int t = blockIdx.x;
  const int lane = threadIdx.x & 31;
  const int nwarps = blockDim.x >> 5;
  const int nh = Hq + 2 * Hkv;
  const int p = pos[t];
  const int64_t sl = slot[t];
  const int64_t blk = sl / block_size, off = sl % block_size;
  // per-lane constants of the token, loaded once for all its heads: rotation and norm weights
  float cs[PER], sn[PER], wq_lo[PER], wq_hi[PER], wk_lo[PER], wk_hi[PER];
#pragma unroll
  for (int i = 0; i < PER; ++i) {
    const int j = lane * PER + i;
    cs[i] = cos_t[(int64_t)p * (D / 2) + j];
    sn[i] = sin_t[(int64_t)p * (D / 2) + j];
    wq_lo[i] = qn ? qn[j] : 1.f;
    wq_hi[i] = qn ? qn[D / 2 + j] : 1.f;
    wk_lo[i] = kn ? kn[j] : 1.f;
    wk_hi[i] = kn ? kn[D / 2 + j] : 1.f;
  }
  for (int h = threadIdx.x >> 5; h < nh; h += nwarps) {
    const __nv_bfloat16* src = qkv + ((int64_t)t * nh + h) * D;
    float lo[PER], hi[PER];
    if constexpr (PER == 2) {
      const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(src + lane * 2));
      const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(src + D / 2 + lane * 2));
      lo[0] = a.x, lo[1] = a.y, hi[0] = b.x, hi[1] = b.y;
    } else {
      lo[0] = bf2f(src[lane]);
      hi[0] = bf2f(src[D / 2 + lane]);
    }
    const bool is_q = h < Hq, is_k = !is_q && h < Hq + Hkv;
    if (is_q || is_k) {
      if (is_q ? qn != nullptr : kn != nullptr) {
        float ss = 0.f;
#pragma unroll
        for (int i = 0; i < PER; ++i) ss += lo[i] * lo[i] + hi[i] * hi[i];
        ss = warp_sum(ss);
        const float r = rsqrtf(ss / (float)D + eps);
#pragma unroll
        for (int i = 0; i < PER; ++i) {
          lo[i] = lo[i] * r * (is_q ? wq_lo[i] : wk_lo[i]);
          hi[i] = hi[i] * r * (is_q ? wq_hi[i] : wk_hi[i]);
        }
      }
#pragma unroll
      for (int i = 0; i < PER; ++i) {
        const float a = lo[i], b = hi[i];
        lo[i] = a * cs[i] - b * sn[i];
        hi[i] = b * cs[i] + a * sn[i];
      }
    }
    __nv_bfloat16* dst;
    if (is_q) {
      dst = q_out + ((int64_t)t * Hq + h) * D;
    } else {
      const int kh = is_k ? h - Hq : h - Hq - Hkv;
      __nv_bfloat16* cache = is_k ? k_cache : v_cache;
      if (sl < 0) continue;  // padded row: no cache write
      dst = cache + (((blk * Hkv + kh) * block_size) + off) * D;
    }
    if constexpr (PER == 2) {
      *reinterpret_cast<__nv_bfloat162*>(dst + lane * 2) = __floats2bfloat162_rn(lo[0], lo[1]);
      *reinterpret_cast<__nv_bfloat162*>(dst + D / 2 + lane * 2) = __floats2bfloat162_rn(hi[0], hi[1]);
    } else {
      dst[lane] = f2bf(lo[0]);
      dst[D / 2 + lane] = f2bf(hi[0]);
    }
  }
}

cudaError_t launch_qk_rope_kv_write(const void* qkv, int T, int Hq, int Hkv, int D, const float* qn, const float* kn,
                                    float eps, const int32_t* pos, const float* cos_t, const float* sin_t,
                                    const int64_t* slot, void* q_out, void* k_cache, void* v_cache, int block_size,
                                    cudaStream_t s) {
  if (T == 0) return cudaSuccess;
  auto qp = reinterpret_cast<const __nv_bfloat16*>(qkv);
  auto qo = reinterpret_cast<__nv_bfloat16*>(q_out);
  auto kc = reinterpret_cast<__nv_bfloat16*>(k_cache);
  auto vc = reinterpret_cast<__nv_bfloat16*>(v_cache);
  if (D == 128)
    qk_rope_kv_write_kernel<128><<<T, 256, 0, s>>>(qp, Hq, Hkv, qn, kn, eps, pos, cos_t, sin_t, slot, qo, kc, vc,
                                                   block_size);
  else if (D == 64)
    qk_rope_kv_write_kernel<64><<<T, 256, 0, s>>>(qp, Hq, Hkv, qn, kn, eps, pos, cos_t, sin_t, slot, qo, kc, vc,
                                                  block_size);
  else
    return cudaErrorInvalidValue;
  return cudaGetLastError();
}

// Embedding gather: out[t] = table[ids[t]] (bf16 table) as f32 residual.
__global__ void embed_kernel(const __nv_bfloat16* __restrict__ table, const int32_t* __restrict__ ids,
                             float* __restrict__ out, int H) {
  const int64_t t = blockIdx.x;
  const int64_t id = ids[t];
  for (int i = threadIdx.x; i < H; i += blockDim.x) out[t * H + i] = bf2f(table[id * H + i]);
}

cudaError_t launch_embed(const void* table, const int32_t* ids, float* out, int T, int H, cudaStream_t s) {
  if (T == 0) return cudaSuccess;
  embed_kernel<<<T, 256, 0, s>>>(reinterpret_cast<const __nv_bfloat16*>(table), ids, out, H);
  return cudaGetLastError();
}

}  // namespace syn
