// MLA decode around the latent attention kernel (DeepSeek-V3 shape): the projections that the
// absorbed form moves onto the query and the output, and the latent-row write, as three
// kernels instead of a chain of f32 tensor ops.
//   mla_q_absorb:  qcat[t][h] = [ q_nope[t][h] . W_uk[h]  (512) | rope(q_pe[t][h]) (64) ]  (bf16)
//   mla_kv_write:  cache[slot[t]] = [ rmsnorm(c[t]) * w (512) | rope(k_pe[t]) (64) ]        (bf16)
//   mla_o_absorb:  out[t][h * 128 + v] = o_lat[t][h] . W_uv[h][v]                            (bf16)
// W_uk [H, 128, 512] and W_uv [H, 128, 512] are bf16 (one read per call: 16 MB each for 128
// heads), products accumulate in f32.  RoPE is the rotate-half form with cos/sin tables
// [max_pos, 32] in f32.  Reference: the absorbed MLA decode of RFC-0040 :474-491 and the f32
// reference path of syntropy_b200/models/mla.py (mla_qkv / mla_attend), which these kernels
// replace on the GPU decode path.
#include "common.cuh"
#include "syn/launch.h"

namespace syn {

namespace {

constexpr int MA_C = 512, MA_DN = 128, MA_DR = 64, MA_DV = 128, MA_W = MA_C + MA_DR;
constexpr int MA_TCH = 8;  // query rows per pass of the q absorb

// grid (H, C / 128), 128 threads: thread = one latent column c of head h, all rows
__global__ void __launch_bounds__(128) mla_q_absorb_kernel(const __nv_bfloat16* __restrict__ q, int T, int H,
                                                           const __nv_bfloat16* __restrict__ w_uk,
                                                           const float* __restrict__ cos_t,
                                                           const float* __restrict__ sin_t,
                                                           const int32_t* __restrict__ pos,
                                                           __nv_bfloat16* __restrict__ qcat) {
  extern __shared__ float sq[];  // [T][128] q_nope of head h in f32
  const int h = blockIdx.x, c = blockIdx.y * 128 + threadIdx.x;
  const int qstride = H * (MA_DN + MA_DR);
  for (int i = threadIdx.x; i < T * MA_DN; i += 128) {
    const int t = i / MA_DN, d = i % MA_DN;
    sq[i] = bf2f(q[(int64_t)t * qstride + h * (MA_DN + MA_DR) + d]);
  }
  __syncthreads();
  const __nv_bfloat16* w = w_uk + (int64_t)h * MA_DN * MA_C + c;
  for (int t0 = 0; t0 < T; t0 += MA_TCH) {
    float acc[MA_TCH];
#pragma unroll
    for (int i = 0; i < MA_TCH; ++i) acc[i] = 0.f;
#pragma unroll 4
    for (int d = 0; d < MA_DN; ++d) {
      const float wv = bf2f(w[(int64_t)d * MA_C]);
#pragma unroll
      for (int i = 0; i < MA_TCH; ++i)
        if (t0 + i < T) acc[i] = fmaf(sq[(t0 + i) * MA_DN + d], wv, acc[i]);
    }
#pragma unroll
    for (int i = 0; i < MA_TCH; ++i)
      if (t0 + i < T) qcat[((int64_t)(t0 + i) * H + h) * MA_W + c] = f2bf(acc[i]);
  }
  if (blockIdx.y == 0) {  // rope of the head's q_pe: thread (t, j) for the 32 rotation pairs
    for (int i = threadIdx.x; i < T * (MA_DR / 2); i += 128) {
      const int t = i / (MA_DR / 2), j = i % (MA_DR / 2);
      const __nv_bfloat16* qp = q + (int64_t)t * qstride + h * (MA_DN + MA_DR) + MA_DN;
      const float a = bf2f(qp[j]), b = bf2f(qp[j + MA_DR / 2]);
      const int p = pos[t];
      const float cs = cos_t[(int64_t)p * (MA_DR / 2) + j], sn = sin_t[(int64_t)p * (MA_DR / 2) + j];
      __nv_bfloat16* o = qcat + ((int64_t)t * H + h) * MA_W + MA_C;
      o[j] = f2bf(a * cs - b * sn);
      o[j + MA_DR / 2] = f2bf(b * cs + a * sn);
    }
  }
}

// one CTA (128 threads) per row t
__global__ void __launch_bounds__(128) mla_kv_write_kernel(const __nv_bfloat16* __restrict__ kva,
                                                           const float* __restrict__ norm_w, float eps,
                                                           const float* __restrict__ cos_t,
                                                           const float* __restrict__ sin_t,
                                                           const int32_t* __restrict__ pos,
                                                           const int64_t* __restrict__ slot,
                                                           __nv_bfloat16* __restrict__ cache) {
  __shared__ float red[4];
  const int t = blockIdx.x;
  const __nv_bfloat16* row = kva + (int64_t)t * MA_W;
  float v[4], ss = 0.f;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    v[i] = bf2f(row[threadIdx.x + i * 128]);
    ss += v[i] * v[i];
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  const float rstd = rsqrtf((red[0] + red[1] + red[2] + red[3]) / MA_C + eps);
  const int64_t s = slot[t] >= 0 ? slot[t] : 0;  // padding rows write the null page
  __nv_bfloat16* out = cache + (int64_t)s * MA_W;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int c = threadIdx.x + i * 128;
    out[c] = f2bf(v[i] * rstd * norm_w[c]);
  }
  if (threadIdx.x < MA_DR / 2) {
    const int j = threadIdx.x, p = pos[t];
    const float a = bf2f(row[MA_C + j]), b = bf2f(row[MA_C + j + MA_DR / 2]);
    const float cs = cos_t[(int64_t)p * (MA_DR / 2) + j], sn = sin_t[(int64_t)p * (MA_DR / 2) + j];
    out[MA_C + j] = f2bf(a * cs - b * sn);
    out[MA_C + j + MA_DR / 2] = f2bf(b * cs + a * sn);
  }
}

// grid (H, row chunks of 16), 256 threads: warp = 16 output columns v, lane = 16 latent columns
__global__ void __launch_bounds__(256) mla_o_absorb_kernel(const float* __restrict__ o_lat, int T, int H,
                                                           const __nv_bfloat16* __restrict__ w_uv,
                                                           __nv_bfloat16* __restrict__ out) {
  __shared__ __align__(16) float so[16][MA_C];  // 32 KB: o_lat rows of this chunk, head h
  const int h = blockIdx.x, t0 = blockIdx.y * 16;
  const int nt = min(16, T - t0);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int i = threadIdx.x; i < nt * (MA_C / 4); i += 256) {
    const int t = i / (MA_C / 4), c4 = i % (MA_C / 4);
    reinterpret_cast<float4*>(so[t])[c4] =
        reinterpret_cast<const float4*>(o_lat + ((int64_t)(t0 + t) * H + h) * MA_C)[c4];
  }
  __syncthreads();
  for (int vi = 0; vi < 16; ++vi) {
    const int v = warp * 16 + vi;
    const uint4* wp = reinterpret_cast<const uint4*>(w_uv + ((int64_t)h * MA_DV + v) * MA_C + lane * 16);
    const uint4 w0 = __ldg(wp), w1 = __ldg(wp + 1);
    float w[16];
    const uint32_t wu[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const float2 f = unpack_bf16x2(wu[k]);
      w[2 * k] = f.x;
      w[2 * k + 1] = f.y;
    }
    for (int t = 0; t < nt; ++t) {
      const float4* op = reinterpret_cast<const float4*>(so[t] + lane * 16);
      float acc = 0.f;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float4 o = op[k];
        acc = fmaf(o.x, w[4 * k], acc);
        acc = fmaf(o.y, w[4 * k + 1], acc);
        acc = fmaf(o.z, w[4 * k + 2], acc);
        acc = fmaf(o.w, w[4 * k + 3], acc);
      }
#pragma unroll
      for (int off = 16; off; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
      if (lane == 0) out[(int64_t)(t0 + t) * H * MA_DV + h * MA_DV + v] = f2bf(acc);
    }
  }
}

}  // namespace

cudaError_t launch_mla_q_absorb(const void* q, int T, int H, const void* w_uk, const float* cos_t, const float* sin_t,
                                const int32_t* pos, void* qcat, cudaStream_t s) {
  if (T <= 0 || H <= 0) return cudaErrorInvalidValue;
  const size_t smem = (size_t)T * MA_DN * sizeof(float);
  if (smem > 227 * 1024) return cudaErrorInvalidValue;
  if (smem > 48 * 1024) {
    const cudaError_t e =
        cudaFuncSetAttribute(mla_q_absorb_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
  }
  mla_q_absorb_kernel<<<dim3((unsigned)H, MA_C / 128), 128, smem, s>>>(
      reinterpret_cast<const __nv_bfloat16*>(q), T, H, reinterpret_cast<const __nv_bfloat16*>(w_uk), cos_t, sin_t,
      pos, reinterpret_cast<__nv_bfloat16*>(qcat));
  return cudaGetLastError();
}

cudaError_t launch_mla_kv_write(const void* kva, int T, const float* norm_w, float eps, const float* cos_t,
                                const float* sin_t, const int32_t* pos, const int64_t* slot, void* cache,
                                cudaStream_t s) {
  if (T <= 0) return cudaErrorInvalidValue;
  mla_kv_write_kernel<<<(unsigned)T, 128, 0, s>>>(reinterpret_cast<const __nv_bfloat16*>(kva), norm_w, eps, cos_t,
                                                  sin_t, pos, slot, reinterpret_cast<__nv_bfloat16*>(cache));
  return cudaGetLastError();
}

cudaError_t launch_mla_o_absorb(const float* o_lat, int T, int H, const void* w_uv, void* out, cudaStream_t s) {
  if (T <= 0 || H <= 0) return cudaErrorInvalidValue;
  mla_o_absorb_kernel<<<dim3((unsigned)H, (unsigned)((T + 15) / 16)), 256, 0, s>>>(
      o_lat, T, H, reinterpret_cast<const __nv_bfloat16*>(w_uv), reinterpret_cast<__nv_bfloat16*>(out));
  return cudaGetLastError();
}

}  // namespace syn
