// 4-bit block format on the device: quantise, repack and dequantise.
//
// Quantisation rule (this framework's own; the file format is the Q4_1 block of
// plan/rfcs/RFC-0042-quantization-and-numerical-fidelity.md §2.1):
//   d = fp16((max - min) / 15), m = fp16(min),
//   q = clamp(rint((x - m) / d), 0, 15)   (q = 0 when d == 0),
// so that the rounding of the stored scale and min is seen by q.  The CPU version in
// csrc/cpu/q4_ref.cpp performs the same operations and is the oracle.
#include "common.cuh"
#include "syn/q4.h"

namespace syn {

template <typename T>
__device__ __forceinline__ float ldf(const T* p) { return (float)(*p); }
template <>
__device__ __forceinline__ float ldf<__nv_bfloat16>(const __nv_bfloat16* p) { return __bfloat162float(*p); }

// One thread per 32-element block: (d, m) pair into the tiled scale array and,
// optionally, into the row-block interchange layout.
template <typename T>
__global__ void q4_block_scales_kernel(const T* __restrict__ w, int64_t N, int64_t K,
                                       half2* __restrict__ sm) {
  const int64_t nb = K / SYN_Q4_BLOCK;
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= N * nb) return;
  const int64_t n = i / nb, kb = i % nb;
  const T* p = w + n * K + kb * SYN_Q4_BLOCK;
  float mn = INFINITY, mx = -INFINITY;
#pragma unroll 8
  for (int j = 0; j < SYN_Q4_BLOCK; ++j) {
    const float v = ldf(p + j);
    mn = fminf(mn, v);
    mx = fmaxf(mx, v);
  }
  const __half d = __float2half_rn((mx - mn) / 15.f);
  const __half m = __float2half_rn(mn);
  sm[q4t_scale_index(K, n, kb)] = __halves2half2(d, m);
}

__device__ __forceinline__ uint32_t q4_code(float x, float d, float m) {
  if (d == 0.f) return 0u;
  float q = rintf((x - m) / d);
  q = fminf(fmaxf(q, 0.f), 15.f);
  return (uint32_t)q;
}

// One thread per output word of qw.
template <typename T>
__global__ void q4_pack_tiled_kernel(const T* __restrict__ w, int64_t N, int64_t K,
                                     const half2* __restrict__ sm, uint32_t* __restrict__ qw) {
  const int64_t nwords = N * K / 8;
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= nwords) return;
  const int wsel = (int)(i & 3);
  const int lane = (int)((i >> 2) & 31);
  const int64_t tk = i >> 7;  // tile * (K/64) + kg
  const int64_t kgs = K >> 6;
  const int64_t tile = tk / kgs, kg = tk % kgs;
  const int blk = wsel >> 1, step = wsel & 1;
  const int g = lane >> 2, t = lane & 3;
  uint32_t word = 0;
#pragma unroll
  for (int nib = 0; nib < 8; ++nib) {
    const int reg = nib & 3, odd = nib >> 2;
    const int hi_row = reg & 1, hi_col = reg >> 1;
    const int64_t n = tile * 16 + g + 8 * hi_row;
    const int kk = 2 * t + odd + 8 * hi_col;
    const int64_t k = kg * 64 + blk * 32 + step * 16 + kk;
    const half2 dm = sm[q4t_scale_index(K, n, k / SYN_Q4_BLOCK)];
    const float d = __low2float(dm), m = __high2float(dm);
    word |= q4_code(ldf(w + n * K + k), d, m) << (4 * nib);
  }
  qw[i] = word;
}

// Row-block interchange layout -> tiled.  One thread per qw word.
__global__ void q4_rows_to_tiled_kernel(const uint8_t* __restrict__ rows, int64_t N, int64_t K,
                                        uint32_t* __restrict__ qw, half2* __restrict__ sm) {
  const int64_t nwords = N * K / 8;
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t nb = K / SYN_Q4_BLOCK;
  if (i < N * nb) {  // scale pairs
    const int64_t n = i / nb, kb = i % nb;
    const uint8_t* b = rows + (n * nb + kb) * SYN_Q4_ROW_BLOCK_BYTES;
    half2 dm;
    memcpy(&dm, b, 4);
    sm[q4t_scale_index(K, n, kb)] = dm;
  }
  if (i >= nwords) return;
  const int wsel = (int)(i & 3);
  const int lane = (int)((i >> 2) & 31);
  const int64_t tk = i >> 7;
  const int64_t kgs = K >> 6;
  const int64_t tile = tk / kgs, kg = tk % kgs;
  const int blk = wsel >> 1, step = wsel & 1;
  const int g = lane >> 2, t = lane & 3;
  uint32_t word = 0;
#pragma unroll
  for (int nib = 0; nib < 8; ++nib) {
    const int reg = nib & 3, odd = nib >> 2;
    const int hi_row = reg & 1, hi_col = reg >> 1;
    const int64_t n = tile * 16 + g + 8 * hi_row;
    const int kin = step * 16 + 2 * t + odd + 8 * hi_col;  // 0..31 inside the block
    const int64_t kb = kg * 2 + blk;
    const uint8_t* qs = rows + (n * nb + kb) * SYN_Q4_ROW_BLOCK_BYTES + 4;
    const uint32_t q = kin < 16 ? (qs[kin] & 15u) : (qs[kin - 16] >> 4);
    word |= q << (4 * nib);
  }
  qw[i] = word;
}

// Tiled -> row-block interchange layout.  One thread per 32-element block.
__global__ void q4_tiled_to_rows_kernel(const uint32_t* __restrict__ qw, const half2* __restrict__ sm,
                                        int64_t N, int64_t K, uint8_t* __restrict__ rows) {
  const int64_t nb = K / SYN_Q4_BLOCK;
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= N * nb) return;
  const int64_t n = i / nb, kb = i % nb;
  uint8_t* b = rows + (n * nb + kb) * SYN_Q4_ROW_BLOCK_BYTES;
  const half2 dm = sm[q4t_scale_index(K, n, kb)];
  memcpy(b, &dm, 4);
  uint8_t qs[16];
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    int64_t wi;
    int nib;
    q4t_locate(N, K, n, kb * 32 + j, &wi, &nib);
    const uint32_t lo = (qw[wi] >> (4 * nib)) & 15u;
    q4t_locate(N, K, n, kb * 32 + j + 16, &wi, &nib);
    const uint32_t hi = (qw[wi] >> (4 * nib)) & 15u;
    qs[j] = (uint8_t)(lo | (hi << 4));
  }
  memcpy(b + 4, qs, 16);
}

// Tiled -> bf16 [N, K].  One thread per element (not a hot path).
__global__ void q4t_dequant_kernel(const uint32_t* __restrict__ qw, const half2* __restrict__ sm,
                                   int64_t N, int64_t K, __nv_bfloat16* __restrict__ out) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= N * K) return;
  const int64_t n = i / K, k = i % K;
  int64_t wi;
  int nib;
  q4t_locate(N, K, n, k, &wi, &nib);
  const float q = (float)((qw[wi] >> (4 * nib)) & 15u);
  const half2 dm = sm[q4t_scale_index(K, n, k / SYN_Q4_BLOCK)];
  out[i] = __float2bfloat16_rn(fmaf(__low2float(dm), q, __high2float(dm)));
}

static inline unsigned nblk(int64_t n, int t) { return (unsigned)((n + t - 1) / t); }

cudaError_t launch_q4_quantize(const void* w, bool is_bf16, int64_t N, int64_t K, uint32_t* qw, void* sm,
                               cudaStream_t s) {
  half2* smp = reinterpret_cast<half2*>(sm);
  if (!is_bf16) {
    const float* p = reinterpret_cast<const float*>(w);
    q4_block_scales_kernel<float><<<nblk(N * K / 32, 256), 256, 0, s>>>(p, N, K, smp);
    q4_pack_tiled_kernel<float><<<nblk(N * K / 8, 256), 256, 0, s>>>(p, N, K, smp, qw);
  } else {
    const __nv_bfloat16* p = reinterpret_cast<const __nv_bfloat16*>(w);
    q4_block_scales_kernel<__nv_bfloat16><<<nblk(N * K / 32, 256), 256, 0, s>>>(p, N, K, smp);
    q4_pack_tiled_kernel<__nv_bfloat16><<<nblk(N * K / 8, 256), 256, 0, s>>>(p, N, K, smp, qw);
  }
  return cudaGetLastError();
}

cudaError_t launch_q4_rows_to_tiled(const uint8_t* rows, int64_t N, int64_t K, uint32_t* qw, void* sm,
                                    cudaStream_t s) {
  q4_rows_to_tiled_kernel<<<nblk(N * K / 8, 256), 256, 0, s>>>(rows, N, K, qw, reinterpret_cast<half2*>(sm));
  return cudaGetLastError();
}

cudaError_t launch_q4_tiled_to_rows(const uint32_t* qw, const void* sm, int64_t N, int64_t K, uint8_t* rows,
                                    cudaStream_t s) {
  q4_tiled_to_rows_kernel<<<nblk(N * K / 32, 256), 256, 0, s>>>(qw, reinterpret_cast<const half2*>(sm), N, K,
                                                                 rows);
  return cudaGetLastError();
}

cudaError_t launch_q4t_dequant(const uint32_t* qw, const void* sm, int64_t N, int64_t K, void* out,
                               cudaStream_t s) {
  q4t_dequant_kernel<<<nblk(N * K, 256), 256, 0, s>>>(qw, reinterpret_cast<const half2*>(sm), N, K,
                                                       reinterpret_cast<__nv_bfloat16*>(out));
  return cudaGetLastError();
}

}  // namespace syn
