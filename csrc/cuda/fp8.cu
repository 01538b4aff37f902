// Block-scaled fp8 (e4m3) decode kernels: weights with one f32 scale per 128x128 block,
// activations quantised per token in 1x128 blocks, products on the fp8 tensor-core path
// (mma.sync m16n8k32 e4m3 x e4m3 -> f32) and the two scales applied once per 128-column
// block:  y[p][n] = sum_b  s_w[n/128][b] * s_x[p][b] * sum_{k in b} q_w[n][k] q_x[p][k].
// Reference: block-scaled fp8 of plan/rfcs/RFC-0042-quantization-and-numerical-fidelity.md
// §2.3 (128x128 weight tiles, 1x128 activation groups); op `Gemv` / `MoeGrouped`.
//
// Tiled weight layout: per (16-row tile, 64-column group) 1024 bytes = 32 lanes x 32 B; lane
// (g = lane/4, t = lane%4) holds, for k32 steps 0 and 1, the four A registers of
// m16n8k32: rows g / g+8, columns 4t..4t+3 / 16+4t..16+4t+3 of the step.  One 2 x 128-bit
// streaming load per lane and group; no shared-memory staging.
#include "common.cuh"
#include "gemv_epilogue.cuh"
#include "sync.cuh"

namespace syn {

// ---- activation quantisation: warp per (row, 128-column block) ----
__global__ void f8_quant_act_kernel(const __nv_bfloat16* __restrict__ x, int rows, int K, int ldx,
                                    uint8_t* __restrict__ xq, float* __restrict__ xs) {
  const int KB = K / 128;
  const int w = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (w >= rows * KB) return;
  const int r = w / KB, b = w % KB;
  const uint2 raw = *reinterpret_cast<const uint2*>(x + (int64_t)r * ldx + b * 128 + lane * 4);
  const float2 v01 = unpack_bf16x2(raw.x), v23 = unpack_bf16x2(raw.y);
  float amax = fmaxf(fmaxf(fabsf(v01.x), fabsf(v01.y)), fmaxf(fabsf(v23.x), fabsf(v23.y)));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  const float s = fmaxf(amax, 1e-12f) / 448.f;
  const float inv = 1.f / s;
  uint16_t lo, hi;
  // the first f32 operand lands in the upper byte: pass (x1, x0) so x0 is the lower address
  asm volatile("{ .reg .b16 r; cvt.rn.satfinite.e4m3x2.f32 r, %1, %2; mov.b16 %0, r; }"
               : "=h"(lo) : "f"(v01.y * inv), "f"(v01.x * inv));
  asm volatile("{ .reg .b16 r; cvt.rn.satfinite.e4m3x2.f32 r, %1, %2; mov.b16 %0, r; }"
               : "=h"(hi) : "f"(v23.y * inv), "f"(v23.x * inv));
  *reinterpret_cast<uint32_t*>(xq + (int64_t)r * K + b * 128 + lane * 4) = (uint32_t)lo | ((uint32_t)hi << 16);
  if (lane == 0) xs[(int64_t)r * KB + b] = s;
}

cudaError_t launch_f8_quant_act(const void* x, int rows, int K, int ldx, uint8_t* xq, float* xs, cudaStream_t s) {
  if (rows == 0) return cudaSuccess;
  if (K % 128 || ldx % 4) return cudaErrorInvalidValue;
  const long warps = (long)rows * (K / 128);
  f8_quant_act_kernel<<<(unsigned)((warps + 7) / 8), 256, 0, s>>>(reinterpret_cast<const __nv_bfloat16*>(x), rows,
                                                                   K, ldx, xq, xs);
  return cudaGetLastError();
}

// ---- row-major e4m3 [N, K] <-> tiled layout: thread per tiled 4-byte register ----
template <bool TO_ROWS>
__global__ void f8_tile_kernel(const uint8_t* __restrict__ q, int N, int K, uint32_t* __restrict__ out) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;  // tiled word
  const int KG = K / 64;
  if (i >= (int64_t)N * K / 4) return;
  const int64_t grp = i >> 8;  // 256 words per (tile, group)
  const int w = (int)(i & 255);
  const int lane = w >> 3, step = (w >> 2) & 1, reg = w & 3;
  const int tile = (int)(grp / KG), kg = (int)(grp % KG);
  const int g = lane >> 2, t = lane & 3;
  const int row = tile * 16 + g + 8 * (reg & 1);
  const int col = kg * 64 + step * 32 + 16 * (reg >> 1) + 4 * t;
  if (TO_ROWS)
    *reinterpret_cast<uint32_t*>(reinterpret_cast<uint8_t*>(out) + (int64_t)row * K + col) =
        reinterpret_cast<const uint32_t*>(q)[i];
  else
    out[i] = *reinterpret_cast<const uint32_t*>(q + (int64_t)row * K + col);
}

cudaError_t launch_f8_rows_to_tiled(const uint8_t* q, int N, int K, uint8_t* tiled, cudaStream_t s) {
  if (N % 16 || K % 128) return cudaErrorInvalidValue;
  const int64_t words = (int64_t)N * K / 4;
  f8_tile_kernel<false><<<(unsigned)((words + 255) / 256), 256, 0, s>>>(q, N, K, reinterpret_cast<uint32_t*>(tiled));
  return cudaGetLastError();
}

cudaError_t launch_f8_tiled_to_rows(const uint8_t* tiled, int N, int K, uint8_t* q, cudaStream_t s) {
  if (N % 16 || K % 128) return cudaErrorInvalidValue;
  const int64_t words = (int64_t)N * K / 4;
  f8_tile_kernel<true><<<(unsigned)((words + 255) / 256), 256, 0, s>>>(tiled, N, K, reinterpret_cast<uint32_t*>(q));
  return cudaGetLastError();
}

// tiled e4m3 -> bf16 row-major with the 128x128 block scales applied (prefill operands of the
// bf16 tensor-core GEMM): thread per tiled 4-byte word, e4m3 pairs widened by cvt to f16x2
__global__ void f8_dequant_tiled_kernel(const uint32_t* __restrict__ tiled, const float* __restrict__ scale, int N,
                                        int K, __nv_bfloat16* __restrict__ out) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int KG = K / 64;
  if (i >= (int64_t)N * K / 4) return;
  const int64_t grp = i >> 8;
  const int w = (int)(i & 255);
  const int lane = w >> 3, step = (w >> 2) & 1, reg = w & 3;
  const int tile = (int)(grp / KG), kg = (int)(grp % KG);
  const int g = lane >> 2, t = lane & 3;
  const int row = tile * 16 + g + 8 * (reg & 1);
  const int col = kg * 64 + step * 32 + 16 * (reg >> 1) + 4 * t;
  const float sc = scale[(int64_t)(row >> 7) * ((K + 127) >> 7) + (col >> 7)];
  const uint32_t v = tiled[i];
  uint32_t h01, h23;
  asm("{ .reg .b16 lo, hi; mov.b32 {lo, hi}, %2; cvt.rn.f16x2.e4m3x2 %0, lo; cvt.rn.f16x2.e4m3x2 %1, hi; }"
      : "=r"(h01), "=r"(h23)
      : "r"(v));
  const float2 f01 = __half22float2(*reinterpret_cast<const __half2*>(&h01));
  const float2 f23 = __half22float2(*reinterpret_cast<const __half2*>(&h23));
  uint2 o;
  o.x = pack_bf16x2(f01.x * sc, f01.y * sc);
  o.y = pack_bf16x2(f23.x * sc, f23.y * sc);
  *reinterpret_cast<uint2*>(out + (int64_t)row * K + col) = o;
}

cudaError_t launch_f8_dequant_tiled(const uint8_t* tiled, const float* scale, int N, int K, void* out_bf16,
                                    cudaStream_t s) {
  if (N % 16 || K % 128) return cudaErrorInvalidValue;
  const int64_t words = (int64_t)N * K / 4;
  f8_dequant_tiled_kernel<<<(unsigned)((words + 255) / 256), 256, 0, s>>>(
      reinterpret_cast<const uint32_t*>(tiled), scale, N, K, reinterpret_cast<__nv_bfloat16*>(out_bf16));
  return cudaGetLastError();
}

__device__ __forceinline__ void mma_e4m3_16832(float* d, const uint32_t* a, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.f32.e4m3.e4m3.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// ---- grouped GEMV: warp = one 16-row tile of one expert, all K; four warps per CTA ----
// U groups (64 columns) of weights in flight per lane (2 x 16 B each); each 128-column
// block is reduced in a fresh accumulator and then scaled into the running sum.
template <int NT, int U>
__global__ void __launch_bounds__(128, 4) f8_gemv_kernel(GemvArgs a) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int g = lane >> 2, t = lane & 3;
  const int e = blockIdx.y;
  const int p0 = a.tok_off[e];
  const int cnt = a.tok_off[e + 1] - p0;
  const int tile = blockIdx.x * 4 + warp;
  // no early return: with done_ctr set every CTA must reach the completion count below
  const bool active = cnt > 0 && tile < a.N / 16;
  const int KG = a.K >> 6, KB = a.K >> 7;
  // K slice (split-K over gridDim.z, dense only): 128-column blocks [kb_lo, kb_hi)
  const int KS = gridDim.z, ks = blockIdx.z;
  const int kb_lo = (int)((int64_t)KB * ks / KS), kb_hi = (int)((int64_t)KB * (ks + 1) / KS);
  const uint4* __restrict__ wq = reinterpret_cast<const uint4*>(a.qw_ptrs[e]) + (int64_t)tile * KG * 64;
  const float* __restrict__ ws = reinterpret_cast<const float*>(a.sm_ptrs[e]) + (int64_t)(tile >> 3) * KB;
  for (int c0 = 0; active && c0 < cnt; c0 += NT * 8) {
    const int ccount = min(cnt - c0, NT * 8);
    // B rows (token g of each n-tile) and the two accumulator tokens (2t, 2t+1) per n-tile
    const uint8_t* xrow[NT];
    const float* srow[NT][2];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      const int jb = min(nt * 8 + g, ccount - 1);
      const int rb = a.tok_idx ? a.tok_idx[p0 + c0 + jb] : p0 + c0 + jb;
      xrow[nt] = a.xq + (int64_t)rb * a.ldx + 4 * t;
#pragma unroll
      for (int hf = 0; hf < 2; ++hf) {
        const int jc = min(nt * 8 + 2 * t + hf, ccount - 1);
        const int rc = a.tok_idx ? a.tok_idx[p0 + c0 + jc] : p0 + c0 + jc;
        srow[nt][hf] = a.xs + (int64_t)rc * KB;
      }
    }
    float acc[NT][4];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int i = 0; i < 4; ++i) acc[nt][i] = 0.f;
    for (int kb0 = 2 * kb_lo; kb0 < 2 * kb_hi; kb0 += U) {
      uint4 wv[U][2];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        if (kb0 + u < 2 * kb_hi) {
          wv[u][0] = __ldcs(wq + (int64_t)(kb0 + u) * 64 + lane * 2);
          wv[u][1] = __ldcs(wq + (int64_t)(kb0 + u) * 64 + lane * 2 + 1);
        }
      }
#pragma unroll
      for (int u = 0; u < U; u += 2) {  // one 128-column scale block = two groups
        const int kg = kb0 + u;
        if (kg >= 2 * kb_hi) break;
        const int kb = kg >> 1;
        const float sw = __ldg(ws + kb);
        float part[NT][4];
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
          for (int i = 0; i < 4; ++i) part[nt][i] = 0.f;
#pragma unroll
        for (int uu = 0; uu < 2; ++uu) {
#pragma unroll
          for (int st = 0; st < 2; ++st) {
            const uint4 v = wv[u + uu][st];
            const uint32_t af[4] = {v.x, v.y, v.z, v.w};
            const int k0 = (kg + uu) * 64 + st * 32;
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
              const uint32_t b0 = __ldg(reinterpret_cast<const uint32_t*>(xrow[nt] + k0));
              const uint32_t b1 = __ldg(reinterpret_cast<const uint32_t*>(xrow[nt] + k0 + 16));
              mma_e4m3_16832(part[nt], af, b0, b1);
            }
          }
        }
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          const float s0 = sw * __ldg(srow[nt][0] + kb), s1 = sw * __ldg(srow[nt][1] + kb);
          acc[nt][0] = fmaf(part[nt][0], s0, acc[nt][0]);
          acc[nt][1] = fmaf(part[nt][1], s1, acc[nt][1]);
          acc[nt][2] = fmaf(part[nt][2], s0, acc[nt][2]);
          acc[nt][3] = fmaf(part[nt][3], s1, acc[nt][3]);
        }
      }
    }
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int hf = 0; hf < 2; ++hf) {
        const int j = nt * 8 + 2 * t + hf;
        if (j >= ccount) continue;
        const int p = p0 + c0 + j;
        if (KS > 1) {  // raw partial sums; the reduce kernel applies the epilogue
          float* w = a.ws_part + ((int64_t)ks * a.ws_rows + p) * a.N;
          w[tile * 16 + g] = acc[nt][hf];
          w[tile * 16 + g + 8] = acc[nt][2 + hf];
          continue;
        }
        if (a.mode == GEMV_SWIGLU) {
          reinterpret_cast<__nv_bfloat16*>(a.out)[(int64_t)p * (a.N / 2) + tile * 8 + g] =
              f2bf(silu(acc[nt][hf]) * acc[nt][2 + hf]);
        } else {
          gemv_store(a, p, tile * 16 + g, acc[nt][hf]);
          gemv_store(a, p, tile * 16 + g + 8, acc[nt][2 + hf]);
        }
      }
  }
  if (a.done_ctr != nullptr) {
    // Expert parallelism: the rows above went to their source ranks' combine slots (mode
    // GEMV_SCALED_F32_PTR); every CTA publishes them and the last one raises this layer's
    // flag on every peer (the counter is reset for the next launch before the release).
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x == 0) {
      const unsigned total = gridDim.x * gridDim.y * gridDim.z;
      const unsigned prev = atomicAdd(a.done_ctr, 1u);
      if (prev == total - 1) {
        *a.done_ctr = 0u;
        __threadfence_system();
        const uint32_t seq = (*a.step_ctr) * (uint32_t)a.n_layers + (uint32_t)a.layer + 1u;
        for (int q = 0; q < a.sig_n; ++q)
          st_release_sys(reinterpret_cast<uint32_t*>(a.sig_peers[q] + a.sig_off) + a.sig_rank, seq);
      }
    }
  }
}

// Split-K reduction in slice order (deterministic) + the epilogue: thread per (row, output).
__global__ void f8_splitk_reduce_kernel(GemvArgs a, int KS) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int rows = a.ws_rows;
  if (i >= (int64_t)rows * a.N) return;
  const int p = (int)(i / a.N), n = (int)(i % a.N);
  if (a.mode == GEMV_SWIGLU && (n & 15) >= 8) return;  // up rows are read by their gate row
  float v = 0.f, u = 0.f;
  for (int k = 0; k < KS; ++k) {
    const float* w = a.ws_part + ((int64_t)k * rows + p) * a.N;
    v += w[n];
    if (a.mode == GEMV_SWIGLU) u += w[n + 8];
  }
  if (a.mode == GEMV_SWIGLU)
    reinterpret_cast<__nv_bfloat16*>(a.out)[(int64_t)p * (a.N / 2) + (n >> 4) * 8 + (n & 7)] = f2bf(silu(v) * u);
  else
    gemv_store(a, p, n, v);
}

int f8_gemv_ksplit(int N, int K, int E, int rows, size_t ws_floats) {
  if (E != 1 || rows <= 0) return 1;
  const int ctas = (N / 16 + 3) / 4;
  int ks = (2 * 148 * 4 + ctas - 1) / ctas;  // ~4 CTAs per SM
  ks = ks < 1 ? 1 : (ks > 16 ? 16 : ks);
  if (ks > K / 128) ks = K / 128;
  while (ks > 1 && (size_t)ks * rows * N > ws_floats) --ks;
  return ks;
}

cudaError_t launch_f8_gemv(const GemvArgs& a_in, cudaStream_t s) {
  if (a_in.N % 16 || a_in.K % 128 || !a_in.xq || !a_in.xs || a_in.ldx % 4) return cudaErrorInvalidValue;
  // split-K finishes in a second kernel, which the completion flags would not wait for
  if (a_in.done_ctr && a_in.ws_part) return cudaErrorInvalidValue;
  GemvArgs a = a_in;
  const int ks = a.ws_part ? f8_gemv_ksplit(a.N, a.K, a.E, a.ws_rows, a.ws_floats) : 1;
  dim3 grid((unsigned)((a.N / 16 + 3) / 4), (unsigned)a.E, (unsigned)ks);
  const int nt = a.nt_hint <= 1 ? 1 : (a.nt_hint <= 2 ? 2 : 4);
  if (nt == 1) f8_gemv_kernel<1, 4><<<grid, 128, 0, s>>>(a);
  else if (nt == 2) f8_gemv_kernel<2, 4><<<grid, 128, 0, s>>>(a);
  else f8_gemv_kernel<4, 2><<<grid, 128, 0, s>>>(a);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess || ks == 1) return e;
  const int64_t n = (int64_t)a.ws_rows * a.N;
  f8_splitk_reduce_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(a, ks);
  return cudaGetLastError();
}

}  // namespace syn
