// Decode-time matrix-vector products with 4-bit tiled weights (see syn/q4.h).
//
// y[p][n] = sum_k W_e[n][k] * x[row(p)][k] for every (expert e, pair p) in a CSR list.
// The dense case is one expert with the identity row map.  Reference op semantics:
// `Gemv` / `MoeGrouped` in crates/kernels/src/op/kind.rs (f32 reference at
// crates/kernels/src/reference/linear.rs:62).
//
// Mapping to the hardware (memory-bound: the weight stream is the roofline):
//  * One 128-bit streaming load per lane covers a 16-row x 64-column weight tile, already
//    in mma.sync m16n8k16 A-fragment order, so no shared-memory staging is needed.
//  * Nibbles become bf16 (128 + q) with one LOP3 per register; tokens are the N=8 side
//    of the MMA ("swap AB"), so 1..8 tokens per expert cost one MMA per k16 step.
//  * Per 32-element block the raw integer dot product and sum(x) (an MMA with an
//    all-ones A) are folded with the fp32 scale and min:
//        acc += d * sum((128+q) x) + (m - 128 d) * sum(x)
//    so the dequantised weight is never rounded to bf16.
//  * Eight warps split K inside the CTA and reduce through shared memory in a fixed
//    order (deterministic); one CTA per (16-row tile, expert).
#include "common.cuh"
#include "gemv_epilogue.cuh"
#include "syn/q4.h"
#include <cstdlib>

#include "sync.cuh"

namespace syn {


// Warp tile: R 16-row tiles x NT 8-token tiles; KS warps split K (KS == 1: every warp of the
// 4-warp CTA is an independent tile, no shared memory).  U k-groups (64 columns each) of
// weights and scales are loaded before any of them is used, so each warp keeps
// U * R * 528 bytes in flight.
template <int R, int NT, int KS, int U = 4, int MINB = 1>
__global__ void __launch_bounds__(KS == 1 ? 128 : KS * 32, MINB)
q4_gemv2_kernel(GemvArgs a) {
  constexpr int WARPS = KS == 1 ? 4 : KS;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int g = lane >> 2, t = lane & 3;
  const int e = blockIdx.y;
  const int p0 = a.tok_off[e];
  // a null weight pointer marks an expert computed elsewhere (the host CPU): its pairs are skipped
  const int cnt = a.qw_ptrs[e] ? a.tok_off[e + 1] - p0 : 0;
  const int n_units = a.N / (16 * R);
  const int unit = KS == 1 ? blockIdx.x * WARPS + warp : blockIdx.x;
  const int kw = KS == 1 ? 0 : warp;
  const int KG = a.K >> 6;
  const bool active = cnt > 0 && unit < n_units;

  extern __shared__ float gsm[];  // KS > 1: [KS][R][NT][4][32]

  if (active || KS > 1) {
    const uint4* __restrict__ qw = reinterpret_cast<const uint4*>(a.qw_ptrs[e]);
    const uint2* __restrict__ sm = reinterpret_cast<const uint2*>(a.sm_ptrs[e]);
    const __nv_bfloat16* xbase = reinterpret_cast<const __nv_bfloat16*>(a.x);
    const uint32_t ones[4] = {0x3F803F80u, 0x3F803F80u, 0x3F803F80u, 0x3F803F80u};
    const int nchunks = active ? (cnt + NT * 8 - 1) / (NT * 8) : 0;
    for (int ch = 0; ch < nchunks; ++ch) {
      const int c0 = ch * NT * 8;
      const int ccount = min(cnt - c0, NT * 8);
      const int ntc = (ccount + 7) >> 3;
      const __nv_bfloat16* xr[NT];
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        const int j = min(nt * 8 + g, ccount - 1);
        const int pp = p0 + c0 + j;
        const int row = a.tok_idx ? a.tok_idx[pp] : pp;
        xr[nt] = xbase + (int64_t)row * a.ldx + 2 * t;
      }
      float acc[R][NT][4];
#pragma unroll
      for (int r = 0; r < R; ++r)
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
          for (int i = 0; i < 4; ++i) acc[r][nt][i] = 0.f;

      uint4 q[U][R];
      uint2 slo[U][R], shi[U][R];
      auto load_batch = [&](int kb0, uint4 (&qq)[U][R], uint2 (&sl)[U][R], uint2 (&sh)[U][R]) {
#pragma unroll
        for (int u = 0; u < U; ++u) {
          const int kg = kb0 + u * KS;
          if (kg < KG) {
#pragma unroll
            for (int r = 0; r < R; ++r) {
              const int64_t tk = (int64_t)(unit * R + r) * KG + kg;
              qq[u][r] = ld_stream_v4(qw + tk * 32 + lane);
              sl[u][r] = ld_stream_v2(sm + tk * 16 + g);
              sh[u][r] = ld_stream_v2(sm + tk * 16 + g + 8);
            }
          }
        }
      };
      for (int kb = kw; kb < KG; kb += KS * U) {
        load_batch(kb, q, slo, shi);
#pragma unroll
        for (int u = 0; u < U; ++u) {
          const int kg = kb + u * KS;
          if (kg >= KG) break;
#pragma unroll
          for (int b = 0; b < 2; ++b) {
            uint32_t af[R][2][4];
#pragma unroll
            for (int r = 0; r < R; ++r) {
              const uint32_t w0 = b ? q[u][r].z : q[u][r].x;
              const uint32_t w1 = b ? q[u][r].w : q[u][r].y;
#pragma unroll
              for (int j = 0; j < 4; ++j) {
                af[r][0][j] = lop3_and_or(w0 >> (4 * j), 0x000F000Fu, 0x43004300u);
                af[r][1][j] = lop3_and_or(w1 >> (4 * j), 0x000F000Fu, 0x43004300u);
              }
            }
            float dlo[R], dhi[R], mlo[R], mhi[R];
#pragma unroll
            for (int r = 0; r < R; ++r) {
              const uint32_t vlo = b ? slo[u][r].y : slo[u][r].x;
              const uint32_t vhi = b ? shi[u][r].y : shi[u][r].x;
              const half2 hl = *reinterpret_cast<const half2*>(&vlo);
              const half2 hh = *reinterpret_cast<const half2*>(&vhi);
              dlo[r] = __low2float(hl);
              dhi[r] = __low2float(hh);
              mlo[r] = fmaf(-128.f, dlo[r], __high2float(hl));
              mhi[r] = fmaf(-128.f, dhi[r], __high2float(hh));
            }
            const int k0 = kg * 64 + b * 32;
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
              if (nt < ntc) {
                uint32_t bf[2][2];
                bf[0][0] = __ldg(reinterpret_cast<const uint32_t*>(xr[nt] + k0));
                bf[0][1] = __ldg(reinterpret_cast<const uint32_t*>(xr[nt] + k0 + 8));
                bf[1][0] = __ldg(reinterpret_cast<const uint32_t*>(xr[nt] + k0 + 16));
                bf[1][1] = __ldg(reinterpret_cast<const uint32_t*>(xr[nt] + k0 + 24));
                float xs[4] = {0.f, 0.f, 0.f, 0.f};
                mma_bf16_16816(xs, ones, bf[0], xs);
                mma_bf16_16816(xs, ones, bf[1], xs);
#pragma unroll
                for (int r = 0; r < R; ++r) {
                  float blk[4] = {0.f, 0.f, 0.f, 0.f};
                  mma_bf16_16816(blk, af[r][0], bf[0], blk);
                  mma_bf16_16816(blk, af[r][1], bf[1], blk);
                  acc[r][nt][0] += fmaf(dlo[r], blk[0], mlo[r] * xs[0]);
                  acc[r][nt][1] += fmaf(dlo[r], blk[1], mlo[r] * xs[1]);
                  acc[r][nt][2] += fmaf(dhi[r], blk[2], mhi[r] * xs[2]);
                  acc[r][nt][3] += fmaf(dhi[r], blk[3], mhi[r] * xs[3]);
                }
              }
            }
          }
        }
      }

      if (KS > 1) {
        // split-K reduction across the CTA's warps in a fixed order
        float* red = gsm;
#pragma unroll
        for (int r = 0; r < R; ++r)
#pragma unroll
          for (int nt = 0; nt < NT; ++nt)
#pragma unroll
            for (int i = 0; i < 4; ++i) red[(((warp * R + r) * NT + nt) * 4 + i) * 32 + lane] = acc[r][nt][i];
        __syncthreads();
        if (warp == 0) {
#pragma unroll
          for (int r = 0; r < R; ++r)
#pragma unroll
            for (int nt = 0; nt < NT; ++nt)
#pragma unroll
              for (int i = 0; i < 4; ++i) {
                float v = 0.f;
                for (int w = 0; w < KS; ++w) v += red[(((w * R + r) * NT + nt) * 4 + i) * 32 + lane];
                acc[r][nt][i] = v;
              }
        }
        __syncthreads();
        if (warp != 0) continue;
      }
      // Epilogue straight from the accumulator fragments:
      // acc[r][nt][0]: row g, token 2t; [1]: row g, token 2t+1; [2], [3]: row g+8.
#pragma unroll
      for (int r = 0; r < R; ++r) {
        const int tile = unit * R + r;
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
          for (int hf = 0; hf < 2; ++hf) {
            const int j = nt * 8 + 2 * t + hf;
            if (j >= ccount) continue;
            const int p = p0 + c0 + j;
            if (a.mode == GEMV_SWIGLU) {
              const float gv = acc[r][nt][hf], uv = acc[r][nt][2 + hf];
              reinterpret_cast<__nv_bfloat16*>(a.out)[(int64_t)p * (a.N / 2) + tile * 8 + g] = f2bf(silu(gv) * uv);
            } else {
              gemv_store(a, p, tile * 16 + g, acc[r][nt][hf]);
              gemv_store(a, p, tile * 16 + g + 8, acc[r][nt][2 + hf]);
            }
          }
        }
      }
    }
  }
  if (a.done_ctr != nullptr) {
    // Completion of the whole grid: every CTA publishes its stores, the last one raises
    // the peers' flags (counter reset for the next launch before the release).
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x == 0) {
      const unsigned total = gridDim.x * gridDim.y;
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

template <int R, int NT, int KS, int U = 4, int MINB = 1>
static cudaError_t launch_v2(const GemvArgs& a, cudaStream_t s) {
  constexpr int WARPS = KS == 1 ? 4 : KS;
  const int units = a.N / (16 * R);
  const int gx = KS == 1 ? (units + WARPS - 1) / WARPS : units;
  const size_t smem = KS > 1 ? (size_t)KS * R * NT * 4 * 32 * sizeof(float) : 0;
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(q4_gemv2_kernel<R, NT, KS, U, MINB>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
  }
  dim3 grid((unsigned)gx, (unsigned)a.E);
  q4_gemv2_kernel<R, NT, KS, U, MINB><<<grid, WARPS * 32, smem, s>>>(a);
  return cudaGetLastError();
}


__device__ __forceinline__ void cp_async16_g(void* smem, const void* gmem) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"((uint32_t)__cvta_generic_to_shared(smem)),
               "l"(gmem));
}
__device__ __forceinline__ void cp_async8_g(void* smem, const void* gmem) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 8;\n" ::"r"((uint32_t)__cvta_generic_to_shared(smem)),
               "l"(gmem));
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N>
__device__ __forceinline__ void cp_wait() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N)); }

// v3: per-warp cp.async ring of packed weight groups (no registers held by loads in
// flight) and per-CTA block sums of x in shared memory (no extra MMAs for the min term).
// Warp tile: R 16-row tiles x NT 8-token tiles over the full K; CTA = 4 warps = 4 tiles
// of the same expert.  S ring slots per warp, D groups prefetched ahead.
template <int R, int NT>
struct GemvV3 {
  static constexpr int WARPS = 4;
  static constexpr int S = 8;        // ring slots per warp
  static constexpr int D = 6;        // groups in flight ahead of the consumer
  static constexpr int SLOT = R * 640;  // bytes per slot: R x (512 B nibbles + 128 B scales)
  static size_t smem(int K, bool xsum_global) {
    return (size_t)WARPS * S * SLOT + (xsum_global ? 0 : (size_t)NT * 8 * (K / 32) * 4);
  }
};

template <int R, int NT>
__global__ void __launch_bounds__(128) q4_gemv3_kernel(GemvArgs a) {
  using C = GemvV3<R, NT>;
  extern __shared__ __align__(16) uint8_t gsm3[];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int g = lane >> 2, t = lane & 3;
  const int e = blockIdx.y;
  const int p0 = a.tok_off[e];
  // a null weight pointer marks an expert computed elsewhere (the host CPU): its pairs are skipped
  const int cnt = a.qw_ptrs[e] ? a.tok_off[e + 1] - p0 : 0;
  const int n_units = a.N / (16 * R);
  const int unit = blockIdx.x * C::WARPS + warp;
  const int KG = a.K >> 6, KB32 = a.K >> 5;
  uint8_t* ring = gsm3 + warp * C::S * C::SLOT;
  float* xsum = reinterpret_cast<float*>(gsm3 + C::WARPS * C::S * C::SLOT);  // [NT*8][KB32]
  const bool cta_active = cnt > 0 && blockIdx.x * C::WARPS < n_units;

  if (cta_active) {
    const uint8_t* qw = reinterpret_cast<const uint8_t*>(a.qw_ptrs[e]);
    const uint8_t* smw = reinterpret_cast<const uint8_t*>(a.sm_ptrs[e]);
    const __nv_bfloat16* xbase = reinterpret_cast<const __nv_bfloat16*>(a.x);
    const bool active = unit < n_units;
    auto issue = [&](int kg) {
      uint8_t* slot = ring + (kg % C::S) * C::SLOT;
      if (active && kg < KG) {
#pragma unroll
        for (int r = 0; r < R; ++r) {
          const int64_t tk = (int64_t)(unit * R + r) * KG + kg;
          cp_async16_g(slot + r * 640 + lane * 16, qw + tk * 512 + lane * 16);
          if (lane < 8) cp_async16_g(slot + r * 640 + 512 + lane * 16, smw + tk * 128 + lane * 16);
        }
      }
      cp_commit();  // empty groups keep the wait_group arithmetic uniform
    };
    for (int c0 = 0; c0 < cnt; c0 += NT * 8) {
      const int ccount = min(cnt - c0, NT * 8);
      const int ntc = (ccount + 7) >> 3;
      // weights start streaming before the block sums are formed
#pragma unroll
      for (int i = 0; i < C::D; ++i) issue(i);
      // ---- block sums of x for this chunk's tokens (fixed order) ----
      const float* xsg = a.xsum;  // optional precomputed [rows][K/32]
      if (xsg == nullptr) {
        __syncthreads();
        for (int idx = threadIdx.x; idx < ntc * 8 * KB32; idx += blockDim.x) {
          const int j = idx / KB32, kb = idx % KB32;
          float sacc = 0.f;
          if (j < ccount) {
            const int pp = p0 + c0 + j;
            const int row = a.tok_idx ? a.tok_idx[pp] : pp;
            const uint4* xp = reinterpret_cast<const uint4*>(xbase + (int64_t)row * a.ldx + kb * 32);
#pragma unroll
            for (int c = 0; c < 4; ++c) {
              const uint4 v = __ldg(xp + c);
              const uint32_t w4[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
              for (int i = 0; i < 4; ++i) {
                const float2 f = unpack_bf16x2(w4[i]);
                sacc += f.x + f.y;
              }
            }
          }
          xsum[j * KB32 + kb] = sacc;
        }
        __syncthreads();
      }
      if (!active) {
        cp_wait<0>();
        continue;
      }
      const __nv_bfloat16* xr[NT];
      const float* xsr[NT][2];
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        const int j = min(nt * 8 + g, ccount - 1);
        const int pp = p0 + c0 + j;
        const int row = a.tok_idx ? a.tok_idx[pp] : pp;
        xr[nt] = xbase + (int64_t)row * a.ldx + 2 * t;
#pragma unroll
        for (int hf = 0; hf < 2; ++hf) {
          const int jj = min(nt * 8 + 2 * t + hf, ccount - 1);
          if (xsg) {
            const int pj = p0 + c0 + jj;
            const int rj = a.tok_idx ? a.tok_idx[pj] : pj;
            xsr[nt][hf] = xsg + (int64_t)rj * KB32;
          } else {
            xsr[nt][hf] = xsum + (nt * 8 + 2 * t + hf) * KB32;
          }
        }
      }
      float acc[R][NT][4];
#pragma unroll
      for (int r = 0; r < R; ++r)
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
          for (int i = 0; i < 4; ++i) acc[r][nt][i] = 0.f;

      for (int kg = 0; kg < KG; ++kg) {
        issue(kg + C::D);
        cp_wait<C::D>();
        __syncwarp();
        const uint8_t* slot = ring + (kg % C::S) * C::SLOT;
#pragma unroll
        for (int b = 0; b < 2; ++b) {
          uint32_t af[R][2][4];
          float dlo[R], dhi[R], mlo[R], mhi[R];
#pragma unroll
          for (int r = 0; r < R; ++r) {
            const uint4 q = *reinterpret_cast<const uint4*>(slot + r * 640 + lane * 16);
            const uint32_t w0 = b ? q.z : q.x;
            const uint32_t w1 = b ? q.w : q.y;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              af[r][0][j] = lop3_and_or(w0 >> (4 * j), 0x000F000Fu, 0x43004300u);
              af[r][1][j] = lop3_and_or(w1 >> (4 * j), 0x000F000Fu, 0x43004300u);
            }
            const half2 hl = *reinterpret_cast<const half2*>(slot + r * 640 + 512 + g * 8 + b * 4);
            const half2 hh = *reinterpret_cast<const half2*>(slot + r * 640 + 512 + (g + 8) * 8 + b * 4);
            dlo[r] = __low2float(hl);
            dhi[r] = __low2float(hh);
            mlo[r] = fmaf(-128.f, dlo[r], __high2float(hl));
            mhi[r] = fmaf(-128.f, dhi[r], __high2float(hh));
          }
          const int k0 = kg * 64 + b * 32;
          const int kb32 = kg * 2 + b;
#pragma unroll
          for (int nt = 0; nt < NT; ++nt) {
            if (nt < ntc) {
              uint32_t bf[2][2];
              bf[0][0] = __ldg(reinterpret_cast<const uint32_t*>(xr[nt] + k0));
              bf[0][1] = __ldg(reinterpret_cast<const uint32_t*>(xr[nt] + k0 + 8));
              bf[1][0] = __ldg(reinterpret_cast<const uint32_t*>(xr[nt] + k0 + 16));
              bf[1][1] = __ldg(reinterpret_cast<const uint32_t*>(xr[nt] + k0 + 24));
              const float xs0 = xsr[nt][0][kb32];
              const float xs1 = xsr[nt][1][kb32];
#pragma unroll
              for (int r = 0; r < R; ++r) {
                float blk[4] = {0.f, 0.f, 0.f, 0.f};
                mma_bf16_16816(blk, af[r][0], bf[0], blk);
                mma_bf16_16816(blk, af[r][1], bf[1], blk);
                acc[r][nt][0] += fmaf(dlo[r], blk[0], mlo[r] * xs0);
                acc[r][nt][1] += fmaf(dlo[r], blk[1], mlo[r] * xs1);
                acc[r][nt][2] += fmaf(dhi[r], blk[2], mhi[r] * xs0);
                acc[r][nt][3] += fmaf(dhi[r], blk[3], mhi[r] * xs1);
              }
            }
          }
        }
        __syncwarp();
      }
      cp_wait<0>();
#pragma unroll
      for (int r = 0; r < R; ++r) {
        const int tile = unit * R + r;
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
          for (int hf = 0; hf < 2; ++hf) {
            const int j = nt * 8 + 2 * t + hf;
            if (j >= ccount) continue;
            const int p = p0 + c0 + j;
            if (a.mode == GEMV_SWIGLU) {
              const float gv = acc[r][nt][hf], uv = acc[r][nt][2 + hf];
              reinterpret_cast<__nv_bfloat16*>(a.out)[(int64_t)p * (a.N / 2) + tile * 8 + g] = f2bf(silu(gv) * uv);
            } else {
              gemv_store(a, p, tile * 16 + g, acc[r][nt][hf]);
              gemv_store(a, p, tile * 16 + g + 8, acc[r][nt][2 + hf]);
            }
          }
        }
      }
    }
  }
  if (a.done_ctr != nullptr) {
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x == 0) {
      const unsigned total = gridDim.x * gridDim.y;
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

template <int R, int NT>
static cudaError_t launch_v3(const GemvArgs& a, cudaStream_t s) {
  using C = GemvV3<R, NT>;
  const int units = a.N / (16 * R);
  const int gx = (units + C::WARPS - 1) / C::WARPS;
  const size_t smem = C::smem(a.K, a.xsum != nullptr);
  static size_t set_for = 0;
  if (smem > 48 * 1024 && smem > set_for) {
    cudaError_t e = cudaFuncSetAttribute(q4_gemv3_kernel<R, NT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)smem);
    if (e != cudaSuccess) return e;
    set_for = smem;
  }
  dim3 grid((unsigned)gx, (unsigned)a.E);
  q4_gemv3_kernel<R, NT><<<grid, C::WARPS * 32, smem, s>>>(a);
  return cudaGetLastError();
}

// Block sums of x: out[r][b] = sum_{i<32} x[r][32 b + i] in f32 (fixed order).
__global__ void block_sums_kernel(const __nv_bfloat16* __restrict__ x, int rows, int K, int ldx,
                                  float* __restrict__ out) {
  const int KB32 = K / 32;
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (int64_t)rows * KB32) return;
  const int r = (int)(idx / KB32), b = (int)(idx % KB32);
  const uint4* xp = reinterpret_cast<const uint4*>(x + (int64_t)r * ldx + b * 32);
  float s = 0.f;
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    const uint4 v = __ldg(xp + c);
    const uint32_t w4[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = unpack_bf16x2(w4[i]);
      s += f.x + f.y;
    }
  }
  out[idx] = s;
}

cudaError_t launch_block_sums(const void* x, int rows, int K, int ldx, float* out, cudaStream_t s) {
  if (rows == 0) return cudaSuccess;
  const int64_t n = (int64_t)rows * (K / 32);
  block_sums_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(reinterpret_cast<const __nv_bfloat16*>(x), rows, K,
                                                                 ldx, out);
  return cudaGetLastError();
}


// ---------------------------------------------------------------------------------------
// v4: TMA-fed GEMV.  A row tile's packed nibbles (K/64 x 512 B) and scales (K/64 x 128 B)
// are contiguous in the tiled layout, so one elected lane per warp streams them with
// cp.async.bulk in 8-group chunks (5 KB) into a 3-stage per-warp ring.  Bytes in flight
// no longer cost registers (15 KB per warp), so a warp streams a whole K without split-K.
// Same fragment math and epilogues as v2.
template <int NT>
struct GemvV4 {
  static constexpr int WARPS = 4;
  static constexpr int CG = 8;      // groups per chunk
  static constexpr int STAGES = 3;
  static constexpr int QB = CG * 512, SB = CG * 128;
  static constexpr int STAGE_BYTES = QB + SB;
  static constexpr size_t SMEM = (size_t)WARPS * STAGES * STAGE_BYTES;
};

__device__ __forceinline__ uint32_t smem_addr_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

template <int NT>
__global__ void __launch_bounds__(128) q4_gemv4_kernel(GemvArgs a) {
  using C = GemvV4<NT>;
  extern __shared__ __align__(128) uint8_t gsm4[];
  __shared__ __align__(8) uint64_t bars[C::WARPS][C::STAGES];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int g = lane >> 2, t = lane & 3;
  const int e = blockIdx.y;
  const int p0 = a.tok_off[e];
  // a null weight pointer marks an expert computed elsewhere (the host CPU): its pairs are skipped
  const int cnt = a.qw_ptrs[e] ? a.tok_off[e + 1] - p0 : 0;
  const int n_units = a.N / 16;
  const int unit = blockIdx.x * C::WARPS + warp;
  const int KG = a.K >> 6;
  const int n_chunks = (KG + C::CG - 1) / C::CG;
  uint8_t* ring = gsm4 + warp * C::STAGES * C::STAGE_BYTES;
  const bool active = cnt > 0 && unit < n_units;
  if (lane == 0) {
    for (int s = 0; s < C::STAGES; ++s)
      asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;\n" ::"r"(smem_addr_u32(&bars[warp][s])));
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
  }
  __syncwarp();
  if (active) {
    const uint8_t* qw = reinterpret_cast<const uint8_t*>(a.qw_ptrs[e]) + (int64_t)unit * KG * 512;
    const uint8_t* smw = reinterpret_cast<const uint8_t*>(a.sm_ptrs[e]) + (int64_t)unit * KG * 128;
    const __nv_bfloat16* xbase = reinterpret_cast<const __nv_bfloat16*>(a.x);
    const uint32_t ones[4] = {0x3F803F80u, 0x3F803F80u, 0x3F803F80u, 0x3F803F80u};
    uint32_t phase_bits = 0;  // bit s: parity to wait for on stage s
    auto issue = [&](int c) {
      if (lane == 0 && c < n_chunks) {
        const int s = c % C::STAGES;
        const int ng = min(C::CG, KG - c * C::CG);
        uint64_t* bar = &bars[warp][s];
        const uint32_t bytes = (uint32_t)ng * 640u;
        asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(smem_addr_u32(bar)),
                     "r"(bytes)
                     : "memory");
        uint8_t* dst = ring + s * C::STAGE_BYTES;
        asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n" ::"r"(
                         smem_addr_u32(dst)),
                     "l"(qw + (int64_t)c * C::CG * 512), "r"((uint32_t)ng * 512u), "r"(smem_addr_u32(bar))
                     : "memory");
        asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n" ::"r"(
                         smem_addr_u32(dst + C::QB)),
                     "l"(smw + (int64_t)c * C::CG * 128), "r"((uint32_t)ng * 128u), "r"(smem_addr_u32(bar))
                     : "memory");
      }
    };
    for (int c0 = 0; c0 < cnt; c0 += NT * 8) {
      const int ccount = min(cnt - c0, NT * 8);
      const int ntc = (ccount + 7) >> 3;
      const __nv_bfloat16* xr[NT];
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        const int j = min(nt * 8 + g, ccount - 1);
        const int pp = p0 + c0 + j;
        const int row = a.tok_idx ? a.tok_idx[pp] : pp;
        xr[nt] = xbase + (int64_t)row * a.ldx + 2 * t;
      }
      float acc[NT][4];
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int i = 0; i < 4; ++i) acc[nt][i] = 0.f;
#pragma unroll
      for (int i = 0; i < C::STAGES; ++i) issue(i);
      bool ok = true;
      for (int c = 0; c < n_chunks && ok; ++c) {
        const int s = c % C::STAGES;
        const uint32_t par = (phase_bits >> s) & 1u;
        {  // bounded wait on this chunk's bytes
          uint32_t done = 0;
          const uint64_t t0 = globaltimer_ns();
          while (true) {
            asm volatile(
                "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
                : "=r"(done)
                : "r"(smem_addr_u32(&bars[warp][s])), "r"(par)
                : "memory");
            if (done) break;
            if (globaltimer_ns() - t0 > 2000000000ull) {
              if (a.status) atomicOr(a.status, 1 << 5);
              ok = false;
              break;
            }
          }
        }
        if (!ok) break;
        phase_bits ^= 1u << s;
        const uint8_t* stq = ring + s * C::STAGE_BYTES;
        const uint8_t* sts = stq + C::QB;
        const int ng = min(C::CG, KG - c * C::CG);
        for (int gi = 0; gi < ng; ++gi) {
          const int kg = c * C::CG + gi;
          const uint4 q = *reinterpret_cast<const uint4*>(stq + gi * 512 + lane * 16);
          const uint2 slo = *reinterpret_cast<const uint2*>(sts + gi * 128 + g * 8);
          const uint2 shi = *reinterpret_cast<const uint2*>(sts + gi * 128 + (g + 8) * 8);
#pragma unroll
          for (int b = 0; b < 2; ++b) {
            const uint32_t w0 = b ? q.z : q.x;
            const uint32_t w1 = b ? q.w : q.y;
            uint32_t af[2][4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              af[0][j] = lop3_and_or(w0 >> (4 * j), 0x000F000Fu, 0x43004300u);
              af[1][j] = lop3_and_or(w1 >> (4 * j), 0x000F000Fu, 0x43004300u);
            }
            const uint32_t vlo = b ? slo.y : slo.x, vhi = b ? shi.y : shi.x;
            const half2 hl = *reinterpret_cast<const half2*>(&vlo);
            const half2 hh = *reinterpret_cast<const half2*>(&vhi);
            const float dlo = __low2float(hl), dhi = __low2float(hh);
            const float mlo = fmaf(-128.f, dlo, __high2float(hl)), mhi = fmaf(-128.f, dhi, __high2float(hh));
            const int k0 = kg * 64 + b * 32;
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
              if (nt < ntc) {
                uint32_t bf[2][2];
                bf[0][0] = __ldg(reinterpret_cast<const uint32_t*>(xr[nt] + k0));
                bf[0][1] = __ldg(reinterpret_cast<const uint32_t*>(xr[nt] + k0 + 8));
                bf[1][0] = __ldg(reinterpret_cast<const uint32_t*>(xr[nt] + k0 + 16));
                bf[1][1] = __ldg(reinterpret_cast<const uint32_t*>(xr[nt] + k0 + 24));
                float xs[4] = {0.f, 0.f, 0.f, 0.f}, blk[4] = {0.f, 0.f, 0.f, 0.f};
                mma_bf16_16816(xs, ones, bf[0], xs);
                mma_bf16_16816(xs, ones, bf[1], xs);
                mma_bf16_16816(blk, af[0], bf[0], blk);
                mma_bf16_16816(blk, af[1], bf[1], blk);
                acc[nt][0] += fmaf(dlo, blk[0], mlo * xs[0]);
                acc[nt][1] += fmaf(dlo, blk[1], mlo * xs[1]);
                acc[nt][2] += fmaf(dhi, blk[2], mhi * xs[2]);
                acc[nt][3] += fmaf(dhi, blk[3], mhi * xs[3]);
              }
            }
          }
        }
        // the stage's generic-proxy reads are ordered before its refill by the bulk copy
        asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
        __syncwarp();
        issue(c + C::STAGES);
      }
      if (!ok) break;
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
        for (int hf = 0; hf < 2; ++hf) {
          const int j = nt * 8 + 2 * t + hf;
          if (j >= ccount) continue;
          const int p = p0 + c0 + j;
          if (a.mode == GEMV_SWIGLU) {
            reinterpret_cast<__nv_bfloat16*>(a.out)[(int64_t)p * (a.N / 2) + unit * 8 + g] =
                f2bf(silu(acc[nt][hf]) * acc[nt][2 + hf]);
          } else {
            gemv_store(a, p, unit * 16 + g, acc[nt][hf]);
            gemv_store(a, p, unit * 16 + g + 8, acc[nt][2 + hf]);
          }
        }
      }
    }
  }
  if (a.done_ctr != nullptr) {
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x == 0) {
      const unsigned total = gridDim.x * gridDim.y;
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

template <int NT>
static cudaError_t launch_v4(const GemvArgs& a, cudaStream_t s) {
  using C = GemvV4<NT>;
  const int units = a.N / 16;
  const int gx = (units + C::WARPS - 1) / C::WARPS;
  static bool set = false;
  if (!set) {
    cudaError_t e = cudaFuncSetAttribute(q4_gemv4_kernel<NT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)C::SMEM);
    if (e != cudaSuccess) return e;
    set = true;
  }
  dim3 grid((unsigned)gx, (unsigned)a.E);
  q4_gemv4_kernel<NT><<<grid, C::WARPS * 32, C::SMEM, s>>>(a);
  return cudaGetLastError();
}


// ---------------------------------------------------------------------------------------
// v5 (dense layers, 1..64 tokens): CTA = 4 warps = 64 output rows x one K slice of KR
// 64-column groups.  The activations of the slice are staged once per CTA in shared memory
// (cp.async) with their 32-column block sums, and shared by the 4 warps (B fragments by
// ldmatrix); each warp issues all KR of its packed-weight loads up front.  NT (8-token
// tiles) and KR are compile-time, so the main loop is straight-line code whose NT
// independent MMA chains interleave.  K is split over gridDim.y CTAs; partial sums go to an
// f32 workspace and the last CTA of a row block (arrival counter) adds them in slice order
// (deterministic) and runs the epilogue.
template <int NT, int KR>
__global__ void __launch_bounds__(128, 4) q4_gemv5_kernel(GemvArgs a, float* __restrict__ ws,
                                                       unsigned* __restrict__ counters) {
  extern __shared__ __align__(16) uint8_t gsm5[];
  constexpr int XS = KR * 64 + 8;  // smem row stride (elements), padded against bank conflicts
  constexpr int TT = NT * 8;       // token rows staged (rows past T repeat the last token)
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int g = lane >> 2, t = lane & 3;
  const int KG = a.K >> 6;
  const int KS = gridDim.y;
  const int ks = blockIdx.y;
  const int rb = blockIdx.x;
  const int tile = rb * 4 + warp;  // 16-row tile of this warp
  const int T = min(a.tok_off[1] - a.tok_off[0], TT);
  __nv_bfloat16* xs_sm = reinterpret_cast<__nv_bfloat16*>(gsm5);
  float* xsum_sm = reinterpret_cast<float*>(gsm5 + (size_t)TT * XS * 2);  // [KR*2][TT]
  __shared__ int s_last;
  const uint4* qw = reinterpret_cast<const uint4*>(a.qw_ptrs[0]);
  const uint2* smw = reinterpret_cast<const uint2*>(a.sm_ptrs[0]);
  const bool active = tile < a.N / 16;

  // 1) weights of this warp's slice: all KR loads in flight at once
  uint4 q[KR];
  uint2 slo[KR], shi[KR];
  if (active) {
    const int64_t tk0 = (int64_t)tile * KG + ks * KR;
#pragma unroll
    for (int i = 0; i < KR; ++i) {
      q[i] = __ldcs(qw + (tk0 + i) * 32 + lane);
      slo[i] = __ldcs(smw + (tk0 + i) * 16 + g);
      shi[i] = __ldcs(smw + (tk0 + i) * 16 + g + 8);
    }
  }
  // 2) activations of the slice into shared memory
  {
    const __nv_bfloat16* xb = reinterpret_cast<const __nv_bfloat16*>(a.x) + (int64_t)ks * KR * 64;
    constexpr int CPR = KR * 8;  // 16-byte chunks per row
#pragma unroll 4
    for (int idx = threadIdx.x; idx < TT * CPR; idx += 128) {
      const int j = idx / CPR, c = idx % CPR;
      const int row = min(j, T - 1);
      const uint4* src = reinterpret_cast<const uint4*>(xb + (int64_t)row * a.ldx) + c;
      const uint32_t dst = (uint32_t)__cvta_generic_to_shared(xs_sm + j * XS + c * 8);
      asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(dst), "l"(src));
    }
    asm volatile("cp.async.commit_group;\n" ::);
    asm volatile("cp.async.wait_group 0;\n" ::);
  }
  __syncthreads();
  // 32-column block sums (the min term of every weight row uses them): xsum_sm[block][token]
  for (int idx = threadIdx.x; idx < KR * 2 * TT; idx += 128) {
    const int j = idx % TT, blk = idx / TT;
    const uint4* src = reinterpret_cast<const uint4*>(xs_sm + j * XS + blk * 32);
    float sum = 0.f;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const uint4 v = src[c];
      const uint32_t u[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 f = unpack_bf16x2(u[e]);
        sum += f.x + f.y;
      }
    }
    xsum_sm[blk * TT + j] = sum;
  }
  __syncthreads();
  float acc[NT][4];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt)
#pragma unroll
    for (int i = 0; i < 4; ++i) acc[nt][i] = 0.f;
  if (active) {
    // ldmatrix row address of this lane: matrix (lane / 8) = k offset 8 * (lane / 8),
    // row (lane % 8) = token inside the 8-token tile
    const uint32_t lds_base = (uint32_t)__cvta_generic_to_shared(xs_sm + (lane & 7) * XS + (lane >> 3) * 8);
#pragma unroll
    for (int i = 0; i < KR; ++i) {
#pragma unroll
      for (int b = 0; b < 2; ++b) {
        const uint32_t w0 = b ? q[i].z : q[i].x;
        const uint32_t w1 = b ? q[i].w : q[i].y;
        uint32_t af[2][4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          af[0][j] = lop3_and_or(w0 >> (4 * j), 0x000F000Fu, 0x43004300u);
          af[1][j] = lop3_and_or(w1 >> (4 * j), 0x000F000Fu, 0x43004300u);
        }
        const uint32_t vlo = b ? slo[i].y : slo[i].x, vhi = b ? shi[i].y : shi[i].x;
        const half2 hl = *reinterpret_cast<const half2*>(&vlo);
        const half2 hh = *reinterpret_cast<const half2*>(&vhi);
        const float dlo = __low2float(hl), dhi = __low2float(hh);
        const float mlo = fmaf(-128.f, dlo, __high2float(hl)), mhi = fmaf(-128.f, dhi, __high2float(hh));
        const float* xsb = xsum_sm + (i * 2 + b) * TT + 2 * t;
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          uint32_t bf[2][2];
          asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
                       : "=r"(bf[0][0]), "=r"(bf[0][1]), "=r"(bf[1][0]), "=r"(bf[1][1])
                       : "r"(lds_base + (uint32_t)((nt * 8 * XS + i * 64 + b * 32) * 2)));
          float blk[4] = {0.f, 0.f, 0.f, 0.f};
          mma_bf16_16816(blk, af[0], bf[0], blk);
          mma_bf16_16816(blk, af[1], bf[1], blk);
          const float2 xs = *reinterpret_cast<const float2*>(xsb + nt * 8);
          acc[nt][0] += fmaf(dlo, blk[0], mlo * xs.x);
          acc[nt][1] += fmaf(dlo, blk[1], mlo * xs.y);
          acc[nt][2] += fmaf(dhi, blk[2], mhi * xs.x);
          acc[nt][3] += fmaf(dhi, blk[3], mhi * xs.y);
        }
      }
    }
  }
  // 3) split-K partials -> workspace [ks][token][N]; the last slice CTA reduces in order
  if (KS == 1) {
    if (active) {
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int hf = 0; hf < 2; ++hf) {
          const int p = nt * 8 + 2 * t + hf;
          if (p >= T) continue;
          if (a.mode == GEMV_SWIGLU) {
            reinterpret_cast<__nv_bfloat16*>(a.out)[(int64_t)p * (a.N / 2) + tile * 8 + g] =
                f2bf(silu(acc[nt][hf]) * acc[nt][2 + hf]);
          } else {
            gemv_store(a, p, tile * 16 + g, acc[nt][hf]);
            gemv_store(a, p, tile * 16 + g + 8, acc[nt][2 + hf]);
          }
        }
    }
    return;
  }
  if (active) {
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int hf = 0; hf < 2; ++hf) {
        const int j = nt * 8 + 2 * t + hf;
        if (j >= T) continue;
        float* w = ws + ((int64_t)ks * TT + j) * a.N;
        w[tile * 16 + g] = acc[nt][hf];
        w[tile * 16 + g + 8] = acc[nt][2 + hf];
      }
  }
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    const unsigned prev = atomicAdd(&counters[rb], 1u);
    s_last = (prev == (unsigned)KS - 1);
    if (s_last) counters[rb] = 0u;
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  // 64 rows x T tokens, summed over the slices in slice order (deterministic).  A thread owns
  // 4 consecutive rows of one token (float4) and issues the loads of up to 8 slices before
  // adding any: the reduction is bound by L2 latency, not bandwidth.
  const bool glu = a.mode == GEMV_SWIGLU;
  for (int idx = threadIdx.x; idx < 16 * T; idx += 128) {
    const int c4 = idx & 15, j = idx >> 4;
    if (glu && (c4 & 2)) continue;  // SwiGLU: rows 8..15 of a 16-row tile are the up halves
    const int n = rb * 64 + c4 * 4;
    const float* src = ws + (int64_t)j * a.N + n;
    const int64_t sstride = (int64_t)TT * a.N;
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f), u = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int s0 = 0; s0 < KS; s0 += 8) {
      float4 bv[8], bu[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        if (s0 + i < KS) {
          bv[i] = __ldcg(reinterpret_cast<const float4*>(src + (s0 + i) * sstride));
          if (glu) bu[i] = __ldcg(reinterpret_cast<const float4*>(src + (s0 + i) * sstride + 8));
        }
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        if (s0 + i < KS) {
          v.x += bv[i].x; v.y += bv[i].y; v.z += bv[i].z; v.w += bv[i].w;
          if (glu) { u.x += bu[i].x; u.y += bu[i].y; u.z += bu[i].z; u.w += bu[i].w; }
        }
      }
    }
    if (glu) {
      __nv_bfloat16* o = reinterpret_cast<__nv_bfloat16*>(a.out) + (int64_t)j * (a.N / 2) + (n >> 4) * 8 + (n & 7);
      o[0] = f2bf(silu(v.x) * u.x);
      o[1] = f2bf(silu(v.y) * u.y);
      o[2] = f2bf(silu(v.z) * u.z);
      o[3] = f2bf(silu(v.w) * u.w);
    } else {
      gemv_store(a, j, n, v.x);
      gemv_store(a, j, n + 1, v.y);
      gemv_store(a, j, n + 2, v.z);
      gemv_store(a, j, n + 3, v.w);
    }
  }
}

template <int NT, int KR>
static cudaError_t launch_v5(const GemvArgs& a, int ksplit, float* ws, unsigned* counters, cudaStream_t s) {
  constexpr size_t smem = (size_t)NT * 8 * (KR * 64 + 8) * 2 + (size_t)KR * 2 * NT * 8 * 4;
  static bool set = false;
  if (smem > 48 * 1024 && !set) {
    cudaError_t e = cudaFuncSetAttribute(q4_gemv5_kernel<NT, KR>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)smem);
    if (e != cudaSuccess) return e;
    set = true;
  }
  dim3 grid((unsigned)((a.N / 16 + 3) / 4), (unsigned)ksplit);
  q4_gemv5_kernel<NT, KR><<<grid, 128, smem, s>>>(a, ws, counters);
  return cudaGetLastError();
}

template <int NT>
static cudaError_t launch_v5_kr(const GemvArgs& a, int kr, float* ws, unsigned* counters, cudaStream_t s) {
  const int ksplit = (a.K >> 6) / kr;
  if (kr == 8) return launch_v5<NT, 8>(a, ksplit, ws, counters, s);
  if (kr == 4) return launch_v5<NT, 4>(a, ksplit, ws, counters, s);
  return launch_v5<NT, 2>(a, ksplit, ws, counters, s);
}

// Split of the dense decode GEMV: 8-token tiles (nt), 64-column groups per K slice (kr) and
// the workspace it needs (floats).  kr is the largest of 8/4/2 dividing K/64, halved while the
// grid is under ~4 CTAs per SM.  Returns false when no split fits (K/64 odd, or more than 64 rows).
bool q4_gemv_dense_plan(int N, int K, int rows, int* nt_out, int* kr_out, size_t* ws_floats_out) {
  if (rows < 1 || rows > 64 || N % 64 || K % 128) return false;
  const int nt = rows <= 8 ? 1 : (rows <= 16 ? 2 : (rows <= 32 ? 4 : 8));
  const int KG = K >> 6;
  int kr = KG % 8 == 0 ? 8 : (KG % 4 == 0 ? 4 : 2);
  const long row_blocks = (N / 16 + 3) / 4;
  while (kr > 2 && row_blocks * (KG / kr) < 148L * 4) kr /= 2;
  const int ksplit = KG / kr;
  *nt_out = nt;
  *kr_out = kr;
  *ws_floats_out = ksplit > 1 ? (size_t)ksplit * nt * 8 * (size_t)N : 0;
  int nt6, ks6;
  size_t ws6;
  if (q4_gemv6_plan(N, K, rows, &nt6, &ks6, &ws6) && ws6 > *ws_floats_out) *ws_floats_out = ws6;  // either kernel fits
  return true;
}

// Dense decode GEMV (one weight matrix, 1..64 rows of x).  ws: f32 workspace of at least
// the planned size; counters: N/64 zeroed unsigned ints (left zeroed on exit).
cudaError_t launch_q4_gemv_dense(const GemvArgs& a, float* ws, unsigned* counters, size_t ws_floats,
                                 cudaStream_t s) {
  // Streaming v6 for large matrices (>= 64M weights: many row blocks, long K), one-slice v5
  // otherwise (measured on B200 at the Qwen3-235B and Llama-3-70B decode shapes).
  // SYN_DENSE_KERNEL=5/6 forces one of them.
  static int kernel = -1;
  if (kernel < 0) {
    const char* v = getenv("SYN_DENSE_KERNEL");
    kernel = v ? atoi(v) : 0;
  }
  const bool big = (long long)a.N * a.K >= (64ll << 20);
  if (a.K % 256 == 0 && (kernel == 6 || (kernel == 0 && big)))
    return launch_q4_gemv_dense6(a, ws, counters, ws_floats, s);
  int nt, kr;
  size_t need;
  if (!q4_gemv_dense_plan(a.N, a.K, a.nt_hint * 8 < 64 ? a.nt_hint * 8 : 64, &nt, &kr, &need))
    return cudaErrorInvalidValue;
  if (need > ws_floats) return cudaErrorInvalidValue;
  if (nt == 1) return launch_v5_kr<1>(a, kr, ws, counters, s);
  if (nt == 2) return launch_v5_kr<2>(a, kr, ws, counters, s);
  if (nt == 4) return launch_v5_kr<4>(a, kr, ws, counters, s);
  return launch_v5_kr<8>(a, kr, ws, counters, s);
}

// ---------------------------------------------------------------------------------------
// v6 (dense layers, 1..64 tokens, large matrices): CTA = 8 warps = 128 output rows that
// stream their K range in rounds of G 64-column groups through an ST-stage cp.async ring in
// shared memory: each stage holds the round's activation chunk (shared by the 8 warps) and
// the 8 warps' packed weights and scales, so ST-1 rounds of weights are always in flight
// while one is computed.  The round's 32-column block sums are computed once per CTA.  K is
// split over gridDim.y CTAs only when the row blocks alone do not fill the GPU; partials
// then go through the f32 workspace and the last CTA of a row block reduces in slice order.
template <int NT, int G, int ST>
__global__ void __launch_bounds__(256, 1) q4_gemv6_kernel(GemvArgs a, float* __restrict__ ws,
                                                       unsigned* __restrict__ counters, int rounds) {
  constexpr int TT = NT * 8;
  constexpr int XS = G * 64 + 8;          // x row stride in smem (elements), padded
  constexpr int XB = TT * XS * 2;         // x bytes per stage
  constexpr int WB = 8 * G * 512;         // packed nibbles per stage (8 warps)
  constexpr int SB = 8 * G * 128;         // scale/min pairs per stage
  constexpr int STB = XB + WB + SB;
  extern __shared__ __align__(16) uint8_t sm6[];
  float* xsum = reinterpret_cast<float*>(sm6 + (size_t)ST * STB);  // [G*2][TT]
  __shared__ int s_last;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int g = lane >> 2, t = lane & 3;
  const int KG = a.K >> 6;
  const int KS = gridDim.y, ks = blockIdx.y, rb = blockIdx.x;
  const int tile = rb * 8 + warp;
  const bool active = tile < a.N / 16;
  const int T = min(a.tok_off[1] - a.tok_off[0], TT);
  const int kg_first = ks * rounds * G;
  const uint8_t* qb = reinterpret_cast<const uint8_t*>(a.qw_ptrs[0]);
  const uint8_t* sb = reinterpret_cast<const uint8_t*>(a.sm_ptrs[0]);
  const __nv_bfloat16* xg = reinterpret_cast<const __nv_bfloat16*>(a.x);

  auto issue = [&](int r) {
    uint8_t* st = sm6 + (size_t)(r % ST) * STB;
    const int kg0 = kg_first + r * G;
    for (int idx = threadIdx.x; idx < TT * G * 8; idx += 256) {
      const int j = idx / (G * 8), c = idx % (G * 8);
      const int row = min(j, T - 1);
      const void* src = xg + (int64_t)row * a.ldx + kg0 * 64 + c * 8;
      const uint32_t dst = (uint32_t)__cvta_generic_to_shared(st + (j * XS + c * 8) * 2);
      asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(dst), "l"(src));
    }
    if (active) {
      const int64_t tk = (int64_t)tile * KG + kg0;
#pragma unroll
      for (int i = 0; i < G; ++i) {
        const uint32_t dst = (uint32_t)__cvta_generic_to_shared(st + XB + (warp * G + i) * 512 + lane * 16);
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(dst), "l"(qb + (tk + i) * 512 + lane * 16));
      }
      if (lane < 8 * G) {
        const uint32_t dst = (uint32_t)__cvta_generic_to_shared(st + XB + WB + warp * G * 128 + lane * 16);
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(dst), "l"(sb + tk * 128 + lane * 16));
      }
    }
    asm volatile("cp.async.commit_group;\n" ::);
  };

#pragma unroll
  for (int r = 0; r < ST - 1; ++r) {
    if (r < rounds) issue(r);
    else asm volatile("cp.async.commit_group;\n" ::);
  }
  float acc[NT][4];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt)
#pragma unroll
    for (int i = 0; i < 4; ++i) acc[nt][i] = 0.f;

  for (int r = 0; r < rounds; ++r) {
    if (r + ST - 1 < rounds) issue(r + ST - 1);
    else asm volatile("cp.async.commit_group;\n" ::);
    asm volatile("cp.async.wait_group %0;\n" ::"n"(ST - 1));
    __syncthreads();
    const uint8_t* st = sm6 + (size_t)(r % ST) * STB;
    const __nv_bfloat16* xs_sm = reinterpret_cast<const __nv_bfloat16*>(st);
    for (int idx = threadIdx.x; idx < G * 2 * TT; idx += 256) {
      const int j = idx % TT, blk = idx / TT;
      const uint4* src = reinterpret_cast<const uint4*>(xs_sm + j * XS + blk * 32);
      float sum = 0.f;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const uint4 v = src[c];
        const uint32_t u[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 f = unpack_bf16x2(u[e]);
          sum += f.x + f.y;
        }
      }
      xsum[blk * TT + j] = sum;
    }
    __syncthreads();
    if (active) {
      const uint32_t lds_base =
          (uint32_t)__cvta_generic_to_shared(xs_sm + (lane & 7) * XS + (lane >> 3) * 8);
#pragma unroll
      for (int i = 0; i < G; ++i) {
        const uint4 q = *reinterpret_cast<const uint4*>(st + XB + (warp * G + i) * 512 + lane * 16);
        const uint2 slo = *reinterpret_cast<const uint2*>(st + XB + WB + (warp * G + i) * 128 + g * 8);
        const uint2 shi = *reinterpret_cast<const uint2*>(st + XB + WB + (warp * G + i) * 128 + (g + 8) * 8);
#pragma unroll
        for (int b = 0; b < 2; ++b) {
          const uint32_t w0 = b ? q.z : q.x;
          const uint32_t w1 = b ? q.w : q.y;
          uint32_t af[2][4];
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            af[0][j] = lop3_and_or(w0 >> (4 * j), 0x000F000Fu, 0x43004300u);
            af[1][j] = lop3_and_or(w1 >> (4 * j), 0x000F000Fu, 0x43004300u);
          }
          const uint32_t vlo = b ? slo.y : slo.x, vhi = b ? shi.y : shi.x;
          const half2 hl = *reinterpret_cast<const half2*>(&vlo);
          const half2 hh = *reinterpret_cast<const half2*>(&vhi);
          const float dlo = __low2float(hl), dhi = __low2float(hh);
          const float mlo = fmaf(-128.f, dlo, __high2float(hl)), mhi = fmaf(-128.f, dhi, __high2float(hh));
          const float* xsb = xsum + (i * 2 + b) * TT + 2 * t;
#pragma unroll
          for (int nt = 0; nt < NT; ++nt) {
            uint32_t bf[2][2];
            asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
                         : "=r"(bf[0][0]), "=r"(bf[0][1]), "=r"(bf[1][0]), "=r"(bf[1][1])
                         : "r"(lds_base + (uint32_t)((nt * 8 * XS + i * 64 + b * 32) * 2)));
            float blk[4] = {0.f, 0.f, 0.f, 0.f};
            mma_bf16_16816(blk, af[0], bf[0], blk);
            mma_bf16_16816(blk, af[1], bf[1], blk);
            const float2 xv = *reinterpret_cast<const float2*>(xsb + nt * 8);
            acc[nt][0] += fmaf(dlo, blk[0], mlo * xv.x);
            acc[nt][1] += fmaf(dlo, blk[1], mlo * xv.y);
            acc[nt][2] += fmaf(dhi, blk[2], mhi * xv.x);
            acc[nt][3] += fmaf(dhi, blk[3], mhi * xv.y);
          }
        }
      }
    }
    __syncthreads();  // the stage is refilled by the next round's issue
  }
  asm volatile("cp.async.wait_group 0;\n" ::);
  // ---- epilogue ----
  if (KS == 1) {
    if (active) {
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int hf = 0; hf < 2; ++hf) {
          const int p = nt * 8 + 2 * t + hf;
          if (p >= T) continue;
          if (a.mode == GEMV_SWIGLU) {
            reinterpret_cast<__nv_bfloat16*>(a.out)[(int64_t)p * (a.N / 2) + tile * 8 + g] =
                f2bf(silu(acc[nt][hf]) * acc[nt][2 + hf]);
          } else {
            gemv_store(a, p, tile * 16 + g, acc[nt][hf]);
            gemv_store(a, p, tile * 16 + g + 8, acc[nt][2 + hf]);
          }
        }
    }
    return;
  }
  if (active) {
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int hf = 0; hf < 2; ++hf) {
        const int j = nt * 8 + 2 * t + hf;
        if (j >= T) continue;
        float* w = ws + ((int64_t)ks * TT + j) * a.N;
        w[tile * 16 + g] = acc[nt][hf];
        w[tile * 16 + g + 8] = acc[nt][2 + hf];
      }
  }
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    const unsigned prev = atomicAdd(&counters[rb], 1u);
    s_last = (prev == (unsigned)KS - 1);
    if (s_last) counters[rb] = 0u;
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  const bool glu = a.mode == GEMV_SWIGLU;
  const int nrows = min(128, a.N - rb * 128);
  for (int idx = threadIdx.x; idx < (nrows / 4) * T; idx += 256) {
    const int c4 = idx % (nrows / 4), j = idx / (nrows / 4);
    if (glu && (c4 & 2)) continue;  // SwiGLU: rows 8..15 of a 16-row tile are the up halves
    const int n = rb * 128 + c4 * 4;
    const float* src = ws + (int64_t)j * a.N + n;
    const int64_t sstride = (int64_t)TT * a.N;
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f), u = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int s0 = 0; s0 < KS; s0 += 8) {
      float4 bv[8], bu[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        if (s0 + i < KS) {
          bv[i] = __ldcg(reinterpret_cast<const float4*>(src + (s0 + i) * sstride));
          if (glu) bu[i] = __ldcg(reinterpret_cast<const float4*>(src + (s0 + i) * sstride + 8));
        }
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        if (s0 + i < KS) {
          v.x += bv[i].x; v.y += bv[i].y; v.z += bv[i].z; v.w += bv[i].w;
          if (glu) { u.x += bu[i].x; u.y += bu[i].y; u.z += bu[i].z; u.w += bu[i].w; }
        }
      }
    }
    if (glu) {
      __nv_bfloat16* o = reinterpret_cast<__nv_bfloat16*>(a.out) + (int64_t)j * (a.N / 2) + (n >> 4) * 8 + (n & 7);
      o[0] = f2bf(silu(v.x) * u.x);
      o[1] = f2bf(silu(v.y) * u.y);
      o[2] = f2bf(silu(v.z) * u.z);
      o[3] = f2bf(silu(v.w) * u.w);
    } else {
      gemv_store(a, j, n, v.x);
      gemv_store(a, j, n + 1, v.y);
      gemv_store(a, j, n + 2, v.z);
      gemv_store(a, j, n + 3, v.w);
    }
  }
}

template <int NT>
static cudaError_t launch_v6(const GemvArgs& a, int ksplit, float* ws, unsigned* counters, cudaStream_t s) {
  constexpr int G = 4, ST = 4;
  constexpr size_t smem = (size_t)ST * (NT * 8 * (G * 64 + 8) * 2 + 8 * G * 512 + 8 * G * 128) +
                          (size_t)G * 2 * NT * 8 * 4;
  static bool set = false;
  if (!set) {
    cudaError_t e = cudaFuncSetAttribute(q4_gemv6_kernel<NT, G, ST>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)smem);
    if (e != cudaSuccess) return e;
    set = true;
  }
  const int rounds = (a.K / 64) / G / ksplit;
  dim3 grid((unsigned)((a.N / 16 + 7) / 8), (unsigned)ksplit);
  q4_gemv6_kernel<NT, G, ST><<<grid, 256, smem, s>>>(a, ws, counters, rounds);
  return cudaGetLastError();
}

// Split of the streaming dense GEMV: K slices (dividing the K/256 rounds) until the row
// blocks x slices reach ~2 CTAs per SM; workspace floats as for v5.
bool q4_gemv6_plan(int N, int K, int rows, int* nt_out, int* ksplit_out, size_t* ws_floats_out) {
  if (rows < 1 || rows > 64 || N % 64 || K % 256) return false;
  const int nt = rows <= 8 ? 1 : (rows <= 16 ? 2 : (rows <= 32 ? 4 : 8));
  const int R = K / 256;
  const long rb = (N / 16 + 7) / 8;
  int ks = 1;
  for (int c = 1; c <= 8; ++c) {
    if (R % c) continue;
    ks = c;
    if (rb * c >= 296) break;
  }
  *nt_out = nt;
  *ksplit_out = ks;
  *ws_floats_out = ks > 1 ? (size_t)ks * nt * 8 * (size_t)N : 0;
  return true;
}

cudaError_t launch_q4_gemv_dense6(const GemvArgs& a, float* ws, unsigned* counters, size_t ws_floats,
                                  cudaStream_t s) {
  int nt, ks;
  size_t need;
  if (!q4_gemv6_plan(a.N, a.K, a.nt_hint * 8 < 64 ? a.nt_hint * 8 : 64, &nt, &ks, &need))
    return cudaErrorInvalidValue;
  if (need > ws_floats) return cudaErrorInvalidValue;
  if (nt == 1) return launch_v6<1>(a, ks, ws, counters, s);
  if (nt == 2) return launch_v6<2>(a, ks, ws, counters, s);
  if (nt == 4) return launch_v6<4>(a, ks, ws, counters, s);
  return launch_v6<8>(a, ks, ws, counters, s);
}

cudaError_t launch_q4_gemv(const GemvArgs& a, cudaStream_t s) {
  // Tile shapes measured on B200 (kernel microbenchmarks at the Qwen3-235B decode shapes):
  //  * one token tile (MoE experts, token groups of dense layers): register pipeline, U=4,
  //    eight 4-warp CTAs per SM (v2<1,1,1,4,8>), ~60% of HBM bandwidth on expert streams;
  //  * few row tiles (dense layers): split K over the warps of a CTA.
  // An explicit variant (a.variant or SYN_GEMV_VARIANT) overrides the choice.
  const int nt = a.nt_hint <= 1 ? 1 : (a.nt_hint <= 2 ? 2 : 4);
  static int env_variant = -1;
  if (env_variant < 0) {
    const char* v = getenv("SYN_GEMV_VARIANT");
    env_variant = v ? atoi(v) : 0;
  }
  const int variant = a.variant ? a.variant : env_variant;
  if (variant == 4 && a.weights_in_vram) {
    if (nt == 1) return launch_v4<1>(a, s);
    if (nt == 2) return launch_v4<2>(a, s);
    return launch_v4<4>(a, s);
  }
  if (variant == 3) {
    if (nt == 1) return launch_v3<1, 1>(a, s);
    if (nt == 2) return launch_v3<1, 2>(a, s);
    return launch_v3<1, 4>(a, s);
  }
  if (nt == 1) {
    switch (variant) {
      case 21: return launch_v2<1, 1, 1, 8>(a, s);
      case 23: return launch_v2<1, 1, 1, 6, 6>(a, s);
      case 24: return launch_v2<1, 1, 1, 4, 10>(a, s);
      case 25: return launch_v2<1, 1, 1, 2, 12>(a, s);
      case 26: return launch_v2<1, 1, 1, 3, 10>(a, s);
      case 27: return launch_v2<1, 1, 8, 4, 1>(a, s);
      case 28: return launch_v2<1, 1, 4, 4, 2>(a, s);
      case 29: return launch_v2<1, 1, 2, 4, 4>(a, s);
      default: break;
    }
    const long units = (long)(a.N / 16) * a.E_active_hint;
    if (units < 148L * 8) return launch_v2<1, 1, 4, 4, 2>(a, s);  // few tiles: split K by 4
    return launch_v2<1, 1, 1, 4, 8>(a, s);
  }
  switch (variant) {
    case 11: return launch_v2<1, 4, 8, 2, 1>(a, s);
    case 12: return launch_v2<1, 4, 4, 2, 1>(a, s);
    case 13: return launch_v2<2, 4, 8, 2, 1>(a, s);
    case 14: return launch_v2<1, 4, 8, 8, 1>(a, s);
    default: break;
  }
  const bool r2 = a.N % 32 == 0;
  const long units = (long)(a.N / (16 * (r2 ? 2 : 1))) * a.E_active_hint;
  if (units < 148L * 16) {
    if (nt == 2) return r2 ? launch_v2<2, 2, 8>(a, s) : launch_v2<1, 2, 8>(a, s);
    return r2 ? launch_v2<2, 4, 8>(a, s) : launch_v2<1, 4, 8>(a, s);
  }
  if (nt == 2) return r2 ? launch_v3<2, 2>(a, s) : launch_v3<1, 2>(a, s);
  return r2 ? launch_v3<2, 4>(a, s) : launch_v3<1, 4>(a, s);
}

}  // namespace syn
