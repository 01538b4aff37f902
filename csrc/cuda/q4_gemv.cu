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
#include "syn/q4.h"
#include "sync.cuh"

namespace syn {

constexpr int GEMV_WARPS = 8;
constexpr int GEMV_NT = 4;  // up to 4 n-tiles of 8 tokens per pass

enum GemvMode : int {
  GEMV_STORE_BF16 = 0,   // out_bf16[p][n]
  GEMV_SWIGLU = 1,       // rows interleaved in 8-row gate/up chunks -> out_bf16[p][n/2]
  GEMV_SCALED_F32 = 2,   // out_f32[p][n] = route_w[p] * y
  GEMV_ADD_F32 = 3,      // out_f32[p][n] += y (residual stream kept in f32)
  GEMV_SCALED_F32_PTR = 4,  // ((float*)out_ptrs[p])[n] = route_w[p] * y (peer memory allowed)
  GEMV_STORE_F32 = 5,    // out_f32[p][n] = y (logits)
};

__global__ void __launch_bounds__(GEMV_WARPS * 32)
q4_gemv_kernel(GemvArgs a) {
  const int tile = blockIdx.x;
  const int e = blockIdx.y;
  const int p0 = a.tok_off[e];
  const int cnt = a.tok_off[e + 1] - p0;
  const uint4* __restrict__ qw = reinterpret_cast<const uint4*>(a.qw_ptrs[e]);
  const uint2* __restrict__ sm = reinterpret_cast<const uint2*>(a.sm_ptrs[e]);

  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int g = lane >> 2, t = lane & 3;
  const int KG = a.K >> 6;

  __shared__ float red[GEMV_WARPS][GEMV_NT][4][32];

  const uint32_t ones[4] = {0x3F803F80u, 0x3F803F80u, 0x3F803F80u, 0x3F803F80u};

  for (int c0 = 0; c0 < cnt; c0 += GEMV_NT * 8) {
    const int ccount = min(cnt - c0, GEMV_NT * 8);
    const int ntc = (ccount + 7) >> 3;
    // Row pointers for the B fragments: token column g of each n-tile.
    const __nv_bfloat16* xr[GEMV_NT];
    const __nv_bfloat16* xbase = reinterpret_cast<const __nv_bfloat16*>(a.x);
#pragma unroll
    for (int nt = 0; nt < GEMV_NT; ++nt) {
      int j = min(nt * 8 + g, ccount - 1);
      int p = p0 + c0 + j;
      int row = a.tok_idx ? a.tok_idx[p] : p;
      xr[nt] = xbase + (int64_t)row * a.ldx + 2 * t;
    }
    float acc[GEMV_NT][4];
#pragma unroll
    for (int nt = 0; nt < GEMV_NT; ++nt)
#pragma unroll
      for (int i = 0; i < 4; ++i) acc[nt][i] = 0.f;

    const uint4* qbase = qw + (int64_t)tile * KG * 32 + lane;
    const uint2* sbase = sm + (int64_t)tile * KG * 16;

#pragma unroll 2
    for (int kg = warp; kg < KG; kg += GEMV_WARPS) {
      const uint4 q = ldg_stream(qbase + (int64_t)kg * 32);
      const uint2 s_lo = __ldg(sbase + (int64_t)kg * 16 + g);      // row g: (d0,m0),(d1,m1)
      const uint2 s_hi = __ldg(sbase + (int64_t)kg * 16 + g + 8);  // row g+8
      const uint32_t qwords[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
      for (int b = 0; b < 2; ++b) {
        float blk[GEMV_NT][4], xs[GEMV_NT][4];
#pragma unroll
        for (int nt = 0; nt < GEMV_NT; ++nt)
#pragma unroll
          for (int i = 0; i < 4; ++i) { blk[nt][i] = 0.f; xs[nt][i] = 0.f; }
#pragma unroll
        for (int s = 0; s < 2; ++s) {
          const uint32_t w = qwords[b * 2 + s];
          uint32_t af[4];
          af[0] = lop3_and_or(w, 0x000F000Fu, 0x43004300u);
          af[1] = lop3_and_or(w >> 4, 0x000F000Fu, 0x43004300u);
          af[2] = lop3_and_or(w >> 8, 0x000F000Fu, 0x43004300u);
          af[3] = lop3_and_or(w >> 12, 0x000F000Fu, 0x43004300u);
          const int k0 = kg * 64 + b * 32 + s * 16;
#pragma unroll
          for (int nt = 0; nt < GEMV_NT; ++nt) {
            if (nt < ntc) {
              uint32_t bf[2];
              bf[0] = __ldg(reinterpret_cast<const uint32_t*>(xr[nt] + k0));
              bf[1] = __ldg(reinterpret_cast<const uint32_t*>(xr[nt] + k0 + 8));
              mma_bf16_16816(blk[nt], af, bf, blk[nt]);
              mma_bf16_16816(xs[nt], ones, bf, xs[nt]);
            }
          }
        }
        const half2 dm_lo = *reinterpret_cast<const half2*>(b ? &s_lo.y : &s_lo.x);
        const half2 dm_hi = *reinterpret_cast<const half2*>(b ? &s_hi.y : &s_hi.x);
        const float d_lo = __low2float(dm_lo), d_hi = __low2float(dm_hi);
        const float m_lo = fmaf(-128.f, d_lo, __high2float(dm_lo));
        const float m_hi = fmaf(-128.f, d_hi, __high2float(dm_hi));
#pragma unroll
        for (int nt = 0; nt < GEMV_NT; ++nt) {
          if (nt < ntc) {
            acc[nt][0] += fmaf(d_lo, blk[nt][0], m_lo * xs[nt][0]);
            acc[nt][1] += fmaf(d_lo, blk[nt][1], m_lo * xs[nt][1]);
            acc[nt][2] += fmaf(d_hi, blk[nt][2], m_hi * xs[nt][2]);
            acc[nt][3] += fmaf(d_hi, blk[nt][3], m_hi * xs[nt][3]);
          }
        }
      }
    }
    // Split-K reduction across warps (fixed order).
#pragma unroll
    for (int nt = 0; nt < GEMV_NT; ++nt)
#pragma unroll
      for (int i = 0; i < 4; ++i) red[warp][nt][i][lane] = acc[nt][i];
    __syncthreads();
    // 16 rows x (ntc*8) tokens; thread -> (row r, token j)
    if (a.mode != GEMV_SWIGLU)
    for (int idx = threadIdx.x; idx < 16 * ntc * 8; idx += blockDim.x) {
      const int r = idx & 15;
      const int j = idx >> 4;  // token inside this chunk
      if (j >= ccount) continue;
      const int nt = j >> 3, jj = j & 7;
      // Fragment position of (row r, token jj): lane = (r%8)*4 + jj/2, reg = (r/8)*2 + jj%2
      const int ln = (r & 7) * 4 + (jj >> 1);
      const int rg = (r >> 3) * 2 + (jj & 1);
      float v = 0.f;
#pragma unroll
      for (int w = 0; w < GEMV_WARPS; ++w) v += red[w][nt][rg][ln];
      const int p = p0 + c0 + j;
      const int n = tile * 16 + r;
      if (a.mode == GEMV_STORE_BF16) {
        reinterpret_cast<__nv_bfloat16*>(a.out)[(int64_t)p * a.N + n] = f2bf(v);
      } else if (a.mode == GEMV_SCALED_F32) {
        reinterpret_cast<float*>(a.out)[(int64_t)p * a.N + n] = a.route_w[p] * v;
      } else if (a.mode == GEMV_ADD_F32) {
        reinterpret_cast<float*>(a.out)[(int64_t)p * a.N + n] += v;
      } else if (a.mode == GEMV_STORE_F32) {
        reinterpret_cast<float*>(a.out)[(int64_t)p * a.N + n] = v;
      } else if (a.mode == GEMV_SCALED_F32_PTR) {
        reinterpret_cast<float*>(a.out_ptrs[p])[n] = a.route_w[p] * v;
      }
    }
    if (a.mode == GEMV_SWIGLU) {
      // Each (feature f, token j): gate = row f, up = row f + 8 of this tile.
      for (int idx = threadIdx.x; idx < 8 * ntc * 8; idx += blockDim.x) {
        const int f = idx & 7;
        const int j = idx >> 3;
        if (j >= ccount) continue;
        const int nt = j >> 3, jj = j & 7;
        const int ln = f * 4 + (jj >> 1);
        float gv = 0.f, uv = 0.f;
#pragma unroll
        for (int w = 0; w < GEMV_WARPS; ++w) {
          gv += red[w][nt][(jj & 1)][ln];
          uv += red[w][nt][2 + (jj & 1)][ln];
        }
        const int p = p0 + c0 + j;
        reinterpret_cast<__nv_bfloat16*>(a.out)[(int64_t)p * (a.N / 2) + tile * 8 + f] = f2bf(silu(gv) * uv);
      }
    }
    __syncthreads();
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

cudaError_t launch_q4_gemv(const GemvArgs& a, cudaStream_t s) {
  dim3 grid((unsigned)(a.N / 16), (unsigned)a.E);
  q4_gemv_kernel<<<grid, GEMV_WARPS * 32, 0, s>>>(a);
  return cudaGetLastError();
}

}  // namespace syn
