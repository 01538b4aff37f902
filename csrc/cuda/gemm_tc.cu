// Prefill GEMM on the 5th-generation tensor cores: C = X * W^T with bf16 activations X
// and 4-bit tiled weights W (syn/q4.h), grouped over experts.
//
// One CTA computes a 256 x BN output tile (BN = 128 or 256) as two 128-row MMA subtiles
// that share every dequantised B stage (half the dequantisation work per FLOP of a 128-row
// tile), with both accumulators in TMEM (2 * BN columns):
//   warp 0      TMA producer: X tiles (2 x 128 rows x 64 bf16, SWIZZLE_128B) -> smem stage
//   warp 2      raw-weight loader: bulk async copies (cp.async.bulk) of the packed 4-bit
//               tiles and their scales, TC_RAW stages ahead of the dequantisers
//   warp 1      TMEM allocator and MMA issuer: one elected thread issues tcgen05.mma
//               (kind::f16, M=128, N=BN, K=16, bf16 x bf16 -> f32) per 16 columns and
//               subtile (the second only when the tile has rows there) and
//               tcgen05.commit's to the stage's "empty" barrier
//   warps 4..11 B producers during the main loop (two per scheduler, so dequantisation
//               latency hides): 4-bit weights -> bf16 (d*q+m, f32 math, one rounding)
//               written straight into the UMMA K-major SWIZZLE_128B layout, then
//               fence.proxy.async; afterwards the epilogue: tcgen05.ld 32x32b of their TMEM
//               lane quarter (warp % 4) and column half of each subtile, fused epilogue,
//               global stores
// Stages are tracked with mbarriers; every wait is bounded (the kernel records an error
// bit and bails out instead of hanging).  Reference op: `Gemm` (crates/kernels/src/op/
// kind.rs; f32 reference crates/kernels/src/reference/linear.rs:71).
#include <cuda.h>

#include "common.cuh"
#include "sync.cuh"
#include "syn/q4.h"
#include "tc_common.cuh"

namespace syn {

constexpr int TC_MSUB = 2;   // subtiles per CTA tile (CTA tile = 256 rows)
constexpr int TC_BK = 64;
constexpr int TC_TILE_RAW = 640;  // bytes per 16-row x 64-col packed tile: 512 nibbles + 128 scales

struct TcGemmArgs {
  int raw_tma;              // 1: packed weights come from the 4-D tensor maps (one bank)
  const int64_t* qw_ptrs;   // [G] tiled 4-bit weights per group
  const int64_t* sm_ptrs;   // [G]
  const int32_t* row_off;   // [G+1] rows of A per group (contiguous)
  const float* route_w;     // [M] (mode SCALED)
  void* out;
  int group_base;           // expert index of group 0 inside the bank (raw_tma)
  int G, M, N, K;
  int mode;                 // 0 store bf16, 1 swiglu bf16 [M, N/2], 2 scaled f32, 3 add f32, 5 store f32
  int* status;
  // two banks (raw_tma): group g's weights are entry grp_sel[g] >> 1 of bank grp_sel[g] & 1
  // (bank 0: tmap_q / tmap_s, bank 1: tmap_q2 / tmap_s2); null: entry group_base + g of bank 0
  const int32_t* grp_sel;
};

template <int BN>
struct TcCfg {
  static constexpr int STAGES = BN == 256 ? 3 : 4;
  static constexpr int RAW = BN == 256 ? 3 : 6;                // packed-weight stages
  static constexpr int A_SUB = TC_BM * TC_BK * 2;              // 16 KB per subtile
  static constexpr int A_BYTES = TC_MSUB * A_SUB;              // 32 KB
  static constexpr int B_BYTES = BN * TC_BK * 2;               // 16 / 32 KB
  static constexpr int RAW_BYTES = (BN / 16) * TC_TILE_RAW;
  static constexpr size_t SMEM = 1024 + (size_t)STAGES * (A_BYTES + B_BYTES) + (size_t)RAW * RAW_BYTES;
  static_assert(SMEM <= 227 * 1024, "shared memory");
};

constexpr int TC_THREADS = 384;
constexpr int TC_PRODUCERS = 8;  // warps 4..11

template <int BN>
__global__ void __launch_bounds__(TC_THREADS, 1) tc_gemm_q4_kernel(const __grid_constant__ CUtensorMap tmap_a,
                                                            const __grid_constant__ CUtensorMap tmap_q,
                                                            const __grid_constant__ CUtensorMap tmap_s,
                                                            const __grid_constant__ CUtensorMap tmap_q2,
                                                            const __grid_constant__ CUtensorMap tmap_s2,
                                                            TcGemmArgs a) {
  constexpr int TC_STAGES = TcCfg<BN>::STAGES;
  constexpr int TC_RAW = TcCfg<BN>::RAW;
  constexpr int A_SUB = TcCfg<BN>::A_SUB;
  constexpr int A_BYTES = TcCfg<BN>::A_BYTES;
  constexpr int B_BYTES = TcCfg<BN>::B_BYTES;
  constexpr int RAW_BYTES = TcCfg<BN>::RAW_BYTES;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + TC_STAGES * A_BYTES;
  uint8_t* sR = sB + TC_STAGES * B_BYTES;
  __shared__ __align__(8) uint64_t full_a[TC_STAGES], full_b[TC_STAGES], empty[TC_STAGES], done_bar;
  __shared__ __align__(8) uint64_t raw_full[TC_RAW], raw_empty[TC_RAW];
  __shared__ uint32_t tmem_base;
  __shared__ int s_group, s_mtile;
  __shared__ volatile int s_abort;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // grid (n-tiles, m-tiles): consecutive CTAs share an activation tile (read from HBM once
  // while its n-tiles run together) and the n-tiles of one group's weights stay in L2
  const int ntile = blockIdx.x;

  // ---- find this CTA's (group, m-tile): warp 0 scans the groups 32 at a time (a prefix sum of
  // the per-group tile counts over the lanes), so a CTA of a late group does not walk every
  // earlier group's offsets one dependent load at a time ----
  if (warp == 0) {
    int base = 0, grp = -1, mt = 0;
    for (int g0 = 0; g0 < a.G && grp < 0; g0 += 32) {
      const int g = g0 + lane;
      const int nt = g < a.G ? (a.row_off[g + 1] - a.row_off[g] + TC_MSUB * TC_BM - 1) / (TC_MSUB * TC_BM) : 0;
      int incl = nt;  // inclusive prefix over the lanes
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int v = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += v;
      }
      const int bx = (int)blockIdx.y - base;
      const unsigned hit = __ballot_sync(0xffffffffu, g < a.G && bx < incl && bx >= incl - nt);
      if (hit) {
        const int src = __ffs(hit) - 1;
        grp = g0 + src;
        mt = bx - __shfl_sync(0xffffffffu, incl - nt, src);
      }
      base += __shfl_sync(0xffffffffu, incl, 31);
    }
    if (lane == 0) {
      s_group = grp;
      s_mtile = mt;
      s_abort = 0;
    }
  }
  __syncthreads();
  const int grp = s_group;
  if (grp < 0) return;  // uniform: beyond the last tile
  const int row0 = a.row_off[grp] + s_mtile * TC_MSUB * TC_BM;
  const int row_end = a.row_off[grp + 1];
  const bool two = row0 + TC_BM < row_end;  // second subtile has rows of this group
  const int KB = a.K / TC_BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < TC_STAGES; ++s) {
      mbar_init(&full_a[s], 1);
      mbar_init(&full_b[s], TC_PRODUCERS * 32);
      mbar_init(&empty[s], 1);
    }
    for (int r = 0; r < TC_RAW; ++r) {
      mbar_init(&raw_full[r], 1);
      mbar_init(&raw_empty[r], TC_PRODUCERS * 32);
    }
    mbar_init(&done_bar, 1);
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(smem_u32(&tmem_base)),
                 "r"(TC_MSUB * BN));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n");
  }
  asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory");
  const uint32_t tmem = tmem_base;

  if (warp == 0) {
    // ---------------- TMA producer (A) ----------------
    if (lane == 0) {
      for (int kb = 0; kb < KB; ++kb) {
        const int s = kb % TC_STAGES;
        const uint32_t ph = (kb / TC_STAGES) & 1;
        if (kb >= TC_STAGES && !mbar_wait(&empty[s], ph ^ 1, a.status, &s_abort)) break;
        mbar_expect_tx(&full_a[s], two ? A_BYTES : A_SUB);
        tma_load_2d(sA + s * A_BYTES, &tmap_a, kb * TC_BK, row0, &full_a[s]);
        if (two) tma_load_2d(sA + s * A_BYTES + A_SUB, &tmap_a, kb * TC_BK, row0 + TC_BM, &full_a[s]);
      }
    }
  } else if (warp == 2) {
    // ---------------- raw 4-bit weight loader ----------------
    if (lane == 0) {
      // pointer tables are read only on the bulk-copy path (the two-bank launch passes none)
      const uint8_t* qw = a.raw_tma ? nullptr : reinterpret_cast<const uint8_t*>(a.qw_ptrs[grp]);
      const uint8_t* sm = a.raw_tma ? nullptr : reinterpret_cast<const uint8_t*>(a.sm_ptrs[grp]);
      const int KG = a.K >> 6;
      const int tile0 = ntile * (BN / 16);
      const CUtensorMap* mq = &tmap_q;
      const CUtensorMap* ms = &tmap_s;
      int entry = a.group_base + grp;
      if (a.raw_tma && a.grp_sel) {
        const int sel = a.grp_sel[grp];
        entry = sel >> 1;
        if (sel & 1) {
          mq = &tmap_q2;
          ms = &tmap_s2;
        }
      }
      for (int kb = 0; kb < KB; ++kb) {
        const int r = kb % TC_RAW;
        const uint32_t ph = (kb / TC_RAW) & 1;
        if (kb >= TC_RAW && !mbar_wait(&raw_empty[r], ph ^ 1, a.status, &s_abort)) break;
        mbar_expect_tx(&raw_full[r], RAW_BYTES);
        uint8_t* dst = sR + r * RAW_BYTES;
        if (a.raw_tma) {
          // [BN/16 tiles x 512 B] of nibbles, then [BN/16 x 128 B] of scales: two copies
          tma_load_4d(dst, mq, 0, kb, tile0, entry, &raw_full[r]);
          tma_load_4d(dst + (BN / 16) * 512, ms, 0, kb, tile0, entry, &raw_full[r]);
        } else {
#pragma unroll 4
          for (int i = 0; i < BN / 16; ++i) {
            const int64_t tk = (int64_t)(tile0 + i) * KG + kb;
            bulk_load(dst + i * 512, qw + tk * 512, 512, &raw_full[r]);
            bulk_load(dst + (BN / 16) * 512 + i * 128, sm + tk * 128, 128, &raw_full[r]);
          }
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_bf16_f32<BN>();
      for (int kb = 0; kb < KB; ++kb) {
        const int s = kb % TC_STAGES;
        const uint32_t ph = (kb / TC_STAGES) & 1;
        if (!mbar_wait(&full_a[s], ph, a.status, &s_abort)) break;
        if (!mbar_wait(&full_b[s], ph, a.status, &s_abort)) break;
        asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory");
        const uint32_t a0 = smem_u32(sA + s * A_BYTES), b0 = smem_u32(sB + s * B_BYTES);
#pragma unroll
        for (int kk = 0; kk < TC_BK / 16; ++kk) {
          umma_bf16(tmem, sw128_desc(a0 + kk * 32), sw128_desc(b0 + kk * 32), idesc, (kb | kk) != 0);
          if (two)
            umma_bf16(tmem + BN, sw128_desc(a0 + A_SUB + kk * 32), sw128_desc(b0 + kk * 32), idesc, (kb | kk) != 0);
        }
        umma_commit(&empty[s]);
      }
      umma_commit(&done_bar);
    }
  } else if (warp >= 4 && warp < 4 + TC_PRODUCERS) {
    // ---------------- B producers: 4-bit -> bf16 in SWIZZLE_128B layout ----------------
    const int pw = warp - 4;  // 0..7
    const int g = lane >> 2, t = lane & 3;
    constexpr int TPW = BN / 16 / TC_PRODUCERS;  // 16-row tiles per producer warp
    for (int kb = 0; kb < KB; ++kb) {
      const int s = kb % TC_STAGES;
      const uint32_t ph = (kb / TC_STAGES) & 1;
      const int rr = kb % TC_RAW;
      if (!mbar_wait(&raw_full[rr], (kb / TC_RAW) & 1, a.status, &s_abort)) break;
      uint4 q[TPW];
      uint2 slo[TPW], shi[TPW];
      const uint8_t* R = sR + rr * RAW_BYTES;
#pragma unroll
      for (int i = 0; i < TPW; ++i) {
        const int ti = pw + TC_PRODUCERS * i;
        q[i] = *reinterpret_cast<const uint4*>(R + ti * 512 + lane * 16);
        const uint8_t* sb = R + (BN / 16) * 512 + ti * 128;
        slo[i] = *reinterpret_cast<const uint2*>(sb + g * 8);
        shi[i] = *reinterpret_cast<const uint2*>(sb + (g + 8) * 8);
      }
      if (kb >= TC_STAGES && !mbar_wait(&empty[s], ph ^ 1, a.status, &s_abort)) break;
      uint8_t* B = sB + s * B_BYTES;
      // Dequantise: value = bf16(fma(d, q, m)) in f32 (one rounding, the reference's
      // dequantised value), stored as pairs of adjacent k into the K-major SWIZZLE_128B tile
      // (16-byte chunk index XOR row%8; row%8 == g for every row this thread writes).
#pragma unroll
      for (int i = 0; i < TPW; ++i) {
        const int rt = pw + TC_PRODUCERS * i;  // 16-row tile inside the BN rows
        const uint32_t words[4] = {q[i].x, q[i].y, q[i].z, q[i].w};
#pragma unroll
        for (int blk = 0; blk < 2; ++blk) {
          const half2 dl = *reinterpret_cast<const half2*>(blk ? &slo[i].y : &slo[i].x);
          const half2 dh = *reinterpret_cast<const half2*>(blk ? &shi[i].y : &shi[i].x);
          const float dd[2] = {__low2float(dl), __low2float(dh)};
          // min folded with the +128 offset of the magic conversion below: m - 128 d (exact
          // in f32 whenever d and m are within 2^13 of each other, i.e. for real blocks)
          const float mm[2] = {fmaf(-128.f, dd[0], __high2float(dl)), fmaf(-128.f, dd[1], __high2float(dh))};
#pragma unroll
          for (int st = 0; st < 2; ++st) {
            const uint32_t w = words[blk * 2 + st];
#pragma unroll
            for (int reg = 0; reg < 4; ++reg) {
              const int hi_row = reg & 1, hi_col = reg >> 1;
              // nibbles reg and reg+4 -> bf16 (128 + q) pair in one LOP3; bf16 -> f32 is a
              // 16-bit shift, so no integer-to-float conversion is issued
              const uint32_t qq = lop3_and_or(w >> (4 * reg), 0x000F000Fu, 0x43004300u);
              const float q0 = __uint_as_float(qq << 16);
              const float q1 = __uint_as_float(qq & 0xFFFF0000u);
              const uint32_t v = pack_bf16x2(fmaf(dd[hi_row], q0, mm[hi_row]), fmaf(dd[hi_row], q1, mm[hi_row]));
              const int row = rt * 16 + g + 8 * hi_row;
              const int chunk = (blk * 4 + st * 2 + hi_col) ^ g;
              *reinterpret_cast<uint32_t*>(B + row * 128 + chunk * 16 + 4 * t) = v;
            }
          }
        }
      }
      // the packed stage is released only now: its values were consumed by the stores above,
      // and the proxy fence orders these generic-proxy reads (and the stores) before the TMA
      // refill of the stage and the MMA reads of the tile (async proxy)
      asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
      mbar_arrive(&raw_empty[rr]);
      mbar_arrive(&full_b[s]);
    }
    // ---------------- epilogue ----------------
    const bool ok = mbar_wait(&done_bar, 0, a.status, &s_abort);
    asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory");
    // the activation stages are free once every MMA has completed (done_bar): each epilogue
    // warp stages its output blocks in 4 KB of them (generic writes after async-proxy use)
    asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
    uint8_t* stg = sA + (warp - 4) * 4096;
    const int quarter = warp & 3;       // TMEM lanes this warp may read
    const int half = (warp - 4) >> 2;   // which half of the columns it stores
#pragma unroll 1
    for (int sub = 0; sub < (two ? 2 : 1); ++sub)
#pragma unroll 1
    for (int c0 = half * (BN / 2); c0 < (half + 1) * (BN / 2); c0 += 32) {
      const int rbase = row0 + sub * TC_BM + quarter * 32;  // first row of this warp's 32 x 32 block
      uint32_t r[32];
      tmem_ld32(tmem + ((uint32_t)(quarter * 32) << 16) + sub * BN + c0, r);
      const int nrows = min(32, min(row_end, a.M) - rbase);  // rows of this group (warp-uniform)
      if (!ok || nrows <= 0) continue;
      const int n0 = ntile * BN + c0;
      // lane = row in TMEM; the block goes through this warp's staging buffer so that each
      // global store instruction writes whole 16-byte pieces of consecutive rows
      float v[32];
#pragma unroll
      for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
      uint8_t* ob = reinterpret_cast<uint8_t*>(a.out);
      if (a.mode == 1) {  // SwiGLU: bf16 [M, N / 2]
        stg_put_swiglu(stg, lane, v);
        stg_flush<2>(stg, lane, ob + ((int64_t)rbase * (a.N / 2) + n0 / 2) * 2, (int64_t)a.N, nrows);
      } else if (a.mode == 0) {  // bf16 [M, N]
        stg_put_bf16(stg, lane, v);
        stg_flush<4>(stg, lane, ob + ((int64_t)rbase * a.N + n0) * 2, (int64_t)a.N * 2, nrows);
      } else {  // f32 [M, N]; mode 2: scaled by the row's routing weight; mode 3: added
        const float sc = (a.mode == 2 && lane < nrows) ? a.route_w[rbase + lane] : 1.f;
        stg_put_f32(stg, lane, v, sc);
        if (a.mode == 3)
          stg_flush<8, true>(stg, lane, ob + ((int64_t)rbase * a.N + n0) * 4, (int64_t)a.N * 4, nrows);
        else
          stg_flush<8>(stg, lane, ob + ((int64_t)rbase * a.N + n0) * 4, (int64_t)a.N * 4, nrows);
      }
    }
  }
  asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory");
  __syncthreads();
  if (warp == 1) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(tmem), "r"(TC_MSUB * BN));
  }
}

// ---- host side ----
template <int BN>
static cudaError_t launch_q4_tiles(dim3 grid, const CUtensorMap& map, const CUtensorMap& mq, const CUtensorMap& ms,
                                   const CUtensorMap& mq2, const CUtensorMap& ms2, const TcGemmArgs& a,
                                   cudaStream_t s) {
  static bool set = false;
  constexpr size_t smem = TcCfg<BN>::SMEM;
  if (!set) {
    const cudaError_t e =
        cudaFuncSetAttribute(tc_gemm_q4_kernel<BN>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    set = true;
  }
  tc_gemm_q4_kernel<BN><<<grid, TC_THREADS, smem, s>>>(map, mq, ms, mq2, ms2, a);
  return cudaGetLastError();
}

// bank_qw/bank_sm: base of a contiguous expert bank (or of one matrix) and the number
// of experts in it; when given (non-null), the packed weights stream with two 4-D TMA copies
// per stage instead of 2 * BN/16 bulk copies.  bank2_* and grp_sel: a second bank (e.g. the
// VRAM residents in bank 0 and the staged host experts in bank 1); group g reads entry
// grp_sel[g] >> 1 of bank grp_sel[g] & 1.
cudaError_t launch_tc_gemm_q4(const void* x, int ldx, const int64_t* qw_ptrs, const int64_t* sm_ptrs,
                              const int32_t* row_off, int G, int M, int N, int K, int mode, const float* route_w,
                              void* out, int* status, int max_mtiles, const void* bank_qw, const void* bank_sm,
                              int bank_experts, int group_base, cudaStream_t s, const void* bank2_qw,
                              const void* bank2_sm, int bank2_experts, const int32_t* grp_sel) {
  if (K % TC_BK != 0 || N % 128 != 0 || M <= 0) return cudaErrorInvalidValue;
  if ((reinterpret_cast<uintptr_t>(x) & 15) != 0 || (ldx * 2) % 16 != 0) return cudaErrorInvalidValue;
  if ((reinterpret_cast<uintptr_t>(out) & 15) != 0) return cudaErrorInvalidValue;  // 16-byte epilogue stores
  PFN_encodeTiled enc = get_encode();
  if (!enc) return cudaErrorNotSupported;
  CUtensorMap map, mq, ms;
  memset(&mq, 0, sizeof(mq));
  memset(&ms, 0, sizeof(ms));
  {
    const cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)M};
    const cuuint64_t strides[1] = {(cuuint64_t)ldx * 2};
    const cuuint32_t box[2] = {(cuuint32_t)TC_BK, (cuuint32_t)TC_BM};
    const cuuint32_t estr[2] = {1, 1};
    CUresult r = enc(&map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(x), dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return cudaErrorInvalidValue;
  }
  const bool wide = (N % 256 == 0);
  const int BN = wide ? 256 : 128;
  auto aligned = [](const void* p) { return p != nullptr && (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
  const int raw_tma = aligned(bank_qw) && aligned(bank_sm);
  if (bank2_qw != nullptr && !(raw_tma && aligned(bank2_qw) && aligned(bank2_sm) && grp_sel != nullptr))
    return cudaErrorInvalidValue;
  CUtensorMap mq2, ms2;
  memset(&mq2, 0, sizeof(mq2));
  memset(&ms2, 0, sizeof(ms2));
  if (raw_tma) {
    if (!encode_q4_raw_maps(enc, &mq, &ms, bank_qw, bank_sm, bank_experts, N, K, BN)) return cudaErrorInvalidValue;
    if (bank2_qw != nullptr && !encode_q4_raw_maps(enc, &mq2, &ms2, bank2_qw, bank2_sm, bank2_experts, N, K, BN))
      return cudaErrorInvalidValue;
  }
  TcGemmArgs a{raw_tma, qw_ptrs, sm_ptrs, row_off, route_w, out, group_base, G, M, N, K, mode, status,
               bank2_qw != nullptr ? grp_sel : nullptr};
  if (max_mtiles > 65535) return cudaErrorInvalidValue;  // grid y limit
  dim3 grid((unsigned)(N / BN), (unsigned)max_mtiles);
  if (wide) return launch_q4_tiles<256>(grid, map, mq, ms, mq2, ms2, a, s);
  return launch_q4_tiles<128>(grid, map, mq, ms, mq2, ms2, a, s);
}


}  // namespace syn
