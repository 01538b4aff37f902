// Decode GEMM with 4-bit weights on the 5th-generation tensor cores, for 16-64 token rows:
// D = W_tile * X^T with the dequantised weights as the M = 128 operand and the tokens as N
// (BT = 32 or 64 columns, rows of X past T zero-filled by TMA), so every weight is read and
// dequantised once per launch whatever the row count, and the MMA issue leaves the SM's
// instruction stream (the mma.sync GEMV of the same rows is instruction-bound: four 8-token
// tiles per 16x16 weight block).  Reference ops `Gemv` / `Gemm` over 4-bit weights
// (crates/kernels/src/op/kind.rs; f32 reference crates/kernels/src/reference/linear.rs:62-132).
//
// One CTA = 128 weight rows x BT tokens over a K slice; the K slices of a row tile form a
// thread-block cluster whose f32 partials meet in shared memory (distributed shared memory,
// rank order: deterministic):
//   warp 0      TMA producer of the X tiles (BT rows x 64 bf16, SWIZZLE_128B)
//   warp 1      TMEM owner and MMA issuer (kind::f16, M = 128, N = BT, K = 16)
//   warp 2      raw-weight loader: two 4-D TMA copies per 64-column block (the eight packed
//               16-row tiles: 8 x 512 B of nibbles, 8 x 128 B of scale/min)
//   warps 4..11 dequantisers (one 16-row tile each): d * q + m in f32, one rounding to bf16,
//               straight into the K-major SWIZZLE_128B A tile; then warps 4..7 run the
//               epilogue of their TMEM lane quarter (shared with the bf16 GEMM: bf16 store,
//               SwiGLU, f32 add / store, tensor-parallel peer push with completion flags).
// Every wait is bounded (bit 4 of *status, never a hang).
#include <cstdlib>

#include "tc_emit.cuh"

namespace syn {

namespace {

constexpr int QD_THREADS = 384;
constexpr int QD_PRODUCERS = 8;
constexpr int QD_STAGES = 3;
constexpr int QD_A_BYTES = 128 * 128;           // 128 rows x 64 bf16
constexpr int QD_RAW_BYTES = 8 * (512 + 128);   // eight 16-row packed tiles

template <int BT, int RAW_ = (BT <= 32 ? 8 : 6)>
struct QdCfg {
  static constexpr int B_BYTES = BT * 128;
  static constexpr int RAW = RAW_;  // packed-weight stages in flight (HBM latency)
  static constexpr size_t SMEM = 1024 + (size_t)QD_STAGES * (QD_A_BYTES + B_BYTES) + (size_t)RAW * QD_RAW_BYTES;
  static_assert(SMEM <= 113 * 1024, "two CTAs per SM");
};

template <int BT, int MODE, int RAWS>
__global__ void __launch_bounds__(QD_THREADS, 2)
    tc_gemm_q4_dec_kernel(const __grid_constant__ CUtensorMap tmap_x, const __grid_constant__ CUtensorMap tmap_q,
                          const __grid_constant__ CUtensorMap tmap_s, DenseGemmArgs a) {
  constexpr int B_BYTES = QdCfg<BT, RAWS>::B_BYTES;
  constexpr int QD_RAW = QdCfg<BT, RAWS>::RAW;
  constexpr int TMEM_COLS = BT < 32 ? 32 : BT;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = sA + QD_STAGES * QD_A_BYTES;
  uint8_t* sR = sB + QD_STAGES * B_BYTES;
  __shared__ __align__(8) uint64_t full_a[QD_STAGES], full_b[QD_STAGES], empty[QD_STAGES], done_bar;
  __shared__ __align__(8) uint64_t raw_full[QD_RAW], raw_empty[QD_RAW];
  __shared__ uint32_t tmem_base;
  __shared__ volatile int s_abort;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tile = blockIdx.x, split = blockIdx.y;
  const int KB = a.K / 64;
  const int kb0 = (int)((int64_t)KB * split / a.splits), kb1 = (int)((int64_t)KB * (split + 1) / a.splits);
  const int nk = kb1 - kb0;

  if (threadIdx.x == 0) {
    s_abort = 0;
    for (int s = 0; s < QD_STAGES; ++s) {
      mbar_init(&full_a[s], QD_PRODUCERS * 32);
      mbar_init(&full_b[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int r = 0; r < QD_RAW; ++r) {
      mbar_init(&raw_full[r], 1);
      mbar_init(&raw_empty[r], QD_PRODUCERS * 32);
    }
    mbar_init(&done_bar, 1);
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(smem_u32(&tmem_base)),
                 "r"(TMEM_COLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n");
  }
  asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory");
  const uint32_t tmem = tmem_base;

  if (warp == 0) {
    // ---------------- X tiles (tokens) ----------------
    if (lane == 0) {
      for (int i = 0; i < nk; ++i) {
        const int s = i % QD_STAGES;
        if (i >= QD_STAGES && !mbar_wait(&empty[s], ((i / QD_STAGES) & 1) ^ 1, a.status, &s_abort)) break;
        mbar_expect_tx(&full_b[s], B_BYTES);
        tma_load_2d(sB + s * B_BYTES, &tmap_x, (kb0 + i) * 64, 0, &full_b[s]);
      }
    }
  } else if (warp == 2) {
    // ---------------- packed 4-bit tiles ----------------
    if (lane == 0) {
      for (int i = 0; i < nk; ++i) {
        const int r = i % QD_RAW;
        if (i >= QD_RAW && !mbar_wait(&raw_empty[r], ((i / QD_RAW) & 1) ^ 1, a.status, &s_abort)) break;
        mbar_expect_tx(&raw_full[r], QD_RAW_BYTES);
        uint8_t* dst = sR + r * QD_RAW_BYTES;
        tma_load_4d(dst, &tmap_q, 0, kb0 + i, tile * 8, 0, &raw_full[r]);
        tma_load_4d(dst + 8 * 512, &tmap_s, 0, kb0 + i, tile * 8, 0, &raw_full[r]);
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_bf16_f32<BT>();
      for (int i = 0; i < nk; ++i) {
        const int s = i % QD_STAGES;
        const uint32_t ph = (i / QD_STAGES) & 1;
        if (!mbar_wait(&full_a[s], ph, a.status, &s_abort)) break;
        if (!mbar_wait(&full_b[s], ph, a.status, &s_abort)) break;
        asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory");
        const uint32_t a0 = smem_u32(sA + s * QD_A_BYTES), b0 = smem_u32(sB + s * B_BYTES);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          umma_bf16(tmem, sw128_desc(a0 + kk * 32), sw128_desc(b0 + kk * 32), idesc, (i | kk) != 0);
        umma_commit(&empty[s]);
      }
      umma_commit(&done_bar);
    }
  } else if (warp >= 4) {
    // ---------------- dequantisers: one 16-row tile per warp ----------------
    const int rt = warp - 4;
    const int g = lane >> 2, t = lane & 3;
    for (int i = 0; i < nk; ++i) {
      const int s = i % QD_STAGES;
      const int rr = i % QD_RAW;
      if (!mbar_wait(&raw_full[rr], (i / QD_RAW) & 1, a.status, &s_abort)) break;
      const uint8_t* R = sR + rr * QD_RAW_BYTES;
      const uint4 q = *reinterpret_cast<const uint4*>(R + rt * 512 + lane * 16);
      const uint8_t* sb = R + 8 * 512 + rt * 128;
      const uint2 slo = *reinterpret_cast<const uint2*>(sb + g * 8);
      const uint2 shi = *reinterpret_cast<const uint2*>(sb + (g + 8) * 8);
      if (i >= QD_STAGES && !mbar_wait(&empty[s], ((i / QD_STAGES) & 1) ^ 1, a.status, &s_abort)) break;
      uint8_t* A = sA + s * QD_A_BYTES;
      const uint32_t words[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
      for (int blk = 0; blk < 2; ++blk) {
        const half2 dl = *reinterpret_cast<const half2*>(blk ? &slo.y : &slo.x);
        const half2 dh = *reinterpret_cast<const half2*>(blk ? &shi.y : &shi.x);
        const float dd[2] = {__low2float(dl), __low2float(dh)};
        // min folded with the +128 offset of the bf16 magic-number conversion: m - 128 d
        const float mm[2] = {fmaf(-128.f, dd[0], __high2float(dl)), fmaf(-128.f, dd[1], __high2float(dh))};
#pragma unroll
        for (int st = 0; st < 2; ++st) {
          const uint32_t w = words[blk * 2 + st];
#pragma unroll
          for (int reg = 0; reg < 4; ++reg) {
            const int hi_row = reg & 1, hi_col = reg >> 1;
            const uint32_t qq = lop3_and_or(w >> (4 * reg), 0x000F000Fu, 0x43004300u);
            const float q0 = __uint_as_float(qq << 16);
            const float q1 = __uint_as_float(qq & 0xFFFF0000u);
            const uint32_t v = pack_bf16x2(fmaf(dd[hi_row], q0, mm[hi_row]), fmaf(dd[hi_row], q1, mm[hi_row]));
            const int row = rt * 16 + g + 8 * hi_row;
            const int chunk = (blk * 4 + st * 2 + hi_col) ^ g;
            *reinterpret_cast<uint32_t*>(A + row * 128 + chunk * 16 + 4 * t) = v;
          }
        }
      }
      // the packed stage is released only now: its values were consumed by the stores above,
      // and the proxy fence orders these generic-proxy reads (and the stores) before the TMA
      // refill of the stage and the MMA reads of the tile (async proxy)
      asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
      mbar_arrive(&raw_empty[rr]);
      mbar_arrive(&full_a[s]);
    }
    // ---------------- epilogue (warps 4..7: one TMEM lane quarter each) ----------------
    if (warp < 8) {
      const int quarter = warp & 3;
      const int r = quarter * 32 + lane;  // weight row inside the tile = TMEM lane
      const bool ok = mbar_wait(&done_bar, 0, a.status, &s_abort) && nk > 0;
      asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory");
      if (a.splits == 1) {
#pragma unroll 1
        for (int c0 = 0; c0 < BT; c0 += 32) {
          uint32_t u[32];
          tmem_ld32(tmem + ((uint32_t)(quarter * 32) << 16) + c0, u);
          float v[32];
#pragma unroll
          for (int j = 0; j < 32; ++j) v[j] = ok ? __uint_as_float(u[j]) : 0.f;
          if (ok) bf16_emit<BT, MODE, true>(a, tile, 0, r, c0, v);
        }
      } else {
        // the stages are idle once the last MMA committed: this slice's partial tile goes there
        float* part = reinterpret_cast<float*>(smem) + r * (BT + 4);
#pragma unroll 1
        for (int c0 = 0; c0 < BT; c0 += 32) {
          uint32_t u[32];
          tmem_ld32(tmem + ((uint32_t)(quarter * 32) << 16) + c0, u);
#pragma unroll
          for (int j = 0; j < 32; j += 4)
            *reinterpret_cast<float4*>(part + c0 + j) =
                make_float4(ok ? __uint_as_float(u[j]) : 0.f, ok ? __uint_as_float(u[j + 1]) : 0.f,
                            ok ? __uint_as_float(u[j + 2]) : 0.f, ok ? __uint_as_float(u[j + 3]) : 0.f);
        }
      }
    }
  }
  if (a.splits > 1) {
    // each CTA of the cluster sums one column share of the tile over the cluster's CTAs in
    // rank order and runs the epilogue on it
    cluster_sync_all();
    if (warp >= 4 && warp < 8) {
      const int r = (warp & 3) * 32 + lane;
      const int w = BT / a.splits, c_lo = split * w;
      const float* part = reinterpret_cast<const float*>(smem) + r * (BT + 4) + c_lo;
      float v[32];
#pragma unroll
      for (int j = 0; j < 32; ++j) v[j] = 0.f;
      for (int p = 0; p < a.splits; ++p) {
#pragma unroll
        for (int j = 0; j < 32; j += 4) {
          if (j < w) {
            const float4 q = ld_dsmem_f4(part + j, p);
            v[j] += q.x;
            v[j + 1] += q.y;
            v[j + 2] += q.z;
            v[j + 3] += q.w;
          }
        }
      }
      bf16_emit<BT, MODE, true>(a, tile, 0, r, c_lo, v, w);
    }
    cluster_sync_all();  // no CTA leaves while a peer still reads its shared memory
  }
  if (MODE == 6 && warp >= 4 && warp < 8) {
    // completion of the whole grid: the last CTA raises one flag per peer
    __threadfence_system();
    asm volatile("bar.sync 1, 128;\n" ::: "memory");
    if (threadIdx.x == 128) {
      const unsigned total = gridDim.x * gridDim.y;
      const unsigned prev = atomicAdd(a.done_ctr, 1u);
      if (prev == total - 1) {
        *a.done_ctr = 0u;
        __threadfence_system();
        const uint32_t seq = (*a.step_ctr) * (uint32_t)a.n_layers + (uint32_t)a.layer + 1u;
        for (int q = 0; q < a.n_peers; ++q)
          st_release_sys(reinterpret_cast<uint32_t*>(a.peers[q] + a.off_flag) + a.rank, seq);
      }
    }
  }
  asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory");
  __syncthreads();
  if (warp == 1) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(tmem), "r"(TMEM_COLS));
  }
}

template <int BT, int MODE, int RAWS>
cudaError_t launch_qd(const CUtensorMap& mx, const CUtensorMap& mq, const CUtensorMap& ms, const DenseGemmArgs& a,
                      cudaStream_t s) {
  static bool set = false;
  constexpr size_t smem = QdCfg<BT, RAWS>::SMEM;
  auto* kern = tc_gemm_q4_dec_kernel<BT, MODE, RAWS>;
  if (!set) {
    const cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    set = true;
  }
  const dim3 grid((unsigned)(a.N / 128), (unsigned)a.splits);
  if (a.splits == 1) {
    kern<<<grid, QD_THREADS, smem, s>>>(mx, mq, ms, a);
    return cudaGetLastError();
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(QD_THREADS);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 1;
  attr[0].val.clusterDim.y = (unsigned)a.splits;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, mx, mq, ms, a);
}

template <int BT>
cudaError_t launch_qd_mode(const CUtensorMap& mx, const CUtensorMap& mq, const CUtensorMap& ms,
                           const DenseGemmArgs& a, cudaStream_t s) {
  // SYN_Q4_DEC_RAW=4: four packed-weight stages (fault isolation / measurement)
  static const bool raw4 = getenv("SYN_Q4_DEC_RAW") && atoi(getenv("SYN_Q4_DEC_RAW")) == 4;
  if (raw4 && a.mode == 5) return launch_qd<BT, 5, 4>(mx, mq, ms, a, s);
  constexpr int R = QdCfg<BT>::RAW;
  switch (a.mode) {
    case 0: return launch_qd<BT, 0, R>(mx, mq, ms, a, s);
    case 1: return launch_qd<BT, 1, R>(mx, mq, ms, a, s);
    case 3: return launch_qd<BT, 3, R>(mx, mq, ms, a, s);
    case 5: return launch_qd<BT, 5, R>(mx, mq, ms, a, s);
    case 6: return launch_qd<BT, 6, R>(mx, mq, ms, a, s);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace

// K slices per 128-row weight tile: about two CTAs per SM (two fit), at least 4 K blocks each.
int q4_dec_splits(int N, int K) {
  const int tiles = N / 128, kb = K / 64;
  int s = 1;
  while (s < 8 && tiles * s * 2 <= 2 * num_sms() && kb / (s * 2) >= 4) s *= 2;
  return s;
}

cudaError_t launch_tc_gemm_q4_dec(const void* x, int T, int ldx, const void* qw, const void* sm, int N, int K,
                                  int mode, void* out, int ldo, const PeerPush* pp, int* status, cudaStream_t s) {
  if (T <= 0 || T > 64 || N % 128 || K % 64 || K < 64) return cudaErrorInvalidValue;
  if ((reinterpret_cast<uintptr_t>(x) & 15) || (ldx * 2) % 16 || (reinterpret_cast<uintptr_t>(qw) & 15) ||
      (reinterpret_cast<uintptr_t>(sm) & 15))
    return cudaErrorInvalidValue;
  if (mode == 6 && pp == nullptr) return cudaErrorInvalidValue;
  DenseGemmArgs a;
  memset(&a, 0, sizeof(a));
  a.decode = 1;
  a.T = T;
  a.N = N;
  a.K = K;
  a.mode = mode;
  a.out = out;
  a.ldo = ldo;
  a.status = status;
  a.splits = q4_dec_splits(N, K);
  // forced K slices (fault isolation / measurement), read once
  static const int forced = [] {
    const char* e = getenv("SYN_Q4_DEC_SPLITS");
    const int f = e ? atoi(e) : 0;
    return (f == 1 || f == 2 || f == 4 || f == 8) ? f : 0;
  }();
  if (forced) a.splits = forced;
  if (pp) {
    a.peers = pp->peers;
    a.n_peers = pp->n_peers;
    a.rank = pp->rank;
    a.cap = pp->cap;
    a.owner_rows = pp->owner_rows;
    a.src_stride = pp->src_stride ? pp->src_stride : (int64_t)pp->cap * ldo;
    a.off_recv = pp->off_recv;
    a.off_flag = pp->off_flag;
    a.done_ctr = pp->done_ctr;
    a.step_ctr = pp->step_ctr;
    a.n_layers = pp->n_layers;
    a.layer = pp->layer;
  }
  PFN_encodeTiled enc = get_encode();
  if (!enc) return cudaErrorNotSupported;
  const int bt = T <= 32 ? 32 : 64;
  CUtensorMap mx;
  const cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)T};
  const cuuint64_t strides[1] = {(cuuint64_t)ldx * 2};
  const cuuint32_t box[2] = {64, (cuuint32_t)bt};
  const cuuint32_t estr[2] = {1, 1};
  if (enc(&mx, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(x), dims, strides, box, estr,
          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return cudaErrorInvalidValue;
  CUtensorMap mq, ms;  // the matrix as a one-entry bank: one box = the eight tiles of a 128-row tile
  if (!encode_q4_raw_maps(enc, &mq, &ms, qw, sm, 1, N, K, 128)) return cudaErrorInvalidValue;
  return bt == 32 ? launch_qd_mode<32>(mx, mq, ms, a, s) : launch_qd_mode<64>(mx, mq, ms, a, s);
}

}  // namespace syn
