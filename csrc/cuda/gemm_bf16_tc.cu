// bf16 GEMM on the 5th-generation tensor cores: C = X W^T with bf16 activations X [T, K] and
// bf16 weights W [N, K], f32 accumulation in TMEM, both operands streamed by TMA
// (SWIZZLE_128B, K-major) from this GPU's own memory.  Reference ops `Gemm` / `Gemv`
// (crates/kernels/src/op/kind.rs; f32 reference crates/kernels/src/reference/linear.rs:62-132)
// for bf16 weights, and the tensor-parallel call sites of plan/rfcs/RFC-0032-distributed-
// execution.md:372-403 when the epilogue pushes to peers.
//
// One CTA computes a 128 x BN tile D = A_tile * B_tile^T over its K range:
//   prefill orientation (T >= 128): A = X (128 tokens), B = W (BN outputs); D[token][output]
//   decode orientation (T <= 256):  A = W (128 outputs), B = X (BN >= T tokens, rows past T
//                                    are zero-filled by TMA); D[output][token].  The weight
//                                    rows stream once; K is split over the CTAs of a thread-
//                                    block cluster when the row tiles alone do not fill the
//                                    GPU; the f32 partials meet in shared memory and each CTA
//                                    sums a column share over distributed shared memory in
//                                    rank order (deterministic, no global workspace).
// Warps: 0 TMA producer, 1 TMEM allocator + MMA issuer (one elected thread issues
// tcgen05.mma kind::f16 M=128 N=BN K=16 and commits each stage to its "empty" barrier),
// 2..5 epilogue (tcgen05.ld 32x32b of their TMEM lane quarter, warp % 4).
// Epilogues: bf16 store, SwiGLU of interleaved 8-row gate/up chunks (bf16), f32 accumulate,
// f32 store, and the peer push of tensor parallelism: every f32 output row goes over NVLink
// into a receive slot of each peer (one-shot all-reduce) or of the row's owner rank
// (reduce-scatter), and the grid's last CTA raises one completion flag per peer.
// Every wait is bounded (an error bit in `status`, never a hang).
#include "tc_emit.cuh"

namespace syn {

template <int BN>
struct Bf16Cfg {
  // decode tiles (BN <= 64) keep 4 stages so that two CTAs fit on an SM (no wave tail when the
  // row tiles x K slices exceed the SM count); prefill tiles take what shared memory allows
  static constexpr int STAGES = BN >= 256 ? 4 : (BN <= 64 ? 4 : 6);
  static constexpr int A_BYTES = 128 * 64 * 2;  // 16 KB
  static constexpr int B_BYTES = BN * 64 * 2;
  static constexpr size_t SMEM = 1024 + (size_t)STAGES * (A_BYTES + B_BYTES);
  static_assert(SMEM <= 227 * 1024, "shared memory");
};

constexpr int BF_THREADS = 192;

template <int BN, int MODE, bool DEC>
__global__ void __launch_bounds__(BF_THREADS, 1) tc_gemm_bf16_kernel(const __grid_constant__ CUtensorMap tmap_a,
                                                                 const __grid_constant__ CUtensorMap tmap_b,
                                                                 DenseGemmArgs a) {
  constexpr int STAGES = Bf16Cfg<BN>::STAGES;
  constexpr int A_BYTES = Bf16Cfg<BN>::A_BYTES;
  constexpr int B_BYTES = Bf16Cfg<BN>::B_BYTES;
  constexpr int TMEM_COLS = BN < 32 ? 32 : BN;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * A_BYTES;
  __shared__ __align__(8) uint64_t full[STAGES], empty[STAGES], done_bar;
  __shared__ uint32_t tmem_base;
  __shared__ volatile int s_abort;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // decode: blockIdx.x = weight row tile, blockIdx.y = K slice; prefill: x = token tile, y = output tile
  const int tile_a = blockIdx.x;
  const int tile_b = DEC ? 0 : blockIdx.y;
  const int split = DEC ? blockIdx.y : 0;
  const int KB = a.K / 64;
  const int kb0 = (int)((int64_t)KB * split / a.splits), kb1 = (int)((int64_t)KB * (split + 1) / a.splits);
  const int a_row0 = tile_a * 128, b_row0 = tile_b * BN;

  if (threadIdx.x == 0) {
    s_abort = 0;
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
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
    if (lane == 0) {
      for (int kb = kb0; kb < kb1; ++kb) {
        const int i = kb - kb0, s = i % STAGES;
        const uint32_t ph = (i / STAGES) & 1;
        if (i >= STAGES && !mbar_wait(&empty[s], ph ^ 1, a.status, &s_abort)) break;
        mbar_expect_tx(&full[s], A_BYTES + B_BYTES);
        tma_load_2d(sA + s * A_BYTES, &tmap_a, kb * 64, a_row0, &full[s]);
        tma_load_2d(sB + s * B_BYTES, &tmap_b, kb * 64, b_row0, &full[s]);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_bf16_f32<BN>();
      for (int kb = kb0; kb < kb1; ++kb) {
        const int i = kb - kb0, s = i % STAGES;
        const uint32_t ph = (i / STAGES) & 1;
        if (!mbar_wait(&full[s], ph, a.status, &s_abort)) break;
        asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory");
        const uint32_t a0 = smem_u32(sA + s * A_BYTES), b0 = smem_u32(sB + s * B_BYTES);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          umma_bf16(tmem, sw128_desc(a0 + kk * 32), sw128_desc(b0 + kk * 32), idesc, (i | kk) != 0);
        umma_commit(&empty[s]);
      }
      umma_commit(&done_bar);
    }
  } else {
    // ---------------- epilogue warps 2..5 ----------------
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;  // D row (TMEM lane)
    const bool ok = mbar_wait(&done_bar, 0, a.status, &s_abort) && kb1 > kb0;
    asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory");
    if (!DEC && MODE != 6 && a.vec_out) {
      // prefill orientation (lane = token): each 32 x 32 block goes through 4 KB of the free
      // pipeline stages and is stored row-major, 16 bytes per lane
      asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
      uint8_t* stg = sA + (warp - 2) * 4096;
      const int tbase = tile_a * 128 + quarter * 32;
      const int nrows = min(32, a.T - tbase);
#pragma unroll 1
      for (int c0 = 0; c0 < BN; c0 += 32) {
        uint32_t u[32];
        tmem_ld32(tmem + ((uint32_t)(quarter * 32) << 16) + c0, u);
        const int n0 = tile_b * BN + c0;
        if (!ok || nrows <= 0 || n0 >= a.N) continue;  // warp-uniform
        float v[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(u[j]);
        uint8_t* ob = reinterpret_cast<uint8_t*>(a.out);
        if constexpr (MODE == 1) {
          stg_put_swiglu(stg, lane, v);
          stg_flush<2>(stg, lane, ob + ((int64_t)tbase * a.ldo + n0 / 2) * 2, (int64_t)a.ldo * 2, nrows);
        } else if constexpr (MODE == 0) {
          stg_put_bf16(stg, lane, v);
          stg_flush<4>(stg, lane, ob + ((int64_t)tbase * a.ldo + n0) * 2, (int64_t)a.ldo * 2, nrows);
        } else {
          stg_put_f32(stg, lane, v, 1.f);
          stg_flush<8, MODE == 3>(stg, lane, ob + ((int64_t)tbase * a.ldo + n0) * 4, (int64_t)a.ldo * 4, nrows);
        }
      }
    } else if (!DEC || a.splits == 1) {
#pragma unroll 1
      for (int c0 = 0; c0 < BN; c0 += 32) {
        uint32_t u[32];
        tmem_ld32(tmem + ((uint32_t)(quarter * 32) << 16) + c0, u);
        float v[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = ok ? __uint_as_float(u[j]) : 0.f;
        if (ok) bf16_emit<BN, MODE, DEC>(a, tile_a, tile_b, r, c0, v);
      }
    } else {
      // split-K over the CTAs of a cluster: the slice's partial tile goes to this CTA's own
      // shared memory (the pipeline stages are free once the last MMA committed)
      float* part = reinterpret_cast<float*>(smem) + r * (BN + 4);
#pragma unroll 1
      for (int c0 = 0; c0 < BN; c0 += 32) {
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
  if (DEC && a.splits > 1) {
    // every slice's partial is in its CTA's shared memory: each CTA sums one column share of
    // the tile over the cluster's CTAs in rank order (distributed shared memory; the same
    // order on every launch: deterministic) and runs the epilogue on it
    cluster_sync_all();
    if (warp >= 2) {
      const int r = (warp & 3) * 32 + lane;
      const int w = BN / a.splits, c_lo = split * w;
      const float* part = reinterpret_cast<const float*>(smem) + r * (BN + 4) + c_lo;
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
      bf16_emit<BN, MODE, DEC>(a, tile_a, tile_b, r, c_lo, v, w);
    }
    cluster_sync_all();  // no CTA leaves while a peer still reads its shared memory
  }
  if (MODE == 6 && warp >= 2) {
    // completion of the whole grid: every CTA publishes its peer stores, the last raises
    // one flag per peer (the arrival counter is reset before the release)
    __threadfence_system();
    asm volatile("bar.sync 1, 128;\n" ::: "memory");
    if (threadIdx.x == 64) {
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

static bool encode_2d(CUtensorMap* map, const void* base, int rows, int cols, int ld_elems, int box_rows) {
  PFN_encodeTiled enc = get_encode();
  if (!enc) return false;
  const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)ld_elems * 2};
  const cuuint32_t box[2] = {64, (cuuint32_t)box_rows};
  const cuuint32_t estr[2] = {1, 1};
  return enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int BN, int MODE, bool DEC>
static cudaError_t launch_bf16(const CUtensorMap& ma, const CUtensorMap& mb, const DenseGemmArgs& a, dim3 grid,
                               cudaStream_t s) {
  static bool set = false;
  constexpr size_t smem = Bf16Cfg<BN>::SMEM;
  auto* kern = tc_gemm_bf16_kernel<BN, MODE, DEC>;
  if (!set) {
    const cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    set = true;
  }
  if (a.splits == 1) {
    kern<<<grid, BF_THREADS, smem, s>>>(ma, mb, a);
    return cudaGetLastError();
  }
  // the K slices of one row tile form a cluster (1 x splits): partials meet in its shared memory
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(BF_THREADS);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 1;
  attr[0].val.clusterDim.y = (unsigned)a.splits;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, ma, mb, a);
}

// One instantiation per (tile width, epilogue, orientation): each kernel carries only its own
// epilogue code (a small kernel's time is otherwise dominated by instruction fetch on every SM).
template <int BN, bool DEC>
static cudaError_t launch_mode(const CUtensorMap& ma, const CUtensorMap& mb, const DenseGemmArgs& a, dim3 grid,
                               cudaStream_t s) {
  switch (a.mode) {
    case 0: return launch_bf16<BN, 0, DEC>(ma, mb, a, grid, s);
    case 1: return launch_bf16<BN, 1, DEC>(ma, mb, a, grid, s);
    case 3: return launch_bf16<BN, 3, DEC>(ma, mb, a, grid, s);
    case 5: return launch_bf16<BN, 5, DEC>(ma, mb, a, grid, s);
    case 6: return launch_bf16<BN, 6, DEC>(ma, mb, a, grid, s);
    default: return cudaErrorInvalidValue;
  }
}

// Split-K plan of the decode orientation: the K slices per row tile so that the grid fills
// about two waves of the SMs, with at least 4 stages of K per slice.
int bf16_gemm_splits(int N, int K, int T) {
  if (T >= 128) return 1;
  const int tiles = (N + 127) / 128, kb = K / 64;
  int s = 1;
  // K slices (a cluster of at most 8 CTAs) while the grid stays within two CTAs per SM and
  // each slice keeps at least 4 K stages
  while (s < 8 && tiles * s * 2 <= 2 * num_sms() && kb / (s * 2) >= 4) s *= 2;
  return s;
}

size_t bf16_gemm_ws_floats(int, int, int) { return 0; }  // split-K partials stay on chip

cudaError_t launch_tc_gemm_bf16(const void* x, int T, int ldx, const void* w, int N, int K, int mode, void* out,
                                int ldo, float* ws, size_t ws_floats, unsigned* counters, const PeerPush* pp,
                                int* status, cudaStream_t s) {
  // N % 32: whole 32-column epilogue groups (prefill orientation); partial 128-row weight tiles
  // of the decode orientation read zeros past N (TMA fill) and store nothing there
  if (T <= 0 || N % 32 || K % 64 || K < 64) return cudaErrorInvalidValue;
  if ((reinterpret_cast<uintptr_t>(x) & 15) || (reinterpret_cast<uintptr_t>(w) & 15) || (ldx * 2) % 16)
    return cudaErrorInvalidValue;
  if (mode == 1 && N % 16) return cudaErrorInvalidValue;
  if (mode == 6 && pp == nullptr) return cudaErrorInvalidValue;
  DenseGemmArgs a;
  memset(&a, 0, sizeof(a));
  a.T = T;
  a.N = N;
  a.K = K;
  a.mode = mode;
  a.out = out;
  a.ldo = ldo;
  a.status = status;
  {
    const int esz = (mode == 0 || mode == 1) ? 2 : 4;
    a.vec_out = (reinterpret_cast<uintptr_t>(out) & 15) == 0 && ((int64_t)ldo * esz) % 16 == 0;
  }
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
  CUtensorMap ma, mb;
  if (T < 128) {
    // decode: weights are the 128-row operand, tokens the N operand (zero-filled past T)
    const int bn = T <= 32 ? 32 : T <= 64 ? 64 : 128;
    a.decode = 1;
    a.splits = bf16_gemm_splits(N, K, T);
    if (!encode_2d(&ma, w, N, K, K, 128) || !encode_2d(&mb, x, T, K, ldx, bn)) return cudaErrorInvalidValue;
    const dim3 grid((unsigned)((N + 127) / 128), (unsigned)a.splits);
    if (bn == 32) return launch_mode<32, true>(ma, mb, a, grid, s);
    if (bn == 64) return launch_mode<64, true>(ma, mb, a, grid, s);
    return launch_mode<128, true>(ma, mb, a, grid, s);
  }
  // prefill: tokens are the 128-row operand, BN output columns per CTA
  const int bn = N % 256 == 0 ? 256 : 128;
  a.decode = 0;
  a.splits = 1;
  if (!encode_2d(&ma, x, T, K, ldx, 128) || !encode_2d(&mb, w, N, K, K, bn)) return cudaErrorInvalidValue;
  const dim3 grid((unsigned)((T + 127) / 128), (unsigned)((N + bn - 1) / bn));
  if (bn == 256) return launch_mode<256, false>(ma, mb, a, grid, s);
  return launch_mode<128, false>(ma, mb, a, grid, s);
}

}  // namespace syn
