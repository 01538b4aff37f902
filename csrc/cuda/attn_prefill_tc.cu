// Causal prefill attention (GQA, head_dim 128) over the paged KV cache on the 5th-generation
// tensor cores: S = Q K^T and O_j = P_j V_j are tcgen05.mma kind::f16 (bf16 operands, f32
// accumulators in TMEM) fed by TMA; the online softmax runs on four warps that read S out of
// TMEM and write P (bf16) back to shared memory for the second product.  Same contract as
// attn_prefill.cu: query row i of sequence s sits at absolute position kv_len[s] - q_len[s] + i
// and attends to keys 0..that position through the sequence's block table (plain prefill and
// chunked prefill after a cached prefix).  Reference op: `AttnPrefill(Gqa)`
// (crates/kernels/src/op/kind.rs; f32 reference crates/kernels/src/reference/attention.rs).
//
// One CTA = 256 query rows of one head (query tiles A and B of 128 rows), 320 threads:
//   warp 0      TMA producer: both Q tiles once (two 64-column halves each), then per 128-key
//               tile the K and V pages (16 keys x 64 columns per box, 16 boxes each) into a
//               2-stage ring;
//   warp 1      TMEM owner and MMA issuer (one elected lane), ping-pong over the two tiles: per
//               key tile j it issues P_A V, S_A(j+1), P_B V, S_B(j+1), so the tensor core works on
//               one tile while the softmax warps of the other run; O_A and O_B accumulate in TMEM;
//   warps 2..5  softmax of tile A, warps 6..9 of tile B (thread = query row = TMEM lane): one
//               read of the S row (its S columns are released at once), causal / length mask,
//               row max, P = 2^(S * scale - m) in bf16 into the shared P buffer (SWIZZLE_128B
//               K-major, as the next MMA reads it; the tiles take it in turn).  The running max
//               is raised lazily: only when a row's new max exceeds it by more than 2^8 is its
//               O (in TMEM) rescaled, after that tile's previous P V.
// TMEM: S_A, S_B, O_A, O_B (128 columns each).  V is the MN-major B operand of P V (its rows are
// keys, 64 head-dim columns per 128-byte row).  Every mbarrier wait is bounded: a wait that
// runs out sets bit 4 of *status and every role leaves its loop.
#include <cuda.h>

#include "common.cuh"
#include "syn/launch.h"
#include "tc_common.cuh"

namespace syn {

namespace {

constexpr int AT_D = 128;
constexpr int AT_BM = 128;                   // query rows per CTA (TMEM lanes)
constexpr int AT_BN = 128;                   // keys per tile
constexpr int AT_HALF = 128 * 128;           // one 64-column half of a 128-row tile: 16 KB
constexpr int AT_TILE = 2 * AT_HALF;         // 32 KB
constexpr int AT_SMEM = 7 * AT_TILE + 1024;  // Q[2 tiles], K[2], V[2], P + alignment slack
constexpr int AT_THREADS = 320;

struct AttnTcArgs {
  const int32_t* block_tables;  // [nseq, max_blocks]
  const int32_t* cu_q;          // [nseq + 1]
  const int32_t* kv_lens;       // [nseq]
  __nv_bfloat16* out;           // [Tq, Hq, D]
  int Hq, Hkv, max_blocks, n_qtiles;
  float scale_log2;
  int* status;
};

__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, int c0, int c1, int c2,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], "
      "[%5];\n" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(smem_u32(bar))
      : "memory");
}

// MN-major SWIZZLE_128B descriptor: 64 MN elements per 128-byte row, the next 64 MN elements
// `lbo` bytes further, K rows 128 bytes apart in 8-row atoms whose groups are 1024 bytes apart.
__device__ __forceinline__ uint64_t sw128_mn_desc(uint32_t saddr, uint32_t lbo) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)(1024 >> 4) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}

__device__ __forceinline__ void tmem_ld32_async(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];\n"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}
// 2^x in one MUFU operation (ex2.approx.ftz: ~2 ulp, flush-to-zero; P is rounded to bf16)
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory"); }

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t* r) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};\n" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]),
      "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]),
      "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}

// kind::f16, bf16 x bf16 -> f32, M = 128, N = 128; b_mn: B operand MN-major
__device__ __forceinline__ constexpr uint32_t at_idesc(bool b_mn) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((b_mn ? 1u : 0u) << 16) | ((uint32_t)(AT_BN >> 3) << 17) |
         ((uint32_t)(AT_BM >> 4) << 24);
}

__global__ void __launch_bounds__(AT_THREADS, 1)
    attn_prefill_tc_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                           const __grid_constant__ CUtensorMap tm_v, AttnTcArgs a) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;                // [2 query tiles]
  uint8_t* sK = sQ + 2 * AT_TILE;    // [2 stages]
  uint8_t* sV = sK + 2 * AT_TILE;    // [2 stages]
  uint8_t* sP = sV + 2 * AT_TILE;    // one P buffer, used by the two query tiles in turn
  __shared__ __align__(8) uint64_t q_full, k_full[2], v_full[2], kv_empty[2], s_full[2], s_free[2], p_full[2],
      pv_done[2], p_free, o_done;
  __shared__ uint32_t tmem_base;
  __shared__ volatile int s_abort;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int s = blockIdx.z, h = blockIdx.y;
  const int qt = a.n_qtiles - 1 - (int)blockIdx.x;  // longest (latest) tiles first
  const int q0 = a.cu_q[s], q_len = a.cu_q[s + 1] - q0;
  const int i0 = qt * 2 * AT_BM;                      // 256 query rows per CTA: tiles A and B
  if (i0 >= q_len) return;  // uniform over the CTA, before any barrier or TMEM use
  const int kv_len = a.kv_lens[s];
  const int pos0 = kv_len - q_len;
  const int hk = h / (a.Hq / a.Hkv);
  // key tiles each query tile needs (0 for a tile past the sequence's rows)
  int n_t[2];
#pragma unroll
  for (int g = 0; g < 2; ++g) {
    const int r0 = i0 + g * AT_BM;
    n_t[g] = r0 < q_len ? (pos0 + min(r0 + AT_BM, q_len) - 1) / AT_BN + 1 : 0;
  }
  const int n_max = max(n_t[0], n_t[1]);

  if (threadIdx.x == 0) {
    s_abort = 0;
    mbar_init(&q_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&v_full[i], 1);
      mbar_init(&kv_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&s_free[i], 128);
      mbar_init(&p_full[i], 128);
      mbar_init(&pv_done[i], 1);
    }
    mbar_init(&p_free, 1);
    mbar_init(&o_done, 1);
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(smem_u32(&tmem_base)),
                 "r"(512));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n");
  }
  asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory");
  const uint32_t tmem = tmem_base;
  // TMEM: S of tile g at columns 128 g, O of tile g at 256 + 128 g

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      const int32_t* bt = a.block_tables + (int64_t)s * a.max_blocks;
      const int n_pages = (kv_len + 15) >> 4;
      mbar_expect_tx(&q_full, 2 * AT_TILE);
#pragma unroll
      for (int g = 0; g < 2; ++g) {  // rows past the tensor read zeros; rows of the next sequence are masked out
        tma_load_3d(sQ + g * AT_TILE, &tm_q, 0, h, q0 + i0 + g * AT_BM, &q_full);
        tma_load_3d(sQ + g * AT_TILE + AT_HALF, &tm_q, 64, h, q0 + i0 + g * AT_BM, &q_full);
      }
      for (int j = 0; j < n_max; ++j) {
        const int st = j & 1;
        if (j >= 2 && !mbar_wait(&kv_empty[st], ((j >> 1) - 1) & 1, a.status, &s_abort)) break;
        int blk[8];
#pragma unroll
        for (int p = 0; p < 8; ++p) blk[p] = bt[min(j * 8 + p, n_pages - 1)];  // past the end: a real page, masked
        mbar_expect_tx(&k_full[st], AT_TILE);
#pragma unroll
        for (int p = 0; p < 8; ++p) {
          tma_load_4d(sK + st * AT_TILE + p * 2048, &tm_k, 0, 0, hk, blk[p], &k_full[st]);
          tma_load_4d(sK + st * AT_TILE + AT_HALF + p * 2048, &tm_k, 64, 0, hk, blk[p], &k_full[st]);
        }
        mbar_expect_tx(&v_full[st], AT_TILE);
#pragma unroll
        for (int p = 0; p < 8; ++p) {
          tma_load_4d(sV + st * AT_TILE + p * 2048, &tm_v, 0, 0, hk, blk[p], &v_full[st]);
          tma_load_4d(sV + st * AT_TILE + AT_HALF + p * 2048, &tm_v, 64, 0, hk, blk[p], &v_full[st]);
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer: S_A(j+1), P_B V and S_B(j+1) overlap the softmax of the other tile ----
    if (lane == 0) {
      constexpr uint32_t id_s = at_idesc(false), id_o = at_idesc(true);
      const uint32_t up = smem_u32(sP);
      auto issue_s = [&](int g, int j) -> bool {  // S_g(j) into tile g's S columns
        if (j >= 1 && !mbar_wait(&s_free[g], (j - 1) & 1, a.status, &s_abort)) return false;
        if (!mbar_wait(&k_full[j & 1], (j >> 1) & 1, a.status, &s_abort)) return false;
        asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory");
        const uint32_t uq = smem_u32(sQ + g * AT_TILE), uk = smem_u32(sK + (j & 1) * AT_TILE);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint32_t off = (kk >> 2) * AT_HALF + (kk & 3) * 32;
          umma_bf16(tmem + g * 128, sw128_desc(uq + off), sw128_desc(uk + off), id_s, kk != 0);
        }
        umma_commit(&s_full[g]);
        return true;
      };
      auto issue_pv = [&](int g, int j) -> bool {  // O_g += P_g(j) V_j
        if (!mbar_wait(&p_full[g], j & 1, a.status, &s_abort)) return false;
        if (!mbar_wait(&v_full[j & 1], (j >> 1) & 1, a.status, &s_abort)) return false;
        asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory");
        const uint32_t uv = smem_u32(sV + (j & 1) * AT_TILE);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint32_t aoff = (kk >> 2) * AT_HALF + (kk & 3) * 32;
          umma_bf16(tmem + 256 + g * 128, sw128_desc(up + aoff), sw128_mn_desc(uv + kk * 2048, AT_HALF), id_o,
                    (j | kk) != 0);
        }
        umma_commit(&pv_done[g]);
        return true;
      };
      bool ok = mbar_wait(&q_full, 0, a.status, &s_abort);
      for (int g = 0; ok && g < 2; ++g)
        if (n_t[g] > 0) ok = issue_s(g, 0);
      for (int j = 0; ok && j < n_max; ++j) {
        // the P buffer serves A(j), B(j), A(j+1), ...: one p_free phase per slot (an empty
        // commit for a tile that has no key tile j), so each softmax waits a fixed parity
#pragma unroll
        for (int g = 0; g < 2; ++g) {
          if (!ok) break;
          if (j < n_t[g]) {
            ok = issue_pv(g, j);
            if (ok && j + 1 < n_t[g]) ok = issue_s(g, j + 1);
          }
          umma_commit(&p_free);
        }
        umma_commit(&kv_empty[j & 1]);
      }
      umma_commit(&o_done);
    }
  } else if (warp >= 2 && warp < 10) {
    // ---------------- softmax: warps 2..5 query tile A, 6..9 tile B ----------------
    const int g = (warp - 2) >> 2;
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;                 // query row in the tile = TMEM lane
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const int row0 = i0 + g * AT_BM;
    const int prow = pos0 + row0 + r;                  // absolute position of this query
    const int pmin = pos0 + row0;                      // first query position of the tile
    const float sl2 = a.scale_log2;
    const uint32_t t_s = tmem + g * 128 + lane_off, t_o = tmem + 256 + g * 128 + lane_off;
    const int nt = n_t[g];
    float m_used = -INFINITY, l_run = 0.f;  // m_used: the max the exponentials subtract
    bool ok = true;
    for (int j = 0; j < nt; ++j) {
      // tcgen05.ld / st are warp-collective: every branch around them is decided warp-uniformly
      if (!__all_sync(0xffffffffu, mbar_wait(&s_full[g], j & 1, a.status, &s_abort))) {
        ok = false;
        break;
      }
      asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory");
      // one read of the S row (four loads, one wait); its S columns are free for S_g(j+1) at once
      uint32_t u[AT_BN];
#pragma unroll
      for (int c0 = 0; c0 < AT_BN; c0 += 32) tmem_ld32_async(t_s + c0, u + c0);
      tmem_wait_ld();
      asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory");
      mbar_arrive(&s_free[g]);
      const int key0 = j * AT_BN;
      if (key0 + AT_BN - 1 > pmin || key0 + AT_BN > kv_len) {  // causal / length mask
#pragma unroll
        for (int i = 0; i < AT_BN; ++i) {
          const int key = key0 + i;
          if (key > prow || key >= kv_len) u[i] = __float_as_uint(-INFINITY);
        }
      }
      float mx = -INFINITY;
#pragma unroll
      for (int i = 0; i < AT_BN; ++i) mx = fmaxf(mx, __uint_as_float(u[i]));
      mx *= sl2;
      const bool raise = mx > m_used + 8.f;  // always on the first tile (m_used = -inf)
      const float m_new = raise ? mx : m_used;
      const float alpha = ex2_approx(m_used - m_new);  // 1 where the max stays, 0 on the first tile
      m_used = m_new;
      // the shared P buffer: tile A's slot j follows tile B's slot j-1 (phase 2j-1), tile B's
      // slot j follows tile A's slot j (phase 2j)
      if ((g == 1 || j >= 1) &&
          !__all_sync(0xffffffffu, mbar_wait(&p_free, g == 0 ? 1u : 0u, a.status, &s_abort))) {
        ok = false;
        break;
      }
      float rs = 0.f;
      uint8_t* pbuf = sP + r * 128;
#pragma unroll
      for (int c0 = 0; c0 < AT_BN; c0 += 32) {
        uint32_t pk[16];
#pragma unroll
        for (int i = 0; i < 32; i += 2) {
          const float p0 = ex2_approx(fmaf(__uint_as_float(u[c0 + i]), sl2, -m_used));
          const float p1 = ex2_approx(fmaf(__uint_as_float(u[c0 + i + 1]), sl2, -m_used));
          rs += p0 + p1;
          pk[i >> 1] = pack_bf16x2(p0, p1);
        }
        uint8_t* prow_base = pbuf + (c0 >> 6) * AT_HALF;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int chunk = ((c0 & 63) >> 3) + q;  // 16-byte chunk of the 128-byte row
          *reinterpret_cast<uint4*>(prow_base + ((chunk ^ (r & 7)) << 4)) =
              make_uint4(pk[4 * q], pk[4 * q + 1], pk[4 * q + 2], pk[4 * q + 3]);
        }
      }
      l_run = l_run * alpha + rs;
      // a raised max: O (tiles 0..j-1) is rescaled now, with the S row out of the registers,
      // after P_g(j-1) V has finished and before P_g(j) V is issued
      if (__any_sync(0xffffffffu, raise) && j > 0) {
        if (!__all_sync(0xffffffffu, mbar_wait(&pv_done[g], (j - 1) & 1, a.status, &s_abort))) {
          ok = false;
          break;
        }
        asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory");
#pragma unroll 1
        for (int c0 = 0; c0 < AT_D; c0 += 32) {
          uint32_t o[32];
          tmem_ld32_async(t_o + c0, o);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
          tmem_st32(t_o + c0, o);
        }
        asm volatile("tcgen05.wait::st.sync.aligned;\n" ::: "memory");
      }
      // P visible to the tensor core (async proxy), then handed over
      asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
      asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory");
      mbar_arrive(&p_full[g]);
    }
    if (ok && nt > 0 && __all_sync(0xffffffffu, mbar_wait(&o_done, 0, a.status, &s_abort))) {
      asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory");
      const int i = row0 + r;
      const float inv = 1.f / l_run;
      uint4* orow = reinterpret_cast<uint4*>(a.out + ((int64_t)(q0 + min(i, q_len - 1)) * a.Hq + h) * AT_D);
#pragma unroll 1
      for (int c0 = 0; c0 < AT_D; c0 += 32) {
        uint32_t o[32];
        tmem_ld32_async(t_o + c0, o);
        tmem_wait_ld();
        if (i < q_len) {
#pragma unroll
          for (int c = 0; c < 32; c += 8)
            orow[(c0 + c) >> 3] =
                make_uint4(pack_bf16x2(__uint_as_float(o[c]) * inv, __uint_as_float(o[c + 1]) * inv),
                           pack_bf16x2(__uint_as_float(o[c + 2]) * inv, __uint_as_float(o[c + 3]) * inv),
                           pack_bf16x2(__uint_as_float(o[c + 4]) * inv, __uint_as_float(o[c + 5]) * inv),
                           pack_bf16x2(__uint_as_float(o[c + 6]) * inv, __uint_as_float(o[c + 7]) * inv));
        }
      }
    }
  }
  asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory");
  __syncthreads();
  if (warp == 1) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(tmem), "r"(512));
  }
}

}  // namespace

cudaError_t launch_attn_prefill_tc(const void* q, int Tq, const void* kc, const void* vc, int n_blocks,
                                   const int32_t* block_tables, const int32_t* cu_q, const int32_t* kv_lens, void* out,
                                   int nseq, int max_q_len, int Hq, int Hkv, int D, int max_blocks, float scale,
                                   int* status, cudaStream_t s) {
  if (D != AT_D || Hq % Hkv || nseq <= 0 || max_q_len <= 0 || Tq <= 0 || n_blocks <= 0) return cudaErrorInvalidValue;
  if ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(kc) | reinterpret_cast<uintptr_t>(vc) |
       reinterpret_cast<uintptr_t>(out)) & 15)
    return cudaErrorMisalignedAddress;
  PFN_encodeTiled enc = get_encode();
  if (!enc) return cudaErrorNotSupported;
  CUtensorMap mq, mk, mv;
  {
    const cuuint64_t dims[3] = {(cuuint64_t)D, (cuuint64_t)Hq, (cuuint64_t)Tq};
    const cuuint64_t strides[2] = {(cuuint64_t)D * 2, (cuuint64_t)Hq * D * 2};
    const cuuint32_t box[3] = {64, 1, AT_BM};
    const cuuint32_t es[3] = {1, 1, 1};
    if (enc(&mq, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(q), dims, strides, box, es,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return cudaErrorInvalidValue;
  }
  for (int w = 0; w < 2; ++w) {
    const cuuint64_t dims[4] = {(cuuint64_t)D, 16, (cuuint64_t)Hkv, (cuuint64_t)n_blocks};
    const cuuint64_t strides[3] = {(cuuint64_t)D * 2, (cuuint64_t)16 * D * 2, (cuuint64_t)Hkv * 16 * D * 2};
    const cuuint32_t box[4] = {64, 16, 1, 1};
    const cuuint32_t es[4] = {1, 1, 1, 1};
    if (enc(w ? &mv : &mk, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(w ? vc : kc), dims, strides, box,
            es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return cudaErrorInvalidValue;
  }
  static bool set = false;
  if (!set) {
    cudaError_t e = cudaFuncSetAttribute(attn_prefill_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, AT_SMEM);
    if (e != cudaSuccess) return e;
    set = true;
  }
  AttnTcArgs a{block_tables, cu_q, kv_lens, reinterpret_cast<__nv_bfloat16*>(out), Hq, Hkv, max_blocks,
               (max_q_len + 2 * AT_BM - 1) / (2 * AT_BM), scale * 1.4426950408889634f, status};
  dim3 grid((unsigned)a.n_qtiles, (unsigned)Hq, (unsigned)nseq);
  attn_prefill_tc_kernel<<<grid, AT_THREADS, AT_SMEM, s>>>(mq, mk, mv, a);
  return cudaGetLastError();
}

}  // namespace syn
