// Shared helpers of the tcgen05 kernels (sm_100a): mbarriers with bounded waits, TMA and
// bulk async copies into shared memory, the SWIZZLE_128B K-major UMMA descriptor, kind::f16
// MMA issue / commit, and TMEM loads.  Every wait is bounded (an error bit, never a hang).
#pragma once
#include <cuda.h>

#include "common.cuh"
#include "sync.cuh"

namespace syn {

constexpr int TC_BM = 128;   // rows of one MMA subtile
constexpr uint64_t TC_WAIT_NS = 2000000000ull;  // 2 s: far above any legitimate stage wait

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint64_t* b, uint32_t n) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(smem_u32(b)), "r"(n));
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* b, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(smem_u32(b)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* b) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" ::"r"(smem_u32(b)) : "memory");
}
__device__ __forceinline__ bool mbar_test(uint64_t* b, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(b)), "r"(parity)
      : "memory");
  return ok != 0;
}
// try_wait with a suspend-time hint: the waiting warp sleeps until the phase completes (or
// the hint, 64 us, runs out) instead of spinning, so waiting warps leave the issue slots to
// the warps that work.
__device__ __forceinline__ bool mbar_test_sleep(uint64_t* b, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(b)), "r"(parity), "r"(65536u)
      : "memory");
  return ok != 0;
}
// Bounded wait on an mbarrier phase; false (with an error bit) after TC_WAIT_NS.
__device__ __forceinline__ bool mbar_wait(uint64_t* b, uint32_t parity, int* status, volatile int* abort) {
  if (mbar_test(b, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  while (!mbar_test_sleep(b, parity)) {
    if (*abort) return false;
    if (globaltimer_ns() - t0 > TC_WAIT_NS) {
      *abort = 1;
      if (status) atomicOr(status, 1 << 4);
      return false;
    }
  }
  return true;
}

__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n" ::"r"(
                   smem_u32(dst)),
               "l"(src), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void tma_load_4d(void* dst, const CUtensorMap* map, int c0, int c1, int c2, int c3,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, %5}], "
      "[%6];\n" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int c0, int c1, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];\n" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(smem_u32(bar))
      : "memory");
}

// K-major, SWIZZLE_128B smem matrix descriptor (rows of 128 bytes, 8-row atoms 1024 B apart).
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)1 << 16;            // leading byte offset (unused for swizzled K-major)
  d |= (uint64_t)(1024 >> 4) << 32;  // stride byte offset: next 8-row group
  d |= (uint64_t)1 << 46;            // descriptor version (sm_100)
  d |= (uint64_t)2 << 61;            // SWIZZLE_128B
  return d;
}

template <int BN>
__device__ __forceinline__ constexpr uint32_t idesc_bf16_f32() {
  return (1u << 4)                 // D: f32
         | (1u << 7)               // A: bf16
         | (1u << 10)              // B: bf16
         | ((uint32_t)(BN >> 3) << 17)
         | ((uint32_t)(TC_BM >> 4) << 24);
}

__device__ __forceinline__ void umma_bf16(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(d_tmem),
      "l"(a), "l"(b), "r"(idesc), "r"(acc));
}
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];\n"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory");
}


// ---- host side: the driver's tensor-map encoder, looked up once through the runtime ----
typedef CUresult (*PFN_encodeTiled)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                    const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                    CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static inline PFN_encodeTiled get_encode() {
  static PFN_encodeTiled fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_encodeTiled>(p);
  }
  return fn;
}

// 4-D tensor maps over a contiguous bank of packed 4-bit matrices [entries][N/16][K/64]:
// nibbles 512 B and scale/min 128 B per (16-row tile, 64-column block); one box = BN/16 tiles.
static inline bool encode_q4_raw_maps(PFN_encodeTiled enc, CUtensorMap* mq, CUtensorMap* ms, const void* bank_qw,
                            const void* bank_sm, int entries, int N, int K, int BN) {
  const cuuint64_t KG = (cuuint64_t)(K / 64), NT = (cuuint64_t)(N / 16);
  const cuuint32_t estr[4] = {1, 1, 1, 1};
  const cuuint64_t dq[4] = {128, KG, NT, (cuuint64_t)entries};  // [entry][tile][kg][128 x u32]
  const cuuint64_t sq[3] = {512, 512 * KG, 512 * KG * NT};
  const cuuint32_t bq[4] = {128, 1, (cuuint32_t)(BN / 16), 1};
  if (enc(mq, CU_TENSOR_MAP_DATA_TYPE_UINT32, 4, const_cast<void*>(bank_qw), dq, sq, bq, estr,
          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return false;
  const cuuint64_t ds[4] = {32, KG, NT, (cuuint64_t)entries};    // [entry][tile][kg][32 x u32]
  const cuuint64_t ss[3] = {128, 128 * KG, 128 * KG * NT};
  const cuuint32_t bs[4] = {32, 1, (cuuint32_t)(BN / 16), 1};
  return enc(ms, CU_TENSOR_MAP_DATA_TYPE_UINT32, 4, const_cast<void*>(bank_sm), ds, ss, bs, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}


// ---- epilogue staging: a warp's 32-row output block stored row-major ----
// After tcgen05.ld each lane holds one output row.  Storing from there writes 32 rows per
// instruction; instead each lane writes its row's 16-byte chunks into a 4 KB staging block
// and the warp stores the block back row-major, 16 bytes per lane.
// stg_off<C>: byte offset of chunk c of row `row`, rows of C chunks (C = 2, 4, 8: 32, 64, 128
// bytes) packed 8 / C to a 128-byte line, chunk position XORed with the line index, so the
// row-per-lane writes (8 lanes = 8 rows per phase) and the row-major reads (8 lanes = one
// line) both touch all 32 banks.
template <int C>
__device__ __forceinline__ uint32_t stg_off(int row, int c) {
  constexpr int L = 8 / C;  // rows per 128-byte line
  const int line = row / L;
  return (uint32_t)(line * 128 + ((((row % L) * C + c) ^ (line & 7)) << 4));
}

// Stores rows [0, nrows) of the staged block to out + row * row_bytes (16-byte aligned rows);
// ADD: f32 elements added to what is there.  Warp-collective.
template <int C, bool ADD = false>
__device__ __forceinline__ void stg_flush(const uint8_t* stg, int lane, uint8_t* out, int64_t row_bytes,
                                          int nrows) {
  __syncwarp();
  constexpr int RPI = 32 / C;  // rows per store instruction
#pragma unroll
  for (int rr = 0; rr < 32; rr += RPI) {
    const int rw = rr + lane / C, c = lane % C;
    if (rw < nrows) {
      uint4* o = reinterpret_cast<uint4*>(out + rw * row_bytes + c * 16);
      uint4 v = *reinterpret_cast<const uint4*>(stg + stg_off<C>(rw, c));
      if constexpr (ADD) {
        const uint4 u = *o;
        v.x = __float_as_uint(__uint_as_float(u.x) + __uint_as_float(v.x));
        v.y = __float_as_uint(__uint_as_float(u.y) + __uint_as_float(v.y));
        v.z = __float_as_uint(__uint_as_float(u.z) + __uint_as_float(v.z));
        v.w = __float_as_uint(__uint_as_float(u.w) + __uint_as_float(v.w));
      }
      *o = v;
    }
  }
  __syncwarp();  // the block is rewritten next
}

// Row r of the staged block from 32 accumulator columns v (lane = row): SwiGLU over the
// interleaved 8-column gate / up chunks (16 bf16 out, C = 2), bf16 (C = 4), f32 * sc (C = 8).
__device__ __forceinline__ void stg_put_swiglu(uint8_t* stg, int lane, const float* v) {
  uint32_t w[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    float o2[2];
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const int jj = 2 * j + e, gi = (jj / 8) * 16 + (jj % 8);
      o2[e] = silu(v[gi]) * v[gi + 8];
    }
    w[j] = pack_bf16x2(o2[0], o2[1]);
  }
#pragma unroll
  for (int c = 0; c < 2; ++c)
    *reinterpret_cast<uint4*>(stg + stg_off<2>(lane, c)) = make_uint4(w[4 * c], w[4 * c + 1], w[4 * c + 2], w[4 * c + 3]);
}
__device__ __forceinline__ void stg_put_bf16(uint8_t* stg, int lane, const float* v) {
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    uint4 w;
    w.x = pack_bf16x2(v[8 * c + 0], v[8 * c + 1]);
    w.y = pack_bf16x2(v[8 * c + 2], v[8 * c + 3]);
    w.z = pack_bf16x2(v[8 * c + 4], v[8 * c + 5]);
    w.w = pack_bf16x2(v[8 * c + 6], v[8 * c + 7]);
    *reinterpret_cast<uint4*>(stg + stg_off<4>(lane, c)) = w;
  }
}
__device__ __forceinline__ void stg_put_f32(uint8_t* stg, int lane, const float* v, float sc) {
#pragma unroll
  for (int c = 0; c < 8; ++c)
    *reinterpret_cast<float4*>(stg + stg_off<8>(lane, c)) =
        make_float4(sc * v[4 * c], sc * v[4 * c + 1], sc * v[4 * c + 2], sc * v[4 * c + 3]);
}

}  // namespace syn
