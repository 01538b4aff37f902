// Cold experts on the host CPU during decode (reference crates/kernels-cpu/src/moe.rs: expert
// misses as tasks per (expert, output-row block); crates/kernels/src/moe/doorbell.rs: the
// hand-off through host-mapped memory).
//
// The weights stay in the device's tiled 4-bit layout (syn/q4.h) inside the pinned host tier
// that the GPU also reads over PCIe, so an expert moves between the CPU and the PCIe path with
// no copy.  In that layout the 64 bytes of lanes 4g..4g+3 of one (16-row tile, 64-column group)
// hold rows g and g+8 over all 64 columns, and ((word >> 4j) & 0x000F000F) is a pair of
// consecutive columns of one row (j = 0, 2: row g; j = 1, 3: row g+8; j = 2, 3 are 8 columns
// further).  Two kernel families consume these pairs (each activation row is packed once per
// layer into the same pair order, with its per-block sums):
//  * BF16: OR-ing 0x4300 into a nibble gives the bf16 number 128 + q exactly, so
//    `vdpbf16ps` multiplies bf16 pairs exactly and
//        sum_k (d q_k + m) x_k = d * sum_k (128 + q_k) x_k + (m - 128 d) * sum_k x_k;
//  * VNNI int16: the activation row is scaled to int16 (s = max|x| / 32767, rounding error at
//    most s / 2 per element), `vpdpwssd` sums q * v exactly in int32 per block, and
//    y ~= s * sum_b d_b * sum_k q_k v_k + sum_b m_b * sum_k x_k (sum x exact).
// Both agree with the f32 product to ~1e-5 relative.  Which one is faster depends on the host's
// `vdpbf16ps` rate, so the default is the faster of the two, timed once per process
// (`calibrate_mode`).
//
// Threads: a fixed pool pinned to the given CPUs.  Thread 0 polls the mailbox's go word; on a
// new sequence it lists the routed pairs of the experts this tier owns for that layer and
// releases the pool through four phases separated by barriers: pack the activation rows; gate
// and up tasks; SiLU-gate + pack; down tasks.  Then it writes the outputs' pair indices and
// release-stores the done word, which the GPU waits on with a time limit.
#ifdef SYN_NO_TORCH  // standalone build (the ThreadSanitizer test of the worker pool)
#include <stdexcept>
#define SYN_REQUIRE(c, msg) \
  do {                      \
    if (!(c)) throw std::runtime_error(msg); \
  } while (0)
#else
#include <torch/extension.h>
#define SYN_REQUIRE(c, msg) TORCH_CHECK(c, msg)
#endif

#include <immintrin.h>
#include <pthread.h>
#include <sched.h>
#include <time.h>

#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <thread>
#include <vector>

#include "syn/cpu_mailbox.h"
#include "syn/q4.h"

namespace syn {
namespace {

inline float bf2f_h(uint16_t v) {
  const uint32_t u = (uint32_t)v << 16;
  float f;
  std::memcpy(&f, &u, 4);
  return f;
}

inline uint16_t f2bf_h(float f) {  // round to nearest even
  uint32_t u;
  std::memcpy(&u, &f, 4);
  if ((u & 0x7fffffffu) > 0x7f800000u) return 0x7fc0;
  u += 0x7fffu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}

inline float h2f_h(uint16_t h) {  // IEEE binary16 -> f32 (scalar path)
  const int s = h >> 15, e = (h >> 10) & 31, m = h & 1023;
  float v;
  if (e == 0)
    v = std::ldexp((float)m, -24);
  else if (e == 31)
    v = m ? NAN : INFINITY;
  else
    v = std::ldexp((float)(m | 1024), e - 25);
  return s ? -v : v;
}

inline uint64_t now_ns() {
  timespec ts;
  clock_gettime(CLOCK_MONOTONIC, &ts);
  return (uint64_t)ts.tv_sec * 1000000000ull + ts.tv_nsec;
}

inline uint32_t load_acquire(const uint32_t* p) { return __atomic_load_n(p, __ATOMIC_ACQUIRE); }
inline void store_release(uint32_t* p, uint32_t v) { __atomic_store_n(p, v, __ATOMIC_RELEASE); }

// Activation row x[K] (bf16) -> per 64-column group kg: 16 pairs for the j = 0, 1 nibbles
// (columns 2t, 2t+1 of k-step w), 16 for j = 2, 3 (8 further), lane i = 4t + w, and the two
// block sums as (s0, 0, s1, 0).
void pack_row(const uint16_t* x, int K, uint32_t* ab, float* sx4) {
  const int KG = K >> 6;
  for (int kg = 0; kg < KG; ++kg) {
    for (int i = 0; i < 16; ++i) {
      const int t = i >> 2, w = i & 3;
      const int k = 64 * kg + 32 * (w >> 1) + 16 * (w & 1) + 2 * t;
      ab[kg * 32 + i] = (uint32_t)x[k] | ((uint32_t)x[k + 1] << 16);
      ab[kg * 32 + 16 + i] = (uint32_t)x[k + 8] | ((uint32_t)x[k + 9] << 16);
    }
    for (int b = 0; b < 2; ++b) {
      float s = 0.f;
      for (int j = 0; j < 32; ++j) s += bf2f_h(x[64 * kg + 32 * b + j]);
      sx4[kg * 4 + 2 * b] = s;
      sx4[kg * 4 + 2 * b + 1] = 0.f;
    }
  }
}

// Integer form of a row for the VNNI kernel: one scale per row, s = max|x| / 32767, and
// v_k = round(x_k / s) as int16 (|x_k - s v_k| <= s / 2: about 1e-4 of the row's largest
// element, far below the bf16 rounding the GPU path applies to the same activations), packed
// in the same pair order as `pack_row`; sxs holds s at every lane of every 64-column group (the
// kernel applies it once per output); sx4 the exact block sums of x as (s0, 0, s1, 0).
void pack_row_i16(const uint16_t* x, int K, uint32_t* ab, float* sxs, float* sx4) {
  const int KG = K >> 6;
  float amax = 0.f;
  for (int k = 0; k < K; ++k) amax = std::max(amax, std::fabs(bf2f_h(x[k])));
  const float sc = amax > 0.f ? amax / 32767.f : 1.f, inv = 1.f / sc;
  for (int kg = 0; kg < KG; ++kg) {
    int16_t v[64];
    for (int b = 0; b < 2; ++b) {
      float sum = 0.f;
      for (int j = 0; j < 32; ++j) {
        const float f = bf2f_h(x[64 * kg + 32 * b + j]);
        sum += f;
        const float q = std::nearbyint(f * inv);
        v[32 * b + j] = (int16_t)std::max(-32767.f, std::min(32767.f, q));
      }
      sx4[kg * 4 + 2 * b] = sum;
      sx4[kg * 4 + 2 * b + 1] = 0.f;
    }
    for (int i = 0; i < 16; ++i) {
      const int t = i >> 2, w = i & 3;
      const int k = 32 * (w >> 1) + 16 * (w & 1) + 2 * t;
      ab[kg * 32 + i] = (uint32_t)(uint16_t)v[k] | ((uint32_t)(uint16_t)v[k + 1] << 16);
      ab[kg * 32 + 16 + i] = (uint32_t)(uint16_t)v[k + 8] | ((uint32_t)(uint16_t)v[k + 9] << 16);
      sxs[kg * 16 + i] = sc;
    }
  }
}

// narrower int16 passes (4 / 2 row pairs) instead of 8 / 4: SYN_CPU_NARROW=1 (measurement)
const bool g_narrow_passes = [] {
  const char* e = getenv("SYN_CPU_NARROW");
  return e && atoi(e) == 1;
}();

// 64-column groups the int16 kernel prefetches ahead: 16 (8 KB of the tile) measured best with
// 14 workers streaming from DRAM (SYN_CPU_PREFETCH overrides, measurement)
const int g_prefetch_groups = [] {
  const char* e = getenv("SYN_CPU_PREFETCH");
  const int v = e ? atoi(e) : 0;
  return v > 0 && v <= 64 ? v : 16;
}();

// VNNI form of the product: nibble pairs as int16 (no magic number), activation pairs as int16,
// vpdpwssd sums q * v exactly in int32 per block; y = s * sum_b d_b * sum(q v) + sum_b m_b * sum(x)
// (s: the row's activation scale, applied once per output).
template <int NR, int GB>
__attribute__((target("avx512f,avx512bw,avx512vl,avx512vnni,f16c,fma"))) void tiles_vnni(
    const uint32_t* qw, const uint16_t* sm, int K, int tile0, int tile1, const uint32_t* const* ab,
    const float* const* sxs, const float* const* sx4, float* const* y, const float* scale) {
  const int KG = K >> 6;
  const __m512i M = _mm512_set1_epi32(0x000F000F);
  __m512i idx[4];
  for (int j = 0; j < 4; ++j)
    idx[j] = _mm512_add_epi32(_mm512_set1_epi32(4 * j), _mm512_set_epi32(2, 2, 0, 0, 2, 2, 0, 0, 2, 2, 0, 0, 2, 2, 0, 0));
  const __m512i swap = _mm512_set_epi32(14, 15, 12, 13, 10, 11, 8, 9, 6, 7, 4, 5, 2, 3, 0, 1);
  for (int tile = tile0; tile < tile1; ++tile) {
    const uint32_t* wt = qw + (int64_t)tile * KG * 128;
    const uint16_t* st = sm + (int64_t)tile * KG * 64;
    alignas(64) float cmin[NR][64];  // m * sum(x): row r of the tile at lanes 4*(r%4) + {0, 2} of vector r/4
    for (int r = 0; r < NR; ++r)
      for (int i = 0; i < 64; ++i) cmin[r][i] = 0.f;
    for (int kg = 0; kg < KG; ++kg) {
      const uint16_t* s = st + kg * 64;
      for (int q = 0; q < 4; ++q) {
        const __m512 F = _mm512_cvtph_ps(_mm256_loadu_si256(reinterpret_cast<const __m256i*>(s + 16 * q)));
        const __m512 G = _mm512_permutexvar_ps(swap, F);  // m at the even lanes
        for (int r = 0; r < NR; ++r) {
          const __m512 S = _mm512_broadcast_f32x4(_mm_loadu_ps(sx4[r] + kg * 4));
          _mm512_store_ps(&cmin[r][16 * q], _mm512_fmadd_ps(G, S, _mm512_load_ps(&cmin[r][16 * q])));
        }
      }
    }
    for (int g0 = 0; g0 < 8; g0 += GB) {
      __m512 alo[GB][NR], ahi[GB][NR];
      for (int gg = 0; gg < GB; ++gg)
        for (int r = 0; r < NR; ++r) {
          alo[gg][r] = _mm512_setzero_ps();
          ahi[gg][r] = _mm512_setzero_ps();
        }
      for (int kg = 0; kg < KG; ++kg) {
        const uint32_t* wp = wt + kg * 128 + 16 * g0;
        // g_prefetch_groups ahead: one thread streams from DRAM at its miss latency
        for (int l = 0; l < GB; ++l)
          _mm_prefetch(reinterpret_cast<const char*>(wp + g_prefetch_groups * 128 + 16 * l), _MM_HINT_T0);
        __m512i xa[NR], xb[NR];
        for (int r = 0; r < NR; ++r) {
          xa[r] = _mm512_loadu_si512(ab[r] + kg * 32);
          xb[r] = _mm512_loadu_si512(ab[r] + kg * 32 + 16);
        }
        const uint16_t* s = st + kg * 64;
#pragma GCC unroll 8
        for (int gg = 0; gg < GB; ++gg) {
          const int g = g0 + gg;
          const __m512 Flo = _mm512_cvtph_ps(_mm256_loadu_si256(reinterpret_cast<const __m256i*>(s + 16 * (g >> 2))));
          const __m512 Fhi =
              _mm512_cvtph_ps(_mm256_loadu_si256(reinterpret_cast<const __m256i*>(s + 16 * ((g + 8) >> 2))));
          const __m512 Dlo = _mm512_permutexvar_ps(idx[g & 3], Flo);
          const __m512 Dhi = _mm512_permutexvar_ps(idx[g & 3], Fhi);
          const __m512i W = _mm512_loadu_si512(wp + 16 * gg);
          const __m512i v0 = _mm512_and_si512(W, M);
          const __m512i v1 = _mm512_and_si512(_mm512_srli_epi32(W, 4), M);
          const __m512i v2 = _mm512_and_si512(_mm512_srli_epi32(W, 8), M);
          const __m512i v3 = _mm512_and_si512(_mm512_srli_epi32(W, 12), M);
          for (int r = 0; r < NR; ++r) {
            const __m512i t = _mm512_dpwssd_epi32(_mm512_dpwssd_epi32(_mm512_setzero_si512(), v0, xa[r]), v2, xb[r]);
            const __m512i u = _mm512_dpwssd_epi32(_mm512_dpwssd_epi32(_mm512_setzero_si512(), v1, xa[r]), v3, xb[r]);
            alo[gg][r] = _mm512_fmadd_ps(_mm512_cvtepi32_ps(t), Dlo, alo[gg][r]);
            ahi[gg][r] = _mm512_fmadd_ps(_mm512_cvtepi32_ps(u), Dhi, ahi[gg][r]);
          }
        }
      }
      for (int gg = 0; gg < GB; ++gg)
        for (int r = 0; r < NR; ++r) {
          const int g = g0 + gg;
          const float* clo = &cmin[r][16 * (g >> 2) + 4 * (g & 3)];
          const float* chi = &cmin[r][16 * ((g + 8) >> 2) + 4 * (g & 3)];
          // the row's activation scale, once per output (the same at every lane and group)
          const float sr = sxs[r][0];
          const float lo = _mm512_reduce_add_ps(alo[gg][r]) * sr + clo[0] + clo[2];
          const float hi = _mm512_reduce_add_ps(ahi[gg][r]) * sr + chi[0] + chi[2];
          y[r][tile * 16 + g] = lo * scale[r];
          y[r][tile * 16 + g + 8] = hi * scale[r];
        }
    }
  }
}

// BF16 family: y[r][n] = scale[r] * sum_k W[n][k] x_r[k] for the rows of tiles [tile0, tile1),
// NR rows; row pairs (g) outer, k-groups inner (the fastest order measured on a B200 node's host).
template <int NR>
__attribute__((target("avx512f,avx512bw,avx512vl,avx512bf16,f16c,fma"))) void tiles_avx512(
    const uint32_t* qw, const uint16_t* sm, int K, int tile0, int tile1, const uint32_t* const* ab,
    const float* const* sx4, float* const* y, const float* scale) {
  const int KG = K >> 6;
  const __m512i M = _mm512_set1_epi32(0x000F000F), C = _mm512_set1_epi32(0x43004300);
  // dword i of a 64-byte row slice belongs to 32-column block ((i & 3) >> 1); the converted
  // scale quad is (d0, m0, d1, m1)
  const __m512i idx = _mm512_set_epi32(2, 2, 0, 0, 2, 2, 0, 0, 2, 2, 0, 0, 2, 2, 0, 0);
  const __m128 c128 = _mm_set1_ps(128.f);
  for (int tile = tile0; tile < tile1; ++tile) {
    const uint32_t* wt = qw + (int64_t)tile * KG * 128;
    const uint16_t* st = sm + (int64_t)tile * KG * 64;
    for (int g = 0; g < 8; ++g) {
      __m512 alo[NR], ahi[NR];
      __m128 clo[NR], chi[NR];
      for (int r = 0; r < NR; ++r) {
        alo[r] = _mm512_setzero_ps();
        ahi[r] = _mm512_setzero_ps();
        clo[r] = _mm_setzero_ps();
        chi[r] = _mm_setzero_ps();
      }
      const uint32_t* wp = wt + 16 * g;
      for (int kg = 0; kg < KG; ++kg) {
        _mm_prefetch(reinterpret_cast<const char*>(wp + (kg + 6) * 128), _MM_HINT_T0);
        const __m512i W = _mm512_loadu_si512(wp + kg * 128);
        const __m512i v0 = _mm512_ternarylogic_epi32(W, M, C, 0xEA);  // (W & M) | C
        const __m512i v1 = _mm512_ternarylogic_epi32(_mm512_srli_epi32(W, 4), M, C, 0xEA);
        const __m512i v2 = _mm512_ternarylogic_epi32(_mm512_srli_epi32(W, 8), M, C, 0xEA);
        const __m512i v3 = _mm512_ternarylogic_epi32(_mm512_srli_epi32(W, 12), M, C, 0xEA);
        const uint16_t* s = st + kg * 64;
        const __m128 flo = _mm_cvtph_ps(_mm_loadl_epi64(reinterpret_cast<const __m128i*>(s + g * 4)));
        const __m128 fhi = _mm_cvtph_ps(_mm_loadl_epi64(reinterpret_cast<const __m128i*>(s + (g + 8) * 4)));
        const __m512 Dlo = _mm512_permutexvar_ps(idx, _mm512_castps128_ps512(flo));
        const __m512 Dhi = _mm512_permutexvar_ps(idx, _mm512_castps128_ps512(fhi));
        // (m - 128 d) in lanes 0 and 2
        const __m128 glo = _mm_fnmadd_ps(c128, flo, _mm_permute_ps(flo, 0xB1));
        const __m128 ghi = _mm_fnmadd_ps(c128, fhi, _mm_permute_ps(fhi, 0xB1));
        for (int r = 0; r < NR; ++r) {
          const uint32_t* xp = ab[r] + kg * 32;
          const __m512i xa = _mm512_loadu_si512(xp), xb = _mm512_loadu_si512(xp + 16);
          __m512 t = _mm512_dpbf16_ps(_mm512_setzero_ps(), (__m512bh)v0, (__m512bh)xa);
          t = _mm512_dpbf16_ps(t, (__m512bh)v2, (__m512bh)xb);
          alo[r] = _mm512_fmadd_ps(t, Dlo, alo[r]);
          __m512 u = _mm512_dpbf16_ps(_mm512_setzero_ps(), (__m512bh)v1, (__m512bh)xa);
          u = _mm512_dpbf16_ps(u, (__m512bh)v3, (__m512bh)xb);
          ahi[r] = _mm512_fmadd_ps(u, Dhi, ahi[r]);
          const __m128 sx = _mm_loadu_ps(sx4[r] + kg * 4);
          clo[r] = _mm_fmadd_ps(glo, sx, clo[r]);
          chi[r] = _mm_fmadd_ps(ghi, sx, chi[r]);
        }
      }
      for (int r = 0; r < NR; ++r) {
        const float lo = _mm512_reduce_add_ps(alo[r]) + _mm_cvtss_f32(clo[r]) +
                         _mm_cvtss_f32(_mm_movehl_ps(clo[r], clo[r]));
        const float hi = _mm512_reduce_add_ps(ahi[r]) + _mm_cvtss_f32(chi[r]) +
                         _mm_cvtss_f32(_mm_movehl_ps(chi[r], chi[r]));
        y[r][tile * 16 + g] = lo * scale[r];
        y[r][tile * 16 + g + 8] = hi * scale[r];
      }
    }
  }
}

// Plain C++ of the same product from the element definition (CPUs without AVX-512 BF16, and
// the oracle of the tests).
void tiles_scalar(const uint32_t* qw, const uint16_t* sm, int K, int tile0, int tile1, const uint16_t* const* x,
                  int nr, float* const* y, const float* scale) {
  const int64_t Kl = K;
  for (int64_t n = (int64_t)tile0 * 16; n < (int64_t)tile1 * 16; ++n)
    for (int r = 0; r < nr; ++r) {
      float acc = 0.f;
      for (int64_t kb = 0; kb < Kl / 32; ++kb) {
        const int64_t si = q4t_scale_index(Kl, n, kb);
        const float d = h2f_h(sm[2 * si]), m = h2f_h(sm[2 * si + 1]);
        float s = 0.f, sx = 0.f;
        for (int64_t k = kb * 32; k < kb * 32 + 32; ++k) {
          int64_t word;
          int nib;
          q4t_locate(0, Kl, n, k, &word, &nib);
          const float q = (float)((qw[word] >> (4 * nib)) & 15u);
          const float xv = bf2f_h(x[r][k]);
          s += q * xv;
          sx += xv;
        }
        acc += d * s + m * sx;
      }
      y[r][n] = acc * scale[r];
    }
}

// Kernel family: 0 plain C++, 1 AVX-512 BF16 (bf16 magic-number pairs, exact products),
// 2 AVX-512 VNNI (int16 activations, vpdpwssd); the default is the faster SIMD family.
bool has_bf16() {
  static const bool ok = __builtin_cpu_supports("avx512f") && __builtin_cpu_supports("avx512bw") &&
                         __builtin_cpu_supports("avx512vl") && __builtin_cpu_supports("avx512bf16");
  return ok;
}
bool has_vnni() {
  static const bool ok = __builtin_cpu_supports("avx512f") && __builtin_cpu_supports("avx512bw") &&
                         __builtin_cpu_supports("avx512vl") && __builtin_cpu_supports("avx512vnni");
  return ok;
}
bool simd_ok() { return has_bf16() || has_vnni(); }

// Issue cost of the dot-product instructions the two families rest on (ns per instruction, eight
// independent accumulator chains, zmm forms): vdpbf16ps, vfmadd231ps, vpdpwssd, vpdpbusd.
// A probe of the host (the figures behind the family choice); -1 where the ISA is missing.
__attribute__((target("avx512f,avx512bw,avx512vl,avx512bf16,avx512vnni"))) static double time_bf16(long n) {
  __m512 a[8];
  for (int i = 0; i < 8; ++i) a[i] = _mm512_set1_ps((float)i);
  __m512i x = _mm512_set1_epi32(0x3f803f80), w = _mm512_set1_epi32(0x3f003f00);
  const uint64_t t0 = now_ns();
  for (long i = 0; i < n; ++i) {
#pragma GCC unroll 8
    for (int j = 0; j < 8; ++j) a[j] = _mm512_dpbf16_ps(a[j], (__m512bh)x, (__m512bh)w);
    asm volatile("" : "+v"(x));
  }
  const uint64_t t1 = now_ns();
  float s = 0.f;
  for (int i = 0; i < 8; ++i) s += _mm512_reduce_add_ps(a[i]);
  asm volatile("" ::"x"(s));
  return (double)(t1 - t0) / (8.0 * n);
}
__attribute__((target("avx512f,fma"))) static double time_fma(long n) {
  __m512 a[8];
  for (int i = 0; i < 8; ++i) a[i] = _mm512_set1_ps((float)i);
  __m512 y = _mm512_set1_ps(0.999f), z = _mm512_set1_ps(0.5f);
  const uint64_t t0 = now_ns();
  for (long i = 0; i < n; ++i) {
#pragma GCC unroll 8
    for (int j = 0; j < 8; ++j) a[j] = _mm512_fmadd_ps(a[j], y, z);
    asm volatile("" : "+v"(y));
  }
  const uint64_t t1 = now_ns();
  float s = 0.f;
  for (int i = 0; i < 8; ++i) s += _mm512_reduce_add_ps(a[i]);
  asm volatile("" ::"x"(s));
  return (double)(t1 - t0) / (8.0 * n);
}
template <bool BYTES>
__attribute__((target("avx512f,avx512bw,avx512vnni"))) static double time_vnni(long n) {
  __m512i a[8];
  for (int i = 0; i < 8; ++i) a[i] = _mm512_set1_epi32(i);
  __m512i u = _mm512_set1_epi32(0x01010101), v = _mm512_set1_epi32(0x02020202);
  const uint64_t t0 = now_ns();
  for (long i = 0; i < n; ++i) {
#pragma GCC unroll 8
    for (int j = 0; j < 8; ++j) a[j] = BYTES ? _mm512_dpbusd_epi32(a[j], u, v) : _mm512_dpwssd_epi32(a[j], u, v);
    asm volatile("" : "+v"(u));
  }
  const uint64_t t1 = now_ns();
  long s = 0;
  for (int i = 0; i < 8; ++i) s += _mm512_reduce_add_epi32(a[i]);
  asm volatile("" ::"r"(s));
  return (double)(t1 - t0) / (8.0 * n);
}

// Which SIMD family is faster depends on the host: on some Xeons `vdpbf16ps` issues at about a
// quarter of the FMA rate, so the int16 VNNI form (two `vpdpwssd` per pair of columns, exact
// integer sums) wins by ~1.4x; where bf16 dot products are cheap the BF16 form saves the
// activation scaling.  Both families are timed once per process on a synthetic, cache-resident
// slice (4 tiles x 1024 columns, 2 rows: the common row count of an expert at decode) and the
// faster one is the default.  A few milliseconds on the calling thread.
int calibrate_mode() {
  if (!(has_bf16() && has_vnni())) return has_bf16() ? 1 : (has_vnni() ? 2 : 0);
  constexpr int Kc = 1024, KGc = Kc / 64, T = 4, R = 2;
  std::vector<uint32_t> qw((size_t)T * KGc * 128);
  std::vector<uint16_t> sm((size_t)T * KGc * 64);
  uint32_t st = 12345u;
  for (auto& v : qw) v = (st = st * 1664525u + 1013904223u);
  for (size_t i = 0; i < sm.size(); ++i) sm[i] = (i & 1) ? 0xA400 : 0x2000;  // m = -1/64, d = 1/128
  std::vector<uint16_t> x((size_t)R * Kc);
  for (auto& v : x) v = f2bf_h((float)(int)((st = st * 1664525u + 1013904223u) >> 22) / 512.f - 1.f);
  std::vector<uint32_t> ab(R * KGc * 32), ab16(R * KGc * 32);
  std::vector<float> sx4(R * KGc * 4), sxs(R * KGc * 16), y(R * T * 16), one(R, 1.f);
  const uint32_t *pa[R], *pa16[R];
  const float *ps4[R], *pss[R];
  float* py[R];
  for (int r = 0; r < R; ++r) {
    pack_row(&x[r * Kc], Kc, &ab[r * KGc * 32], &sx4[r * KGc * 4]);
    pack_row_i16(&x[r * Kc], Kc, &ab16[r * KGc * 32], &sxs[r * KGc * 16], &sx4[r * KGc * 4]);
    pa[r] = &ab[r * KGc * 32];
    pa16[r] = &ab16[r * KGc * 32];
    ps4[r] = &sx4[r * KGc * 4];
    pss[r] = &sxs[r * KGc * 16];
    py[r] = &y[r * T * 16];
  }
  auto best_of = [](auto&& f) {
    uint64_t best = ~0ull;
    for (int rep = 0; rep < 7; ++rep) {
      const uint64_t t0 = now_ns();
      for (int i = 0; i < 16; ++i) f();
      best = std::min(best, now_ns() - t0);
    }
    return best;
  };
  const uint64_t t_bf = best_of([&] { tiles_avx512<R>(qw.data(), sm.data(), Kc, 0, T, pa, ps4, py, one.data()); });
  const uint64_t t_i16 =
      best_of([&] { tiles_vnni<R, 4>(qw.data(), sm.data(), Kc, 0, T, pa16, pss, ps4, py, one.data()); });
  return t_i16 < t_bf ? 2 : 1;
}

int pick_mode(int want) {
  if (want < 0) {
    if (const char* e = getenv("SYN_CPU_GEMV_MODE")) {
      want = atoi(e);
    } else {
      static const int fastest = calibrate_mode();
      want = fastest;
    }
  }
  if (want == 1 && !has_bf16()) want = has_vnni() ? 2 : 0;
  if (want == 2 && !has_vnni()) want = has_bf16() ? 1 : 0;
  return want;
}

std::vector<double> isa_rates(long n) {
  std::vector<double> r(4, -1.0);
  if (has_bf16()) r[0] = time_bf16(n);
  if (__builtin_cpu_supports("avx512f") && __builtin_cpu_supports("fma")) r[1] = time_fma(n);
  if (has_vnni()) {
    r[2] = time_vnni<false>(n);
    r[3] = time_vnni<true>(n);
  }
  return r;
}

// Packs one activation row for `mode` (ab: [K/64][32] pairs, sxs: [K/64][16] VNNI scales,
// sx4: [K/64][4] block sums).
void pack_for(int mode, const uint16_t* x, int K, uint32_t* ab, float* sxs, float* sx4) {
  if (mode == 2)
    pack_row_i16(x, K, ab, sxs, sx4);
  else if (mode == 1)
    pack_row(x, K, ab, sx4);
}

// Rows of one expert against one weight matrix.
void expert_tiles(int mode, const uint32_t* qw, const uint16_t* sm, int K, int t0, int t1, int nr,
                  const uint32_t* const* ab, const float* const* sxs, const float* const* sx4,
                  const uint16_t* const* xr, float* const* y, const float* scale) {
  if (mode == 0) {
    tiles_scalar(qw, sm, K, t0, t1, xr, nr, y, scale);
    return;
  }
  for (int r0 = 0; r0 < nr;) {
    const int n = nr - r0;
    if (mode == 2) {
      // up to four rows per pass over the weights (one pass for 3 rows is ~28 % faster than 2 + 1,
      // for 4 rows ~18 % faster than 2 + 2); fewer row pairs per pass as rows grow (registers)
      // row pairs per pass: all 8 for 1-2 rows (each 512-byte group of the tile streamed whole),
      // 4 for 3-4 rows (registers); SYN_CPU_NARROW=1 keeps the narrower passes (measurement)
      const int take = std::min(4, n);
      if (g_narrow_passes) {
        switch (take) {
          case 1: tiles_vnni<1, 4>(qw, sm, K, t0, t1, ab + r0, sxs + r0, sx4 + r0, y + r0, scale + r0); break;
          case 2: tiles_vnni<2, 4>(qw, sm, K, t0, t1, ab + r0, sxs + r0, sx4 + r0, y + r0, scale + r0); break;
          case 3: tiles_vnni<3, 2>(qw, sm, K, t0, t1, ab + r0, sxs + r0, sx4 + r0, y + r0, scale + r0); break;
          default: tiles_vnni<4, 2>(qw, sm, K, t0, t1, ab + r0, sxs + r0, sx4 + r0, y + r0, scale + r0); break;
        }
      } else {
        switch (take) {
          case 1: tiles_vnni<1, 8>(qw, sm, K, t0, t1, ab + r0, sxs + r0, sx4 + r0, y + r0, scale + r0); break;
          case 2: tiles_vnni<2, 8>(qw, sm, K, t0, t1, ab + r0, sxs + r0, sx4 + r0, y + r0, scale + r0); break;
          case 3: tiles_vnni<3, 4>(qw, sm, K, t0, t1, ab + r0, sxs + r0, sx4 + r0, y + r0, scale + r0); break;
          default: tiles_vnni<4, 4>(qw, sm, K, t0, t1, ab + r0, sxs + r0, sx4 + r0, y + r0, scale + r0); break;
        }
      }
      r0 += take;
    } else {
      const int nb = std::min(4, n);
      switch (nb) {
        case 1: tiles_avx512<1>(qw, sm, K, t0, t1, ab + r0, sx4 + r0, y + r0, scale + r0); break;
        case 2: tiles_avx512<2>(qw, sm, K, t0, t1, ab + r0, sx4 + r0, y + r0, scale + r0); break;
        case 3: tiles_avx512<3>(qw, sm, K, t0, t1, ab + r0, sx4 + r0, y + r0, scale + r0); break;
        default: tiles_avx512<4>(qw, sm, K, t0, t1, ab + r0, sx4 + r0, y + r0, scale + r0); break;
      }
      r0 += nb;
    }
  }
}

}  // namespace

// ------------------------------------------------------------------ the worker pool
class CpuExpertTier {
 public:
  CpuExpertTier(int64_t n_layers, int64_t E, int64_t H, int64_t I, int64_t k, int64_t max_rows, int64_t mailbox,
                std::vector<int64_t> cpus, int64_t n_threads, int64_t mode)
      : L_(n_layers), E_(E), H_(H), I_(I), k_(k), R_(max_rows), cpus_(std::move(cpus)),
        nt_((int)std::max<int64_t>(1, n_threads)), mode_(pick_mode((int)mode)),
        mb_(reinterpret_cast<uint8_t*>(mailbox)), lay_(cpu_mailbox_layout(E, k, max_rows, H)),
        own_(n_layers * E * 4, 0) {
    SYN_REQUIRE(H % 64 == 0 && I % 64 == 0 && (2 * I) % 16 == 0, "cpu experts: H, I multiples of 64");
    const int64_t P = max_rows * k;
    hab_.resize(R_ * (H_ / 64) * 32);
    hsx_.resize(R_ * (H_ / 64) * 4);
    hss_.resize(R_ * (H_ / 64) * 16);
    ygu_.resize(P * 2 * I_);
    mid_.resize(P * I_);
    mab_.resize(P * (I_ / 64) * 32);
    msx_.resize(P * (I_ / 64) * 4);
    mss_.resize(P * (I_ / 64) * 16);
    row_used_.resize(R_);
  }
  ~CpuExpertTier() { stop(); }

  // Expert e of layer l is computed here when its gate_up / down weight pointers are given
  // (host addresses of its tiled rows); zeros hand it back to the GPU.
  void set_expert(int64_t l, int64_t e, int64_t qgu, int64_t sgu, int64_t qdn, int64_t sdn) {
    SYN_REQUIRE(l >= 0 && l < L_ && e >= 0 && e < E_, "set_expert: layer/expert out of range");
    int64_t* o = &own_[(l * E_ + e) * 4];
    o[0] = qgu;
    o[1] = sgu;
    o[2] = qdn;
    o[3] = sdn;
  }

  void start() {
    if (!th_.empty()) return;
    stop_.store(false);
    seen_ = load_acquire(word(MB_GO));
    // every thread starts from the same job generation, read before any of them runs (a thread
    // that read it after thread 0 published the first job would skip that job)
    const uint32_t gen0 = job_gen_.load(std::memory_order_acquire);
    for (int t = 0; t < nt_; ++t) th_.emplace_back([this, t, gen0] { loop(t, gen0); });
  }

  void stop() {
    stop_.store(true);
    for (auto& t : th_) t.join();
    th_.clear();
  }

  struct Stats {
    int64_t jobs, pairs;
    double busy_ms, phase_ms[4];  // phases per thread, averaged: pack, gate/up, SiLU + pack, down
    int threads, mode;             // mode: 0 plain C++, 1 AVX-512 BF16, 2 AVX-512 VNNI
  };
  Stats stats() const {
    Stats st;
    st.jobs = jobs_.load();
    st.pairs = pairs_.load();
    st.busy_ms = busy_ns_.load() / 1e6;
    for (int i = 0; i < 4; ++i) st.phase_ms[i] = phase_ns_[i].load() / 1e6 / nt_;
    st.threads = nt_;
    st.mode = mode_;
    return st;
  }

 private:
  uint32_t* word(int i) { return reinterpret_cast<uint32_t*>(mb_) + i; }

  void pin(int t) {
    if (cpus_.empty()) return;
    cpu_set_t set;
    CPU_ZERO(&set);
    CPU_SET((int)cpus_[t % cpus_.size()], &set);
    pthread_setaffinity_np(pthread_self(), sizeof(set), &set);
  }

  // spin, then sleep in short naps while idle; false once stop() was called
  template <typename F>
  bool wait_until(F ready) {
    uint64_t t0 = 0;
    for (uint32_t it = 0;; ++it) {
      if (ready()) return true;
      if (stop_.load(std::memory_order_relaxed)) return false;
      if (it < 4096) {
        _mm_pause();
        continue;
      }
      if (!t0) t0 = now_ns();
      if (now_ns() - t0 < 2000000ull) {
        _mm_pause();
      } else {
        timespec ts{0, 20000};
        nanosleep(&ts, nullptr);
      }
    }
  }

  // A thread that left on stop() never arrives, so waits give up on stop() too (the job's
  // results are then not published).
  void barrier() {
    const uint32_t g = bar_gen_.load(std::memory_order_acquire);
    if (bar_count_.fetch_add(1, std::memory_order_acq_rel) == nt_ - 1) {
      bar_count_.store(0, std::memory_order_relaxed);
      bar_gen_.store(g + 1, std::memory_order_release);
    } else {
      while (bar_gen_.load(std::memory_order_acquire) == g) {
        if (stop_.load(std::memory_order_relaxed)) return;
        _mm_pause();
      }
    }
  }

  struct Expert {
    int e, p0, n, q0;
  };
  struct Task {
    int j, t0, t1;
  };

  void prepare(uint32_t seq) {
    t_start_ = now_ns();
    seq_ = seq;
    layer_ = (int)*word(MB_LAYER);
    rows_ = (int)*word(MB_ROWS);
    const int32_t* off = reinterpret_cast<const int32_t*>(mb_ + lay_.tok_off);
    const int32_t* tidx = reinterpret_cast<const int32_t*>(mb_ + lay_.tok_idx);
    int32_t* out_pairs = reinterpret_cast<int32_t*>(mb_ + lay_.out_pairs);
    experts_.clear();
    gu_tasks_.clear();
    dn_tasks_.clear();
    pack_rows_.clear();
    std::fill(row_used_.begin(), row_used_.end(), 0);
    n_out_ = 0;
    bad_ = layer_ < 0 || layer_ >= L_ || rows_ < 0 || rows_ > R_;
    if (!bad_) {
      const int GT = (int)(2 * I_ / 16), DT = (int)(H_ / 16);
      for (int e = 0; e < E_; ++e) {
        const int64_t* o = &own_[((int64_t)layer_ * E_ + e) * 4];
        if (!o[0]) continue;
        const int p0 = off[e], n = off[e + 1] - off[e];
        if (n <= 0) continue;
        if (p0 < 0 || p0 + n > rows_ * k_) {
          bad_ = true;
          break;
        }
        const int j = (int)experts_.size();
        experts_.push_back({e, p0, n, n_out_});
        for (int i = 0; i < n; ++i) {
          out_pairs[n_out_ + i] = p0 + i;
          const int tok = tidx[p0 + i];
          if (tok < 0 || tok >= rows_) {
            bad_ = true;
          } else if (!row_used_[tok]) {
            row_used_[tok] = 1;
            pack_rows_.push_back(tok);
          }
        }
        n_out_ += n;
        for (int t = 0; t < GT; t += gu_tiles_) gu_tasks_.push_back({j, t, std::min(GT, t + gu_tiles_)});
        for (int t = 0; t < DT; t += dn_tiles_) dn_tasks_.push_back({j, t, std::min(DT, t + dn_tiles_)});
      }
    }
    if (bad_) {
      experts_.clear();
      gu_tasks_.clear();
      dn_tasks_.clear();
      pack_rows_.clear();
      n_out_ = 0;
    }
    next_.store(0, std::memory_order_relaxed);
  }

  // dynamic task claiming within one phase; the counter is reset by the last arriver
  template <typename F>
  void run_phase(int n_tasks, F fn) {
    for (;;) {
      const int i = next_.fetch_add(1, std::memory_order_relaxed);
      if (i >= n_tasks) break;
      fn(i);
    }
    barrier();
    if (bar_reset_.fetch_add(1, std::memory_order_acq_rel) == nt_ - 1) {
      bar_reset_.store(0, std::memory_order_relaxed);
      next_.store(0, std::memory_order_relaxed);
    }
    barrier();
  }

  void work() {
    const uint16_t* h = reinterpret_cast<const uint16_t*>(mb_ + lay_.h);
    const int32_t* tidx = reinterpret_cast<const int32_t*>(mb_ + lay_.tok_idx);
    const float* pw = reinterpret_cast<const float*>(mb_ + lay_.pair_w);
    float* out = reinterpret_cast<float*>(mb_ + lay_.out);
    const int KGH = (int)(H_ / 64), KGI = (int)(I_ / 64);
    // 1. pack the activation rows
    if (mode_)
      run_phase((int)pack_rows_.size(), [&](int i) {
        const int r = pack_rows_[i];
        pack_for(mode_, h + (int64_t)r * H_, (int)H_, &hab_[(int64_t)r * KGH * 32], &hss_[(int64_t)r * KGH * 16],
                 &hsx_[(int64_t)r * KGH * 4]);
      });
    uint64_t tp = now_ns();
    auto lap = [&](int ph) {
      const uint64_t t = now_ns();
      phase_ns_[ph].fetch_add(t - tp, std::memory_order_relaxed);
      tp = t;
    };
    lap(0);
    // 2. gate / up blocks of every owned expert
    run_phase((int)gu_tasks_.size(), [&](int i) {
      const Task& t = gu_tasks_[i];
      const Expert& x = experts_[t.j];
      const int64_t* o = &own_[((int64_t)layer_ * E_ + x.e) * 4];
      std::vector<const uint32_t*> ab(x.n);
      std::vector<const float*> sx(x.n), ss(x.n);
      std::vector<const uint16_t*> xr(x.n);
      std::vector<float*> y(x.n);
      std::vector<float> one(x.n, 1.f);
      for (int r = 0; r < x.n; ++r) {
        const int tok = tidx[x.p0 + r];
        ab[r] = &hab_[(int64_t)tok * KGH * 32];
        sx[r] = &hsx_[(int64_t)tok * KGH * 4];
        ss[r] = &hss_[(int64_t)tok * KGH * 16];
        xr[r] = h + (int64_t)tok * H_;
        y[r] = &ygu_[(int64_t)(x.q0 + r) * 2 * I_];
      }
      expert_tiles(mode_, reinterpret_cast<const uint32_t*>(o[0]), reinterpret_cast<const uint16_t*>(o[1]), (int)H_,
                   t.t0, t.t1, x.n, ab.data(), ss.data(), sx.data(), xr.data(), y.data(), one.data());
    });
    lap(1);
    // 3. SiLU gate (rows interleaved in 8-row gate / up chunks), bf16 rounding, packing
    run_phase(n_out_, [&](int q) {
      const float* g = &ygu_[(int64_t)q * 2 * I_];
      uint16_t* m = &mid_[(int64_t)q * I_];
      for (int64_t c = 0; c < I_ / 8; ++c)
        for (int i = 0; i < 8; ++i) {
          const float gv = g[16 * c + i], uv = g[16 * c + 8 + i];
          m[8 * c + i] = f2bf_h(gv / (1.f + std::exp(-gv)) * uv);
        }
      if (mode_)
        pack_for(mode_, m, (int)I_, &mab_[(int64_t)q * KGI * 32], &mss_[(int64_t)q * KGI * 16],
                 &msx_[(int64_t)q * KGI * 4]);
    });
    lap(2);
    // 4. down blocks, scaled by the routing weight, straight into the mailbox
    run_phase((int)dn_tasks_.size(), [&](int i) {
      const Task& t = dn_tasks_[i];
      const Expert& x = experts_[t.j];
      const int64_t* o = &own_[((int64_t)layer_ * E_ + x.e) * 4];
      std::vector<const uint32_t*> ab(x.n);
      std::vector<const float*> sx(x.n), ss(x.n);
      std::vector<const uint16_t*> xr(x.n);
      std::vector<float*> y(x.n);
      std::vector<float> sc(x.n);
      for (int r = 0; r < x.n; ++r) {
        const int q = x.q0 + r;
        ab[r] = &mab_[(int64_t)q * KGI * 32];
        sx[r] = &msx_[(int64_t)q * KGI * 4];
        ss[r] = &mss_[(int64_t)q * KGI * 16];
        xr[r] = &mid_[(int64_t)q * I_];
        y[r] = out + (int64_t)q * H_;
        sc[r] = pw[x.p0 + r];
      }
      expert_tiles(mode_, reinterpret_cast<const uint32_t*>(o[2]), reinterpret_cast<const uint16_t*>(o[3]), (int)I_,
                   t.t0, t.t1, x.n, ab.data(), ss.data(), sx.data(), xr.data(), y.data(), sc.data());
    });
    lap(3);
  }

  void loop(int t, uint32_t gen0) {
    pin(t);
    uint32_t my_gen = gen0;
    while (true) {
      if (t == 0) {
        uint32_t go = 0;
        if (!wait_until([&] { return (go = load_acquire(word(MB_GO))) != seen_; })) break;
        if (stop_.load()) break;
        seen_ = go;
        prepare(go);
        job_gen_.store(my_gen + 1, std::memory_order_release);
      } else if (!wait_until([&] { return job_gen_.load(std::memory_order_acquire) != my_gen; })) {
        break;
      }
      my_gen = job_gen_.load(std::memory_order_acquire);
      work();
      if (t == 0 && !stop_.load()) {
        *word(MB_NOUT) = (uint32_t)n_out_;
        *word(MB_ERR) = bad_ ? 1u : 0u;
        std::atomic_thread_fence(std::memory_order_seq_cst);
        store_release(word(MB_DONE), seq_);
        jobs_.fetch_add(1);
        pairs_.fetch_add(n_out_);
        busy_ns_.fetch_add(now_ns() - t_start_);
      }
    }
  }

  const int64_t L_, E_, H_, I_, k_, R_;
  std::vector<int64_t> cpus_;
  const int nt_;
  const int mode_;
  uint8_t* mb_;
  CpuMailboxLayout lay_;
  std::vector<int64_t> own_;
  std::vector<uint32_t> hab_, mab_;
  std::vector<float> hsx_, msx_, hss_, mss_, ygu_;
  std::vector<uint16_t> mid_;
  std::vector<char> row_used_;
  std::vector<int> pack_rows_;
  std::vector<Expert> experts_;
  std::vector<Task> gu_tasks_, dn_tasks_;
  // 16-row tiles per task (gate/up, down): 4 / 8 measured best on the B200 node's 14 workers
  // (with 16 groups of prefetch: 61 GB/s against 46 GB/s for 8 / 16 tiles and 8 groups, the
  // pool alone); SYN_CPU_TASK_TILES="gu,dn" overrides (measurement)
  int gu_tiles_ = env_pair(0, 4), dn_tiles_ = env_pair(1, 8);
  static int env_pair(int which, int dflt) {
    const char* e = getenv("SYN_CPU_TASK_TILES");
    int a = 0, b = 0;
    if (e && sscanf(e, "%d,%d", &a, &b) == 2 && a > 0 && b > 0) return which ? b : a;
    return dflt;
  }
  int layer_ = 0, rows_ = 0, n_out_ = 0;
  bool bad_ = false;
  uint32_t seq_ = 0, seen_ = 0;
  uint64_t t_start_ = 0;
  std::vector<std::thread> th_;
  std::atomic<bool> stop_{false};
  std::atomic<uint32_t> job_gen_{0}, bar_gen_{0};
  std::atomic<int> bar_count_{0}, bar_reset_{0}, next_{0};
  std::atomic<int64_t> jobs_{0}, pairs_{0};
  std::atomic<uint64_t> busy_ns_{0};
  std::atomic<uint64_t> phase_ns_[4] = {};  // summed over threads: pack, gate/up, SiLU, down
};

#ifndef SYN_NO_TORCH
// y [R, N] f32 = x [R, K] (bf16) @ W^T for a tiled 4-bit matrix held in host memory, with
// kernel family `mode` (0 plain C++, 1 AVX-512 BF16, 2 AVX-512 VNNI, -1 the default).
torch::Tensor cpu_q4t_gemv(torch::Tensor qw, torch::Tensor sm, torch::Tensor x, int64_t N, int64_t mode) {
  TORCH_CHECK(!qw.is_cuda() && !sm.is_cuda() && !x.is_cuda(), "cpu_q4t_gemv: host tensors");
  TORCH_CHECK(qw.is_contiguous() && sm.is_contiguous() && x.is_contiguous(), "contiguous inputs");
  TORCH_CHECK(x.scalar_type() == torch::kBFloat16 && x.dim() == 2, "x bf16 [R, K]");
  const int64_t R = x.size(0), K = x.size(1);
  TORCH_CHECK(N % 16 == 0 && K % 64 == 0, "N % 16, K % 64");
  TORCH_CHECK(qw.numel() * qw.element_size() >= N * K / 2 && sm.numel() * sm.element_size() >= N * K / 32 * 4,
              "weight sizes");
  const int md = mode == 0 ? 0 : pick_mode((int)mode);
  auto y = torch::zeros({R, N}, torch::kFloat32);
  const uint16_t* xp = reinterpret_cast<const uint16_t*>(x.data_ptr());
  const int64_t KG = K / 64;
  std::vector<uint32_t> ab(R * KG * 32);
  std::vector<float> sx(R * KG * 4), ss(R * KG * 16);
  std::vector<const uint32_t*> abp(R);
  std::vector<const float*> sxp(R), ssp(R);
  std::vector<const uint16_t*> xr(R);
  std::vector<float*> yp(R);
  std::vector<float> one(R, 1.f);
  for (int64_t r = 0; r < R; ++r) {
    pack_for(md, xp + r * K, (int)K, &ab[r * KG * 32], &ss[r * KG * 16], &sx[r * KG * 4]);
    abp[r] = &ab[r * KG * 32];
    sxp[r] = &sx[r * KG * 4];
    ssp[r] = &ss[r * KG * 16];
    xr[r] = xp + r * K;
    yp[r] = y.data_ptr<float>() + r * N;
  }
  expert_tiles(md, reinterpret_cast<const uint32_t*>(qw.data_ptr()), reinterpret_cast<const uint16_t*>(sm.data_ptr()),
               (int)K, 0, (int)(N / 16), (int)R, abp.data(), ssp.data(), sxp.data(), xr.data(), yp.data(), one.data());
  return y;
}

#endif  // SYN_NO_TORCH

namespace {
__attribute__((target("avx512f"))) double read_chunk(const uint8_t* p, int64_t n) {
  __m512 acc = _mm512_setzero_ps();
  for (int64_t i = 0; i + 256 <= n; i += 256) {
    const __m512 a = _mm512_loadu_ps(reinterpret_cast<const float*>(p + i));
    const __m512 b = _mm512_loadu_ps(reinterpret_cast<const float*>(p + i + 64));
    const __m512 c = _mm512_loadu_ps(reinterpret_cast<const float*>(p + i + 128));
    const __m512 d = _mm512_loadu_ps(reinterpret_cast<const float*>(p + i + 192));
    acc = _mm512_add_ps(acc, _mm512_add_ps(_mm512_add_ps(a, b), _mm512_add_ps(c, d)));
  }
  return _mm512_reduce_add_ps(acc);
}
}  // namespace

// Host read bandwidth (GB/s) of `threads` threads streaming disjoint parts of one buffer
// (a probe for sizing the CPU share of the cold experts).
double cpu_read_gbs(int64_t nbytes, int64_t threads, int64_t reps) {
  SYN_REQUIRE(simd_ok(), "cpu_read_gbs: needs AVX-512");
  std::vector<uint8_t> buf(nbytes, 1);
  const int64_t per = (nbytes / threads) & ~int64_t(255);
  std::vector<double> sink(threads);
  double best = 0.0;
  for (int64_t r = 0; r < reps; ++r) {
    const uint64_t t0 = now_ns();
    std::vector<std::thread> th;
    for (int64_t t = 0; t < threads; ++t)
      th.emplace_back([&, t] { sink[t] = read_chunk(buf.data() + t * per, per); });
    for (auto& x : th) x.join();
    const double s = (now_ns() - t0) * 1e-9;
    best = std::max(best, (double)(per * threads) / s / 1e9);
  }
  return best;
}

#ifndef SYN_NO_TORCH
void register_cpu_experts(pybind11::module& m) {
  m.def("cpu_read_gbs", &cpu_read_gbs, pybind11::call_guard<pybind11::gil_scoped_release>());
  m.def("cpu_q4t_gemv", &cpu_q4t_gemv, "host GEMV over the tiled 4-bit layout (AVX-512 BF16 or plain C++)",
        pybind11::call_guard<pybind11::gil_scoped_release>());
  m.def("cpu_simd_available", [] { return simd_ok(); });
  m.def("cpu_gemv_mode", [] { return pick_mode(-1); }, "default kernel family: 0 C++, 1 AVX-512 BF16, 2 VNNI");
  m.def("cpu_isa_rates", [](int64_t n) { return isa_rates((long)n); }, pybind11::arg("n") = 20000000,
        "ns per instruction (8 chains): vdpbf16ps, vfmadd231ps, vpdpwssd, vpdpbusd (-1: not supported)",
        pybind11::call_guard<pybind11::gil_scoped_release>());
  m.def("cpu_mailbox_bytes", [](int64_t E, int64_t k, int64_t R, int64_t H) {
    const CpuMailboxLayout l = cpu_mailbox_layout(E, k, R, H);
    return std::vector<int64_t>{l.tok_off, l.tok_idx, l.pair_w, l.h, l.out_pairs, l.out, l.bytes};
  });
  pybind11::class_<CpuExpertTier>(m, "CpuExpertTier")
      .def(pybind11::init<int64_t, int64_t, int64_t, int64_t, int64_t, int64_t, int64_t, std::vector<int64_t>, int64_t,
                          int64_t>())
      .def("set_expert", &CpuExpertTier::set_expert)
      .def("start", &CpuExpertTier::start)
      .def("stop", &CpuExpertTier::stop, pybind11::call_guard<pybind11::gil_scoped_release>())
      .def("stats", [](const CpuExpertTier& t) {
        const auto st = t.stats();
        pybind11::dict d;
        d["jobs"] = st.jobs;
        d["busy_ms"] = st.busy_ms;
        d["pairs"] = st.pairs;
        d["threads"] = st.threads;
        d["mode"] = st.mode;
        d["phase_ms"] = std::vector<double>(st.phase_ms, st.phase_ms + 4);
        return d;
      });
}

#endif  // SYN_NO_TORCH

}  // namespace syn
