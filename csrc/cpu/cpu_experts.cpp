// Cold experts on the host CPU during decode (reference crates/kernels-cpu/src/moe.rs: expert
// misses as tasks per (expert, output-row block); crates/kernels/src/moe/doorbell.rs: the
// hand-off through host-mapped memory).
//
// The weights stay in the device's tiled 4-bit layout (syn/q4.h) inside the pinned host tier
// that the GPU also reads over PCIe, so an expert moves between the CPU and the PCIe path with
// no copy.  In that layout the 64 bytes of lanes 4g..4g+3 of one (16-row tile, 64-column group)
// hold rows g and g+8 over all 64 columns, and ((word >> 4j) & 0x000F000F) is a pair of
// consecutive columns of one row (j = 0, 2: row g; j = 1, 3: row g+8; j = 2, 3 are 8 columns
// further).  OR-ing 0x4300 into a nibble gives the bf16 number 128 + q exactly, so one
// `vdpbf16ps` multiplies 16 weight pairs by the matching bf16 activation pairs exactly and adds
// them in f32.  Per 32-column block with scale d and min m:
//     sum_k (d q_k + m) x_k = d * sum_k (128 + q_k) x_k + (m - 128 d) * sum_k x_k.
// Each activation row is packed once per layer into the pair order of the layout, with its
// per-block sums.  Products are exact, sums are f32: the result differs from the GPU kernels
// only by the order of f32 additions.
//
// Threads: a fixed pool pinned to the given CPUs.  Thread 0 polls the mailbox's go word; on a
// new sequence it lists the routed pairs of the experts this tier owns for that layer and
// releases the pool through four phases separated by barriers: pack the activation rows; gate
// and up tasks; SiLU-gate + pack; down tasks.  Then it writes the outputs' pair indices and
// release-stores the done word, which the GPU waits on with a time limit.
#include <torch/extension.h>

#include <immintrin.h>
#include <pthread.h>
#include <sched.h>
#include <time.h>

#include <algorithm>
#include <atomic>
#include <cmath>
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

// y[r][n] = scale[r] * sum_k W[n][k] x_r[k] for the rows of tiles [tile0, tile1), NR rows.
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

bool simd_ok() {
  static const bool ok = __builtin_cpu_supports("avx512f") && __builtin_cpu_supports("avx512bw") &&
                         __builtin_cpu_supports("avx512vl") && __builtin_cpu_supports("avx512bf16");
  return ok;
}

// Rows of one expert against one weight matrix: SIMD in groups of up to 4 rows.
void expert_tiles(bool simd, const uint32_t* qw, const uint16_t* sm, int K, int t0, int t1, int nr,
                  const uint32_t* const* ab, const float* const* sx4, const uint16_t* const* xr, float* const* y,
                  const float* scale) {
  if (!simd) {
    tiles_scalar(qw, sm, K, t0, t1, xr, nr, y, scale);
    return;
  }
  for (int r0 = 0; r0 < nr; r0 += 4) {
    const int n = std::min(4, nr - r0);
    switch (n) {
      case 1: tiles_avx512<1>(qw, sm, K, t0, t1, ab + r0, sx4 + r0, y + r0, scale + r0); break;
      case 2: tiles_avx512<2>(qw, sm, K, t0, t1, ab + r0, sx4 + r0, y + r0, scale + r0); break;
      case 3: tiles_avx512<3>(qw, sm, K, t0, t1, ab + r0, sx4 + r0, y + r0, scale + r0); break;
      default: tiles_avx512<4>(qw, sm, K, t0, t1, ab + r0, sx4 + r0, y + r0, scale + r0); break;
    }
  }
}

}  // namespace

// ------------------------------------------------------------------ the worker pool
class CpuExpertTier {
 public:
  CpuExpertTier(int64_t n_layers, int64_t E, int64_t H, int64_t I, int64_t k, int64_t max_rows, int64_t mailbox,
                std::vector<int64_t> cpus, int64_t n_threads, bool simd)
      : L_(n_layers), E_(E), H_(H), I_(I), k_(k), R_(max_rows), cpus_(std::move(cpus)),
        nt_((int)std::max<int64_t>(1, n_threads)), simd_(simd && simd_ok()),
        mb_(reinterpret_cast<uint8_t*>(mailbox)), lay_(cpu_mailbox_layout(E, k, max_rows, H)),
        own_(n_layers * E * 4, 0) {
    TORCH_CHECK(H % 64 == 0 && I % 64 == 0 && (2 * I) % 16 == 0, "cpu experts: H, I multiples of 64");
    const int64_t P = max_rows * k;
    hab_.resize(R_ * (H_ / 64) * 32);
    hsx_.resize(R_ * (H_ / 64) * 4);
    ygu_.resize(P * 2 * I_);
    mid_.resize(P * I_);
    mab_.resize(P * (I_ / 64) * 32);
    msx_.resize(P * (I_ / 64) * 4);
    row_used_.resize(R_);
  }
  ~CpuExpertTier() { stop(); }

  // Expert e of layer l is computed here when its gate_up / down weight pointers are given
  // (host addresses of its tiled rows); zeros hand it back to the GPU.
  void set_expert(int64_t l, int64_t e, int64_t qgu, int64_t sgu, int64_t qdn, int64_t sdn) {
    TORCH_CHECK(l >= 0 && l < L_ && e >= 0 && e < E_, "set_expert: layer/expert out of range");
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
    for (int t = 0; t < nt_; ++t) th_.emplace_back([this, t] { loop(t); });
  }

  void stop() {
    stop_.store(true);
    for (auto& t : th_) t.join();
    th_.clear();
  }

  pybind11::dict stats() const {
    pybind11::dict d;
    d["jobs"] = jobs_.load();
    d["busy_ms"] = busy_ns_.load() / 1e6;
    d["pairs"] = pairs_.load();
    d["threads"] = nt_;
    d["simd"] = simd_;
    return d;
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
        for (int t = 0; t < GT; t += 8) gu_tasks_.push_back({j, t, std::min(GT, t + 8)});
        for (int t = 0; t < DT; t += 16) dn_tasks_.push_back({j, t, std::min(DT, t + 16)});
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
    if (simd_)
      run_phase((int)pack_rows_.size(), [&](int i) {
        const int r = pack_rows_[i];
        pack_row(h + (int64_t)r * H_, (int)H_, &hab_[(int64_t)r * KGH * 32], &hsx_[(int64_t)r * KGH * 4]);
      });
    // 2. gate / up blocks of every owned expert
    run_phase((int)gu_tasks_.size(), [&](int i) {
      const Task& t = gu_tasks_[i];
      const Expert& x = experts_[t.j];
      const int64_t* o = &own_[((int64_t)layer_ * E_ + x.e) * 4];
      std::vector<const uint32_t*> ab(x.n);
      std::vector<const float*> sx(x.n);
      std::vector<const uint16_t*> xr(x.n);
      std::vector<float*> y(x.n);
      std::vector<float> one(x.n, 1.f);
      for (int r = 0; r < x.n; ++r) {
        const int tok = tidx[x.p0 + r];
        ab[r] = &hab_[(int64_t)tok * KGH * 32];
        sx[r] = &hsx_[(int64_t)tok * KGH * 4];
        xr[r] = h + (int64_t)tok * H_;
        y[r] = &ygu_[(int64_t)(x.q0 + r) * 2 * I_];
      }
      expert_tiles(simd_, reinterpret_cast<const uint32_t*>(o[0]), reinterpret_cast<const uint16_t*>(o[1]), (int)H_,
                   t.t0, t.t1, x.n, ab.data(), sx.data(), xr.data(), y.data(), one.data());
    });
    // 3. SiLU gate (rows interleaved in 8-row gate / up chunks), bf16 rounding, packing
    run_phase(n_out_, [&](int q) {
      const float* g = &ygu_[(int64_t)q * 2 * I_];
      uint16_t* m = &mid_[(int64_t)q * I_];
      for (int64_t c = 0; c < I_ / 8; ++c)
        for (int i = 0; i < 8; ++i) {
          const float gv = g[16 * c + i], uv = g[16 * c + 8 + i];
          m[8 * c + i] = f2bf_h(gv / (1.f + std::exp(-gv)) * uv);
        }
      if (simd_) pack_row(m, (int)I_, &mab_[(int64_t)q * KGI * 32], &msx_[(int64_t)q * KGI * 4]);
    });
    // 4. down blocks, scaled by the routing weight, straight into the mailbox
    run_phase((int)dn_tasks_.size(), [&](int i) {
      const Task& t = dn_tasks_[i];
      const Expert& x = experts_[t.j];
      const int64_t* o = &own_[((int64_t)layer_ * E_ + x.e) * 4];
      std::vector<const uint32_t*> ab(x.n);
      std::vector<const float*> sx(x.n);
      std::vector<const uint16_t*> xr(x.n);
      std::vector<float*> y(x.n);
      std::vector<float> sc(x.n);
      for (int r = 0; r < x.n; ++r) {
        const int q = x.q0 + r;
        ab[r] = &mab_[(int64_t)q * KGI * 32];
        sx[r] = &msx_[(int64_t)q * KGI * 4];
        xr[r] = &mid_[(int64_t)q * I_];
        y[r] = out + (int64_t)q * H_;
        sc[r] = pw[x.p0 + r];
      }
      expert_tiles(simd_, reinterpret_cast<const uint32_t*>(o[2]), reinterpret_cast<const uint16_t*>(o[3]), (int)I_,
                   t.t0, t.t1, x.n, ab.data(), sx.data(), xr.data(), y.data(), sc.data());
    });
  }

  void loop(int t) {
    pin(t);
    uint32_t my_gen = job_gen_.load(std::memory_order_acquire);
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
  const bool simd_;
  uint8_t* mb_;
  CpuMailboxLayout lay_;
  std::vector<int64_t> own_;
  std::vector<uint32_t> hab_, mab_;
  std::vector<float> hsx_, msx_, ygu_;
  std::vector<uint16_t> mid_;
  std::vector<char> row_used_;
  std::vector<int> pack_rows_;
  std::vector<Expert> experts_;
  std::vector<Task> gu_tasks_, dn_tasks_;
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
};

// y [R, N] f32 = x [R, K] (bf16) @ W^T for a tiled 4-bit matrix held in host memory.
torch::Tensor cpu_q4t_gemv(torch::Tensor qw, torch::Tensor sm, torch::Tensor x, int64_t N, bool simd) {
  TORCH_CHECK(!qw.is_cuda() && !sm.is_cuda() && !x.is_cuda(), "cpu_q4t_gemv: host tensors");
  TORCH_CHECK(qw.is_contiguous() && sm.is_contiguous() && x.is_contiguous(), "contiguous inputs");
  TORCH_CHECK(x.scalar_type() == torch::kBFloat16 && x.dim() == 2, "x bf16 [R, K]");
  const int64_t R = x.size(0), K = x.size(1);
  TORCH_CHECK(N % 16 == 0 && K % 64 == 0, "N % 16, K % 64");
  TORCH_CHECK(qw.numel() * qw.element_size() >= N * K / 2 && sm.numel() * sm.element_size() >= N * K / 32 * 4,
              "weight sizes");
  auto y = torch::zeros({R, N}, torch::kFloat32);
  const bool use_simd = simd && simd_ok();
  const uint16_t* xp = reinterpret_cast<const uint16_t*>(x.data_ptr());
  std::vector<uint32_t> ab(R * (K / 64) * 32);
  std::vector<float> sx(R * (K / 64) * 4);
  std::vector<const uint32_t*> abp(R);
  std::vector<const float*> sxp(R);
  std::vector<const uint16_t*> xr(R);
  std::vector<float*> yp(R);
  std::vector<float> one(R, 1.f);
  for (int64_t r = 0; r < R; ++r) {
    if (use_simd) pack_row(xp + r * K, (int)K, &ab[r * (K / 64) * 32], &sx[r * (K / 64) * 4]);
    abp[r] = &ab[r * (K / 64) * 32];
    sxp[r] = &sx[r * (K / 64) * 4];
    xr[r] = xp + r * K;
    yp[r] = y.data_ptr<float>() + r * N;
  }
  expert_tiles(use_simd, reinterpret_cast<const uint32_t*>(qw.data_ptr()),
               reinterpret_cast<const uint16_t*>(sm.data_ptr()), (int)K, 0, (int)(N / 16), (int)R, abp.data(),
               sxp.data(), xr.data(), yp.data(), one.data());
  return y;
}

void register_cpu_experts(pybind11::module& m) {
  m.def("cpu_q4t_gemv", &cpu_q4t_gemv, "host GEMV over the tiled 4-bit layout (AVX-512 BF16 or plain C++)");
  m.def("cpu_simd_available", [] { return simd_ok(); });
  m.def("cpu_mailbox_bytes", [](int64_t E, int64_t k, int64_t R, int64_t H) {
    const CpuMailboxLayout l = cpu_mailbox_layout(E, k, R, H);
    return std::vector<int64_t>{l.tok_off, l.tok_idx, l.pair_w, l.h, l.out_pairs, l.out, l.bytes};
  });
  pybind11::class_<CpuExpertTier>(m, "CpuExpertTier")
      .def(pybind11::init<int64_t, int64_t, int64_t, int64_t, int64_t, int64_t, int64_t, std::vector<int64_t>, int64_t,
                          bool>())
      .def("set_expert", &CpuExpertTier::set_expert)
      .def("start", &CpuExpertTier::start)
      .def("stop", &CpuExpertTier::stop, pybind11::call_guard<pybind11::gil_scoped_release>())
      .def("stats", &CpuExpertTier::stats);
}

}  // namespace syn
