// Token selection on the device: greedy argmax and seeded sampling with temperature,
// top-k and top-p.  Reference ops: `Argmax`, `LogitsProcess`, `TopKTopP`, `SampleSeeded`
// (plan/rfcs/RFC-0040-kernel-providers-and-backends.md:855; counter contract in
// plan/decisions/ADR-0107-counter-based-sampling-rng.md).
//
// Exact and deterministic by construction:
//  * thresholds come from radix select over the f32 key bits (top-k) and over integer
//    probability mass (top-p): histograms hold integer counts / fixed-point masses, so
//    atomic accumulation order cannot change a decision;
//  * p_i = exp(z_i - max) is held as a 2^32 fixed-point integer; the draw u picks the
//    first token (ascending id) whose cumulative mass exceeds floor(u * total);
//  * ties at the top-k threshold are all kept.
#include "common.cuh"
#include "syn/philox.h"

namespace syn {

constexpr int SMP_THREADS = 1024;

__device__ __forceinline__ uint32_t f2key(float f) {
  uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);  // monotone: larger float -> larger key
}

__global__ void argmax_kernel(const float* __restrict__ logits, int V, int32_t* __restrict__ out) {
  const int t = blockIdx.x;
  const float* lg = logits + (int64_t)t * V;
  float best = -INFINITY;
  int bi = 0x7fffffff;
  for (int i = threadIdx.x; i < V; i += blockDim.x) {
    const float v = lg[i];
    if (v > best || (v == best && i < bi)) { best = v; bi = i; }
  }
  __shared__ float sb[32];
  __shared__ int si[32];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ob = __shfl_xor_sync(0xffffffffu, best, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (ob > best || (ob == best && oi < bi)) { best = ob; bi = oi; }
  }
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  if (lane == 0) { sb[w] = best; si[w] = bi; }
  __syncthreads();
  if (threadIdx.x == 0) {
    float b = sb[0];
    int id = si[0];
    for (int i = 1; i < (int)(blockDim.x >> 5); ++i)
      if (sb[i] > b || (sb[i] == b && si[i] < id)) { b = sb[i]; id = si[i]; }
    out[t] = id;
  }
}

struct SampleArgs {
  const float* logits;       // [T, V]
  int V;
  const float* temperature;  // [T]; <= 0 means greedy
  const int32_t* top_k;      // [T]; <= 0 or >= V: disabled
  const float* top_p;        // [T]; >= 1: disabled
  const int64_t* seed;       // [T]
  const int64_t* stream;     // [T]
  int64_t* counter;          // [T] rng_counter, incremented by one per sampled row
  int32_t* out;              // [T]
};

__global__ void __launch_bounds__(SMP_THREADS) sample_kernel(SampleArgs a) {
  const int t = blockIdx.x;
  const float* lg = a.logits + (int64_t)t * a.V;
  const float temp = a.temperature[t];
  __shared__ float s_red[32];
  __shared__ uint32_t s_hist[256];
  __shared__ unsigned long long s_mass[256];
  __shared__ uint32_t s_prefix, s_want;
  __shared__ unsigned long long s_scan[SMP_THREADS];
  __shared__ int s_pick;

  if (!(temp > 0.f)) {  // greedy
    float best = -INFINITY;
    int bi = 0x7fffffff;
    for (int i = threadIdx.x; i < a.V; i += blockDim.x) {
      const float v = lg[i];
      if (v > best || (v == best && i < bi)) { best = v; bi = i; }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ob = __shfl_xor_sync(0xffffffffu, best, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ob > best || (ob == best && oi < bi)) { best = ob; bi = oi; }
    }
    __shared__ float sb[32];
    __shared__ int si[32];
    if ((threadIdx.x & 31) == 0) { sb[threadIdx.x >> 5] = best; si[threadIdx.x >> 5] = bi; }
    __syncthreads();
    if (threadIdx.x == 0) {
      float b = sb[0];
      int id = si[0];
      for (int i = 1; i < (int)(blockDim.x >> 5); ++i)
        if (sb[i] > b || (sb[i] == b && si[i] < id)) { b = sb[i]; id = si[i]; }
      a.out[t] = id;
    }
    return;
  }
  const float inv_t = 1.f / temp;
  float mx = -INFINITY;
  for (int i = threadIdx.x; i < a.V; i += blockDim.x) mx = fmaxf(mx, lg[i] * inv_t);
  mx = block_max(mx, s_red);

  // ---- top-k threshold key (radix select on f32 key bits, 4 x 8-bit digits) ----
  const int k = a.top_k[t];
  uint32_t kth_key = 0;  // keep z with key >= kth_key
  if (k > 0 && k < a.V) {
    uint32_t prefix = 0;
    uint32_t want = (uint32_t)k;  // rank from the top
    for (int shift = 24; shift >= 0; shift -= 8) {
      for (int i = threadIdx.x; i < 256; i += blockDim.x) s_hist[i] = 0;
      __syncthreads();
      const uint32_t hmask = shift == 24 ? 0u : (0xFFFFFFFFu << (shift + 8));
      for (int i = threadIdx.x; i < a.V; i += blockDim.x) {
        const uint32_t key = f2key(lg[i] * inv_t);
        if ((key & hmask) == (prefix & hmask)) atomicAdd(&s_hist[(key >> shift) & 255u], 1u);
      }
      __syncthreads();
      if (threadIdx.x == 0) {
        uint32_t acc = 0;
        int d = 255;
        for (; d > 0; --d) {
          if (acc + s_hist[d] >= want) break;
          acc += s_hist[d];
        }
        s_prefix = prefix | ((uint32_t)d << shift);
        s_want = want - acc;
      }
      __syncthreads();
      prefix = s_prefix;
      want = s_want;
    }
    kth_key = prefix;
  }

  // ---- fixed-point masses of the top-k candidates ----
  // mass_i = floor(exp(z_i - max) * 2^32)
  auto mass_of = [&](int i) -> unsigned long long {
    const float z = lg[i] * inv_t;
    if (f2key(z) < kth_key) return 0ull;
    return (unsigned long long)(__expf(z - mx) * 4294967296.0f);
  };

  // ---- top-p threshold on mass (radix select over the 64-bit mass, top 40 bits) ----
  const float tp = a.top_p[t];
  unsigned long long mass_floor = 0;  // keep mass >= mass_floor
  if (tp < 1.f) {
    unsigned long long total = 0;
    for (int i = threadIdx.x; i < a.V; i += blockDim.x) total += mass_of(i);
    s_scan[threadIdx.x] = total;
    __syncthreads();
    if (threadIdx.x == 0) {
      unsigned long long s = 0;
      for (int i = 0; i < (int)blockDim.x; ++i) s += s_scan[i];
      s_scan[0] = s;
    }
    __syncthreads();
    total = s_scan[0];
    __syncthreads();
    const unsigned long long need = (unsigned long long)((double)tp * (double)total);
    // masses are < 2^33; select over bits 32..8 in 8-bit digits from the top
    unsigned long long prefix = 0, acc_above = 0;
    for (int shift = 32; shift >= 0; shift -= 8) {
      for (int i = threadIdx.x; i < 256; i += blockDim.x) s_mass[i] = 0;
      __syncthreads();
      const unsigned long long hmask = shift == 32 ? 0ull : (~0ull << (shift + 8));
      for (int i = threadIdx.x; i < a.V; i += blockDim.x) {
        const unsigned long long m = mass_of(i);
        if (m && (m & hmask) == (prefix & hmask)) atomicAdd(&s_mass[(m >> shift) & 255ull], m);
      }
      __syncthreads();
      if (threadIdx.x == 0) {
        unsigned long long acc = acc_above;
        int d = 255;
        for (; d > 0; --d) {
          if (acc + s_mass[d] >= need) break;
          acc += s_mass[d];
        }
        s_scan[0] = prefix | ((unsigned long long)d << shift);
        s_scan[1] = acc;
      }
      __syncthreads();
      prefix = s_scan[0];
      acc_above = s_scan[1];
      __syncthreads();
    }
    mass_floor = prefix;
  }

  // ---- inverse CDF in ascending token order ----
  const int per = (a.V + blockDim.x - 1) / blockDim.x;
  const int i0 = threadIdx.x * per, i1 = min(a.V, i0 + per);
  unsigned long long local = 0;
  for (int i = i0; i < i1; ++i) {
    const unsigned long long m = mass_of(i);
    if (m >= mass_floor) local += m;
  }
  s_scan[threadIdx.x] = local;
  __syncthreads();
  if (threadIdx.x == 0) {  // exclusive scan (fixed order)
    unsigned long long s = 0;
    for (int i = 0; i < (int)blockDim.x; ++i) {
      const unsigned long long v = s_scan[i];
      s_scan[i] = s;
      s += v;
    }
    const uint64_t ctr = (uint64_t)a.counter[t];
    const uint32_t x0 = philox_draw((uint64_t)a.seed[t], (uint64_t)a.stream[t], ctr);
    // target = floor(u * total), u = x0 / 2^32
    const unsigned long long target = __umul64hi((unsigned long long)x0 << 32, s);
    s_hist[0] = (uint32_t)(target >> 32);
    s_hist[1] = (uint32_t)target;
    s_pick = -1;
    a.counter[t] = (int64_t)(ctr + 1);
  }
  __syncthreads();
  const unsigned long long target = ((unsigned long long)s_hist[0] << 32) | s_hist[1];
  unsigned long long run = s_scan[threadIdx.x];
  if (run <= target) {
    for (int i = i0; i < i1; ++i) {
      const unsigned long long m = mass_of(i);
      if (m < mass_floor || m == 0) continue;
      if (run + m > target) { s_pick = i; break; }
      run += m;
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) a.out[t] = s_pick >= 0 ? s_pick : 0;
}

__global__ void philox_kernel(uint64_t seed, uint64_t stream, uint64_t counter0, int n, uint32_t* out) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) out[i] = philox_draw(seed, stream, counter0 + (uint64_t)i);
}

cudaError_t launch_argmax(const float* logits, int T, int V, int32_t* out, cudaStream_t s) {
  if (T == 0) return cudaSuccess;
  argmax_kernel<<<T, 1024, 0, s>>>(logits, V, out);
  return cudaGetLastError();
}

cudaError_t launch_sample(const float* logits, int T, int V, const float* temperature, const int32_t* top_k,
                          const float* top_p, const int64_t* seed, const int64_t* stream, int64_t* counter,
                          int32_t* out, cudaStream_t s) {
  if (T == 0) return cudaSuccess;
  SampleArgs a{logits, V, temperature, top_k, top_p, seed, stream, counter, out};
  sample_kernel<<<T, SMP_THREADS, 0, s>>>(a);
  return cudaGetLastError();
}

cudaError_t launch_philox(uint64_t seed, uint64_t stream, uint64_t counter0, int n, uint32_t* out, cudaStream_t s) {
  philox_kernel<<<(n + 255) / 256, 256, 0, s>>>(seed, stream, counter0, n, out);
  return cudaGetLastError();
}

}  // namespace syn

namespace syn {

// ---------------------------------------------------------------------------------------
// Speculative verification (reference op `VerifyAccept`, plan/rfcs/RFC-0012-execution-
// scheduler.md :605-617; draw order plan/decisions/ADR-0107-counter-based-sampling-rng.md).
// Point-mass drafts d_1..d_g per sequence against target logits rows 0..g:
//   greedy rows : accept d_j while d_j == argmax_j; at the first mismatch emit argmax_j;
//                 if all accepted emit the bonus argmax_g.  No draws.
//   sampled rows: draw u_j; accept iff u_j < p_j(d_j) (p after temperature/top-k/top-p);
//                 at the first rejection draw once more from p_j with d_j removed (the
//                 residual of a point-mass draft); if all accepted draw the bonus from p_g.
//   stochastic drafts (d_j sampled from a draft distribution q_j, given as f32 rows):
//                 accept iff u_j < min(1, p_j(d_j) / q_j(d_j)); at the first rejection draw
//                 from the residual max(0, p_j - q_j) (renormalised); same draw order.  p and q
//                 are compared in units of 2^-32 with exact integer rules (floor(q * 2^32)
//                 masses; r = floor((2^64-1) / total), each (m * r) >> 32), so the host oracle
//                 reproduces every decision bit for bit.
// The output distribution equals sampling from the target alone.


// Argmax over a row (all threads participate; ties to the lower index).
__device__ int block_argmax(const float* lg, int V, float* sb, int* si) {
  float best = -INFINITY;
  int bi = 0x7fffffff;
  for (int i = threadIdx.x; i < V; i += blockDim.x) {
    const float v = lg[i];
    if (v > best || (v == best && i < bi)) { best = v; bi = i; }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ob = __shfl_xor_sync(0xffffffffu, best, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (ob > best || (ob == best && oi < bi)) { best = ob; bi = oi; }
  }
  __syncthreads();
  if ((threadIdx.x & 31) == 0) { sb[threadIdx.x >> 5] = best; si[threadIdx.x >> 5] = bi; }
  __syncthreads();
  if (threadIdx.x == 0) {
    float b = sb[0];
    int id = si[0];
    for (int i = 1; i < (int)(blockDim.x >> 5); ++i)
      if (sb[i] > b || (sb[i] == b && si[i] < id)) { b = sb[i]; id = si[i]; }
    si[0] = id;
  }
  __syncthreads();
  const int r = si[0];
  __syncthreads();
  return r;
}

// Fixed-point masses with temperature and top-k / top-p thresholds, as in sample_kernel.
struct RowDist {
  float inv_t, mx;
  uint32_t kth_key;
  unsigned long long floor_mass;
};

__device__ __forceinline__ unsigned long long row_mass(const float* lg, const RowDist& d, int i) {
  const float z = lg[i] * d.inv_t;
  if (f2key(z) < d.kth_key) return 0ull;
  const unsigned long long m = (unsigned long long)(__expf(z - d.mx) * 4294967296.0f);
  return m >= d.floor_mass ? m : 0ull;
}

__device__ void row_setup(const float* lg, int V, float temp, int k, float tp, RowDist& d, float* red,
                          uint32_t* hist, unsigned long long* mhist, unsigned long long* scan) {
  d.inv_t = 1.f / temp;
  float mx = -INFINITY;
  for (int i = threadIdx.x; i < V; i += blockDim.x) mx = fmaxf(mx, lg[i] * d.inv_t);
  d.mx = block_max(mx, red);
  d.kth_key = 0;
  d.floor_mass = 0;
  if (k > 0 && k < V) {
    uint32_t prefix = 0, want = (uint32_t)k;
    for (int shift = 24; shift >= 0; shift -= 8) {
      for (int i = threadIdx.x; i < 256; i += blockDim.x) hist[i] = 0;
      __syncthreads();
      const uint32_t hmask = shift == 24 ? 0u : (0xFFFFFFFFu << (shift + 8));
      for (int i = threadIdx.x; i < V; i += blockDim.x) {
        const uint32_t key = f2key(lg[i] * d.inv_t);
        if ((key & hmask) == (prefix & hmask)) atomicAdd(&hist[(key >> shift) & 255u], 1u);
      }
      __syncthreads();
      if (threadIdx.x == 0) {
        uint32_t acc = 0;
        int dd = 255;
        for (; dd > 0; --dd) {
          if (acc + hist[dd] >= want) break;
          acc += hist[dd];
        }
        hist[256] = prefix | ((uint32_t)dd << shift);
        hist[257] = want - acc;
      }
      __syncthreads();
      prefix = hist[256];
      want = hist[257];
      __syncthreads();
    }
    d.kth_key = prefix;
  }
  if (tp < 1.f) {
    unsigned long long tot = 0;
    for (int i = threadIdx.x; i < V; i += blockDim.x) tot += row_mass(lg, d, i);
    scan[threadIdx.x] = tot;
    __syncthreads();
    if (threadIdx.x == 0) {
      unsigned long long s = 0;
      for (int i = 0; i < (int)blockDim.x; ++i) s += scan[i];
      scan[0] = s;
    }
    __syncthreads();
    const unsigned long long need = (unsigned long long)((double)tp * (double)scan[0]);
    __syncthreads();
    unsigned long long prefix = 0, acc_above = 0;
    for (int shift = 32; shift >= 0; shift -= 8) {
      for (int i = threadIdx.x; i < 256; i += blockDim.x) mhist[i] = 0;
      __syncthreads();
      const unsigned long long hmask = shift == 32 ? 0ull : (~0ull << (shift + 8));
      for (int i = threadIdx.x; i < V; i += blockDim.x) {
        const unsigned long long m = row_mass(lg, d, i);
        if (m && (m & hmask) == (prefix & hmask)) atomicAdd(&mhist[(m >> shift) & 255ull], m);
      }
      __syncthreads();
      if (threadIdx.x == 0) {
        unsigned long long acc = acc_above;
        int dd = 255;
        for (; dd > 0; --dd) {
          if (acc + mhist[dd] >= need) break;
          acc += mhist[dd];
        }
        scan[0] = prefix | ((unsigned long long)dd << shift);
        scan[1] = acc;
      }
      __syncthreads();
      prefix = scan[0];
      acc_above = scan[1];
      __syncthreads();
    }
    d.floor_mass = prefix;
  }
}

// Inverse-CDF draw over the row's masses with token `exclude` removed (-1: none).
__device__ int row_draw(const float* lg, int V, const RowDist& d, int exclude, uint32_t x0,
                        unsigned long long* scan, int* pick) {
  const int per = (V + blockDim.x - 1) / blockDim.x;
  const int i0 = threadIdx.x * per, i1 = min(V, i0 + per);
  unsigned long long local = 0;
  for (int i = i0; i < i1; ++i)
    if (i != exclude) local += row_mass(lg, d, i);
  scan[threadIdx.x] = local;
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned long long s = 0;
    for (int i = 0; i < (int)blockDim.x; ++i) {
      const unsigned long long v = scan[i];
      scan[i] = s;
      s += v;
    }
    scan[blockDim.x] = __umul64hi((unsigned long long)x0 << 32, s);
    *pick = -1;
  }
  __syncthreads();
  const unsigned long long target = scan[blockDim.x];
  unsigned long long run = scan[threadIdx.x];
  if (run <= target) {
    for (int i = i0; i < i1; ++i) {
      if (i == exclude) continue;
      const unsigned long long m = row_mass(lg, d, i);
      if (m == 0) continue;
      if (run + m > target) { *pick = i; break; }
      run += m;
    }
  }
  __syncthreads();
  const int r = *pick >= 0 ? *pick : 0;
  __syncthreads();
  return r;
}

__device__ __forceinline__ unsigned long long draft_mass(const float* q, int i) {
  const float v = q[i];
  return v > 0.f ? (unsigned long long)(v * 4294967296.0f) : 0ull;
}

// Residual draw max(0, pn - qn) over the row (or from pn when the residual is empty).
__device__ int resid_draw(const float* lg, const float* q, int V, const RowDist& d, unsigned long long rp,
                          unsigned long long rq, uint32_t x0, unsigned long long* scan, int* pick) {
  const int per = (V + blockDim.x - 1) / blockDim.x;
  const int i0 = threadIdx.x * per, i1 = min(V, i0 + per);
  __shared__ int s_plain;
  for (int pass = 0; pass < 2; ++pass) {
    // pass 0: residual masses; pass 1 (only if the residual sums to 0): the target's own
    unsigned long long local = 0;
    for (int i = i0; i < i1; ++i) {
      const unsigned long long pn = (row_mass(lg, d, i) * rp) >> 32;
      const unsigned long long qn = (draft_mass(q, i) * rq) >> 32;
      local += pass ? pn : (pn > qn ? pn - qn : 0ull);
    }
    scan[threadIdx.x] = local;
    __syncthreads();
    if (threadIdx.x == 0) {
      unsigned long long s = 0;
      for (int i = 0; i < (int)blockDim.x; ++i) {
        const unsigned long long v = scan[i];
        scan[i] = s;
        s += v;
      }
      s_plain = s == 0ull;
      scan[blockDim.x] = __umul64hi((unsigned long long)x0 << 32, s);
      *pick = -1;
    }
    __syncthreads();
    if (pass == 0 && s_plain) {
      __syncthreads();
      continue;
    }
    const unsigned long long target = scan[blockDim.x];
    unsigned long long run = scan[threadIdx.x];
    if (run <= target) {
      for (int i = i0; i < i1; ++i) {
        const unsigned long long pn = (row_mass(lg, d, i) * rp) >> 32;
        const unsigned long long qn = (draft_mass(q, i) * rq) >> 32;
        const unsigned long long m = pass ? pn : (pn > qn ? pn - qn : 0ull);
        if (m == 0) continue;
        if (run + m > target) { *pick = i; break; }
        run += m;
      }
    }
    __syncthreads();
    break;
  }
  const int r = *pick >= 0 ? *pick : 0;
  __syncthreads();
  return r;
}

__global__ void __launch_bounds__(SMP_THREADS) verify_accept_kernel(VerifyArgs a) {
  __shared__ float red[32];
  __shared__ float sb[32];
  __shared__ int si[32];
  __shared__ uint32_t hist[258];
  __shared__ unsigned long long mhist[256];
  __shared__ unsigned long long scan[SMP_THREADS + 1];
  __shared__ int pick;
  __shared__ unsigned long long s_tot, s_md;
  const int sq = blockIdx.x;
  const int g = a.g;
  const float temp = a.temperature[sq];
  uint64_t ctr = (uint64_t)a.counter[sq];
  int n_acc = g;
  int last = 0;
  for (int j = 0; j <= g; ++j) {
    const float* lg = a.logits + ((int64_t)sq * (g + 1) + j) * a.V;
    const int dj = j < g ? a.draft[sq * g + j] : -1;
    int tok;
    if (!(temp > 0.f)) {
      tok = block_argmax(lg, a.V, sb, si);
      if (j < g && tok == dj) {
        if (threadIdx.x == 0) a.out_tokens[sq * (g + 1) + j] = dj;
        continue;
      }
    } else {
      RowDist d;
      row_setup(lg, a.V, temp, a.top_k[sq], a.top_p[sq], d, red, hist, mhist, scan);
      if (j < g) {
        unsigned long long loc = 0;
        for (int i = threadIdx.x; i < a.V; i += blockDim.x) loc += row_mass(lg, d, i);
        scan[threadIdx.x] = loc;
        __syncthreads();
        if (threadIdx.x == 0) {
          unsigned long long s = 0;
          for (int i = 0; i < (int)blockDim.x; ++i) s += scan[i];
          s_tot = s;
          s_md = (dj >= 0 && dj < a.V) ? row_mass(lg, d, dj) : 0ull;
        }
        __syncthreads();
        const uint32_t u = philox_draw((uint64_t)a.seed[sq], (uint64_t)a.stream[sq], ctr++);
        if (a.draft_probs != nullptr) {
          // stochastic draft: accept iff u * qn(d) < pn(d) * 2^32, else draw the residual
          const float* q = a.draft_probs + ((int64_t)sq * g + j) * a.V;
          unsigned long long ql = 0;
          for (int i = threadIdx.x; i < a.V; i += blockDim.x) ql += draft_mass(q, i);
          scan[threadIdx.x] = ql;
          __syncthreads();
          __shared__ unsigned long long s_rp, s_rq;
          __shared__ int s_acc;
          if (threadIdx.x == 0) {
            unsigned long long qs = 0;
            for (int i = 0; i < (int)blockDim.x; ++i) qs += scan[i];
            s_rp = s_tot ? ~0ull / s_tot : 0ull;
            s_rq = qs ? ~0ull / qs : 0ull;
            const bool in = dj >= 0 && dj < a.V;
            const unsigned long long pn = (s_md * s_rp) >> 32;
            const unsigned long long qn = in ? (draft_mass(q, dj) * s_rq) >> 32 : 0ull;
            s_acc = in && (unsigned long long)u * qn < (pn << 32);
          }
          __syncthreads();
          if (s_acc) {
            if (threadIdx.x == 0) a.out_tokens[sq * (g + 1) + j] = dj;
            __syncthreads();
            continue;
          }
          tok = resid_draw(lg, q, a.V, d, s_rp, s_rq,
                           philox_draw((uint64_t)a.seed[sq], (uint64_t)a.stream[sq], ctr++), scan, &pick);
          if (threadIdx.x == 0) a.out_tokens[sq * (g + 1) + j] = tok;
          n_acc = j;
          break;
        }
        const unsigned long long thr = __umul64hi((unsigned long long)u << 32, s_tot);  // floor(u * total)
        if (thr < s_md) {
          if (threadIdx.x == 0) a.out_tokens[sq * (g + 1) + j] = dj;
          __syncthreads();
          continue;
        }
        tok = row_draw(lg, a.V, d, dj, philox_draw((uint64_t)a.seed[sq], (uint64_t)a.stream[sq], ctr++), scan,
                       &pick);
      } else {
        tok = row_draw(lg, a.V, d, -1, philox_draw((uint64_t)a.seed[sq], (uint64_t)a.stream[sq], ctr++), scan,
                       &pick);
      }
    }
    if (threadIdx.x == 0) a.out_tokens[sq * (g + 1) + j] = tok;
    n_acc = j < g ? j : g;
    last = j;
    break;
  }
  (void)last;
  if (threadIdx.x == 0) {
    a.n_accept[sq] = n_acc;
    a.counter[sq] = (int64_t)ctr;
  }
}

cudaError_t launch_verify_accept(const VerifyArgs& a, cudaStream_t s) {
  if (a.S == 0) return cudaSuccess;
  verify_accept_kernel<<<a.S, SMP_THREADS, 0, s>>>(a);
  return cudaGetLastError();
}

}  // namespace syn
