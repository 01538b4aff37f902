// Ordered two-shot all-reduce of f32 partials over NVLink peer memory (tensor-parallel prefill,
// MiB-scale messages), in two kernels:
//   tp_twoshot_rs_kernel   every rank publishes that its partial [T, H] (in its symmetric region)
//                          is complete, then sums ITS 1/N element slice over all ranks' partials
//                          in rank order 0..N-1 (plain 16-byte loads of peer memory), and stores
//                          the sum into the same slice of every rank's gather buffer; the last
//                          CTA raises this rank's done flag on every rank.
//   tp_twoshot_add_kernel  waits for every rank's done flag, adds the gathered sums to the
//                          residual x [T, H] and optionally applies the next RMSNorm.
// Each element is summed once, by its slice owner, so every rank ends with the same bits, and
// the result does not depend on timing (the order is fixed).  Per rank, (N-1)/N of the message
// crosses NVLink in each direction: the bandwidth-optimal volume of a ring, in two steps.
// Every wait is bounded (a status bit, then the kernel skips the data it waited for).
// Buffer reuse: a rank rewrites its partial only after its add kernel saw every done flag,
// i.e. after every peer finished reading it; a peer pushes into this rank's gather buffer only
// after this rank published its next partial, i.e. after its previous add kernel.
// Reference: plan/rfcs/RFC-0040-kernel-providers-and-backends.md:990 (one-shot for small
// messages, two-shot reduce-scatter + all-gather for large ones, rank order for determinism).
#include "common.cuh"
#include "sync.cuh"
#include "syn/launch.h"

namespace syn {

namespace {

__global__ void __launch_bounds__(256) tp_twoshot_rs_kernel(TwoShotArgs a) {
  __shared__ int s_ok;
  uint8_t* mine = reinterpret_cast<uint8_t*>(a.peers[a.rank]);
  // publish: the partial was written by earlier work on this stream; every CTA stores the same
  // sequence number, so the flag is up whichever CTAs run first
  if (threadIdx.x < a.N) {
    __threadfence_system();
    uint8_t* peer = reinterpret_cast<uint8_t*>(a.peers[threadIdx.x]);
    st_release_sys(reinterpret_cast<uint32_t*>(peer + a.off_flag_ready) + a.rank, a.seq);
  }
  if (threadIdx.x == 0) s_ok = 1;
  __syncthreads();
  if (threadIdx.x < a.N) {
    const uint32_t* f = reinterpret_cast<const uint32_t*>(mine + a.off_flag_ready) + threadIdx.x;
    if (!wait_flag(f, a.seq, a.timeout_ns, a.status, 3)) s_ok = 0;
  }
  __syncthreads();
  const int64_t n4 = a.n_elems / 4;
  const int64_t lo = n4 * a.rank / a.N, hi = n4 * (a.rank + 1) / a.N;  // this rank's float4 slice
  if (s_ok) {
    // four float4 per thread in flight from every rank before any add: remote loads take
    // microseconds, so the memory-level parallelism sets the rate
    constexpr int U = 4;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t i0 = lo + (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i0 < hi; i0 += U * stride) {
      float4 acc[U];
#pragma unroll
      for (int u = 0; u < U; ++u) acc[u] = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int r = 0; r < a.N; ++r) {  // rank order: identical bits on every rank
        const float4* src = reinterpret_cast<const float4*>(reinterpret_cast<const uint8_t*>(a.peers[r]) + a.off_part);
        float4 v[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
          const int64_t i = i0 + u * stride;
          v[u] = i < hi ? __ldcg(src + i) : make_float4(0.f, 0.f, 0.f, 0.f);
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
          acc[u].x += v[u].x;
          acc[u].y += v[u].y;
          acc[u].z += v[u].z;
          acc[u].w += v[u].w;
        }
      }
      for (int r = 0; r < a.N; ++r) {
        float4* dst = reinterpret_cast<float4*>(reinterpret_cast<uint8_t*>(a.peers[r]) + a.off_gather);
#pragma unroll
        for (int u = 0; u < U; ++u) {
          const int64_t i = i0 + u * stride;
          if (i < hi) dst[i] = acc[u];
        }
      }
    }
  }
  // completion of this rank's slice: the last CTA raises the done flag on every rank
  __shared__ bool s_last;
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    const unsigned prev = atomicAdd(a.done_ctr, 1u);
    s_last = prev == gridDim.x - 1;
  }
  __syncthreads();
  if (s_last && threadIdx.x < a.N) {
    if (threadIdx.x == 0) *a.done_ctr = 0u;
    __threadfence_system();
    uint8_t* peer = reinterpret_cast<uint8_t*>(a.peers[threadIdx.x]);
    st_release_sys(reinterpret_cast<uint32_t*>(peer + a.off_flag_done) + a.rank, a.seq);
  }
}

// grid = T rows, block 256: x[t] += gathered[t]; h = rmsnorm(x[t]) * wn (when wn is given)
__global__ void __launch_bounds__(256) tp_twoshot_add_kernel(TwoShotArgs a, float* __restrict__ x,
                                                             const float* __restrict__ wn,
                                                             __nv_bfloat16* __restrict__ hout, float eps) {
  __shared__ float red[32];
  __shared__ int s_ok;
  const int t = blockIdx.x;
  const uint8_t* mine = reinterpret_cast<const uint8_t*>(a.peers[a.rank]);
  if (threadIdx.x == 0) s_ok = 1;
  __syncthreads();
  if (threadIdx.x < a.N) {
    const uint32_t* f = reinterpret_cast<const uint32_t*>(mine + a.off_flag_done) + threadIdx.x;
    if (!wait_flag(f, a.seq, a.timeout_ns, a.status, 3)) s_ok = 0;
  }
  __syncthreads();
  const float4* g = reinterpret_cast<const float4*>(mine + a.off_gather) + (int64_t)t * (a.H / 4);
  float4* xr4 = reinterpret_cast<float4*>(x + (int64_t)t * a.H);
  const float* xr = x + (int64_t)t * a.H;
  float ss = 0.f;
  for (int i = threadIdx.x; i < a.H / 4; i += blockDim.x) {
    float4 v = xr4[i];
    if (s_ok) {
      const float4 d = __ldcg(g + i);
      v.x += d.x;
      v.y += d.y;
      v.z += d.z;
      v.w += d.w;
    }
    xr4[i] = v;
    ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
  }
  __syncthreads();  // x rows are re-read by other threads for the norm below
  if (wn == nullptr) return;
  ss = block_sum(ss, red);
  const float rr = rsqrtf(ss / (float)a.H + eps);
  for (int i = threadIdx.x; i < a.H; i += blockDim.x) hout[(int64_t)t * a.H + i] = f2bf(xr[i] * rr * wn[i]);
}

}  // namespace

cudaError_t launch_tp_twoshot(const TwoShotArgs& a, float* x, const float* wn, void* hout, float eps, int T,
                              cudaStream_t s) {
  if (T <= 0) return cudaSuccess;
  if (a.N < 1 || a.N > 32 || a.H % 4 != 0 || a.n_elems != (int64_t)T * a.H || (a.off_part | a.off_gather) & 15 ||
      (reinterpret_cast<uintptr_t>(x) & 15))
    return cudaErrorInvalidValue;
  static int n_sm = 0;
  if (n_sm == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n_sm, cudaDevAttrMultiProcessorCount, dev);
  }
  const int64_t slice4 = a.n_elems / 4 / a.N + 1;
  const int blocks = (int)std::min<int64_t>(4 * n_sm, (slice4 + 255) / 256);
  tp_twoshot_rs_kernel<<<blocks, 256, 0, s>>>(a);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  tp_twoshot_add_kernel<<<T, 256, 0, s>>>(a, x, wn, reinterpret_cast<__nv_bfloat16*>(hout), eps);
  return cudaGetLastError();
}

}  // namespace syn
