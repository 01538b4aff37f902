// GPU side of the CPU expert hand-off during decode (mailbox in syn/cpu_mailbox.h; the host
// side is csrc/cpu/cpu_experts.cpp).  Reference: crates/kernels/src/moe/doorbell.rs (doorbell
// layer in host-mapped memory) and the MoE split of RFC-0040 §3.4 (hit / miss / CPU sites).
//
//  * cpu_handoff_kernel: after routing, copies the layer's rows and routing CSR into the
//    mailbox, then the last CTA to arrive raises the go word to the next sequence number
//    (data, system fence, arrival counter, release store).
//  * cpu_collect_kernel: after the GPU's own expert GEMVs, waits (bounded by a time limit; on
//    timeout it sets a status bit and returns, never hangs) for the done word to reach that
//    sequence, then copies each CPU output row into the pair slot the combine reads.
#include "common.cuh"
#include "sync.cuh"
#include "syn/cpu_mailbox.h"
#include "syn/launch.h"

namespace syn {

__global__ void __launch_bounds__(256) cpu_handoff_kernel(CpuHandoffArgs a) {
  const int64_t gtid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  const CpuMailboxLayout lay = cpu_mailbox_layout(a.E, a.k, a.max_rows, a.H);
  const int64_t nh = (int64_t)a.B * a.H / 8;
  const uint4* src = reinterpret_cast<const uint4*>(a.h);
  uint4* dst = reinterpret_cast<uint4*>(a.mb + lay.h);
  for (int64_t i = gtid; i < nh; i += stride) dst[i] = src[i];
  int32_t* off = reinterpret_cast<int32_t*>(a.mb + lay.tok_off);
  for (int64_t i = gtid; i <= a.E; i += stride) off[i] = a.tok_off[i];
  const int64_t P = (int64_t)a.B * a.k;
  int32_t* tidx = reinterpret_cast<int32_t*>(a.mb + lay.tok_idx);
  float* pw = reinterpret_cast<float*>(a.mb + lay.pair_w);
  for (int64_t i = gtid; i < P; i += stride) {
    tidx[i] = a.tok_idx[i];
    pw[i] = a.pair_w[i];
  }
  __threadfence_system();
  __syncthreads();
  __shared__ int last;
  if (threadIdx.x == 0) last = atomicAdd(&a.ctr[1], 1u) == gridDim.x - 1;
  __syncthreads();
  if (!last || threadIdx.x != 0) return;
  __threadfence();
  const uint32_t seq = a.ctr[0] + 1;
  a.ctr[0] = seq;
  a.ctr[1] = 0;
  uint32_t* w = reinterpret_cast<uint32_t*>(a.mb);
  w[MB_LAYER] = (uint32_t)a.layer;
  w[MB_ROWS] = (uint32_t)a.B;
  __threadfence_system();
  st_release_sys(&w[MB_GO], seq);
}

__global__ void __launch_bounds__(256) cpu_collect_kernel(CpuCollectArgs a) {
  __shared__ int n_out;
  const uint32_t* w = reinterpret_cast<const uint32_t*>(a.mb);
  if (threadIdx.x == 0) {
    const uint32_t seq = a.ctr[0];
    int n = 0;
    if (wait_flag(&w[MB_DONE], seq, a.timeout_ns, a.status, 0)) {
      n = (int)ld_acquire_sys(&w[MB_NOUT]);
      if (ld_acquire_sys(&w[MB_ERR]) != 0u || n < 0 || n > a.max_rows * a.k) {
        atomicOr(a.status, 2);
        n = 0;
      }
    }
    n_out = n;
  }
  __syncthreads();
  const CpuMailboxLayout lay = cpu_mailbox_layout(a.E, a.k, a.max_rows, a.H);
  const int32_t* pairs = reinterpret_cast<const int32_t*>(a.mb + lay.out_pairs);
  const float4* out = reinterpret_cast<const float4*>(a.mb + lay.out);
  const int H4 = a.H / 4;
  // host memory written by the CPU since the last layer: uncached loads
  for (int i = blockIdx.x; i < n_out; i += gridDim.x) {
    const int p = __ldcv(pairs + i);
    if (p < 0 || p >= a.max_rows * a.k) continue;
    float4* y = a.pair_dst ? reinterpret_cast<float4*>(a.pair_dst[p])
                           : reinterpret_cast<float4*>(a.yp + (int64_t)p * a.H);
    if (y == nullptr) continue;
    for (int c = threadIdx.x; c < H4; c += blockDim.x) y[c] = __ldcv(out + (int64_t)i * H4 + c);
  }
  if (a.sig_n > 0) {
    // the GEMV of this layer left the flags to this kernel: every CTA publishes its stores,
    // the last one to arrive raises every rank's flag (counter reset before the release)
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x == 0) {
      const unsigned prev = atomicAdd(a.done_ctr, 1u);
      if (prev == gridDim.x - 1) {
        *a.done_ctr = 0u;
        __threadfence_system();
        const uint32_t seq = (*a.step_ctr) * (uint32_t)a.n_layers + (uint32_t)a.layer + 1u;
        for (int q = 0; q < a.sig_n; ++q)
          st_release_sys(reinterpret_cast<uint32_t*>(a.sig_peers[q] + a.sig_off) + a.sig_rank, seq);
      }
    }
  }
}

cudaError_t launch_cpu_handoff(const CpuHandoffArgs& a, cudaStream_t s) {
  if (a.H % 8 || a.B > a.max_rows) return cudaErrorInvalidValue;
  const int64_t nh = (int64_t)a.B * a.H / 8;
  const int blocks = (int)std::min<int64_t>(32, std::max<int64_t>(1, (nh + 255) / 256));
  cpu_handoff_kernel<<<blocks, 256, 0, s>>>(a);
  return cudaGetLastError();
}

cudaError_t launch_cpu_collect(const CpuCollectArgs& a, cudaStream_t s) {
  if (a.H % 4) return cudaErrorInvalidValue;
  cpu_collect_kernel<<<64, 256, 0, s>>>(a);
  return cudaGetLastError();
}

}  // namespace syn
