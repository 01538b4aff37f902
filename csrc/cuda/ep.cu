// Expert-parallel MoE dispatch and combine over NVLink peer memory (decode path).
//
// Reference semantics: EP dispatch / combine (plan/rfcs/RFC-0032-distributed-execution.md
// :415-424; frame codec crates/net/src/frame/ep.rs) — each row is sent once per owner
// rank with its expert ids and weights; owners return per-(token, expert) f32 outputs that
// the source sums in ascending expert order.
//
// Data path (one process per GPU, symmetric region mapped by CUDA IPC on every rank):
//   ep_dispatch  (source)  : P2P stores of each routed row + routing metadata into the
//                            owner's receive slots, then a release flag per owner.
//   ep_build     (owner)   : bounded acquire-waits on every source's flag, then CSR lists
//                            of the owner's local experts and, per pair, the peer address
//                            its result row goes to.
//   grouped GEMV (owner)   : gate_up (SwiGLU) on the received rows; down projection whose
//                            epilogue stores each f32 row straight into the source's
//                            combine buffer over NVLink, last CTA raising the flags
//                            (csrc/cuda/q4_gemv.cu, mode GEMV_SCALED_F32_PTR).
//   ep_combine   (source)  : bounded waits on every owner's flag, x += sum of the k rows
//                            in ascending expert order, then the next RMSNorm.
// Sequence numbers (step * n_layers + layer + 1) make every flag monotone, so nothing is
// ever reset and CUDA-graph replays need no host work.
#include "common.cuh"
#include "sync.cuh"

namespace syn {

__device__ __forceinline__ uint32_t ep_seq(const uint32_t* step_ctr, int n_layers, int layer) {
  return (*step_ctr) * (uint32_t)n_layers + (uint32_t)layer + 1u;
}

__global__ void ep_step_begin_kernel(uint32_t* step_ctr) { *step_ctr += 1u; }

cudaError_t launch_ep_step_begin(uint32_t* step_ctr, cudaStream_t s) {
  ep_step_begin_kernel<<<1, 1, 0, s>>>(step_ctr);
  return cudaGetLastError();
}

// grid = N (destination rank), block = 256.  T <= 256.
__global__ void __launch_bounds__(256) ep_dispatch_kernel(EpArgs a, const __nv_bfloat16* __restrict__ h,
                                                          const int32_t* __restrict__ ids,
                                                          const float* __restrict__ w, int T) {
  const int r = blockIdx.x;
  const int t = threadIdx.x;
  const int lane = t & 31, warp = t >> 5;
  __shared__ int s_slot[256];
  __shared__ int s_warp[8];
  __shared__ int s_total;
  const int e_lo = r * a.E_loc, e_hi = e_lo + a.E_loc;
  int send = 0;
  if (t < T) {
    for (int j = 0; j < a.k; ++j) {
      const int e = ids[t * a.k + j];
      send |= (e >= e_lo && e < e_hi);
    }
  }
  // block exclusive scan of `send`
  const unsigned m = __ballot_sync(0xffffffffu, send);
  const int pre = __popc(m & ((1u << lane) - 1u));
  if (lane == 0) s_warp[warp] = __popc(m);
  __syncthreads();
  int base = 0;
  for (int i = 0; i < warp; ++i) base += s_warp[i];
  s_slot[t] = send ? base + pre : -1;
  if (t == 0) {
    int tot = 0;
    for (int i = 0; i < (int)(blockDim.x >> 5); ++i) tot += s_warp[i];
    s_total = tot;
  }
  __syncthreads();
  uint8_t* peer = reinterpret_cast<uint8_t*>(a.peers[r]);
  const int me = a.rank;
  // metadata: per slot [t, (e_local, w bits, comb_row) x k]
  const int MS = 1 + 3 * a.k;
  int32_t* meta = reinterpret_cast<int32_t*>(peer + a.off_meta) + ((int64_t)me * a.cap) * MS;
  __nv_bfloat16* rx = reinterpret_cast<__nv_bfloat16*>(peer + a.off_x) + ((int64_t)me * a.cap) * a.H;
  if (t < T && s_slot[t] >= 0) {
    const int slot = s_slot[t];
    int32_t* mrow = meta + (int64_t)slot * MS;
    mrow[0] = t;
    for (int j = 0; j < a.k; ++j) {
      const int e = ids[t * a.k + j];
      int rank_in_tok = 0;  // ascending-expert slot of choice j
      for (int j2 = 0; j2 < a.k; ++j2) rank_in_tok += ids[t * a.k + j2] < e;
      const bool mine = e >= e_lo && e < e_hi;
      mrow[1 + 3 * j] = mine ? e - e_lo : -1;
      mrow[2 + 3 * j] = __float_as_int(w[t * a.k + j]);
      mrow[3 + 3 * j] = t * a.k + rank_in_tok;
    }
  }
  // rows: one warp per sending token, 16-byte stores
  const int nchunk = a.H / 8;
  for (int tt = warp; tt < T; tt += blockDim.x >> 5) {
    const int slot = s_slot[tt];
    if (slot < 0) continue;
    const uint4* src = reinterpret_cast<const uint4*>(h + (int64_t)tt * a.H);
    uint4* dst = reinterpret_cast<uint4*>(rx + (int64_t)slot * a.H);
    for (int c = lane; c < nchunk; c += 32) dst[c] = src[c];
  }
  if (t == 0) reinterpret_cast<int32_t*>(peer + a.off_cnt)[me] = s_total;
  __threadfence_system();
  __syncthreads();
  if (t == 0) {
    const uint32_t seq = ep_seq(a.step_ctr, a.n_layers, a.layer);
    st_release_sys(reinterpret_cast<uint32_t*>(peer + a.off_flag_disp) + me, seq);
  }
}

// 1 CTA x 1024 threads on the owner rank.
__global__ void __launch_bounds__(1024) ep_build_kernel(EpArgs a, int32_t* __restrict__ tok_off,
                                                        int32_t* __restrict__ tok_idx, float* __restrict__ pair_w,
                                                        int64_t* __restrict__ pair_dst) {
  __shared__ int s_cnt[512];
  __shared__ int s_src_cnt[64];
  uint8_t* mine = reinterpret_cast<uint8_t*>(a.peers[a.rank]);
  const uint32_t seq = ep_seq(a.step_ctr, a.n_layers, a.layer);
  const int tid = threadIdx.x;
  if (tid < a.N) {
    const uint32_t* f = reinterpret_cast<const uint32_t*>(mine + a.off_flag_disp) + tid;
    const bool ok = wait_flag(f, seq, a.timeout_ns, a.status, 0);
    s_src_cnt[tid] = ok ? reinterpret_cast<volatile int32_t*>(mine + a.off_cnt)[tid] : 0;
  }
  for (int e = tid; e < a.E_loc; e += blockDim.x) s_cnt[e] = 0;
  __syncthreads();
  const int MS = 1 + 3 * a.k;
  const int32_t* meta = reinterpret_cast<const int32_t*>(mine + a.off_meta);
  // counts per local expert
  for (int s = 0; s < a.N; ++s) {
    const int n = min(s_src_cnt[s], a.cap);
    for (int idx = tid; idx < n * a.k; idx += blockDim.x) {
      const int slot = idx / a.k, j = idx % a.k;
      const int el = meta[((int64_t)s * a.cap + slot) * MS + 1 + 3 * j];
      if (el >= 0) atomicAdd(&s_cnt[el], 1);
    }
  }
  __syncthreads();
  if (tid == 0) {
    int acc = 0;
    for (int e = 0; e < a.E_loc; ++e) {
      tok_off[e] = acc;
      const int c = s_cnt[e];
      s_cnt[e] = acc;
      acc += c;
    }
    tok_off[a.E_loc] = acc;
  }
  __syncthreads();
  // fill in (source, slot) order per expert: deterministic
  for (int e = tid; e < a.E_loc; e += blockDim.x) {
    int p = s_cnt[e];
    for (int s = 0; s < a.N; ++s) {
      const int n = min(s_src_cnt[s], a.cap);
      for (int slot = 0; slot < n; ++slot) {
        const int32_t* mrow = meta + ((int64_t)s * a.cap + slot) * MS;
        for (int j = 0; j < a.k; ++j) {
          if (mrow[1 + 3 * j] == e) {
            tok_idx[p] = s * a.cap + slot;
            pair_w[p] = __int_as_float(mrow[2 + 3 * j]);
            pair_dst[p] = a.peers[s] + a.off_comb + (int64_t)mrow[3 + 3 * j] * a.H * 4;
            ++p;
          }
        }
      }
    }
  }
}

// grid = T, block = 256.  x[t] += sum_j comb[t*k + j]; h = rmsnorm(x) * w (if w).
__global__ void ep_combine_kernel(EpArgs a, float* __restrict__ x, const float* __restrict__ wn,
                                  __nv_bfloat16* __restrict__ hout, float eps) {
  __shared__ float red[32];
  __shared__ int s_ok;
  const int t = blockIdx.x;
  uint8_t* mine = reinterpret_cast<uint8_t*>(a.peers[a.rank]);
  const uint32_t seq = ep_seq(a.step_ctr, a.n_layers, a.layer);
  if (threadIdx.x == 0) s_ok = 1;
  __syncthreads();
  if (threadIdx.x < a.N) {
    const uint32_t* f = reinterpret_cast<const uint32_t*>(mine + a.off_flag_comb) + threadIdx.x;
    if (!wait_flag(f, seq, a.timeout_ns, a.status, 1)) s_ok = 0;
  }
  __syncthreads();
  const float* comb = reinterpret_cast<const float*>(mine + a.off_comb) + (int64_t)t * a.k * a.H;
  float* xr = x + (int64_t)t * a.H;
  float ss = 0.f;
  for (int i = threadIdx.x; i < a.H; i += blockDim.x) {
    float acc = 0.f;
    if (s_ok)
      for (int j = 0; j < a.k; ++j) acc += comb[(int64_t)j * a.H + i];
    const float v = xr[i] + acc;
    xr[i] = v;
    ss += v * v;
  }
  if (wn == nullptr) return;
  ss = block_sum(ss, red);
  const float r = rsqrtf(ss / (float)a.H + eps);
  for (int i = threadIdx.x; i < a.H; i += blockDim.x) hout[(int64_t)t * a.H + i] = f2bf(xr[i] * r * wn[i]);
}

// TP one-shot all-reduce, receive side: every rank pushed its f32 partial rows into slot
// [src][row] of this rank's receive area; sum them in rank order (identical bits on every
// rank), add to the residual, and apply the next RMSNorm.  grid = T, block = 256.
__global__ void tp_reduce_norm_kernel(EpArgs a, int64_t off_recv, int64_t off_flag, float* __restrict__ x,
                                      const float* __restrict__ wn, __nv_bfloat16* __restrict__ hout, float eps) {
  __shared__ float red[32];
  __shared__ int s_ok;
  const int t = blockIdx.x;
  uint8_t* mine = reinterpret_cast<uint8_t*>(a.peers[a.rank]);
  const uint32_t seq = ep_seq(a.step_ctr, a.n_layers, a.layer);
  if (threadIdx.x == 0) s_ok = 1;
  __syncthreads();
  if (threadIdx.x < a.N) {
    const uint32_t* f = reinterpret_cast<const uint32_t*>(mine + off_flag) + threadIdx.x;
    if (!wait_flag(f, seq, a.timeout_ns, a.status, 2)) s_ok = 0;
  }
  __syncthreads();
  const float* recv = reinterpret_cast<const float*>(mine + off_recv);
  float* xr = x + (int64_t)t * a.H;
  float ss = 0.f;
  for (int i = threadIdx.x; i < a.H; i += blockDim.x) {
    float acc = 0.f;
    if (s_ok)
      for (int r = 0; r < a.N; ++r) acc += recv[((int64_t)r * a.cap + t) * a.H + i];
    const float v = xr[i] + acc;
    xr[i] = v;
    ss += v * v;
  }
  if (wn == nullptr) return;
  ss = block_sum(ss, red);
  const float rr = rsqrtf(ss / (float)a.H + eps);
  for (int i = threadIdx.x; i < a.H; i += blockDim.x) hout[(int64_t)t * a.H + i] = f2bf(xr[i] * rr * wn[i]);
}

cudaError_t launch_tp_reduce_norm(const EpArgs& a, int64_t off_recv, int64_t off_flag, float* x, const float* wn,
                                  void* hout, float eps, int T, cudaStream_t s) {
  if (T == 0) return cudaSuccess;
  tp_reduce_norm_kernel<<<T, 256, 0, s>>>(a, off_recv, off_flag, x, wn, reinterpret_cast<__nv_bfloat16*>(hout), eps);
  return cudaGetLastError();
}

cudaError_t launch_ep_dispatch(const EpArgs& a, const void* h, const int32_t* ids, const float* w, int T,
                               cudaStream_t s) {
  if (T > 256) return cudaErrorInvalidValue;
  ep_dispatch_kernel<<<a.N, 256, 0, s>>>(a, reinterpret_cast<const __nv_bfloat16*>(h), ids, w, T);
  return cudaGetLastError();
}

cudaError_t launch_ep_build(const EpArgs& a, int32_t* tok_off, int32_t* tok_idx, float* pair_w, int64_t* pair_dst,
                            cudaStream_t s) {
  if (a.E_loc > 512 || a.N > 64) return cudaErrorInvalidValue;
  ep_build_kernel<<<1, 1024, 0, s>>>(a, tok_off, tok_idx, pair_w, pair_dst);
  return cudaGetLastError();
}

cudaError_t launch_ep_combine(const EpArgs& a, float* x, const float* wn, void* hout, float eps, int T,
                              cudaStream_t s) {
  if (T == 0) return cudaSuccess;
  ep_combine_kernel<<<T, 256, 0, s>>>(a, x, wn, reinterpret_cast<__nv_bfloat16*>(hout), eps);
  return cudaGetLastError();
}

}  // namespace syn
