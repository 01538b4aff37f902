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

// 1 CTA x 1024 threads on the owner rank.  Every source's routing metadata is staged in
// shared memory once (coalesced loads after the bounded flag waits); then one warp per local
// expert scans the (source, slot, choice) entries in order with ballots: a first pass counts
// the expert's pairs, warp 0 scans the counts into the CSR offsets, a second pass writes each
// pair at its ordered position.  The order, and so the output, is deterministic.
__global__ void __launch_bounds__(1024) ep_build_kernel(EpArgs a, int32_t* __restrict__ tok_off,
                                                        int32_t* __restrict__ tok_idx, float* __restrict__ pair_w,
                                                        int64_t* __restrict__ pair_dst) {
  extern __shared__ int32_t s_meta[];  // [N * cap][MS]
  __shared__ int s_cnt[512];
  __shared__ int s_base[512];
  __shared__ int s_src_cnt[64];
  uint8_t* mine = reinterpret_cast<uint8_t*>(a.peers[a.rank]);
  const uint32_t seq = ep_seq(a.step_ctr, a.n_layers, a.layer);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, n_warps = blockDim.x >> 5;
  if (tid < a.N) {
    const uint32_t* f = reinterpret_cast<const uint32_t*>(mine + a.off_flag_disp) + tid;
    const bool ok = wait_flag(f, seq, a.timeout_ns, a.status, 0);
    const int c = ok ? __ldcg(reinterpret_cast<const int32_t*>(mine + a.off_cnt) + tid) : 0;
    s_src_cnt[tid] = c < 0 ? 0 : (c > a.cap ? a.cap : c);
  }
  __syncthreads();
  const int MS = 1 + 3 * a.k;
  const int rows = a.N * a.cap;
  const int32_t* meta = reinterpret_cast<const int32_t*>(mine + a.off_meta);
  for (int i = tid; i < rows * MS; i += blockDim.x) {
    const int row = i / MS;
    const bool valid = (row % a.cap) < s_src_cnt[row / a.cap];
    s_meta[i] = valid ? __ldcg(meta + i) : -1;  // an invalid slot routes to no expert
  }
  __syncthreads();
  const int n_ent = rows * a.k;
  for (int e = warp; e < a.E_loc; e += n_warps) {
    int c = 0;
    for (int b = 0; b < n_ent; b += 32) {
      const int idx = b + lane;
      const int el = idx < n_ent ? s_meta[(idx / a.k) * MS + 1 + 3 * (idx % a.k)] : -1;
      c += __popc(__ballot_sync(0xffffffffu, el == e));
    }
    if (lane == 0) s_cnt[e] = c;
  }
  __syncthreads();
  if (warp == 0) {
    int carry = 0;
    for (int e0 = 0; e0 < a.E_loc; e0 += 32) {
      const int e = e0 + lane;
      const int c = e < a.E_loc ? s_cnt[e] : 0;
      int v = c;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, v, o);
        if (lane >= o) v += y;
      }
      if (e < a.E_loc) {
        s_base[e] = carry + v - c;
        tok_off[e] = carry + v - c;
      }
      carry += __shfl_sync(0xffffffffu, v, 31);
    }
    if (lane == 0) tok_off[a.E_loc] = carry;
  }
  __syncthreads();
  for (int e = warp; e < a.E_loc; e += n_warps) {
    int p = s_base[e];
    for (int b = 0; b < n_ent; b += 32) {
      const int idx = b + lane;
      const int row = idx / a.k, j = idx % a.k;
      const int el = idx < n_ent ? s_meta[row * MS + 1 + 3 * j] : -1;
      const unsigned m = __ballot_sync(0xffffffffu, el == e);
      if (el == e) {
        const int q = p + __popc(m & ((1u << lane) - 1u));
        const int32_t* mrow = s_meta + row * MS;
        tok_idx[q] = row;  // = source * cap + slot: the received row
        pair_w[q] = __int_as_float(mrow[2 + 3 * j]);
        pair_dst[q] = a.peers[row / a.cap] + a.off_comb + (int64_t)mrow[3 + 3 * j] * a.H * 4;
      }
      p += __popc(m);
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

// Bounded wait of one CTA: thread q waits for rank q's flag at off_flag in this rank's region.
__global__ void flags_wait_kernel(const int64_t* __restrict__ peers, int n, int rank, int64_t off_flag,
                                  const uint32_t* step_ctr, int n_layers, int layer, uint64_t timeout_ns, int* status) {
  if ((int)threadIdx.x >= n) return;
  const uint8_t* mine = reinterpret_cast<const uint8_t*>(peers[rank]);
  const uint32_t seq = ep_seq(step_ctr, n_layers, layer);
  wait_flag(reinterpret_cast<const uint32_t*>(mine + off_flag) + threadIdx.x, seq, timeout_ns, status, 2);
}

cudaError_t launch_flags_wait(const int64_t* peers, int n, int rank, int64_t off_flag, const uint32_t* step_ctr,
                              int n_layers, int layer, uint64_t timeout_ns, int* status, cudaStream_t s) {
  if (n <= 0 || n > 1024) return cudaErrorInvalidValue;
  flags_wait_kernel<<<1, ((n + 31) / 32) * 32, 0, s>>>(peers, n, rank, off_flag, step_ctr, n_layers, layer, timeout_ns,
                                                       status);
  return cudaGetLastError();
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
  const size_t smem = (size_t)a.N * a.cap * (1 + 3 * a.k) * sizeof(int32_t);
  if (smem > 200 * 1024) return cudaErrorInvalidValue;
  if (smem > 48 * 1024) {
    const cudaError_t e = cudaFuncSetAttribute(ep_build_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
  }
  ep_build_kernel<<<1, 1024, smem, s>>>(a, tok_off, tok_idx, pair_w, pair_dst);
  return cudaGetLastError();
}

cudaError_t launch_ep_combine(const EpArgs& a, float* x, const float* wn, void* hout, float eps, int T,
                              cudaStream_t s) {
  if (T == 0) return cudaSuccess;
  ep_combine_kernel<<<T, 256, 0, s>>>(a, x, wn, reinterpret_cast<__nv_bfloat16*>(hout), eps);
  return cudaGetLastError();
}

}  // namespace syn
