// Raw-pointer launchers for every CUDA kernel.  The .cu files include no torch header
// (fast builds); csrc/torch_ops*.cpp validate tensors and call these.  Every launcher
// returns the cudaError_t of its launch.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace syn {

// ---- q4 format ----
cudaError_t launch_q4_quantize(const void* w, bool is_bf16, int64_t N, int64_t K, uint32_t* qw, void* sm,
                               cudaStream_t s);
cudaError_t launch_q4_rows_to_tiled(const uint8_t* rows, int64_t N, int64_t K, uint32_t* qw, void* sm,
                                    cudaStream_t s);
cudaError_t launch_q4_tiled_to_rows(const uint32_t* qw, const void* sm, int64_t N, int64_t K, uint8_t* rows,
                                    cudaStream_t s);
cudaError_t launch_q4t_dequant(const uint32_t* qw, const void* sm, int64_t N, int64_t K, void* out_bf16,
                               cudaStream_t s);

// ---- decode GEMV over 4-bit tiled weights ----
struct GemvArgs {
  const void* x;               // bf16 [rows, ldx]
  const int64_t* qw_ptrs;      // [E] device pointers
  const int64_t* sm_ptrs;      // [E] device pointers
  const int32_t* tok_off;      // [E+1]
  const int32_t* tok_idx;      // [P] or nullptr (identity)
  const float* route_w;        // [P] (mode 2)
  const void* res;             // bf16 [P, N] (mode 3)
  void* out;
  int N, K, ldx;
  int mode;
  int E;
  // mode 4 (GEMV_SCALED_F32_PTR): row p goes to (float*)out_ptrs[p]
  const int64_t* out_ptrs;
  // completion signal (optional): the last CTA stores seq into every peer's flag array
  unsigned* done_ctr;
  const int64_t* sig_peers;   // [sig_n] symmetric-region bases
  int64_t sig_off;            // byte offset of the flag array in the region
  int sig_n, sig_rank;
  const uint32_t* step_ctr;
  int n_layers, layer;
  // mode 6 (GEMV_PEERS_F32): every output row p goes to slot [sig_rank][p] of each peer's
  // receive area at byte offset peer_off (rows of N floats, peer_cap rows per source)
  int64_t peer_off;
  int peer_cap;
  // launch shape hints: max rows (tokens) per expert -> n-tiles of 8; experts likely active
  int nt_hint;
  int E_active_hint;
  // optional precomputed block sums of x: f32 [rows][K/32] (nullptr: computed per CTA)
  const float* xsum;
  int variant;  // 0 auto; 2 force v2 (register pipeline); 3 force v3 (cp.async ring); 4 TMA-fed
  int* status;  // error bits of bounded waits (v4), may be null
  int weights_in_vram;  // 1: every weight pointer is device memory (bulk-copy path allowed)
  // fp8 path: activations quantised to e4m3 [rows][ldx] with f32 scales [rows][K/128]
  const uint8_t* xq;
  const float* xs;
  // fp8 dense split-K: f32 partials [ksplit][ws_rows][N] (null: no split)
  float* ws_part;
  int ws_rows;
  size_t ws_floats;
};
// ---- fp8 (e4m3, 128x128 weight blocks, 1x128 activation blocks) ----
// Tiled weight layout: per (16-row tile, 64-column group) 1024 bytes, lane-major in
// mma.sync m16n8k32 A-fragment order (see fp8.cu); scales f32 [ceil(N/128)][K/128].
cudaError_t launch_f8_quant_act(const void* x, int rows, int K, int ldx, uint8_t* xq, float* xs, cudaStream_t s);
cudaError_t launch_f8_rows_to_tiled(const uint8_t* q, int N, int K, uint8_t* tiled, cudaStream_t s);
cudaError_t launch_f8_tiled_to_rows(const uint8_t* tiled, int N, int K, uint8_t* q, cudaStream_t s);
// tiled e4m3 + block scales -> bf16 row-major [N, K]
cudaError_t launch_f8_dequant_tiled(const uint8_t* tiled, const float* scale, int N, int K, void* out_bf16,
                                    cudaStream_t s);
// qw_ptrs: tiled e4m3 per expert; sm_ptrs: f32 scales per expert; a.xq / a.xs: quantised x
cudaError_t launch_f8_gemv(const GemvArgs& a, cudaStream_t s);
cudaError_t launch_block_sums(const void* x, int rows, int K, int ldx, float* out, cudaStream_t s);

// ---- prefill GEMM on tcgen05 (4-bit weights, grouped) ----
cudaError_t launch_tc_gemm_q4(const void* x, int ldx, const int64_t* qw_ptrs, const int64_t* sm_ptrs,
                              const int32_t* row_off, int G, int M, int N, int K, int mode, const float* route_w,
                              void* out, int* status, int max_mtiles, const void* bank_qw, const void* bank_sm,
                              int bank_experts, int group_base, cudaStream_t s, const void* bank2_qw = nullptr,
                              const void* bank2_sm = nullptr, int bank2_experts = 0, const int32_t* grp_sel = nullptr);

// ---- expert parallelism over NVLink peer memory ----
struct EpArgs {
  const int64_t* peers;  // device array [N] of symmetric-region bases (own included)
  int N, rank, cap, H, k, E_loc;
  int64_t off_x, off_meta, off_cnt, off_flag_disp, off_comb, off_flag_comb;
  const uint32_t* step_ctr;
  int n_layers, layer;
  uint64_t timeout_ns;
  int* status;
};
cudaError_t launch_ep_step_begin(uint32_t* step_ctr, cudaStream_t s);
cudaError_t launch_ep_dispatch(const EpArgs& a, const void* h, const int32_t* ids, const float* w, int T,
                               cudaStream_t s);
cudaError_t launch_ep_build(const EpArgs& a, int32_t* tok_off, int32_t* tok_idx, float* pair_w, int64_t* pair_dst,
                            cudaStream_t s);
// Ordered two-shot all-reduce of f32 partials in symmetric regions (tensor-parallel prefill):
// rank-order reduce-scatter by peer loads, all-gather by peer stores, then x += sum (+ RMSNorm).
struct TwoShotArgs {
  const int64_t* peers;  // device array [N] of symmetric-region bases (own included)
  int N, rank, H;
  int64_t n_elems;       // T * H
  int64_t off_part, off_gather, off_flag_ready, off_flag_done;
  uint32_t seq;          // monotone per use; flags compare against it
  uint64_t timeout_ns;
  int* status;
  unsigned* done_ctr;    // CTA arrivals of the reduce-scatter (left zero)
};
cudaError_t launch_tp_twoshot(const TwoShotArgs& a, float* x, const float* wn, void* hout, float eps, int T,
                              cudaStream_t s);
cudaError_t launch_tp_reduce_norm(const EpArgs& a, int64_t off_recv, int64_t off_flag, float* x, const float* wn,
                                  void* hout, float eps, int T, cudaStream_t s);
cudaError_t launch_ep_combine(const EpArgs& a, float* x, const float* wn, void* hout, float eps, int T,
                              cudaStream_t s);
cudaError_t launch_q4_gemv(const GemvArgs& a, cudaStream_t s);
// Split plan of the dense decode GEMV (see q4_gemv.cu); false if the shape is unsupported.
bool q4_gemv_dense_plan(int N, int K, int rows, int* nt, int* kr, size_t* ws_floats);
bool q4_gemv6_plan(int N, int K, int rows, int* nt, int* ksplit, size_t* ws_floats);
// Streaming dense GEMV (v6): K % 256 == 0; counters: N/128 + 1 zeroed ints.
cudaError_t launch_q4_gemv_dense6(const GemvArgs& a, float* ws, unsigned* counters, size_t ws_floats,
                                  cudaStream_t s);
// ---- causal prefill attention over the paged cache (head_dim 128) ----
cudaError_t launch_attn_prefill(const void* q, const void* kc, const void* vc, const int32_t* block_tables,
                                const int32_t* cu_q, const int32_t* kv_lens, void* out, int nseq, int max_q_len,
                                int Hq, int Hkv, int D, int max_blocks, float scale, cudaStream_t s);
// tcgen05 variant (TMA-fed, S and P V on the tensor cores, softmax warps between); Tq: rows
// of q, n_blocks: pages of the cache; *status bit 4: a pipeline wait timed out.
cudaError_t launch_attn_prefill_tc(const void* q, int Tq, const void* kc, const void* vc, int n_blocks,
                                   const int32_t* block_tables, const int32_t* cu_q, const int32_t* kv_lens, void* out,
                                   int nseq, int max_q_len, int Hq, int Hkv, int D, int max_blocks, float scale,
                                   int* status, cudaStream_t s);
// ---- MLA decode attention (absorbed; latent 512 + rope 64) over the paged latent cache ----
cudaError_t launch_mla_decode(const void* q, const void* cache, const int32_t* block_tables, const int32_t* ctx_lens,
                              float* part_o, float* part_ml, float* out, int B, int H, int max_blocks,
                              int pages_per_split, int n_splits, float scale, cudaStream_t s);
// ---- MLA decode projections around the latent attention (C 512, nope 128, rope 64, v 128) ----
cudaError_t launch_mla_q_absorb(const void* q, int T, int H, const void* w_uk, const float* cos_t, const float* sin_t,
                                const int32_t* pos, void* qcat, cudaStream_t s);
cudaError_t launch_mla_kv_write(const void* kva, int T, const float* norm_w, float eps, const float* cos_t,
                                const float* sin_t, const int32_t* pos, const int64_t* slot, void* cache,
                                cudaStream_t s);
cudaError_t launch_mla_o_absorb(const float* o_lat, int T, int H, const void* w_uv, void* out, cudaStream_t s);
// ---- runtime kernels: doorbells (bounded wait), timestamps, parity taps, KV page pack ----
cudaError_t launch_doorbell_wait(const uint32_t* flag, uint32_t want, uint64_t timeout_ns, int* status,
                                 uint64_t* waited_ns, cudaStream_t s);
cudaError_t launch_doorbell_ring(uint32_t* flag, uint32_t value, cudaStream_t s);
cudaError_t launch_timestamp(uint64_t* out, int slot, cudaStream_t s);
cudaError_t launch_tap_gather(const void* src, bool src_bf16, const int32_t* idx, int n, int H, float* dst,
                              cudaStream_t s);
cudaError_t launch_tap_compare(const float* a, const float* b, int n, int H, float* out, cudaStream_t s);
cudaError_t launch_kv_pages(void* kc, void* vc, const int32_t* pages, int n, int64_t page_bytes, void* packed,
                            bool pack, cudaStream_t s);
// ---- router-predicted expert prefetch (decode) ----
cudaError_t launch_expert_prefetch(const int32_t* pred, const int32_t* host_row, int e0, int El,
                                   const void* const* host, void* const* stage, const int64_t* row_bytes,
                                   int64_t* const* live, const int64_t* const* home, int n_parts, int ctas,
                                   cudaStream_t s);
cudaError_t launch_q4_gemv_dense(const GemvArgs& a, float* ws, unsigned* counters, size_t ws_floats,
                                 cudaStream_t s);

// ---- norms, RoPE, KV writes, embedding ----
cudaError_t launch_rmsnorm(const void* x, bool x_bf16, const float* w, void* y, int T, int H, float eps,
                           cudaStream_t s);
cudaError_t launch_moe_combine_rmsnorm(float* x, const float* yp, const int32_t* pair_of, int top_k,
                                       const float* shared, const float* w, void* y, int T, int H, float eps,
                                       cudaStream_t s);
cudaError_t launch_qk_rope_kv_write(const void* qkv, int T, int Hq, int Hkv, int D, const float* qn, const float* kn,
                                    float eps, const int32_t* pos, const float* cos_t, const float* sin_t,
                                    const int64_t* slot, void* q_out, void* k_cache, void* v_cache, int block_size,
                                    cudaStream_t s);
cudaError_t launch_embed(const void* table, const int32_t* ids, float* out, int T, int H, cudaStream_t s);

// ---- paged decode attention ----
cudaError_t launch_attn_decode(const void* q, const void* kc, const void* vc, const int32_t* block_tables,
                               const int32_t* ctx_lens, float* part_o, float* part_ml, void* out, int T, int Hq,
                               int Hkv, int D, int max_blocks, int pages_per_split, int n_splits, float scale,
                               cudaStream_t s);

// ---- MoE routing ----
cudaError_t launch_router_logits(const void* h, const void* W, float* logits, int T, int H, int E_rows,
                                 cudaStream_t s);
struct TopkArgs {
  const float* logits;   // [T, E_rows]
  const float* bias;     // [E] selection bias (sigmoid routing) or null
  int T, E, E_rows, k;
  int scoring;           // 0 softmax, 1 sigmoid
  int n_groups, topk_groups;
  int norm;              // renormalise the k weights
  float scaling;
  int pred;              // also top-k of logits[:, E:2E] (next-layer prediction)
  int32_t* topk_ids;     // [T, k]
  float* topk_w;         // [T, k]
  int32_t* tok_off;      // [E+1]
  int32_t* tok_idx;      // [T*k] token of each pair (pairs sorted by expert, then token)
  float* pair_w;         // [T*k]
  int32_t* pair_of;      // [T, k] pair index of each choice, choices sorted by expert
  int32_t* pred_mask;    // [E] 1 if any token is predicted to use expert e at the next layer
  uint32_t* ws;          // zeroed workspace of TOPK_WS_WORDS words, left zeroed on exit
  int32_t* counts;       // [E] or null: += the number of pairs routed to each expert (usage statistics)
  const int64_t* count_rows;  // [T] or null: only rows t with count_rows[t] >= 0 are counted (padding rows are not)
};
constexpr int TOPK_WS_WORDS = 512 * 8 + 16 + 1;
cudaError_t launch_moe_topk(const TopkArgs& a, cudaStream_t s);
// Any T (no next-layer prediction); ws: zeroed E * ceil(T/32) + E words (not restored).
cudaError_t launch_moe_route_large(const TopkArgs& a, cudaStream_t s);

// ---- CPU expert hand-off (mailbox layout: syn/cpu_mailbox.h) ----
struct CpuHandoffArgs {
  const void* h;          // [B, H] bf16 rows of this layer (device)
  int B, H, E, k, max_rows, layer;
  const int32_t* tok_off; // [E+1] routing CSR (device)
  const int32_t* tok_idx; // [B*k]
  const float* pair_w;    // [B*k]
  uint8_t* mb;            // host-mapped mailbox
  uint32_t* ctr;          // device [2]: last sequence number, CTA arrivals (zero between launches)
};
struct CpuCollectArgs {
  const uint8_t* mb;
  int H, E, k, max_rows;
  const uint32_t* ctr;    // the sequence number the hand-off raised
  float* yp;              // [B*k, H] pair outputs of the grouped GEMVs (device)
  uint64_t timeout_ns;
  int* status;            // bit 0: the CPU did not answer in time; bit 1: the CPU reported bad input
  // expert parallelism: pair p's row goes to the address pair_dst[p] (a source rank's combine
  // slot, possibly in a peer's memory) instead of yp; then, when sig_n > 0, the completion
  // flags of this layer are release-stored into every rank's region (flag array at sig_off,
  // slot sig_rank, value step * n_layers + layer + 1), as the down-projection GEMV does
  const int64_t* pair_dst;
  const int64_t* sig_peers;
  int64_t sig_off;
  int sig_n, sig_rank, n_layers, layer;
  const uint32_t* step_ctr;
  unsigned* done_ctr;     // CTA arrival counter (zero between launches)
};
cudaError_t launch_cpu_handoff(const CpuHandoffArgs& a, cudaStream_t s);
cudaError_t launch_cpu_collect(const CpuCollectArgs& a, cudaStream_t s);

// ---- sampling ----
cudaError_t launch_argmax(const float* logits, int T, int V, int32_t* out, cudaStream_t s);
cudaError_t launch_sample(const float* logits, int T, int V, const float* temperature, const int32_t* top_k,
                          const float* top_p, const int64_t* seed, const int64_t* stream, int64_t* counter,
                          int32_t* out, cudaStream_t s);
struct VerifyArgs {
  const float* logits;       // [S * (g+1), V]
  const int32_t* draft;      // [S, g]
  int S, g, V;
  const float* temperature;  // [S]
  const int32_t* top_k;      // [S]
  const float* top_p;        // [S]
  const int64_t* seed;
  const int64_t* stream;
  int64_t* counter;          // [S], advanced by the number of draws taken
  int32_t* out_tokens;       // [S, g+1]
  int32_t* n_accept;         // [S]
  const float* draft_probs;  // [S, g, V] distributions the drafts were sampled from, or null (point masses)
};
cudaError_t launch_verify_accept(const VerifyArgs& a, cudaStream_t s);

// ---- bf16 GEMM on tcgen05 (csrc/cuda/gemm_bf16_tc.cu) ----
// Peer push of a tensor-parallel partial: row t, column n of the f32 product goes to
// peers[d] + off_recv + (rank * src_stride + t' * ldo + n) * 4 (src_stride defaults to
// cap * ldo: one receive slot per source; the column width of a vocab slice turns it into a
// gather of column slices) for every rank d (owner_rows == 0,
// t' = t: one-shot all-reduce) or for d = t / owner_rows (t' = t % owner_rows: reduce-scatter);
// the grid's last CTA then release-stores step * n_layers + layer + 1 into each peer's flag
// slot `rank` at off_flag.
struct PeerPush {
  const int64_t* peers;
  int n_peers, rank, cap, owner_rows;
  int64_t src_stride;  // elements between two source ranks' areas (0: cap * ldo, the receive slots)
  int64_t off_recv, off_flag;
  unsigned* done_ctr;
  const uint32_t* step_ctr;
  int n_layers, layer;
};
// out = x [T, K] (row stride ldx) @ w [N, K]^T, bf16 operands; mode 0 bf16 store, 1 SwiGLU of
// interleaved 8-row gate/up chunks (bf16 [T, N/2]), 3 f32 +=, 5 f32 store, 6 peer push (pp).
// T < 128 runs the decode orientation (split-K partials in ws, per-row-tile counters).
cudaError_t launch_tc_gemm_bf16(const void* x, int T, int ldx, const void* w, int N, int K, int mode, void* out,
                                int ldo, float* ws, size_t ws_floats, unsigned* counters, const PeerPush* pp,
                                int* status, cudaStream_t s);
int bf16_gemm_splits(int N, int K, int T);
// 4-bit tiled weights (syn/q4.h), 1..64 token rows, decode orientation on tcgen05 (weights as the
// M operand); N % 128 == 0, K % 64 == 0; modes as launch_tc_gemm_bf16.
cudaError_t launch_tc_gemm_q4_dec(const void* x, int T, int ldx, const void* qw, const void* sm, int N, int K,
                                  int mode, void* out, int ldo, const PeerPush* pp, int* status, cudaStream_t s);
int q4_dec_splits(int N, int K);
// Bounded wait (grid of one CTA) until every rank's flag slot at off_flag holds this layer's
// sequence number; a timeout sets bit 2 of status.
cudaError_t launch_flags_wait(const int64_t* peers, int n, int rank, int64_t off_flag, const uint32_t* step_ctr,
                              int n_layers, int layer, uint64_t timeout_ns, int* status, cudaStream_t s);
size_t bf16_gemm_ws_floats(int N, int K, int T);
cudaError_t launch_philox(uint64_t seed, uint64_t stream, uint64_t counter0, int n, uint32_t* out, cudaStream_t s);

}  // namespace syn
