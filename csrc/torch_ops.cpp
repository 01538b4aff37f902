// Tensor-level wrappers: validate shapes, dtypes and devices, then call the raw-pointer
// launchers of syn/launch.h on the current CUDA stream.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "ops.h"
#include "syn/launch.h"

#define SYN_CHECK_CUDA(expr)                                                              \
  do {                                                                                    \
    cudaError_t _e = (expr);                                                              \
    TORCH_CHECK(_e == cudaSuccess, "CUDA error ", cudaGetErrorString(_e), " at ", __FILE__, \
                ":", __LINE__);                                                           \
  } while (0)

#define SYN_CHECK_INPUT(x)                                   \
  TORCH_CHECK((x).is_cuda(), #x " must be a CUDA tensor");   \
  TORCH_CHECK((x).is_contiguous(), #x " must be contiguous")

namespace syn {

static inline cudaStream_t cur_stream() { return at::cuda::getCurrentCUDAStream(); }

std::vector<torch::Tensor> q4_quantize(torch::Tensor w) {
  SYN_CHECK_INPUT(w);
  TORCH_CHECK(w.dim() == 2, "q4_quantize expects [N, K]");
  const int64_t N = w.size(0), K = w.size(1);
  TORCH_CHECK(N % 16 == 0 && K % 64 == 0, "q4 tiled layout needs N%16==0 and K%64==0");
  TORCH_CHECK(w.scalar_type() == torch::kFloat32 || w.scalar_type() == torch::kBFloat16,
              "q4_quantize: float32 or bfloat16");
  const at::cuda::CUDAGuard guard(w.device());
  auto qw = torch::empty({N * K / 8}, w.options().dtype(torch::kInt32));
  auto sm = torch::empty({N * K / 16}, w.options().dtype(torch::kFloat16));
  SYN_CHECK_CUDA(launch_q4_quantize(w.data_ptr(), w.scalar_type() == torch::kBFloat16, N, K,
                                    reinterpret_cast<uint32_t*>(qw.data_ptr()), sm.data_ptr(), cur_stream()));
  return {qw, sm};
}

std::vector<torch::Tensor> q4_rows_to_tiled(torch::Tensor rows, int64_t N, int64_t K) {
  SYN_CHECK_INPUT(rows);
  TORCH_CHECK(N % 16 == 0 && K % 64 == 0, "q4 tiled layout needs N%16==0 and K%64==0");
  TORCH_CHECK(rows.numel() == N * K / 32 * 20, "q4 rows: wrong byte count");
  const at::cuda::CUDAGuard guard(rows.device());
  auto qw = torch::empty({N * K / 8}, rows.options().dtype(torch::kInt32));
  auto sm = torch::empty({N * K / 16}, rows.options().dtype(torch::kFloat16));
  SYN_CHECK_CUDA(launch_q4_rows_to_tiled(rows.data_ptr<uint8_t>(), N, K, reinterpret_cast<uint32_t*>(qw.data_ptr()),
                                         sm.data_ptr(), cur_stream()));
  return {qw, sm};
}

torch::Tensor q4_tiled_to_rows(torch::Tensor qw, torch::Tensor sm, int64_t N, int64_t K) {
  SYN_CHECK_INPUT(qw);
  SYN_CHECK_INPUT(sm);
  TORCH_CHECK(qw.numel() * 8 == N * K && sm.numel() * 16 == N * K, "q4_tiled_to_rows: sizes");
  const at::cuda::CUDAGuard guard(qw.device());
  auto rows = torch::empty({N * K / 32 * 20}, qw.options().dtype(torch::kUInt8));
  SYN_CHECK_CUDA(launch_q4_tiled_to_rows(reinterpret_cast<const uint32_t*>(qw.data_ptr()), sm.data_ptr(), N, K,
                                         rows.data_ptr<uint8_t>(), cur_stream()));
  return rows;
}

torch::Tensor q4t_dequant(torch::Tensor qw, torch::Tensor sm, int64_t N, int64_t K) {
  SYN_CHECK_INPUT(qw);
  SYN_CHECK_INPUT(sm);
  TORCH_CHECK(qw.numel() * 8 == N * K && sm.numel() * 16 == N * K, "q4t_dequant: sizes");
  const at::cuda::CUDAGuard guard(qw.device());
  auto out = torch::empty({N, K}, qw.options().dtype(torch::kBFloat16));
  SYN_CHECK_CUDA(launch_q4t_dequant(reinterpret_cast<const uint32_t*>(qw.data_ptr()), sm.data_ptr(), N, K,
                                    out.data_ptr(), cur_stream()));
  return out;
}

void q4_gemv(torch::Tensor x, torch::Tensor qw_ptrs, torch::Tensor sm_ptrs, torch::Tensor tok_off,
             torch::Tensor tok_idx, torch::Tensor route_w, torch::Tensor res, torch::Tensor out, int64_t N,
             int64_t K, int64_t mode, int64_t nt_hint, int64_t e_active, torch::Tensor xsum, bool in_vram) {
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == torch::kBFloat16, "x must be cuda bf16");
  TORCH_CHECK(x.dim() == 2 && x.stride(1) == 1, "x must be [rows, K] with unit inner stride");
  TORCH_CHECK(N % 16 == 0 && K % 64 == 0, "q4_gemv: N%16, K%64");
  TORCH_CHECK(x.size(1) == K, "q4_gemv: x width != K");
  TORCH_CHECK((reinterpret_cast<uintptr_t>(x.data_ptr()) & 3) == 0 && x.stride(0) % 2 == 0,
              "q4_gemv: x rows must be 4-byte aligned");
  TORCH_CHECK(qw_ptrs.is_cuda() && sm_ptrs.is_cuda() && tok_off.is_cuda(), "index arrays must be on the device");
  TORCH_CHECK(qw_ptrs.scalar_type() == torch::kInt64 && sm_ptrs.scalar_type() == torch::kInt64, "ptr arrays int64");
  TORCH_CHECK(tok_off.scalar_type() == torch::kInt32, "tok_off int32");
  const int E = (int)qw_ptrs.numel();
  TORCH_CHECK(sm_ptrs.numel() == E && tok_off.numel() == E + 1, "tok_off must have E+1 entries");
  TORCH_CHECK(out.is_cuda() && out.is_contiguous(), "out must be contiguous cuda");
  GemvArgs a;
  a.x = x.data_ptr();
  a.qw_ptrs = qw_ptrs.data_ptr<int64_t>();
  a.sm_ptrs = sm_ptrs.data_ptr<int64_t>();
  a.tok_off = tok_off.data_ptr<int32_t>();
  a.tok_idx = tok_idx.numel() ? tok_idx.data_ptr<int32_t>() : nullptr;
  a.route_w = route_w.numel() ? route_w.data_ptr<float>() : nullptr;
  a.res = res.numel() ? res.data_ptr() : nullptr;
  a.out = out.data_ptr();
  a.N = (int)N;
  a.K = (int)K;
  a.ldx = (int)x.stride(0);
  a.mode = (int)mode;
  a.E = E;
  a.out_ptrs = nullptr;
  a.done_ctr = nullptr;
  a.sig_peers = nullptr;
  a.sig_off = 0;
  a.sig_n = 0;
  a.sig_rank = 0;
  a.step_ctr = nullptr;
  a.n_layers = 0;
  a.layer = 0;
  a.nt_hint = (int)nt_hint;
  a.E_active_hint = (int)std::max<int64_t>(1, e_active);
  a.xsum = nullptr;
  a.variant = 0;
  a.peer_off = 0;
  a.peer_cap = 0;
  a.status = nullptr;
  a.weights_in_vram = in_vram ? 1 : 0;
  if (xsum.defined() && xsum.numel() > 0) {
    TORCH_CHECK(xsum.is_cuda() && xsum.scalar_type() == torch::kFloat32 && xsum.size(-1) == K / 32, "xsum f32 [rows, K/32]");
    a.xsum = xsum.data_ptr<float>();
  }
  if (mode == 0) TORCH_CHECK(out.scalar_type() == torch::kBFloat16 && out.size(-1) == N, "out bf16 [P, N]");
  if (mode == 3 || mode == 5) TORCH_CHECK(out.scalar_type() == torch::kFloat32 && out.size(-1) == N, "out f32 [P, N]");
  if (mode == 1) TORCH_CHECK(out.scalar_type() == torch::kBFloat16 && out.size(-1) == N / 2, "out bf16 [P, N/2]");
  if (mode == 2) TORCH_CHECK(a.route_w && out.scalar_type() == torch::kFloat32 && out.size(-1) == N, "mode 2: route_w, fp32 [P, N]");
  TORCH_CHECK(mode >= 0 && mode <= 5 && mode != 4, "q4_gemv: bad mode (mode 4 goes through q4_gemv_ep)");
  const at::cuda::CUDAGuard guard(x.device());
  SYN_CHECK_CUDA(launch_q4_gemv(a, cur_stream()));
}


static inline const float* fptr_or_null(const torch::Tensor& t) {
  if (!t.defined() || t.numel() == 0) return nullptr;
  TORCH_CHECK(t.is_cuda() && t.scalar_type() == torch::kFloat32 && t.is_contiguous(), "expected contiguous cuda f32");
  return t.data_ptr<float>();
}

void rmsnorm(torch::Tensor x, torch::Tensor w, double eps, torch::Tensor out) {
  SYN_CHECK_INPUT(x);
  SYN_CHECK_INPUT(out);
  TORCH_CHECK(x.dim() == 2 && out.sizes() == x.sizes() && out.scalar_type() == torch::kBFloat16, "rmsnorm shapes");
  TORCH_CHECK(x.scalar_type() == torch::kFloat32 || x.scalar_type() == torch::kBFloat16, "rmsnorm x dtype");
  TORCH_CHECK(w.numel() == x.size(1), "rmsnorm weight size");
  const at::cuda::CUDAGuard guard(x.device());
  SYN_CHECK_CUDA(launch_rmsnorm(x.data_ptr(), x.scalar_type() == torch::kBFloat16, fptr_or_null(w), out.data_ptr(),
                                (int)x.size(0), (int)x.size(1), (float)eps, cur_stream()));
}

void moe_combine_rmsnorm(torch::Tensor x, torch::Tensor yp, torch::Tensor pair_of, torch::Tensor shared,
                         torch::Tensor w, torch::Tensor out, double eps) {
  SYN_CHECK_INPUT(x);
  SYN_CHECK_INPUT(yp);
  SYN_CHECK_INPUT(pair_of);
  TORCH_CHECK(x.scalar_type() == torch::kFloat32 && yp.scalar_type() == torch::kFloat32, "f32 x, yp");
  TORCH_CHECK(pair_of.scalar_type() == torch::kInt32 && pair_of.dim() == 2 && pair_of.size(0) == x.size(0), "pair_of");
  TORCH_CHECK(yp.size(-1) == x.size(1), "yp width");
  const float* wp = fptr_or_null(w);
  if (wp) TORCH_CHECK(out.is_cuda() && out.scalar_type() == torch::kBFloat16 && out.sizes() == x.sizes(), "out");
  const at::cuda::CUDAGuard guard(x.device());
  SYN_CHECK_CUDA(launch_moe_combine_rmsnorm(x.data_ptr<float>(), yp.data_ptr<float>(), pair_of.data_ptr<int32_t>(),
                                            (int)pair_of.size(1), fptr_or_null(shared), wp,
                                            wp ? out.data_ptr() : nullptr, (int)x.size(0), (int)x.size(1),
                                            (float)eps, cur_stream()));
}

void qk_rope_kv_write(torch::Tensor qkv, int64_t Hq, int64_t Hkv, int64_t D, torch::Tensor qn, torch::Tensor kn,
                      double eps, torch::Tensor pos, torch::Tensor cos_t, torch::Tensor sin_t, torch::Tensor slot,
                      torch::Tensor q_out, torch::Tensor k_cache, torch::Tensor v_cache) {
  SYN_CHECK_INPUT(qkv);
  SYN_CHECK_INPUT(pos);
  SYN_CHECK_INPUT(slot);
  SYN_CHECK_INPUT(q_out);
  SYN_CHECK_INPUT(k_cache);
  SYN_CHECK_INPUT(v_cache);
  TORCH_CHECK(qkv.scalar_type() == torch::kBFloat16 && qkv.size(-1) == (Hq + 2 * Hkv) * D, "qkv shape");
  const int64_t T = qkv.size(0);
  TORCH_CHECK(pos.numel() == T && pos.scalar_type() == torch::kInt32, "pos");
  TORCH_CHECK(slot.numel() == T && slot.scalar_type() == torch::kInt64, "slot");
  TORCH_CHECK(q_out.numel() == T * Hq * D && q_out.scalar_type() == torch::kBFloat16, "q_out");
  TORCH_CHECK(k_cache.dim() == 4 && k_cache.size(1) == Hkv && k_cache.size(3) == D, "k_cache [nb, Hkv, bs, D]");
  TORCH_CHECK(cos_t.size(-1) == D / 2 && sin_t.size(-1) == D / 2, "rope table");
  const at::cuda::CUDAGuard guard(qkv.device());
  SYN_CHECK_CUDA(launch_qk_rope_kv_write(qkv.data_ptr(), (int)T, (int)Hq, (int)Hkv, (int)D, fptr_or_null(qn),
                                         fptr_or_null(kn), (float)eps, pos.data_ptr<int32_t>(),
                                         cos_t.data_ptr<float>(), sin_t.data_ptr<float>(), slot.data_ptr<int64_t>(),
                                         q_out.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(),
                                         (int)k_cache.size(2), cur_stream()));
}

void embed(torch::Tensor table, torch::Tensor ids, torch::Tensor out) {
  SYN_CHECK_INPUT(table);
  SYN_CHECK_INPUT(ids);
  SYN_CHECK_INPUT(out);
  TORCH_CHECK(table.scalar_type() == torch::kBFloat16 && ids.scalar_type() == torch::kInt32 &&
                  out.scalar_type() == torch::kFloat32, "embed dtypes");
  const at::cuda::CUDAGuard guard(table.device());
  SYN_CHECK_CUDA(launch_embed(table.data_ptr(), ids.data_ptr<int32_t>(), out.data_ptr<float>(), (int)ids.numel(),
                              (int)table.size(1), cur_stream()));
}

void attn_decode(torch::Tensor q, torch::Tensor kc, torch::Tensor vc, torch::Tensor block_tables,
                 torch::Tensor ctx_lens, torch::Tensor part_o, torch::Tensor part_ml, torch::Tensor out,
                 int64_t pages_per_split, double scale) {
  SYN_CHECK_INPUT(q);
  SYN_CHECK_INPUT(kc);
  SYN_CHECK_INPUT(vc);
  SYN_CHECK_INPUT(block_tables);
  SYN_CHECK_INPUT(ctx_lens);
  SYN_CHECK_INPUT(part_o);
  SYN_CHECK_INPUT(part_ml);
  SYN_CHECK_INPUT(out);
  TORCH_CHECK(q.dim() == 3 && q.scalar_type() == torch::kBFloat16, "q [T, Hq, D] bf16");
  TORCH_CHECK(kc.dim() == 4 && kc.size(2) == 16 && kc.scalar_type() == torch::kBFloat16, "cache [nb, Hkv, 16, D] bf16");
  const int64_t T = q.size(0), Hq = q.size(1), D = q.size(2), Hkv = kc.size(1);
  TORCH_CHECK(block_tables.dim() == 2 && block_tables.size(0) >= T && block_tables.scalar_type() == torch::kInt32, "block_tables");
  const int64_t max_blocks = block_tables.size(1);
  const int64_t n_splits = (max_blocks + pages_per_split - 1) / pages_per_split;
  TORCH_CHECK(part_o.numel() >= T * Hkv * n_splits * 16 * D, "part_o too small");
  TORCH_CHECK(part_ml.numel() >= T * Hkv * n_splits * 16 * 2, "part_ml too small");
  TORCH_CHECK(out.numel() == T * Hq * D && out.scalar_type() == torch::kBFloat16, "out");
  const at::cuda::CUDAGuard guard(q.device());
  SYN_CHECK_CUDA(launch_attn_decode(q.data_ptr(), kc.data_ptr(), vc.data_ptr(), block_tables.data_ptr<int32_t>(),
                                    ctx_lens.data_ptr<int32_t>(), part_o.data_ptr<float>(), part_ml.data_ptr<float>(),
                                    out.data_ptr(), (int)T, (int)Hq, (int)Hkv, (int)D, (int)max_blocks,
                                    (int)pages_per_split, (int)n_splits, (float)scale, cur_stream()));
}

void router_logits(torch::Tensor h, torch::Tensor W, torch::Tensor logits) {
  SYN_CHECK_INPUT(h);
  SYN_CHECK_INPUT(W);
  SYN_CHECK_INPUT(logits);
  TORCH_CHECK(h.scalar_type() == torch::kBFloat16 && W.scalar_type() == torch::kBFloat16, "bf16 h, W");
  TORCH_CHECK(logits.scalar_type() == torch::kFloat32 && logits.size(0) == h.size(0) && logits.size(1) == W.size(0), "logits");
  const at::cuda::CUDAGuard guard(h.device());
  SYN_CHECK_CUDA(launch_router_logits(h.data_ptr(), W.data_ptr(), logits.data_ptr<float>(), (int)h.size(0),
                                      (int)h.size(1), (int)W.size(0), cur_stream()));
}

void moe_topk(torch::Tensor logits, torch::Tensor bias, int64_t E, int64_t k, int64_t scoring, int64_t n_groups,
              int64_t topk_groups, bool norm, double scaling, bool pred, torch::Tensor topk_ids, torch::Tensor topk_w,
              torch::Tensor tok_off, torch::Tensor tok_idx, torch::Tensor pair_w, torch::Tensor pair_of,
              torch::Tensor pred_mask, torch::Tensor ws, torch::Tensor counts, torch::Tensor count_rows) {
  SYN_CHECK_INPUT(logits);
  TORCH_CHECK(logits.scalar_type() == torch::kFloat32, "logits f32");
  const bool large = logits.size(0) > 256;
  const int64_t need = large ? E * ((logits.size(0) + 31) / 32) + E : TOPK_WS_WORDS;
  TORCH_CHECK(ws.is_cuda() && ws.scalar_type() == torch::kInt32 && ws.numel() >= need,
              "moe_topk workspace: zeroed int32 of at least ", need, " words");
  TORCH_CHECK(!(large && pred), "moe_topk: next-layer prediction needs at most 256 tokens");
  const int64_t T = logits.size(0);
  TORCH_CHECK(logits.size(1) == (pred ? 2 * E : E), "logits width");
  TORCH_CHECK(topk_ids.numel() >= T * k && topk_w.numel() >= T * k && tok_idx.numel() >= T * k &&
                  pair_w.numel() >= T * k && pair_of.numel() >= T * k && tok_off.numel() >= E + 1, "topk outputs");
  TopkArgs a;
  a.logits = logits.data_ptr<float>();
  a.bias = fptr_or_null(bias);
  a.T = (int)T;
  a.E = (int)E;
  a.E_rows = (int)logits.size(1);
  a.k = (int)k;
  a.scoring = (int)scoring;
  a.n_groups = (int)n_groups;
  a.topk_groups = (int)topk_groups;
  a.norm = norm ? 1 : 0;
  a.scaling = (float)scaling;
  a.pred = pred ? 1 : 0;
  a.topk_ids = topk_ids.data_ptr<int32_t>();
  a.topk_w = topk_w.data_ptr<float>();
  a.tok_off = tok_off.data_ptr<int32_t>();
  a.tok_idx = tok_idx.data_ptr<int32_t>();
  a.pair_w = pair_w.data_ptr<float>();
  a.pair_of = pair_of.data_ptr<int32_t>();
  a.pred_mask = pred_mask.numel() ? pred_mask.data_ptr<int32_t>() : nullptr;
  a.ws = reinterpret_cast<uint32_t*>(ws.data_ptr<int32_t>());
  TORCH_CHECK(!counts.numel() || (counts.is_cuda() && counts.scalar_type() == torch::kInt32 && counts.numel() >= E &&
                                  counts.is_contiguous()), "moe_topk counts: int32 [E] on the device");
  a.counts = counts.numel() ? counts.data_ptr<int32_t>() : nullptr;
  TORCH_CHECK(!count_rows.numel() || (count_rows.is_cuda() && count_rows.scalar_type() == torch::kInt64 &&
                                      count_rows.numel() >= T), "moe_topk count_rows: int64 [T] on the device (step slots)");
  a.count_rows = count_rows.numel() ? count_rows.data_ptr<int64_t>() : nullptr;
  TORCH_CHECK(!(large && a.count_rows), "moe_topk: count_rows is for decode batches (at most 256 rows)");
  const at::cuda::CUDAGuard guard(logits.device());
  if (large) {
    SYN_CHECK_CUDA(launch_moe_route_large(a, cur_stream()));
  } else {
    SYN_CHECK_CUDA(launch_moe_topk(a, cur_stream()));
  }
}

void argmax(torch::Tensor logits, torch::Tensor out) {
  SYN_CHECK_INPUT(logits);
  TORCH_CHECK(logits.scalar_type() == torch::kFloat32 && logits.dim() == 2, "logits f32 [T, V]");
  TORCH_CHECK(out.scalar_type() == torch::kInt32 && out.numel() >= logits.size(0), "out int32");
  const at::cuda::CUDAGuard guard(logits.device());
  SYN_CHECK_CUDA(launch_argmax(logits.data_ptr<float>(), (int)logits.size(0), (int)logits.size(1),
                               out.data_ptr<int32_t>(), cur_stream()));
}

void sample(torch::Tensor logits, torch::Tensor temperature, torch::Tensor top_k, torch::Tensor top_p,
            torch::Tensor seed, torch::Tensor stream, torch::Tensor counter, torch::Tensor out) {
  SYN_CHECK_INPUT(logits);
  TORCH_CHECK(logits.scalar_type() == torch::kFloat32 && logits.dim() == 2, "logits f32 [T, V]");
  const int64_t T = logits.size(0);
  TORCH_CHECK(temperature.numel() >= T && top_k.numel() >= T && top_p.numel() >= T && seed.numel() >= T &&
                  stream.numel() >= T && counter.numel() >= T && out.numel() >= T, "sample params");
  TORCH_CHECK(seed.scalar_type() == torch::kInt64 && stream.scalar_type() == torch::kInt64 &&
                  counter.scalar_type() == torch::kInt64, "seed/stream/counter int64");
  const at::cuda::CUDAGuard guard(logits.device());
  SYN_CHECK_CUDA(launch_sample(logits.data_ptr<float>(), (int)T, (int)logits.size(1), temperature.data_ptr<float>(),
                               top_k.data_ptr<int32_t>(), top_p.data_ptr<float>(), seed.data_ptr<int64_t>(),
                               stream.data_ptr<int64_t>(), counter.data_ptr<int64_t>(), out.data_ptr<int32_t>(),
                               cur_stream()));
}

torch::Tensor philox(int64_t seed, int64_t stream, int64_t counter0, int64_t n, torch::Tensor like) {
  const at::cuda::CUDAGuard guard(like.device());
  auto out = torch::empty({n}, like.options().dtype(torch::kInt32));
  SYN_CHECK_CUDA(launch_philox((uint64_t)seed, (uint64_t)stream, (uint64_t)counter0, (int)n,
                               reinterpret_cast<uint32_t*>(out.data_ptr()), cur_stream()));
  return out;
}


static EpArgs make_ep_args(torch::Tensor peers, int64_t N, int64_t rank, int64_t cap, int64_t H, int64_t k,
                           int64_t E_loc, std::vector<int64_t> offs, torch::Tensor step_ctr, int64_t n_layers,
                           int64_t layer, int64_t timeout_ns, torch::Tensor status) {
  TORCH_CHECK(peers.is_cuda() && peers.scalar_type() == torch::kInt64 && peers.numel() == N, "peers: cuda int64 [N]");
  TORCH_CHECK(offs.size() == 6, "6 region offsets");
  TORCH_CHECK(step_ctr.is_cuda() && step_ctr.scalar_type() == torch::kInt32, "step_ctr cuda int32");
  TORCH_CHECK(status.is_cuda() && status.scalar_type() == torch::kInt32, "status cuda int32");
  EpArgs a;
  a.peers = peers.data_ptr<int64_t>();
  a.N = (int)N;
  a.rank = (int)rank;
  a.cap = (int)cap;
  a.H = (int)H;
  a.k = (int)k;
  a.E_loc = (int)E_loc;
  a.off_x = offs[0];
  a.off_meta = offs[1];
  a.off_cnt = offs[2];
  a.off_flag_disp = offs[3];
  a.off_comb = offs[4];
  a.off_flag_comb = offs[5];
  a.step_ctr = reinterpret_cast<const uint32_t*>(step_ctr.data_ptr());
  a.n_layers = (int)n_layers;
  a.layer = (int)layer;
  a.timeout_ns = (uint64_t)timeout_ns;
  a.status = status.data_ptr<int32_t>();
  return a;
}

void ep_step_begin(torch::Tensor step_ctr) {
  TORCH_CHECK(step_ctr.is_cuda() && step_ctr.scalar_type() == torch::kInt32, "step_ctr");
  const at::cuda::CUDAGuard guard(step_ctr.device());
  SYN_CHECK_CUDA(launch_ep_step_begin(reinterpret_cast<uint32_t*>(step_ctr.data_ptr()), cur_stream()));
}

void ep_dispatch(torch::Tensor peers, int64_t N, int64_t rank, int64_t cap, int64_t H, int64_t k, int64_t E_loc,
                 std::vector<int64_t> offs, torch::Tensor step_ctr, int64_t n_layers, int64_t layer,
                 int64_t timeout_ns, torch::Tensor status, torch::Tensor h, torch::Tensor ids, torch::Tensor w) {
  auto a = make_ep_args(peers, N, rank, cap, H, k, E_loc, offs, step_ctr, n_layers, layer, timeout_ns, status);
  TORCH_CHECK(h.is_cuda() && h.scalar_type() == torch::kBFloat16 && h.size(1) == H, "h bf16 [T, H]");
  TORCH_CHECK(h.size(0) <= cap, "ep_dispatch: more local rows than capacity");
  TORCH_CHECK(ids.scalar_type() == torch::kInt32 && w.scalar_type() == torch::kFloat32, "ids int32, w f32");
  const at::cuda::CUDAGuard guard(h.device());
  SYN_CHECK_CUDA(launch_ep_dispatch(a, h.data_ptr(), ids.data_ptr<int32_t>(), w.data_ptr<float>(), (int)h.size(0),
                                    cur_stream()));
}

void ep_build(torch::Tensor peers, int64_t N, int64_t rank, int64_t cap, int64_t H, int64_t k, int64_t E_loc,
              std::vector<int64_t> offs, torch::Tensor step_ctr, int64_t n_layers, int64_t layer, int64_t timeout_ns,
              torch::Tensor status, torch::Tensor tok_off, torch::Tensor tok_idx, torch::Tensor pair_w,
              torch::Tensor pair_dst) {
  auto a = make_ep_args(peers, N, rank, cap, H, k, E_loc, offs, step_ctr, n_layers, layer, timeout_ns, status);
  TORCH_CHECK(tok_off.numel() >= E_loc + 1 && tok_idx.numel() >= N * cap * k && pair_w.numel() >= N * cap * k &&
                  pair_dst.numel() >= N * cap * k, "ep_build outputs too small");
  const at::cuda::CUDAGuard guard(tok_off.device());
  SYN_CHECK_CUDA(launch_ep_build(a, tok_off.data_ptr<int32_t>(), tok_idx.data_ptr<int32_t>(), pair_w.data_ptr<float>(),
                                 pair_dst.data_ptr<int64_t>(), cur_stream()));
}

void ep_combine(torch::Tensor peers, int64_t N, int64_t rank, int64_t cap, int64_t H, int64_t k, int64_t E_loc,
                std::vector<int64_t> offs, torch::Tensor step_ctr, int64_t n_layers, int64_t layer,
                int64_t timeout_ns, torch::Tensor status, torch::Tensor x, torch::Tensor wn, torch::Tensor hout,
                double eps) {
  auto a = make_ep_args(peers, N, rank, cap, H, k, E_loc, offs, step_ctr, n_layers, layer, timeout_ns, status);
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == torch::kFloat32 && x.size(1) == H, "x f32 [T, H]");
  const float* wp = fptr_or_null(wn);
  if (wp) TORCH_CHECK(hout.scalar_type() == torch::kBFloat16 && hout.sizes() == x.sizes(), "hout");
  const at::cuda::CUDAGuard guard(x.device());
  SYN_CHECK_CUDA(launch_ep_combine(a, x.data_ptr<float>(), wp, wp ? hout.data_ptr() : nullptr, (float)eps,
                                   (int)x.size(0), cur_stream()));
}

// Grouped GEMV whose epilogue stores row p to out_ptrs[p] (peer memory allowed) and whose
// last CTA raises flag `sig_rank` in every peer's flag array at byte offset sig_off.
void q4_gemv_ep(torch::Tensor x, torch::Tensor qw_ptrs, torch::Tensor sm_ptrs, torch::Tensor tok_off,
                torch::Tensor tok_idx, torch::Tensor route_w, torch::Tensor out_ptrs, int64_t N, int64_t K,
                torch::Tensor done_ctr, torch::Tensor peers, int64_t sig_off, int64_t sig_rank,
                torch::Tensor step_ctr, int64_t n_layers, int64_t layer, int64_t nt_hint, int64_t e_active,
                bool in_vram) {
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == torch::kBFloat16 && x.dim() == 2 && x.stride(1) == 1, "x");
  TORCH_CHECK(N % 16 == 0 && K % 64 == 0 && x.size(1) == K, "q4_gemv_ep shapes");
  TORCH_CHECK(done_ctr.is_cuda() && done_ctr.scalar_type() == torch::kInt32, "done_ctr cuda int32");
  GemvArgs a;
  memset(&a, 0, sizeof(a));
  a.x = x.data_ptr();
  a.qw_ptrs = qw_ptrs.data_ptr<int64_t>();
  a.sm_ptrs = sm_ptrs.data_ptr<int64_t>();
  a.tok_off = tok_off.data_ptr<int32_t>();
  a.tok_idx = tok_idx.numel() ? tok_idx.data_ptr<int32_t>() : nullptr;
  a.route_w = route_w.data_ptr<float>();
  a.res = nullptr;
  a.out = nullptr;
  a.N = (int)N;
  a.K = (int)K;
  a.ldx = (int)x.stride(0);
  a.mode = 4;
  a.E = (int)qw_ptrs.numel();
  a.out_ptrs = out_ptrs.data_ptr<int64_t>();
  // an empty done_ctr: this launch raises no flags (a later kernel of the layer does)
  a.done_ctr = done_ctr.numel() ? reinterpret_cast<unsigned*>(done_ctr.data_ptr()) : nullptr;
  a.sig_peers = peers.data_ptr<int64_t>();
  a.sig_off = sig_off;
  a.sig_n = (int)peers.numel();
  a.sig_rank = (int)sig_rank;
  a.step_ctr = reinterpret_cast<const uint32_t*>(step_ctr.data_ptr());
  a.n_layers = (int)n_layers;
  a.layer = (int)layer;
  a.nt_hint = (int)nt_hint;
  a.E_active_hint = (int)std::max<int64_t>(1, e_active);
  a.xsum = nullptr;
  a.variant = 0;
  a.peer_off = 0;
  a.peer_cap = 0;
  a.status = nullptr;
  a.weights_in_vram = in_vram ? 1 : 0;
  TORCH_CHECK(tok_off.numel() == a.E + 1, "tok_off E+1");
  const at::cuda::CUDAGuard guard(x.device());
  SYN_CHECK_CUDA(launch_q4_gemv(a, cur_stream()));
}


// C = X W^T on tcgen05 with 4-bit weights, grouped over contiguous row ranges.
//   x: bf16 [M, K]; row_off: int32 [G+1] (device); qw/sm ptrs: int64 [G]
//   mode 0: out bf16 [M, N]; 1: SwiGLU out bf16 [M, N/2]; 2: out f32 [M, N] * route_w[m];
//   3: out f32 [M, N] += ; 5: out f32 [M, N]
void tc_gemm_q4(torch::Tensor x, torch::Tensor qw_ptrs, torch::Tensor sm_ptrs, torch::Tensor row_off, int64_t N,
                int64_t K, int64_t mode, torch::Tensor route_w, torch::Tensor out, torch::Tensor status,
                int64_t max_mtiles, torch::Tensor bank_qw, torch::Tensor bank_sm, int64_t group_base) {
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == torch::kBFloat16 && x.dim() == 2 && x.stride(1) == 1, "x bf16 [M, K]");
  TORCH_CHECK(x.size(1) == K && K % 64 == 0 && N % 128 == 0, "tc_gemm_q4 shapes (K%64, N%128)");
  TORCH_CHECK(row_off.is_cuda() && row_off.scalar_type() == torch::kInt32 && row_off.numel() == qw_ptrs.numel() + 1,
              "row_off int32 [G+1]");
  TORCH_CHECK(status.is_cuda() && status.scalar_type() == torch::kInt32, "status int32");
  const int64_t M = x.size(0);
  if (mode == 1) TORCH_CHECK(out.scalar_type() == torch::kBFloat16 && out.size(-1) == N / 2 && out.size(0) >= M, "out swiglu");
  if (mode == 0) TORCH_CHECK(out.scalar_type() == torch::kBFloat16 && out.size(-1) == N && out.size(0) >= M, "out bf16");
  if (mode == 2 || mode == 3 || mode == 5)
    TORCH_CHECK(out.scalar_type() == torch::kFloat32 && out.size(-1) == N && out.size(0) >= M, "out f32");
  if (mode == 2) TORCH_CHECK(route_w.numel() >= M, "route_w");
  TORCH_CHECK(out.is_contiguous(), "out contiguous");
  if (M == 0) return;
  const at::cuda::CUDAGuard guard(x.device());
  SYN_CHECK_CUDA(launch_tc_gemm_q4(x.data_ptr(), (int)x.stride(0), qw_ptrs.data_ptr<int64_t>(), sm_ptrs.data_ptr<int64_t>(),
                                   row_off.data_ptr<int32_t>(), (int)qw_ptrs.numel(), (int)M, (int)N, (int)K, (int)mode,
                                   mode == 2 ? route_w.data_ptr<float>() : nullptr, out.data_ptr(),
                                   status.data_ptr<int32_t>(), (int)max_mtiles,
                                   bank_qw.numel() ? bank_qw.data_ptr() : nullptr,
                                   bank_sm.numel() ? bank_sm.data_ptr() : nullptr,
                                   bank_qw.numel() ? (int)(bank_qw.dim() == 2 ? bank_qw.size(0) : 1) : 0,
                                   (int)group_base, cur_stream()));
}


// The grouped 4-bit GEMM over two contiguous banks: group g reads entry sel[g] >> 1 of bank
// sel[g] & 1 (bank 0: b0_qw / b0_sm [entries, N*K/8 u32 / N*K/16 f16], bank 1 likewise).
void tc_gemm_q4_banks(torch::Tensor x, torch::Tensor row_off, int64_t N, int64_t K, int64_t mode, torch::Tensor route_w,
                      torch::Tensor out, torch::Tensor status, int64_t max_mtiles, torch::Tensor b0_qw,
                      torch::Tensor b0_sm, torch::Tensor b1_qw, torch::Tensor b1_sm, torch::Tensor sel) {
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == torch::kBFloat16 && x.dim() == 2 && x.stride(1) == 1, "x bf16 [M, K]");
  TORCH_CHECK(x.size(1) == K && K % 64 == 0 && N % 128 == 0, "tc_gemm_q4_banks shapes (K%64, N%128)");
  TORCH_CHECK(row_off.is_cuda() && row_off.scalar_type() == torch::kInt32 && sel.is_cuda() &&
                  sel.scalar_type() == torch::kInt32 && sel.numel() + 1 == row_off.numel(),
              "row_off int32 [G+1], sel int32 [G]");
  const int64_t per_q = N * K / 8, per_s = N * K / 16;
  TORCH_CHECK(b0_qw.is_cuda() && b0_qw.dim() == 2 && b0_qw.size(1) == per_q && b0_sm.dim() == 2 &&
                  b0_sm.size(1) == per_s && b0_sm.size(0) == b0_qw.size(0) && b0_qw.is_contiguous() &&
                  b0_sm.is_contiguous(), "bank 0 [entries, words]");
  TORCH_CHECK(b1_qw.is_cuda() && b1_qw.dim() == 2 && b1_qw.size(1) == per_q && b1_sm.dim() == 2 &&
                  b1_sm.size(1) == per_s && b1_sm.size(0) == b1_qw.size(0) && b1_qw.is_contiguous() &&
                  b1_sm.is_contiguous(), "bank 1 [entries, words]");
  TORCH_CHECK(status.is_cuda() && status.scalar_type() == torch::kInt32, "status int32");
  const int64_t M = x.size(0);
  if (mode == 1) TORCH_CHECK(out.scalar_type() == torch::kBFloat16 && out.size(-1) == N / 2 && out.size(0) >= M, "out swiglu");
  if (mode == 0) TORCH_CHECK(out.scalar_type() == torch::kBFloat16 && out.size(-1) == N && out.size(0) >= M, "out bf16");
  if (mode == 2 || mode == 3 || mode == 5)
    TORCH_CHECK(out.scalar_type() == torch::kFloat32 && out.size(-1) == N && out.size(0) >= M, "out f32");
  if (mode == 2) TORCH_CHECK(route_w.numel() >= M, "route_w");
  TORCH_CHECK(out.is_contiguous(), "out contiguous");
  if (M == 0) return;
  const at::cuda::CUDAGuard guard(x.device());
  SYN_CHECK_CUDA(launch_tc_gemm_q4(x.data_ptr(), (int)x.stride(0), nullptr, nullptr, row_off.data_ptr<int32_t>(),
                                   (int)sel.numel(), (int)M, (int)N, (int)K, (int)mode,
                                   mode == 2 ? route_w.data_ptr<float>() : nullptr, out.data_ptr(),
                                   status.data_ptr<int32_t>(), (int)max_mtiles, b0_qw.data_ptr(), b0_sm.data_ptr(),
                                   (int)b0_qw.size(0), 0, cur_stream(), b1_qw.data_ptr(), b1_sm.data_ptr(),
                                   (int)b1_qw.size(0), sel.data_ptr<int32_t>()));
}

void block_sums(torch::Tensor x, torch::Tensor out) {
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == torch::kBFloat16 && x.dim() == 2 && x.stride(1) == 1, "x bf16 [rows, K]");
  TORCH_CHECK(x.size(1) % 32 == 0, "K % 32");
  TORCH_CHECK(out.is_cuda() && out.scalar_type() == torch::kFloat32 && out.is_contiguous() &&
                  out.numel() >= x.size(0) * (x.size(1) / 32), "out f32 [rows, K/32]");
  const at::cuda::CUDAGuard guard(x.device());
  SYN_CHECK_CUDA(launch_block_sums(x.data_ptr(), (int)x.size(0), (int)x.size(1), (int)x.stride(0),
                                   out.data_ptr<float>(), cur_stream()));
}


// TP row-parallel GEMV whose epilogue pushes the f32 partial rows into every peer's receive
// slot (one-shot all-reduce); the last CTA raises flag `rank` in every peer's flag array.
void q4_gemv_tp(torch::Tensor x, torch::Tensor qw_ptrs, torch::Tensor sm_ptrs, torch::Tensor tok_off, int64_t N,
                int64_t K, torch::Tensor done_ctr, torch::Tensor peers, int64_t peer_off, int64_t peer_cap,
                int64_t sig_off, int64_t rank, torch::Tensor step_ctr, int64_t n_layers, int64_t layer) {
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == torch::kBFloat16 && x.dim() == 2 && x.stride(1) == 1, "x");
  TORCH_CHECK(N % 16 == 0 && K % 64 == 0 && x.size(1) == K, "q4_gemv_tp shapes");
  TORCH_CHECK(x.size(0) <= peer_cap, "more rows than the receive capacity");
  GemvArgs a;
  memset(&a, 0, sizeof(a));
  a.x = x.data_ptr();
  a.qw_ptrs = qw_ptrs.data_ptr<int64_t>();
  a.sm_ptrs = sm_ptrs.data_ptr<int64_t>();
  a.tok_off = tok_off.data_ptr<int32_t>();
  a.N = (int)N;
  a.K = (int)K;
  a.ldx = (int)x.stride(0);
  a.mode = 6;
  a.E = (int)qw_ptrs.numel();
  // an empty done_ctr: this launch raises no flags (a later kernel of the layer does)
  a.done_ctr = done_ctr.numel() ? reinterpret_cast<unsigned*>(done_ctr.data_ptr()) : nullptr;
  a.sig_peers = peers.data_ptr<int64_t>();
  a.sig_off = sig_off;
  a.sig_n = (int)peers.numel();
  a.sig_rank = (int)rank;
  a.step_ctr = reinterpret_cast<const uint32_t*>(step_ctr.data_ptr());
  a.n_layers = (int)n_layers;
  a.layer = (int)layer;
  a.peer_off = peer_off;
  a.peer_cap = (int)peer_cap;
  a.nt_hint = (int)((x.size(0) + 7) / 8);
  a.E_active_hint = 1;
  a.weights_in_vram = 1;
  const at::cuda::CUDAGuard guard(x.device());
  SYN_CHECK_CUDA(launch_q4_gemv(a, cur_stream()));
}

void tp_reduce_norm(torch::Tensor peers, int64_t N, int64_t rank, int64_t cap, int64_t H, std::vector<int64_t> offs,
                    torch::Tensor step_ctr, int64_t n_layers, int64_t layer, int64_t timeout_ns, torch::Tensor status,
                    int64_t off_recv, int64_t off_flag, torch::Tensor x, torch::Tensor wn, torch::Tensor hout,
                    double eps) {
  auto a = make_ep_args(peers, N, rank, cap, H, 1, 1, offs, step_ctr, n_layers, layer, timeout_ns, status);
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == torch::kFloat32 && x.size(1) == H, "x f32 [T, H]");
  const float* wp = fptr_or_null(wn);
  const at::cuda::CUDAGuard guard(x.device());
  SYN_CHECK_CUDA(launch_tp_reduce_norm(a, off_recv, off_flag, x.data_ptr<float>(), wp, wp ? hout.data_ptr() : nullptr,
                                       (float)eps, (int)x.size(0), cur_stream()));
}


// Two-shot all-reduce of this rank's f32 partial (at off_part of its symmetric region, [T, H])
// into x [T, H] (+ RMSNorm into hout when wn is given).
void tp_twoshot(torch::Tensor peers, int64_t rank, int64_t off_part, int64_t off_gather, int64_t off_flag_ready,
                int64_t off_flag_done, int64_t seq, int64_t timeout_ns, torch::Tensor status, torch::Tensor done_ctr,
                torch::Tensor x, torch::Tensor wn, torch::Tensor hout, double eps) {
  TORCH_CHECK(peers.is_cuda() && peers.scalar_type() == torch::kInt64, "peers int64 (device)");
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == torch::kFloat32 && x.dim() == 2 && x.is_contiguous(), "x f32 [T, H]");
  TORCH_CHECK(status.is_cuda() && status.scalar_type() == torch::kInt32, "status int32 (device)");
  TORCH_CHECK(done_ctr.is_cuda() && done_ctr.scalar_type() == torch::kInt32 && done_ctr.numel() >= 1, "done_ctr int32");
  TwoShotArgs a;
  a.peers = peers.data_ptr<int64_t>();
  a.N = (int)peers.numel();
  a.rank = (int)rank;
  a.H = (int)x.size(1);
  a.n_elems = x.numel();
  a.off_part = off_part;
  a.off_gather = off_gather;
  a.off_flag_ready = off_flag_ready;
  a.off_flag_done = off_flag_done;
  a.seq = (uint32_t)seq;
  a.timeout_ns = (uint64_t)timeout_ns;
  a.status = status.data_ptr<int32_t>();
  a.done_ctr = reinterpret_cast<unsigned*>(done_ctr.data_ptr<int32_t>());
  const float* wp = fptr_or_null(wn);
  if (wp) TORCH_CHECK(hout.is_cuda() && hout.scalar_type() == torch::kBFloat16 && hout.numel() >= x.numel(), "hout bf16");
  const at::cuda::CUDAGuard guard(x.device());
  SYN_CHECK_CUDA(launch_tp_twoshot(a, x.data_ptr<float>(), wp, wp ? hout.data_ptr() : nullptr, (float)eps,
                                   (int)x.size(0), cur_stream()));
}

// Exact acceptance of point-mass drafts, or of drafts sampled from the distributions
// draft_probs [S, g, V] (f32; empty for point masses) (see csrc/cuda/sampler.cu).
void verify_accept(torch::Tensor logits, torch::Tensor draft, torch::Tensor temperature, torch::Tensor top_k,
                   torch::Tensor top_p, torch::Tensor seed, torch::Tensor stream, torch::Tensor counter,
                   torch::Tensor out_tokens, torch::Tensor n_accept, torch::Tensor draft_probs) {
  SYN_CHECK_INPUT(logits);
  SYN_CHECK_INPUT(draft);
  TORCH_CHECK(logits.scalar_type() == torch::kFloat32 && draft.scalar_type() == torch::kInt32 && draft.dim() == 2,
              "logits f32, draft int32 [S, g]");
  const int64_t S = draft.size(0), g = draft.size(1);
  TORCH_CHECK(logits.size(0) == S * (g + 1), "logits rows must be S*(g+1)");
  TORCH_CHECK(out_tokens.numel() >= S * (g + 1) && n_accept.numel() >= S, "outputs");
  VerifyArgs a{logits.data_ptr<float>(), draft.data_ptr<int32_t>(), (int)S, (int)g, (int)logits.size(1),
               temperature.data_ptr<float>(), top_k.data_ptr<int32_t>(), top_p.data_ptr<float>(),
               seed.data_ptr<int64_t>(), stream.data_ptr<int64_t>(), counter.data_ptr<int64_t>(),
               out_tokens.data_ptr<int32_t>(), n_accept.data_ptr<int32_t>(), nullptr};
  if (draft_probs.defined() && draft_probs.numel()) {
    SYN_CHECK_INPUT(draft_probs);
    TORCH_CHECK(draft_probs.scalar_type() == torch::kFloat32 && draft_probs.numel() == S * g * logits.size(1),
                "draft_probs f32 [S, g, V]");
    a.draft_probs = draft_probs.data_ptr<float>();
  }
  const at::cuda::CUDAGuard guard(logits.device());
  SYN_CHECK_CUDA(launch_verify_accept(a, cur_stream()));
}


// Dense decode GEMV for 9..64 rows (split-K, activations staged per CTA).
void q4_gemv_dense(torch::Tensor x, torch::Tensor qw_ptrs, torch::Tensor sm_ptrs, torch::Tensor tok_off,
                   torch::Tensor out, int64_t N, int64_t K, int64_t mode, torch::Tensor ws, torch::Tensor counters) {
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == torch::kBFloat16 && x.dim() == 2 && x.stride(1) == 1, "x");
  TORCH_CHECK(N % 64 == 0 && K % 128 == 0 && x.size(1) == K, "q4_gemv_dense shapes (N%64, K%128)");
  TORCH_CHECK(x.size(0) <= 64, "q4_gemv_dense: at most 64 rows");
  TORCH_CHECK((reinterpret_cast<uintptr_t>(x.data_ptr()) & 15) == 0 && (x.stride(0) * 2) % 16 == 0,
              "x rows must be 16-byte aligned");
  TORCH_CHECK(ws.is_cuda() && ws.scalar_type() == torch::kFloat32, "ws f32");
  TORCH_CHECK(counters.is_cuda() && counters.scalar_type() == torch::kInt32 && counters.numel() >= N / 64, "counters");
  GemvArgs a;
  memset(&a, 0, sizeof(a));
  a.x = x.data_ptr();
  a.qw_ptrs = qw_ptrs.data_ptr<int64_t>();
  a.sm_ptrs = sm_ptrs.data_ptr<int64_t>();
  a.tok_off = tok_off.data_ptr<int32_t>();
  a.out = out.data_ptr();
  a.N = (int)N;
  a.K = (int)K;
  a.ldx = (int)x.stride(0);
  a.mode = (int)mode;
  a.E = 1;
  a.nt_hint = (int)((x.size(0) + 7) / 8);
  if (mode == 0) TORCH_CHECK(out.scalar_type() == torch::kBFloat16 && out.size(-1) == N, "out bf16 [T, N]");
  if (mode == 1) TORCH_CHECK(out.scalar_type() == torch::kBFloat16 && out.size(-1) == N / 2, "out bf16 [T, N/2]");
  if (mode == 3 || mode == 5) TORCH_CHECK(out.scalar_type() == torch::kFloat32 && out.size(-1) == N, "out f32 [T, N]");
  TORCH_CHECK(mode == 0 || mode == 1 || mode == 3 || mode == 5, "q4_gemv_dense: mode");
  const at::cuda::CUDAGuard guard(x.device());
  SYN_CHECK_CUDA(launch_q4_gemv_dense(a, ws.data_ptr<float>(), reinterpret_cast<unsigned*>(counters.data_ptr()),
                                      (size_t)ws.numel(), cur_stream()));
}

int64_t q4_gemv_dense_ws(int64_t N, int64_t K, int64_t rows) {
  int nt, kr;
  size_t need;
  if (!q4_gemv_dense_plan((int)N, (int)K, (int)rows, &nt, &kr, &need)) return -1;
  return (int64_t)need;
}


void attn_prefill(torch::Tensor q, torch::Tensor kc, torch::Tensor vc, torch::Tensor block_tables, torch::Tensor cu_q,
                  torch::Tensor kv_lens, torch::Tensor out, int64_t max_q_len, double scale) {
  SYN_CHECK_INPUT(q);
  TORCH_CHECK(q.scalar_type() == torch::kBFloat16 && q.dim() == 3 && q.is_contiguous(), "q bf16 [T, Hq, D]");
  TORCH_CHECK(kc.scalar_type() == torch::kBFloat16 && kc.dim() == 4 && kc.size(2) == 16 && kc.is_contiguous(),
              "k cache bf16 [blocks, Hkv, 16, D]");
  TORCH_CHECK(vc.sizes() == kc.sizes() && vc.is_contiguous() && vc.scalar_type() == torch::kBFloat16, "v cache");
  TORCH_CHECK(out.sizes() == q.sizes() && out.scalar_type() == torch::kBFloat16 && out.is_contiguous(), "out");
  TORCH_CHECK(block_tables.scalar_type() == torch::kInt32 && block_tables.dim() == 2 && block_tables.is_contiguous(),
              "block tables int32 [nseq, max_blocks]");
  const int64_t nseq = block_tables.size(0);
  TORCH_CHECK(cu_q.scalar_type() == torch::kInt32 && cu_q.numel() == nseq + 1, "cu_q int32 [nseq + 1]");
  TORCH_CHECK(kv_lens.scalar_type() == torch::kInt32 && kv_lens.numel() == nseq, "kv_lens int32 [nseq]");
  TORCH_CHECK(q.size(2) == 128 && kc.size(3) == 128, "head_dim 128");
  TORCH_CHECK(q.size(1) % kc.size(1) == 0, "query heads must be a multiple of KV heads");
  if (nseq == 0 || q.size(0) == 0) return;
  const at::cuda::CUDAGuard guard(q.device());
  SYN_CHECK_CUDA(launch_attn_prefill(q.data_ptr(), kc.data_ptr(), vc.data_ptr(), block_tables.data_ptr<int32_t>(),
                                     cu_q.data_ptr<int32_t>(), kv_lens.data_ptr<int32_t>(), out.data_ptr(), (int)nseq,
                                     (int)max_q_len, (int)q.size(1), (int)kc.size(1), (int)q.size(2),
                                     (int)block_tables.size(1), (float)scale, cur_stream()));
}

// The same contract on tcgen05 (status: int32 error word, bit 4 = a pipeline wait timed out).
void attn_prefill_tc(torch::Tensor q, torch::Tensor kc, torch::Tensor vc, torch::Tensor block_tables,
                     torch::Tensor cu_q, torch::Tensor kv_lens, torch::Tensor out, int64_t max_q_len, double scale,
                     torch::Tensor status) {
  SYN_CHECK_INPUT(q);
  TORCH_CHECK(q.scalar_type() == torch::kBFloat16 && q.dim() == 3 && q.is_contiguous(), "q bf16 [T, Hq, D]");
  TORCH_CHECK(kc.scalar_type() == torch::kBFloat16 && kc.dim() == 4 && kc.size(2) == 16 && kc.is_contiguous(),
              "k cache bf16 [blocks, Hkv, 16, D]");
  TORCH_CHECK(vc.sizes() == kc.sizes() && vc.is_contiguous() && vc.scalar_type() == torch::kBFloat16, "v cache");
  TORCH_CHECK(out.sizes() == q.sizes() && out.scalar_type() == torch::kBFloat16 && out.is_contiguous(), "out");
  TORCH_CHECK(block_tables.scalar_type() == torch::kInt32 && block_tables.dim() == 2 && block_tables.is_contiguous(),
              "block tables int32 [nseq, max_blocks]");
  const int64_t nseq = block_tables.size(0);
  TORCH_CHECK(cu_q.scalar_type() == torch::kInt32 && cu_q.numel() == nseq + 1, "cu_q int32 [nseq + 1]");
  TORCH_CHECK(kv_lens.scalar_type() == torch::kInt32 && kv_lens.numel() == nseq, "kv_lens int32 [nseq]");
  TORCH_CHECK(q.size(2) == 128 && kc.size(3) == 128, "head_dim 128");
  TORCH_CHECK(q.size(1) % kc.size(1) == 0, "query heads must be a multiple of KV heads");
  TORCH_CHECK(status.is_cuda() && status.scalar_type() == torch::kInt32, "status int32");
  if (nseq == 0 || q.size(0) == 0) return;
  const at::cuda::CUDAGuard guard(q.device());
  SYN_CHECK_CUDA(launch_attn_prefill_tc(q.data_ptr(), (int)q.size(0), kc.data_ptr(), vc.data_ptr(), (int)kc.size(0),
                                        block_tables.data_ptr<int32_t>(), cu_q.data_ptr<int32_t>(),
                                        kv_lens.data_ptr<int32_t>(), out.data_ptr(), (int)nseq, (int)max_q_len,
                                        (int)q.size(1), (int)kc.size(1), (int)q.size(2), (int)block_tables.size(1),
                                        (float)scale, status.data_ptr<int32_t>(), cur_stream()));
}

std::vector<torch::Tensor> f8_quant_act(torch::Tensor x) {
  SYN_CHECK_INPUT(x);
  TORCH_CHECK(x.scalar_type() == torch::kBFloat16 && x.dim() == 2 && x.stride(1) == 1, "x bf16 [T, K]");
  const int64_t T = x.size(0), K = x.size(1);
  TORCH_CHECK(K % 128 == 0, "K % 128 == 0 (1x128 activation blocks), got K=", K);
  auto xq = torch::empty({T, K}, x.options().dtype(torch::kUInt8));
  auto xs = torch::empty({T, K / 128}, x.options().dtype(torch::kFloat32));
  const at::cuda::CUDAGuard guard(x.device());
  SYN_CHECK_CUDA(launch_f8_quant_act(x.data_ptr(), (int)T, (int)K, (int)x.stride(0), xq.data_ptr<uint8_t>(),
                                     xs.data_ptr<float>(), cur_stream()));
  return {xq, xs};
}

torch::Tensor f8_rows_to_tiled(torch::Tensor q, int64_t N, int64_t K) {
  SYN_CHECK_INPUT(q);
  TORCH_CHECK(q.scalar_type() == torch::kUInt8 && q.numel() == N * K, "e4m3 bytes [N, K]");
  TORCH_CHECK(N % 16 == 0 && K % 128 == 0, "fp8 tiled layout needs N % 16 == 0 and K % 128 == 0, got N=", N, " K=", K);
  auto out = torch::empty({N * K}, q.options());
  const at::cuda::CUDAGuard guard(q.device());
  SYN_CHECK_CUDA(launch_f8_rows_to_tiled(q.data_ptr<uint8_t>(), (int)N, (int)K, out.data_ptr<uint8_t>(), cur_stream()));
  return out;
}

torch::Tensor f8_tiled_to_rows(torch::Tensor tiled, int64_t N, int64_t K) {
  SYN_CHECK_INPUT(tiled);
  TORCH_CHECK(tiled.scalar_type() == torch::kUInt8 && tiled.numel() == N * K, "tiled e4m3 bytes");
  TORCH_CHECK(N % 16 == 0 && K % 128 == 0, "fp8 tiled layout needs N % 16 == 0 and K % 128 == 0, got N=", N, " K=", K);
  auto out = torch::empty({N, K}, tiled.options());
  const at::cuda::CUDAGuard guard(tiled.device());
  SYN_CHECK_CUDA(launch_f8_tiled_to_rows(tiled.data_ptr<uint8_t>(), (int)N, (int)K, out.data_ptr<uint8_t>(), cur_stream()));
  return out;
}

torch::Tensor f8_dequant_tiled(torch::Tensor tiled, torch::Tensor scale, int64_t N, int64_t K) {
  SYN_CHECK_INPUT(tiled);
  TORCH_CHECK(tiled.scalar_type() == torch::kUInt8 && tiled.numel() == N * K, "tiled e4m3 bytes");
  TORCH_CHECK(scale.is_cuda() && scale.scalar_type() == torch::kFloat32 && scale.is_contiguous() &&
                  scale.numel() == ((N + 127) / 128) * ((K + 127) / 128), "scale f32 [ceil(N/128), ceil(K/128)]");
  TORCH_CHECK(N % 16 == 0 && K % 128 == 0, "fp8 tiled layout needs N % 16 == 0 and K % 128 == 0");
  auto out = torch::empty({N, K}, tiled.options().dtype(torch::kBFloat16));
  const at::cuda::CUDAGuard guard(tiled.device());
  SYN_CHECK_CUDA(launch_f8_dequant_tiled(tiled.data_ptr<uint8_t>(), scale.data_ptr<float>(), (int)N, (int)K,
                                         out.data_ptr(), cur_stream()));
  return out;
}

void f8_gemv(torch::Tensor xq, torch::Tensor xs, torch::Tensor qw_ptrs, torch::Tensor sm_ptrs, torch::Tensor tok_off,
             torch::Tensor tok_idx, torch::Tensor route_w, torch::Tensor out, int64_t N, int64_t K, int64_t mode,
             int64_t nt_hint, torch::Tensor ws) {
  SYN_CHECK_INPUT(xq);
  TORCH_CHECK(xq.scalar_type() == torch::kUInt8 && xq.dim() == 2 && xq.size(1) == K && xq.stride(1) == 1, "xq");
  TORCH_CHECK(xs.scalar_type() == torch::kFloat32 && xs.dim() == 2 && xs.size(1) == K / 128 && xs.is_contiguous(),
              "xs f32 [rows, K/128]");
  TORCH_CHECK(qw_ptrs.scalar_type() == torch::kInt64 && sm_ptrs.scalar_type() == torch::kInt64 &&
                  qw_ptrs.numel() == sm_ptrs.numel() && tok_off.numel() == qw_ptrs.numel() + 1,
              "pointer tables / CSR");
  TORCH_CHECK(mode == 0 || mode == 1 || mode == 2 || mode == 3 || mode == 5, "f8_gemv: mode ", mode);
  GemvArgs a;
  memset(&a, 0, sizeof(a));
  a.xq = xq.data_ptr<uint8_t>();
  a.xs = xs.data_ptr<float>();
  a.ldx = (int)xq.stride(0);
  a.qw_ptrs = qw_ptrs.data_ptr<int64_t>();
  a.sm_ptrs = sm_ptrs.data_ptr<int64_t>();
  a.tok_off = tok_off.data_ptr<int32_t>();
  a.tok_idx = tok_idx.numel() ? tok_idx.data_ptr<int32_t>() : nullptr;
  a.route_w = route_w.numel() ? route_w.data_ptr<float>() : nullptr;
  TORCH_CHECK(mode != 2 || a.route_w, "mode 2 needs route_w");
  a.out = out.data_ptr();
  a.N = (int)N;
  a.K = (int)K;
  a.mode = (int)mode;
  a.E = (int)qw_ptrs.numel();
  a.nt_hint = (int)nt_hint;
  if (ws.numel() && a.E == 1) {  // dense: split-K allowed into this f32 workspace
    TORCH_CHECK(ws.is_cuda() && ws.scalar_type() == torch::kFloat32, "ws f32");
    a.ws_part = ws.data_ptr<float>();
    a.ws_rows = (int)xq.size(0);
    a.ws_floats = (size_t)ws.numel();
  }
  const at::cuda::CUDAGuard guard(xq.device());
  SYN_CHECK_CUDA(launch_f8_gemv(a, cur_stream()));
}

// Expert-parallel down projection over fp8 experts: xq/xs are the quantised SwiGLU rows of
// every pair (contiguous, pair order), row p goes scaled by route_w[p] to the address
// out_ptrs[p] (a source rank's combine slot, local or peer), and the last CTA raises this
// layer's flags on every peer unless done_ctr is empty.
void f8_gemv_ep(torch::Tensor xq, torch::Tensor xs, torch::Tensor qw_ptrs, torch::Tensor sm_ptrs,
                torch::Tensor tok_off, torch::Tensor route_w, torch::Tensor out_ptrs, int64_t N, int64_t K,
                torch::Tensor done_ctr, torch::Tensor peers, int64_t sig_off, int64_t sig_rank, torch::Tensor step_ctr,
                int64_t n_layers, int64_t layer, int64_t nt_hint) {
  SYN_CHECK_INPUT(xq);
  TORCH_CHECK(xq.scalar_type() == torch::kUInt8 && xq.dim() == 2 && xq.size(1) == K && xq.stride(1) == 1, "xq");
  TORCH_CHECK(xs.scalar_type() == torch::kFloat32 && xs.dim() == 2 && xs.size(1) == K / 128 && xs.is_contiguous(),
              "xs f32 [rows, K/128]");
  TORCH_CHECK(qw_ptrs.scalar_type() == torch::kInt64 && sm_ptrs.scalar_type() == torch::kInt64 &&
                  qw_ptrs.numel() == sm_ptrs.numel() && tok_off.numel() == qw_ptrs.numel() + 1,
              "pointer tables / CSR");
  TORCH_CHECK(out_ptrs.scalar_type() == torch::kInt64 && route_w.scalar_type() == torch::kFloat32, "out_ptrs / route_w");
  TORCH_CHECK(done_ctr.is_cuda() && done_ctr.scalar_type() == torch::kInt32, "done_ctr cuda int32");
  GemvArgs a;
  memset(&a, 0, sizeof(a));
  a.xq = xq.data_ptr<uint8_t>();
  a.xs = xs.data_ptr<float>();
  a.ldx = (int)xq.stride(0);
  a.qw_ptrs = qw_ptrs.data_ptr<int64_t>();
  a.sm_ptrs = sm_ptrs.data_ptr<int64_t>();
  a.tok_off = tok_off.data_ptr<int32_t>();
  a.route_w = route_w.data_ptr<float>();
  a.out_ptrs = out_ptrs.data_ptr<int64_t>();
  a.N = (int)N;
  a.K = (int)K;
  a.mode = 4;
  a.E = (int)qw_ptrs.numel();
  a.nt_hint = (int)nt_hint;
  a.done_ctr = done_ctr.numel() ? reinterpret_cast<unsigned*>(done_ctr.data_ptr()) : nullptr;
  a.sig_peers = peers.data_ptr<int64_t>();
  a.sig_off = sig_off;
  a.sig_n = (int)peers.numel();
  a.sig_rank = (int)sig_rank;
  a.step_ctr = reinterpret_cast<const uint32_t*>(step_ctr.data_ptr());
  a.n_layers = (int)n_layers;
  a.layer = (int)layer;
  const at::cuda::CUDAGuard guard(xq.device());
  SYN_CHECK_CUDA(launch_f8_gemv(a, cur_stream()));
}

// MLA decode projections: q bf16 [T, H*(128+64)] -> qcat bf16 [T, H, 576]; kva bf16 [T, 576] ->
// cache rows (normed latent | roped k_pe); o_lat f32 [T, H, 512] -> out bf16 [T, H*128].
void mla_q_absorb(torch::Tensor q, torch::Tensor w_uk, torch::Tensor cos_t, torch::Tensor sin_t, torch::Tensor pos,
                  torch::Tensor qcat) {
  SYN_CHECK_INPUT(q);
  const int64_t T = qcat.size(0), H = qcat.size(1);
  TORCH_CHECK(q.scalar_type() == torch::kBFloat16 && q.is_contiguous() && q.numel() == T * H * 192, "q bf16 [T, H*192]");
  TORCH_CHECK(w_uk.scalar_type() == torch::kBFloat16 && w_uk.is_contiguous() && w_uk.numel() == H * 128 * 512,
              "w_uk bf16 [H, 128, 512]");
  TORCH_CHECK(qcat.scalar_type() == torch::kBFloat16 && qcat.is_contiguous() && qcat.dim() == 3 && qcat.size(2) == 576,
              "qcat bf16 [T, H, 576]");
  TORCH_CHECK(cos_t.scalar_type() == torch::kFloat32 && sin_t.scalar_type() == torch::kFloat32 && cos_t.size(-1) == 32,
              "rope tables f32 [max_pos, 32]");
  TORCH_CHECK(pos.scalar_type() == torch::kInt32 && pos.numel() >= T, "pos int32 [T]");
  if (T == 0) return;
  const at::cuda::CUDAGuard guard(q.device());
  SYN_CHECK_CUDA(launch_mla_q_absorb(q.data_ptr(), (int)T, (int)H, w_uk.data_ptr(), cos_t.data_ptr<float>(),
                                     sin_t.data_ptr<float>(), pos.data_ptr<int32_t>(), qcat.data_ptr(), cur_stream()));
}

void mla_kv_write(torch::Tensor kva, torch::Tensor norm_w, double eps, torch::Tensor cos_t, torch::Tensor sin_t,
                  torch::Tensor pos, torch::Tensor slot, torch::Tensor cache) {
  SYN_CHECK_INPUT(kva);
  TORCH_CHECK(kva.scalar_type() == torch::kBFloat16 && kva.is_contiguous() && kva.dim() == 2 && kva.size(1) == 576,
              "kva bf16 [T, 576]");
  TORCH_CHECK(norm_w.scalar_type() == torch::kFloat32 && norm_w.numel() == 512, "norm weight f32 [512]");
  TORCH_CHECK(cache.scalar_type() == torch::kBFloat16 && cache.is_contiguous() && cache.size(-1) == 576,
              "latent cache bf16 [.., 576]");
  const int64_t T = kva.size(0);
  TORCH_CHECK(pos.scalar_type() == torch::kInt32 && slot.scalar_type() == torch::kInt64 && pos.numel() >= T &&
                  slot.numel() >= T, "pos int32 / slot int64 [T]");
  if (T == 0) return;
  const at::cuda::CUDAGuard guard(kva.device());
  SYN_CHECK_CUDA(launch_mla_kv_write(kva.data_ptr(), (int)T, norm_w.data_ptr<float>(), (float)eps,
                                     cos_t.data_ptr<float>(), sin_t.data_ptr<float>(), pos.data_ptr<int32_t>(),
                                     slot.data_ptr<int64_t>(), cache.data_ptr(), cur_stream()));
}

void mla_o_absorb(torch::Tensor o_lat, torch::Tensor w_uv, torch::Tensor out) {
  SYN_CHECK_INPUT(o_lat);
  TORCH_CHECK(o_lat.scalar_type() == torch::kFloat32 && o_lat.is_contiguous() && o_lat.dim() == 3 &&
                  o_lat.size(2) == 512, "o_lat f32 [T, H, 512]");
  const int64_t T = o_lat.size(0), H = o_lat.size(1);
  TORCH_CHECK(w_uv.scalar_type() == torch::kBFloat16 && w_uv.is_contiguous() && w_uv.numel() == H * 128 * 512,
              "w_uv bf16 [H, 128, 512]");
  TORCH_CHECK(out.scalar_type() == torch::kBFloat16 && out.is_contiguous() && out.numel() == T * H * 128,
              "out bf16 [T, H*128]");
  if (T == 0) return;
  const at::cuda::CUDAGuard guard(o_lat.device());
  SYN_CHECK_CUDA(launch_mla_o_absorb(o_lat.data_ptr<float>(), (int)T, (int)H, w_uv.data_ptr(), out.data_ptr(),
                                     cur_stream()));
}

void mla_decode(torch::Tensor q, torch::Tensor cache, torch::Tensor block_tables, torch::Tensor ctx_lens,
                torch::Tensor out, double scale, torch::Tensor part_o, torch::Tensor part_ml, int64_t pages_per_split) {
  SYN_CHECK_INPUT(q);
  TORCH_CHECK(q.scalar_type() == torch::kBFloat16 && q.dim() == 3 && q.size(2) == 576 && q.is_contiguous(),
              "q bf16 [B, H, 576] = [q_lat | q_pe]");
  TORCH_CHECK(cache.scalar_type() == torch::kBFloat16 && cache.size(-1) == 576 && cache.is_contiguous() &&
                  cache.numel() % (16 * 576) == 0,
              "latent cache bf16 [blocks, 16, 576]");
  const int64_t B = q.size(0), H = q.size(1);
  TORCH_CHECK(H % 16 == 0, "heads must be a multiple of 16, got ", H);
  TORCH_CHECK(out.scalar_type() == torch::kFloat32 && out.numel() == B * H * 512 && out.is_contiguous(),
              "out f32 [B, H, 512]");
  TORCH_CHECK(block_tables.scalar_type() == torch::kInt32 && block_tables.dim() == 2 && block_tables.size(0) >= B &&
                  block_tables.stride(1) == 1,
              "block tables int32 [B, max_blocks]");
  TORCH_CHECK(ctx_lens.scalar_type() == torch::kInt32 && ctx_lens.numel() >= B, "ctx_lens int32 [B]");
  const int64_t max_blocks = block_tables.size(1);
  const int64_t n_splits = (max_blocks + pages_per_split - 1) / pages_per_split;
  TORCH_CHECK(part_o.numel() >= B * H * n_splits * 512 && part_ml.numel() >= B * H * n_splits * 2,
              "split workspace too small");
  if (B == 0) return;
  const at::cuda::CUDAGuard guard(q.device());
  SYN_CHECK_CUDA(launch_mla_decode(q.data_ptr(), cache.data_ptr(), block_tables.data_ptr<int32_t>(),
                                   ctx_lens.data_ptr<int32_t>(), part_o.data_ptr<float>(), part_ml.data_ptr<float>(),
                                   out.data_ptr<float>(), (int)B, (int)H, (int)block_tables.stride(0),
                                   (int)pages_per_split, (int)n_splits, (float)scale, cur_stream()));
}


void doorbell_wait(torch::Tensor flag, int64_t want, double timeout_s, torch::Tensor status, torch::Tensor waited_ns) {
  SYN_CHECK_INPUT(flag);
  TORCH_CHECK(flag.scalar_type() == torch::kInt32 && status.scalar_type() == torch::kInt32, "int32 flag / status");
  TORCH_CHECK(timeout_s > 0 && timeout_s <= 60.0, "doorbell timeout must be in (0, 60] s, got ", timeout_s);
  const at::cuda::CUDAGuard guard(flag.device());
  SYN_CHECK_CUDA(launch_doorbell_wait(reinterpret_cast<const uint32_t*>(flag.data_ptr()), (uint32_t)want,
                                      (uint64_t)(timeout_s * 1e9), status.data_ptr<int32_t>(),
                                      waited_ns.numel() ? reinterpret_cast<uint64_t*>(waited_ns.data_ptr()) : nullptr,
                                      cur_stream()));
}

void doorbell_ring(torch::Tensor flag, int64_t value) {
  SYN_CHECK_INPUT(flag);
  TORCH_CHECK(flag.scalar_type() == torch::kInt32, "int32 flag");
  const at::cuda::CUDAGuard guard(flag.device());
  SYN_CHECK_CUDA(launch_doorbell_ring(reinterpret_cast<uint32_t*>(flag.data_ptr()), (uint32_t)value, cur_stream()));
}

void timestamp(torch::Tensor out, int64_t slot) {
  SYN_CHECK_INPUT(out);
  TORCH_CHECK(out.scalar_type() == torch::kInt64 && slot >= 0 && slot < out.numel(), "int64 slots");
  const at::cuda::CUDAGuard guard(out.device());
  SYN_CHECK_CUDA(launch_timestamp(reinterpret_cast<uint64_t*>(out.data_ptr()), (int)slot, cur_stream()));
}

void tap_gather(torch::Tensor src, torch::Tensor idx, torch::Tensor dst) {
  SYN_CHECK_INPUT(src);
  TORCH_CHECK(src.dim() == 2 && src.is_contiguous() &&
                  (src.scalar_type() == torch::kBFloat16 || src.scalar_type() == torch::kFloat32), "src [R, H]");
  TORCH_CHECK(idx.scalar_type() == torch::kInt32 && dst.scalar_type() == torch::kFloat32 &&
                  dst.size(0) == idx.numel() && dst.size(1) == src.size(1) && dst.is_contiguous(), "idx / dst");
  const at::cuda::CUDAGuard guard(src.device());
  SYN_CHECK_CUDA(launch_tap_gather(src.data_ptr(), src.scalar_type() == torch::kBFloat16, idx.data_ptr<int32_t>(),
                                   (int)idx.numel(), (int)src.size(1), dst.data_ptr<float>(), cur_stream()));
}

void tap_compare(torch::Tensor a, torch::Tensor b, torch::Tensor out) {
  SYN_CHECK_INPUT(a);
  TORCH_CHECK(a.sizes() == b.sizes() && a.dim() == 2 && a.scalar_type() == torch::kFloat32 &&
                  b.scalar_type() == torch::kFloat32 && a.is_contiguous() && b.is_contiguous(), "a, b f32 [n, H]");
  TORCH_CHECK(out.scalar_type() == torch::kFloat32 && out.numel() == a.size(0) * 2, "out f32 [n, 2]");
  const at::cuda::CUDAGuard guard(a.device());
  SYN_CHECK_CUDA(launch_tap_compare(a.data_ptr<float>(), b.data_ptr<float>(), (int)a.size(0), (int)a.size(1),
                                    out.data_ptr<float>(), cur_stream()));
}

void kv_pages(torch::Tensor kc, torch::Tensor vc, torch::Tensor pages, torch::Tensor packed, bool pack) {
  SYN_CHECK_INPUT(kc);
  TORCH_CHECK(kc.sizes() == vc.sizes() && kc.is_contiguous() && vc.is_contiguous() &&
                  kc.scalar_type() == vc.scalar_type(), "k/v caches");
  TORCH_CHECK(pages.scalar_type() == torch::kInt32 && pages.dim() == 1, "pages int32");
  const int64_t page_bytes = kc.numel() / kc.size(0) * kc.element_size();
  TORCH_CHECK(packed.is_contiguous() && packed.numel() * packed.element_size() == pages.numel() * 2 * page_bytes,
              "packed buffer must hold 2 x pages x page bytes");
  const at::cuda::CUDAGuard guard(kc.device());
  SYN_CHECK_CUDA(launch_kv_pages(kc.data_ptr(), vc.data_ptr(), pages.data_ptr<int32_t>(), (int)pages.numel(),
                                 page_bytes, packed.data_ptr(), pack, cur_stream()));
}


void expert_prefetch(torch::Tensor pred, torch::Tensor host_row, int64_t e0, std::vector<torch::Tensor> host,
                     std::vector<torch::Tensor> stage, std::vector<torch::Tensor> live, std::vector<torch::Tensor> home,
                     int64_t ctas) {
  SYN_CHECK_INPUT(pred);
  TORCH_CHECK(pred.scalar_type() == torch::kInt32 && host_row.scalar_type() == torch::kInt32 && host_row.is_cuda(),
              "int32 pred / host_row");
  const int n = (int)host.size();
  TORCH_CHECK(n >= 1 && n <= 4 && stage.size() == host.size() && live.size() == host.size() &&
                  home.size() == host.size(), "1..4 parts");
  const void* hp[4];
  void* sp[4];
  int64_t rb[4];
  int64_t* lp[4];
  const int64_t* op[4];
  const int64_t El = host_row.numel();
  for (int p = 0; p < n; ++p) {
    TORCH_CHECK(host[p].is_pinned() && stage[p].is_cuda() && host[p].sizes() == stage[p].sizes() &&
                    host[p].is_contiguous() && stage[p].is_contiguous(), "host rows pinned, staging rows on device");
    TORCH_CHECK(live[p].scalar_type() == torch::kInt64 && home[p].scalar_type() == torch::kInt64 &&
                    live[p].numel() == El && home[p].numel() == El, "pointer tables int64 [El]");
    hp[p] = host[p].data_ptr();
    sp[p] = stage[p].data_ptr();
    rb[p] = host[p].numel() ? host[p].nbytes() / host[p].size(0) : 0;
    lp[p] = live[p].data_ptr<int64_t>();
    op[p] = home[p].data_ptr<int64_t>();
  }
  const at::cuda::CUDAGuard guard(pred.device());
  SYN_CHECK_CUDA(launch_expert_prefetch(pred.data_ptr<int32_t>(), host_row.data_ptr<int32_t>(), (int)e0, (int)El, hp,
                                        sp, rb, lp, op, n, (int)ctas, cur_stream()));
}


void cpu_handoff(torch::Tensor h, torch::Tensor tok_off, torch::Tensor tok_idx, torch::Tensor pair_w, int64_t E,
                 int64_t k, int64_t max_rows, int64_t mailbox, int64_t layer, torch::Tensor ctr) {
  SYN_CHECK_INPUT(h);
  TORCH_CHECK(h.scalar_type() == torch::kBFloat16 && h.dim() == 2, "h bf16 [B, H]");
  TORCH_CHECK(tok_off.is_cuda() && tok_idx.is_cuda() && pair_w.is_cuda() && ctr.is_cuda(), "device CSR / counter");
  TORCH_CHECK(tok_off.numel() >= E + 1 && tok_idx.numel() >= h.size(0) * k && pair_w.numel() >= h.size(0) * k,
              "CSR sizes");
  TORCH_CHECK(ctr.scalar_type() == torch::kInt32 && ctr.numel() >= 2, "ctr int32 [2]");
  TORCH_CHECK(h.size(0) <= max_rows, "more rows than the mailbox holds");
  CpuHandoffArgs a;
  a.h = h.data_ptr();
  a.B = (int)h.size(0);
  a.H = (int)h.size(1);
  a.E = (int)E;
  a.k = (int)k;
  a.max_rows = (int)max_rows;
  a.layer = (int)layer;
  a.tok_off = tok_off.data_ptr<int32_t>();
  a.tok_idx = tok_idx.data_ptr<int32_t>();
  a.pair_w = pair_w.data_ptr<float>();
  a.mb = reinterpret_cast<uint8_t*>(mailbox);
  a.ctr = reinterpret_cast<uint32_t*>(ctr.data_ptr<int32_t>());
  const at::cuda::CUDAGuard guard(h.device());
  SYN_CHECK_CUDA(launch_cpu_handoff(a, cur_stream()));
}

void cpu_collect(int64_t mailbox, int64_t E, int64_t k, int64_t max_rows, torch::Tensor ctr, torch::Tensor yp,
                 double timeout_s, torch::Tensor status) {
  SYN_CHECK_INPUT(yp);
  TORCH_CHECK(yp.scalar_type() == torch::kFloat32 && yp.dim() == 2, "yp f32 [P, H]");
  TORCH_CHECK(ctr.is_cuda() && status.is_cuda() && status.scalar_type() == torch::kInt32, "device ctr / status");
  TORCH_CHECK(yp.size(0) >= 1, "yp rows");
  CpuCollectArgs a;
  a.mb = reinterpret_cast<const uint8_t*>(mailbox);
  a.H = (int)yp.size(1);
  a.E = (int)E;
  a.k = (int)k;
  a.max_rows = (int)max_rows;
  a.ctr = reinterpret_cast<const uint32_t*>(ctr.data_ptr<int32_t>());
  a.yp = yp.data_ptr<float>();
  a.timeout_ns = (uint64_t)(timeout_s * 1e9);
  a.status = status.data_ptr<int32_t>();
  a.pair_dst = nullptr;
  a.sig_peers = nullptr;
  a.sig_off = 0;
  a.sig_n = a.sig_rank = a.n_layers = a.layer = 0;
  a.step_ctr = nullptr;
  a.done_ctr = nullptr;
  const at::cuda::CUDAGuard guard(yp.device());
  SYN_CHECK_CUDA(launch_cpu_collect(a, cur_stream()));
}

// Expert-parallel form: the CPU's rows go to pair_dst[p] (source ranks' combine slots over
// NVLink), then this layer's completion flags are raised in every rank's region (the
// down-projection GEMV ran without raising them).
void cpu_collect_ep(int64_t mailbox, int64_t E, int64_t k, int64_t max_rows, int64_t H, torch::Tensor ctr,
                    torch::Tensor pair_dst, double timeout_s, torch::Tensor status, torch::Tensor peers,
                    int64_t sig_off, int64_t sig_rank, torch::Tensor step_ctr, int64_t n_layers, int64_t layer,
                    torch::Tensor done_ctr) {
  TORCH_CHECK(ctr.is_cuda() && status.is_cuda() && status.scalar_type() == torch::kInt32, "device ctr / status");
  TORCH_CHECK(pair_dst.is_cuda() && pair_dst.scalar_type() == torch::kInt64 && pair_dst.numel() >= max_rows * k,
              "pair_dst int64 [max_rows * k]");
  TORCH_CHECK(peers.is_cuda() && peers.scalar_type() == torch::kInt64, "peers int64");
  TORCH_CHECK(done_ctr.is_cuda() && done_ctr.scalar_type() == torch::kInt32 && done_ctr.numel() >= 1, "done_ctr");
  TORCH_CHECK(step_ctr.is_cuda(), "step_ctr");
  CpuCollectArgs a;
  a.mb = reinterpret_cast<const uint8_t*>(mailbox);
  a.H = (int)H;
  a.E = (int)E;
  a.k = (int)k;
  a.max_rows = (int)max_rows;
  a.ctr = reinterpret_cast<const uint32_t*>(ctr.data_ptr<int32_t>());
  a.yp = nullptr;
  a.timeout_ns = (uint64_t)(timeout_s * 1e9);
  a.status = status.data_ptr<int32_t>();
  a.pair_dst = pair_dst.data_ptr<int64_t>();
  a.sig_peers = peers.data_ptr<int64_t>();
  a.sig_off = sig_off;
  a.sig_n = (int)peers.numel();
  a.sig_rank = (int)sig_rank;
  a.n_layers = (int)n_layers;
  a.layer = (int)layer;
  a.step_ctr = reinterpret_cast<const uint32_t*>(step_ctr.data_ptr());
  a.done_ctr = reinterpret_cast<unsigned*>(done_ctr.data_ptr());
  const at::cuda::CUDAGuard guard(pair_dst.device());
  SYN_CHECK_CUDA(launch_cpu_collect(a, cur_stream()));
}


// out = x @ w^T on tcgen05 with bf16 weights (csrc/cuda/gemm_bf16_tc.cu).  mode: 0 bf16 [T, N],
// 1 SwiGLU bf16 [T, N/2], 3 f32 += [T, N], 5 f32 [T, N].  ws / counters: split-K workspace
// (f32, at least gemm_bf16_ws(N, K, T) floats) and N/128 zeroed counters (decode shapes).
void gemm_bf16(torch::Tensor x, torch::Tensor w, torch::Tensor out, int64_t mode, torch::Tensor ws,
               torch::Tensor counters, torch::Tensor status) {
  TORCH_CHECK(x.is_cuda() && w.is_cuda() && out.is_cuda(), "gemm_bf16: cuda tensors");
  TORCH_CHECK(x.scalar_type() == torch::kBFloat16 && w.scalar_type() == torch::kBFloat16 && x.dim() == 2 &&
                  w.dim() == 2 && x.stride(1) == 1 && w.is_contiguous(),
              "gemm_bf16: x bf16 [T, K] (unit column stride), w bf16 [N, K] contiguous");
  const int64_t T = x.size(0), K = x.size(1), N = w.size(0);
  TORCH_CHECK(w.size(1) == K, "gemm_bf16: K mismatch");
  TORCH_CHECK(mode == 0 || mode == 1 || mode == 3 || mode == 5, "gemm_bf16: mode 0, 1, 3 or 5");
  const int64_t ncol = mode == 1 ? N / 2 : N;
  TORCH_CHECK(out.dim() == 2 && out.size(0) == T && out.size(1) == ncol && out.stride(1) == 1, "gemm_bf16: out shape");
  TORCH_CHECK((mode <= 1 && out.scalar_type() == torch::kBFloat16) || (mode >= 3 && out.scalar_type() == torch::kFloat32),
              "gemm_bf16: out dtype");
  const at::cuda::CUDAGuard guard(x.device());
  SYN_CHECK_CUDA(launch_tc_gemm_bf16(x.data_ptr(), (int)T, (int)x.stride(0), w.data_ptr(), (int)N, (int)K, (int)mode,
                                     out.data_ptr(), (int)out.stride(0), ws.numel() ? ws.data_ptr<float>() : nullptr,
                                     (size_t)ws.numel(),
                                     counters.numel() ? reinterpret_cast<unsigned*>(counters.data_ptr<int32_t>()) : nullptr,
                                     nullptr, status.data_ptr<int32_t>(), cur_stream()));
}

int64_t gemm_bf16_ws(int64_t N, int64_t K, int64_t T) { return (int64_t)bf16_gemm_ws_floats((int)N, (int)K, (int)T); }

// Tensor-parallel row-parallel product with the peer push epilogue: each f32 row of x @ w^T
// goes into every peer's receive slot [rank][row] (owner_rows == 0) or into the row owner's
// slot (owner_rows > 0), then the completion flags (see PeerPush in syn/launch.h).
void gemm_bf16_tp(torch::Tensor x, torch::Tensor w, torch::Tensor peers, int64_t off_recv, int64_t cap, int64_t ldo,
                  int64_t owner_rows, int64_t off_flag, int64_t rank, torch::Tensor done_ctr, torch::Tensor step_ctr,
                  int64_t n_layers, int64_t layer, torch::Tensor ws, torch::Tensor counters, torch::Tensor status,
                  int64_t src_stride) {
  TORCH_CHECK(x.is_cuda() && w.is_cuda() && x.scalar_type() == torch::kBFloat16 && w.scalar_type() == torch::kBFloat16 &&
                  x.dim() == 2 && x.stride(1) == 1 && w.is_contiguous(),
              "gemm_bf16_tp: bf16 x [T, K], w [N, K]");
  const int64_t T = x.size(0), K = x.size(1), N = w.size(0);
  TORCH_CHECK(w.size(1) == K && ldo >= N, "gemm_bf16_tp: shapes");
  TORCH_CHECK(owner_rows > 0 ? T <= owner_rows * peers.numel() && owner_rows <= cap : T <= cap,
              "gemm_bf16_tp: rows exceed the receive slots");
  TORCH_CHECK(src_stride == 0 || src_stride * (peers.numel() - 1) + N + (T - 1) * ldo <= cap * ldo,
              "gemm_bf16_tp: column slices exceed the gather area");
  TORCH_CHECK(peers.is_cuda() && peers.scalar_type() == torch::kInt64, "peers int64 (device)");
  TORCH_CHECK(done_ctr.is_cuda() && done_ctr.scalar_type() == torch::kInt32, "done_ctr int32 (device)");
  PeerPush pp{peers.data_ptr<int64_t>(), (int)peers.numel(), (int)rank, (int)cap, (int)owner_rows, src_stride,
              off_recv, off_flag,
              reinterpret_cast<unsigned*>(done_ctr.data_ptr<int32_t>()),
              reinterpret_cast<const uint32_t*>(step_ctr.data_ptr()), (int)n_layers, (int)layer};
  const at::cuda::CUDAGuard guard(x.device());
  SYN_CHECK_CUDA(launch_tc_gemm_bf16(x.data_ptr(), (int)T, (int)x.stride(0), w.data_ptr(), (int)N, (int)K, 6, nullptr,
                                     (int)ldo, ws.numel() ? ws.data_ptr<float>() : nullptr, (size_t)ws.numel(),
                                     counters.numel() ? reinterpret_cast<unsigned*>(counters.data_ptr<int32_t>()) : nullptr,
                                     &pp, status.data_ptr<int32_t>(), cur_stream()));
}


// 4-bit weights, 16-64 token rows, on tcgen05 (decode orientation): out = x @ W^T with the
// epilogues of gemm_bf16 (mode 0, 1, 3, 5); q4_gemm_dec_tp: the peer push (mode 6).
void q4_gemm_dec(torch::Tensor x, torch::Tensor qw, torch::Tensor sm, int64_t N, int64_t K, int64_t mode,
                 torch::Tensor out, torch::Tensor status) {
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == torch::kBFloat16 && x.dim() == 2 && x.stride(1) == 1 && x.size(1) == K,
              "q4_gemm_dec: x bf16 [T, K]");
  TORCH_CHECK(qw.is_cuda() && sm.is_cuda() && qw.numel() * 4 == N * K / 2 && sm.numel() * 2 == N * K / 8,
              "q4_gemm_dec: tiled 4-bit weights [N, K]");
  TORCH_CHECK(mode == 0 || mode == 1 || mode == 3 || mode == 5, "q4_gemm_dec: mode 0, 1, 3 or 5");
  const int64_t T = x.size(0), ncol = mode == 1 ? N / 2 : N;
  TORCH_CHECK(out.dim() == 2 && out.size(0) == T && out.size(1) == ncol && out.stride(1) == 1, "q4_gemm_dec: out shape");
  TORCH_CHECK((mode <= 1 && out.scalar_type() == torch::kBFloat16) || (mode >= 3 && out.scalar_type() == torch::kFloat32),
              "q4_gemm_dec: out dtype");
  const at::cuda::CUDAGuard guard(x.device());
  SYN_CHECK_CUDA(launch_tc_gemm_q4_dec(x.data_ptr(), (int)T, (int)x.stride(0), qw.data_ptr(), sm.data_ptr(), (int)N,
                                       (int)K, (int)mode, out.data_ptr(), (int)out.stride(0), nullptr,
                                       status.data_ptr<int32_t>(), cur_stream()));
}

void q4_gemm_dec_tp(torch::Tensor x, torch::Tensor qw, torch::Tensor sm, int64_t N, int64_t K, torch::Tensor peers,
                    int64_t off_recv, int64_t cap, int64_t ldo, int64_t off_flag, int64_t rank, torch::Tensor done_ctr,
                    torch::Tensor step_ctr, int64_t n_layers, int64_t layer, torch::Tensor status) {
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == torch::kBFloat16 && x.dim() == 2 && x.stride(1) == 1 && x.size(1) == K,
              "q4_gemm_dec_tp: x bf16 [T, K]");
  TORCH_CHECK(qw.numel() * 4 == N * K / 2 && sm.numel() * 2 == N * K / 8, "q4_gemm_dec_tp: tiled 4-bit weights");
  TORCH_CHECK(x.size(0) <= cap && ldo >= N, "q4_gemm_dec_tp: rows exceed the receive slots");
  TORCH_CHECK(peers.is_cuda() && peers.scalar_type() == torch::kInt64, "peers int64 (device)");
  TORCH_CHECK(done_ctr.is_cuda() && done_ctr.scalar_type() == torch::kInt32, "done_ctr int32 (device)");
  PeerPush pp{peers.data_ptr<int64_t>(), (int)peers.numel(), (int)rank, (int)cap, 0, 0, off_recv, off_flag,
              reinterpret_cast<unsigned*>(done_ctr.data_ptr<int32_t>()),
              reinterpret_cast<const uint32_t*>(step_ctr.data_ptr()), (int)n_layers, (int)layer};
  const at::cuda::CUDAGuard guard(x.device());
  SYN_CHECK_CUDA(launch_tc_gemm_q4_dec(x.data_ptr(), (int)x.size(0), (int)x.stride(0), qw.data_ptr(), sm.data_ptr(),
                                       (int)N, (int)K, 6, nullptr, (int)ldo, &pp, status.data_ptr<int32_t>(),
                                       cur_stream()));
}

void flags_wait(torch::Tensor peers, int64_t rank, int64_t off_flag, torch::Tensor step_ctr, int64_t n_layers,
                int64_t layer, int64_t timeout_ns, torch::Tensor status) {
  TORCH_CHECK(peers.is_cuda() && peers.scalar_type() == torch::kInt64, "peers int64 (device)");
  const at::cuda::CUDAGuard guard(peers.device());
  SYN_CHECK_CUDA(launch_flags_wait(peers.data_ptr<int64_t>(), (int)peers.numel(), (int)rank, off_flag,
                                   reinterpret_cast<const uint32_t*>(step_ctr.data_ptr()), (int)n_layers, (int)layer,
                                   (uint64_t)timeout_ns, status.data_ptr<int32_t>(), cur_stream()));
}

}  // namespace syn
