// Declarations of every function exported by syntropy_b200._C.
#pragma once
#include <torch/extension.h>
#include <vector>

namespace syn {
// q4 format (CPU oracle)
torch::Tensor q4_quantize_rows_cpu(torch::Tensor w);
torch::Tensor q4_dequant_rows_cpu(torch::Tensor rows, int64_t N, int64_t K);
std::vector<torch::Tensor> q4_rows_to_tiled_cpu(torch::Tensor rows, int64_t N, int64_t K);
// q4 format (device)
std::vector<torch::Tensor> q4_quantize(torch::Tensor w);
std::vector<torch::Tensor> q4_rows_to_tiled(torch::Tensor rows, int64_t N, int64_t K);
torch::Tensor q4_tiled_to_rows(torch::Tensor qw, torch::Tensor sm, int64_t N, int64_t K);
torch::Tensor q4t_dequant(torch::Tensor qw, torch::Tensor sm, int64_t N, int64_t K);
void q4_gemv(torch::Tensor x, torch::Tensor qw_ptrs, torch::Tensor sm_ptrs, torch::Tensor tok_off,
             torch::Tensor tok_idx, torch::Tensor route_w, torch::Tensor res, torch::Tensor out,
             int64_t N, int64_t K, int64_t mode, int64_t nt_hint, int64_t e_active, torch::Tensor xsum,
             bool in_vram);
void tc_gemm_q4_banks(torch::Tensor x, torch::Tensor row_off, int64_t N, int64_t K, int64_t mode, torch::Tensor route_w,
                      torch::Tensor out, torch::Tensor status, int64_t max_mtiles, torch::Tensor b0_qw,
                      torch::Tensor b0_sm, torch::Tensor b1_qw, torch::Tensor b1_sm, torch::Tensor sel);
void block_sums(torch::Tensor x, torch::Tensor out);

void rmsnorm(torch::Tensor x, torch::Tensor w, double eps, torch::Tensor out);
void moe_combine_rmsnorm(torch::Tensor x, torch::Tensor yp, torch::Tensor pair_of, torch::Tensor shared,
                         torch::Tensor w, torch::Tensor out, double eps);
void qk_rope_kv_write(torch::Tensor qkv, int64_t Hq, int64_t Hkv, int64_t D, torch::Tensor qn, torch::Tensor kn,
                      double eps, torch::Tensor pos, torch::Tensor cos_t, torch::Tensor sin_t, torch::Tensor slot,
                      torch::Tensor q_out, torch::Tensor k_cache, torch::Tensor v_cache);
void embed(torch::Tensor table, torch::Tensor ids, torch::Tensor out);
void attn_decode(torch::Tensor q, torch::Tensor kc, torch::Tensor vc, torch::Tensor block_tables,
                 torch::Tensor ctx_lens, torch::Tensor part_o, torch::Tensor part_ml, torch::Tensor out,
                 int64_t pages_per_split, double scale);
void router_logits(torch::Tensor h, torch::Tensor W, torch::Tensor logits);
void moe_topk(torch::Tensor logits, torch::Tensor bias, int64_t E, int64_t k, int64_t scoring, int64_t n_groups,
              int64_t topk_groups, bool norm, double scaling, bool pred, torch::Tensor topk_ids, torch::Tensor topk_w,
              torch::Tensor tok_off, torch::Tensor tok_idx, torch::Tensor pair_w, torch::Tensor pair_of,
              torch::Tensor pred_mask, torch::Tensor ws, torch::Tensor counts,
              torch::Tensor count_rows);
void argmax(torch::Tensor logits, torch::Tensor out);
void sample(torch::Tensor logits, torch::Tensor temperature, torch::Tensor top_k, torch::Tensor top_p,
            torch::Tensor seed, torch::Tensor stream, torch::Tensor counter, torch::Tensor out);
torch::Tensor philox(int64_t seed, int64_t stream, int64_t counter0, int64_t n, torch::Tensor like);
torch::Tensor philox_cpu(int64_t seed, int64_t stream, int64_t counter0, int64_t n);

std::vector<torch::Tensor> symm_alloc(int64_t nbytes);
int64_t symm_open(torch::Tensor handle);
void symm_close(int64_t ptr);
bool p2p_access(int64_t a, int64_t b);
void ep_step_begin(torch::Tensor step_ctr);
void ep_dispatch(torch::Tensor peers, int64_t N, int64_t rank, int64_t cap, int64_t H, int64_t k, int64_t E_loc,
                 std::vector<int64_t> offs, torch::Tensor step_ctr, int64_t n_layers, int64_t layer,
                 int64_t timeout_ns, torch::Tensor status, torch::Tensor h, torch::Tensor ids, torch::Tensor w);
void ep_build(torch::Tensor peers, int64_t N, int64_t rank, int64_t cap, int64_t H, int64_t k, int64_t E_loc,
              std::vector<int64_t> offs, torch::Tensor step_ctr, int64_t n_layers, int64_t layer, int64_t timeout_ns,
              torch::Tensor status, torch::Tensor tok_off, torch::Tensor tok_idx, torch::Tensor pair_w,
              torch::Tensor pair_dst);
void ep_combine(torch::Tensor peers, int64_t N, int64_t rank, int64_t cap, int64_t H, int64_t k, int64_t E_loc,
                std::vector<int64_t> offs, torch::Tensor step_ctr, int64_t n_layers, int64_t layer,
                int64_t timeout_ns, torch::Tensor status, torch::Tensor x, torch::Tensor wn, torch::Tensor hout,
                double eps);
void q4_gemv_ep(torch::Tensor x, torch::Tensor qw_ptrs, torch::Tensor sm_ptrs, torch::Tensor tok_off,
                torch::Tensor tok_idx, torch::Tensor route_w, torch::Tensor out_ptrs, int64_t N, int64_t K,
                torch::Tensor done_ctr, torch::Tensor peers, int64_t sig_off, int64_t sig_rank,
                torch::Tensor step_ctr, int64_t n_layers, int64_t layer, int64_t nt_hint, int64_t e_active,
                bool in_vram);

void tc_gemm_q4(torch::Tensor x, torch::Tensor qw_ptrs, torch::Tensor sm_ptrs, torch::Tensor row_off, int64_t N,
                int64_t K, int64_t mode, torch::Tensor route_w, torch::Tensor out, torch::Tensor status,
                int64_t max_mtiles, torch::Tensor bank_qw, torch::Tensor bank_sm, int64_t group_base);

void q4_gemv_tp(torch::Tensor x, torch::Tensor qw_ptrs, torch::Tensor sm_ptrs, torch::Tensor tok_off, int64_t N,
                int64_t K, torch::Tensor done_ctr, torch::Tensor peers, int64_t peer_off, int64_t peer_cap,
                int64_t sig_off, int64_t rank, torch::Tensor step_ctr, int64_t n_layers, int64_t layer);
void tp_twoshot(torch::Tensor peers, int64_t rank, int64_t off_part, int64_t off_gather, int64_t off_flag_ready,
                int64_t off_flag_done, int64_t seq, int64_t timeout_ns, torch::Tensor status, torch::Tensor done_ctr,
                torch::Tensor x, torch::Tensor wn, torch::Tensor hout, double eps);
void tp_reduce_norm(torch::Tensor peers, int64_t N, int64_t rank, int64_t cap, int64_t H, std::vector<int64_t> offs,
                    torch::Tensor step_ctr, int64_t n_layers, int64_t layer, int64_t timeout_ns, torch::Tensor status,
                    int64_t off_recv, int64_t off_flag, torch::Tensor x, torch::Tensor wn, torch::Tensor hout,
                    double eps);
void verify_accept(torch::Tensor logits, torch::Tensor draft, torch::Tensor temperature, torch::Tensor top_k,
                   torch::Tensor top_p, torch::Tensor seed, torch::Tensor stream, torch::Tensor counter,
                   torch::Tensor out_tokens, torch::Tensor n_accept, torch::Tensor draft_probs);
int64_t q4_gemv_dense_ws(int64_t N, int64_t K, int64_t rows);
void attn_prefill(torch::Tensor q, torch::Tensor kc, torch::Tensor vc, torch::Tensor block_tables, torch::Tensor cu_q,
                  torch::Tensor kv_lens, torch::Tensor out, int64_t max_q_len, double scale);
void attn_prefill_tc(torch::Tensor q, torch::Tensor kc, torch::Tensor vc, torch::Tensor block_tables,
                     torch::Tensor cu_q, torch::Tensor kv_lens, torch::Tensor out, int64_t max_q_len, double scale,
                     torch::Tensor status);
std::vector<torch::Tensor> f8_quant_act(torch::Tensor x);
torch::Tensor f8_rows_to_tiled(torch::Tensor q, int64_t N, int64_t K);
torch::Tensor f8_tiled_to_rows(torch::Tensor tiled, int64_t N, int64_t K);
torch::Tensor f8_dequant_tiled(torch::Tensor tiled, torch::Tensor scale, int64_t N, int64_t K);
void f8_gemv(torch::Tensor xq, torch::Tensor xs, torch::Tensor qw_ptrs, torch::Tensor sm_ptrs, torch::Tensor tok_off,
             torch::Tensor tok_idx, torch::Tensor route_w, torch::Tensor out, int64_t N, int64_t K, int64_t mode,
             int64_t nt_hint, torch::Tensor ws);
void f8_gemv_ep(torch::Tensor xq, torch::Tensor xs, torch::Tensor qw_ptrs, torch::Tensor sm_ptrs,
                torch::Tensor tok_off, torch::Tensor route_w, torch::Tensor out_ptrs, int64_t N, int64_t K,
                torch::Tensor done_ctr, torch::Tensor peers, int64_t sig_off, int64_t sig_rank, torch::Tensor step_ctr,
                int64_t n_layers, int64_t layer, int64_t nt_hint);
void mla_q_absorb(torch::Tensor q, torch::Tensor w_uk, torch::Tensor cos_t, torch::Tensor sin_t, torch::Tensor pos,
                  torch::Tensor qcat);
void mla_kv_write(torch::Tensor kva, torch::Tensor norm_w, double eps, torch::Tensor cos_t, torch::Tensor sin_t,
                  torch::Tensor pos, torch::Tensor slot, torch::Tensor cache);
void mla_o_absorb(torch::Tensor o_lat, torch::Tensor w_uv, torch::Tensor out);
void mla_decode(torch::Tensor q, torch::Tensor cache, torch::Tensor block_tables, torch::Tensor ctx_lens,
                torch::Tensor out, double scale, torch::Tensor part_o, torch::Tensor part_ml, int64_t pages_per_split);
void doorbell_wait(torch::Tensor flag, int64_t want, double timeout_s, torch::Tensor status, torch::Tensor waited_ns);
void doorbell_ring(torch::Tensor flag, int64_t value);
void timestamp(torch::Tensor out, int64_t slot);
void tap_gather(torch::Tensor src, torch::Tensor idx, torch::Tensor dst);
void tap_compare(torch::Tensor a, torch::Tensor b, torch::Tensor out);
void kv_pages(torch::Tensor kc, torch::Tensor vc, torch::Tensor pages, torch::Tensor packed, bool pack);
void expert_prefetch(torch::Tensor pred, torch::Tensor host_row, int64_t e0, std::vector<torch::Tensor> host,
                     std::vector<torch::Tensor> stage, std::vector<torch::Tensor> live, std::vector<torch::Tensor> home,
                     int64_t ctas);
void q4_gemv_dense(torch::Tensor x, torch::Tensor qw_ptrs, torch::Tensor sm_ptrs, torch::Tensor tok_off,
                   torch::Tensor out, int64_t N, int64_t K, int64_t mode, torch::Tensor ws, torch::Tensor counters);
void register_all(pybind11::module& m);
void register_runtime(pybind11::module& m);
void cpu_handoff(torch::Tensor h, torch::Tensor tok_off, torch::Tensor tok_idx, torch::Tensor pair_w, int64_t E,
                 int64_t k, int64_t max_rows, int64_t mailbox, int64_t layer, torch::Tensor ctr);
void cpu_collect(int64_t mailbox, int64_t E, int64_t k, int64_t max_rows, torch::Tensor ctr, torch::Tensor yp,
                 double timeout_s, torch::Tensor status);
void cpu_collect_ep(int64_t mailbox, int64_t E, int64_t k, int64_t max_rows, int64_t H, torch::Tensor ctr,
                    torch::Tensor pair_dst, double timeout_s, torch::Tensor status, torch::Tensor peers,
                    int64_t sig_off, int64_t sig_rank, torch::Tensor step_ctr, int64_t n_layers, int64_t layer,
                    torch::Tensor done_ctr);
void register_dispatcher(pybind11::module& m);
void register_tier(pybind11::module& m);
void register_cpu_experts(pybind11::module& m);
void register_constrain(pybind11::module& m);
void register_formats(pybind11::module& m);
void register_ggml(pybind11::module& m);
void register_blake3(pybind11::module& m);
void gemm_bf16(torch::Tensor x, torch::Tensor w, torch::Tensor out, int64_t mode, torch::Tensor ws,
               torch::Tensor counters, torch::Tensor status);
int64_t gemm_bf16_ws(int64_t N, int64_t K, int64_t T);
void gemm_bf16_tp(torch::Tensor x, torch::Tensor w, torch::Tensor peers, int64_t off_recv, int64_t cap, int64_t ldo,
                  int64_t owner_rows, int64_t off_flag, int64_t rank, torch::Tensor done_ctr, torch::Tensor step_ctr,
                  int64_t n_layers, int64_t layer, torch::Tensor ws, torch::Tensor counters, torch::Tensor status,
                  int64_t src_stride);
void q4_gemm_dec(torch::Tensor x, torch::Tensor qw, torch::Tensor sm, int64_t N, int64_t K, int64_t mode,
                 torch::Tensor out, torch::Tensor status);
void q4_gemm_dec_tp(torch::Tensor x, torch::Tensor qw, torch::Tensor sm, int64_t N, int64_t K, torch::Tensor peers,
                    int64_t off_recv, int64_t cap, int64_t ldo, int64_t off_flag, int64_t rank, torch::Tensor done_ctr,
                    torch::Tensor step_ctr, int64_t n_layers, int64_t layer, torch::Tensor status);
void flags_wait(torch::Tensor peers, int64_t rank, int64_t off_flag, torch::Tensor step_ctr, int64_t n_layers,
                int64_t layer, int64_t timeout_ns, torch::Tensor status);

}  // namespace syn
