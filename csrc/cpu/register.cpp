#include <string>
// Registration of every exported function (one place, so the surface is easy to audit).
#include "ops.h"

#if __has_include("syn_build_stamp.h")
#include "syn_build_stamp.h"  // written by setup.py: the source hash and ABI version
#endif
#ifndef SYN_BUILD_ID
#define SYN_BUILD_ID "unstamped"
#endif
#ifndef SYN_ABI_VERSION
#define SYN_ABI_VERSION 0
#endif

// Build identity for loaders (plain C, exported): the hash of the native sources this object
// was built from and the ABI version of its interface.
extern "C" __attribute__((visibility("default"))) const char* syn_build_id() { return SYN_BUILD_ID; }
extern "C" __attribute__((visibility("default"))) int syn_abi_version() { return SYN_ABI_VERSION; }

namespace syn {

void register_all(pybind11::module& m) {
  m.def("build_id", [] { return std::string(syn_build_id()); });
  m.def("abi_version", [] { return syn_abi_version(); });
  m.def("q4_quantize_rows_cpu", &q4_quantize_rows_cpu);
  m.def("q4_dequant_rows_cpu", &q4_dequant_rows_cpu);
  m.def("q4_rows_to_tiled_cpu", &q4_rows_to_tiled_cpu);
  m.def("q4_quantize", &q4_quantize);
  m.def("q4_rows_to_tiled", &q4_rows_to_tiled);
  m.def("q4_tiled_to_rows", &q4_tiled_to_rows);
  m.def("q4t_dequant", &q4t_dequant);
  m.def("q4_gemv", &q4_gemv);
  m.def("block_sums", &block_sums);
  m.def("q4_gemv_dense", &q4_gemv_dense);
  m.def("expert_prefetch", &expert_prefetch, "router-predicted copy of next-layer host experts into VRAM staging");
  m.def("doorbell_wait", &doorbell_wait, "bounded device wait on a flag (error bit 0 on timeout)");
  m.def("doorbell_ring", &doorbell_ring, "release store of a flag value");
  m.def("timestamp", &timestamp, "globaltimer sample into out[slot]");
  m.def("tap_gather", &tap_gather, "rows of a hidden state -> f32 tap buffer");
  m.def("tap_compare", &tap_compare, "per-row max abs diff and relative L2 of two taps");
  m.def("kv_pages", &kv_pages, "pack (true) or unpack (false) the K/V pages of a block list");
  m.def("mla_decode", &mla_decode, "MLA decode attention (absorbed) over the paged latent cache");
  m.def("mla_q_absorb", &mla_q_absorb, "MLA decode: q_nope . W_uk and rope(q_pe) into the 576-wide query rows");
  m.def("mla_kv_write", &mla_kv_write, "MLA decode: normed latent + rope(k_pe) into the latent cache");
  m.def("mla_o_absorb", &mla_o_absorb, "MLA decode: o_lat . W_uv^T per head (bf16 out)");
  m.def("f8_quant_act", &f8_quant_act, "bf16 [T, K] -> e4m3 [T, K] + f32 1x128 scales");
  m.def("f8_rows_to_tiled", &f8_rows_to_tiled, "row-major e4m3 bytes -> mma-fragment tiled layout");
  m.def("f8_tiled_to_rows", &f8_tiled_to_rows, "inverse of f8_rows_to_tiled");
  m.def("f8_dequant_tiled", &f8_dequant_tiled, "tiled e4m3 + 128x128 block scales -> bf16 rows");
  m.def("f8_gemv", &f8_gemv, "block-scaled fp8 grouped GEMV (e4m3 x e4m3 tensor cores)");
  m.def("f8_gemv_ep", &f8_gemv_ep, "fp8 expert down projection into source ranks' combine slots + layer flags");
  m.def("attn_prefill", &attn_prefill, "causal prefill attention over the paged KV cache (GQA, head_dim 128)");
  m.def("attn_prefill_tc", &attn_prefill_tc, "causal paged prefill attention on tcgen05 (TMA, TMEM)");
  m.def("q4_gemv_dense_ws", &q4_gemv_dense_ws, "split-K workspace (floats) of the dense GEMV, -1 if unsupported");
  m.def("rmsnorm", &rmsnorm);
  m.def("moe_combine_rmsnorm", &moe_combine_rmsnorm);
  m.def("qk_rope_kv_write", &qk_rope_kv_write);
  m.def("embed", &embed);
  m.def("attn_decode", &attn_decode);
  m.def("router_logits", &router_logits);
  m.def("moe_topk", &moe_topk);
  m.def("cpu_handoff", &cpu_handoff);
  m.def("cpu_collect", &cpu_collect);
  m.def("cpu_collect_ep", &cpu_collect_ep);
  m.def("gemm_bf16", &gemm_bf16);
  m.def("gemm_bf16_ws", &gemm_bf16_ws);
  m.def("gemm_bf16_tp", &gemm_bf16_tp);
  m.def("flags_wait", &flags_wait);
  m.def("q4_gemm_dec", &q4_gemm_dec, "4-bit weights x 16-64 token rows on tcgen05 (decode orientation)");
  m.def("q4_gemm_dec_tp", &q4_gemm_dec_tp, "4-bit decode GEMM on tcgen05 with the TP peer push epilogue");
  m.def("argmax", &argmax);
  m.def("sample", &sample);
  m.def("philox", &philox);
  m.def("philox_cpu", &philox_cpu);
  m.def("symm_alloc", &symm_alloc);
  m.def("symm_open", &symm_open);
  m.def("symm_close", &symm_close);
  m.def("p2p_access", &p2p_access);
  m.def("ep_step_begin", &ep_step_begin);
  m.def("ep_dispatch", &ep_dispatch);
  m.def("ep_build", &ep_build);
  m.def("ep_combine", &ep_combine);
  m.def("q4_gemv_ep", &q4_gemv_ep);
  m.def("tc_gemm_q4", &tc_gemm_q4);
  m.def("tc_gemm_q4_banks", &tc_gemm_q4_banks, "grouped 4-bit tcgen05 GEMM over two weight banks (TMA)");
  m.def("verify_accept", &verify_accept);
  m.def("q4_gemv_tp", &q4_gemv_tp);
  m.def("tp_reduce_norm", &tp_reduce_norm);
  m.def("tp_twoshot", &tp_twoshot, "ordered two-shot all-reduce (peer-load reduce-scatter, peer-store all-gather) + residual + RMSNorm");
  register_runtime(m);
  register_formats(m);
  register_dispatcher(m);
  register_tier(m);
  register_cpu_experts(m);
  register_constrain(m);
  register_ggml(m);
  register_blake3(m);
}

}  // namespace syn
