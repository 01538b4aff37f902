// Per-step host hot loop in C++: fills the pinned step descriptor (syn/step_desc.h) for the
// live rows and the bucket's padding rows in one call, and launches a captured decode graph
// (descriptor upload + graph launch on the caller's stream).  Replaces a per-row Python loop
// of tensor element writes.  Reference: the per-GPU dispatcher of crates/exec (step
// descriptor write, graph launch per bucket).
#include <cuda_runtime.h>
#include <torch/extension.h>

#include <cstring>
#include <vector>

#include "syn/step_desc.h"

namespace syn {

void step_desc_fill(torch::Tensor host, int64_t rows_cap, int64_t max_blocks, std::vector<int32_t> tokens,
                    std::vector<int32_t> pos, std::vector<int32_t> top_k, std::vector<int64_t> slot,
                    std::vector<int64_t> seed, std::vector<int64_t> stream, std::vector<int64_t> counter,
                    std::vector<double> temperature, std::vector<double> top_p,
                    std::vector<std::vector<int32_t>> block_lists, int64_t bucket) {
  const StepDescLayout L(rows_cap, max_blocks);
  TORCH_CHECK(host.device().is_cpu() && host.scalar_type() == torch::kUInt8 && host.is_contiguous() &&
                  (size_t)host.numel() == L.nbytes,
              "step descriptor host buffer: uint8 [", L.nbytes, "]");
  const int64_t n = (int64_t)tokens.size();
  TORCH_CHECK(n <= bucket && bucket <= rows_cap, "rows ", n, " bucket ", bucket, " capacity ", rows_cap);
  TORCH_CHECK(pos.size() == (size_t)n && top_k.size() == (size_t)n && slot.size() == (size_t)n &&
                  seed.size() == (size_t)n && stream.size() == (size_t)n && counter.size() == (size_t)n &&
                  temperature.size() == (size_t)n && top_p.size() == (size_t)n && block_lists.size() == (size_t)n,
              "per-row field lengths differ");
  uint8_t* b = host.data_ptr<uint8_t>();
  auto i32 = [&](size_t off) { return reinterpret_cast<int32_t*>(b + off); };
  auto i64 = [&](size_t off) { return reinterpret_cast<int64_t*>(b + off); };
  auto f32 = [&](size_t off) { return reinterpret_cast<float*>(b + off); };
  for (int64_t r = 0; r < bucket; ++r) {
    const bool live = r < n;
    i32(L.off_tokens)[r] = live ? tokens[r] : 0;
    i32(L.off_pos)[r] = live ? pos[r] : 0;
    i32(L.off_ctx)[r] = live ? pos[r] + 1 : 1;
    i32(L.off_topk)[r] = live ? top_k[r] : 0;
    f32(L.off_temp)[r] = live ? (float)temperature[r] : 0.f;
    f32(L.off_topp)[r] = live ? (float)top_p[r] : 1.f;
    i64(L.off_slot)[r] = live ? slot[r] : -1;
    i64(L.off_seed)[r] = live ? seed[r] : 0;
    i64(L.off_stream)[r] = live ? stream[r] : 0;
    i64(L.off_counter)[r] = live ? counter[r] : 0;
    int32_t* bt = i32(L.off_bt) + r * max_blocks;
    if (live) {
      const auto& bl = block_lists[r];
      TORCH_CHECK((int64_t)bl.size() <= max_blocks, "row ", r, ": ", bl.size(), " blocks > table width ", max_blocks);
      std::memcpy(bt, bl.data(), bl.size() * sizeof(int32_t));
    } else {
      bt[0] = 0;  // the null page
    }
  }
}

// Upload the descriptor and launch a captured graph exec on `stream` (both raw handles).
void step_launch(torch::Tensor host, torch::Tensor dev, int64_t graph_exec, int64_t stream) {
  TORCH_CHECK(host.numel() == dev.numel() && dev.is_cuda(), "descriptor buffers");
  auto s = reinterpret_cast<cudaStream_t>(stream);
  cudaError_t e = cudaMemcpyAsync(dev.data_ptr(), host.data_ptr(), (size_t)host.numel(), cudaMemcpyHostToDevice, s);
  TORCH_CHECK(e == cudaSuccess, "descriptor upload: ", cudaGetErrorString(e));
  e = cudaGraphLaunch(reinterpret_cast<cudaGraphExec_t>(graph_exec), s);
  TORCH_CHECK(e == cudaSuccess, "graph launch: ", cudaGetErrorString(e));
}

void register_dispatcher(pybind11::module& m) {
  m.def("step_desc_fill", &step_desc_fill, "fill the pinned step descriptor for live + padding rows");
  m.def("step_launch", &step_launch, "descriptor upload + CUDA graph launch on a stream");
}

}  // namespace syn
