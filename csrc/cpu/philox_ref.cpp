// CPU Philox4x32-10 draws (same header as the device sampler): the oracle for
// bit-exact tests of the device generator.
#include <torch/extension.h>

#include "syn/philox.h"

namespace syn {

torch::Tensor philox_cpu(int64_t seed, int64_t stream, int64_t counter0, int64_t n) {
  auto out = torch::empty({n}, torch::kInt32);
  uint32_t* o = reinterpret_cast<uint32_t*>(out.data_ptr());
  for (int64_t i = 0; i < n; ++i) o[i] = philox_draw((uint64_t)seed, (uint64_t)stream, (uint64_t)(counter0 + i));
  return out;
}

}  // namespace syn
