// CPU oracle for the 4-bit block format (syn/q4.h): quantise, dequantise and the
// row-block <-> tiled repack.  Same operation order as csrc/cuda/q4.cu so the two agree
// bit for bit.  The f32 dequantised value is d * q + m with one rounding (fmaf), the
// reference's "fl32(element x scale)" rule (plan/rfcs/RFC-0042-quantization-and-
// numerical-fidelity.md §2).
#include <torch/extension.h>
#include <c10/util/Half.h>
#include <cmath>
#include <cstring>

#include "syn/q4.h"

namespace syn {

static inline uint16_t f2h_bits(float v) { return c10::Half(v).x; }
static inline float h2f_bits(uint16_t b) {
  c10::Half h;
  h.x = b;
  return (float)h;
}

// w: f32 [N, K] -> rows uint8 [N * K/32 * 20]
torch::Tensor q4_quantize_rows_cpu(torch::Tensor w) {
  TORCH_CHECK(w.device().is_cpu() && w.scalar_type() == torch::kFloat32 && w.dim() == 2, "f32 cpu [N,K]");
  w = w.contiguous();
  const int64_t N = w.size(0), K = w.size(1);
  TORCH_CHECK(K % SYN_Q4_BLOCK == 0, "K % 32");
  const int64_t nb = K / SYN_Q4_BLOCK;
  auto rows = torch::empty({N * nb * SYN_Q4_ROW_BLOCK_BYTES}, torch::kUInt8);
  const float* x = w.data_ptr<float>();
  uint8_t* o = rows.data_ptr<uint8_t>();
  at::parallel_for(0, N * nb, 1024, [&](int64_t b0, int64_t b1) {
    for (int64_t i = b0; i < b1; ++i) {
      const float* p = x + i * SYN_Q4_BLOCK;  // rows are contiguous blocks
      float mn = INFINITY, mx = -INFINITY;
      for (int j = 0; j < SYN_Q4_BLOCK; ++j) {
        mn = std::fmin(mn, p[j]);
        mx = std::fmax(mx, p[j]);
      }
      const uint16_t db = f2h_bits((mx - mn) / 15.f), mb = f2h_bits(mn);
      const float d = h2f_bits(db), m = h2f_bits(mb);
      uint8_t* b = o + i * SYN_Q4_ROW_BLOCK_BYTES;
      memcpy(b, &db, 2);
      memcpy(b + 2, &mb, 2);
      uint8_t q[32];
      for (int j = 0; j < 32; ++j) {
        if (d == 0.f) {
          q[j] = 0;
        } else {
          float v = std::rint((p[j] - m) / d);
          v = std::fmin(std::fmax(v, 0.f), 15.f);
          q[j] = (uint8_t)v;
        }
      }
      for (int j = 0; j < 16; ++j) b[4 + j] = (uint8_t)(q[j] | (q[j + 16] << 4));
    }
  });
  return rows;
}

torch::Tensor q4_dequant_rows_cpu(torch::Tensor rows, int64_t N, int64_t K) {
  TORCH_CHECK(rows.device().is_cpu() && rows.scalar_type() == torch::kUInt8, "uint8 cpu");
  TORCH_CHECK(rows.numel() == N * K / 32 * SYN_Q4_ROW_BLOCK_BYTES, "byte count");
  rows = rows.contiguous();
  auto out = torch::empty({N, K}, torch::kFloat32);
  const uint8_t* r = rows.data_ptr<uint8_t>();
  float* y = out.data_ptr<float>();
  const int64_t nb = N * K / 32;
  at::parallel_for(0, nb, 1024, [&](int64_t b0, int64_t b1) {
    for (int64_t i = b0; i < b1; ++i) {
      const uint8_t* b = r + i * SYN_Q4_ROW_BLOCK_BYTES;
      uint16_t db, mb;
      memcpy(&db, b, 2);
      memcpy(&mb, b + 2, 2);
      const float d = h2f_bits(db), m = h2f_bits(mb);
      for (int j = 0; j < 16; ++j) {
        y[i * 32 + j] = std::fma(d, (float)(b[4 + j] & 15), m);
        y[i * 32 + j + 16] = std::fma(d, (float)(b[4 + j] >> 4), m);
      }
    }
  });
  return out;
}

// rows -> tiled (qw int32 [N*K/8], sm fp16 [N*K/16])
std::vector<torch::Tensor> q4_rows_to_tiled_cpu(torch::Tensor rows, int64_t N, int64_t K) {
  TORCH_CHECK(N % 16 == 0 && K % 64 == 0, "q4 tiled layout needs N % 16 == 0 and K % 64 == 0, got N=", N, " K=", K);
  rows = rows.contiguous();
  auto qw = torch::zeros({N * K / 8}, torch::kInt32);
  auto sm = torch::empty({N * K / 16}, torch::kFloat16);
  uint32_t* q = reinterpret_cast<uint32_t*>(qw.data_ptr());
  uint16_t* s = reinterpret_cast<uint16_t*>(sm.data_ptr());
  const uint8_t* r = rows.data_ptr<uint8_t>();
  const int64_t nb = K / 32;
  for (int64_t n = 0; n < N; ++n) {
    for (int64_t kb = 0; kb < nb; ++kb) {
      const uint8_t* b = r + (n * nb + kb) * SYN_Q4_ROW_BLOCK_BYTES;
      const int64_t si = q4t_scale_index(K, n, kb);
      memcpy(s + 2 * si, b, 4);
      for (int j = 0; j < 32; ++j) {
        const uint32_t v = j < 16 ? (b[4 + j] & 15u) : (b[4 + j - 16] >> 4);
        int64_t wi;
        int nib;
        q4t_locate(N, K, n, kb * 32 + j, &wi, &nib);
        q[wi] |= v << (4 * nib);
      }
    }
  }
  return {qw, sm};
}

}  // namespace syn
