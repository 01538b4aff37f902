// Dequantisation of GGML block formats (GGUF tensor data) on the host, multi-threaded over
// blocks.  Used when a GGUF checkpoint is read tensor by tensor; the PyTorch restatement in
// syntropy_b200/formats/ggml_blocks.py is the oracle in the tests.  The reference gets the same
// operation from its vendored ggml (crates/kernels-ggml/src/lib.rs:61-325, `dequantize`).
//
// Block layouts (public GGML definitions; bytes read as written, little-endian):
//   Q8_0  32 values / 34 B : f16 d, 32 x int8 q                          -> d q
//   Q4_0  32 values / 18 B : f16 d, 16 B nibbles (value j: low nibble of byte j, j+16: high)
//                                                                         -> d (q - 8)
//   Q4_1  32 values / 20 B : f16 d, f16 m, 16 B nibbles                  -> d q + m
//   Q4_K 256 values / 144 B: f16 d, f16 dmin, 12 B of 6-bit scales / mins for eight
//         32-value sub-blocks, 128 B nibbles (32 B per sub-block pair: low nibbles the
//         first sub-block, high nibbles the second)                      -> d sc q - dmin mn
//   Q6_K 256 values / 210 B: 128 B low 4 bits, 64 B high 2 bits, 16 int8 scales (one per
//         16 values), f16 d                                              -> d sc (q - 32)
#include <torch/extension.h>

#include <ATen/Parallel.h>

#include <cmath>
#include <cstdint>
#include <cstring>
#include <string>
#include <thread>
#include <vector>
#include <algorithm>

namespace syn {
namespace {

// IEEE 754 binary16 -> binary32 from the format's definition (sign, 5-bit exponent bias 15,
// 10-bit fraction; subnormals scaled by 2^-24).
inline float half_bits_to_float(uint16_t h) {
  const uint32_t s = (uint32_t)(h & 0x8000u) << 16, e = (h >> 10) & 0x1fu, m = h & 0x3ffu;
  uint32_t bits;
  if (e == 0) {
    const float f = std::ldexp((float)m, -24);
    return s ? -f : f;
  }
  bits = e == 31 ? (s | 0x7f800000u | (m << 13)) : (s | ((e + 112u) << 23) | (m << 13));
  float f;
  std::memcpy(&f, &bits, 4);
  return f;
}

inline float f16_at(const uint8_t* p) { return half_bits_to_float((uint16_t)(p[0] | (p[1] << 8))); }

void q8_0(const uint8_t* __restrict__ b, float* __restrict__ y) {
  const float d = f16_at(b);
  const int8_t* q = reinterpret_cast<const int8_t*>(b + 2);
  for (int j = 0; j < 32; ++j) y[j] = d * q[j];
}

void q4_0(const uint8_t* __restrict__ b, float* __restrict__ y) {
  const float d = f16_at(b);
  for (int j = 0; j < 16; ++j) {
    y[j] = d * ((b[2 + j] & 15) - 8);
    y[j + 16] = d * ((b[2 + j] >> 4) - 8);
  }
}

void q4_1(const uint8_t* __restrict__ b, float* __restrict__ y) {
  const float d = f16_at(b), m = f16_at(b + 2);
  for (int j = 0; j < 16; ++j) {
    y[j] = d * (b[4 + j] & 15) + m;
    y[j + 16] = d * (b[4 + j] >> 4) + m;
  }
}

void q4_k(const uint8_t* __restrict__ b, float* __restrict__ y) {
  const float d = f16_at(b), dmin = f16_at(b + 2);
  const uint8_t* s = b + 4;
  const uint8_t* qs = b + 16;
  float a[8], c[8];
  for (int j = 0; j < 4; ++j) {
    a[j] = d * (s[j] & 63);
    c[j] = dmin * (s[j + 4] & 63);
    a[j + 4] = d * ((s[j + 8] & 15) | ((s[j] >> 6) << 4));
    c[j + 4] = dmin * ((s[j + 8] >> 4) | ((s[j + 4] >> 6) << 4));
  }
  for (int p = 0; p < 4; ++p) {  // 32 bytes hold sub-blocks 2p (low nibbles) and 2p+1 (high)
    const uint8_t* q = qs + p * 32;
    float* lo = y + (2 * p) * 32;
    float* hi = lo + 32;
    for (int l = 0; l < 32; ++l) {
      lo[l] = a[2 * p] * (q[l] & 15) - c[2 * p];
      hi[l] = a[2 * p + 1] * (q[l] >> 4) - c[2 * p + 1];
    }
  }
}

void q6_k(const uint8_t* __restrict__ b, float* __restrict__ y) {
  const int8_t* sc = reinterpret_cast<const int8_t*>(b + 192);
  const float d = f16_at(b + 208);
  for (int h = 0; h < 2; ++h) {
    const uint8_t* lo = b + h * 64;         // low 4 bits: groups 0 / 2 (low / high nibble)
    const uint8_t* hi = lo + 32;            //             groups 1 / 3
    const uint8_t* qq = b + 128 + h * 32;   // high 2 bits: groups 0..3 at bit 0, 2, 4, 6
    float* out = y + h * 128;
    for (int r = 0; r < 2; ++r) {           // 16 values share one scale
      const float s0 = d * sc[h * 8 + 0 + r], s1 = d * sc[h * 8 + 2 + r], s2 = d * sc[h * 8 + 4 + r],
                  s3 = d * sc[h * 8 + 6 + r];
      for (int l = r * 16; l < r * 16 + 16; ++l) {
        out[l] = s0 * (((lo[l] & 15) | ((qq[l] & 3) << 4)) - 32);
        out[32 + l] = s1 * (((hi[l] & 15) | (((qq[l] >> 2) & 3) << 4)) - 32);
        out[64 + l] = s2 * (((lo[l] >> 4) | (((qq[l] >> 4) & 3) << 4)) - 32);
        out[96 + l] = s3 * (((hi[l] >> 4) | (((qq[l] >> 6) & 3) << 4)) - 32);
      }
    }
  }
}

struct Fmt {
  int values, bytes;
  void (*fn)(const uint8_t*, float*);
};

Fmt fmt_of(const std::string& t) {
  if (t == "Q8_0") return {32, 34, q8_0};
  if (t == "Q4_0") return {32, 18, q4_0};
  if (t == "Q4_1") return {32, 20, q4_1};
  if (t == "Q4_K") return {256, 144, q4_k};
  if (t == "Q6_K") return {256, 210, q6_k};
  TORCH_CHECK(false, "ggml_dequant: unsupported block type ", t);
}

}  // namespace

// raw: uint8 bytes of whole blocks -> f32 [blocks * values per block]
torch::Tensor ggml_dequant(torch::Tensor raw, const std::string& type) {
  TORCH_CHECK(!raw.is_cuda() && raw.scalar_type() == torch::kUInt8 && raw.is_contiguous(),
              "ggml_dequant: contiguous host uint8 bytes");
  const Fmt f = fmt_of(type);
  TORCH_CHECK(raw.numel() % f.bytes == 0, "ggml_dequant: ", raw.numel(), " bytes is not a whole number of ", type,
              " blocks");
  const int64_t nb = raw.numel() / f.bytes;
  auto y = torch::empty({nb * f.values}, torch::kFloat32);
  const uint8_t* src = raw.data_ptr<uint8_t>();
  float* dst = y.data_ptr<float>();
  // plain threads: the extension is built without OpenMP, so at::parallel_for would run serially
  const int64_t per = 2048;
  const int64_t nt = std::max<int64_t>(1, std::min<int64_t>((nb + per - 1) / per, at::get_num_threads()));
  auto work = [&](int64_t t) {
    const int64_t a = nb * t / nt, b = nb * (t + 1) / nt;
    for (int64_t i = a; i < b; ++i) f.fn(src + i * f.bytes, dst + i * f.values);
  };
  std::vector<std::thread> th;
  for (int64_t t = 1; t < nt; ++t) th.emplace_back(work, t);
  work(0);
  for (auto& x : th) x.join();
  return y;
}

void register_ggml(pybind11::module& m) {
  m.def("ggml_dequant", &ggml_dequant, "GGML block bytes -> f32 values (Q8_0, Q4_0, Q4_1, Q4_K, Q6_K)",
        pybind11::call_guard<pybind11::gil_scoped_release>());
}

}  // namespace syn
