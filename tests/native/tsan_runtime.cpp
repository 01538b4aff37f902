// ThreadSanitizer driver for the native runtime's concurrent pieces (built and run by
// tests/test_native_tsan.py with -fsanitize=thread):
//  1. the lock-free SPSC ring: one producer and one consumer thread move 200000 sequenced
//     messages through a small ring;
//  2. the CPU expert worker pool: this thread plays the GPU, publishing a layer's rows and
//     routing CSR in the mailbox and raising the go word, then waiting (bounded) for the done
//     word and reading the outputs, for 300 jobs over two layers.
// Exit code 0 and no sanitizer report mean no data race was observed.
#define SYN_NO_TORCH
#include "../../csrc/cpu/cpu_experts.cpp"
#include "../../csrc/include/syn/spsc.h"

#include <chrono>
#include <cstdio>
#include <cstdlib>
#include <random>

using namespace syn;

static int test_spsc() {
  const uint64_t cap = 64;
  std::vector<uint8_t> mem(SpscRing::bytes_needed(cap, 32) + 64);
  void* base = reinterpret_cast<void*>((reinterpret_cast<uintptr_t>(mem.data()) + 63) & ~uintptr_t(63));
  SpscRing* r = SpscRing::init(base, cap, 32);
  const uint64_t N = 200000;
  std::thread prod([&] {
    for (uint64_t i = 0; i < N;) {
      if (r->push(&i, sizeof(i))) ++i;
      else std::this_thread::yield();
    }
  });
  uint64_t want = 0;
  while (want < N) {
    uint64_t v = 0;
    const int64_t n = r->pop(&v, sizeof(v));
    if (n < 0) {
      std::this_thread::yield();
      continue;
    }
    if (n != 8 || v != want) {
      std::fprintf(stderr, "spsc: got %llu want %llu\n", (unsigned long long)v, (unsigned long long)want);
      prod.join();
      return 1;
    }
    ++want;
  }
  prod.join();
  return 0;
}

static int test_pool() {
  const int E = 8, k = 2, H = 128, I = 64, R = 4, L = 2;
  std::mt19937 rng(1);
  // tiled 4-bit weights (any bits: the test checks ordering, not values) and fp16 scales
  auto words = [&](size_t n) {
    std::vector<uint32_t> v(n);
    for (auto& x : v) x = rng();
    return v;
  };
  auto scales = [&](size_t n) {
    std::vector<uint16_t> v(n);
    for (auto& x : v) x = (uint16_t)(0x2000 + (rng() & 0x3ff));  // small positive halves
    return v;
  };
  std::vector<std::vector<uint32_t>> qg, qd;
  std::vector<std::vector<uint16_t>> sg, sd;
  for (int e = 0; e < E; ++e) {
    qg.push_back(words((size_t)2 * I * H / 8));
    sg.push_back(scales((size_t)2 * I * H / 32 * 2));
    qd.push_back(words((size_t)H * I / 8));
    sd.push_back(scales((size_t)H * I / 32 * 2));
  }
  const CpuMailboxLayout lay = cpu_mailbox_layout(E, k, R, H);
  std::vector<uint8_t> mbv(lay.bytes + 256, 0);
  uint8_t* mb = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(mbv.data()) + 255) & ~uintptr_t(255));
  uint32_t* w = reinterpret_cast<uint32_t*>(mb);
  CpuExpertTier tier(L, E, H, I, k, R, (int64_t)mb, {}, 4, -1);
  for (int l = 0; l < L; ++l)
    for (int e : {1, 4, 6})
      tier.set_expert(l, e, (int64_t)qg[e].data(), (int64_t)sg[e].data(), (int64_t)qd[e].data(),
                      (int64_t)sd[e].data());
  tier.start();
  int32_t* off = reinterpret_cast<int32_t*>(mb + lay.tok_off);
  int32_t* tidx = reinterpret_cast<int32_t*>(mb + lay.tok_idx);
  float* pw = reinterpret_cast<float*>(mb + lay.pair_w);
  uint16_t* h = reinterpret_cast<uint16_t*>(mb + lay.h);
  const float* out = reinterpret_cast<const float*>(mb + lay.out);
  double sink = 0;
  for (uint32_t seq = 1; seq <= 300; ++seq) {
    // routing: token t picks experts (t + seq) % E and (t + seq + 3) % E
    std::vector<std::pair<int, int>> pairs;
    for (int t = 0; t < R; ++t) {
      pairs.push_back({(int)((t + seq) % E), t});
      pairs.push_back({(int)((t + seq + 3) % E), t});
    }
    std::sort(pairs.begin(), pairs.end());
    for (int e = 0; e <= E; ++e) off[e] = 0;
    for (auto& p : pairs) off[p.first + 1]++;
    for (int e = 0; e < E; ++e) off[e + 1] += off[e];
    for (size_t i = 0; i < pairs.size(); ++i) {
      tidx[i] = pairs[i].second;
      pw[i] = 0.5f;
    }
    for (int i = 0; i < R * H; ++i) h[i] = (uint16_t)(0x3c00 + (rng() & 0xff));
    w[MB_LAYER] = seq % L;
    w[MB_ROWS] = R;
    __atomic_store_n(&w[MB_GO], seq, __ATOMIC_RELEASE);
    const auto t0 = std::chrono::steady_clock::now();
    while (__atomic_load_n(&w[MB_DONE], __ATOMIC_ACQUIRE) != seq) {
      if (std::chrono::steady_clock::now() - t0 > std::chrono::seconds(20)) {
        std::fprintf(stderr, "pool: job %u not answered\n", seq);
        tier.stop();
        return 1;
      }
      std::this_thread::yield();
    }
    const uint32_t n_out = w[MB_NOUT];
    if (w[MB_ERR] != 0 || n_out == 0) {
      std::fprintf(stderr, "pool: job %u err %u n_out %u\n", seq, w[MB_ERR], n_out);
      tier.stop();
      return 1;
    }
    for (uint32_t q = 0; q < n_out; ++q) sink += out[(size_t)q * H];
  }
  tier.stop();
  const auto st = tier.stats();
  std::printf("pool: %lld jobs, %lld pairs (checksum %g)\n", (long long)st.jobs, (long long)st.pairs, sink);
  return st.jobs == 300 ? 0 : 1;
}

int main() {
  if (test_spsc()) return 1;
  std::printf("spsc ok\n");
  if (test_pool()) return 1;
  std::printf("pool ok\n");
  return 0;
}
