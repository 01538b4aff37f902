// BLAKE3 (O'Connor, Aumasson, Neves, Wilcox-O'Hearn, 2020: "BLAKE3 - one function, fast
// everywhere", the published specification), unkeyed hash with a 32-byte output, written from
// the specification: 1024-byte chunks of 64-byte blocks compressed with the BLAKE2s-derived
// 7-round function, chunk chaining values merged pairwise into a binary tree (left subtrees
// a power of two chunks, built with a stack of pending values), ROOT flag on the final
// compression.  Portable scalar code: it hashes pairing fields and other short inputs, not
// bulk data.  Used by the LAN pairing commitments and codes (reference
// crates/cluster/src/pairing.rs:28-100).
#include <pybind11/pybind11.h>

#include <cstdint>
#include <cstring>
#include <string>
#include <vector>

namespace syn {
namespace {

constexpr uint32_t IV[8] = {0x6A09E667u, 0xBB67AE85u, 0x3C6EF372u, 0xA54FF53Au,
                            0x510E527Fu, 0x9B05688Cu, 0x1F83D9ABu, 0x5BE0CD19u};
constexpr int PERM[16] = {2, 6, 3, 10, 7, 0, 4, 13, 1, 11, 12, 5, 9, 14, 15, 8};
constexpr uint32_t CHUNK_START = 1, CHUNK_END = 2, PARENT = 4, ROOT = 8;
constexpr size_t BLOCK = 64, CHUNK = 1024;

inline uint32_t rotr(uint32_t x, int n) { return (x >> n) | (x << (32 - n)); }

inline void g(uint32_t* s, int a, int b, int c, int d, uint32_t mx, uint32_t my) {
  s[a] = s[a] + s[b] + mx;
  s[d] = rotr(s[d] ^ s[a], 16);
  s[c] = s[c] + s[d];
  s[b] = rotr(s[b] ^ s[c], 12);
  s[a] = s[a] + s[b] + my;
  s[d] = rotr(s[d] ^ s[a], 8);
  s[c] = s[c] + s[d];
  s[b] = rotr(s[b] ^ s[c], 7);
}

// The full 16-word output of one compression.
void compress(const uint32_t cv[8], const uint32_t block[16], uint64_t counter, uint32_t len, uint32_t flags,
              uint32_t out[16]) {
  uint32_t s[16] = {cv[0], cv[1], cv[2], cv[3], cv[4], cv[5], cv[6], cv[7],
                    IV[0], IV[1], IV[2], IV[3], (uint32_t)counter, (uint32_t)(counter >> 32), len, flags};
  uint32_t m[16];
  std::memcpy(m, block, sizeof(m));
  for (int r = 0; r < 7; ++r) {
    g(s, 0, 4, 8, 12, m[0], m[1]);
    g(s, 1, 5, 9, 13, m[2], m[3]);
    g(s, 2, 6, 10, 14, m[4], m[5]);
    g(s, 3, 7, 11, 15, m[6], m[7]);
    g(s, 0, 5, 10, 15, m[8], m[9]);
    g(s, 1, 6, 11, 12, m[10], m[11]);
    g(s, 2, 7, 8, 13, m[12], m[13]);
    g(s, 3, 4, 9, 14, m[14], m[15]);
    uint32_t p[16];
    for (int i = 0; i < 16; ++i) p[i] = m[PERM[i]];
    std::memcpy(m, p, sizeof(m));
  }
  for (int i = 0; i < 8; ++i) {
    out[i] = s[i] ^ s[i + 8];
    out[i + 8] = s[i + 8] ^ cv[i];
  }
}

void load_block(const uint8_t* p, size_t n, uint32_t w[16]) {
  uint8_t buf[BLOCK] = {0};
  std::memcpy(buf, p, n);
  for (int i = 0; i < 16; ++i)
    w[i] = (uint32_t)buf[4 * i] | ((uint32_t)buf[4 * i + 1] << 8) | ((uint32_t)buf[4 * i + 2] << 16) |
           ((uint32_t)buf[4 * i + 3] << 24);
}

// A compression not yet performed: the root one needs the ROOT flag added.
struct Output {
  uint32_t cv[8], block[16];
  uint64_t counter;
  uint32_t len, flags;
  void chaining(uint32_t out8[8]) const {
    uint32_t o[16];
    compress(cv, block, counter, len, flags, o);
    std::memcpy(out8, o, 32);
  }
};

// The last block of a chunk (its earlier blocks folded into cv).
Output chunk_output(const uint8_t* p, size_t n, uint64_t index) {
  uint32_t cv[8];
  std::memcpy(cv, IV, sizeof(cv));
  size_t nblocks = n == 0 ? 1 : (n + BLOCK - 1) / BLOCK;
  for (size_t b = 0; b + 1 < nblocks; ++b) {
    uint32_t w[16], o[16];
    load_block(p + b * BLOCK, BLOCK, w);
    compress(cv, w, index, BLOCK, b == 0 ? CHUNK_START : 0, o);
    std::memcpy(cv, o, 32);
  }
  Output out;
  std::memcpy(out.cv, cv, sizeof(cv));
  const size_t last = (nblocks - 1) * BLOCK;
  load_block(p + last, n - last, out.block);
  out.counter = index;
  out.len = (uint32_t)(n - last);
  out.flags = CHUNK_END | (nblocks == 1 ? CHUNK_START : 0);
  return out;
}

Output parent_output(const uint32_t left[8], const uint32_t right[8]) {
  Output o;
  std::memcpy(o.cv, IV, sizeof(o.cv));
  std::memcpy(o.block, left, 32);
  std::memcpy(o.block + 8, right, 32);
  o.counter = 0;
  o.len = BLOCK;
  o.flags = PARENT;
  return o;
}

}  // namespace

std::string blake3_hash(const std::string& data) {
  const uint8_t* p = reinterpret_cast<const uint8_t*>(data.data());
  const size_t n = data.size();
  const uint64_t nchunks = n == 0 ? 1 : (n + CHUNK - 1) / CHUNK;
  std::vector<std::vector<uint32_t>> stack;  // chaining values of complete left subtrees
  for (uint64_t c = 0; c + 1 < nchunks; ++c) {
    std::vector<uint32_t> cv(8);
    chunk_output(p + c * CHUNK, CHUNK, c).chaining(cv.data());
    uint64_t total = c + 1;  // merge as many subtrees as complete chunk counts allow
    while ((total & 1) == 0) {
      std::vector<uint32_t> merged(8);
      parent_output(stack.back().data(), cv.data()).chaining(merged.data());
      stack.pop_back();
      cv = merged;
      total >>= 1;
    }
    stack.push_back(cv);
  }
  const uint64_t lastc = nchunks - 1;
  Output out = chunk_output(p + lastc * CHUNK, n - lastc * CHUNK, lastc);
  while (!stack.empty()) {
    uint32_t right[8];
    out.chaining(right);
    out = parent_output(stack.back().data(), right);
    stack.pop_back();
  }
  uint32_t o[16];
  compress(out.cv, out.block, out.counter, out.len, out.flags | ROOT, o);
  std::string digest(32, '\0');
  for (int i = 0; i < 8; ++i)
    for (int b = 0; b < 4; ++b) digest[4 * i + b] = (char)((o[i] >> (8 * b)) & 0xff);
  return digest;
}

void register_blake3(pybind11::module& m) {
  m.def("blake3", [](pybind11::bytes b) { return pybind11::bytes(blake3_hash(std::string(b))); },
        "BLAKE3 of the bytes (32-byte digest)");
}

}  // namespace syn
