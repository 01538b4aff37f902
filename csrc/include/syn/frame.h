// Data-plane frame header: 64 bytes, little-endian, the same byte layout as the reference
// wire format (crates/net/src/frame/header.rs; RFC-0031 §6.1) so frames interoperate:
//   0..4   magic "SYNF"           4      wire minor       5      frame type
//   6..8   flags                  8..16  instance id      16..24 epoch term
//   24..32 epoch seq              32..40 step             40..48 channel seq
//   48..52 extension length (multiple of 64)              52..56 payload length
//   56..60 CRC32C(payload)        60..64 CRC32C(header[0..60] ++ extension)
// The extension is zero-padded so the payload starts 64-byte aligned.
#pragma once
#include <cstddef>
#include <cstdint>
#include <cstring>

namespace syn {

// CRC32C (Castagnoli, reflected polynomial 0x82F63B78), table-driven.
struct Crc32c {
  uint32_t table[256];
  Crc32c() {
    for (uint32_t i = 0; i < 256; ++i) {
      uint32_t c = i;
      for (int k = 0; k < 8; ++k) c = (c & 1u) ? (0x82F63B78u ^ (c >> 1)) : (c >> 1);
      table[i] = c;
    }
  }
  // Continue a CRC: pass the previous result (0 to start).
  uint32_t update(uint32_t crc, const uint8_t* p, size_t n) const {
    uint32_t c = ~crc;
    for (size_t i = 0; i < n; ++i) c = table[(c ^ p[i]) & 0xFFu] ^ (c >> 8);
    return ~c;
  }
};

inline const Crc32c& crc32c_table() {
  static Crc32c t;
  return t;
}
inline uint32_t crc32c(const uint8_t* p, size_t n, uint32_t prev = 0) { return crc32c_table().update(prev, p, n); }

constexpr size_t kFrameHeader = 64;
constexpr uint8_t kWireMinor = 1;

struct FrameSpec {
  uint8_t wire_minor = kWireMinor;
  uint8_t ftype = 0;
  uint16_t flags = 0;
  uint64_t instance = 0;
  uint64_t epoch_term = 0;
  uint64_t epoch_seq = 0;
  uint64_t step = 0;
  uint64_t chan_seq = 0;
};

inline size_t frame_len(size_t ext, size_t payload) { return kFrameHeader + ((ext + 63) / 64) * 64 + payload; }

template <typename T>
inline void put_le(uint8_t* p, T v) {
  for (size_t i = 0; i < sizeof(T); ++i) p[i] = (uint8_t)(v >> (8 * i));
}
template <typename T>
inline T get_le(const uint8_t* p) {
  T v = 0;
  for (size_t i = 0; i < sizeof(T); ++i) v |= (T)p[i] << (8 * i);
  return v;
}

// Encodes into `out` (frame_len() bytes); returns the length.
inline size_t frame_encode(const FrameSpec& s, const uint8_t* ext, size_t ext_n, const uint8_t* payload,
                           size_t pay_n, uint8_t* out) {
  const size_t ext_len = ((ext_n + 63) / 64) * 64;
  memset(out, 0, kFrameHeader);
  if (ext_n) memcpy(out + kFrameHeader, ext, ext_n);
  memset(out + kFrameHeader + ext_n, 0, ext_len - ext_n);
  if (pay_n) memcpy(out + kFrameHeader + ext_len, payload, pay_n);
  uint8_t* h = out;
  memcpy(h, "SYNF", 4);
  h[4] = s.wire_minor;
  h[5] = s.ftype;
  put_le<uint16_t>(h + 6, s.flags);
  put_le<uint64_t>(h + 8, s.instance);
  put_le<uint64_t>(h + 16, s.epoch_term);
  put_le<uint64_t>(h + 24, s.epoch_seq);
  put_le<uint64_t>(h + 32, s.step);
  put_le<uint64_t>(h + 40, s.chan_seq);
  put_le<uint32_t>(h + 48, (uint32_t)ext_len);
  put_le<uint32_t>(h + 52, (uint32_t)pay_n);
  const uint32_t pcrc = pay_n ? crc32c(out + kFrameHeader + ext_len, pay_n) : 0u;
  put_le<uint32_t>(h + 56, pcrc);
  uint32_t hcrc = crc32c(h, 60);
  hcrc = crc32c(out + kFrameHeader, ext_len, hcrc);
  put_le<uint32_t>(h + 60, hcrc);
  return kFrameHeader + ext_len + pay_n;
}

enum FrameError : int {
  FRAME_OK = 0,
  FRAME_SHORT = 1,
  FRAME_BAD_MAGIC = 2,
  FRAME_BAD_HEADER_CRC = 3,
  FRAME_BAD_PAYLOAD_CRC = 4,
  FRAME_BAD_EXT_ALIGN = 5,
};

// Decodes and verifies a frame at the start of buf; on success fills spec, offsets, lengths.
inline int frame_decode(const uint8_t* buf, size_t n, FrameSpec* s, size_t* ext_off, size_t* ext_len,
                        size_t* pay_off, size_t* pay_len) {
  if (n < kFrameHeader) return FRAME_SHORT;
  if (memcmp(buf, "SYNF", 4) != 0) return FRAME_BAD_MAGIC;
  const uint32_t el = get_le<uint32_t>(buf + 48), pl = get_le<uint32_t>(buf + 52);
  if (el % 64 != 0) return FRAME_BAD_EXT_ALIGN;
  if (n < kFrameHeader + (size_t)el + pl) return FRAME_SHORT;
  uint32_t hcrc = crc32c(buf, 60);
  hcrc = crc32c(buf + kFrameHeader, el, hcrc);
  if (hcrc != get_le<uint32_t>(buf + 60)) return FRAME_BAD_HEADER_CRC;
  const uint32_t pcrc = pl ? crc32c(buf + kFrameHeader + el, pl) : 0u;
  if (pcrc != get_le<uint32_t>(buf + 56)) return FRAME_BAD_PAYLOAD_CRC;
  s->wire_minor = buf[4];
  s->ftype = buf[5];
  s->flags = get_le<uint16_t>(buf + 6);
  s->instance = get_le<uint64_t>(buf + 8);
  s->epoch_term = get_le<uint64_t>(buf + 16);
  s->epoch_seq = get_le<uint64_t>(buf + 24);
  s->step = get_le<uint64_t>(buf + 32);
  s->chan_seq = get_le<uint64_t>(buf + 40);
  *ext_off = kFrameHeader;
  *ext_len = el;
  *pay_off = kFrameHeader + el;
  *pay_len = pl;
  return FRAME_OK;
}

}  // namespace syn
