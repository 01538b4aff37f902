// Data-plane payload codecs on top of the 64-byte frame header (syn/frame.h): the Activation
// frame (hidden-state rows handed from one pipeline stage to the next) and the Token frame
// (sampled tokens returned to the ingress).  Reference semantics: crates/net/src/frame/
// activation.rs:82-482 (kind, spans of sequences, rows of `streams x hidden` elements with a
// 64-byte row stride, chunks split into parts at row boundaries) and crates/net/src/frame/
// token.rs (tokens per sequence with a finish flag).  The frame header is byte-compatible with
// the reference's; these extension and payload layouts are this framework's own.
//
// Activation extension: 64-byte fixed part, then n_spans x 32-byte spans, zero-padded to 64:
//   fixed  0 from_stage u16   2 to_stage u16    4 kind u8 (1 prefill, 2 decode, 3 verify,
//          5 dtype u8 (1 f32, 2 bf16)   6 streams u8   4 replay, 5 canary)
//          8 hidden u32      12 n_rows u32     16 n_spans u16   18 part_index u16
//         20 part_count u16  24 kind_arg u32   28 kind_flags u32   (the rest reserved, zero)
//   span   0 sequence id u64  8 first_position u32  12 n_positions u32  16 row_offset u32
// Payload: n_rows rows of streams * hidden elements, each row padded to a 64-byte stride.
//
// Token extension: 64-byte fixed part (0 n_entries u32, 4 total_tokens u32), then 16-byte
// entries (0 sequence id u64, 8 n_tokens u32, 12 flags u16: bit 0 finished, bits 8..15 finish
// reason code); payload: every entry's tokens as u32, in entry order.
#pragma once
#include <cstdint>
#include <cstring>
#include <string>
#include <vector>

#include "syn/frame.h"

namespace syn {

constexpr uint8_t FRAME_ACTIVATION = 1;
constexpr uint8_t FRAME_TOKEN = 2;

enum PayloadError : int {
  PAYLOAD_OK = 0,
  PAYLOAD_BAD_TYPE = 10,
  PAYLOAD_BAD_DTYPE = 11,
  PAYLOAD_BAD_LENGTH = 12,
  PAYLOAD_BAD_SPAN = 13,
};

struct ActivationHeader {
  uint16_t from_stage = 0, to_stage = 0;
  uint8_t kind = 2, dtype = 2, streams = 1;
  uint32_t hidden = 0, n_rows = 0;
  uint16_t part_index = 0, part_count = 1;
  uint32_t kind_arg = 0, kind_flags = 0;
};

struct ActivationSpan {
  uint64_t seq = 0;
  uint32_t first_position = 0, n_positions = 0, row_offset = 0;
};

inline size_t act_elem_bytes(uint8_t dtype) { return dtype == 1 ? 4 : dtype == 2 ? 2 : 0; }
inline size_t act_row_stride(const ActivationHeader& h) {
  const size_t row = (size_t)h.streams * h.hidden * act_elem_bytes(h.dtype);
  return (row + 63) / 64 * 64;
}

// Encodes a full frame; rows holds n_rows dense rows of streams * hidden elements.
inline std::string activation_encode(const FrameSpec& fs, const ActivationHeader& h,
                                     const std::vector<ActivationSpan>& spans, const uint8_t* rows) {
  std::vector<uint8_t> ext(64 + 32 * spans.size(), 0);
  uint8_t* f = ext.data();
  put_le<uint16_t>(f + 0, h.from_stage);
  put_le<uint16_t>(f + 2, h.to_stage);
  f[4] = h.kind;
  f[5] = h.dtype;
  f[6] = h.streams;
  put_le<uint32_t>(f + 8, h.hidden);
  put_le<uint32_t>(f + 12, h.n_rows);
  put_le<uint16_t>(f + 16, (uint16_t)spans.size());
  put_le<uint16_t>(f + 18, h.part_index);
  put_le<uint16_t>(f + 20, h.part_count);
  put_le<uint32_t>(f + 24, h.kind_arg);
  put_le<uint32_t>(f + 28, h.kind_flags);
  for (size_t i = 0; i < spans.size(); ++i) {
    uint8_t* s = f + 64 + 32 * i;
    put_le<uint64_t>(s + 0, spans[i].seq);
    put_le<uint32_t>(s + 8, spans[i].first_position);
    put_le<uint32_t>(s + 12, spans[i].n_positions);
    put_le<uint32_t>(s + 16, spans[i].row_offset);
  }
  const size_t row = (size_t)h.streams * h.hidden * act_elem_bytes(h.dtype), stride = act_row_stride(h);
  std::vector<uint8_t> pay(stride * h.n_rows, 0);
  for (uint32_t r = 0; r < h.n_rows; ++r) memcpy(pay.data() + r * stride, rows + r * row, row);
  FrameSpec s = fs;
  s.ftype = FRAME_ACTIVATION;
  std::string out(frame_len(ext.size(), pay.size()), '\0');
  frame_encode(s, ext.data(), ext.size(), pay.data(), pay.size(), reinterpret_cast<uint8_t*>(&out[0]));
  return out;
}

// Decodes and checks a frame; rows_out receives n_rows dense rows (strides removed).
inline int activation_decode(const uint8_t* buf, size_t n, FrameSpec* fs, ActivationHeader* h,
                             std::vector<ActivationSpan>* spans, std::vector<uint8_t>* rows_out) {
  size_t eo, el, po, pl;
  const int rc = frame_decode(buf, n, fs, &eo, &el, &po, &pl);
  if (rc != FRAME_OK) return rc;
  if (fs->ftype != FRAME_ACTIVATION) return PAYLOAD_BAD_TYPE;
  if (el < 64) return PAYLOAD_BAD_LENGTH;
  const uint8_t* f = buf + eo;
  h->from_stage = get_le<uint16_t>(f + 0);
  h->to_stage = get_le<uint16_t>(f + 2);
  h->kind = f[4];
  h->dtype = f[5];
  h->streams = f[6];
  h->hidden = get_le<uint32_t>(f + 8);
  h->n_rows = get_le<uint32_t>(f + 12);
  const uint16_t n_spans = get_le<uint16_t>(f + 16);
  h->part_index = get_le<uint16_t>(f + 18);
  h->part_count = get_le<uint16_t>(f + 20);
  h->kind_arg = get_le<uint32_t>(f + 24);
  h->kind_flags = get_le<uint32_t>(f + 28);
  if (act_elem_bytes(h->dtype) == 0) return PAYLOAD_BAD_DTYPE;
  if (64 + 32 * (size_t)n_spans > el) return PAYLOAD_BAD_LENGTH;
  const size_t row = (size_t)h->streams * h->hidden * act_elem_bytes(h->dtype), stride = act_row_stride(*h);
  if (pl != stride * h->n_rows) return PAYLOAD_BAD_LENGTH;
  spans->clear();
  for (uint16_t i = 0; i < n_spans; ++i) {
    const uint8_t* s = f + 64 + 32 * i;
    ActivationSpan sp;
    sp.seq = get_le<uint64_t>(s + 0);
    sp.first_position = get_le<uint32_t>(s + 8);
    sp.n_positions = get_le<uint32_t>(s + 12);
    sp.row_offset = get_le<uint32_t>(s + 16);
    if ((uint64_t)sp.row_offset + sp.n_positions > h->n_rows) return PAYLOAD_BAD_SPAN;
    spans->push_back(sp);
  }
  rows_out->assign(row * h->n_rows, 0);
  for (uint32_t r = 0; r < h->n_rows; ++r) memcpy(rows_out->data() + r * row, buf + po + r * stride, row);
  return PAYLOAD_OK;
}

struct TokenEntry {
  uint64_t seq = 0;
  uint16_t flags = 0;  // bit 0 finished; bits 8..15 finish reason code
  std::vector<uint32_t> tokens;
};

inline std::string token_encode(const FrameSpec& fs, const std::vector<TokenEntry>& entries) {
  std::vector<uint8_t> ext(64 + 16 * entries.size(), 0);
  uint32_t total = 0;
  for (size_t i = 0; i < entries.size(); ++i) {
    uint8_t* e = ext.data() + 64 + 16 * i;
    put_le<uint64_t>(e + 0, entries[i].seq);
    put_le<uint32_t>(e + 8, (uint32_t)entries[i].tokens.size());
    put_le<uint16_t>(e + 12, entries[i].flags);
    total += (uint32_t)entries[i].tokens.size();
  }
  put_le<uint32_t>(ext.data() + 0, (uint32_t)entries.size());
  put_le<uint32_t>(ext.data() + 4, total);
  std::vector<uint8_t> pay(4 * (size_t)total);
  size_t o = 0;
  for (const auto& e : entries)
    for (uint32_t t : e.tokens) {
      put_le<uint32_t>(pay.data() + o, t);
      o += 4;
    }
  FrameSpec s = fs;
  s.ftype = FRAME_TOKEN;
  std::string out(frame_len(ext.size(), pay.size()), '\0');
  frame_encode(s, ext.data(), ext.size(), pay.data(), pay.size(), reinterpret_cast<uint8_t*>(&out[0]));
  return out;
}

inline int token_decode(const uint8_t* buf, size_t n, FrameSpec* fs, std::vector<TokenEntry>* entries) {
  size_t eo, el, po, pl;
  const int rc = frame_decode(buf, n, fs, &eo, &el, &po, &pl);
  if (rc != FRAME_OK) return rc;
  if (fs->ftype != FRAME_TOKEN) return PAYLOAD_BAD_TYPE;
  if (el < 64) return PAYLOAD_BAD_LENGTH;
  const uint32_t ne = get_le<uint32_t>(buf + eo), total = get_le<uint32_t>(buf + eo + 4);
  if (64 + 16 * (size_t)ne > el || pl != 4 * (size_t)total) return PAYLOAD_BAD_LENGTH;
  entries->clear();
  size_t o = 0;
  for (uint32_t i = 0; i < ne; ++i) {
    const uint8_t* e = buf + eo + 64 + 16 * i;
    TokenEntry t;
    t.seq = get_le<uint64_t>(e + 0);
    const uint32_t nt = get_le<uint32_t>(e + 8);
    t.flags = get_le<uint16_t>(e + 12);
    if (o + 4 * (size_t)nt > pl) return PAYLOAD_BAD_LENGTH;
    for (uint32_t k = 0; k < nt; ++k) t.tokens.push_back(get_le<uint32_t>(buf + po + o + 4 * k));
    o += 4 * (size_t)nt;
    entries->push_back(std::move(t));
  }
  return o == pl ? PAYLOAD_OK : PAYLOAD_BAD_LENGTH;
}

}  // namespace syn
