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
//
// Collective extension (one member's part of a group reduction or gather), 64 bytes:
//   0 phase u8 (1 attention all-reduce, 2 FFN all-reduce, 3 exit gather, 4 logits gather)
//   1 dtype u8 (1 f32, 2 bf16)   2 member u16   4 n_members u16   8 layer u32   12 n_rows u32
//   16 width u32 (elements per row)   20 row_offset u32 (first row of the part)   24 epoch u32
// Payload: n_rows rows of width elements at a 64-byte stride.
// EP dispatch extension (rows sent to the owner of some of their experts): 64-byte fixed part
//   0 src_rank u16   2 dst_rank u16   4 dtype u8   5 top_k u8   8 layer u32   12 n_rows u32
//   16 hidden u32   20 epoch u32
// then n_rows route records of 8 + 8 * top_k bytes padded to 16 (0 source row u32, 4 n_routes u16;
// then per route: expert u16, 2 reserved, weight f32), zero-padded to 64; payload: the rows.
// EP combine extension (the owner's weighted sum over its experts, per row, back to the source):
//   64-byte fixed part (0 src_rank u16, 2 dst_rank u16, 8 layer u32, 12 n_rows u32, 16 hidden
//   u32, 20 epoch u32), then the n_rows source rows as u32, zero-padded to 64; payload: f32 rows.
#pragma once
#include <cstdint>
#include <cstring>
#include <string>
#include <vector>

#include "syn/frame.h"

namespace syn {

constexpr uint8_t FRAME_ACTIVATION = 1;
constexpr uint8_t FRAME_TOKEN = 2;
// frame type codes of the header (the channel's table: 3 sequence control, 4 credit, 5 KV chunk,
// 9 step descriptor, 0x0A-0x0C hello / ack / close, 0x10 ping)
constexpr uint8_t FRAME_COLLECTIVE = 0x08;
constexpr uint8_t FRAME_EP_DISPATCH = 0x0E;
constexpr uint8_t FRAME_EP_COMBINE = 0x0F;

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


// ---- rows at a 64-byte stride (Collective, EP dispatch, EP combine payloads) ----
inline size_t rows_stride(size_t row_bytes) { return (row_bytes + 63) / 64 * 64; }
inline std::vector<uint8_t> rows_pack(const uint8_t* rows, uint32_t n, size_t row_bytes) {
  const size_t st = rows_stride(row_bytes);
  std::vector<uint8_t> pay(st * n, 0);
  for (uint32_t r = 0; r < n; ++r) memcpy(pay.data() + r * st, rows + r * row_bytes, row_bytes);
  return pay;
}
inline void rows_unpack(const uint8_t* pay, uint32_t n, size_t row_bytes, std::vector<uint8_t>* out) {
  const size_t st = rows_stride(row_bytes);
  out->assign(row_bytes * n, 0);
  for (uint32_t r = 0; r < n; ++r) memcpy(out->data() + r * row_bytes, pay + r * st, row_bytes);
}
inline std::string frame_with(const FrameSpec& fs, uint8_t type, const std::vector<uint8_t>& ext,
                              const std::vector<uint8_t>& pay) {
  FrameSpec s = fs;
  s.ftype = type;
  std::string out(frame_len(ext.size(), pay.size()), '\0');
  frame_encode(s, ext.data(), ext.size(), pay.data(), pay.size(), reinterpret_cast<uint8_t*>(&out[0]));
  return out;
}

struct CollectiveHeader {
  uint8_t phase = 1, dtype = 1;
  uint16_t member = 0, n_members = 1;
  uint32_t layer = 0, n_rows = 0, width = 0, row_offset = 0, epoch = 0;
};

inline std::string collective_encode(const FrameSpec& fs, const CollectiveHeader& h, const uint8_t* rows) {
  std::vector<uint8_t> ext(64, 0);
  uint8_t* f = ext.data();
  f[0] = h.phase;
  f[1] = h.dtype;
  put_le<uint16_t>(f + 2, h.member);
  put_le<uint16_t>(f + 4, h.n_members);
  put_le<uint32_t>(f + 8, h.layer);
  put_le<uint32_t>(f + 12, h.n_rows);
  put_le<uint32_t>(f + 16, h.width);
  put_le<uint32_t>(f + 20, h.row_offset);
  put_le<uint32_t>(f + 24, h.epoch);
  return frame_with(fs, FRAME_COLLECTIVE, ext, rows_pack(rows, h.n_rows, (size_t)h.width * act_elem_bytes(h.dtype)));
}

inline int collective_decode(const uint8_t* buf, size_t n, FrameSpec* fs, CollectiveHeader* h,
                             std::vector<uint8_t>* rows_out) {
  size_t eo, el, po, pl;
  const int rc = frame_decode(buf, n, fs, &eo, &el, &po, &pl);
  if (rc != FRAME_OK) return rc;
  if (fs->ftype != FRAME_COLLECTIVE) return PAYLOAD_BAD_TYPE;
  if (el < 64) return PAYLOAD_BAD_LENGTH;
  const uint8_t* f = buf + eo;
  h->phase = f[0];
  h->dtype = f[1];
  h->member = get_le<uint16_t>(f + 2);
  h->n_members = get_le<uint16_t>(f + 4);
  h->layer = get_le<uint32_t>(f + 8);
  h->n_rows = get_le<uint32_t>(f + 12);
  h->width = get_le<uint32_t>(f + 16);
  h->row_offset = get_le<uint32_t>(f + 20);
  h->epoch = get_le<uint32_t>(f + 24);
  if (act_elem_bytes(h->dtype) == 0) return PAYLOAD_BAD_DTYPE;
  if (h->n_members == 0 || h->member >= h->n_members) return PAYLOAD_BAD_SPAN;
  const size_t rb = (size_t)h->width * act_elem_bytes(h->dtype);
  if (pl != rows_stride(rb) * h->n_rows) return PAYLOAD_BAD_LENGTH;
  rows_unpack(buf + po, h->n_rows, rb, rows_out);
  return PAYLOAD_OK;
}

struct EpRoute {
  uint32_t row = 0;                    // the row's index at the source rank
  std::vector<uint16_t> experts;       // this owner's experts for the row (<= top_k)
  std::vector<float> weights;          // their routing weights
};
struct EpHeader {
  uint16_t src_rank = 0, dst_rank = 0;
  uint8_t dtype = 2, top_k = 1;
  uint32_t layer = 0, n_rows = 0, hidden = 0, epoch = 0;
};
inline size_t ep_record_bytes(uint8_t top_k) { return (8 + 8 * (size_t)top_k + 15) / 16 * 16; }
inline void ep_put_fixed(uint8_t* f, const EpHeader& h) {
  put_le<uint16_t>(f + 0, h.src_rank);
  put_le<uint16_t>(f + 2, h.dst_rank);
  f[4] = h.dtype;
  f[5] = h.top_k;
  put_le<uint32_t>(f + 8, h.layer);
  put_le<uint32_t>(f + 12, h.n_rows);
  put_le<uint32_t>(f + 16, h.hidden);
  put_le<uint32_t>(f + 20, h.epoch);
}
inline void ep_get_fixed(const uint8_t* f, EpHeader* h) {
  h->src_rank = get_le<uint16_t>(f + 0);
  h->dst_rank = get_le<uint16_t>(f + 2);
  h->dtype = f[4];
  h->top_k = f[5];
  h->layer = get_le<uint32_t>(f + 8);
  h->n_rows = get_le<uint32_t>(f + 12);
  h->hidden = get_le<uint32_t>(f + 16);
  h->epoch = get_le<uint32_t>(f + 20);
}

inline std::string ep_dispatch_encode(const FrameSpec& fs, const EpHeader& h, const std::vector<EpRoute>& routes,
                                      const uint8_t* rows) {
  const size_t rec = ep_record_bytes(h.top_k);
  std::vector<uint8_t> ext((64 + rec * routes.size() + 63) / 64 * 64, 0);
  ep_put_fixed(ext.data(), h);
  for (size_t i = 0; i < routes.size(); ++i) {
    uint8_t* r = ext.data() + 64 + rec * i;
    put_le<uint32_t>(r + 0, routes[i].row);
    put_le<uint16_t>(r + 4, (uint16_t)routes[i].experts.size());
    for (size_t j = 0; j < routes[i].experts.size(); ++j) {
      put_le<uint16_t>(r + 8 + 8 * j, routes[i].experts[j]);
      float w = routes[i].weights[j];
      uint32_t wb;
      memcpy(&wb, &w, 4);
      put_le<uint32_t>(r + 8 + 8 * j + 4, wb);
    }
  }
  return frame_with(fs, FRAME_EP_DISPATCH, ext, rows_pack(rows, h.n_rows, (size_t)h.hidden * act_elem_bytes(h.dtype)));
}

inline int ep_dispatch_decode(const uint8_t* buf, size_t n, FrameSpec* fs, EpHeader* h, std::vector<EpRoute>* routes,
                              std::vector<uint8_t>* rows_out) {
  size_t eo, el, po, pl;
  const int rc = frame_decode(buf, n, fs, &eo, &el, &po, &pl);
  if (rc != FRAME_OK) return rc;
  if (fs->ftype != FRAME_EP_DISPATCH) return PAYLOAD_BAD_TYPE;
  if (el < 64) return PAYLOAD_BAD_LENGTH;
  ep_get_fixed(buf + eo, h);
  if (act_elem_bytes(h->dtype) == 0) return PAYLOAD_BAD_DTYPE;
  const size_t rec = ep_record_bytes(h->top_k);
  if (h->top_k == 0 || 64 + rec * (size_t)h->n_rows > el) return PAYLOAD_BAD_LENGTH;
  const size_t rb = (size_t)h->hidden * act_elem_bytes(h->dtype);
  if (pl != rows_stride(rb) * h->n_rows) return PAYLOAD_BAD_LENGTH;
  routes->clear();
  for (uint32_t i = 0; i < h->n_rows; ++i) {
    const uint8_t* r = buf + eo + 64 + rec * i;
    EpRoute e;
    e.row = get_le<uint32_t>(r + 0);
    const uint16_t nr = get_le<uint16_t>(r + 4);
    if (nr == 0 || nr > h->top_k) return PAYLOAD_BAD_SPAN;
    for (uint16_t j = 0; j < nr; ++j) {
      e.experts.push_back(get_le<uint16_t>(r + 8 + 8 * j));
      const uint32_t wb = get_le<uint32_t>(r + 8 + 8 * j + 4);
      float w;
      memcpy(&w, &wb, 4);
      e.weights.push_back(w);
    }
    routes->push_back(std::move(e));
  }
  rows_unpack(buf + po, h->n_rows, rb, rows_out);
  return PAYLOAD_OK;
}

// EP combine: f32 rows (dtype is always 1); row_ids: the source rows they answer.
inline std::string ep_combine_encode(const FrameSpec& fs, const EpHeader& h, const std::vector<uint32_t>& row_ids,
                                     const uint8_t* rows) {
  std::vector<uint8_t> ext((64 + 4 * row_ids.size() + 63) / 64 * 64, 0);
  EpHeader c = h;
  c.dtype = 1;
  c.top_k = 0;
  ep_put_fixed(ext.data(), c);
  for (size_t i = 0; i < row_ids.size(); ++i) put_le<uint32_t>(ext.data() + 64 + 4 * i, row_ids[i]);
  return frame_with(fs, FRAME_EP_COMBINE, ext, rows_pack(rows, h.n_rows, (size_t)h.hidden * 4));
}

inline int ep_combine_decode(const uint8_t* buf, size_t n, FrameSpec* fs, EpHeader* h,
                             std::vector<uint32_t>* row_ids, std::vector<uint8_t>* rows_out) {
  size_t eo, el, po, pl;
  const int rc = frame_decode(buf, n, fs, &eo, &el, &po, &pl);
  if (rc != FRAME_OK) return rc;
  if (fs->ftype != FRAME_EP_COMBINE) return PAYLOAD_BAD_TYPE;
  if (el < 64) return PAYLOAD_BAD_LENGTH;
  ep_get_fixed(buf + eo, h);
  if (h->dtype != 1) return PAYLOAD_BAD_DTYPE;
  if (64 + 4 * (size_t)h->n_rows > el) return PAYLOAD_BAD_LENGTH;
  const size_t rb = (size_t)h->hidden * 4;
  if (pl != rows_stride(rb) * h->n_rows) return PAYLOAD_BAD_LENGTH;
  row_ids->clear();
  for (uint32_t i = 0; i < h->n_rows; ++i) row_ids->push_back(get_le<uint32_t>(buf + eo + 64 + 4 * i));
  rows_unpack(buf + po, h->n_rows, rb, rows_out);
  return PAYLOAD_OK;
}

}  // namespace syn
