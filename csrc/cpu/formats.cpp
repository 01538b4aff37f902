// Model-file header parsers: safetensors (8-byte length + JSON header) and GGUF (v2/v3
// binary metadata + tensor infos).  Both read only the header bytes (range reads); tensor
// data is mapped or streamed separately.  Reference: crates/manifest/src/{safetensors.rs:
// 143-235, gguf.rs:75-335}.
#include <torch/extension.h>

#include <cstdio>
#include <cstring>
#include <fstream>
#include <map>
#include <stdexcept>
#include <string>
#include <vector>

namespace py = pybind11;

namespace syn {

// ------------------------------------------------------------------ minimal JSON
struct JVal {
  enum T { NUL, BOOL, NUM, STR, ARR, OBJ } t = NUL;
  bool b = false;
  double n = 0;
  std::string s;
  std::vector<JVal> a;
  std::vector<std::pair<std::string, JVal>> o;
  const JVal* get(const std::string& k) const {
    for (auto& kv : o)
      if (kv.first == k) return &kv.second;
    return nullptr;
  }
};

class JParser {
 public:
  explicit JParser(const std::string& s) : s_(s) {}
  JVal parse() {
    JVal v = value();
    ws();
    if (i_ != s_.size()) fail("trailing bytes");
    return v;
  }

 private:
  const std::string& s_;
  size_t i_ = 0;
  [[noreturn]] void fail(const char* m) { throw std::runtime_error(std::string("JSON: ") + m + " at " + std::to_string(i_)); }
  void ws() {
    while (i_ < s_.size() && (s_[i_] == ' ' || s_[i_] == '\n' || s_[i_] == '\r' || s_[i_] == '\t')) ++i_;
  }
  char peek() {
    ws();
    if (i_ >= s_.size()) fail("unexpected end");
    return s_[i_];
  }
  JVal value() {
    const char c = peek();
    if (c == '{') return object();
    if (c == '[') return array();
    if (c == '"') {
      JVal v;
      v.t = JVal::STR;
      v.s = str();
      return v;
    }
    if (c == 't' || c == 'f') {
      JVal v;
      v.t = JVal::BOOL;
      if (s_.compare(i_, 4, "true") == 0) { v.b = true; i_ += 4; }
      else if (s_.compare(i_, 5, "false") == 0) { i_ += 5; }
      else fail("bad literal");
      return v;
    }
    if (c == 'n') {
      if (s_.compare(i_, 4, "null") != 0) fail("bad literal");
      i_ += 4;
      return JVal();
    }
    JVal v;
    v.t = JVal::NUM;
    size_t end;
    v.n = std::stod(s_.substr(i_, 64), &end);
    i_ += end;
    return v;
  }
  std::string str() {
    if (s_[i_] != '"') fail("expected string");
    ++i_;
    std::string out;
    while (i_ < s_.size() && s_[i_] != '"') {
      if (s_[i_] == '\\') {
        ++i_;
        if (i_ >= s_.size()) fail("bad escape");
        const char e = s_[i_];
        if (e == 'u') {
          out += '?';  // names in model headers are ASCII; keep the length sane
          i_ += 4;
        } else {
          out += (e == 'n' ? '\n' : e == 't' ? '\t' : e);
        }
        ++i_;
      } else {
        out += s_[i_++];
      }
    }
    if (i_ >= s_.size()) fail("unterminated string");
    ++i_;
    return out;
  }
  JVal array() {
    JVal v;
    v.t = JVal::ARR;
    ++i_;
    if (peek() == ']') { ++i_; return v; }
    for (;;) {
      v.a.push_back(value());
      const char c = peek();
      ++i_;
      if (c == ']') break;
      if (c != ',') fail("expected , or ]");
    }
    return v;
  }
  JVal object() {
    JVal v;
    v.t = JVal::OBJ;
    ++i_;
    if (peek() == '}') { ++i_; return v; }
    for (;;) {
      peek();
      std::string k = str();
      if (peek() != ':') fail("expected :");
      ++i_;
      v.o.emplace_back(k, value());
      const char c = peek();
      ++i_;
      if (c == '}') break;
      if (c != ',') fail("expected , or }");
    }
    return v;
  }
};

// Returns (header_len, [(name, dtype, shape, begin, end)], metadata dict).  Offsets are
// relative to the data section (which starts at 8 + header_len).
py::tuple safetensors_header(const std::string& path) {
  std::ifstream f(path, std::ios::binary);
  TORCH_CHECK(f.good(), "cannot open ", path);
  uint64_t n = 0;
  f.read(reinterpret_cast<char*>(&n), 8);
  TORCH_CHECK(f.good() && n > 0 && n < (1ull << 30), "bad safetensors header length in ", path);
  std::string hdr(n, '\0');
  f.read(&hdr[0], (std::streamsize)n);
  TORCH_CHECK(f.good(), "truncated safetensors header in ", path);
  JVal root;
  try {
    root = JParser(hdr).parse();
  } catch (const std::exception& e) {
    TORCH_CHECK(false, path, ": ", e.what());
  }
  TORCH_CHECK(root.t == JVal::OBJ, "safetensors header is not an object");
  py::list tensors;
  py::dict meta;
  for (auto& kv : root.o) {
    if (kv.first == "__metadata__") {
      for (auto& m : kv.second.o)
        if (m.second.t == JVal::STR) meta[py::str(m.first)] = m.second.s;
      continue;
    }
    const JVal* dt = kv.second.get("dtype");
    const JVal* sh = kv.second.get("shape");
    const JVal* off = kv.second.get("data_offsets");
    TORCH_CHECK(dt && sh && off && off->a.size() == 2, "tensor ", kv.first, ": missing fields");
    py::list shape;
    for (auto& d : sh->a) shape.append((int64_t)d.n);
    tensors.append(py::make_tuple(kv.first, dt->s, shape, (int64_t)off->a[0].n, (int64_t)off->a[1].n));
  }
  return py::make_tuple((int64_t)n, tensors, meta);
}

// ------------------------------------------------------------------ GGUF
class Reader {
 public:
  explicit Reader(const std::string& p) : f_(p, std::ios::binary) { TORCH_CHECK(f_.good(), "cannot open ", p); }
  template <typename T>
  T get() {
    T v;
    f_.read(reinterpret_cast<char*>(&v), sizeof(T));
    TORCH_CHECK(f_.good(), "truncated GGUF");
    return v;
  }
  std::string str() {
    const uint64_t n = get<uint64_t>();
    TORCH_CHECK(n < (1ull << 24), "GGUF string too long");
    std::string s(n, '\0');
    f_.read(&s[0], (std::streamsize)n);
    return s;
  }
  uint64_t tell() { return (uint64_t)f_.tellg(); }

 private:
  std::ifstream f_;
};

static py::object gguf_value(Reader& r, uint32_t type) {
  switch (type) {
    case 0: return py::int_(r.get<uint8_t>());
    case 1: return py::int_(r.get<int8_t>());
    case 2: return py::int_(r.get<uint16_t>());
    case 3: return py::int_(r.get<int16_t>());
    case 4: return py::int_(r.get<uint32_t>());
    case 5: return py::int_(r.get<int32_t>());
    case 6: return py::float_(r.get<float>());
    case 7: return py::bool_(r.get<uint8_t>() != 0);
    case 8: return py::str(r.str());
    case 9: {
      const uint32_t et = r.get<uint32_t>();
      const uint64_t n = r.get<uint64_t>();
      py::list l;
      for (uint64_t i = 0; i < n; ++i) l.append(gguf_value(r, et));
      return l;
    }
    case 10: return py::int_(r.get<uint64_t>());
    case 11: return py::int_(r.get<int64_t>());
    case 12: return py::float_(r.get<double>());
    default: TORCH_CHECK(false, "unknown GGUF value type ", type);
  }
}

// Returns (version, metadata dict, [(name, ggml_type, dims, offset)], data_offset).
py::tuple gguf_header(const std::string& path) {
  Reader r(path);
  const uint32_t magic = r.get<uint32_t>();
  TORCH_CHECK(magic == 0x46554747u, "not a GGUF file: ", path);  // "GGUF"
  const uint32_t version = r.get<uint32_t>();
  TORCH_CHECK(version == 2 || version == 3, "unsupported GGUF version ", version);
  const uint64_t n_tensors = r.get<uint64_t>();
  const uint64_t n_kv = r.get<uint64_t>();
  py::dict meta;
  for (uint64_t i = 0; i < n_kv; ++i) {
    std::string k = r.str();
    const uint32_t t = r.get<uint32_t>();
    meta[py::str(k)] = gguf_value(r, t);
  }
  py::list tensors;
  for (uint64_t i = 0; i < n_tensors; ++i) {
    std::string name = r.str();
    const uint32_t nd = r.get<uint32_t>();
    py::list dims;
    for (uint32_t d = 0; d < nd; ++d) dims.append(r.get<uint64_t>());
    const uint32_t type = r.get<uint32_t>();
    const uint64_t off = r.get<uint64_t>();
    tensors.append(py::make_tuple(name, type, dims, off));
  }
  uint64_t align = 32;
  if (meta.contains("general.alignment")) align = meta["general.alignment"].cast<uint64_t>();
  const uint64_t pos = r.tell();
  const uint64_t data = (pos + align - 1) / align * align;
  return py::make_tuple(version, meta, tensors, data);
}

void register_formats(py::module& m) {
  m.def("safetensors_header", &safetensors_header);
  m.def("gguf_header", &gguf_header);
}

}  // namespace syn
