// Grammar-constrained decoding on the host (reference crates/text/src/constraint/{engine.rs,
// schema.rs}: token masks from a grammar over the vocabulary, with a vocabulary cache).
//
// The vocabulary's byte strings go into a trie once.  A constraint is a byte-level automaton
// (here: any JSON value of RFC 8259 with an object at the top level, or one of a list of
// strings).  The mask of allowed next tokens is a depth-first walk of the trie that advances a
// copy of the automaton along each edge and prunes at the first rejected byte, so a subtree of
// tokens sharing a rejected prefix costs one step.  Masks are cached per automaton state (the
// part of the state that the longest token can observe), which makes repeated states — most
// of the steps inside a JSON string — a lookup.
#include <torch/extension.h>

#include <algorithm>
#include <cctype>
#include <cstring>
#include <memory>
#include <string>
#include <unordered_map>
#include <vector>

namespace syn {
namespace {

struct TrieNode {
  std::vector<std::pair<uint8_t, int>> kids;  // sorted by byte
  std::vector<int32_t> tokens;                // ids whose byte string ends here
  int child(unsigned char c) const {
    auto it = std::lower_bound(kids.begin(), kids.end(), std::make_pair((uint8_t)c, -1));
    return (it != kids.end() && it->first == c) ? it->second : -1;
  }
};

}  // namespace

class TokenTrie {
 public:
  explicit TokenTrie(const std::vector<std::string>& vocab) : V_((int64_t)vocab.size()), bytes_(vocab) {
    nodes_.emplace_back();
    std::unordered_map<uint64_t, int> edge;  // (node << 8 | byte) -> child, while building
    for (int32_t id = 0; id < (int32_t)vocab.size(); ++id) {
      const std::string& s = vocab[id];
      if (s.empty()) continue;  // special tokens: never produced under a constraint
      max_len_ = std::max<int>(max_len_, (int)s.size());
      int n = 0;
      for (unsigned char c : s) {
        const uint64_t key = ((uint64_t)n << 8) | c;
        auto it = edge.find(key);
        if (it == edge.end()) {
          const int nn = (int)nodes_.size();
          nodes_.emplace_back();
          nodes_[n].kids.emplace_back(c, nn);
          edge.emplace(key, nn);
          n = nn;
        } else {
          n = it->second;
        }
      }
      nodes_[n].tokens.push_back(id);
    }
    for (auto& nd : nodes_) std::sort(nd.kids.begin(), nd.kids.end());
  }
  int64_t vocab_size() const { return V_; }
  int64_t n_nodes() const { return (int64_t)nodes_.size(); }
  int max_len() const { return max_len_; }
  const TrieNode& node(int i) const { return nodes_[i]; }
  const std::string& bytes(int32_t id) const { return bytes_[id]; }
  // JSON masks by observable automaton state, shared by every sequence of this vocabulary
  std::unordered_map<std::string, std::vector<uint32_t>> json_cache;

 private:
  int64_t V_;
  int max_len_ = 0;
  std::vector<TrieNode> nodes_;
  std::vector<std::string> bytes_;
};

namespace {

// ------------------------------------------------------------------ JSON automaton
enum JMode : uint8_t {
  J_START,        // before the top-level value (whitespace, then '{')
  J_VALUE,        // expecting a value
  J_OBJ_FIRST,    // after '{': key or '}'
  J_OBJ_KEY,      // after ',' in an object: key
  J_COLON,        // after a key
  J_ARR_FIRST,    // after '[': value or ']'
  J_AFTER,        // after a value: ',' or the container's closer
  J_STRING,       // inside a string
  J_ESC,          // after a backslash
  J_HEX,          // inside \uXXXX (hex_left digits to go)
  J_NUM,          // inside a number (num_state)
  J_LIT,          // inside true / false / null
  J_DONE,         // top-level value complete
};
enum NumState : uint8_t { N_MINUS, N_ZERO, N_INT, N_DOT, N_FRAC, N_E, N_ESIGN, N_EXP };

struct Json {
  std::string stack;  // open containers: '{' or '['
  JMode mode = J_START;
  bool key = false;   // the string being read is an object key
  uint8_t hex_left = 0, num = 0, ws = 0;
  uint8_t u8_need = 0, u8_lo = 0x80, u8_hi = 0xBF;  // UTF-8 continuation bytes still expected in a string
  const char* lit = nullptr;
  uint8_t lit_pos = 0;
  static constexpr int kMaxWs = 8;  // longest run of insignificant whitespace

  static bool is_ws(unsigned char c) { return c == ' ' || c == '\n' || c == '\t' || c == '\r'; }

  bool ws_ok(unsigned char c) {
    if (!is_ws(c)) return false;
    if (ws >= kMaxWs) return false;
    ++ws;
    return true;
  }

  void value_done() {
    mode = stack.empty() ? J_DONE : J_AFTER;
  }

  bool start_value(unsigned char c) {
    switch (c) {
      case '{': stack.push_back('{'); mode = J_OBJ_FIRST; return true;
      case '[': stack.push_back('['); mode = J_ARR_FIRST; return true;
      case '"': key = false; mode = J_STRING; return true;
      case 't': lit = "true"; lit_pos = 1; mode = J_LIT; return true;
      case 'f': lit = "false"; lit_pos = 1; mode = J_LIT; return true;
      case 'n': lit = "null"; lit_pos = 1; mode = J_LIT; return true;
      case '-': num = N_MINUS; mode = J_NUM; return true;
      case '0': num = N_ZERO; mode = J_NUM; return true;
      default:
        if (c >= '1' && c <= '9') {
          num = N_INT;
          mode = J_NUM;
          return true;
        }
        return false;
    }
  }

  bool close(unsigned char c) {
    if (stack.empty()) return false;
    if ((c == '}' && stack.back() != '{') || (c == ']' && stack.back() != '[')) return false;
    stack.pop_back();
    value_done();
    return true;
  }

  bool step(unsigned char c) {
    if (mode != J_STRING && mode != J_ESC && mode != J_HEX && !is_ws(c)) ws = 0;
    switch (mode) {
      case J_START:
        if (ws_ok(c)) return true;
        if (c != '{') return false;
        stack.push_back('{');
        mode = J_OBJ_FIRST;
        return true;
      case J_VALUE:
        if (ws_ok(c)) return true;
        return start_value(c);
      case J_OBJ_FIRST:
        if (ws_ok(c)) return true;
        if (c == '}') return close(c);
        if (c != '"') return false;
        key = true;
        mode = J_STRING;
        return true;
      case J_OBJ_KEY:
        if (ws_ok(c)) return true;
        if (c != '"') return false;
        key = true;
        mode = J_STRING;
        return true;
      case J_COLON:
        if (ws_ok(c)) return true;
        if (c != ':') return false;
        mode = J_VALUE;
        return true;
      case J_ARR_FIRST:
        if (ws_ok(c)) return true;
        if (c == ']') return close(c);
        return start_value(c);
      case J_AFTER:
        if (ws_ok(c)) return true;
        if (c == ',') {
          mode = stack.back() == '{' ? J_OBJ_KEY : J_VALUE;
          return true;
        }
        if (c == '}' || c == ']') return close(c);
        return false;
      case J_STRING:
        if (u8_need) {  // inside a multi-byte UTF-8 character
          if (c < u8_lo || c > u8_hi) return false;
          --u8_need;
          u8_lo = 0x80;
          u8_hi = 0xBF;
          return true;
        }
        if (c >= 0x80) {  // lead byte of a well-formed UTF-8 sequence (RFC 3629 table)
          if (c >= 0xC2 && c <= 0xDF) {
            u8_need = 1;
          } else if (c >= 0xE0 && c <= 0xEF) {
            u8_need = 2;
            if (c == 0xE0) u8_lo = 0xA0;
            if (c == 0xED) u8_hi = 0x9F;
          } else if (c >= 0xF0 && c <= 0xF4) {
            u8_need = 3;
            if (c == 0xF0) u8_lo = 0x90;
            if (c == 0xF4) u8_hi = 0x8F;
          } else {
            return false;
          }
          return true;
        }
        if (c == '"') {
          if (key) {
            key = false;
            mode = J_COLON;
          } else {
            value_done();
          }
          return true;
        }
        if (c == '\\') {
          mode = J_ESC;
          return true;
        }
        return c >= 0x20;  // no raw control characters
      case J_ESC:
        if (c == 'u') {
          hex_left = 4;
          mode = J_HEX;
          return true;
        }
        if (std::strchr("\"\\/bfnrt", c) && c) {
          mode = J_STRING;
          return true;
        }
        return false;
      case J_HEX:
        if (!std::isxdigit(c)) return false;
        if (--hex_left == 0) mode = J_STRING;
        return true;
      case J_LIT:
        if (c != (unsigned char)lit[lit_pos]) return false;
        if (lit[++lit_pos] == 0) value_done();
        return true;
      case J_NUM: {
        const bool digit = c >= '0' && c <= '9';
        switch (num) {
          case N_MINUS:
            if (c == '0') { num = N_ZERO; return true; }
            if (digit) { num = N_INT; return true; }
            return false;
          case N_ZERO:
          case N_INT:
            if (digit && num == N_INT) return true;
            if (c == '.') { num = N_DOT; return true; }
            if (c == 'e' || c == 'E') { num = N_E; return true; }
            break;  // the number ends here
          case N_DOT:
            if (digit) { num = N_FRAC; return true; }
            return false;
          case N_FRAC:
            if (digit) return true;
            if (c == 'e' || c == 'E') { num = N_E; return true; }
            break;
          case N_E:
            if (c == '+' || c == '-') { num = N_ESIGN; return true; }
            if (digit) { num = N_EXP; return true; }
            return false;
          case N_ESIGN:
            if (digit) { num = N_EXP; return true; }
            return false;
          case N_EXP:
            if (digit) return true;
            break;
        }
        // a complete number followed by a delimiter: close the number, re-read the byte
        value_done();
        return step(c);
      }
      case J_DONE:
        return false;
    }
    return false;
  }

  bool accepting() const { return mode == J_DONE; }
  bool finished() const { return mode == J_DONE; }

  // the part of the state a token of at most `lmax` bytes can observe
  std::string key_of(int lmax) const {
    std::string k;
    k.push_back((char)mode);
    k.push_back((char)key);
    k.push_back((char)hex_left);
    k.push_back((char)num);
    k.push_back((char)ws);
    k.push_back((char)lit_pos);
    k.push_back((char)u8_need);
    k.push_back((char)u8_lo);
    k.push_back((char)u8_hi);
    k.push_back(lit ? lit[0] : 0);
    const int keep = std::min<int>((int)stack.size(), lmax);
    k.push_back((char)std::min<size_t>(stack.size(), (size_t)lmax + 1));
    k.append(stack.end() - keep, stack.end());
    return k;
  }
};

// ------------------------------------------------------------------ choice automaton
struct Choices {
  std::shared_ptr<TokenTrie> trie;  // trie of the allowed strings (ids = choice index)
  int node = 0;
  bool dead = false;
  bool step(unsigned char c) {
    const int n = trie->node(node).child(c);
    if (n < 0) return false;
    node = n;
    return true;
  }
  bool accepting() const { return !trie->node(node).tokens.empty(); }
  bool finished() const { return accepting() && trie->node(node).kids.empty(); }
  std::string key_of(int) const { return std::to_string(node); }
};

template <typename A>
void walk(const TokenTrie& T, int n, const A& st, uint32_t* mask) {
  for (const auto& kv : T.node(n).kids) {
    A s2 = st;
    if (!s2.step(kv.first)) continue;
    for (int32_t id : T.node(kv.second).tokens) mask[id >> 5] |= 1u << (id & 31);
    walk(T, kv.second, s2, mask);
  }
}

}  // namespace

// One sequence's constraint: its automaton state, the shared vocabulary trie and mask cache.
class Constraint {
 public:
  static std::unique_ptr<Constraint> json(std::shared_ptr<TokenTrie> trie, int64_t eos) {
    auto c = std::unique_ptr<Constraint>(new Constraint(std::move(trie), eos));
    c->kind_ = 0;
    return c;
  }
  static std::unique_ptr<Constraint> choices(std::shared_ptr<TokenTrie> trie, int64_t eos,
                                             const std::vector<std::string>& options) {
    TORCH_CHECK(!options.empty(), "choice constraint: at least one option");
    auto c = std::unique_ptr<Constraint>(new Constraint(std::move(trie), eos));
    c->kind_ = 1;
    c->ch_.trie = std::make_shared<TokenTrie>(options);
    return c;
  }

  // Allowed next tokens as int32 words of a bitmask over the vocabulary (EOS allowed exactly
  // when the text so far is complete).
  torch::Tensor mask() {
    auto& cache = kind_ == 0 ? trie_->json_cache[js_.key_of(trie_->max_len())] : cache_[ch_.key_of(0)];
    if (cache.empty()) {
      cache.assign((trie_->vocab_size() + 31) / 32, 0u);
      if (kind_ == 0)
        walk(*trie_, 0, js_, cache.data());
      else
        walk(*trie_, 0, ch_, cache.data());
    }
    auto out = torch::empty({(int64_t)cache.size()}, torch::kInt32);
    std::memcpy(out.data_ptr(), cache.data(), cache.size() * 4);
    const bool acc = kind_ == 0 ? js_.accepting() : ch_.accepting();
    if (eos_ >= 0 && eos_ < trie_->vocab_size()) {
      uint32_t* w = reinterpret_cast<uint32_t*>(out.data_ptr());
      if (acc)
        w[eos_ >> 5] |= 1u << (eos_ & 31);
      else
        w[eos_ >> 5] &= ~(1u << (eos_ & 31));
    }
    return out;
  }

  // Advances over a chosen token; false (state unchanged) if the token breaks the grammar.
  bool advance(int64_t id) {
    if (id == eos_) return kind_ == 0 ? js_.accepting() : ch_.accepting();
    TORCH_CHECK(id >= 0 && id < trie_->vocab_size(), "token id out of range");
    const std::string& b = trie_->bytes((int32_t)id);
    if (b.empty()) return false;
    if (kind_ == 0) {
      Json s = js_;
      for (unsigned char c : b)
        if (!s.step(c)) return false;
      js_ = s;
    } else {
      Choices s = ch_;
      for (unsigned char c : b)
        if (!s.step(c)) return false;
      ch_ = s;
    }
    return true;
  }

  bool accepting() const { return kind_ == 0 ? js_.accepting() : ch_.accepting(); }
  bool finished() const { return kind_ == 0 ? js_.finished() : ch_.finished(); }

 private:
  Constraint(std::shared_ptr<TokenTrie> trie, int64_t eos) : trie_(std::move(trie)), eos_(eos) {}
  std::shared_ptr<TokenTrie> trie_;
  int64_t eos_;
  int kind_ = 0;
  Json js_;
  Choices ch_;
  std::unordered_map<std::string, std::vector<uint32_t>> cache_;  // choice masks by trie node
};

void register_constrain(pybind11::module& m) {
  pybind11::class_<TokenTrie, std::shared_ptr<TokenTrie>>(m, "TokenTrie")
      .def(pybind11::init([](std::vector<pybind11::bytes> vocab) {
        std::vector<std::string> v;
        v.reserve(vocab.size());
        for (auto& b : vocab) v.emplace_back(std::string(b));
        return std::make_shared<TokenTrie>(v);
      }))
      .def("vocab_size", &TokenTrie::vocab_size)
      .def("n_nodes", &TokenTrie::n_nodes)
      .def("max_len", &TokenTrie::max_len);
  pybind11::class_<Constraint>(m, "Constraint")
      .def_static("json", &Constraint::json, "any JSON text whose top-level value is an object")
      .def_static("choices", [](std::shared_ptr<TokenTrie> t, int64_t eos, std::vector<pybind11::bytes> options) {
        std::vector<std::string> v;
        for (auto& b : options) v.emplace_back(std::string(b));
        return Constraint::choices(std::move(t), eos, v);
      }, "exactly one of the given byte strings")
      .def("mask", &Constraint::mask)
      .def("advance", &Constraint::advance)
      .def("accepting", &Constraint::accepting)
      .def("finished", &Constraint::finished);
}

}  // namespace syn
