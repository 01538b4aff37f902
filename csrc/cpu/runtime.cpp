// Host-side native runtime exposed to Python: SPSC rings (in-process or in a POSIX shared
// memory region), the data-plane frame codec, the MoE split rule, an O_DIRECT pread pool
// into pinned buffers, and lock-free metric counters / log-linear histograms.
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <atomic>
#include <chrono>
#include <condition_variable>
#include <cstdlib>
#include <cstring>
#include <deque>
#include <mutex>
#include <string>
#include <thread>
#include <algorithm>
#include <vector>

#include <torch/extension.h>

#include "syn/frame.h"
#include "syn/payload.h"
#include "syn/moe_assign.h"
#include "syn/spsc.h"

namespace py = pybind11;

namespace syn {

// ------------------------------------------------------------------ shared memory region
// A named POSIX shm object holding a header and any number of SPSC rings (the daemon <->
// runner "local plane"; reference crates/ipc/src/shm.rs:75-468).
class ShmRegion {
 public:
  ShmRegion(const std::string& name, int64_t nbytes, bool create) : name_(name), size_(nbytes), owner_(create) {
    int fd = shm_open(name.c_str(), create ? (O_CREAT | O_RDWR | O_EXCL) : O_RDWR, 0600);
    TORCH_CHECK(fd >= 0, "shm_open(", name, ") failed: ", strerror(errno));
    if (create) TORCH_CHECK(ftruncate(fd, nbytes) == 0, "ftruncate failed");
    base_ = mmap(nullptr, (size_t)nbytes, PROT_READ | PROT_WRITE, MAP_SHARED, fd, 0);
    close(fd);
    TORCH_CHECK(base_ != MAP_FAILED, "mmap failed");
  }
  ~ShmRegion() {
    if (base_ && base_ != MAP_FAILED) munmap(base_, (size_t)size_);
    if (owner_) shm_unlink(name_.c_str());
  }
  int64_t address() const { return (int64_t)(uintptr_t)base_; }
  int64_t size() const { return size_; }

 private:
  std::string name_;
  int64_t size_;
  bool owner_;
  void* base_ = nullptr;
};

// ------------------------------------------------------------------ SPSC ring wrapper
class Ring {
 public:
  // Own memory (in-process ring).
  Ring(int64_t capacity, int64_t slot_bytes) {
    TORCH_CHECK(capacity > 0 && (capacity & (capacity - 1)) == 0, "capacity must be a power of two");
    own_.resize(SpscRing::bytes_needed(capacity, (uint32_t)slot_bytes) + 64);
    void* p = reinterpret_cast<void*>((reinterpret_cast<uintptr_t>(own_.data()) + 63) & ~uintptr_t(63));
    r_ = SpscRing::init(p, (uint64_t)capacity, (uint32_t)slot_bytes);
    buf_.resize(slot_bytes);
  }
  // Ring at an address (e.g. inside a ShmRegion); init=true formats it.
  Ring(int64_t address, int64_t capacity, int64_t slot_bytes, bool init) {
    void* p = (void*)(uintptr_t)address;
    TORCH_CHECK((address & 63) == 0, "ring address must be 64-byte aligned");
    r_ = init ? SpscRing::init(p, (uint64_t)capacity, (uint32_t)slot_bytes) : SpscRing::attach(p);
    TORCH_CHECK(r_ != nullptr, "no ring at this address");
    buf_.resize(r_->hdr()->slot_bytes);
  }
  static int64_t bytes_needed(int64_t capacity, int64_t slot_bytes) {
    return (int64_t)SpscRing::bytes_needed((uint64_t)capacity, (uint32_t)slot_bytes);
  }
  bool push(py::bytes b) {
    std::string s = b;
    return r_->push(s.data(), (uint32_t)s.size());
  }
  py::object pop() {
    const int64_t n = r_->pop(buf_.data(), (uint32_t)buf_.size());
    if (n < 0) return py::none();
    return py::bytes(reinterpret_cast<const char*>(buf_.data()), (size_t)n);
  }
  int64_t size() { return (int64_t)r_->size(); }
  int64_t capacity() { return (int64_t)r_->capacity(); }

 private:
  std::vector<uint8_t> own_;
  std::vector<uint8_t> buf_;
  SpscRing* r_ = nullptr;
};

// ------------------------------------------------------------------ frames
py::bytes frame_encode_py(int64_t ftype, int64_t flags, int64_t instance, int64_t term, int64_t seq, int64_t step,
                          int64_t chan_seq, py::bytes ext, py::bytes payload) {
  std::string e = ext, p = payload;
  FrameSpec s;
  s.ftype = (uint8_t)ftype;
  s.flags = (uint16_t)flags;
  s.instance = (uint64_t)instance;
  s.epoch_term = (uint64_t)term;
  s.epoch_seq = (uint64_t)seq;
  s.step = (uint64_t)step;
  s.chan_seq = (uint64_t)chan_seq;
  std::string out(frame_len(e.size(), p.size()), '\0');
  frame_encode(s, reinterpret_cast<const uint8_t*>(e.data()), e.size(), reinterpret_cast<const uint8_t*>(p.data()),
               p.size(), reinterpret_cast<uint8_t*>(&out[0]));
  return py::bytes(out);
}

py::tuple frame_decode_py(py::bytes buf) {
  std::string b = buf;
  FrameSpec s;
  size_t eo, el, po, pl;
  const int rc = frame_decode(reinterpret_cast<const uint8_t*>(b.data()), b.size(), &s, &eo, &el, &po, &pl);
  if (rc != FRAME_OK) return py::make_tuple(rc, py::none(), py::none(), py::none());
  py::dict spec;
  spec["wire_minor"] = s.wire_minor;
  spec["ftype"] = s.ftype;
  spec["flags"] = s.flags;
  spec["instance"] = s.instance;
  spec["epoch_term"] = s.epoch_term;
  spec["epoch_seq"] = s.epoch_seq;
  spec["step"] = s.step;
  spec["chan_seq"] = s.chan_seq;
  return py::make_tuple(0, spec, py::bytes(b.data() + eo, el), py::bytes(b.data() + po, pl));
}

// ------------------------------------------------------------------ payload codecs (syn/payload.h)
static FrameSpec spec_from(py::dict d) {
  FrameSpec s;
  if (d.contains("flags")) s.flags = (uint16_t)py::cast<int64_t>(d["flags"]);
  if (d.contains("instance")) s.instance = (uint64_t)py::cast<int64_t>(d["instance"]);
  if (d.contains("epoch_term")) s.epoch_term = (uint64_t)py::cast<int64_t>(d["epoch_term"]);
  if (d.contains("epoch_seq")) s.epoch_seq = (uint64_t)py::cast<int64_t>(d["epoch_seq"]);
  if (d.contains("step")) s.step = (uint64_t)py::cast<int64_t>(d["step"]);
  if (d.contains("chan_seq")) s.chan_seq = (uint64_t)py::cast<int64_t>(d["chan_seq"]);
  return s;
}

static py::dict spec_to(const FrameSpec& s) {
  py::dict d;
  d["wire_minor"] = s.wire_minor;
  d["ftype"] = s.ftype;
  d["flags"] = s.flags;
  d["instance"] = s.instance;
  d["epoch_term"] = s.epoch_term;
  d["epoch_seq"] = s.epoch_seq;
  d["step"] = s.step;
  d["chan_seq"] = s.chan_seq;
  return d;
}

// rows: contiguous CPU tensor [n_rows, streams * hidden], f32 (dtype 1) or bf16 (dtype 2).
py::bytes activation_encode_py(py::dict frame, py::dict hdr, std::vector<std::tuple<int64_t, int64_t, int64_t, int64_t>> spans,
                               torch::Tensor rows) {
  TORCH_CHECK(!rows.is_cuda() && rows.is_contiguous() && rows.dim() == 2, "rows: contiguous host tensor [n, width]");
  ActivationHeader h;
  h.from_stage = (uint16_t)py::cast<int64_t>(hdr["from_stage"]);
  h.to_stage = (uint16_t)py::cast<int64_t>(hdr["to_stage"]);
  h.kind = (uint8_t)py::cast<int64_t>(hdr["kind"]);
  h.streams = (uint8_t)(hdr.contains("streams") ? py::cast<int64_t>(hdr["streams"]) : 1);
  h.dtype = rows.scalar_type() == torch::kFloat32 ? 1 : rows.scalar_type() == torch::kBFloat16 ? 2 : 0;
  TORCH_CHECK(h.dtype, "rows dtype must be f32 or bf16");
  TORCH_CHECK(rows.size(1) % h.streams == 0, "row width must be streams * hidden");
  h.hidden = (uint32_t)(rows.size(1) / h.streams);
  h.n_rows = (uint32_t)rows.size(0);
  if (hdr.contains("part_index")) h.part_index = (uint16_t)py::cast<int64_t>(hdr["part_index"]);
  if (hdr.contains("part_count")) h.part_count = (uint16_t)py::cast<int64_t>(hdr["part_count"]);
  if (hdr.contains("kind_arg")) h.kind_arg = (uint32_t)py::cast<int64_t>(hdr["kind_arg"]);
  if (hdr.contains("kind_flags")) h.kind_flags = (uint32_t)py::cast<int64_t>(hdr["kind_flags"]);
  std::vector<ActivationSpan> sp;
  for (const auto& t : spans) {
    ActivationSpan a;
    a.seq = (uint64_t)std::get<0>(t);
    a.first_position = (uint32_t)std::get<1>(t);
    a.n_positions = (uint32_t)std::get<2>(t);
    a.row_offset = (uint32_t)std::get<3>(t);
    TORCH_CHECK((uint64_t)a.row_offset + a.n_positions <= h.n_rows, "span rows beyond the frame's rows");
    sp.push_back(a);
  }
  return py::bytes(activation_encode(spec_from(frame), h, sp, reinterpret_cast<const uint8_t*>(rows.data_ptr())));
}

py::tuple activation_decode_py(py::bytes buf) {
  std::string b = buf;
  FrameSpec fs;
  ActivationHeader h;
  std::vector<ActivationSpan> sp;
  std::vector<uint8_t> rows;
  const int rc = activation_decode(reinterpret_cast<const uint8_t*>(b.data()), b.size(), &fs, &h, &sp, &rows);
  if (rc != 0) return py::make_tuple(rc, py::none(), py::none(), py::none(), py::none());
  py::dict hd;
  hd["from_stage"] = h.from_stage;
  hd["to_stage"] = h.to_stage;
  hd["kind"] = h.kind;
  hd["dtype"] = h.dtype;
  hd["streams"] = h.streams;
  hd["hidden"] = h.hidden;
  hd["n_rows"] = h.n_rows;
  hd["part_index"] = h.part_index;
  hd["part_count"] = h.part_count;
  hd["kind_arg"] = h.kind_arg;
  hd["kind_flags"] = h.kind_flags;
  py::list sl;
  for (const auto& a : sp) sl.append(py::make_tuple(a.seq, a.first_position, a.n_positions, a.row_offset));
  auto t = torch::empty({(int64_t)h.n_rows, (int64_t)h.streams * h.hidden},
                        h.dtype == 1 ? torch::kFloat32 : torch::kBFloat16);
  if (!rows.empty()) memcpy(t.data_ptr(), rows.data(), rows.size());
  return py::make_tuple(0, spec_to(fs), hd, sl, t);
}

py::bytes token_encode_py(py::dict frame, std::vector<std::tuple<int64_t, std::vector<int64_t>, int64_t>> entries) {
  std::vector<TokenEntry> es;
  for (const auto& t : entries) {
    TokenEntry e;
    e.seq = (uint64_t)std::get<0>(t);
    for (int64_t x : std::get<1>(t)) e.tokens.push_back((uint32_t)x);
    e.flags = (uint16_t)std::get<2>(t);
    es.push_back(std::move(e));
  }
  return py::bytes(token_encode(spec_from(frame), es));
}

py::tuple token_decode_py(py::bytes buf) {
  std::string b = buf;
  FrameSpec fs;
  std::vector<TokenEntry> es;
  const int rc = token_decode(reinterpret_cast<const uint8_t*>(b.data()), b.size(), &fs, &es);
  if (rc != 0) return py::make_tuple(rc, py::none(), py::none());
  py::list out;
  for (const auto& e : es) {
    std::vector<int64_t> toks(e.tokens.begin(), e.tokens.end());
    out.append(py::make_tuple(e.seq, toks, e.flags));
  }
  return py::make_tuple(0, spec_to(fs), out);
}

static uint8_t rows_dtype(const torch::Tensor& rows) {
  TORCH_CHECK(!rows.is_cuda() && rows.is_contiguous() && rows.dim() == 2, "rows: contiguous host tensor [n, width]");
  const uint8_t d = rows.scalar_type() == torch::kFloat32 ? 1 : rows.scalar_type() == torch::kBFloat16 ? 2 : 0;
  TORCH_CHECK(d, "rows dtype must be f32 or bf16");
  return d;
}
static torch::Tensor rows_tensor(const std::vector<uint8_t>& rows, uint32_t n, uint32_t width, uint8_t dtype) {
  auto t = torch::empty({(int64_t)n, (int64_t)width}, dtype == 1 ? torch::kFloat32 : torch::kBFloat16);
  if (!rows.empty()) memcpy(t.data_ptr(), rows.data(), rows.size());
  return t;
}

// Collective: hdr {phase, member, n_members, layer, row_offset, epoch}; rows [n, width]
py::bytes collective_encode_py(py::dict frame, py::dict hdr, torch::Tensor rows) {
  CollectiveHeader h;
  h.dtype = rows_dtype(rows);
  h.phase = (uint8_t)py::cast<int64_t>(hdr["phase"]);
  h.member = (uint16_t)py::cast<int64_t>(hdr["member"]);
  h.n_members = (uint16_t)py::cast<int64_t>(hdr["n_members"]);
  TORCH_CHECK(h.n_members > 0 && h.member < h.n_members, "member outside the group");
  h.layer = (uint32_t)py::cast<int64_t>(hdr["layer"]);
  h.row_offset = hdr.contains("row_offset") ? (uint32_t)py::cast<int64_t>(hdr["row_offset"]) : 0;
  h.epoch = hdr.contains("epoch") ? (uint32_t)py::cast<int64_t>(hdr["epoch"]) : 0;
  h.n_rows = (uint32_t)rows.size(0);
  h.width = (uint32_t)rows.size(1);
  return py::bytes(collective_encode(spec_from(frame), h, reinterpret_cast<const uint8_t*>(rows.data_ptr())));
}

py::tuple collective_decode_py(py::bytes buf) {
  std::string b = buf;
  FrameSpec fs;
  CollectiveHeader h;
  std::vector<uint8_t> rows;
  const int rc = collective_decode(reinterpret_cast<const uint8_t*>(b.data()), b.size(), &fs, &h, &rows);
  if (rc != 0) return py::make_tuple(rc, py::none(), py::none(), py::none());
  py::dict hd;
  hd["phase"] = h.phase;
  hd["member"] = h.member;
  hd["n_members"] = h.n_members;
  hd["layer"] = h.layer;
  hd["row_offset"] = h.row_offset;
  hd["epoch"] = h.epoch;
  return py::make_tuple(0, spec_to(fs), hd, rows_tensor(rows, h.n_rows, h.width, h.dtype));
}

static EpHeader ep_header_from(py::dict hdr, const torch::Tensor& rows) {
  EpHeader h;
  h.src_rank = (uint16_t)py::cast<int64_t>(hdr["src_rank"]);
  h.dst_rank = (uint16_t)py::cast<int64_t>(hdr["dst_rank"]);
  h.layer = (uint32_t)py::cast<int64_t>(hdr["layer"]);
  h.epoch = hdr.contains("epoch") ? (uint32_t)py::cast<int64_t>(hdr["epoch"]) : 0;
  h.n_rows = (uint32_t)rows.size(0);
  h.hidden = (uint32_t)rows.size(1);
  return h;
}
static py::dict ep_header_to(const EpHeader& h) {
  py::dict hd;
  hd["src_rank"] = h.src_rank;
  hd["dst_rank"] = h.dst_rank;
  hd["layer"] = h.layer;
  hd["epoch"] = h.epoch;
  hd["top_k"] = h.top_k;
  return hd;
}

// routes: per row (source row, [(expert, weight)...]) with at most top_k routes
py::bytes ep_dispatch_encode_py(py::dict frame, py::dict hdr,
                                std::vector<std::tuple<int64_t, std::vector<std::tuple<int64_t, double>>>> routes,
                                torch::Tensor rows) {
  EpHeader h = ep_header_from(hdr, rows);
  h.dtype = rows_dtype(rows);
  h.top_k = (uint8_t)py::cast<int64_t>(hdr["top_k"]);
  TORCH_CHECK(h.top_k > 0 && routes.size() == h.n_rows, "one route record per row, top_k > 0");
  std::vector<EpRoute> rs;
  for (const auto& t : routes) {
    EpRoute e;
    e.row = (uint32_t)std::get<0>(t);
    TORCH_CHECK(!std::get<1>(t).empty() && std::get<1>(t).size() <= h.top_k, "1..top_k routes per row");
    for (const auto& r : std::get<1>(t)) {
      e.experts.push_back((uint16_t)std::get<0>(r));
      e.weights.push_back((float)std::get<1>(r));
    }
    rs.push_back(std::move(e));
  }
  return py::bytes(ep_dispatch_encode(spec_from(frame), h, rs, reinterpret_cast<const uint8_t*>(rows.data_ptr())));
}

py::tuple ep_dispatch_decode_py(py::bytes buf) {
  std::string b = buf;
  FrameSpec fs;
  EpHeader h;
  std::vector<EpRoute> rs;
  std::vector<uint8_t> rows;
  const int rc = ep_dispatch_decode(reinterpret_cast<const uint8_t*>(b.data()), b.size(), &fs, &h, &rs, &rows);
  if (rc != 0) return py::make_tuple(rc, py::none(), py::none(), py::none(), py::none());
  py::list rl;
  for (const auto& e : rs) {
    py::list r;
    for (size_t j = 0; j < e.experts.size(); ++j) r.append(py::make_tuple(e.experts[j], e.weights[j]));
    rl.append(py::make_tuple(e.row, r));
  }
  return py::make_tuple(0, spec_to(fs), ep_header_to(h), rl, rows_tensor(rows, h.n_rows, h.hidden, h.dtype));
}

py::bytes ep_combine_encode_py(py::dict frame, py::dict hdr, std::vector<int64_t> row_ids, torch::Tensor rows) {
  TORCH_CHECK(rows_dtype(rows) == 1, "combine rows are f32");
  EpHeader h = ep_header_from(hdr, rows);
  TORCH_CHECK(row_ids.size() == h.n_rows, "one source row id per row");
  std::vector<uint32_t> ids(row_ids.begin(), row_ids.end());
  return py::bytes(ep_combine_encode(spec_from(frame), h, ids, reinterpret_cast<const uint8_t*>(rows.data_ptr())));
}

py::tuple ep_combine_decode_py(py::bytes buf) {
  std::string b = buf;
  FrameSpec fs;
  EpHeader h;
  std::vector<uint32_t> ids;
  std::vector<uint8_t> rows;
  const int rc = ep_combine_decode(reinterpret_cast<const uint8_t*>(b.data()), b.size(), &fs, &h, &ids, &rows);
  if (rc != 0) return py::make_tuple(rc, py::none(), py::none(), py::none(), py::none());
  std::vector<int64_t> out(ids.begin(), ids.end());
  return py::make_tuple(0, spec_to(fs), ep_header_to(h), out, rows_tensor(rows, h.n_rows, h.hidden, 1));
}

int64_t crc32c_py(py::bytes b) {
  std::string s = b;
  return crc32c(reinterpret_cast<const uint8_t*>(s.data()), s.size());
}

// ------------------------------------------------------------------ MoE split rule
// route: int64 [n, 3] (expert, tokens, cache_slot); eligible: int32 bitmap words.
torch::Tensor moe_assign_py(torch::Tensor route, torch::Tensor eligible, int64_t n_experts, int64_t b_copy,
                            int64_t expert_bytes, int64_t copy_slots) {
  route = route.to(torch::kInt64).contiguous();
  eligible = eligible.to(torch::kInt32).contiguous();
  const int64_t n = route.size(0);
  std::vector<syn_route_slot> r(n);
  auto ra = route.accessor<int64_t, 2>();
  for (int64_t i = 0; i < n; ++i) {
    r[i].expert = (uint16_t)ra[i][0];
    r[i].tokens = (uint16_t)ra[i][1];
    r[i].cache_slot = (uint32_t)ra[i][2];
  }
  std::vector<uint32_t> order(n), out(n);
  syn_moe_assign(r.data(), (uint32_t)n, reinterpret_cast<const uint32_t*>(eligible.data_ptr()), (uint32_t)n_experts,
                 (uint32_t)b_copy, (uint64_t)expert_bytes, (uint32_t)copy_slots, order.data(), out.data());
  auto t = torch::empty({n}, torch::kInt64);
  for (int64_t i = 0; i < n; ++i) t[i] = (int64_t)out[i];
  return t;
}

// ------------------------------------------------------------------ I/O pool
// Reads (fd, offset, length) extents into caller buffers (pinned host memory for the
// host->VRAM weight path) with N worker threads using pread; files opened with O_DIRECT
// when the extent and buffer alignments allow (reference: crates/io/src/pool/linux.rs).
class IoPool {
 public:
  explicit IoPool(int threads) {
    for (int i = 0; i < threads; ++i) workers_.emplace_back([this] { run(); });
  }
  ~IoPool() {
    {
      std::lock_guard<std::mutex> g(mu_);
      stop_ = true;
    }
    cv_.notify_all();
    for (auto& t : workers_) t.join();
  }
  // Submit a read; returns a ticket.  dst is a host address with room for `len` bytes.
  int64_t submit(const std::string& path, int64_t offset, int64_t len, int64_t dst) {
    std::lock_guard<std::mutex> g(mu_);
    const int64_t id = next_++;
    q_.push_back({id, path, offset, len, dst});
    pending_++;
    cv_.notify_one();
    return id;
  }
  // Wait for all submitted reads; returns total bytes read (negative errno of the first failure).
  int64_t wait_all() {
    std::unique_lock<std::mutex> g(mu_);
    done_cv_.wait(g, [this] { return pending_ == 0; });
    const int64_t r = first_error_ ? first_error_ : bytes_;
    bytes_ = 0;
    first_error_ = 0;
    return r;
  }

 private:
  struct Job {
    int64_t id;
    std::string path;
    int64_t offset, len, dst;
  };
  void run() {
    for (;;) {
      Job j;
      {
        std::unique_lock<std::mutex> g(mu_);
        cv_.wait(g, [this] { return stop_ || !q_.empty(); });
        if (stop_ && q_.empty()) return;
        j = q_.front();
        q_.pop_front();
      }
      int64_t got = do_read(j);
      {
        std::lock_guard<std::mutex> g(mu_);
        if (got < 0 && !first_error_) first_error_ = got;
        if (got > 0) bytes_ += got;
        if (--pending_ == 0) done_cv_.notify_all();
      }
    }
  }
  static int64_t do_read(const Job& j) {
    const bool aligned = (j.offset % 4096 == 0) && (j.len % 4096 == 0) && (j.dst % 4096 == 0);
    int fd = open(j.path.c_str(), O_RDONLY | (aligned ? O_DIRECT : 0));
    if (fd < 0 && aligned) fd = open(j.path.c_str(), O_RDONLY);
    if (fd < 0) return -errno;
    int64_t done = 0;
    while (done < j.len) {
      const ssize_t n = pread(fd, (char*)(uintptr_t)j.dst + done, (size_t)(j.len - done), (off_t)(j.offset + done));
      if (n < 0) {
        if (errno == EINTR) continue;
        const int64_t e = -errno;
        close(fd);
        return e;
      }
      if (n == 0) break;
      done += n;
    }
    close(fd);
    return done;
  }
  std::vector<std::thread> workers_;
  std::deque<Job> q_;
  std::mutex mu_;
  std::condition_variable cv_, done_cv_;
  bool stop_ = false;
  int64_t next_ = 0, pending_ = 0, bytes_ = 0, first_error_ = 0;
};

// ------------------------------------------------------------------ metrics
// Counters and log-linear histograms with relaxed atomics (hot-thread safe; reference
// crates/obs/src/metrics/{registry.rs,histogram.rs}).  Histogram buckets: 8 linear
// sub-buckets per power of two from 1 unit to 2^40 units.
class Histogram {
 public:
  static constexpr int kSub = 8, kPow = 41, kBuckets = kSub * kPow;
  Histogram() {
    for (auto& b : b_) b.store(0, std::memory_order_relaxed);
  }
  static int bucket(uint64_t v) {
    if (v < kSub) return (int)v;
    const int p = 63 - __builtin_clzll(v);  // floor(log2 v) >= 3
    const int sub = (int)((v >> (p - 3)) & (kSub - 1));
    const int idx = (p - 2) * kSub + sub;
    return idx < kBuckets ? idx : kBuckets - 1;
  }
  static double lower(int idx) {
    if (idx < kSub) return idx;
    const int p = idx / kSub + 2, sub = idx % kSub;
    return std::ldexp(1.0 + sub / (double)kSub, p);
  }
  void record(int64_t v) {
    b_[bucket(v < 0 ? 0 : (uint64_t)v)].fetch_add(1, std::memory_order_relaxed);
    n_.fetch_add(1, std::memory_order_relaxed);
    sum_.fetch_add(v, std::memory_order_relaxed);
  }
  double quantile(double q) {
    const uint64_t n = n_.load(std::memory_order_relaxed);
    if (!n) return 0.0;
    const uint64_t target = (uint64_t)std::ceil(q * n);
    uint64_t acc = 0;
    for (int i = 0; i < kBuckets; ++i) {
      acc += b_[i].load(std::memory_order_relaxed);
      if (acc >= target) return lower(i);
    }
    return lower(kBuckets - 1);
  }
  int64_t count() { return (int64_t)n_.load(); }
  int64_t sum() { return (int64_t)sum_.load(); }

 private:
  std::atomic<uint64_t> b_[kBuckets];
  std::atomic<uint64_t> n_{0};
  std::atomic<int64_t> sum_{0};
};

class Counter {
 public:
  void add(int64_t v) { v_.fetch_add(v, std::memory_order_relaxed); }
  int64_t get() { return v_.load(std::memory_order_relaxed); }

 private:
  std::atomic<int64_t> v_{0};
};

// Prompt-lookup drafting for a batch of sequences: for each history, the most recent earlier
// occurrence of its last n tokens (n from max_n down to 1) and the g tokens that followed it,
// padded with the last of them; without any match, g copies of the last token.  One linear
// scan per (sequence, n), in native code because the host builds the drafts of every running
// sequence each decode step.
static std::vector<std::vector<int64_t>> ngram_propose_py(const std::vector<std::vector<int64_t>>& histories,
                                                          int max_n, int g) {
  std::vector<std::vector<int64_t>> out;
  out.reserve(histories.size());
  for (const auto& h : histories) {
    const int64_t L = (int64_t)h.size();
    std::vector<int64_t> d;
    for (int n = (int)std::min<int64_t>(max_n, L - 1); n >= 1 && d.empty(); --n) {
      const int64_t* key = h.data() + L - n;
      for (int64_t i = L - n - 1; i >= 0; --i) {
        if (std::equal(key, key + n, h.data() + i)) {
          const int64_t c0 = i + n, c1 = std::min<int64_t>(L, c0 + g);
          if (c1 > c0) {
            d.assign(h.begin() + c0, h.begin() + c1);
            break;
          }
        }
      }
    }
    if (d.empty()) d.assign(g, L > 0 ? h.back() : 0);
    while ((int)d.size() < g) d.push_back(d.back());
    out.push_back(std::move(d));
  }
  return out;
}

void register_runtime(py::module& m) {
  m.def("ngram_propose", &ngram_propose_py, "prompt-lookup drafts for a batch of token histories");
  py::class_<ShmRegion>(m, "ShmRegion")
      .def(py::init<const std::string&, int64_t, bool>())
      .def("address", &ShmRegion::address)
      .def("size", &ShmRegion::size);
  py::class_<Ring>(m, "SpscRing")
      .def(py::init<int64_t, int64_t>())
      .def(py::init<int64_t, int64_t, int64_t, bool>())
      .def_static("bytes_needed", &Ring::bytes_needed)
      .def("push", &Ring::push)
      .def("pop", &Ring::pop)
      .def("size", &Ring::size)
      .def("capacity", &Ring::capacity);
  m.def("frame_encode", &frame_encode_py);
  m.def("frame_decode", &frame_decode_py);
  m.def("crc32c", &crc32c_py);
  m.def("activation_encode", &activation_encode_py);
  m.def("collective_encode", &collective_encode_py);
  m.def("collective_decode", &collective_decode_py);
  m.def("ep_dispatch_encode", &ep_dispatch_encode_py);
  m.def("ep_dispatch_decode", &ep_dispatch_decode_py);
  m.def("ep_combine_encode", &ep_combine_encode_py);
  m.def("ep_combine_decode", &ep_combine_decode_py);
  m.def("activation_decode", &activation_decode_py);
  m.def("token_encode", &token_encode_py);
  m.def("token_decode", &token_decode_py);
  m.def("moe_assign", &moe_assign_py);
  py::class_<IoPool>(m, "IoPool")
      .def(py::init<int>())
      .def("submit", &IoPool::submit)
      .def("wait_all", &IoPool::wait_all, py::call_guard<py::gil_scoped_release>());
  py::class_<Histogram>(m, "Histogram")
      .def(py::init<>())
      .def("record", &Histogram::record)
      .def("quantile", &Histogram::quantile)
      .def("count", &Histogram::count)
      .def("sum", &Histogram::sum);
  py::class_<Counter>(m, "Counter").def(py::init<>()).def("add", &Counter::add).def("get", &Counter::get);
}

}  // namespace syn
