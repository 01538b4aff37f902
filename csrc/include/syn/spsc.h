// Lock-free single-producer / single-consumer ring of fixed-size slots.
//
// Capacity is a power of two; head and tail live on their own cache lines; the producer
// publishes a slot with a release store of `tail`, the consumer frees it with a release store
// of `head`.  The ring is position-independent (no pointers inside), so the same layout works
// in process memory and in a shared-memory region mapped by two processes.
// Reference: crates/spsc/src/ring.rs:61-243 (same contract: power-of-two capacity, padded
// indices, wait-free push/pop, blocking left to the caller).
#pragma once
#include <atomic>
#include <cstddef>
#include <cstdint>
#include <cstring>

namespace syn {

struct alignas(64) SpscHeader {
  uint32_t magic;      // 'SPSC'
  uint32_t slot_bytes; // payload bytes per slot (a 4-byte length prefix precedes each payload)
  uint64_t capacity;   // slots, power of two
  alignas(64) std::atomic<uint64_t> head;  // next slot to read (consumer-owned)
  alignas(64) std::atomic<uint64_t> tail;  // next slot to write (producer-owned)
  alignas(64) uint8_t pad[64];
};

class SpscRing {
 public:
  static constexpr uint32_t kMagic = 0x43535053u;  // "SPSC"

  static size_t bytes_needed(uint64_t capacity, uint32_t slot_bytes) {
    return sizeof(SpscHeader) + capacity * (uint64_t)(slot_bytes + 4);
  }

  // Initialise a ring in `mem` (bytes_needed() bytes, 64-byte aligned).
  static SpscRing* init(void* mem, uint64_t capacity, uint32_t slot_bytes) {
    auto* h = new (mem) SpscHeader();
    h->magic = kMagic;
    h->slot_bytes = slot_bytes;
    h->capacity = capacity;
    h->head.store(0, std::memory_order_relaxed);
    h->tail.store(0, std::memory_order_relaxed);
    return reinterpret_cast<SpscRing*>(mem);
  }
  // Attach to an already initialised ring.
  static SpscRing* attach(void* mem) {
    auto* h = reinterpret_cast<SpscHeader*>(mem);
    return h->magic == kMagic ? reinterpret_cast<SpscRing*>(mem) : nullptr;
  }

  SpscHeader* hdr() { return reinterpret_cast<SpscHeader*>(this); }
  uint8_t* slot(uint64_t i) {
    SpscHeader* h = hdr();
    return reinterpret_cast<uint8_t*>(h) + sizeof(SpscHeader) + (i & (h->capacity - 1)) * (h->slot_bytes + 4);
  }

  // Producer: copy `n` bytes in; false when full or too large.
  bool push(const void* data, uint32_t n) {
    SpscHeader* h = hdr();
    if (n > h->slot_bytes) return false;
    const uint64_t t = h->tail.load(std::memory_order_relaxed);
    const uint64_t hd = h->head.load(std::memory_order_acquire);
    if (t - hd >= h->capacity) return false;
    uint8_t* s = slot(t);
    memcpy(s, &n, 4);
    memcpy(s + 4, data, n);
    h->tail.store(t + 1, std::memory_order_release);
    return true;
  }

  // Consumer: copy the oldest message out; returns its length or -1 when empty.
  int64_t pop(void* out, uint32_t cap) {
    SpscHeader* h = hdr();
    const uint64_t hd = h->head.load(std::memory_order_relaxed);
    const uint64_t t = h->tail.load(std::memory_order_acquire);
    if (hd == t) return -1;
    uint8_t* s = slot(hd);
    uint32_t n;
    memcpy(&n, s, 4);
    if (n > cap) return -2;  // caller buffer too small; message stays queued
    memcpy(out, s + 4, n);
    h->head.store(hd + 1, std::memory_order_release);
    return n;
  }

  uint64_t size() {
    SpscHeader* h = hdr();
    return h->tail.load(std::memory_order_acquire) - h->head.load(std::memory_order_acquire);
  }
  uint64_t capacity() { return hdr()->capacity; }
};

}  // namespace syn
