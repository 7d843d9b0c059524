// ExpertCache: the slot-table policy of MoEStream, rebuilt for this library.
//
// Interface and decisions follow the reference class moestream::ExpertCache
// (src/expert_cache.hpp:61-147, src/expert_cache.cpp): S3-FIFO with SMALL /
// MAIN / GHOST queues per layer, a frequency ceiling of 3, refcounted slots
// that are never evicted while in use, a LIFO free-slot stack that hands out
// slot 0 first, per-layer quotas rebalanced from ghost hits, and an optional
// PINNED set. Given the same call sequence it returns the same slot for every
// request as the reference; the tests replay random traces through both.
//
// Differences from the reference, both outside its production configuration
// (one cache per layer with n_layer = 1 and pin_ratio = 0):
//   - build_pinned breaks frequency ties by the lower expert id (the
//     reference uses std::partial_sort, whose tie order is unspecified);
//   - queues are fixed-capacity rings sized n_expert per layer instead of
//     std::deque; every queue holds each expert at most once, so the capacity
//     is never exceeded.
//
// Single-threaded, no locks (like the reference).
#pragma once

#include <cstddef>
#include <cstdint>
#include <string>
#include <vector>

namespace moestream {

enum class Origin : uint8_t { Demand, PrefetchHigh, PrefetchLow, Sweep };
enum class Seg : uint8_t { None, Pinned, Small, Main };

struct CacheStats {
  uint64_t hit = 0, miss = 0, hit_pinned = 0, hit_small = 0, hit_main = 0,
           ghost_hit = 0, admit = 0, evict = 0, bypass = 0, promote = 0,
           bytes_fetched = 0;
  double hit_rate() const {
    const uint64_t t = hit + miss;
    return t ? double(hit) / double(t) : 0.0;
  }
};

class ExpertCache {
 public:
  struct Config {
    uint32_t n_layer = 40;
    uint32_t n_expert = 256;
    uint32_t n_slot = 0;
    double cache_frac = 0.25;
    double pin_ratio = 0.05;
    double small_ratio = 0.10;
    uint32_t ghost_mult = 2;
    bool layer_quota_adapt = true;
    uint32_t quota_period = 512;
    double quota_eta = 0.10;
    uint32_t quota_min = 8;
  };
  static constexpr uint32_t kNoSlot = 0xFFFFFFFFu;

  explicit ExpertCache(const Config &cfg);

  bool acquire(uint32_t layer, uint32_t expert, Origin origin,
               uint32_t *out_slot);
  void mark_resident(uint32_t layer, uint32_t expert, uint64_t nbytes);
  void release(uint32_t layer, uint32_t expert);
  void end_step();
  void build_pinned(const std::vector<uint32_t> &freq_per_layer_expert);

  const CacheStats &stats() const { return stats_; }
  uint32_t n_slot() const { return n_slot_; }
  uint32_t slot_of(uint32_t layer, uint32_t expert) const {
    return entries_[key(layer, expert)].slot;
  }
  std::vector<uint32_t> layer_quota() const { return quota_; }
  std::string quota_summary() const;

 private:
  static constexpr uint32_t kFreqCap = 3;

  // Fixed-capacity FIFO of expert ids with order-preserving removal.
  class Ring {
   public:
    void init(uint32_t cap) { buf_.assign(cap ? cap : 1, 0); head_ = n_ = 0; }
    uint32_t size() const { return n_; }
    uint32_t front() const { return buf_[head_]; }
    void pop_front() { head_ = wrap(head_ + 1); --n_; }
    void push_back(uint32_t v) { buf_[wrap(head_ + n_)] = v; ++n_; }
    void push_front(uint32_t v) { head_ = wrap(head_ + cap() - 1); buf_[head_] = v; ++n_; }
    bool remove(uint32_t v);  // first occurrence; true if found
   private:
    uint32_t cap() const { return uint32_t(buf_.size()); }
    uint32_t wrap(uint32_t i) const { return i >= cap() ? i - cap() : i; }
    std::vector<uint32_t> buf_;
    uint32_t head_ = 0, n_ = 0;
  };

  struct Entry {
    uint32_t slot = kNoSlot;
    uint16_t refs = 0;
    Seg seg = Seg::None;
    bool loaded = false;
    uint32_t freq = 0;
    uint32_t last_step = 0;
  };
  struct Layer {
    Ring small, main, ghost;
    uint32_t ghost_hits = 0;
    uint32_t resident = 0;
    uint32_t pinned = 0;
  };

  size_t key(uint32_t l, uint32_t e) const {
    return size_t(l) * cfg_.n_expert + e;
  }
  uint32_t take_slot(uint32_t layer);
  bool evict_from(uint32_t layer);
  void rebalance();

  Config cfg_;
  uint32_t n_slot_ = 0;
  std::vector<Entry> entries_;
  std::vector<Layer> layers_;
  std::vector<uint32_t> quota_;
  std::vector<uint32_t> free_slots_;  // stack; back() is handed out next
  CacheStats stats_;
  uint32_t step_ = 0;
};

}  // namespace moestream
