// ExpertCache policy implementation; see expert_cache.hpp for what it mirrors.
#include "expert_cache.hpp"

#include <algorithm>
#include <climits>
#include <cstdio>
#include <numeric>

namespace moestream {

bool ExpertCache::Ring::remove(uint32_t v) {
  for (uint32_t i = 0; i < n_; ++i) {
    if (buf_[wrap(head_ + i)] != v) continue;
    // Close the gap by shifting the later elements one place forward.
    for (uint32_t j = i; j + 1 < n_; ++j)
      buf_[wrap(head_ + j)] = buf_[wrap(head_ + j + 1)];
    --n_;
    return true;
  }
  return false;
}

ExpertCache::ExpertCache(const Config &cfg) : cfg_(cfg) {
  const uint32_t total = cfg_.n_layer * cfg_.n_expert;
  // Slot count: explicit, or the resident fraction of all (layer, expert)
  // pairs rounded half up (src/expert_cache.cpp:11-13).
  n_slot_ = cfg_.n_slot ? cfg_.n_slot
                        : uint32_t(double(total) * cfg_.cache_frac + 0.5);
  entries_.assign(total, Entry{});
  layers_.resize(cfg_.n_layer);
  for (Layer &L : layers_) {
    L.small.init(cfg_.n_expert);
    L.main.init(cfg_.n_expert);
    L.ghost.init(cfg_.n_expert);
  }
  // Even split; the remainder goes one each to the leading layers.
  quota_.assign(cfg_.n_layer, n_slot_ / cfg_.n_layer);
  uint32_t rest = n_slot_ - quota_[0] * cfg_.n_layer;
  for (uint32_t l = 0; rest > 0; --rest, ++l) quota_[l % cfg_.n_layer]++;
  // Stack of free slots with slot 0 on top.
  free_slots_.resize(n_slot_);
  for (uint32_t i = 0; i < n_slot_; ++i) free_slots_[i] = n_slot_ - 1 - i;
}

void ExpertCache::build_pinned(const std::vector<uint32_t> &freq) {
  if (cfg_.pin_ratio <= 0.0 || freq.size() != entries_.size()) return;
  const uint32_t per_layer = std::max<uint32_t>(
      1, uint32_t(cfg_.n_expert * cfg_.pin_ratio + 0.5));
  std::vector<uint32_t> order(cfg_.n_expert);
  for (uint32_t l = 0; l < cfg_.n_layer; ++l) {
    const size_t base = size_t(l) * cfg_.n_expert;
    std::iota(order.begin(), order.end(), 0u);
    std::stable_sort(order.begin(), order.end(), [&](uint32_t a, uint32_t b) {
      return freq[base + a] > freq[base + b];
    });
    for (uint32_t i = 0; i < per_layer && !free_slots_.empty(); ++i) {
      Entry &en = entries_[base + order[i]];
      if (en.seg != Seg::None) continue;
      en.slot = free_slots_.back();
      free_slots_.pop_back();
      en.seg = Seg::Pinned;
      en.loaded = true;  // pinned experts are loaded during warm-up
      layers_[l].pinned++;
      layers_[l].resident++;
    }
  }
}

bool ExpertCache::acquire(uint32_t layer, uint32_t expert, Origin origin,
                          uint32_t *out_slot) {
  Entry &en = entries_[key(layer, expert)];
  Layer &L = layers_[layer];
  en.last_step = step_;

  if (en.seg != Seg::None) {  // hit
    stats_.hit++;
    if (en.freq < kFreqCap) en.freq++;
    en.refs++;
    if (en.seg == Seg::Pinned) {
      stats_.hit_pinned++;
    } else if (en.seg == Seg::Small) {
      stats_.hit_small++;
      // A second reference while in SMALL moves the expert to MAIN's tail.
      if (en.freq >= 2 && L.small.remove(expert)) {
        L.main.push_back(expert);
        en.seg = Seg::Main;
        stats_.promote++;
      }
    } else {
      stats_.hit_main++;
    }
    if (out_slot) *out_slot = en.slot;
    return true;
  }

  // miss
  stats_.miss++;
  en.freq = 1;
  const bool from_ghost = L.ghost.remove(expert);
  if (from_ghost) {
    L.ghost_hits++;
    stats_.ghost_hit++;
  }
  if (origin == Origin::Sweep) {  // sweeps never take a slot
    stats_.bypass++;
    if (out_slot) *out_slot = kNoSlot;
    return false;
  }
  const uint32_t s = take_slot(layer);
  if (s == kNoSlot) {  // every candidate is referenced: exhausted
    if (out_slot) *out_slot = kNoSlot;
    return false;
  }
  en.slot = s;
  en.refs = 1;
  en.loaded = false;
  stats_.admit++;
  if (from_ghost) {  // proven useful: straight to MAIN
    L.main.push_back(expert);
    en.seg = Seg::Main;
  } else if (origin == Origin::PrefetchLow) {  // first in line for eviction
    L.small.push_front(expert);
    en.seg = Seg::Small;
  } else {
    L.small.push_back(expert);
    en.seg = Seg::Small;
  }
  L.resident++;
  if (out_slot) *out_slot = s;
  return false;
}

void ExpertCache::mark_resident(uint32_t layer, uint32_t expert,
                                uint64_t nbytes) {
  Entry &en = entries_[key(layer, expert)];
  if (en.loaded) return;
  en.loaded = true;
  stats_.bytes_fetched += nbytes;
}

void ExpertCache::release(uint32_t layer, uint32_t expert) {
  Entry &en = entries_[key(layer, expert)];
  if (en.refs) en.refs--;
}

uint32_t ExpertCache::take_slot(uint32_t layer) {
  // Over quota: this layer gives one up first.
  if (layers_[layer].resident >= quota_[layer] && !evict_from(layer))
    return kNoSlot;
  if (free_slots_.empty()) {
    // Take one from the layer furthest over its quota that still holds an
    // unpinned expert; ties keep the earliest layer.
    uint32_t victim = layer;
    int32_t worst = INT32_MIN;
    for (uint32_t l = 0; l < cfg_.n_layer; ++l) {
      const int32_t over = int32_t(layers_[l].resident) - int32_t(quota_[l]);
      if (over > worst && layers_[l].resident > layers_[l].pinned) {
        worst = over;
        victim = l;
      }
    }
    if (!evict_from(victim) || free_slots_.empty()) return kNoSlot;
  }
  const uint32_t s = free_slots_.back();
  free_slots_.pop_back();
  return s;
}

bool ExpertCache::evict_from(uint32_t layer) {
  Layer &L = layers_[layer];
  // Sweep 0 walks SMALL from its head; sweep 1 walks MAIN granting one more
  // round to entries with freq > 1 (and spending it); sweep 2 walks MAIN with
  // no second chances. Referenced entries rotate to the tail untouched.
  for (int sweep = 0; sweep < 3; ++sweep) {
    Ring &q = sweep == 0 ? L.small : L.main;
    for (uint32_t left = q.size(); left > 0; --left) {
      const uint32_t e = q.front();
      q.pop_front();
      Entry &en = entries_[key(layer, e)];
      if (en.refs > 0 || (sweep == 1 && en.freq > 1)) {
        if (en.refs == 0) en.freq--;
        q.push_back(e);
        continue;
      }
      free_slots_.push_back(en.slot);
      en.slot = kNoSlot;
      en.seg = Seg::None;
      en.loaded = false;
      en.freq = 0;
      L.resident--;
      stats_.evict++;
      L.ghost.push_back(e);
      const size_t ghost_cap = size_t(quota_[layer]) * cfg_.ghost_mult;
      while (L.ghost.size() > ghost_cap) L.ghost.pop_front();
      return true;
    }
  }
  return false;
}

void ExpertCache::end_step() {
  step_++;
  if (cfg_.layer_quota_adapt && step_ % cfg_.quota_period == 0) rebalance();
}

void ExpertCache::rebalance() {
  // Layers with more ghost hits than average gain quota in proportion; the
  // total is renormalised to the slot count with a floor of quota_min.
  const uint32_t nl = cfg_.n_layer;
  double mean = 0;
  for (const Layer &L : layers_) mean += L.ghost_hits;
  mean /= double(nl);
  if (mean <= 0) {
    for (Layer &L : layers_) L.ghost_hits = 0;
    return;
  }
  std::vector<int64_t> q(nl);
  int64_t sum = 0;
  for (uint32_t l = 0; l < nl; ++l) {
    const double d = cfg_.quota_eta * (double(layers_[l].ghost_hits) - mean) /
                     mean * double(quota_[l]);
    int64_t v = int64_t(quota_[l]) + int64_t(d + (d >= 0 ? 0.5 : -0.5));
    v = std::min<int64_t>(std::max<int64_t>(v, cfg_.quota_min),
                          cfg_.n_expert);
    q[l] = v;
    sum += v;
  }
  const double scale = double(n_slot_) / double(sum);
  sum = 0;
  for (uint32_t l = 0; l < nl; ++l) {
    q[l] = std::max<int64_t>(cfg_.quota_min, int64_t(q[l] * scale));
    sum += q[l];
  }
  for (uint32_t l = 0; sum < int64_t(n_slot_); ++l) {
    q[l % nl]++;
    sum++;
  }
  for (uint32_t l = 0; l < nl; ++l) quota_[l] = uint32_t(q[l]);
  for (Layer &L : layers_) L.ghost_hits = 0;
}

std::string ExpertCache::quota_summary() const {
  const uint32_t nl = cfg_.n_layer;
  char buf[256];
  snprintf(buf, sizeof buf, "L0=%u L%u=%u L%u=%u L%u=%u L%u=%u", quota_[0],
           nl / 4, quota_[nl / 4], nl / 2, quota_[nl / 2], 3 * nl / 4,
           quota_[3 * nl / 4], nl - 1, quota_[nl - 1]);
  return buf;
}

}  // namespace moestream
