// Host half of the C ABI: errors, slab sizing, the expert cache and the slot
// streamer (the host side of the reference's ms_remap_fn).
#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <new>
#include <vector>

#include "expert_cache.hpp"
#include "msb_internal.h"

namespace msb {

static thread_local char g_err[512];

int fail(int code, const char *fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof g_err, fmt, ap);
  va_end(ap);
  return code;
}
void clear_error() { g_err[0] = 0; }

static std::atomic<uint64_t> g_launches{0};
void count_launch(int n) { g_launches.fetch_add(uint64_t(n), std::memory_order_relaxed); }

}  // namespace msb

using moestream::ExpertCache;
using moestream::Origin;

struct msb_cache_s {
  ExpertCache cache;
  explicit msb_cache_s(const ExpertCache::Config &c) : cache(c) {}
};

// Per-layer caches plus the references each layer holds until its next call.
struct msb_streamer_s {
  uint32_t n_expert = 0, n_slot = 0;
  uint64_t expert_bytes = 0;
  std::vector<ExpertCache> caches;
  std::vector<std::vector<uint32_t>> held;
  uint64_t exhausted = 0;
};

static void fill_stats(const moestream::CacheStats &s, msb_cache_stats_t *o) {
  o->hit = s.hit; o->miss = s.miss; o->hit_pinned = s.hit_pinned;
  o->hit_small = s.hit_small; o->hit_main = s.hit_main;
  o->ghost_hit = s.ghost_hit; o->admit = s.admit; o->evict = s.evict;
  o->bypass = s.bypass; o->promote = s.promote;
  o->bytes_fetched = s.bytes_fetched;
}

extern "C" {

int msb_version(void) { return 100; }

uint64_t msb_kernel_launches(void) { return msb::g_launches.load(); }

const char *msb_last_error(void) { return msb::g_err; }

int64_t msb_expert_bytes(int wtype, int64_t K, int64_t N) {
  msb::BlockFormat f;
  if (!msb::block_format(wtype, &f) || K <= 0 || N <= 0 || K % 32) return -1;
  return (K / 32) * f.block_bytes * N;
}

uint32_t msb_slab_slots(int64_t n_expert, double frac, int top_k,
                        int max_ubatch) {
  // Plain-fraction sizing of slab_slots (src/llama-moestream.cpp:1017-1086):
  // round(frac * n_expert), then at least the expected union of one
  // micro-batch's experts, n*(1-(1-k/n)^ub), times 1.15 plus top_k.
  if (n_expert <= 1) return 0;
  uint32_t s = uint32_t(double(n_expert) * frac + 0.5);
  const double tk = top_k > 0 ? double(top_k) : 8.0;
  const double u = double(n_expert) *
                   (1.0 - std::pow(1.0 - tk / double(n_expert),
                                   double(max_ubatch > 0 ? max_ubatch : 2)));
  const uint32_t need = uint32_t(
      std::min<int64_t>(n_expert, int64_t(u * 1.15) + int64_t(tk)));
  s = std::max(s, need);
  s = std::max<uint32_t>(8, std::min<uint32_t>(s, uint32_t(n_expert)));
  return s;
}

int msb_arena_threshold(int64_t n_expert, int top_k, uint32_t n_slot) {
  // Largest n with union(n + 1) * 1.15 + top_k <= n_slot, starting at 1
  // (src/llama-moestream.cpp:1530-1543).
  const double tk = double(top_k > 0 ? top_k : 8);
  int n = 1;
  while (n < 4096) {
    const double u = double(n_expert) *
                     (1.0 - std::pow(1.0 - tk / double(n_expert), double(n + 1)));
    if (u * 1.15 + tk > double(n_slot)) break;
    ++n;
  }
  return n;
}

void msb_cache_config_default(msb_cache_config_t *cfg) {
  const ExpertCache::Config d;
  cfg->n_layer = d.n_layer; cfg->n_expert = d.n_expert; cfg->n_slot = d.n_slot;
  cfg->cache_frac = d.cache_frac; cfg->pin_ratio = d.pin_ratio;
  cfg->small_ratio = d.small_ratio; cfg->ghost_mult = d.ghost_mult;
  cfg->layer_quota_adapt = d.layer_quota_adapt ? 1 : 0;
  cfg->quota_period = d.quota_period; cfg->quota_eta = d.quota_eta;
  cfg->quota_min = d.quota_min;
}

int msb_cache_create(const msb_cache_config_t *cfg, msb_cache_t *out) {
  MSB_CHECK_ARG(cfg && out, "msb_cache_create: null argument");
  MSB_CHECK_ARG(cfg->n_layer > 0 && cfg->n_expert > 0,
                "msb_cache_create: n_layer and n_expert must be positive");
  MSB_CHECK_ARG(cfg->quota_period > 0 || !cfg->layer_quota_adapt,
                "msb_cache_create: quota_period must be positive");
  ExpertCache::Config c;
  c.n_layer = cfg->n_layer; c.n_expert = cfg->n_expert; c.n_slot = cfg->n_slot;
  c.cache_frac = cfg->cache_frac; c.pin_ratio = cfg->pin_ratio;
  c.small_ratio = cfg->small_ratio; c.ghost_mult = cfg->ghost_mult;
  c.layer_quota_adapt = cfg->layer_quota_adapt != 0;
  c.quota_period = cfg->quota_period; c.quota_eta = cfg->quota_eta;
  c.quota_min = cfg->quota_min;
  *out = new (std::nothrow) msb_cache_s(c);
  return *out ? MSB_OK : msb::fail(MSB_ERR_NOMEM, "msb_cache_create: out of memory");
}

void msb_cache_destroy(msb_cache_t c) { delete c; }

int msb_cache_acquire(msb_cache_t c, uint32_t layer, uint32_t expert,
                      int origin, uint32_t *slot) {
  return c->cache.acquire(layer, expert, Origin(origin), slot) ? 1 : 0;
}
void msb_cache_mark_resident(msb_cache_t c, uint32_t layer, uint32_t expert,
                             uint64_t nbytes) {
  c->cache.mark_resident(layer, expert, nbytes);
}
void msb_cache_release(msb_cache_t c, uint32_t layer, uint32_t expert) {
  c->cache.release(layer, expert);
}
void msb_cache_end_step(msb_cache_t c) { c->cache.end_step(); }
void msb_cache_build_pinned(msb_cache_t c, const uint32_t *freq, size_t n) {
  c->cache.build_pinned(std::vector<uint32_t>(freq, freq + n));
}
void msb_cache_get_stats(msb_cache_t c, msb_cache_stats_t *out) {
  fill_stats(c->cache.stats(), out);
}
uint32_t msb_cache_n_slot(msb_cache_t c) { return c->cache.n_slot(); }
uint32_t msb_cache_slot_of(msb_cache_t c, uint32_t layer, uint32_t expert) {
  return c->cache.slot_of(layer, expert);
}
void msb_cache_layer_quota(msb_cache_t c, uint32_t *out) {
  const std::vector<uint32_t> q = c->cache.layer_quota();
  std::copy(q.begin(), q.end(), out);
}

int msb_streamer_create(uint32_t n_layer, uint32_t n_expert, uint32_t n_slot,
                        uint64_t expert_bytes_total, msb_streamer_t *out) {
  MSB_CHECK_ARG(out && n_layer > 0 && n_expert > 0 && n_slot > 0,
                "msb_streamer_create: bad arguments");
  msb_streamer_s *s = new (std::nothrow) msb_streamer_s();
  if (!s) return msb::fail(MSB_ERR_NOMEM, "msb_streamer_create: out of memory");
  s->n_expert = n_expert;
  s->n_slot = n_slot;
  s->expert_bytes = expert_bytes_total;
  // One cache per layer, configured as finalize does
  // (src/llama-moestream.cpp:1438-1447).
  ExpertCache::Config cfg;
  cfg.n_layer = 1;
  cfg.n_expert = n_expert;
  cfg.n_slot = n_slot;
  cfg.pin_ratio = 0.0;
  cfg.layer_quota_adapt = false;
  s->caches.reserve(n_layer);
  for (uint32_t l = 0; l < n_layer; ++l) s->caches.emplace_back(cfg);
  s->held.assign(n_layer, {});
  *out = s;
  return MSB_OK;
}

void msb_streamer_destroy(msb_streamer_t s) { delete s; }

int msb_streamer_remap(msb_streamer_t s, uint32_t layer, const int32_t *ids,
                       int64_t nb0, int64_t nb1, int32_t top_k, int32_t n_tok,
                       int32_t *out_slots, int32_t *n_miss,
                       int32_t *miss_experts, int32_t *miss_slots,
                       int32_t *table_out) {
  MSB_CHECK_ARG(s && ids && out_slots && n_miss && miss_experts && miss_slots,
                "msb_streamer_remap: null argument");
  MSB_CHECK_ARG(layer < s->caches.size(), "msb_streamer_remap: layer %u out of range",
                layer);
  MSB_CHECK_ARG(top_k > 0 && n_tok >= 0, "msb_streamer_remap: bad shape");
  ExpertCache &cache = s->caches[layer];
  std::vector<uint32_t> &held = s->held[layer];
  // The previous call's mul_mat_id has finished by the time this layer runs
  // again, so its references can be dropped before new ones are taken.
  for (uint32_t e : held) cache.release(0, e);
  held.clear();
  const int32_t zero_slot = int32_t(s->n_slot);
  const char *base = reinterpret_cast<const char *>(ids);
  int32_t nm = 0;
  for (int32_t t = 0; t < n_tok; ++t) {
    for (int32_t k = 0; k < top_k; ++k) {
      int32_t e;
      std::memcpy(&e, base + int64_t(k) * nb0 + int64_t(t) * nb1, sizeof e);
      int32_t sid = zero_slot;
      if (e >= 0 && uint32_t(e) < s->n_expert) {
        uint32_t slot = 0;
        const bool hit = cache.acquire(0, uint32_t(e), Origin::Demand, &slot);
        if (slot == ExpertCache::kNoSlot) {
          // Exhausted: a wrong slot would corrupt the output, the zero slot
          // only drops this expert's contribution.
          s->exhausted++;
        } else {
          if (!hit) {
            miss_experts[nm] = e;
            miss_slots[nm] = int32_t(slot);
            nm++;
            cache.mark_resident(0, uint32_t(e), s->expert_bytes);
          }
          sid = int32_t(slot);
          held.push_back(uint32_t(e));
        }
      }
      out_slots[int64_t(t) * top_k + k] = sid;
    }
  }
  *n_miss = nm;
  if (table_out) {
    for (uint32_t e = 0; e < s->n_expert; ++e) {
      const uint32_t sl = cache.slot_of(0, e);
      table_out[e] = sl == ExpertCache::kNoSlot ? -1 : int32_t(sl);
    }
  }
  return MSB_OK;
}

int msb_streamer_stats(msb_streamer_t s, msb_cache_stats_t *out,
                       uint64_t *n_exhausted) {
  MSB_CHECK_ARG(s && out, "msb_streamer_stats: null argument");
  moestream::CacheStats sum;
  for (const ExpertCache &c : s->caches) {
    const moestream::CacheStats &x = c.stats();
    sum.hit += x.hit; sum.miss += x.miss; sum.hit_pinned += x.hit_pinned;
    sum.hit_small += x.hit_small; sum.hit_main += x.hit_main;
    sum.ghost_hit += x.ghost_hit; sum.admit += x.admit; sum.evict += x.evict;
    sum.bypass += x.bypass; sum.promote += x.promote;
    sum.bytes_fetched += x.bytes_fetched;
  }
  fill_stats(sum, out);
  if (n_exhausted) *n_exhausted = s->exhausted;
  return MSB_OK;
}

}  // extern "C"
