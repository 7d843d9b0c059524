// ref_shim.cpp -- C entry points over the reference's own ExpertCache.
//
// TEST INFRASTRUCTURE ONLY: the checker for the product's expert cache and
// remap. Linked by oracle/Makefile against the reference source
// src/expert_cache.cpp compiled where it lies (the reference is not copied
// into this repository); the result goes to oracle/_ref/libref_cache.so.
//
// orc_remap_call restates the decode remap loop of ms_remap_fn
// (src/llama-moestream.cpp:1799-2105) over that cache, without its
// diagnostics (sweep passes, drop mode, no-op levels):
//   - release every reference this layer took on its previous call
//     (:1839-1852);
//   - for each (t, k) in order (:1900-1952): out-of-range id -> zero slot;
//     acquire(Demand); NO_SLOT -> zero slot (exhaustion, :1913-1928);
//     a miss is appended to the pending list and marked resident at once
//     (:1940-1945); the id is held until the next call.
#include <cstdint>
#include <cstring>
#include <vector>

#include "expert_cache.hpp"

using moestream::CacheStats;
using moestream::ExpertCache;
using moestream::Origin;

namespace {
struct RemapState {
  ExpertCache cache;
  std::vector<uint32_t> held;
  uint32_t n_expert, n_slot;
  uint64_t exhausted = 0;
  RemapState(const ExpertCache::Config &c, uint32_t ne, uint32_t ns)
      : cache(c), n_expert(ne), n_slot(ns) {}
};
}  // namespace

extern "C" {

void *orc_cache_new_cfg(uint32_t n_layer, uint32_t n_expert, uint32_t n_slot, double cache_frac,
                        double pin_ratio, double small_ratio, uint32_t ghost_mult, int adapt,
                        uint32_t quota_period, double quota_eta, uint32_t quota_min) {
  ExpertCache::Config c;
  c.n_layer = n_layer;
  c.n_expert = n_expert;
  c.n_slot = n_slot;
  c.cache_frac = cache_frac;
  c.pin_ratio = pin_ratio;
  c.small_ratio = small_ratio;
  c.ghost_mult = ghost_mult;
  c.layer_quota_adapt = adapt != 0;
  c.quota_period = quota_period;
  c.quota_eta = quota_eta;
  c.quota_min = quota_min;
  return new ExpertCache(c);
}

void orc_cache_free(void *c) { delete static_cast<ExpertCache *>(c); }

int orc_cache_acquire(void *c, uint32_t layer, uint32_t e, int origin, uint32_t *slot) {
  return static_cast<ExpertCache *>(c)->acquire(layer, e, Origin(origin), slot) ? 1 : 0;
}
void orc_cache_mark_resident(void *c, uint32_t layer, uint32_t e, uint64_t nbytes) {
  static_cast<ExpertCache *>(c)->mark_resident(layer, e, nbytes);
}
void orc_cache_release(void *c, uint32_t layer, uint32_t e) {
  static_cast<ExpertCache *>(c)->release(layer, e);
}
void orc_cache_end_step(void *c) { static_cast<ExpertCache *>(c)->end_step(); }
uint32_t orc_cache_slot_of(void *c, uint32_t layer, uint32_t e) {
  return static_cast<ExpertCache *>(c)->slot_of(layer, e);
}
void orc_cache_build_pinned(void *c, const uint32_t *freq, size_t n) {
  static_cast<ExpertCache *>(c)->build_pinned(std::vector<uint32_t>(freq, freq + n));
}
void orc_cache_quota(void *c, uint32_t *out) {
  const std::vector<uint32_t> q = static_cast<ExpertCache *>(c)->layer_quota();
  std::memcpy(out, q.data(), q.size() * sizeof(uint32_t));
}
void orc_cache_stats(void *c, uint64_t *out) {
  const CacheStats &s = static_cast<ExpertCache *>(c)->stats();
  const uint64_t v[11] = {s.hit,   s.miss,  s.hit_pinned, s.hit_small, s.hit_main,     s.ghost_hit,
                          s.admit, s.evict, s.bypass,     s.promote,   s.bytes_fetched};
  std::memcpy(out, v, sizeof v);
}

// One layer's remap state, configured as finalize does
// (src/llama-moestream.cpp:1438-1447).
void *orc_remap_new(uint32_t n_expert, uint32_t n_slot) {
  ExpertCache::Config c;
  c.n_layer = 1;
  c.n_expert = n_expert;
  c.n_slot = n_slot;
  c.pin_ratio = 0.0;
  c.layer_quota_adapt = false;
  return new RemapState(c, n_expert, n_slot);
}
void orc_remap_free(void *s) { delete static_cast<RemapState *>(s); }

int orc_remap_call(void *sp, const int32_t *ids, int64_t nb0, int64_t nb1, int tk, int nt,
                   uint64_t expert_bytes, int32_t *out, int32_t *pend_e, int32_t *pend_s,
                   int32_t *n_pend) {
  RemapState &st = *static_cast<RemapState *>(sp);
  for (uint32_t e : st.held) st.cache.release(0, e);
  st.held.clear();
  const char *src = reinterpret_cast<const char *>(ids);
  const int32_t zero = int32_t(st.n_slot);
  int32_t np = 0;
  for (int j = 0; j < nt; ++j) {
    for (int k = 0; k < tk; ++k) {
      int32_t e;
      std::memcpy(&e, src + size_t(j) * nb1 + size_t(k) * nb0, sizeof e);
      int32_t sid = zero;
      if (e >= 0 && uint32_t(e) < st.n_expert) {
        uint32_t slot = 0;
        const bool hit = st.cache.acquire(0, uint32_t(e), Origin::Demand, &slot);
        if (slot == 0xFFFFFFFFu) {
          st.exhausted++;
          out[size_t(j) * tk + k] = zero;
          continue;
        }
        if (!hit) {
          pend_e[np] = e;
          pend_s[np] = int32_t(slot);
          np++;
          st.cache.mark_resident(0, uint32_t(e), expert_bytes);
        }
        sid = int32_t(slot);
        st.held.push_back(uint32_t(e));
      }
      out[size_t(j) * tk + k] = sid;
    }
  }
  *n_pend = np;
  return 0;
}

void orc_remap_stats(void *sp, uint64_t *out, uint64_t *exhausted) {
  RemapState &st = *static_cast<RemapState *>(sp);
  orc_cache_stats(&st.cache, out);
  *exhausted = st.exhausted;
}

}  // extern "C"
