// The slot streamer's per-layer cache decisions as plain functions over one
// int32 state block, compiled for both the host and the device.
//
// This is the decision procedure of msb_streamer_remap (one ExpertCache per
// layer configured as the reference's finalize builds them:
// src/llama-moestream.cpp:1438-1447, n_layer 1, pin_ratio 0, no quota
// adaptation, so the layer's quota is all n_slot slots; demand requests
// only) and of the reference cache's acquire / release / eviction
// (src/expert_cache.cpp:62-224), restated over fixed arrays so that one
// CTA can run it out of shared memory. Given the same ids it produces the
// same slots, misses and counters as the host streamer; the tests compare
// both on random traces.
//
// State block of one layer (int32 words, offsets from dc_layout):
//   slot[E]   slot of each expert, -1 if none      refs[E]  references held
//   seg[E]    0 none, 2 SMALL, 3 MAIN               freq[E]  0..3
//   small[E], main[E], ghost[E]   FIFO rings of expert ids
//   free[n_slot]                  stack of free slots, top at free[n_free-1]
//   hdr: small head/n, main head/n, ghost head/n, n_free, resident, n_held
//   held[max_pairs]               experts this layer referenced last call
//   stats: 12 uint64 (hit, miss, hit_pinned, hit_small, hit_main,
//          ghost_hit, admit, evict, bypass, promote, bytes_fetched,
//          exhausted)
#pragma once

#include <cstdint>

#if defined(__CUDACC__)
#define MSB_HD __host__ __device__ __forceinline__
#else
#define MSB_HD inline
#endif

namespace msb {

enum : int32_t { kSegNone = 0, kSegSmall = 2, kSegMain = 3 };
enum : int { kStHit = 0, kStMiss, kStHitPinned, kStHitSmall, kStHitMain, kStGhostHit, kStAdmit,
             kStEvict, kStBypass, kStPromote, kStBytes, kStExhausted, kNumStats };
enum : int { kHdrSmallHead = 0, kHdrSmallN, kHdrMainHead, kHdrMainN, kHdrGhostHead, kHdrGhostN,
             kHdrFree, kHdrResident, kHdrHeld, kHdrWords = 16 };
constexpr int32_t kFreqCap = 3;
constexpr int32_t kGhostMult = 2;

struct DcLayout {
  int32_t E, n_slot, max_pairs;
  int32_t slot, refs, seg, freq, small, main, ghost, free_, hdr, held, stats, words;
};

MSB_HD DcLayout dc_layout(int32_t E, int32_t n_slot, int32_t max_pairs) {
  DcLayout L;
  L.E = E;
  L.n_slot = n_slot;
  L.max_pairs = max_pairs;
  L.slot = 0;
  L.refs = E;
  L.seg = 2 * E;
  L.freq = 3 * E;
  L.small = 4 * E;
  L.main = 5 * E;
  L.ghost = 6 * E;
  L.free_ = 7 * E;
  L.hdr = (7 * E + n_slot + 3) & ~3;
  L.held = L.hdr + kHdrWords;
  L.stats = (L.held + max_pairs + 3) & ~3;       // 16-byte aligned
  L.words = L.stats + 2 * kNumStats;
  L.words = (L.words + 3) & ~3;
  return L;
}

// Initial state: every slot free with slot 0 on top, empty queues.
MSB_HD void dc_init(int32_t *s, const DcLayout &L) {
  for (int32_t i = 0; i < L.words; ++i) s[i] = 0;
  for (int32_t e = 0; e < L.E; ++e) s[L.slot + e] = -1;
  for (int32_t i = 0; i < L.n_slot; ++i) s[L.free_ + i] = L.n_slot - 1 - i;
  s[L.hdr + kHdrFree] = L.n_slot;
}

struct DcRing {
  int32_t *buf, *head, *n;
  int32_t cap;
  MSB_HD int32_t wrap(int32_t i) const { return i >= cap ? i - cap : i; }
  MSB_HD int32_t front() const { return buf[*head]; }
  MSB_HD void pop_front() {
    *head = wrap(*head + 1);
    --*n;
  }
  MSB_HD void push_back(int32_t v) {
    buf[wrap(*head + *n)] = v;
    ++*n;
  }
  // Removes the first occurrence of v, keeping the order of the rest.
  MSB_HD bool remove(int32_t v) {
    for (int32_t i = 0; i < *n; ++i) {
      if (buf[wrap(*head + i)] != v) continue;
      for (int32_t j = i; j + 1 < *n; ++j) buf[wrap(*head + j)] = buf[wrap(*head + j + 1)];
      --*n;
      return true;
    }
    return false;
  }
};

struct DcState {
  int32_t *s;
  DcLayout L;
  MSB_HD int32_t &slot(int32_t e) const { return s[L.slot + e]; }
  MSB_HD int32_t &refs(int32_t e) const { return s[L.refs + e]; }
  MSB_HD int32_t &seg(int32_t e) const { return s[L.seg + e]; }
  MSB_HD int32_t &freq(int32_t e) const { return s[L.freq + e]; }
  MSB_HD int32_t &hdr(int i) const { return s[L.hdr + i]; }
  MSB_HD DcRing small() const { return DcRing{s + L.small, &hdr(kHdrSmallHead), &hdr(kHdrSmallN), L.E}; }
  MSB_HD DcRing main() const { return DcRing{s + L.main, &hdr(kHdrMainHead), &hdr(kHdrMainN), L.E}; }
  MSB_HD DcRing ghost() const { return DcRing{s + L.ghost, &hdr(kHdrGhostHead), &hdr(kHdrGhostN), L.E}; }
  MSB_HD void stat_add(int i, uint64_t v) const {
    uint64_t x = uint32_t(s[L.stats + 2 * i]) | uint64_t(uint32_t(s[L.stats + 2 * i + 1])) << 32;
    x += v;
    s[L.stats + 2 * i] = int32_t(uint32_t(x));
    s[L.stats + 2 * i + 1] = int32_t(uint32_t(x >> 32));
  }

  // Evicts one unreferenced expert (src/expert_cache.cpp:194-224): sweep 0
  // over SMALL, sweep 1 over MAIN granting one more round to freq > 1
  // (spending it), sweep 2 over MAIN without second chances; referenced
  // entries rotate to the tail.
  MSB_HD bool evict() const {
    for (int sweep = 0; sweep < 3; ++sweep) {
      DcRing q = sweep == 0 ? small() : main();
      for (int32_t left = *q.n; left > 0; --left) {
        const int32_t e = q.front();
        q.pop_front();
        if (refs(e) > 0 || (sweep == 1 && freq(e) > 1)) {
          if (refs(e) == 0) freq(e)--;
          q.push_back(e);
          continue;
        }
        s[L.free_ + hdr(kHdrFree)] = slot(e);
        hdr(kHdrFree)++;
        slot(e) = -1;
        seg(e) = kSegNone;
        freq(e) = 0;
        hdr(kHdrResident)--;
        stat_add(kStEvict, 1);
        DcRing g = ghost();
        g.push_back(e);
        while (*g.n > L.n_slot * kGhostMult) g.pop_front();
        return true;
      }
    }
    return false;
  }

  // A slot for a newly admitted expert, -1 when every candidate is
  // referenced (src/expert_cache.cpp:169-192 with one layer whose quota is
  // every slot).
  MSB_HD int32_t take_slot() const {
    if (hdr(kHdrResident) >= L.n_slot && !evict()) return -1;
    if (hdr(kHdrFree) == 0) {
      if (!evict() || hdr(kHdrFree) == 0) return -1;
    }
    hdr(kHdrFree)--;
    return s[L.free_ + hdr(kHdrFree)];
  }

  // Demand acquire (src/expert_cache.cpp:62-153). Returns true on a hit;
  // *out = slot or -1 (exhausted).
  MSB_HD bool acquire(int32_t e, int32_t *out) const {
    if (seg(e) != kSegNone) {
      stat_add(kStHit, 1);
      if (freq(e) < kFreqCap) freq(e)++;
      refs(e)++;
      if (seg(e) == kSegSmall) {
        stat_add(kStHitSmall, 1);
        if (freq(e) >= 2) {
          DcRing sm = small();
          if (sm.remove(e)) {
            main().push_back(e);
            seg(e) = kSegMain;
            stat_add(kStPromote, 1);
          }
        }
      } else {
        stat_add(kStHitMain, 1);
      }
      *out = slot(e);
      return true;
    }
    stat_add(kStMiss, 1);
    freq(e) = 1;
    const bool from_ghost = ghost().remove(e);
    if (from_ghost) stat_add(kStGhostHit, 1);
    const int32_t sl = take_slot();
    if (sl < 0) {
      *out = -1;
      return false;
    }
    slot(e) = sl;
    refs(e) = 1;
    stat_add(kStAdmit, 1);
    if (from_ghost) {
      main().push_back(e);
      seg(e) = kSegMain;
    } else {
      small().push_back(e);
      seg(e) = kSegSmall;
    }
    hdr(kHdrResident)++;
    *out = sl;
    return false;
  }
};

// One layer's decode remap (msb_streamer_remap): drop the previous call's
// references, then acquire every (t, k) in order. ids are dense in pair
// order (p = t * top_k + k). out_slots[p] = slot, or n_slot (the zero slot)
// for an invalid id or on exhaustion; misses are appended in first-seen
// order. Returns the miss count.
MSB_HD int32_t dc_remap(int32_t *s, const DcLayout &L, const int32_t *ids, int32_t n_pairs,
                        uint64_t expert_bytes, int32_t *out_slots, int32_t *miss_e,
                        int32_t *miss_s) {
  DcState st{s, L};
  int32_t *held = s + L.held;
  for (int32_t i = 0; i < st.hdr(kHdrHeld); ++i)
    if (st.refs(held[i]) > 0) st.refs(held[i])--;
  st.hdr(kHdrHeld) = 0;
  int32_t nm = 0;
  for (int32_t p = 0; p < n_pairs; ++p) {
    const int32_t e = ids[p];
    int32_t sid = L.n_slot;
    if (e >= 0 && e < L.E) {
      int32_t sl;
      const bool hit = st.acquire(e, &sl);
      if (sl < 0) {
        st.stat_add(kStExhausted, 1);
      } else {
        if (!hit) {
          miss_e[nm] = e;
          miss_s[nm] = sl;
          ++nm;
          st.stat_add(kStBytes, expert_bytes);
        }
        sid = sl;
        held[st.hdr(kHdrHeld)++] = e;
      }
    }
    out_slots[p] = sid;
  }
  return nm;
}

}  // namespace msb
