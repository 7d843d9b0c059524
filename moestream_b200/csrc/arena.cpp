// Prefill arena on the device: every expert of one layer resident in HBM,
// loaded from the GGUF, with the next layer's load running in the background.
//
// The reference switches a micro-batch whose expected expert union exceeds
// the slots to a per-layer arena holding all n_expert experts, so that ids
// index experts directly (prefill_exps, src/llama-moestream.cpp:2147-2155).
// load_layer_arena (:2167-2283) reads into arena il % n_buf the experts the
// batch needs (the union, or all of them) that the arena does not already
// hold for that layer, resetting what it holds when the arena switches
// layers. pf_kick (:2285-2317) starts that load for the next layer on a
// background thread, using the same layer's union from the previous pass as
// the hint (all experts on the first pass); whatever the hint missed is read
// once the ids are known, so a bad hint never changes the output.
//
// Here an arena buffer is three slot pools (gate, up, down) with one slot per
// expert (slot e = expert e, slot n_expert the zero slot), so the
// ids route through msb_remap_group with no table and the FFN runs unchanged.
// The reads are the GGUF source's (pinned staging, parallel preads) and the
// uploads are stream-ordered on the caller's copy stream. Two events per
// buffer order the streams: `filled` (after its last upload; the compute
// stream waits on it in msb_arena_ready) and `used` (after the last kernel
// that reads it; its next load waits on it before writing slots).
#include <cuda_runtime.h>

#include <array>
#include <string>
#include <thread>
#include <vector>

#include "msb_internal.h"

using msb::fail;

struct msb_arena_s {
  msb_gguf_t g = nullptr;
  int32_t n_layer = 0, n_expert = 0, n_buf = 0, n_threads = 1, device = 0;
  std::vector<std::array<int64_t, 3>> tensor;  // per layer and role, -1 if absent
  struct Buf {
    msb_pool_t pool[3] = {nullptr, nullptr, nullptr};
    int type[3] = {-1, -1, -1};
    int64_t K[3] = {0, 0, 0}, N[3] = {0, 0, 0};
    int32_t layer = -1;
    std::vector<uint8_t> have;
    cudaEvent_t filled = nullptr, used = nullptr;
    bool used_recorded = false;
  };
  std::vector<Buf> bufs;
  std::thread pf;
  int32_t pf_layer = -1;
  int pf_rc = MSB_OK;
  std::string pf_err;
  msb_arena_stats_t stats{};

  ~msb_arena_s() {
    if (pf.joinable()) pf.join();
    for (Buf &b : bufs) {
      if (b.filled) cudaEventSynchronize(b.filled);
      if (b.used) cudaEventSynchronize(b.used);
      for (msb_pool_t p : b.pool)
        if (p) msb_pool_destroy(p);
      if (b.filled) cudaEventDestroy(b.filled);
      if (b.used) cudaEventDestroy(b.used);
    }
    if (g) msb_gguf_close(g);
  }
};

namespace {

// Joins the background load, if any; returns its status (message restored on
// the calling thread).
int join_prefetch(msb_arena_s *a) {
  if (!a->pf.joinable()) return MSB_OK;
  a->pf.join();
  a->pf_layer = -1;
  const int rc = a->pf_rc;
  a->pf_rc = MSB_OK;
  if (rc != MSB_OK) return fail(rc, "arena prefetch: %s", a->pf_err.c_str());
  return MSB_OK;
}

// (Re)creates the buffer's pool for `role` when the layer's tensor has another
// type or shape (per-layer quantization types differ in some models).
int ensure_pool(msb_arena_s *a, msb_arena_s::Buf &b, int role, const msb_gguf_tensor_t &t) {
  if (b.pool[role] && b.type[role] == t.type && b.K[role] == t.ne[0] && b.N[role] == t.ne[1])
    return MSB_OK;
  if (b.pool[role]) {
    if (b.used_recorded) MSB_CUDA_TRY(cudaEventSynchronize(b.used));
    MSB_CUDA_TRY(cudaEventSynchronize(b.filled));
    msb_pool_destroy(b.pool[role]);
    b.pool[role] = nullptr;
  }
  const int rc = msb_pool_create(t.type, t.ne[0], t.ne[1], a->n_expert, 0, &b.pool[role]);
  if (rc != MSB_OK) return rc;
  b.type[role] = t.type;
  b.K[role] = t.ne[0];
  b.N[role] = t.ne[1];
  return MSB_OK;
}

int load(msb_arena_s *a, int32_t il, const uint8_t *need, cudaStream_t st) {
  MSB_CHECK_ARG(il >= 0 && il < a->n_layer, "arena: layer %d of %d", il, a->n_layer);
  for (int r = 0; r < 3; ++r)
    MSB_CHECK_ARG(a->tensor[size_t(il)][size_t(r)] >= 0,
                  "arena: layer %d has no expert tensor for role %d", il, r);
  msb_arena_s::Buf &b = a->bufs[size_t(il % a->n_buf)];
  msb_gguf_tensor_t t[3];
  for (int r = 0; r < 3; ++r) {
    int rc = msb_gguf_tensor_info(a->g, a->tensor[size_t(il)][size_t(r)], &t[r]);
    if (rc != MSB_OK) return rc;
    rc = ensure_pool(a, b, r, t[r]);
    if (rc != MSB_OK) return rc;
  }
  if (b.layer != il) {
    b.have.assign(size_t(a->n_expert), 0);
    b.layer = il;
  }
  std::vector<int32_t> ex;
  for (int32_t e = 0; e < a->n_expert; ++e)
    if ((!need || need[e]) && !b.have[size_t(e)]) ex.push_back(e);
  a->stats.experts_asked += uint64_t(a->n_expert);
  if (ex.empty()) {
    ++a->stats.hits;
    return MSB_OK;
  }
  // Slots of this buffer may still be read by the layer it held before; and
  // `filled` must cover the uploads of earlier loads made on other streams.
  if (b.used_recorded) MSB_CUDA_TRY(cudaStreamWaitEvent(st, b.used, 0));
  MSB_CUDA_TRY(cudaStreamWaitEvent(st, b.filled, 0));
  // Chunks of kChunk experts per role bound the pinned staging (two chunks)
  // and let the reads of one chunk overlap the uploads of the one before.
  constexpr int32_t kChunk = 8;
  const int32_t n = int32_t(ex.size());
  for (int32_t c0 = 0; c0 < n; c0 += kChunk) {
    const int32_t m = n - c0 < kChunk ? n - c0 : kChunk;
    for (int r = 0; r < 3; ++r) {
      const int rc = msb_gguf_fill_slots_async(a->g, a->tensor[size_t(il)][size_t(r)],
                                               b.pool[r], m, ex.data() + c0, ex.data() + c0,
                                               a->n_threads, st);
      if (rc != MSB_OK) {
        b.layer = -1;  // partly written: hold nothing
        return rc;
      }
      a->stats.bytes_read += uint64_t(t[r].nbytes / t[r].ne[2]) * uint64_t(m);
    }
  }
  MSB_CUDA_TRY(cudaEventRecord(b.filled, st));
  for (int32_t e : ex) b.have[size_t(e)] = 1;
  a->stats.experts_read += uint64_t(n);
  ++a->stats.loads;
  return MSB_OK;
}

}  // namespace

extern "C" {

int msb_arena_create(const char *gguf_path, int32_t n_buf, int32_t n_threads,
                     msb_arena_t *out) {
  MSB_CHECK_ARG(gguf_path && out && n_buf >= 1, "msb_arena_create: bad argument");
  *out = nullptr;
  msb_arena_s *a = new (std::nothrow) msb_arena_s();
  if (!a) return fail(MSB_ERR_NOMEM, "msb_arena_create: out of memory");
  int rc = msb_gguf_open(gguf_path, &a->g);
  if (rc != MSB_OK) {
    delete a;
    return rc;
  }
  int64_t n_layer = 0;
  if (msb_gguf_kv_int(a->g, ".block_count", &n_layer) != MSB_OK || n_layer <= 0) {
    n_layer = 0;  // no metadata: the highest layer with expert tensors
    for (int32_t il = 0; il < 4096; ++il)
      if (msb_gguf_expert_tensor(a->g, il, MSB_ROLE_GATE) >= 0) n_layer = il + 1;
  }
  msb::clear_error();
  a->n_layer = int32_t(n_layer);
  a->tensor.resize(size_t(n_layer));
  for (int32_t il = 0; il < a->n_layer; ++il) {
    for (int r = 0; r < 3; ++r) {
      const int64_t ti = msb_gguf_expert_tensor(a->g, il, r);
      a->tensor[size_t(il)][size_t(r)] = ti;
      if (ti < 0) continue;
      msb_gguf_tensor_t t;
      msb_gguf_tensor_info(a->g, ti, &t);
      if (a->n_expert == 0) a->n_expert = int32_t(t.ne[2]);
      if (t.ne[2] != a->n_expert) {
        const int rc2 = fail(MSB_ERR_INVALID, "arena: %s has %lld experts, the others %d",
                             t.name, (long long)t.ne[2], a->n_expert);
        delete a;
        return rc2;
      }
    }
  }
  if (a->n_expert <= 1) {
    delete a;
    return fail(MSB_ERR_INVALID, "arena: %s has no expert tensors", gguf_path);
  }
  a->n_buf = n_buf;
  a->n_threads = n_threads < 1 ? 1 : n_threads;
  cudaGetDevice(&a->device);
  a->bufs.resize(size_t(n_buf));
  // Pools for the first complete layer's shapes are made here (creation
  // synchronizes the device); a background load only makes new ones for a
  // layer of another type or shape.
  int32_t first = -1;
  for (int32_t il = 0; il < a->n_layer && first < 0; ++il)
    if (a->tensor[size_t(il)][0] >= 0 && a->tensor[size_t(il)][1] >= 0 &&
        a->tensor[size_t(il)][2] >= 0)
      first = il;
  for (msb_arena_s::Buf &b : a->bufs) {
    if (cudaEventCreateWithFlags(&b.filled, cudaEventDisableTiming) != cudaSuccess ||
        cudaEventCreateWithFlags(&b.used, cudaEventDisableTiming) != cudaSuccess) {
      delete a;
      return fail(MSB_ERR_CUDA, "arena: cudaEventCreate failed");
    }
    for (int r = 0; r < 3 && first >= 0; ++r) {
      msb_gguf_tensor_t t;
      msb_gguf_tensor_info(a->g, a->tensor[size_t(first)][size_t(r)], &t);
      rc = ensure_pool(a, b, r, t);
      if (rc != MSB_OK) {
        delete a;
        return rc;
      }
    }
  }
  *out = a;
  return MSB_OK;
}

int msb_arena_destroy(msb_arena_t a) {
  delete a;
  return MSB_OK;
}

int msb_arena_info(msb_arena_t a, int32_t *n_layer, int32_t *n_expert, int32_t *n_buf) {
  MSB_CHECK_ARG(a, "msb_arena_info: null arena");
  if (n_layer) *n_layer = a->n_layer;
  if (n_expert) *n_expert = a->n_expert;
  if (n_buf) *n_buf = a->n_buf;
  return MSB_OK;
}

int msb_arena_load(msb_arena_t a, int32_t layer, const uint8_t *need, void *stream) {
  MSB_CHECK_ARG(a, "msb_arena_load: null arena");
  int rc = join_prefetch(a);
  if (rc != MSB_OK) return rc;
  msb::clear_error();
  return load(a, layer, need, static_cast<cudaStream_t>(stream));
}

int msb_arena_prefetch(msb_arena_t a, int32_t layer, const uint8_t *hint, void *stream) {
  MSB_CHECK_ARG(a, "msb_arena_prefetch: null arena");
  MSB_CHECK_ARG(layer >= 0 && layer < a->n_layer, "msb_arena_prefetch: layer %d of %d", layer,
                a->n_layer);
  MSB_CHECK_ARG(a->n_buf >= 2, "msb_arena_prefetch: needs two arena buffers or more");
  int rc = join_prefetch(a);  // never more than one load in flight
  if (rc != MSB_OK) return rc;
  std::vector<uint8_t> h;
  if (hint) h.assign(hint, hint + a->n_expert);
  a->pf_layer = layer;
  a->pf = std::thread([a, layer, h = std::move(h), stream] {
    cudaSetDevice(a->device);
    const int r = load(a, layer, h.empty() ? nullptr : h.data(), static_cast<cudaStream_t>(stream));
    a->pf_rc = r;
    if (r != MSB_OK) a->pf_err = msb_last_error();
  });
  return MSB_OK;
}

int msb_arena_wait(msb_arena_t a) {
  MSB_CHECK_ARG(a, "msb_arena_wait: null arena");
  return join_prefetch(a);
}

int msb_arena_ready(msb_arena_t a, int32_t layer, void *compute_stream, msb_pool_t *gate,
                    msb_pool_t *up, msb_pool_t *down) {
  MSB_CHECK_ARG(a && gate && up && down, "msb_arena_ready: null argument");
  MSB_CHECK_ARG(layer >= 0 && layer < a->n_layer, "msb_arena_ready: layer %d of %d", layer,
                a->n_layer);
  msb_arena_s::Buf &b = a->bufs[size_t(layer % a->n_buf)];
  if (a->pf_layer >= 0 && a->pf_layer % a->n_buf == layer % a->n_buf) {
    const int rc = join_prefetch(a);
    if (rc != MSB_OK) return rc;
  }
  MSB_CHECK_ARG(b.layer == layer, "msb_arena_ready: the arena buffer holds layer %d, not %d",
                b.layer, layer);
  MSB_CUDA_TRY(cudaStreamWaitEvent(static_cast<cudaStream_t>(compute_stream), b.filled, 0));
  *gate = b.pool[0];
  *up = b.pool[1];
  *down = b.pool[2];
  return MSB_OK;
}

int msb_arena_release(msb_arena_t a, int32_t layer, void *compute_stream) {
  MSB_CHECK_ARG(a, "msb_arena_release: null arena");
  MSB_CHECK_ARG(layer >= 0 && layer < a->n_layer, "msb_arena_release: layer %d of %d", layer,
                a->n_layer);
  msb_arena_s::Buf &b = a->bufs[size_t(layer % a->n_buf)];
  if (a->pf_layer >= 0 && a->pf_layer % a->n_buf == layer % a->n_buf) {
    const int rc = join_prefetch(a);
    if (rc != MSB_OK) return rc;
  }
  MSB_CUDA_TRY(cudaEventRecord(b.used, static_cast<cudaStream_t>(compute_stream)));
  b.used_recorded = true;
  return MSB_OK;
}

int msb_arena_stats(msb_arena_t a, msb_arena_stats_t *out) {
  MSB_CHECK_ARG(a && out, "msb_arena_stats: null argument");
  const int rc = join_prefetch(a);
  *out = a->stats;
  return rc;
}

}  // extern "C"
