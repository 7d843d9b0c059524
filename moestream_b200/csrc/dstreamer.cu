// Device slot streamer: the decode remap with no host round trip.
//
// The reference's decode remap (ms_remap_fn, src/llama-moestream.cpp:
// 1799-2105) is a CPU op: every layer the router's ids travel to the host,
// the ExpertCache decides, missing experts are read and uploaded, and the
// slot ids travel back (2.24 ms of GPU<->CPU synchronisation per token on
// the reference's hardware). Its own stated fix is a device-resident slot
// table with the miss queue in mapped memory.
//
// Here the whole decision runs on the device, in stream order:
//   dc_remap_kernel   one CTA: loads the layer's cache state (dcache.cuh) and
//                     its ids into shared memory, one thread runs the
//                     streamer's decisions (the same code the host path
//                     compiles), the CTA writes back the state, the slot ids
//                     and the miss queue (experts and slots, first-seen
//                     order), into device memory for the fills and into
//                     mapped pinned memory for the host;
//   dfill_kernel      copies each missed expert (of up to three roles in one
//                     launch), in ggml layout, from pinned
//                     host memory (read by the kernel over the bus) or device
//                     memory into its slot, repacking into the pool layout;
//                     it reads the miss count from the device copy of the
//                     queue, so the launch does not depend on it (reading it
//                     from the mapped copy in every CTA serialises on the
//                     bus: 1.8 ms per launch with nothing to fill);
// after which msb_remap_group groups the slot ids (no table) and the FFN
// runs. Every launch is stream-ordered with no host decision between them,
// so a whole decode step, misses and fills included, can be captured in a
// CUDA graph. A streamer made with on_host runs the identical decisions on
// the host (for tests on machines without a GPU).
#include <cuda_runtime.h>

#include <cstring>
#include <new>
#include <vector>

#include "dcache.cuh"
#include "msb_internal.h"
#include "pool.cuh"

using msb::fail;

struct msb_dstreamer_s {
  bool on_host = false;
  int device = 0;
  uint32_t n_layer = 0;
  msb::DcLayout L{};
  uint64_t expert_bytes = 0;
  int32_t *state = nullptr;     // n_layer blocks of L.words (device, or host when on_host)
  int32_t *queue = nullptr;     // pinned, mapped: per layer [n_miss, 3 pad, experts, slots]
  int32_t *queue_dev = nullptr; // device address of `queue`
  int32_t *dqueue = nullptr;    // device-memory copy the fill kernels read
  int64_t queue_words = 0;      // per layer
  size_t remap_smem = 0;

  ~msb_dstreamer_s() {
    if (on_host) {
      delete[] state;
      delete[] queue;
      return;
    }
    if (state) cudaFree(state);
    if (dqueue) cudaFree(dqueue);
    if (queue) cudaFreeHost(queue);
  }
  int32_t *layer_queue(uint32_t l) const { return queue + int64_t(l) * queue_words; }
};

namespace msb {
namespace {

constexpr int kRemapThreads = 256;

__global__ void __launch_bounds__(kRemapThreads) dc_remap_kernel(
    int32_t *state, DcLayout L, const char *ids, int64_t nb0, int64_t nb1, int32_t top_k,
    int32_t n_tok, uint64_t expert_bytes, int32_t *out_slots, int32_t *dqueue, int32_t *queue) {
  extern __shared__ int4 smem4[];
  int32_t *sm = reinterpret_cast<int32_t *>(smem4);
  const int32_t n_pairs = top_k * n_tok;
  int32_t *sids = sm + L.words;
  int32_t *sout = sids + n_pairs;
  int32_t *sme = sout + n_pairs;
  int32_t *sms = sme + n_pairs;
  __shared__ int32_t n_miss;
  pdl_wait();
  const int4 *g4 = reinterpret_cast<const int4 *>(state);
  for (int i = threadIdx.x; i < L.words / 4; i += blockDim.x) smem4[i] = g4[i];
  for (int32_t p = threadIdx.x; p < n_pairs; p += blockDim.x) {
    const int32_t t = p / top_k, k = p - t * top_k;
    sids[p] = *reinterpret_cast<const int32_t *>(ids + int64_t(k) * nb0 + int64_t(t) * nb1);
  }
  __syncthreads();
  if (threadIdx.x == 0) n_miss = dc_remap(sm, L, sids, n_pairs, expert_bytes, sout, sme, sms);
  __syncthreads();
  int4 *w4 = reinterpret_cast<int4 *>(state);
  for (int i = threadIdx.x; i < L.words / 4; i += blockDim.x) w4[i] = smem4[i];
  for (int32_t p = threadIdx.x; p < n_pairs; p += blockDim.x) out_slots[p] = sout[p];
  const int32_t cap = L.max_pairs;
  for (int32_t i = threadIdx.x; i < n_miss; i += blockDim.x) {
    dqueue[4 + i] = sme[i];
    dqueue[4 + cap + i] = sms[i];
    queue[4 + i] = sme[i];
    queue[4 + cap + i] = sms[i];
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    dqueue[0] = n_miss;
    __threadfence_system();  // the queue entries before the count
    queue[0] = n_miss;
  }
  pdl_trigger();
}

// The pools and sources of up to three roles filled by one launch.
struct FillRoles {
  const uint8_t *src[3];
  int64_t src_stride[3];
  uint8_t *base[3];
  int64_t slot_stride[3], N[3], nb[3];
  int block_bytes[3], scale_bytes[3], tiles[3];
  int n;
};

// Persistent grid over (role, miss, 32-row tile) items, the roles' items
// interleaved miss by miss so that every role's bytes are in flight at once.
__global__ void __launch_bounds__(256) dfill_kernel(const int32_t *queue, int32_t cap,
                                                    const __grid_constant__ FillRoles f) {
  extern __shared__ uint8_t tile[];
  pdl_wait();
  const int32_t n_miss = queue[0];
  int per_miss = 0;
  for (int r = 0; r < f.n; ++r) per_miss += f.tiles[r];
  const int64_t items = int64_t(n_miss) * per_miss;
  for (int64_t w = blockIdx.x; w < items; w += gridDim.x) {
    const int32_t m = int32_t(w / per_miss);
    int t = int(w - int64_t(m) * per_miss), r = 0;
    while (t >= f.tiles[r]) t -= f.tiles[r++];
    const int32_t e = queue[4 + m], s = queue[4 + cap + m];
    repack_tile(tile, f.src[r] + int64_t(e) * f.src_stride[r],
                f.base[r] + int64_t(s) * f.slot_stride[r], int64_t(t) * kRepackRows, f.N[r],
                f.nb[r], f.block_bytes[r], f.scale_bytes[r]);
  }
  pdl_trigger();
}

}  // namespace
}  // namespace msb

extern "C" {

int msb_dstreamer_create(uint32_t n_layer, uint32_t n_expert, uint32_t n_slot, int32_t max_pairs,
                         uint64_t expert_bytes_total, int on_host, msb_dstreamer_t *out) {
  MSB_CHECK_ARG(out && n_layer > 0 && n_expert > 0 && n_slot > 0 && max_pairs > 0,
                "msb_dstreamer_create: bad arguments");
  MSB_CHECK_ARG(n_expert <= 65536 && n_slot <= 65536 && max_pairs <= (1 << 20),
                "msb_dstreamer_create: sizes too large");
  *out = nullptr;
  msb_dstreamer_s *s = new (std::nothrow) msb_dstreamer_s();
  if (!s) return fail(MSB_ERR_NOMEM, "msb_dstreamer_create: out of memory");
  s->on_host = on_host != 0;
  s->n_layer = n_layer;
  s->L = msb::dc_layout(int32_t(n_expert), int32_t(n_slot), max_pairs);
  s->expert_bytes = expert_bytes_total;
  s->queue_words = 4 + 2 * int64_t(max_pairs);
  s->remap_smem = (size_t(s->L.words) + 4 * size_t(max_pairs)) * sizeof(int32_t);
  if (!s->on_host && s->remap_smem > 220 * 1024) {
    const size_t need = s->remap_smem;
    delete s;
    return fail(MSB_ERR_UNSUPPORTED,
                "msb_dstreamer_create: %u experts and %d pairs need %zu bytes of shared memory",
                n_expert, max_pairs, need);
  }
  std::vector<int32_t> init(size_t(s->L.words) * n_layer);
  for (uint32_t l = 0; l < n_layer; ++l) msb::dc_init(init.data() + size_t(l) * s->L.words, s->L);
  const size_t qbytes = size_t(s->queue_words) * n_layer * sizeof(int32_t);
  if (s->on_host) {
    s->state = new (std::nothrow) int32_t[init.size()];
    s->queue = new (std::nothrow) int32_t[qbytes / sizeof(int32_t)];
    if (!s->state || !s->queue) {
      delete s;
      return fail(MSB_ERR_NOMEM, "msb_dstreamer_create: out of memory");
    }
    std::memcpy(s->state, init.data(), init.size() * sizeof(int32_t));
    std::memset(s->queue, 0, qbytes);
    *out = s;
    return MSB_OK;
  }
  cudaGetDevice(&s->device);
  cudaError_t e = cudaMalloc(&s->state, init.size() * sizeof(int32_t));
  if (e == cudaSuccess)
    e = cudaMemcpy(s->state, init.data(), init.size() * sizeof(int32_t), cudaMemcpyHostToDevice);
  if (e == cudaSuccess) e = cudaMalloc(&s->dqueue, qbytes);
  if (e == cudaSuccess) e = cudaMemset(s->dqueue, 0, qbytes);
  if (e == cudaSuccess)
    e = cudaHostAlloc(reinterpret_cast<void **>(&s->queue), qbytes,
                      cudaHostAllocMapped | cudaHostAllocPortable);
  if (e == cudaSuccess) {
    std::memset(s->queue, 0, qbytes);
    e = cudaHostGetDevicePointer(reinterpret_cast<void **>(&s->queue_dev), s->queue, 0);
  }
  if (e == cudaSuccess) e = cudaDeviceSynchronize();  // the memset and copies above
  if (e == cudaSuccess && s->remap_smem > 48 * 1024)
    e = cudaFuncSetAttribute(msb::dc_remap_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             int(s->remap_smem));
  if (e != cudaSuccess) {
    delete s;
    return fail(MSB_ERR_CUDA, "msb_dstreamer_create: %s", cudaGetErrorString(e));
  }
  *out = s;
  return MSB_OK;
}

int msb_dstreamer_destroy(msb_dstreamer_t s) {
  if (s && !s->on_host) cudaDeviceSynchronize();
  delete s;
  return MSB_OK;
}

int msb_dstreamer_remap(msb_dstreamer_t s, uint32_t layer, const int32_t *ids, int64_t nb0,
                        int64_t nb1, int32_t top_k, int32_t n_tok, int32_t *out_slots,
                        void *stream) {
  MSB_CHECK_ARG(s && layer < s->n_layer, "msb_dstreamer_remap: bad streamer or layer");
  MSB_CHECK_ARG(top_k > 0 && n_tok >= 0 && (n_tok == 0 || (ids && out_slots)),
                "msb_dstreamer_remap: bad shape or null pointer");
  MSB_CHECK_ARG(int64_t(top_k) * n_tok <= s->L.max_pairs,
                "msb_dstreamer_remap: %lld pairs exceed max_pairs %d",
                (long long)(int64_t(top_k) * n_tok), s->L.max_pairs);
  MSB_CHECK_ARG(nb0 % 4 == 0 && nb1 % 4 == 0, "msb_dstreamer_remap: id strides must be multiples of 4");
  int32_t *st = s->state + int64_t(layer) * s->L.words;
  if (s->on_host) {
    const int32_t n_pairs = top_k * n_tok;
    std::vector<int32_t> dense(size_t(n_pairs) + 1), me(size_t(n_pairs) + 1),
        ms(size_t(n_pairs) + 1);
    const char *base = reinterpret_cast<const char *>(ids);
    for (int32_t t = 0; t < n_tok; ++t)
      for (int32_t k = 0; k < top_k; ++k)
        std::memcpy(&dense[size_t(t) * top_k + k], base + k * nb0 + t * nb1, sizeof(int32_t));
    const int32_t nm = msb::dc_remap(st, s->L, dense.data(), n_pairs, s->expert_bytes, out_slots,
                                     me.data(), ms.data());
    int32_t *q = s->layer_queue(layer);
    std::memcpy(q + 4, me.data(), size_t(nm) * sizeof(int32_t));
    std::memcpy(q + 4 + s->L.max_pairs, ms.data(), size_t(nm) * sizeof(int32_t));
    q[0] = nm;
    return MSB_OK;
  }
  MSB_CUDA_TRY(msb::launch_pdl(msb::dc_remap_kernel, dim3(1), dim3(msb::kRemapThreads),
                               size_t(s->L.words + 4 * top_k * n_tok) * sizeof(int32_t),
                               static_cast<cudaStream_t>(stream), st, s->L,
                               reinterpret_cast<const char *>(ids), nb0, nb1, top_k, n_tok,
                               s->expert_bytes, out_slots,
                               s->dqueue + int64_t(layer) * s->queue_words,
                               s->queue_dev + int64_t(layer) * s->queue_words));
  msb::count_launch();
  return MSB_OK;
}

int msb_dstreamer_fill_roles(msb_dstreamer_t s, uint32_t layer, int32_t n_roles,
                             const msb_pool_t *pools, const void *const *srcs,
                             const int64_t *src_expert_strides, void *stream) {
  MSB_CHECK_ARG(s && layer < s->n_layer && n_roles >= 1 && n_roles <= 3 && pools && srcs &&
                    src_expert_strides,
                "msb_dstreamer_fill_roles: bad argument");
  MSB_CHECK_ARG(!s->on_host, "msb_dstreamer_fill: a host streamer has no device fills");
  msb::FillRoles f{};
  f.n = n_roles;
  size_t smem = 0;
  int device = 0;
  int64_t per_miss = 0;
  for (int r = 0; r < n_roles; ++r) {
    const msb_pool_s *p = pools[r];
    MSB_CHECK_ARG(p && srcs[r], "msb_dstreamer_fill: null pool or source");
    MSB_CHECK_ARG(p->n_slot == s->L.n_slot,
                  "msb_dstreamer_fill: the pool has %d slots, the streamer %d", p->n_slot,
                  s->L.n_slot);
    MSB_CHECK_ARG(src_expert_strides[r] >= p->expert_bytes,
                  "msb_dstreamer_fill: expert stride %lld below the expert's %lld bytes",
                  (long long)src_expert_strides[r], (long long)p->expert_bytes);
    const size_t sm = size_t(msb::kRepackRows) * p->nb * p->block_bytes;
    MSB_CHECK_ARG(sm <= 227 * 1024, "msb_dstreamer_fill: rows too long for the repack tile");
    smem = sm > smem ? sm : smem;
    f.src[r] = static_cast<const uint8_t *>(srcs[r]);
    f.src_stride[r] = src_expert_strides[r];
    f.base[r] = p->data;
    f.slot_stride[r] = p->slot_stride;
    f.N[r] = p->N;
    f.nb[r] = p->nb;
    f.block_bytes[r] = p->block_bytes;
    f.scale_bytes[r] = p->scale_bytes;
    f.tiles[r] = int((p->N + msb::kRepackRows - 1) / msb::kRepackRows);
    per_miss += f.tiles[r];
    device = p->device;
  }
  if (smem > 48 * 1024)
    MSB_CUDA_TRY(cudaFuncSetAttribute(msb::dfill_kernel,
                                      cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)));
  int n_sm = 0;
  MSB_CUDA_TRY(cudaDeviceGetAttribute(&n_sm, cudaDevAttrMultiProcessorCount, device));
  const int64_t most =
      int64_t(s->L.max_pairs < s->L.n_slot ? s->L.max_pairs : s->L.n_slot) * per_miss;
  const int grid = int(most < 2 * n_sm ? most : 2 * n_sm);
  MSB_CUDA_TRY(msb::launch_pdl(msb::dfill_kernel, dim3(grid), dim3(256), smem,
                               static_cast<cudaStream_t>(stream),
                               s->dqueue + int64_t(layer) * s->queue_words, s->L.max_pairs, f));
  msb::count_launch();
  return MSB_OK;
}

int msb_dstreamer_fill(msb_dstreamer_t s, uint32_t layer, msb_pool_t pool, const void *src,
                       int64_t src_expert_stride, void *stream) {
  return msb_dstreamer_fill_roles(s, layer, 1, &pool, &src, &src_expert_stride, stream);
}

int msb_dstreamer_misses(msb_dstreamer_t s, uint32_t layer, int32_t *n_miss, int32_t *experts,
                         int32_t *slots) {
  MSB_CHECK_ARG(s && layer < s->n_layer && n_miss, "msb_dstreamer_misses: bad argument");
  const int32_t *q = s->layer_queue(layer);
  const int32_t nm = *reinterpret_cast<const volatile int32_t *>(q);
  *n_miss = nm;
  if (experts) std::memcpy(experts, q + 4, size_t(nm) * sizeof(int32_t));
  if (slots) std::memcpy(slots, q + 4 + s->L.max_pairs, size_t(nm) * sizeof(int32_t));
  return MSB_OK;
}

int msb_dstreamer_table(msb_dstreamer_t s, uint32_t layer, int32_t *table) {
  MSB_CHECK_ARG(s && layer < s->n_layer && table, "msb_dstreamer_table: bad argument");
  const int32_t *st = s->state + int64_t(layer) * s->L.words + s->L.slot;
  if (s->on_host) {
    std::memcpy(table, st, size_t(s->L.E) * sizeof(int32_t));
    return MSB_OK;
  }
  // The remap may have run on any stream: wait for all of them.
  MSB_CUDA_TRY(cudaDeviceSynchronize());
  MSB_CUDA_TRY(cudaMemcpy(table, st, size_t(s->L.E) * sizeof(int32_t), cudaMemcpyDeviceToHost));
  return MSB_OK;
}

int msb_dstreamer_stats(msb_dstreamer_t s, msb_cache_stats_t *out, uint64_t *n_exhausted) {
  MSB_CHECK_ARG(s && out, "msb_dstreamer_stats: bad argument");
  std::vector<int32_t> all(size_t(s->L.words) * s->n_layer);
  if (s->on_host) {
    std::memcpy(all.data(), s->state, all.size() * sizeof(int32_t));
  } else {
    MSB_CUDA_TRY(cudaDeviceSynchronize());
    MSB_CUDA_TRY(cudaMemcpy(all.data(), s->state, all.size() * sizeof(int32_t),
                            cudaMemcpyDeviceToHost));
  }
  uint64_t sum[msb::kNumStats] = {0};
  for (uint32_t l = 0; l < s->n_layer; ++l) {
    const int32_t *st = all.data() + size_t(l) * s->L.words + s->L.stats;
    for (int i = 0; i < msb::kNumStats; ++i)
      sum[i] += uint64_t(uint32_t(st[2 * i])) | uint64_t(uint32_t(st[2 * i + 1])) << 32;
  }
  out->hit = sum[msb::kStHit];
  out->miss = sum[msb::kStMiss];
  out->hit_pinned = sum[msb::kStHitPinned];
  out->hit_small = sum[msb::kStHitSmall];
  out->hit_main = sum[msb::kStHitMain];
  out->ghost_hit = sum[msb::kStGhostHit];
  out->admit = sum[msb::kStAdmit];
  out->evict = sum[msb::kStEvict];
  out->bypass = sum[msb::kStBypass];
  out->promote = sum[msb::kStPromote];
  out->bytes_fetched = sum[msb::kStBytes];
  if (n_exhausted) *n_exhausted = sum[msb::kStExhausted];
  return MSB_OK;
}

}  // extern "C"
