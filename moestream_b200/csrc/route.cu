// Remap router expert ids to slot ids and group the (token, k) pairs by slot.
//
// The reference produces slot ids on the CPU (ms_remap_fn core loop,
// src/llama-moestream.cpp:1900-1952) and ggml then groups rows by expert
// inside mul_mat_id. Here both happen in one single-CTA kernel:
//   1. every thread maps its pairs through the expert -> slot table (zero
//      slot for invalid ids or experts without a slot) and counts per slot
//      with shared-memory atomics (order independent);
//   2. a block scan turns counts into offsets and lists the active slots;
//   3. one warp scatters pair indices into their slot's range, 32 pairs per
//      step: __match_any_sync finds the lanes sharing a slot, the lowest such
//      lane advances that slot's cursor, and each lane's rank among them
//      gives its position. Steps run in pair order, so each slot's list is in
//      increasing pair order and the output is deterministic.
#include <cuda_runtime.h>

#include "msb_internal.h"

namespace msb {

struct RouteArgs {
  const char *ids;
  int64_t nb0, nb1;
  int32_t top_k, n_tok;
  const int32_t *table;
  int32_t n_expert, n_slot;
  int32_t *slot_ids, *counts, *offsets, *rows, *active;
  FlagWait wait;   // ids arriving from other GPUs (expert parallelism)
  int stash;       // pairs' slots also kept in shared memory (n_pairs <= kStashPairs)
};

// Pairs whose slots the scatter reads from shared memory instead of global
// memory (the scatter is one warp's dependent chain: a shared-memory read
// per step instead of a round trip to L2).
static constexpr int kStashPairs = 12288;

static constexpr int kRouteThreads = 1024;

// Exclusive scan of v[0..n) in place over the whole block; returns the total.
__device__ int block_exclusive_scan(int *v, int n, int *warp_sums) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int per = (n + kRouteThreads - 1) / kRouteThreads;
  const int lo = tid * per, hi = min(lo + per, n);
  int local = 0;
  for (int i = lo; i < hi; ++i) local += v[i];
  int incl = local;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += y;
  }
  if (lane == 31) warp_sums[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    int w = warp_sums[lane];
    int wi = w;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, wi, o);
      if (lane >= o) wi += y;
    }
    warp_sums[lane] = wi - w;  // exclusive prefix of warp totals
    if (lane == 31) warp_sums[32] = wi;
  }
  __syncthreads();
  int run = warp_sums[warp] + incl - local;
  for (int i = lo; i < hi; ++i) {
    const int x = v[i];
    v[i] = run;
    run += x;
  }
  const int total = warp_sums[32];
  __syncthreads();
  return total;
}

__global__ void __launch_bounds__(kRouteThreads) route_kernel(RouteArgs a) {
  pdl_wait();
  pdl_trigger();
  flag_wait_block(a.wait);
  extern __shared__ int sm[];
  const int S = a.n_slot + 1;
  int *cnt = sm;             // [S]
  int *cursor = sm + S;      // [S]
  int *flag = sm + 2 * S;    // [S]
  int *warp_sums = sm + 3 * S;  // [33]
  int *stash = sm + 3 * S + 33;  // [n_pairs] when a.stash
  const int tid = threadIdx.x;
  const int n_pairs = a.top_k * a.n_tok;

  for (int s = tid; s < S; s += kRouteThreads) cnt[s] = 0;
  __syncthreads();

  for (int i = tid; i < n_pairs; i += kRouteThreads) {
    const int t = i / a.top_k, k = i - t * a.top_k;
    const int e = *reinterpret_cast<const int32_t *>(a.ids + k * a.nb0 + t * a.nb1);
    int slot = a.n_slot;  // zero slot
    if (a.table) {
      if (e >= 0 && e < a.n_expert) {
        const int s = a.table[e];
        if (s >= 0 && s < a.n_slot) slot = s;
      }
    } else if (e >= 0 && e <= a.n_slot) {
      slot = e;  // ids already hold slot ids
    }
    a.slot_ids[i] = slot;
    if (a.stash) stash[i] = slot;
    atomicAdd(&cnt[slot], 1);
  }
  __syncthreads();

  for (int s = tid; s < S; s += kRouteThreads) {
    a.counts[s] = cnt[s];
    cursor[s] = cnt[s];
    flag[s] = cnt[s] > 0;
  }
  __syncthreads();
  block_exclusive_scan(cursor, S, warp_sums);
  const int n_active = block_exclusive_scan(flag, S, warp_sums);
  for (int s = tid; s < S; s += kRouteThreads) {
    a.offsets[s] = cursor[s];
    if (cnt[s] > 0) a.active[1 + flag[s]] = s;
  }
  if (tid == 0) {
    a.offsets[S] = n_pairs;
    a.active[0] = n_active;
  }
  __syncthreads();

  if (tid < 32) {
    const int lane = tid;
    const unsigned lt = (1u << lane) - 1u;
    for (int base = 0; base < n_pairs; base += 32) {
      const int i = base + lane;
      const bool valid = i < n_pairs;
      const int s = valid ? (a.stash ? stash[i] : a.slot_ids[i]) : -1 - lane;
      const unsigned same = __match_any_sync(0xffffffffu, s);
      const int leader = __ffs(same) - 1;
      int start = 0;
      if (valid && lane == leader) {
        start = cursor[s];
        cursor[s] = start + __popc(same);
      }
      start = __shfl_sync(0xffffffffu, start, leader);
      if (valid) a.rows[start + __popc(same & lt)] = i;
      __syncwarp();
    }
  }
}

}  // namespace msb

extern "C" int msb_remap_group(const int32_t *ids_dev, int64_t nb0, int64_t nb1, int32_t top_k,
                               int32_t n_tok, const int32_t *table_dev, int32_t n_expert,
                               int32_t n_slot, const msb_route_t *route, void *stream) {
  return msb::remap_group_wait(ids_dev, nb0, nb1, top_k, n_tok, table_dev, n_expert, n_slot,
                               route, msb::FlagWait{}, stream);
}

int msb::remap_group_wait(const int32_t *ids_dev, int64_t nb0, int64_t nb1, int32_t top_k,
                          int32_t n_tok, const int32_t *table_dev, int32_t n_expert,
                          int32_t n_slot, const msb_route_t *route, const FlagWait &wait,
                          void *stream) {
  MSB_CHECK_ARG(route && route->slot_ids && route->counts && route->offsets && route->rows &&
                    route->active,
                "msb_remap_group: route arrays must all be set");
  MSB_CHECK_ARG(top_k > 0 && n_tok >= 0 && n_slot > 0, "msb_remap_group: bad shape");
  MSB_CHECK_ARG(ids_dev || n_tok == 0, "msb_remap_group: null ids");
  MSB_CHECK_ARG(nb0 % 4 == 0 && nb1 % 4 == 0, "msb_remap_group: id strides must be multiples of 4 bytes");
  MSB_CHECK_ARG(int64_t(top_k) * n_tok < (int64_t(1) << 30), "msb_remap_group: too many pairs");
  const int S = n_slot + 1;
  const int64_t n_pairs = int64_t(top_k) * n_tok;
  size_t smem = (size_t(3) * S + 33) * sizeof(int);
  MSB_CHECK_ARG(smem <= 200 * 1024, "msb_remap_group: n_slot %d too large", n_slot);
  const bool stash = n_pairs <= msb::kStashPairs && smem + size_t(n_pairs) * 4 <= 200 * 1024;
  if (stash) smem += size_t(n_pairs) * sizeof(int);
  msb::RouteArgs a{reinterpret_cast<const char *>(ids_dev), nb0, nb1, top_k, n_tok,
                   table_dev, n_expert, n_slot, route->slot_ids, route->counts,
                   route->offsets, route->rows, route->active, wait, stash ? 1 : 0};
  if (smem > 48 * 1024)
    MSB_CUDA_TRY(cudaFuncSetAttribute(msb::route_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)));
  MSB_CUDA_TRY(msb::launch_pdl(msb::route_kernel, dim3(1), dim3(msb::kRouteThreads), smem,
                               static_cast<cudaStream_t>(stream), a));
  msb::count_launch();
  MSB_CUDA_TRY(cudaGetLastError());
  return MSB_OK;
}
