// Expert-parallel exchange over NVLink peer memory.
//
// The reference is single-process and single-GPU; this replaces the two
// all-to-all collectives of an expert-parallel MoE layer with kernels that
// store the rows straight into the other GPUs' memory. Every rank owns one
// exchange buffer (cudaMalloc, shared with the other ranks by CUDA IPC):
//
//   [recv rows: n_rank*cap rows of row_bytes]   block s = rows from rank s:
//                                               K bf16 activations, then
//                                               the int32 local expert id
//   [y_back: n_rank*cap rows of K f32]          block d = results from rank d
//   [control: 32 u32]                           flags[2][8] (written by the
//                                               peers), sent[2], done[2]
//                                               (this rank's own)
//
// A sending kernel stores its rows into the destinations' buffers, and its
// last CTA to finish (a done counter) raises this rank's flag in every
// destination to the next sequence number. A waiting kernel spins, bounded
// (about a second), until every peer's flag reached the number of layers
// this rank has dispatched (its own sent[0]: every rank runs the same
// layers, so a rank waiting for layer L's rows or results expects L). The counters live in device memory, so a captured CUDA graph
// replays the protocol correctly. Ordering: each CTA's stores are followed by
// a system-scope fence before it counts itself done; the last CTA fences
// again and publishes the flags with release stores; waiters load them with
// acquire loads.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstring>

#include "msb_internal.h"

namespace msb {
namespace ep {

constexpr int kThreads = 256;
constexpr int kFlags = 0, kSent = 16, kDone = 20;   // control u32 offsets

struct Layout {
  char *peer[MSB_EP_MAX_RANKS];
  int32_t n_rank, rank, cap;
  int64_t K, row_bytes, yback_off, ctrl_off;
};

__host__ __device__ inline int64_t align256(int64_t x) { return (x + 255) / 256 * 256; }
__host__ __device__ inline int64_t row_bytes_of(int64_t K) { return (2 * K + 4 + 15) / 16 * 16; }

__device__ __forceinline__ void store_release_sys(uint32_t *p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t load_acquire_sys(const uint32_t *p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ uint32_t *ctrl_of(const Layout &L, int r) {
  return reinterpret_cast<uint32_t *>(L.peer[r] + L.ctrl_off);
}

// Called by every CTA after its stores: the last one to finish publishes
// phase `ph`'s next sequence number in every rank's flag for this rank.
__device__ void publish(const Layout &L, int ph) {
  __syncthreads();
  if (threadIdx.x != 0) return;
  uint32_t *own = ctrl_of(L, L.rank);
  __threadfence_system();
  const uint32_t prev = atomicAdd(&own[kDone + ph], 1u);
  if (prev != gridDim.x - 1) return;
  own[kDone + ph] = 0;
  __threadfence_system();
  const uint32_t seq = own[kSent + ph] + 1;
  own[kSent + ph] = seq;
  for (int d = 0; d < L.n_rank; ++d) store_release_sys(ctrl_of(L, d) + kFlags + ph * 8 + L.rank, seq);
}

// Pairs p < n_pairs: the row of pair p (token p / top_k) goes to the rank
// owning its expert, at block `rank` row (its rank among earlier pairs with
// that destination); pos[p] = that destination's block row here. CTA
// n_pairs + d marks the rows this rank leaves unused in rank d's block
// (expert id -1).
template <typename T>
__global__ void __launch_bounds__(kThreads) dispatch_kernel(const __grid_constant__ Layout L, const int32_t *ids,
                                                            const char *x, int64_t x_nb1,
                                                            int32_t top_k, int32_t n_pairs,
                                                            int32_t n_local, int32_t *pos) {
  pdl_wait();
  pdl_trigger();
  __shared__ int warp_cnt[kThreads / 32];
  const int n_exp = n_local * L.n_rank;
  const bool fill = int(blockIdx.x) >= n_pairs;
  const int p = blockIdx.x;
  int dest;
  if (fill) {
    dest = p - n_pairs;
  } else {
    const int e = ids[p];
    dest = (e >= 0 && e < n_exp) ? e / n_local : -1;
  }
  // Pairs before p (all pairs for a fill CTA) with this destination.
  int c = 0;
  if (dest >= 0) {
    const int end = fill ? n_pairs : p;
    for (int q = threadIdx.x; q < end; q += kThreads) {
      const int eq = ids[q];
      c += (eq >= 0 && eq < n_exp && eq / n_local == dest);
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) c += __shfl_xor_sync(0xffffffffu, c, o);
  if ((threadIdx.x & 31) == 0) warp_cnt[threadIdx.x >> 5] = c;
  __syncthreads();
  int rank = 0;
  for (int w = 0; w < kThreads / 32; ++w) rank += warp_cnt[w];
  char *recv = dest >= 0 ? L.peer[dest] + int64_t(L.rank) * L.cap * L.row_bytes : nullptr;
  if (fill) {
    for (int r = (rank < L.cap ? rank : L.cap) + threadIdx.x; r < L.cap; r += kThreads)
      *reinterpret_cast<int32_t *>(recv + r * L.row_bytes + 2 * L.K) = -1;
  } else if (dest < 0 || rank >= L.cap) {
    if (threadIdx.x == 0) pos[p] = -1;
  } else {
    char *row = recv + rank * L.row_bytes;
    if (threadIdx.x == 0) {
      pos[p] = dest * L.cap + rank;
      *reinterpret_cast<int32_t *>(row + 2 * L.K) = ids[p] - dest * n_local;
    }
    const T *src = reinterpret_cast<const T *>(x + int64_t(p / top_k) * x_nb1);
    __nv_bfloat16 *dst = reinterpret_cast<__nv_bfloat16 *>(row);
    if (sizeof(T) == 2 && L.K % 8 == 0 && (reinterpret_cast<uintptr_t>(src) & 15) == 0) {
      const uint4 *s4 = reinterpret_cast<const uint4 *>(src);
      uint4 *d4 = reinterpret_cast<uint4 *>(dst);
      for (int64_t i = threadIdx.x; i < L.K / 8; i += kThreads) d4[i] = s4[i];
    } else {
      for (int64_t i = threadIdx.x; i < L.K; i += kThreads) {
        if constexpr (sizeof(T) == 2) dst[i] = src[i];
        else dst[i] = __float2bfloat16_rn(src[i]);
      }
    }
  }
  publish(L, 0);
}

// Row r of y_loc (block s = rows received from rank s) goes back to rank s,
// block `rank`; rows whose expert id is -1 were never asked for.
__global__ void __launch_bounds__(kThreads) return_kernel(const __grid_constant__ Layout L, const float *y_loc) {
  pdl_wait();
  pdl_trigger();
  const int r = blockIdx.x;
  const int s = r / L.cap, i = r % L.cap;
  const char *recv_row = L.peer[L.rank] + int64_t(r) * L.row_bytes;
  if (*reinterpret_cast<const int32_t *>(recv_row + 2 * L.K) >= 0) {
    const float4 *src = reinterpret_cast<const float4 *>(y_loc + int64_t(r) * L.K);
    float4 *dst = reinterpret_cast<float4 *>(L.peer[s] + L.yback_off +
                                             (int64_t(L.rank) * L.cap + i) * L.K * 4);
    for (int64_t j = threadIdx.x; j < L.K / 4; j += kThreads) dst[j] = src[j];
  }
  publish(L, 1);
}

// Waits until every rank published phase `ph` of the current layer here.
__global__ void wait_kernel(FlagWait w) {
  pdl_wait();
  pdl_trigger();
  flag_wait_block(w);
}

inline FlagWait phase_wait(const Layout &L, int ph, int *status) {
  FlagWait w;
  const uint32_t *own = reinterpret_cast<const uint32_t *>(L.peer[L.rank] + L.ctrl_off);
  w.flags = own + kFlags + ph * 8;
  w.seq = own + kSent;
  w.n = L.n_rank;
  w.status = status;
  w.bit = 32 << ph;
  return w;
}

}  // namespace ep
}  // namespace msb

using namespace msb;

static int make_layout(const msb_ep_peers_t *p, ep::Layout *L) {
  MSB_CHECK_ARG(p, "null peers");
  MSB_CHECK_ARG(p->n_rank >= 1 && p->n_rank <= MSB_EP_MAX_RANKS && p->rank >= 0 &&
                    p->rank < p->n_rank && p->cap > 0 && p->K > 0 && p->K % 4 == 0,
                "bad expert-parallel layout (n_rank %d, rank %d, cap %d, K %lld)", p->n_rank,
                p->rank, p->cap, (long long)p->K);
  for (int r = 0; r < p->n_rank; ++r) MSB_CHECK_ARG(p->peer[r], "peer %d buffer missing", r);
  *L = {};
  for (int r = 0; r < p->n_rank; ++r) L->peer[r] = static_cast<char *>(p->peer[r]);
  L->n_rank = p->n_rank;
  L->rank = p->rank;
  L->cap = p->cap;
  L->K = p->K;
  L->row_bytes = ep::row_bytes_of(p->K);
  const int64_t R = int64_t(p->n_rank) * p->cap;
  L->yback_off = ep::align256(R * L->row_bytes);
  L->ctrl_off = L->yback_off + ep::align256(R * p->K * 4);
  return MSB_OK;
}

extern "C" int64_t msb_ep_buffer_bytes(int32_t n_rank, int32_t cap, int64_t K) {
  if (n_rank < 1 || n_rank > MSB_EP_MAX_RANKS || cap < 1 || K < 1 || K % 4) return -1;
  const int64_t R = int64_t(n_rank) * cap;
  return ep::align256(R * ep::row_bytes_of(K)) + ep::align256(R * K * 4) + 256;
}

extern "C" int64_t msb_ep_row_bytes(int64_t K) { return K > 0 ? ep::row_bytes_of(K) : -1; }

extern "C" int64_t msb_ep_yback_offset(int32_t n_rank, int32_t cap, int64_t K) {
  if (n_rank < 1 || cap < 1 || K < 1) return -1;
  return ep::align256(int64_t(n_rank) * cap * ep::row_bytes_of(K));
}

extern "C" int msb_ep_buffer_create(int64_t bytes, void **buf, void *ipc_handle) {
  MSB_CHECK_ARG(bytes > 0 && buf && ipc_handle, "msb_ep_buffer_create: bad argument");
  void *p = nullptr;
  MSB_CUDA_TRY(cudaMalloc(&p, size_t(bytes)));
  cudaError_t e = cudaMemset(p, 0, size_t(bytes));
  cudaIpcMemHandle_t h;
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, p);
  if (e != cudaSuccess) {
    cudaFree(p);
    return fail(MSB_ERR_CUDA, "msb_ep_buffer_create: %s", cudaGetErrorString(e));
  }
  static_assert(sizeof(h) == MSB_EP_HANDLE_BYTES, "IPC handle size");
  memcpy(ipc_handle, &h, sizeof(h));
  *buf = p;
  return MSB_OK;
}

extern "C" int msb_ep_buffer_open(const void *ipc_handle, void **peer_buf) {
  MSB_CHECK_ARG(ipc_handle && peer_buf, "msb_ep_buffer_open: bad argument");
  cudaIpcMemHandle_t h;
  memcpy(&h, ipc_handle, sizeof(h));
  MSB_CUDA_TRY(cudaIpcOpenMemHandle(peer_buf, h, cudaIpcMemLazyEnablePeerAccess));
  return MSB_OK;
}

extern "C" int msb_ep_buffer_close(void *peer_buf) {
  MSB_CHECK_ARG(peer_buf, "msb_ep_buffer_close: null");
  MSB_CUDA_TRY(cudaIpcCloseMemHandle(peer_buf));
  return MSB_OK;
}

extern "C" int msb_ep_buffer_destroy(void *buf) {
  if (buf) MSB_CUDA_TRY(cudaFree(buf));
  return MSB_OK;
}

extern "C" int msb_ep_dispatch_peers(const msb_ep_peers_t *peers, const int32_t *ids_dev,
                                     const void *x_dev, int x_type, int64_t x_nb1, int32_t top_k,
                                     int32_t n_tok, int32_t n_local, int32_t *pos_dev,
                                     void *stream) {
  ep::Layout L{};
  if (int rc = make_layout(peers, &L)) return rc;
  MSB_CHECK_ARG(top_k > 0 && n_tok >= 0 && n_local > 0, "msb_ep_dispatch_peers: bad shape");
  MSB_CHECK_ARG(n_tok == 0 || (ids_dev && x_dev && pos_dev), "msb_ep_dispatch_peers: null");
  const int n_pairs = top_k * n_tok;
  const unsigned grid = unsigned(n_pairs + L.n_rank);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const char *x = static_cast<const char *>(x_dev);
  if (x_type == MSB_TYPE_BF16)
    MSB_CUDA_TRY(launch_pdl(ep::dispatch_kernel<__nv_bfloat16>, dim3(grid), dim3(ep::kThreads), 0, st,
                            L, ids_dev, x, x_nb1, top_k, n_pairs, n_local, pos_dev));
  else if (x_type == MSB_TYPE_F32)
    MSB_CUDA_TRY(launch_pdl(ep::dispatch_kernel<float>, dim3(grid), dim3(ep::kThreads), 0, st, L,
                            ids_dev, x, x_nb1, top_k, n_pairs, n_local, pos_dev));
  else
    return fail(MSB_ERR_INVALID, "msb_ep_dispatch_peers: activation type %d", x_type);
  count_launch();
  MSB_CUDA_TRY(cudaGetLastError());
  return MSB_OK;
}

extern "C" int msb_ep_return_peers(const msb_ep_peers_t *peers, const float *y_loc_dev,
                                   void *stream) {
  ep::Layout L{};
  if (int rc = make_layout(peers, &L)) return rc;
  MSB_CHECK_ARG(y_loc_dev && (reinterpret_cast<uintptr_t>(y_loc_dev) & 15) == 0,
                "msb_ep_return_peers: y_loc must be 16-byte aligned");
  MSB_CUDA_TRY(launch_pdl(ep::return_kernel, dim3(unsigned(L.n_rank * L.cap)), dim3(ep::kThreads),
                          0, static_cast<cudaStream_t>(stream), L, y_loc_dev));
  count_launch();
  MSB_CUDA_TRY(cudaGetLastError());
  return MSB_OK;
}

extern "C" int msb_ep_wait(const msb_ep_peers_t *peers, int32_t phase, void *stream) {
  ep::Layout L{};
  if (int rc = make_layout(peers, &L)) return rc;
  MSB_CHECK_ARG(phase == 0 || phase == 1, "msb_ep_wait: phase must be 0 or 1");
  int *status = nullptr;
  if (int rc = status_word(&status)) return rc;
  MSB_CUDA_TRY(launch_pdl(ep::wait_kernel, dim3(1), dim3(32), 0, static_cast<cudaStream_t>(stream),
                          ep::phase_wait(L, phase, status)));
  count_launch();
  MSB_CUDA_TRY(cudaGetLastError());
  return MSB_OK;
}

extern "C" int msb_ep_remap_group(const msb_ep_peers_t *peers, int32_t n_slot,
                                  const msb_route_t *route, void *stream) {
  ep::Layout L{};
  if (int rc = make_layout(peers, &L)) return rc;
  int *status = nullptr;
  if (int rc = status_word(&status)) return rc;
  const int32_t *ids = reinterpret_cast<const int32_t *>(L.peer[L.rank] + 2 * L.K);
  return remap_group_wait(ids, 4, L.row_bytes, 1, L.n_rank * L.cap, nullptr, 0, n_slot, route,
                          ep::phase_wait(L, 0, status), stream);
}

extern "C" int msb_ep_combine_peers(const msb_ep_peers_t *peers, const int32_t *pos_dev,
                                    const float *w_dev, int32_t top_k, int32_t n_tok,
                                    float *y_dev, void *stream) {
  ep::Layout L{};
  if (int rc = make_layout(peers, &L)) return rc;
  int *status = nullptr;
  if (int rc = status_word(&status)) return rc;
  const float *back = reinterpret_cast<const float *>(L.peer[L.rank] + L.yback_off);
  return ep_combine_wait(back, pos_dev, w_dev, top_k, n_tok, L.K, y_dev,
                         ep::phase_wait(L, 1, status), stream);
}
