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
//   [control: 32 u32]                           flags[2][8] (arrival counts
//                                               the peers add to), sent[0]
//                                               (this rank's layer count),
//                                               done (results sent, per
//                                               launch)
//
// The dispatch kernel runs kCtas CTAs per peer; each stores its share of the
// rows into that peer's buffer and then adds one to the peer's flag for this
// rank (a system-scope release reduction after an acquire-release fence).
// Results go back either from the down projection's epilogue itself
// (msb_ep_moe_ffn_peers) or by return_kernel; in both the last CTA to finish
// (a done counter) adds one to each source's result flag for this rank. A
// waiting kernel spins, bounded (about a second), until every peer's flag
// reached kCtas (rows) or 1 (results) times the number of layers this rank
// has dispatched (its own sent[0]: every rank runs the same layers). The counters
// live in device memory, so a captured CUDA graph replays the protocol
// correctly. Waiters read the flags with system-scope acquire loads.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstring>

#include "msb_internal.h"

namespace msb {
namespace ep {

constexpr int kThreads = 256;
constexpr int kFlags = 0, kSent = 16, kDone = 17;   // control u32 offsets
constexpr int kCtas = 32;                // CTAs per (this rank, peer) block

struct Layout {
  char *peer[MSB_EP_MAX_RANKS];
  int32_t n_rank, rank, cap;
  int64_t K, row_bytes, yback_off, ctrl_off;
};

__host__ __device__ inline int64_t align256(int64_t x) { return (x + 255) / 256 * 256; }
__host__ __device__ inline int64_t row_bytes_of(int64_t K) { return (2 * K + 4 + 15) / 16 * 16; }

__device__ __forceinline__ uint32_t *ctrl_of(const Layout &L, int r) {
  return reinterpret_cast<uint32_t *>(L.peer[r] + L.ctrl_off);
}

__device__ __forceinline__ int32_t e_local(int32_t e, int d, int32_t n_local) {
  return e - d * n_local;
}

// After a CTA's stores into rank d's buffer: one arrival on d's flag for
// this rank in phase `ph`. The barrier orders every thread's stores before
// thread 0's acquire-release fence at system scope, which orders them before
// the arrival (a release reduction) for any GPU that acquires the flag.
__device__ __forceinline__ void arrive(const Layout &L, int d, int ph) {
  __syncthreads();
  if (threadIdx.x == 0) {
    asm volatile("fence.acq_rel.sys;" ::: "memory");
    uint32_t *f = ctrl_of(L, d) + kFlags + ph * 8 + L.rank;
    asm volatile("red.release.sys.global.add.u32 [%0], 1;" ::"l"(f) : "memory");
  }
}

// The CTA copies n16 16-byte words, each thread issuing all of its loads
// (up to kBatch) before its stores, so the requests overlap instead of
// waiting one round trip per word.
constexpr int kBatch = 4;
__device__ __forceinline__ void cta_copy16(uint4 *__restrict__ dst, const uint4 *__restrict__ src,
                                           int64_t n16) {
  for (int64_t b = 0; b < n16; b += int64_t(kThreads) * kBatch) {
    uint4 r[kBatch];
#pragma unroll
    for (int u = 0; u < kBatch; ++u) {
      const int64_t i = b + u * kThreads + threadIdx.x;
      if (i < n16) r[u] = src[i];
    }
#pragma unroll
    for (int u = 0; u < kBatch; ++u) {
      const int64_t i = b + u * kThreads + threadIdx.x;
      if (i < n16) dst[i] = r[u];
    }
  }
}

// One activation row (K values) into a bf16 row, by the whole CTA.
template <typename T>
__device__ __forceinline__ void cta_copy_row_bf16(__nv_bfloat16 *dst, const T *src, int64_t K) {
  if (sizeof(T) == 2 && K % 8 == 0 && (reinterpret_cast<uintptr_t>(src) & 15) == 0) {
    cta_copy16(reinterpret_cast<uint4 *>(dst), reinterpret_cast<const uint4 *>(src), K / 8);
  } else {
    for (int64_t i = threadIdx.x; i < K; i += kThreads) {
      if constexpr (sizeof(T) == 2) dst[i] = src[i];
      else dst[i] = __float2bfloat16_rn(src[i]);
    }
  }
}

// kCtas CTAs per destination rank d. Pair p goes to d's block `rank` at
// row = its rank among the pairs with destination d (pair order); CTA c of d
// copies the rows whose index is c mod kCtas, writes their pos and local
// expert ids, marks its share of the unused rows with -1, then arrives once
// on d's flag. CTA 0 also counts the layer (sent[0]) and writes pos -1 for
// pairs with an invalid expert.
template <typename T>
__global__ void __launch_bounds__(kThreads) dispatch_kernel(const __grid_constant__ Layout L,
                                                            const int32_t *ids, const char *x,
                                                            int64_t x_nb1, int32_t top_k,
                                                            int32_t n_pairs, int32_t n_local,
                                                            int32_t *pos) {
  pdl_wait();
  pdl_trigger();
  __shared__ int warp_tot[kThreads / 32];
  __shared__ int s_pair[kThreads], s_row[kThreads];
  __shared__ int s_n;
  const int d = blockIdx.x / kCtas, c = blockIdx.x % kCtas;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_exp = n_local * L.n_rank;
  char *recv = L.peer[d] + int64_t(L.rank) * L.cap * L.row_bytes;
  int base = 0;
  for (int p0 = 0; p0 < n_pairs; p0 += kThreads) {
    const int p = p0 + threadIdx.x;
    const int e = p < n_pairs ? ids[p] : -1;
    const bool valid = e >= 0 && e < n_exp;
    const bool mine = valid && e / n_local == d;
    if (p < n_pairs && !valid && blockIdx.x == 0) pos[p] = -1;
    const unsigned bal = __ballot_sync(0xffffffffu, mine);
    if (lane == 0) warp_tot[warp] = __popc(bal);
    if (threadIdx.x == 0) s_n = 0;
    __syncthreads();
    int before = 0, total = 0;
    for (int w = 0; w < kThreads / 32; ++w) {
      before += w < warp ? warp_tot[w] : 0;
      total += warp_tot[w];
    }
    const int row = base + before + __popc(bal & ((1u << lane) - 1));
    if (mine && row % kCtas == c) {
      if (row < L.cap) {
        pos[p] = d * L.cap + row;
        const int k = atomicAdd(&s_n, 1);
        s_pair[k] = p;
        s_row[k] = row;
      } else {
        pos[p] = -1;
      }
    }
    __syncthreads();
    for (int k = 0; k < s_n; ++k) {
      const int q = s_pair[k];
      char *dst = recv + int64_t(s_row[k]) * L.row_bytes;
      if (threadIdx.x == 0) *reinterpret_cast<int32_t *>(dst + 2 * L.K) = e_local(ids[q], d, n_local);
      cta_copy_row_bf16(reinterpret_cast<__nv_bfloat16 *>(dst),
                        reinterpret_cast<const T *>(x + int64_t(q / top_k) * x_nb1), L.K);
    }
    base += total;
    __syncthreads();
  }
  for (int r = base + threadIdx.x; r < L.cap; r += kThreads)
    if (r % kCtas == c) *reinterpret_cast<int32_t *>(recv + r * L.row_bytes + 2 * L.K) = -1;
  if (blockIdx.x == 0 && threadIdx.x == 0) ctrl_of(L, L.rank)[kSent] += 1;
  arrive(L, d, 0);
}

// kCtas CTAs per source rank s: rows i = c, c + kCtas, ... of the block
// received from s go back into s's buffer (block `rank`), by the whole CTA;
// rows whose expert id is -1 were never asked for. The last CTA to finish
// adds one to every source's result flag for this rank.
__global__ void __launch_bounds__(kThreads) return_kernel(const __grid_constant__ Layout L,
                                                          const float *y_loc) {
  pdl_wait();
  pdl_trigger();
  const int s = blockIdx.x / kCtas, c = blockIdx.x % kCtas;
  for (int i = c; i < L.cap; i += kCtas) {
    const int64_t r = int64_t(s) * L.cap + i;
    const char *recv_row = L.peer[L.rank] + r * L.row_bytes;
    if (*reinterpret_cast<const int32_t *>(recv_row + 2 * L.K) < 0) continue;
    cta_copy16(reinterpret_cast<uint4 *>(L.peer[s] + L.yback_off +
                                         (int64_t(L.rank) * L.cap + i) * L.K * 4),
               reinterpret_cast<const uint4 *>(y_loc + r * L.K), L.K / 4);
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    uint32_t *own = ctrl_of(L, L.rank);
    asm volatile("fence.acq_rel.sys;" ::: "memory");
    if (atomicAdd(own + kDone, 1u) == gridDim.x - 1) {
      own[kDone] = 0;
      asm volatile("fence.acq_rel.sys;" ::: "memory");
      for (int d = 0; d < L.n_rank; ++d) {
        uint32_t *f = ctrl_of(L, d) + kFlags + 8 + L.rank;
        asm volatile("red.release.sys.global.add.u32 [%0], 1;" ::"l"(f) : "memory");
      }
    }
  }
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
  w.mult = ph == 0 ? kCtas : 1;   // rows: kCtas arrivals per peer per layer
  w.n = L.n_rank;
  w.status = status;
  w.bit = 32 << ph;
  w.limit_ns = wait_limit_ns();
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
  const unsigned grid = unsigned(L.n_rank * ep::kCtas);
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
  MSB_CUDA_TRY(launch_pdl(ep::return_kernel, dim3(unsigned(L.n_rank * ep::kCtas)), dim3(ep::kThreads),
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

extern "C" int msb_ep_moe_ffn_peers(const msb_ep_peers_t *peers, msb_pool_t gate, msb_pool_t up,
                                    int64_t up_row0, msb_pool_t down, const msb_route_t *route,
                                    void *workspace, int64_t workspace_bytes, void *stream) {
  ep::Layout L{};
  if (int rc = make_layout(peers, &L)) return rc;
  RowTarget rows;
  for (int s = 0; s < L.n_rank; ++s) {
    rows.blk[s] = reinterpret_cast<float *>(L.peer[s] + L.yback_off) + int64_t(L.rank) * L.cap * L.K;
    rows.arrive[s] = reinterpret_cast<uint32_t *>(L.peer[s] + L.ctrl_off) + ep::kFlags + 8 + L.rank;
  }
  rows.cap = L.cap;
  rows.ld = L.K;
  rows.skip_zero = true;   // rows with expert -1 are padding nobody reads
  rows.done = reinterpret_cast<uint32_t *>(L.peer[L.rank] + L.ctrl_off) + ep::kDone;
  rows.n_arrive = L.n_rank;
  return moe_ffn_to_rows(gate, up, up_row0, down, L.peer[L.rank], MSB_TYPE_BF16, L.row_bytes, route,
                         L.n_rank * L.cap, rows, workspace, workspace_bytes, stream);
}
