// Internal helpers shared by the host and device translation units.
#pragma once

#include <cstdarg>
#include <cstdint>
#include <utility>

#ifdef __CUDACC__
#include <cuda_runtime.h>
#endif

#include "../../include/msb.h"

namespace msb {

// Records a formatted message as the calling thread's last error and returns
// `code`, so call sites read `return fail(MSB_ERR_INVALID, "...")`.
int fail(int code, const char *fmt, ...);
void clear_error();

// Counts a kernel launch (reported by msb_kernel_launches).
void count_launch(int n = 1);

// Device address of the library's status word on the current device (bits
// set by kernels whose bounded waits gave up; msb_device_status reads it).
int status_word(int **out);

// How long a bounded device wait spins before it gives up, in nanoseconds
// (MSB_OPT_WAIT_LIMIT_US; one second by default). Read when a launch is set
// up, so a captured CUDA graph keeps the limit it was captured with.
int64_t wait_limit_ns();

// An optional wait at the start of a kernel for flags that other GPUs raise
// (expert-parallel exchange): threads 0..n-1 of every CTA spin, bounded
// (limit_ns), until flags[t] reached *seq * mult, then the CTA synchronizes. A
// wait that gives up sets `bit` in *status. n == 0: no wait.
struct FlagWait {
  const uint32_t *flags = nullptr;
  const uint32_t *seq = nullptr;
  uint32_t mult = 1;
  int n = 0;
  int *status = nullptr;
  int bit = 0;
  long long limit_ns = 1000000000ll;
};

// Where a projection's f32 result rows go when they are not one contiguous
// [pairs][n_out] array: row r at blk[r / cap] + (r % cap) * ld floats (the
// blocks may be other GPUs' memory). Rows routed to the zero slot are not
// written when skip_zero. With done set, the kernel's last CTA to finish
// adds one to every arrive[i] (a system-scope release) once all rows are
// stored; done is a counter of this GPU that starts at and returns to 0.
struct RowTarget {
  float *blk[MSB_EP_MAX_RANKS] = {};
  int32_t cap = 0;
  int64_t ld = 0;
  bool skip_zero = false;
  uint32_t *done = nullptr;
  uint32_t *arrive[MSB_EP_MAX_RANKS] = {};
  int32_t n_arrive = 0;
};

// The router-weighted combine fused into the down projection's epilogue:
// y[t][n] = sum_k w[t][k] * r[t*top_k + k][n] in k order (one f32 fma per
// k, starting from 0), where r is the projection's result rows. Each warp
// that stores a 32-row block of one pair's row counts itself on cnt[t][blk];
// the warp that brings the count to top_k (all of the token's rows of that
// block are stored) reads them back and writes y's block, so the sum runs in
// the same order whichever CTA finishes last. cnt starts at zero (zeroed by
// the kernel that prepares the call's activations).
struct Combine {
  const float *w = nullptr;   // [n_tok][top_k]; null: no combine
  float *y = nullptr;         // [n_tok][n_out]
  const float *r = nullptr;   // [n_tok * top_k][n_out], the rows just stored
  uint32_t *cnt = nullptr;    // [n_tok][nblk]
  int32_t top_k = 0;
  int64_t n_out = 0, nblk = 0;
  bool accumulate = false;    // y += the sum instead of y = the sum
};

// Expert biases (gpt-oss): f32 rows indexed by expert id, added to the f32
// result of every pair not routed to the zero slot. The expert of pair p =
// t * top_k + k is ids[t * nb1 + k * nb0] (byte strides; the router's ids,
// before the remap); ids outside [0, n_expert) add nothing. View v's row of
// expert e starts at b[v] + e * ld[v]. Null b[v]: no bias for that view.
struct FfnBias {
  const float *b[2] = {nullptr, nullptr};
  int64_t ld[2] = {0, 0};
  const char *ids = nullptr;
  int64_t nb0 = 0, nb1 = 0;
  int32_t top_k = 1, n_expert = 0;
};

// The activation between the gate/up and down projections: kind 0 is
// silu(g) * u; kind 1 (MSB_ACT_SWIGLU_OAI) is gpt-oss's clamped form
// min(g, limit) * sigmoid(alpha * min(g, limit)) * (clamp(u, -limit, limit) + 1).
struct FfnAct {
  int kind = 0;
  float alpha = 1.f;
  float limit = 0.f;
};

// msb_moe_ffn whose down projection writes its rows to `rows` (top_k 1, no
// router weights, tensor-core shapes only; MSB_ERR_UNSUPPORTED otherwise,
// before any launch).
int moe_ffn_to_rows(msb_pool_t gate, msb_pool_t up, int64_t up_row0, msb_pool_t down,
                    const void *x_dev, int x_type, int64_t x_nb1, const msb_route_t *route,
                    int32_t n_tok, const RowTarget &rows, void *workspace,
                    int64_t workspace_bytes, void *stream, const FfnAct &fa = FfnAct{});

// msb_remap_group whose kernel first waits on `wait` (route.cu), and
// msb_ep_combine likewise (ep.cu).
int remap_group_wait(const int32_t *ids_dev, int64_t nb0, int64_t nb1, int32_t top_k,
                     int32_t n_tok, const int32_t *table_dev, int32_t n_expert, int32_t n_slot,
                     const msb_route_t *route, const FlagWait &wait, void *stream);
int ep_combine_wait(const float *back_dev, const int32_t *pos_dev, const float *w_dev,
                    int32_t top_k, int32_t n_tok, int64_t K, float *y_dev, const FlagWait &wait,
                    void *stream);

// ggml block geometry of the two weight types.
struct BlockFormat {
  int block_bytes;  // bytes per 32-element block in ggml layout
  int scale_bytes;  // bytes of the per-block scale (e8m0: 1, fp16: 2)
};
inline bool block_format(int wtype, BlockFormat *f) {
  if (wtype == MSB_TYPE_IQ4_NL) { *f = {18, 2}; return true; }
  if (wtype == MSB_TYPE_MXFP4)  { *f = {17, 1}; return true; }
  return false;
}

#ifdef __CUDACC__
// Programmatic dependent launch. Hot-path kernels are launched with
// launch_pdl, which lets a kernel start (and run its prologue) while the
// previous kernel in the stream finishes; every such kernel calls pdl_wait()
// before it reads or writes memory that earlier work uses (the wait returns
// once the previous grid has completed and its writes are visible; without
// the launch attribute it returns at once), and pdl_trigger() once its own
// CTAs are all running, so the next kernel can be scheduled early.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void flag_wait_block(const FlagWait &w) {
  if (w.n == 0) return;
  bool ok = true;
  if (int(threadIdx.x) < w.n) {
    const uint32_t seq = *reinterpret_cast<const volatile uint32_t *>(w.seq) * w.mult;
    const uint32_t *f = w.flags + threadIdx.x;
    // Bounded in SM cycles, 2 per ns of the limit (as sm100::wait_cycles).
    const long long c0 = clock64(), lim = 2 * w.limit_ns;
    for (;;) {
      uint32_t v;
      asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(f) : "memory");
      if (int32_t(v - seq) >= 0) break;
      if (clock64() - c0 > lim) { ok = false; break; }
    }
  }
  if (!ok) atomicOr(w.status, w.bit);
  __syncthreads();
}

template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                              cudaStream_t st, Args &&...args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}
// Called by all 32 lanes of a warp after the warp stored its 32-row block
// `blk` (row n = blk*32 + lane, rows past n_out skipped) of the result rows of
// m pairs; lane l < m passes the l-th pair. One acquire-release atomic per
// pair counts the block (the warp barrier orders every lane's stores before
// it, and release is cumulative); for each pair whose count reached top_k --
// all of its token's rows of the block are stored -- the warp sums them in
// k order and writes y's block (see Combine).
__device__ __forceinline__ void combine_arrive(const Combine &c, int64_t my_pair, int m,
                                               int64_t blk, int lane) {
  if (!c.w || blk >= c.nblk) return;
  __syncwarp();
  uint32_t old = 0;
  int64_t t = 0;
  if (lane < m) {
    t = my_pair / c.top_k;
    asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;"
                 : "=r"(old)
                 : "l"(c.cnt + t * c.nblk + blk)
                 : "memory");
  }
  unsigned last = __ballot_sync(0xffffffffu, lane < m && old == uint32_t(c.top_k - 1));
  const int64_t n = blk * 32 + lane;
  while (last) {
    const int j = __ffs(last) - 1;
    last &= last - 1;
    const int64_t tj = __shfl_sync(0xffffffffu, t, j);
    if (n < c.n_out) {
      float s = 0.f;
      for (int k = 0; k < c.top_k; ++k)
        s = fmaf(c.w[tj * c.top_k + k], __ldcg(c.r + (tj * c.top_k + k) * c.n_out + n), s);
      float *yp = c.y + tj * c.n_out + n;
      *yp = c.accumulate ? *yp + s : s;
    }
  }
}

// Result row r of a RowTarget.
__device__ __forceinline__ float *out_row(const RowTarget &t, int64_t r) {
  const int64_t b = r / t.cap;
  return t.blk[b] + (r - b * t.cap) * t.ld;
}

// Zeroes n words with every thread of the grid (grid-stride).
__device__ __forceinline__ void grid_zero(uint32_t *p, int64_t n) {
  if (!p) return;
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += int64_t(gridDim.x) * blockDim.x)
    p[i] = 0u;
}

// Row of view v's bias for `pair` (null when none applies).
__device__ __forceinline__ const float *bias_row(const FfnBias &f, int v, int64_t pair) {
  if (!f.b[v]) return nullptr;
  const int64_t t = pair / f.top_k, k = pair - t * f.top_k;
  const int32_t e = *reinterpret_cast<const int32_t *>(f.ids + t * f.nb1 + k * f.nb0);
  return (e >= 0 && e < f.n_expert) ? f.b[v] + int64_t(e) * f.ld[v] : nullptr;
}

// h = act(g, u) of FfnAct, in f32 with expf.
__device__ __forceinline__ float ffn_act(const FfnAct &f, float g, float u) {
  if (f.kind == 1) {
    const float x = g < f.limit ? g : f.limit;
    const float y = u < -f.limit ? -f.limit : (u > f.limit ? f.limit : u);
    return x / (1.f + expf(-f.alpha * x)) * (y + 1.f);
  }
  return g / (1.f + expf(-g)) * u;
}
#endif

}  // namespace msb

#define MSB_CUDA_TRY(expr)                                                   \
  do {                                                                       \
    cudaError_t e_ = (expr);                                                 \
    if (e_ != cudaSuccess)                                                   \
      return msb::fail(MSB_ERR_CUDA, "%s failed: %s", #expr,                \
                       cudaGetErrorString(e_));                              \
  } while (0)

#define MSB_CHECK_ARG(cond, ...)                                             \
  do {                                                                       \
    if (!(cond)) return msb::fail(MSB_ERR_INVALID, __VA_ARGS__);             \
  } while (0)
