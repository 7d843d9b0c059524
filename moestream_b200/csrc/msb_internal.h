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
    uint64_t t0;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t0));
    for (;;) {
      uint32_t v;
      asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(f) : "memory");
      if (int32_t(v - seq) >= 0) break;
      uint64_t t;
      asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
      if (t - t0 > uint64_t(w.limit_ns)) { ok = false; break; }
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
