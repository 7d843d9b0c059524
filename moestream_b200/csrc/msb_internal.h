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
