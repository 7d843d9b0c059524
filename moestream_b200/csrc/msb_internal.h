// Internal helpers shared by the host and device translation units.
#pragma once

#include <cstdarg>
#include <cstdint>

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
