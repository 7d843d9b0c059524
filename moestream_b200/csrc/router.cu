// Router on the device: the top_k experts of every token and their weights.
//
// In the reference the router runs in llama.cpp's MoE graph ahead of the
// remap (build_remap, src/llama-moestream.cpp:2555, receives the selected
// ids): ggml argsort-top-k over the router logits, then either a
// softmax over the k selected logits (gpt-oss) or a softmax over all
// experts whose selected probabilities are used as they are, or after
// renormalisation (which equals the first form). Here it is one kernel so
// the ids never leave the device before the remap.
//
// One warp per token. Lane l holds the logits of experts l, l + 32, ... in
// registers (n_expert <= 1024). Each of the top_k rounds takes the warp's
// largest remaining logit, lower expert index first among equal values (the
// order of a stable descending sort), with a butterfly of shuffles; the
// owning lane marks it taken. NaN logits count as -inf. Lane k keeps the
// k-th pick; the weights are a softmax computed in f32 with expf (uniform
// when every logit of the token is -inf).
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cfloat>
#include <climits>

#include "msb_internal.h"

namespace msb {

namespace {

constexpr int kRouterWarps = 8;

struct RouterArgs {
  const char *logits;
  int64_t nb1;
  int type;
  int32_t n_tok, n_expert, top_k, mode;
  int32_t *ids;
  float *w;
};

__device__ __forceinline__ float load_logit(const char *row, int type, int e) {
  float v;
  if (type == MSB_TYPE_F32) {
    v = reinterpret_cast<const float *>(row)[e];
  } else if (type == MSB_TYPE_BF16) {
    v = __uint_as_float(uint32_t(reinterpret_cast<const uint16_t *>(row)[e]) << 16);
  } else {
    v = __half2float(reinterpret_cast<const __half *>(row)[e]);
  }
  return v != v ? -INFINITY : v;
}

template <int PER>
__global__ void __launch_bounds__(kRouterWarps * 32) router_kernel(RouterArgs a) {
  pdl_wait();
  const int lane = threadIdx.x & 31;
  const int t = blockIdx.x * kRouterWarps + int(threadIdx.x >> 5);
  if (t >= a.n_tok) return;
  const char *row = a.logits + int64_t(t) * a.nb1;
  float v[PER];
#pragma unroll
  for (int j = 0; j < PER; ++j) {
    const int e = j * 32 + lane;
    v[j] = e < a.n_expert ? load_logit(row, a.type, e) : -INFINITY;
  }
  uint32_t taken = 0;
  // Padding entries (e >= n_expert) are never picked: they are marked taken.
#pragma unroll
  for (int j = 0; j < PER; ++j)
    if (j * 32 + lane >= a.n_expert) taken |= 1u << j;
  float my_v = -INFINITY;
  int my_e = -1;
  for (int k = 0; k < a.top_k; ++k) {
    float bv = -INFINITY;
    int be = INT_MAX;
#pragma unroll
    for (int j = 0; j < PER; ++j) {
      const bool free = !(taken >> j & 1u);
      // Ascending j is ascending expert index: strict > keeps the lowest.
      if (free && (v[j] > bv || be == INT_MAX)) {
        bv = v[j];
        be = j * 32 + lane;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oe = __shfl_xor_sync(0xffffffffu, be, o);
      if (ov > bv || (ov == bv && oe < be)) {
        bv = ov;
        be = oe;
      }
    }
    if ((be & 31) == lane) taken |= 1u << (be >> 5);
    if (lane == k) {
      my_v = bv;
      my_e = be;
    }
  }
  const float m = __shfl_sync(0xffffffffu, my_v, 0);  // the largest logit
  // Every logit -inf (or NaN): the limit of equal logits, uniform weights.
  const bool flat = m == -INFINITY;
  float ex = lane < a.top_k ? (flat ? 1.f : expf(my_v - m)) : 0.f;
  float z;
  if (a.mode == MSB_ROUTER_SOFTMAX_TOPK) {
    z = ex;
  } else {
    z = 0.f;
#pragma unroll
    for (int j = 0; j < PER; ++j)
      if (j * 32 + lane < a.n_expert) z += flat ? 1.f : expf(v[j] - m);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) z += __shfl_xor_sync(0xffffffffu, z, o);
  if (lane < a.top_k) {
    a.ids[int64_t(t) * a.top_k + lane] = my_e;
    a.w[int64_t(t) * a.top_k + lane] = ex / z;
  }
  pdl_trigger();
}

template <int PER>
cudaError_t launch(const RouterArgs &a, cudaStream_t st) {
  const dim3 grid((a.n_tok + kRouterWarps - 1) / kRouterWarps);
  return launch_pdl(router_kernel<PER>, grid, dim3(kRouterWarps * 32), 0, st, a);
}

}  // namespace
}  // namespace msb

extern "C" int msb_router_topk(const void *logits_dev, int logits_type, int64_t nb1,
                               int32_t n_tok, int32_t n_expert, int32_t top_k, int mode,
                               int32_t *ids_dev, float *w_dev, void *stream) {
  MSB_CHECK_ARG(logits_type == MSB_TYPE_F32 || logits_type == MSB_TYPE_F16 ||
                    logits_type == MSB_TYPE_BF16,
                "msb_router_topk: logits must be f32, f16 or bf16");
  MSB_CHECK_ARG(n_expert >= 1 && n_expert <= 1024, "msb_router_topk: n_expert %d not in [1, 1024]",
                n_expert);
  MSB_CHECK_ARG(top_k >= 1 && top_k <= 32 && top_k <= n_expert,
                "msb_router_topk: top_k %d not in [1, min(32, n_expert)]", top_k);
  MSB_CHECK_ARG(mode == MSB_ROUTER_SOFTMAX_TOPK || mode == MSB_ROUTER_SOFTMAX_ALL,
                "msb_router_topk: unknown mode %d", mode);
  MSB_CHECK_ARG(n_tok >= 0, "msb_router_topk: n_tok < 0");
  if (n_tok == 0) return MSB_OK;
  const int es = logits_type == MSB_TYPE_F32 ? 4 : 2;
  MSB_CHECK_ARG(logits_dev && ids_dev && w_dev, "msb_router_topk: null pointer");
  MSB_CHECK_ARG(nb1 >= int64_t(n_expert) * es && nb1 % es == 0 &&
                    reinterpret_cast<uintptr_t>(logits_dev) % es == 0,
                "msb_router_topk: bad row stride %lld", (long long)nb1);
  const msb::RouterArgs a{static_cast<const char *>(logits_dev), nb1, logits_type, n_tok,
                          n_expert, top_k, mode, ids_dev, w_dev};
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e;
  if (n_expert <= 32) e = msb::launch<1>(a, st);
  else if (n_expert <= 64) e = msb::launch<2>(a, st);
  else if (n_expert <= 128) e = msb::launch<4>(a, st);
  else if (n_expert <= 256) e = msb::launch<8>(a, st);
  else if (n_expert <= 512) e = msb::launch<16>(a, st);
  else e = msb::launch<32>(a, st);
  if (e != cudaSuccess) return msb::fail(MSB_ERR_CUDA, "router launch: %s", cudaGetErrorString(e));
  msb::count_launch();
  return MSB_OK;
}
