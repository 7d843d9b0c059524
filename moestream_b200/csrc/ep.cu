// Expert-parallel packing around the all-to-all exchanges.
//
// The reference runs in one process on one GPU and has no expert
// parallelism; this is the layer's token dispatch and combine when the
// experts are split evenly over the GPUs of one node (expert e on rank
// e / n_local). Each rank packs its (token, k) rows into fixed-capacity
// per-destination blocks, so the exchange is an equal-split all-to-all that
// needs no host round trip for counts; rows a destination does not receive
// carry expert -1 and land in the zero slot there.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include "msb_internal.h"

namespace msb {

static constexpr int kEpThreads = 256;

// One CTA per (token, k) pair: its rank among earlier pairs with the same
// destination fixes its row in the send buffer; the CTA then copies the
// token's activation row there as bf16.
template <typename T>
__global__ void __launch_bounds__(kEpThreads) ep_dispatch_kernel(
    const int32_t *ids, const char *x, int64_t x_nb1, int32_t top_k, int32_t n_pairs,
    int64_t K, int32_t n_local, int32_t n_rank, int32_t cap, char *send_x, int64_t send_nb1,
    char *send_e, int64_t send_e_nb, int32_t *pos) {
  pdl_wait();
  pdl_trigger();
  __shared__ int warp_cnt[kEpThreads / 32];
  const int p = blockIdx.x;
  const int e = ids[p];
  const int dest = (e >= 0 && e < n_local * n_rank) ? e / n_local : -1;
  int c = 0;
  if (dest >= 0) {
    for (int q = threadIdx.x; q < p; q += kEpThreads) {
      const int eq = ids[q];
      c += (eq >= 0 && eq < n_local * n_rank && eq / n_local == dest);
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) c += __shfl_xor_sync(0xffffffffu, c, o);
  if ((threadIdx.x & 31) == 0) warp_cnt[threadIdx.x >> 5] = c;
  __syncthreads();
  int rank = 0;
  for (int w = 0; w < kEpThreads / 32; ++w) rank += warp_cnt[w];
  if (dest < 0 || rank >= cap) {
    if (threadIdx.x == 0) pos[p] = -1;
    return;
  }
  const int row = dest * cap + rank;
  if (threadIdx.x == 0) {
    pos[p] = row;
    *reinterpret_cast<int32_t *>(send_e + int64_t(row) * send_e_nb) = e - dest * n_local;
  }
  const int t = p / top_k;
  const T *src = reinterpret_cast<const T *>(x + int64_t(t) * x_nb1);
  __nv_bfloat16 *dst = reinterpret_cast<__nv_bfloat16 *>(send_x + int64_t(row) * send_nb1);
  for (int64_t i = threadIdx.x; i < K; i += kEpThreads) {
    if constexpr (sizeof(T) == 2) dst[i] = src[i];
    else dst[i] = __float2bfloat16_rn(src[i]);
  }
}

// y[t, n] = sum_k w[t, k] * back[pos[t, k], n], k ascending; pos -1 adds 0.
__global__ void ep_combine_kernel(const float *back, const int32_t *pos, const float *w,
                                  int32_t top_k, int64_t K, int64_t n_tok, float *y,
                                  FlagWait wait) {
  pdl_wait();
  pdl_trigger();
  flag_wait_block(wait);
  const int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= n_tok * K) return;
  const int64_t t = i / K, n = i - t * K;
  float s = 0.f;
  for (int k = 0; k < top_k; ++k) {
    const int r = pos[t * top_k + k];
    if (r >= 0) s = fmaf(w[t * top_k + k], back[int64_t(r) * K + n], s);
  }
  y[i] = s;
}

}  // namespace msb

extern "C" int msb_ep_dispatch(const int32_t *ids_dev, const void *x_dev, int x_type,
                               int64_t x_nb1, int32_t top_k, int32_t n_tok, int64_t K,
                               int32_t n_local, int32_t n_rank, int32_t cap, void *send_x_dev,
                               int64_t send_nb1, int32_t *send_e_dev, int64_t send_e_nb,
                               int32_t *pos_dev, void *stream) {
  MSB_CHECK_ARG(top_k > 0 && n_tok >= 0 && K > 0 && n_local > 0 && n_rank > 0 && cap > 0,
                "msb_ep_dispatch: bad shape");
  MSB_CHECK_ARG(send_x_dev && send_e_dev && pos_dev && (n_tok == 0 || (ids_dev && x_dev)),
                "msb_ep_dispatch: null argument");
  MSB_CHECK_ARG(send_nb1 >= 2 * K && send_nb1 % 2 == 0 && send_e_nb >= 4 && send_e_nb % 4 == 0 &&
                    reinterpret_cast<uintptr_t>(send_e_dev) % 4 == 0,
                "msb_ep_dispatch: bad send strides");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // Every id starts as -1 (unused row): one 4-byte column of send_e_nb pitch.
  MSB_CUDA_TRY(cudaMemset2DAsync(send_e_dev, size_t(send_e_nb), 0xFF, sizeof(int32_t),
                                 size_t(n_rank) * cap, st));
  const int n_pairs = top_k * n_tok;
  if (n_pairs == 0) return MSB_OK;
  const char *x = static_cast<const char *>(x_dev);
  auto *sx = static_cast<char *>(send_x_dev);
  auto *se = reinterpret_cast<char *>(send_e_dev);
  if (x_type == MSB_TYPE_BF16)
    MSB_CUDA_TRY(msb::launch_pdl(msb::ep_dispatch_kernel<__nv_bfloat16>, dim3(n_pairs),
                                 dim3(msb::kEpThreads), 0, st, ids_dev, x, x_nb1, top_k, n_pairs,
                                 K, n_local, n_rank, cap, sx, send_nb1, se, send_e_nb, pos_dev));
  else if (x_type == MSB_TYPE_F32)
    MSB_CUDA_TRY(msb::launch_pdl(msb::ep_dispatch_kernel<float>, dim3(n_pairs),
                                 dim3(msb::kEpThreads), 0, st, ids_dev, x, x_nb1, top_k, n_pairs,
                                 K, n_local, n_rank, cap, sx, send_nb1, se, send_e_nb, pos_dev));
  else
    return msb::fail(MSB_ERR_INVALID, "msb_ep_dispatch: activation type %d", x_type);
  msb::count_launch();
  MSB_CUDA_TRY(cudaGetLastError());
  return MSB_OK;
}

extern "C" int msb_ep_combine(const float *back_dev, const int32_t *pos_dev, const float *w_dev,
                              int32_t top_k, int32_t n_tok, int64_t K, float *y_dev,
                              void *stream) {
  return msb::ep_combine_wait(back_dev, pos_dev, w_dev, top_k, n_tok, K, y_dev, msb::FlagWait{},
                              stream);
}

int msb::ep_combine_wait(const float *back_dev, const int32_t *pos_dev, const float *w_dev,
                         int32_t top_k, int32_t n_tok, int64_t K, float *y_dev,
                         const FlagWait &wait, void *stream) {
  MSB_CHECK_ARG(top_k > 0 && n_tok >= 0 && K > 0, "msb_ep_combine: bad shape");
  MSB_CHECK_ARG(n_tok == 0 || (back_dev && pos_dev && w_dev && y_dev),
                "msb_ep_combine: null argument");
  const int64_t total = int64_t(n_tok) * K;
  if (total == 0) return MSB_OK;
  MSB_CUDA_TRY(msb::launch_pdl(msb::ep_combine_kernel, dim3(unsigned((total + 255) / 256)),
                               dim3(256), 0, static_cast<cudaStream_t>(stream), back_dev, pos_dev,
                               w_dev, top_k, K, int64_t(n_tok), y_dev, wait));
  msb::count_launch();
  MSB_CUDA_TRY(cudaGetLastError());
  return MSB_OK;
}
