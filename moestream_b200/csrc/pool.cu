// Slot pool: device slab of n_slot + 1 expert slots, slot fills (ggml block
// layout in, device layout out) and device quantizers.
//
// The reference allocates each expert tensor as [K, N, n_slot + 1]
// (src/apply.py:47-83), zero-fills the last slot (ensure_zero_slot,
// src/llama-moestream.cpp:1749-1792) and fills missing experts with pread into
// the slot's bytes (:1954-2028). Here a fill is a host-to-device copy into a
// staging area owned by the pool, followed by a repack kernel that transposes
// the expert into the block-major layout the matmul reads (quant.cuh).
#include <cuda_runtime.h>

#include <cmath>
#include <cstring>
#include <new>

#include "msb_internal.h"
#include "pool.cuh"
#include "quant.cuh"

namespace msb {

// ggml-layout expert (rows of `nb` blocks) -> device layout, one CTA per
// (expert, 32-row tile) (repack_tile in pool.cuh).
__global__ void __launch_bounds__(256) repack_to_device_kernel(
    const uint8_t *const *srcs, const int32_t *slots, uint8_t *pool_base,
    int64_t slot_stride, int64_t N, int64_t nb, int block_bytes,
    int scale_bytes, int tiles_per_expert) {
  extern __shared__ uint8_t tile[];
  const int ex = blockIdx.x / tiles_per_expert;
  const int64_t n0 = int64_t(blockIdx.x % tiles_per_expert) * kRepackRows;
  repack_tile(tile, srcs[ex], pool_base + int64_t(slots[ex]) * slot_stride, n0, N, nb,
              block_bytes, scale_bytes);
}

// Device layout -> ggml layout for one slot (used to check fills).
__global__ void __launch_bounds__(256) repack_to_ggml_kernel(
    const uint8_t *slot_base, uint8_t *dst, int64_t N, int64_t nb,
    int block_bytes, int scale_bytes) {
  const int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= N * nb) return;
  const int64_t n = i / nb, b = i % nb;
  const uint8_t *qs = slot_base + (b * N + n) * 16;
  const uint8_t *sc = slot_base + nb * N * 16 + scale_offset(scale_bytes == 1, b, n, N, nb);
  uint8_t *o = dst + (n * nb + b) * block_bytes;
  for (int j = 0; j < scale_bytes; ++j) o[j] = sc[j];
  for (int j = 0; j < 16; ++j) o[scale_bytes + j] = qs[j];
}

// ---------------------------------------------------------------------------
// Quantizers: one thread per 32-element block. Products and differences use
// explicit round-to-nearest intrinsics so no fused multiply-add changes the
// result; the CPU oracle is compiled without contraction and matches bit for
// bit.
// ---------------------------------------------------------------------------

// floor(log2(x)) for finite x > 0, exact (frexp exponent minus one).
__device__ __forceinline__ int floor_log2(float x) {
  int ex;
  frexpf(x, &ex);
  return ex - 1;
}

__device__ __forceinline__ int nearest_code(float x, float d, const int8_t *cb) {
  int best = 0;
  float best_err = fabsf(__fsub_rn(__fmul_rn(d, float(cb[0])), x));
  for (int i = 1; i < 16; ++i) {
    const float err = fabsf(__fsub_rn(__fmul_rn(d, float(cb[i])), x));
    if (err < best_err) { best_err = err; best = i; }
  }
  return best;
}

__constant__ int8_t c_kv_mxfp4[16] = {0, 1, 2, 3, 4, 6, 8, 12,
                                      0, -1, -2, -3, -4, -6, -8, -12};
__constant__ int8_t c_kv_iq4nl[16] = {-127, -104, -83, -65, -49, -35, -22, -10,
                                      1, 13, 25, 38, 53, 69, 89, 113};

__global__ void quantize_mxfp4_kernel(const float *src, uint8_t *dst,
                                      int64_t n_blocks) {
  const int64_t blk = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (blk >= n_blocks) return;
  const float *x = src + blk * 32;
  float amax = 0.f;
  for (int j = 0; j < 32; ++j) amax = fmaxf(amax, fabsf(x[j]));
  // ggml/gguf MXFP4: e = floor(log2(amax)) - 2 + 127, scale 2^(e-128).
  const uint32_t e = amax > 0.f ? uint32_t(uint8_t(floor_log2(amax) - 2 + 127)) : 0u;
  const float d = e8m0_half(e);
  uint8_t *o = dst + blk * 17;
  o[0] = uint8_t(e);
  for (int j = 0; j < 16; ++j) {
    const int lo = nearest_code(x[j], d, c_kv_mxfp4);
    const int hi = nearest_code(x[j + 16], d, c_kv_mxfp4);
    o[1 + j] = uint8_t(lo | (hi << 4));
  }
}

// Squared error of a block coded at scale d; optionally accumulates the
// least-squares terms sum(x*l) and sum(l*l) of the chosen codes l.
__device__ float iq4nl_block_sse(const float *x, float d, float *sxl, float *sll) {
  float sse = 0.f, a = 0.f, b = 0.f;
  for (int j = 0; j < 32; ++j) {
    const float l = float(c_kv_iq4nl[nearest_code(x[j], d, c_kv_iq4nl)]);
    const float r = __fsub_rn(x[j], __fmul_rn(d, l));
    sse = __fadd_rn(sse, __fmul_rn(r, r));
    a = __fadd_rn(a, __fmul_rn(x[j], l));
    b = __fadd_rn(b, __fmul_rn(l, l));
  }
  if (sxl) *sxl = a;
  if (sll) *sll = b;
  return sse;
}

// IQ4_NL scale search: start from the scale that maps the largest-magnitude
// element onto the codebook's end (-127), refine once by least squares for
// the chosen codes, keep whichever fp16 scale has the smaller squared error.
// Codes are those nearest to each element at the kept scale.
__global__ void quantize_iq4nl_kernel(const float *src, uint8_t *dst,
                                      int64_t n_blocks) {
  const int64_t blk = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (blk >= n_blocks) return;
  const float *x = src + blk * 32;
  float amax = 0.f, vmax = 0.f;
  for (int j = 0; j < 32; ++j) {
    const float a = fabsf(x[j]);
    if (a > amax) { amax = a; vmax = x[j]; }
  }
  float d = 0.f;
  if (amax != 0.f) {
    d = __half2float(__float2half_rn(vmax / -127.f));
    float sxl, sll;
    const float sse0 = iq4nl_block_sse(x, d, &sxl, &sll);
    const float d1 = __half2float(__float2half_rn(sxl / sll));
    const float sse1 = iq4nl_block_sse(x, d1, nullptr, nullptr);
    if (sse1 < sse0) d = d1;
  }
  // Block bytes as nine 16-bit words (the block starts on an even byte).
  unsigned short *o = reinterpret_cast<unsigned short *>(dst + blk * 18);
  o[0] = __half_as_ushort(__float2half_rn(d));
  for (int j = 0; j < 16; j += 2) {
    unsigned short w = 0;
    for (int h = 0; h < 2; ++h) {
      const int lo = amax != 0.f ? nearest_code(x[j + h], d, c_kv_iq4nl) : 8;
      const int hi = amax != 0.f ? nearest_code(x[j + h + 16], d, c_kv_iq4nl) : 8;
      w |= (unsigned short)((lo | (hi << 4)) << (8 * h));
    }
    o[1 + j / 2] = w;
  }
}

}  // namespace msb

namespace msb {

bool encode_tmap_u64_3d(CUtensorMap *map, const void *base, const uint64_t dims[3],
                        const uint64_t strides[2], const uint32_t box[3]) {
  typedef CUresult (*EncodeFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *,
                               const cuuint64_t *, const cuuint64_t *, const cuuint32_t *,
                               const cuuint32_t *, CUtensorMapInterleave, CUtensorMapSwizzle,
                               CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
  static EncodeFn fn = nullptr;
  static bool looked = false;
  if (!looked) {
    looked = true;
    void *ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeFn>(ptr);
  }
  if (!fn) return false;
  const cuuint32_t estr[3] = {1, 1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT64, 3, const_cast<void *>(base), dims, strides, box,
            estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace msb

using namespace msb;

static int64_t round_up(int64_t x, int64_t a) { return (x + a - 1) / a * a; }

extern "C" int msb_pool_create(int wtype, int64_t K, int64_t N, int32_t n_slot,
                               int32_t max_fill_batch, msb_pool_t *out) {
  BlockFormat f;
  MSB_CHECK_ARG(out, "msb_pool_create: null out");
  MSB_CHECK_ARG(block_format(wtype, &f), "msb_pool_create: weight type %d is not IQ4_NL or MXFP4", wtype);
  MSB_CHECK_ARG(K > 0 && K % 32 == 0 && N > 0, "msb_pool_create: K must be a positive multiple of 32 and N positive");
  MSB_CHECK_ARG(n_slot > 0, "msb_pool_create: n_slot must be positive");
  if (max_fill_batch <= 0) max_fill_batch = 4;
  msb_pool_s *p = new (std::nothrow) msb_pool_s();
  if (!p) return fail(MSB_ERR_NOMEM, "msb_pool_create: out of memory");
  p->wtype = wtype;
  p->K = K;
  p->N = N;
  p->nb = K / 32;
  p->n_slot = n_slot;
  p->block_bytes = f.block_bytes;
  p->scale_bytes = f.scale_bytes;
  p->expert_bytes = p->nb * f.block_bytes * N;
  p->slot_stride = round_up(p->nb * N * 16 + scale_region_bytes(wtype == MSB_TYPE_MXFP4, p->nb, N), 256);
  p->max_fill = max_fill_batch;
  cudaGetDevice(&p->device);
  const int64_t slab = p->slot_stride * (int64_t(n_slot) + 1);
  const int64_t meta = round_up(int64_t(max_fill_batch) * (sizeof(int32_t) + sizeof(void *)) + 16, 256);
  cudaError_t e = cudaMalloc(&p->data, slab);
  if (e != cudaSuccess) { delete p; return fail(MSB_ERR_NOMEM, "msb_pool_create: cudaMalloc(%lld) failed: %s", (long long)slab, cudaGetErrorString(e)); }
  e = cudaMalloc(&p->stage_meta, meta);
  if (e != cudaSuccess) { cudaFree(p->data); delete p; return fail(MSB_ERR_NOMEM, "msb_pool_create: metadata cudaMalloc failed: %s", cudaGetErrorString(e)); }
  e = cudaMallocHost(&p->host_meta, meta);
  if (e != cudaSuccess) { cudaFree(p->stage_meta); cudaFree(p->data); delete p; return fail(MSB_ERR_NOMEM, "msb_pool_create: pinned metadata failed: %s", cudaGetErrorString(e)); }
  e = cudaEventCreateWithFlags(&p->meta_free, cudaEventDisableTiming);
  if (e == cudaSuccess) e = cudaMemset(p->data, 0, slab);  // every slot starts as zeros
  if (e == cudaSuccess && wtype == MSB_TYPE_MXFP4) {
    const uint64_t dims[3] = {uint64_t(N) * 2, uint64_t(p->nb), uint64_t(n_slot) + 1};
    const uint64_t strides[2] = {uint64_t(N) * 16, uint64_t(p->slot_stride)};
    const uint32_t box[3] = {256, 4, 1}, box8[3] = {256, 8, 1};
    p->has_tmap = encode_tmap_u64_3d(&p->tmap_w, p->data, dims, strides, box) &&
                  encode_tmap_u64_3d(&p->tmap_w8, p->data, dims, strides, box8);
  }
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e != cudaSuccess) { msb_pool_destroy(p); return fail(MSB_ERR_CUDA, "msb_pool_create: init failed: %s", cudaGetErrorString(e)); }
  *out = p;
  return MSB_OK;
}

extern "C" int msb_pool_destroy(msb_pool_t p) {
  if (!p) return MSB_OK;
  if (p->meta_free) { cudaEventSynchronize(p->meta_free); cudaEventDestroy(p->meta_free); }
  if (p->host_meta) cudaFreeHost(p->host_meta);
  if (p->stage) cudaFree(p->stage);
  if (p->stage_meta) cudaFree(p->stage_meta);
  if (p->data) cudaFree(p->data);
  delete p;
  return MSB_OK;
}

extern "C" int msb_pool_get_info(msb_pool_t p, msb_pool_info_t *out) {
  MSB_CHECK_ARG(p && out, "msb_pool_get_info: null argument");
  out->wtype = p->wtype;
  out->K = p->K;
  out->N = p->N;
  out->n_slot = p->n_slot;
  out->device = p->device;
  out->expert_bytes = p->expert_bytes;
  out->slot_stride = p->slot_stride;
  out->data = p->data;
  return MSB_OK;
}

// Launches the repack of `n` ggml-layout experts whose device addresses and
// destination slots are first staged in pinned host memory and copied to
// the pool's device metadata block (so the kernel reads them by pointer).
static int launch_repack(msb_pool_s *p, int32_t n, const int32_t *slots,
                         const void *const *src_dev, cudaStream_t st) {
  // The pinned metadata block may still be read by a previous copy.
  MSB_CUDA_TRY(cudaEventSynchronize(p->meta_free));
  int32_t *hs = reinterpret_cast<int32_t *>(p->host_meta);
  const uint8_t **hp = reinterpret_cast<const uint8_t **>(
      p->host_meta + round_up(int64_t(p->max_fill) * sizeof(int32_t), 16));
  for (int i = 0; i < n; ++i) {
    hs[i] = slots[i];
    hp[i] = static_cast<const uint8_t *>(src_dev[i]);
  }
  const int64_t meta = round_up(int64_t(p->max_fill) * sizeof(int32_t), 16) + int64_t(p->max_fill) * sizeof(void *);
  MSB_CUDA_TRY(cudaMemcpyAsync(p->stage_meta, p->host_meta, meta, cudaMemcpyHostToDevice, st));
  MSB_CUDA_TRY(cudaEventRecord(p->meta_free, st));
  const int32_t *ds = reinterpret_cast<const int32_t *>(p->stage_meta);
  const uint8_t *const *dp = reinterpret_cast<const uint8_t *const *>(
      p->stage_meta + round_up(int64_t(p->max_fill) * sizeof(int32_t), 16));
  const int tiles = int((p->N + kRepackRows - 1) / kRepackRows);
  const size_t smem = size_t(kRepackRows) * p->nb * p->block_bytes;
  if (smem > 48 * 1024)
    MSB_CUDA_TRY(cudaFuncSetAttribute(repack_to_device_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)));
  repack_to_device_kernel<<<n * tiles, 256, smem, st>>>(
      dp, ds, p->data, p->slot_stride, p->N, p->nb, p->block_bytes, p->scale_bytes, tiles); count_launch();
  MSB_CUDA_TRY(cudaGetLastError());
  return MSB_OK;
}

static int check_slots(msb_pool_s *p, int32_t n, const int32_t *slots) {
  for (int i = 0; i < n; ++i)
    MSB_CHECK_ARG(slots[i] >= 0 && slots[i] < p->n_slot,
                  "fill: slot %d out of range [0, %d) (the zero slot cannot be filled)", slots[i], p->n_slot);
  const int64_t smem = int64_t(kRepackRows) * p->nb * p->block_bytes;
  if (smem > 227 * 1024)
    return fail(MSB_ERR_UNSUPPORTED, "fill: rows of %lld bytes exceed the repack tile", (long long)(p->nb * p->block_bytes));
  return MSB_OK;
}

extern "C" int msb_fill_slots_async(msb_pool_t p, int32_t n, const int32_t *slots,
                                    const void *const *src_host, void *stream) {
  MSB_CHECK_ARG(p && (n == 0 || (slots && src_host)), "msb_fill_slots_async: null argument");
  if (int rc = check_slots(p, n, slots)) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int64_t pitch = round_up(p->expert_bytes, 256);
  if (!p->stage && n > 0) {
    // Staging for host sources is allocated on the first host fill; pools
    // filled only from device memory never need it.
    const cudaError_t e = cudaMalloc(&p->stage, pitch * p->max_fill);
    if (e != cudaSuccess)
      return fail(MSB_ERR_NOMEM, "fill: staging cudaMalloc(%lld) failed: %s",
                  (long long)(pitch * p->max_fill), cudaGetErrorString(e));
  }
  for (int32_t i0 = 0; i0 < n; i0 += p->max_fill) {
    const int32_t m = n - i0 < p->max_fill ? n - i0 : p->max_fill;
    const void *dev[64];
    int32_t sl[64];
    for (int32_t j0 = 0; j0 < m; j0 += 64) {
      const int32_t mm = m - j0 < 64 ? m - j0 : 64;
      for (int32_t j = 0; j < mm; ++j) {
        uint8_t *dst = p->stage + int64_t(j0 + j) * pitch;
        MSB_CUDA_TRY(cudaMemcpyAsync(dst, src_host[i0 + j0 + j], p->expert_bytes, cudaMemcpyHostToDevice, st));
        dev[j] = dst;
        sl[j] = slots[i0 + j0 + j];
      }
      if (int rc = launch_repack(p, mm, sl, dev, st)) return rc;
    }
  }
  return MSB_OK;
}

extern "C" int msb_fill_slots_from_device_async(msb_pool_t p, int32_t n, const int32_t *slots,
                                                const void *const *src_dev, void *stream) {
  MSB_CHECK_ARG(p && (n == 0 || (slots && src_dev)), "msb_fill_slots_from_device_async: null argument");
  if (int rc = check_slots(p, n, slots)) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  for (int32_t i0 = 0; i0 < n; i0 += p->max_fill) {
    const int32_t m = n - i0 < p->max_fill ? n - i0 : p->max_fill;
    if (int rc = launch_repack(p, m, slots + i0, src_dev + i0, st)) return rc;
  }
  return MSB_OK;
}

extern "C" int msb_read_slot_async(msb_pool_t p, int32_t slot, void *dst_dev, void *stream) {
  MSB_CHECK_ARG(p && dst_dev && slot >= 0 && slot <= p->n_slot, "msb_read_slot_async: bad argument");
  const int64_t total = p->N * p->nb;
  repack_to_ggml_kernel<<<int((total + 255) / 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      p->data + int64_t(slot) * p->slot_stride, static_cast<uint8_t *>(dst_dev), p->N, p->nb,
      p->block_bytes, p->scale_bytes); count_launch();
  MSB_CUDA_TRY(cudaGetLastError());
  return MSB_OK;
}

extern "C" int msb_quantize_rows(int wtype, const float *src_dev, int64_t n_rows, int64_t K,
                                 void *dst_dev, void *stream) {
  MSB_CHECK_ARG(src_dev && dst_dev && n_rows >= 0 && K > 0 && K % 32 == 0, "msb_quantize_rows: bad argument");
  const int64_t n_blocks = n_rows * (K / 32);
  if (n_blocks == 0) return MSB_OK;
  const int threads = 128;
  const int64_t grid = (n_blocks + threads - 1) / threads;
  MSB_CHECK_ARG(grid < (int64_t(1) << 31), "msb_quantize_rows: too many blocks in one call");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  MSB_CHECK_ARG((reinterpret_cast<uintptr_t>(dst_dev) & 1) == 0,
                "msb_quantize_rows: dst must be 2-byte aligned");
  if (wtype == MSB_TYPE_MXFP4)
    quantize_mxfp4_kernel<<<unsigned(grid), threads, 0, st>>>(src_dev, static_cast<uint8_t *>(dst_dev), n_blocks);
  else if (wtype == MSB_TYPE_IQ4_NL)
    quantize_iq4nl_kernel<<<unsigned(grid), threads, 0, st>>>(src_dev, static_cast<uint8_t *>(dst_dev), n_blocks);
  else
    return fail(MSB_ERR_INVALID, "msb_quantize_rows: weight type %d is not IQ4_NL or MXFP4", wtype);
  count_launch();
  MSB_CUDA_TRY(cudaGetLastError());
  return MSB_OK;
}
