// Slot pool object shared by the fill and matmul translation units.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "msb_internal.h"
#include "quant.cuh"

struct msb_pool_s {
  int wtype = 0;
  int64_t K = 0, N = 0, nb = 0;  // nb = K / 32 blocks per row
  int32_t n_slot = 0;            // slot n_slot is the zero slot
  int32_t device = 0;
  int block_bytes = 0, scale_bytes = 0;
  int64_t expert_bytes = 0;      // ggml bytes of one expert
  int64_t slot_stride = 0;       // device bytes between slots (256-aligned)
  int32_t max_fill = 0;          // experts staged per fill batch
  uint8_t *data = nullptr;       // slot 0; slot s at data + s * slot_stride
  uint8_t *stage = nullptr;      // fill staging, max_fill * expert pitch (lazy)
  uint8_t *stage_meta = nullptr; // device copy of (slots, source pointers)
  uint8_t *host_meta = nullptr;  // pinned host block for that copy
  cudaEvent_t meta_free = nullptr;
  // 3-D tensor maps of the nibbles in 8-byte elements: (2 per row over the
  // N rows of a block, blocks, slots), box (256, 4, 1) = a 128-row tile of
  // 4 blocks (tmap_w) or (256, 8, 1) = of 8 blocks (tmap_w8), one 2 KB line
  // per block; valid when has_tmap (MXFP4 pools).
  alignas(64) CUtensorMap tmap_w;
  alignas(64) CUtensorMap tmap_w8;
  bool has_tmap = false;
};

namespace msb {

// Encodes a 3-D tensor map of 8-byte elements (dims innermost first, byte
// strides of dims 1..2, box sizes). False when the driver call is
// unavailable or fails.
bool encode_tmap_u64_3d(CUtensorMap *map, const void *base, const uint64_t dims[3],
                        const uint64_t strides[2], const uint32_t box[3]);

// Read-only view of one pool for the matmul kernels. Row n of block b of
// slot s: qs at base + s*slot_stride + (b*N + row0 + n)*16, scale at
// base + s*slot_stride + nb*N*16 + scale_offset(mx, b, row0 + n, N, nb).
struct PoolView {
  const uint8_t *base;
  int64_t slot_stride;
  int64_t N;      // rows stored per slot
  int64_t nb;     // blocks per row
  int64_t row0;   // first row of this view inside the slot
};

inline PoolView view_of(const msb_pool_s *p, int64_t row0 = 0) {
  return PoolView{p->data, p->slot_stride, p->N, p->nb, row0};
}

constexpr int kRepackRows = 32;  // rows per repack tile

#ifdef __CUDACC__
// Rows [n0, n0 + 32) of one ggml-layout expert (rows of `nb` blocks of
// block_bytes, the scale first) -> the device layout of the slot at `dst`.
// The tile's bytes are contiguous in the source: they are staged in shared
// memory with the widest aligned loads (the source may be pinned host
// memory read over the bus) and written out one block column at a time
// (32 rows x 16 bytes contiguous). Uses kRepackRows * nb * block_bytes
// bytes of `tile`; every thread of the block must call it.
__device__ __forceinline__ void repack_tile(uint8_t *tile, const uint8_t *src_expert,
                                            uint8_t *dst, int64_t n0, int64_t N, int64_t nb,
                                            int block_bytes, int scale_bytes) {
  const int rows = int(N - n0 < kRepackRows ? N - n0 : kRepackRows);
  const int64_t row_bytes = nb * block_bytes;
  const uint8_t *src = src_expert + n0 * row_bytes;
  const int64_t tile_bytes = rows * row_bytes;
  if ((reinterpret_cast<uintptr_t>(src) & 15) == 0 && (tile_bytes & 15) == 0) {
    const uint4 *s16 = reinterpret_cast<const uint4 *>(src);
    uint4 *t16 = reinterpret_cast<uint4 *>(tile);
    for (int64_t i = threadIdx.x; i < tile_bytes / 16; i += blockDim.x) t16[i] = s16[i];
  } else if ((reinterpret_cast<uintptr_t>(src) & 3) == 0 && (tile_bytes & 3) == 0) {
    const uint32_t *s4 = reinterpret_cast<const uint32_t *>(src);
    uint32_t *t4 = reinterpret_cast<uint32_t *>(tile);
    for (int64_t i = threadIdx.x; i < tile_bytes / 4; i += blockDim.x) t4[i] = s4[i];
  } else {
    for (int64_t i = threadIdx.x; i < tile_bytes; i += blockDim.x) tile[i] = src[i];
  }
  __syncthreads();
  uint8_t *dst_scale = dst + nb * N * 16;
  const bool mx = scale_bytes == 1;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane < rows) {
    const int64_t n = n0 + lane;
    for (int64_t b = warp; b < nb; b += blockDim.x / 32) {
      const uint8_t *blk = tile + lane * row_bytes + b * block_bytes;
      uint8_t q[16];
#pragma unroll
      for (int j = 0; j < 16; ++j) q[j] = blk[scale_bytes + j];
      uint4 v;
      memcpy(&v, q, 16);
      *reinterpret_cast<uint4 *>(dst + (b * N + n) * 16) = v;
      uint8_t *sd = dst_scale + scale_offset(mx, b, n, N, nb);
      for (int j = 0; j < scale_bytes; ++j) sd[j] = blk[j];
    }
  }
  __syncthreads();  // the tile may be reused by the caller
}
#endif

}  // namespace msb
