// Slot pool object shared by the fill and matmul translation units.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "msb_internal.h"

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
  // 3-D tensor map of the nibbles in 8-byte elements: (2 per row over the
  // N rows of a block, blocks, slots), box (256, 4, 1) = a 128-row tile of
  // 4 blocks, one 2 KB line per block; valid when has_tmap (MXFP4 pools).
  alignas(64) CUtensorMap tmap_w;
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
// base + s*slot_stride + nb*N*16 + scale_offset(mx, b, row0 + n, N).
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

}  // namespace msb
