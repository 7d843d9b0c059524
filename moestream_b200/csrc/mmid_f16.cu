// Tensor-core mul_mat_id for IQ4_NL slot pools: codebook dequantization into
// shared memory, then tcgen05 kind::f16 MMAs.
//
// IQ4_NL stores per 32-element block an fp16 scale d and 16 bytes of 4-bit
// indices into a 16-entry int8 codebook; no tensor-core format takes those
// values directly (the codebook is not an FP4/FP6/FP8 grid). So the weights
// are dequantized by CUDA cores into shared memory: w = fp16(d * kv) (the
// product of an fp16 and a 7-bit integer is exact in f32 and rounds once to
// fp16), laid out as the MMA's K-major A operand. Activations are rounded to
// fp16 (exact for bf16 input within fp16's range) and the products
// accumulate in f32 in tensor memory.
//
// Inside each 32-element block K is permuted the same way for weights and
// activations: the nibble decoder emits elements (j, j+16, j+1, j+17, ...)
// of a 4-byte word (quant.cuh's interleaved order), so a word's 8 values are
// one 16-byte row of a core matrix without any repacking.
//
// Persistent CTAs (one per SM, 320 threads) walk work items (active slot x
// 128-row tile x pass of up to 64 pairs):
//   warp 0, lane 0 : producer -- per stage (2 blocks = K of 64), one tiled TMA
//                    copy of each view's packed indices (128 rows x 2 blocks),
//                    one bulk copy of each block's 128 scales, one tiled TMA
//                    copy of the pass's fp16 activations (64 rows x 64);
//   warp 1, lane 0 : issues the MMAs (M = 128, N = 64, K = 16; 4 per view
//                    and stage) into one of two accumulator buffers;
//   warps 2-5      : dequantize -- thread t owns weight row t of the tile;
//   warps 6-9      : epilogue -- warp w reads TMEM lanes 32*(w%4)..+31.
// Two views (gate and up) apply the activation in the epilogue and write the
// down projection's fp16 activations directly. Every mbarrier wait is
// bounded (the library's wait limit); a wait that gives up sets a bit of the
// device status word and the CTA stops issuing work.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "msb_internal.h"
#include "pool.cuh"
#include "quant.cuh"
#include "sm100.cuh"

namespace msb {
namespace f16 {

constexpr int kPairs = 64;         // (token, k) pairs per pass = MMA N
constexpr int kBlocks = 2;         // 32-element blocks per stage (K = 64)
constexpr int kThreads = 320;      // producer, MMA, 4 dequant, 4 epilogue warps
constexpr int kMaxActive = 1024;   // slots (with the zero slot) one launch can walk

template <int NV>
struct Cfg {
  static constexpr int kStages = NV == 2 ? 4 : 6;
  static constexpr int kQ = NV * kBlocks * 2048;            // indices, [view][block][row][16 B]
  static constexpr int kS = NV * kBlocks * 256;             // scales, [view][block][row] fp16
  static constexpr int kA = NV * kBlocks * 4 * 128 * 16;    // f16 weights, [view][kcol][row][16 B]
  static constexpr int kB = kBlocks * 4 * kPairs * 16;      // f16 activations, [kcol][pair][16 B]
  static constexpr int kStage = kQ + kS + kA + kB;
  static constexpr int kBarOff = kStages * kStage;
  static constexpr int kItemOff = kBarOff + 256;
  static constexpr int kSmem = kItemOff + (kMaxActive + 1) * 4;
  static constexpr int kAccCols = NV * kPairs;
  static constexpr int kTmemCols = 2 * kAccCols <= 128 ? 128 : 256;
  static_assert(2 * kAccCols <= kTmemCols, "double-buffered accumulators");
  static_assert(kSmem + 1024 <= 228 * 1024, "shared memory per SM");
  static_assert(kStage % 128 == 0, "TMA destinations stay 128-byte aligned");
};

struct Args {
  CUtensorMap tm_w[2];       // each view's indices: (8 B x 2 x rows, blocks, slots), box 2 blocks
  CUtensorMap tm_x;          // activations: (8 B x 2 x pairs, kcols, 1), box 64 pairs x 8 kcols
  const uint8_t *pool[2];    // slot 0 of each view's pool
  int64_t slot_stride[2], N[2];
  int64_t nb;                // blocks per row (K / 32)
  int64_t row0[2];           // first row of each view (multiple of 128)
  int64_t n_out;             // rows per view
  int tiles;
  const int32_t *counts, *offsets, *rows, *active;
  int32_t zero_slot;
  int64_t a_rows;            // rows of the activation buffers (= pairs)
  RowTarget out;             // one view: result row of each pair
  __half *xo;                // two views: the down projection's f16 activations
  float *act;                // two views, optional: f32 activation rows
  FfnAct fa;
  FfnBias bias;
  Combine comb;
  long long wait_ns;
};

constexpr int kStatusProducer = 1, kStatusAccEmpty = 2, kStatusFull = 4, kStatusAccFull = 8,
              kStatusDrain = 16;

// Byte offset of activation element (kcol c, row r) in a [kcols][rows][8]
// f16 buffer.
__device__ __forceinline__ int64_t x_off(int64_t c, int64_t rows, int64_t r) {
  return (c * rows + r) * 16;
}

// Position of row n's value in the permuted f16 activation layout: kcol and
// element within it.
__device__ __forceinline__ void perm_pos(int64_t n, int64_t &kcol, int &e) {
  const int p = interleaved_pos(int(n & 31));
  kcol = (n >> 5) * 4 + (p >> 3);
  e = p & 7;
}

// The pairs' activations in grouped order, rounded to f16 and permuted:
// xo[kcol][pos][8] for kcol = block * 4 + word. One thread per (pos, kcol).
template <typename T>
__global__ void __launch_bounds__(256) act_f16_kernel(const char *b, int64_t nb1, int64_t nb2,
                                                      int32_t ne1, int32_t top_k,
                                                      const int32_t *rows, int64_t n_pairs,
                                                      int64_t kcols, __half *xo, uint32_t *zero,
                                                      int64_t zero_n) {
  pdl_wait();
  pdl_trigger();
  grid_zero(zero, zero_n);
  const int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= n_pairs * kcols) return;
  const int64_t c = i / n_pairs, pos = i - c * n_pairs;
  const int64_t pair = rows[pos];
  const int64_t tok = pair / top_k, k1 = (pair % top_k) % ne1;
  const T *x = reinterpret_cast<const T *>(b + tok * nb2 + k1 * nb1) + (c >> 2) * 32;
  const int w = int(c & 3);
  __align__(16) __half v[8];
#pragma unroll
  for (int p = 0; p < 8; ++p) {
    const int j = 4 * w + (p >> 1) + 16 * (p & 1);
    float f;
    if constexpr (sizeof(T) == 4) f = float(x[j]);
    else f = __bfloat162float(x[j]);
    v[p] = __float2half_rn(f);
  }
  *reinterpret_cast<uint4 *>(reinterpret_cast<uint8_t *>(xo) + x_off(c, n_pairs, pos)) =
      *reinterpret_cast<const uint4 *>(v);
}

struct Item {
  int slot, pass;
  int64_t n0;
};
__device__ __forceinline__ Item locate(const Args &a, const int *item0, int64_t w, int &cur) {
  while (item0[cur + 1] <= w) ++cur;
  const int slot = a.active[1 + cur];
  const int64_t local = w - item0[cur];
  const int64_t passes = (item0[cur + 1] - item0[cur]) / a.tiles;
  return Item{slot, int(local % passes), (local / passes) * 128};
}

__device__ __forceinline__ __half2 u32_as_h2(uint32_t v) {
  __half2 h;
  memcpy(&h, &v, 4);
  return h;
}
__device__ __forceinline__ uint32_t h2_as_u32(__half2 h) {
  uint32_t v;
  memcpy(&v, &h, 4);
  return v;
}

template <int NV>
__global__ void __launch_bounds__(kThreads, 1) f16_kernel(const __grid_constant__ Args a,
                                                         int *status) {
  using C = Cfg<NV>;
  constexpr int kStages = C::kStages;
  extern __shared__ __align__(1024) uint8_t smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t n_stages_item = (a.nb + kBlocks - 1) / kBlocks;

  uint64_t *full = reinterpret_cast<uint64_t *>(smem + C::kBarOff);
  uint64_t *dq = full + kStages;          // dequant warps -> MMA
  uint64_t *empty = dq + kStages;         // MMA -> producer
  uint64_t *acc_full = empty + kStages;   // [2]
  uint64_t *acc_empty = acc_full + 2;     // [2]
  uint64_t *drained = acc_empty + 2;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(drained + 1);
  int *abort_flag = reinterpret_cast<int *>(tmem_slot + 1);
  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      sm100::mbar_init(&full[s], 1);
      sm100::mbar_init(&dq[s], 4);
      sm100::mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      sm100::mbar_init(&acc_full[b], 1);
      sm100::mbar_init(&acc_empty[b], 4);
    }
    sm100::mbar_init(drained, 1);
    *abort_flag = 0;
    sm100::fence_mbar_init();
  }
  if (warp == 0) {
    sm100::tmem_alloc(tmem_slot, C::kTmemCols);
    sm100::tmem_relinquish();
  }
  sm100::tc_fence_before();
  __syncthreads();
  sm100::tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  volatile int *abort_v = abort_flag;
  pdl_wait();
  pdl_trigger();
  int *item0 = reinterpret_cast<int *>(smem + C::kItemOff);
  const int n_active = a.active[0];
  for (int i = threadIdx.x; i < n_active; i += kThreads) {
    const int slot = a.active[1 + i];
    const int passes = slot == a.zero_slot ? 1 : (a.counts[slot] + kPairs - 1) / kPairs;
    item0[i + 1] = passes * a.tiles;
  }
  __syncthreads();
  if (warp == 0) {
    int carry = 0;
    if (lane == 0) item0[0] = 0;
    for (int b = 0; b < n_active; b += 32) {
      int v = b + lane < n_active ? item0[b + lane + 1] : 0;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, v, o);
        if (lane >= o) v += y;
      }
      if (b + lane < n_active) item0[b + lane + 1] = carry + v;
      carry += __shfl_sync(0xffffffffu, v, 31);
    }
  }
  __syncthreads();
  const int64_t n_items = item0[n_active];

  if (warp == 0) {
    // ---- producer ----
    if (lane == 0) {
      uint32_t it = 0;
      int cur = 0;
      for (int64_t w = blockIdx.x; w < n_items && !*abort_v; w += gridDim.x) {
        const Item item = locate(a, item0, w, cur);
        if (item.slot == a.zero_slot) continue;
        const int pos = int(a.offsets[item.slot] + int64_t(item.pass) * kPairs);
        for (int64_t i = 0; i < n_stages_item; ++i, ++it) {
          const int s = it % kStages;
          if (!sm100::mbar_wait_bounded(&empty[s], ((it / kStages) & 1) ^ 1, a.wait_ns)) {
            atomicOr(status, kStatusProducer);
            *abort_v = 1;
            break;
          }
          uint8_t *st = smem + s * C::kStage;
          uint8_t *sQ = st, *sS = st + C::kQ, *sB = sS + C::kS + C::kA;
          const int64_t b0 = i * kBlocks;
          sm100::mbar_expect_tx(&full[s], uint32_t(C::kQ + C::kS + C::kB));
          for (int v = 0; v < NV; ++v) {
            const int64_t r0 = a.row0[v] + item.n0;
            sm100::tma_3d(sQ + v * kBlocks * 2048, &a.tm_w[v], int(r0) * 2, int(b0), item.slot,
                          &full[s]);
            const uint8_t *sc = a.pool[v] + int64_t(item.slot) * a.slot_stride[v] +
                                a.nb * a.N[v] * 16;
            for (int bb = 0; bb < kBlocks; ++bb) {
              // Blocks past the row end: any in-bounds scales (their indices
              // arrive as zeros).
              const int64_t blk = b0 + bb < a.nb ? b0 + bb : a.nb - 1;
              sm100::bulk_g2s(sS + (v * kBlocks + bb) * 256, sc + (blk * a.N[v] + r0) * 2, 256,
                              &full[s]);
            }
          }
          sm100::tma_3d(sB, &a.tm_x, pos * 2, int(b0 * 4), 0, &full[s]);
        }
      }
      for (uint32_t k = it > uint32_t(kStages) ? it - kStages : 0; k < it; ++k)
        if (!sm100::mbar_wait_bounded(&full[k % kStages], (k / kStages) & 1, a.wait_ns))
          atomicOr(status, kStatusDrain);
    }
  } else if (warp == 1) {
    // ---- MMA issue ----
    if (lane == 0) {
      uint32_t it = 0, acc = 0;
      int cur = 0;
      for (int64_t w = blockIdx.x; w < n_items && !*abort_v; w += gridDim.x) {
        const Item item = locate(a, item0, w, cur);
        if (item.slot == a.zero_slot) continue;
        const int buf = acc & 1;
        if (!sm100::mbar_wait_bounded(&acc_empty[buf], ((acc >> 1) & 1) ^ 1, a.wait_ns)) {
          atomicOr(status, kStatusAccEmpty);
          *abort_v = 1;
          break;
        }
        sm100::tc_fence_after();
        for (int64_t i = 0; i < n_stages_item; ++i, ++it) {
          const int s = it % kStages;
          // The stage's copies (the activations are read straight from
          // shared memory) and the dequantized weights.
          if (!sm100::mbar_wait_bounded(&full[s], (it / kStages) & 1, a.wait_ns) ||
              !sm100::mbar_wait_bounded(&dq[s], (it / kStages) & 1, a.wait_ns)) {
            atomicOr(status, kStatusFull);
            *abort_v = 1;
            break;
          }
          sm100::tc_fence_after();
          const uint8_t *st = smem + s * C::kStage;
          const uint8_t *sA = st + C::kQ + C::kS, *sB = sA + C::kA;
          const int kk = int(a.nb - i * kBlocks < kBlocks ? a.nb - i * kBlocks : kBlocks);
          for (int v = 0; v < NV; ++v) {
            const uint32_t d = tmem + buf * C::kAccCols + v * kPairs;
            for (int k16 = 0; k16 < 2 * kk; ++k16) {
              // K = 16 per MMA: two 16-byte core columns (LBO apart), 8-row
              // groups 128 B apart.
              const uint64_t adesc = sm100::smem_desc(
                  sm100::smem_u32(sA + (v * kBlocks * 4 + 2 * k16) * 128 * 16), 128 * 16, 128);
              const uint64_t bdesc = sm100::smem_desc(
                  sm100::smem_u32(sB + 2 * k16 * kPairs * 16), kPairs * 16, 128);
              sm100::mma_f16(d, adesc, bdesc, sm100::idesc_f16(kPairs),
                             (i == 0 && k16 == 0) ? 0u : 1u);
            }
          }
          sm100::tc_commit(&empty[s]);
        }
        sm100::tc_commit(&acc_full[buf]);
        ++acc;
      }
      sm100::tc_commit(drained);
      if (!sm100::mbar_wait_bounded(drained, 0, a.wait_ns)) atomicOr(status, kStatusDrain);
    }
  } else if (warp <= 5) {
    // ---- dequantize: thread t owns row t of the tile ----
    const int r = threadIdx.x - 64;
    const Codebook cb = {0x3F2D1801u, 0x766A5D4Fu, 0xA6998D81u, 0xF1D9C5B5u};  // kvalues + 128
    const __half2 off = __float2half2_rn(1152.f);   // 1024 (the 0x64 exponent) + 128
    uint32_t it = 0;
    int cur = 0;
    for (int64_t w = blockIdx.x; w < n_items && !__shfl_sync(0xffffffffu, *abort_v, 0);
         w += gridDim.x) {
      const Item item = locate(a, item0, w, cur);
      if (item.slot == a.zero_slot) continue;
      bool ok = true;
      for (int64_t i = 0; i < n_stages_item; ++i, ++it) {
        const int s = it % kStages;
        if (!__all_sync(0xffffffffu,
                        sm100::mbar_wait_bounded(&full[s], (it / kStages) & 1, a.wait_ns))) {
          if (lane == 0) {
            atomicOr(status, kStatusFull);
            *abort_v = 1;
          }
          ok = false;
          break;
        }
        uint8_t *st = smem + s * C::kStage;
        const uint8_t *sQ = st, *sS = st + C::kQ;
        uint8_t *sA = st + C::kQ + C::kS;
#pragma unroll
        for (int v = 0; v < NV; ++v) {
#pragma unroll
          for (int bb = 0; bb < kBlocks; ++bb) {
            const uint4 q = *reinterpret_cast<const uint4 *>(sQ + ((v * kBlocks + bb) * 128 + r) * 16);
            const __half d = reinterpret_cast<const __half *>(sS + (v * kBlocks + bb) * 256)[r];
            const __half2 d2 = __half2half2(d);
            const uint32_t words[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
            for (int wd = 0; wd < 4; ++wd) {
              uint32_t lo, hi;
              decode_nibbles(words[wd], cb, lo, hi);
              uint4 o;
              o.x = h2_as_u32(__hmul2(__hsub2(u32_as_h2(__byte_perm(lo, 0x64646464u, 0x4140)), off), d2));
              o.y = h2_as_u32(__hmul2(__hsub2(u32_as_h2(__byte_perm(lo, 0x64646464u, 0x4342)), off), d2));
              o.z = h2_as_u32(__hmul2(__hsub2(u32_as_h2(__byte_perm(hi, 0x64646464u, 0x4140)), off), d2));
              o.w = h2_as_u32(__hmul2(__hsub2(u32_as_h2(__byte_perm(hi, 0x64646464u, 0x4342)), off), d2));
              *reinterpret_cast<uint4 *>(sA + (((v * kBlocks + bb) * 4 + wd) * 128 + r) * 16) = o;
            }
          }
        }
        sm100::fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0)
          asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(sm100::smem_u32(&dq[s]))
                       : "memory");
      }
      if (!ok) break;
    }
  } else {
    // ---- epilogue (warps 6-9) ----
    const int quad = warp & 3;
    const uint32_t lane_addr = uint32_t(quad * 32) << 16;
    uint32_t acc = 0;
    int cur = 0;
    for (int64_t w = blockIdx.x; w < n_items && !*abort_v; w += gridDim.x) {
      const Item item = locate(a, item0, w, cur);
      const int slot = item.slot;
      const int64_t n = item.n0 + quad * 32 + lane;
      const bool valid = n < a.n_out;
      const int64_t blk = (item.n0 >> 5) + quad;
      const int c_total = a.counts[slot];
      const int64_t pos0 = a.offsets[slot];
      int64_t kcol = 0;
      int e = 0;
      perm_pos(n, kcol, e);
      if (slot == a.zero_slot) {
        // Every weight of the zero slot is 0: the result is exactly 0.
        for (int j = 0; j < c_total; ++j) {
          const int64_t pair = a.rows[pos0 + j];
          if constexpr (NV == 1) {
            if (valid && !a.out.skip_zero) out_row(a.out, pair)[n] = 0.f;
          } else {
            if (a.act && valid) a.act[pair * a.n_out + n] = 0.f;
            if (valid)
              *reinterpret_cast<__half *>(reinterpret_cast<uint8_t *>(a.xo) +
                                          x_off(kcol, a.a_rows, pos0 + j) + e * 2) = __float2half(0.f);
          }
        }
        if constexpr (NV == 1) {
          for (int j0 = 0; j0 < c_total; j0 += 32) {
            const int m = min(32, c_total - j0);
            combine_arrive(a.comb, lane < m ? a.rows[pos0 + j0 + lane] : 0, m, blk, lane);
          }
        }
        continue;
      }
      const uint32_t a_i = acc++;
      const int buf = a_i & 1;
      if (!sm100::mbar_wait_bounded(&acc_full[buf], (a_i >> 1) & 1, a.wait_ns)) {
        atomicOr(status, kStatusAccFull);
        *abort_v = 1;
        break;
      }
      sm100::tc_fence_after();
      const int g0 = item.pass * kPairs;
      const int cc = min(kPairs, c_total - g0);
      const int64_t pos = pos0 + g0;
      const uint32_t col = tmem + lane_addr + buf * C::kAccCols;
      const int n_groups = (cc + 31) / 32;
      for (int gq = 0; gq < n_groups; ++gq) {
        uint32_t dg[32], du[32];
        sm100::tmem_ld_32cols(col + gq * 32, dg);
        if constexpr (NV == 2) sm100::tmem_ld_32cols(col + kPairs + gq * 32, du);
        sm100::tmem_ld_wait();
        if (gq == n_groups - 1) {
          sm100::tc_fence_before();
          __syncwarp();
          if (lane == 0)
            asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(
                             sm100::smem_u32(&acc_empty[buf]))
                         : "memory");
        }
        const int gcc = min(32, cc - gq * 32);
        const int64_t my_pair = lane < gcc ? a.rows[pos + gq * 32 + lane] : 0;
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          if (j >= gcc) break;
          const int64_t pair = __shfl_sync(0xffffffffu, my_pair, j);
          float g = __uint_as_float(dg[j]);
          if constexpr (NV == 1) {
            if (valid) {
              if (const float *br = bias_row(a.bias, 0, pair)) g += br[n];
              out_row(a.out, pair)[n] = g;
            }
          } else {
            float u = __uint_as_float(du[j]);
            if (valid) {
              if (const float *br = bias_row(a.bias, 0, pair)) g += br[n];
              if (const float *br = bias_row(a.bias, 1, pair)) u += br[n];
            }
            const float h = valid ? ffn_act(a.fa, g, u) : 0.f;
            if (a.act && valid) a.act[pair * a.n_out + n] = h;
            if (valid)
              *reinterpret_cast<__half *>(reinterpret_cast<uint8_t *>(a.xo) +
                                          x_off(kcol, a.a_rows, pos + gq * 32 + j) + e * 2) =
                  __float2half_rn(h);
          }
        }
        if constexpr (NV == 1)
          combine_arrive(a.comb, my_pair, gcc, blk, lane);
      }
    }
  }

  sm100::tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    sm100::tc_fence_after();
    sm100::tmem_dealloc(tmem, C::kTmemCols);
  }
}

}  // namespace f16

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
// Bytes of the f16 activation buffer of `rows` pairs over K inputs.
int64_t f16_act_bytes(int64_t K, int64_t rows) { return K * rows * 2; }

// Whether an IQ4_NL pool's shapes suit the f16 tensor-core path: K a
// multiple of 64 (whole stages) and rows a multiple of 8 (16-byte aligned
// scale rows).
int f16_supported(const msb_pool_s *p) {
  return p->wtype == MSB_TYPE_IQ4_NL && p->nb % 2 == 0 && p->N % 8 == 0;
}

int f16_act(const void *b, int b_type, int64_t ne1, int64_t nb1, int64_t nb2, int32_t top_k,
            const int32_t *rows, int64_t n_pairs, int64_t K, void *xo, cudaStream_t st,
            uint32_t *zero, int64_t zero_n) {
  if (n_pairs == 0) return MSB_OK;
  const int64_t kcols = K / 8;
  const int64_t grid = (n_pairs * kcols + 255) / 256;
  const char *p = static_cast<const char *>(b);
  __half *o = static_cast<__half *>(xo);
  if (b_type == MSB_TYPE_F32)
    MSB_CUDA_TRY(launch_pdl(f16::act_f16_kernel<float>, dim3(unsigned(grid)), dim3(256), 0, st, p,
                            nb1, nb2, int32_t(ne1), top_k, rows, n_pairs, kcols, o, zero, zero_n));
  else if (b_type == MSB_TYPE_BF16)
    MSB_CUDA_TRY(launch_pdl(f16::act_f16_kernel<__nv_bfloat16>, dim3(unsigned(grid)), dim3(256), 0,
                            st, p, nb1, nb2, int32_t(ne1), top_k, rows, n_pairs, kcols, o, zero,
                            zero_n));
  else
    return fail(MSB_ERR_INVALID, "activation type %d is not F32 or BF16", b_type);
  count_launch();
  MSB_CUDA_TRY(cudaGetLastError());
  return MSB_OK;
}

template <int NV>
static int launch_f16_t(const f16::Args &a, int max_active, int64_t n_pairs, cudaStream_t st) {
  using C = f16::Cfg<NV>;
  MSB_CUDA_TRY(cudaFuncSetAttribute(f16::f16_kernel<NV>,
                                    cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmem));
  static int n_sm = 0;
  if (!n_sm) {
    int dev = 0;
    MSB_CUDA_TRY(cudaGetDevice(&dev));
    MSB_CUDA_TRY(cudaDeviceGetAttribute(&n_sm, cudaDevAttrMultiProcessorCount, dev));
  }
  const int64_t passes = int64_t(max_active) + n_pairs / f16::kPairs + 1;
  int64_t grid = passes * a.tiles;
  if (grid > n_sm) grid = n_sm;
  if (grid == 0) return MSB_OK;
  int *status = nullptr;
  if (int rc = status_word(&status)) return rc;
  MSB_CUDA_TRY(launch_pdl(f16::f16_kernel<NV>, dim3(unsigned(grid)), dim3(f16::kThreads), C::kSmem,
                          st, a, status));
  count_launch();
  MSB_CUDA_TRY(cudaGetLastError());
  return MSB_OK;
}

// One IQ4_NL projection over rows [row0[v], row0[v] + n_out) of each view's
// pool (nv == 2: gate and up, writing the down projection's f16 activations
// to x_out; nv == 1: result rows).
int f16_projection(const msb_pool_s *const *pools, int nv, const int64_t *row0, int64_t n_out,
                   const msb_route_t *route, int64_t n_pairs, const void *x_in, float *res,
                   void *x_out, float *act_f32, int max_active, cudaStream_t st,
                   const RowTarget *res_rows, const FfnAct *fa, const FfnBias *bias,
                   const Combine *comb) {
  const msb_pool_s *pool = pools[0];
  f16::Args a{};
  for (int v = 0; v < 2; ++v) {
    const msb_pool_s *p = pools[nv == 2 ? v : 0];
    const int64_t r0 = nv == 2 ? row0[v] : row0[0];
    if (r0 % 128) return fail(MSB_ERR_UNSUPPORTED, "IQ4_NL tensor cores: view row %lld", (long long)r0);
    const uint64_t dims[3] = {uint64_t(p->N) * 2, uint64_t(p->nb), uint64_t(p->n_slot) + 1};
    const uint64_t strides[2] = {uint64_t(p->N) * 16, uint64_t(p->slot_stride)};
    const uint32_t box[3] = {256, uint32_t(f16::kBlocks), 1};
    if (!encode_tmap_u64_3d(&a.tm_w[v], p->data, dims, strides, box))
      return fail(MSB_ERR_CUDA, "IQ4_NL tensor cores: weight tensor map could not be encoded");
    a.pool[v] = p->data;
    a.slot_stride[v] = p->slot_stride;
    a.N[v] = p->N;
    a.row0[v] = r0;
  }
  if (pool->n_slot + 1 > f16::kMaxActive)
    return fail(MSB_ERR_UNSUPPORTED, "IQ4_NL tensor cores: %d slots exceed %d", pool->n_slot,
                f16::kMaxActive - 1);
  a.nb = pool->nb;
  a.n_out = n_out;
  a.tiles = int((n_out + 127) / 128);
  a.counts = route->counts;
  a.offsets = route->offsets;
  a.rows = route->rows;
  a.active = route->active;
  a.zero_slot = pool->n_slot;
  a.a_rows = n_pairs;
  if (res_rows) {
    a.out = *res_rows;
  } else {
    a.out.blk[0] = res;
    a.out.cap = n_pairs > 0 ? int32_t(n_pairs) : 1;
    a.out.ld = n_out;
  }
  a.xo = static_cast<__half *>(x_out);
  a.act = act_f32;
  a.fa = fa ? *fa : FfnAct{};
  if (bias) a.bias = *bias;
  if (comb) a.comb = *comb;
  a.wait_ns = wait_limit_ns();
  {
    // Activations [kcols][pairs][16 B] as 8-byte elements: a box of the
    // pass's 64 pairs x 8 kcols (one stage's K of 64) lands as
    // [kcol][pair][16 B], the K-major B operand.
    const uint64_t kcols = uint64_t(pool->K / 8);
    const uint64_t dims[3] = {uint64_t(n_pairs) * 2, kcols, 1};
    const uint64_t strides[2] = {uint64_t(n_pairs) * 16, uint64_t(n_pairs) * 16 * kcols};
    const uint32_t box[3] = {uint32_t(f16::kPairs * 2), uint32_t(f16::kBlocks * 4), 1};
    if (!encode_tmap_u64_3d(&a.tm_x, x_in, dims, strides, box))
      return fail(MSB_ERR_CUDA, "IQ4_NL tensor cores: activation tensor map could not be encoded");
  }
  return nv == 2 ? launch_f16_t<2>(a, max_active, n_pairs, st)
                 : launch_f16_t<1>(a, max_active, n_pairs, st);
}

}  // namespace msb
