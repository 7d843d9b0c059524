// Tensor-core mul_mat_id for MXFP4 slot pools (tcgen05, kind::mxf4).
//
// Weights are consumed as stored: e2m1 nibbles with one e8m0 scale per 32
// elements are exactly the tensor core's block-scaled FP4 format, so no
// weight is decoded by the CUDA cores. ggml's nibble order (byte j = elements
// j and j+16) is a fixed permutation of K inside each 32-element block; the
// activations are written with the same permutation, so every product pairs
// the right elements and the block scales line up.
//
// Activations are split into kTerms e2m1 terms per 32-element block, each
// with its own power-of-two scale (a residual expansion: term t encodes what
// terms 0..t-1 left over). Four terms are ~30x closer to exact than ggml's
// int8 (q8_0) activations. The terms of a pass's 8 pairs are stacked along
// the MMA's N (row 4p + t of B is term t of pair p, each row with its own
// block scales), so one M=128 N=32 K=64 MMA reads each weight tile from
// shared memory once for all four terms; the epilogue adds the four f32
// partial sums of a pair.
//
// Persistent CTAs walk the work items (active slot x 128-row tile x pass)
// with a stride of the grid; a pass is 8 of the slot's (token, k) pairs
// (narrow: two CTAs per SM, 256 threads) or 24 (wide, prompt-sized batches:
// one CTA per SM, 512 threads). The pipeline never drains between items:
// the producer streams the next item's tiles while the accumulators of the
// previous one are read out. Roles:
//   warp 0, lane 0 : producer -- per stage (4 or 8 blocks of K), one tiled
//                    TMA copy per weight view (128 rows x the stage's
//                    blocks), one bulk copy per view of the stage's scale
//                    records (a tile's chunks are contiguous in the pool),
//                    and one tiled TMA copy of the pass's activation lines
//                    (per chunk: 4 blocks of terms, then the scale records),
//                    into a shared-memory ring;
//   warps 1-2, lane 0 : copy each chunk's scale factors into tensor memory
//                    (tcgen05.cp) and issue the MMAs (one per K=64 step)
//                    into one of two accumulator buffers -- with two views
//                    each takes one view, with one view they take the chunks
//                    in turn (each warp its own stage ring), each into its
//                    own accumulator;
//                    tcgen05.commit frees the stage / hands over a buffer;
//   warps 4-7      : epilogue -- warp w reads TMEM lanes 32*(w%4)..+31
//                    (rows), releases the buffer, then stores (wide passes:
//                    warps 4-15, three sets of four, one 8-pair group each).
// With two views (gate and up) the epilogue applies SwiGLU and writes the
// down projection's activation terms directly.
// Batches of up to 8 pairs leave most CTAs without an item, so there a work
// item is also one of up to 4 segments of the K chunks: the epilogue stores
// f32 partial sums and counts its segment in; the warp that completes a
// 32-row block's count adds the segments in order and runs the epilogue
// (every CTA derives the same split from the route).
// Every mbarrier wait is bounded (the library's wait limit, one second by
// default); a wait that gives up sets
// a bit of the device status word (msb_device_status) and the CTA stops
// issuing work, waits (bounded) for its copies and MMAs in flight and
// releases its tensor memory.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdio>
#include <mutex>

#include "msb_internal.h"
#include "pool.cuh"
#include "quant.cuh"
#include "sm100.cuh"

namespace msb {
namespace tc {

constexpr int kTerms = 4;        // e2m1 terms per activation block
constexpr int kMaxActive = 1024; // slots (with the zero slot) one launch can walk

// Shapes of one launch with NV weight views (2: gate and up); a work item
// is one pass of up to kPairs pairs over one 128-row weight tile.
//   narrow (W false): 8 pairs per pass (MMA N = 32), two CTAs per SM with
//     256 tensor-memory columns each -- decode batches, where a slot has a
//     few pairs and many CTAs streaming different tiles keep HBM busy;
//   wide (W true): 24 pairs per pass (N = 96), one CTA per SM with all 512
//     columns (two accumulator buffers of 2 x 96 columns plus each stage's
//     scale factors) -- prompt-sized batches, where a tile's weights are
//     streamed once per pass and 3x fewer passes mean 3x fewer re-reads.
//     Three sets of 4 epilogue warps take the pass's three 8-pair groups
//     (one each): a pass's epilogue costs about as much per group as the
//     MMAs of the whole pass, so one set would leave the MMAs waiting.
// (Feeding four narrow passes' accumulators from one staged tile -- one CTA
// per SM, single-buffered tensor memory -- ran a 2048-token layer 1.4x
// slower: the four passes' epilogue serialized with the MMAs.)
template <int NV, bool W>
struct Cfg {
  static constexpr int kPairs = W ? 24 : 8;              // (token, k) pairs per pass
  static constexpr int kN = kTerms * kPairs;             // MMA N: the pass's terms stacked
  static constexpr int kCtasPerSm = W ? 1 : 2;
  // Epilogue warp sets (4 warps each, one per TMEM lane quadrant); set s
  // takes the pass's 8-pair groups s, s + kEpiSets, ...
  static constexpr int kEpiSets = W ? 3 : 1;
  // Warp 0 producer, warps 1-2 MMA issue (warp 3 idle), then the epilogue sets.
  static constexpr int kThreads = 128 + 128 * kEpiSets;
  // MMA-issuing warps: one per view (gate and up), or two taking turns
  // over the chunks of a single view. One accumulator buffer holds one
  // N = kN accumulator per MMA warp.
  static constexpr int kMma = 2;
  // Stage rings. With two views every MMA warp consumes every stage: one
  // ring. With one view each MMA warp owns a ring of kStages / kMma stages
  // (stages m * kRing ..), filled with its chunks in order, so that each
  // warp waits on every phase of the stages it reads. (A parity wait on a
  // barrier two phases behind -- a stage whose previous copy, for another
  // warp, has not landed -- would report the older phase as complete.)
  static constexpr int kRings = NV == 2 ? 1 : kMma;
  // K blocks per stage: 4 (two K=64 MMAs per view) for narrow two-view
  // passes, else 8. A stage costs its copy instructions more than its bytes
  // (each tiled or bulk copy occupies the SM's copy engine for a few hundred
  // cycles), so wide passes and one-view launches move twice the bytes per
  // instruction. (A narrow two-view stage of 8 blocks would take ~40 KB:
  // two stages per CTA at two CTAs per SM.)
  static constexpr int kCh = (W || NV == 1) ? 8 : 4;
  static constexpr int kSfc = kCh / 4;                   // 4-block scale chunks per stage
  static constexpr int kStages = W ? (NV == 2 ? 4 : 6) : (NV == 2 ? 5 : 4);
  static constexpr int kRing = kStages / kRings;
  static_assert(kStages % kRings == 0, "whole rings per MMA warp");
  static constexpr int kA = NV * kCh * 2048;             // 128 rows x 16 B per block
  // Scale factors of a weight view: one 512-byte record per 128-row tile and
  // chunk, a tile's chunks contiguous in the pool. View 0 starts on the tile
  // grid; view 1 of a two-view launch (the up half of a fused gate_up
  // tensor, rows from N/2) may not, so its window also takes the next
  // tile's records.
  static constexpr int kSfa0 = kSfc * 512;
  static constexpr int kSfa1 = NV == 2 ? 2 * kSfc * 512 : 0;
  static constexpr int kSFA = kSfa0 + kSfa1;
  // The pass's activation lines of the stage, [chunk][4 blocks, then the
  // scale records][pair][term] 16 B rows: kB bytes of terms and kSfbRec of
  // scale records (a chunk's 4 block scales in the first word). With 8
  // pairs a chunk's records are the MMA's 32-row scale atom as they stand;
  // with 24 each MMA warp gathers rows 32j + l into word j of atom row l
  // (kSfbAtom, per chunk, after the lines).
  static constexpr int kB = kCh * kN * 16;
  static constexpr int kSfbRec = kSfc * kN * 16;
  static constexpr int kSfbAtom = W ? 512 * kMma * kSfc : 0;
  static constexpr int kStage = kA + kSFA + kB + kSfbRec + kSfbAtom;
  static constexpr int kBarOff = kStages * kStage;
  static constexpr int kItemOff = kBarOff + 256;           // item prefix, kMaxActive + 1 ints
  // Gate/up epilogue: each epilogue warp stages the activation of one
  // 8-pair group over its 32 rows ([pair][row] f32) to re-split it with 4
  // lanes per 32-row block.
  static constexpr int kStageHOff = kItemOff + (kMaxActive + 1) * 4;
  static constexpr int kStageH = NV == 2 ? 4 * kEpiSets * 8 * 32 * 4 : 0;
  static constexpr int kSmem = kStageHOff + kStageH;
  static constexpr int kAccCols = kMma * kN;
  // TMEM columns per stage: each MMA warp's scale factors (A then B), 8
  // per chunk.
  static constexpr int kSfCols = (NV == 2 ? 16 : 8) * kSfc;
  static constexpr int kTmemCols = W ? 512 : 256;
  static constexpr int kAccBufs = 2 * kAccCols + kStages * kSfCols <= kTmemCols ? 2 : 1;
  static constexpr int kSfBase = kAccBufs * kAccCols;    // after the buffers
  static_assert(kSfBase + kStages * kSfCols <= kTmemCols, "tensor memory map");
  static_assert(kAccBufs == 2, "double-buffered accumulators");
  static_assert(kCtasPerSm * (kSmem + 1024) <= 228 * 1024, "shared memory per SM");
  static_assert(kStage % 128 == 0, "TMA destinations stay 128-byte aligned");
  static_assert(kPairs % 8 == 0 && kPairs <= 32, "passes of whole 8-pair column groups");
};

struct Args {
  CUtensorMap tm_w[2];       // each view's pool: (8 B x 2 x rows, blocks, slots)
  CUtensorMap tm_aq;         // activation terms and scales: (8 B x 8 x pairs, 5 lines, chunks)
  const uint8_t *pool[2];    // slot 0 of each view's pool
  int64_t slot_stride[2], N[2];
  int64_t nb;                // blocks per row (K / 32), same for both views
  int64_t row0[2];           // first row of each view: a multiple of 128, or of 32
                             // for view 1 of a two-view launch
  int64_t n_out;             // rows per view
  int tiles;                 // ceil(n_out / 128)
  const int32_t *counts, *offsets, *rows, *active;
  int32_t zero_slot;
  const uint8_t *aq;         // activation terms and scales (grouped pair order)
  int64_t a_rows;            // rows of the activation buffers (= pairs)
  RowTarget out;              // one view: result row of each pair
  uint8_t *oq;               // two views: terms and scales of silu(gate) * up
  int64_t o_nb;              // n_out / 32
  float *act;                // two views, optional: f32 silu(gate) * up
  FfnAct fa;                 // two views: the activation
  // Split over K for small batches (split_max > 0): a work item is also a
  // segment of the K chunks; the epilogue stores f32 partial sums
  // part[((seg * NV + view) * a_rows + position) * n_out + row] and counts
  // the segment in at split_cnt[item * 4 + 32-row block of the tile]
  // (zeroed before the launch); the warp that brings a count to the split
  // finishes those rows (sums in segment order, then the activation and
  // terms, or the result rows and the combine).
  int split_max;
  float *part;
  unsigned *split_cnt;
  long long wait_ns;         // bound of every mbarrier wait (wait_limit_ns)
  FfnBias bias;              // expert biases of each view (optional)
  Combine comb;              // one view: the fused router-weighted combine (optional)
};

// Status bits of the tensor-core kernels on this device (see
// msb_device_status): which bounded wait gave up.
__device__ int g_status;
constexpr int kStatusProducer = 1, kStatusAccEmpty = 2, kStatusFull = 4, kStatusAccFull = 8,
              kStatusDrain = 16;

// Activation-term buffers of `rows` rows (grouped pair positions) are lines
// of [r][t][16 B] records, five per chunk of 4 blocks: the chunk's four
// blocks' packed terms, then the chunk's scale records (the 4 block scales in
// the first word). The records of one pass (8 or 24 consecutive rows, all
// terms) of one line are contiguous -- the stacked B operand of one MMA
// K-half (row 4p + t) or its scale rows -- so one tiled copy moves a pass's
// blocks and scales of a stage together. Byte offset of the record of
// (term t, line, row r):
__device__ __forceinline__ int64_t act_line_off(int t, int64_t line, int64_t rows, int64_t r) {
  return ((line * rows + r) * kTerms + t) * 16;
}
// ... of block b's packed terms, and of chunk c's scale records.
__device__ __forceinline__ int64_t act_q_off(int t, int64_t b, int64_t rows, int64_t r) {
  return act_line_off(t, (b >> 2) * 5 + (b & 3), rows, r);
}
__device__ __forceinline__ int64_t act_sf_off(int t, int64_t c, int64_t rows, int64_t r) {
  return act_line_off(t, c * 5 + 4, rows, r);
}

// Splits the block held by the warp (lane j = element j) into kTerms e2m1
// terms and writes, per term, its 16 packed bytes (byte e = code(e) |
// code(e + 16) << 4) and its scale byte k + 127.
__device__ __forceinline__ void warp_e2m1_terms(float r, int lane, uint8_t *q_t0, int64_t q_step,
                                                uint8_t *sf_t0, int64_t sf_step) {
#pragma unroll
  for (int t = 0; t < kTerms; ++t) {
    float amax = fabsf(r);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    int k = -127;
    if (amax > 0.f) {
      int ex;
      const float m = frexpf(amax, &ex);
      k = m > 0.75f ? ex - 2 : ex - 3;
    }
    const bool skip = k < -126;
    int code = 0, neg = 0;
    if (!skip) {
      const float v = fabsf(r) * __int_as_float((127 - k) << 23);  // |r| / 2^k, exact
      code = (v >= 0.25f) + (v >= 0.75f) + (v >= 1.25f) + (v >= 1.75f) + (v >= 2.5f) +
             (v >= 3.5f) + (v >= 5.f);
      neg = (r < 0.f) && code > 0;
      const float mag = code < 5 ? 0.5f * code : (code == 5 ? 3.f : (code == 6 ? 4.f : 6.f));
      const float q = mag * __int_as_float((k + 127) << 23);        // exact
      r = neg ? r + q : r - q;                                      // exact (Sterbenz)
    }
    const int nib = code | (neg << 3);
    const int hi = __shfl_down_sync(0xffffffffu, nib, 16);
    if (lane < 16) q_t0[t * q_step + lane] = uint8_t(nib | (hi << 4));
    if (lane == 0) sf_t0[t * sf_step] = skip ? uint8_t(0) : uint8_t(k > 127 ? 254 : k + 127);
  }
}

// The same split with 8 lanes per block: lane l of the group holds elements
// 2l, 2l+1, 2l+16, 2l+17 (r[0..3]) and writes packed bytes 2l and 2l+1 of
// each term. All 32 lanes of the warp must call it (the amax reduction
// shuffles within each 8-lane group); `store` masks the writes.
__device__ __forceinline__ void group_e2m1_terms(float (&r)[4], int l, bool store, uint8_t *q_t0,
                                                 int64_t q_step, uint8_t *sf_t0, int64_t sf_step) {
#pragma unroll
  for (int t = 0; t < kTerms; ++t) {
    float amax = fmaxf(fmaxf(fabsf(r[0]), fabsf(r[1])), fmaxf(fabsf(r[2]), fabsf(r[3])));
#pragma unroll
    for (int o = 4; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    int k = -127;
    if (amax > 0.f) {
      int ex;
      const float m = frexpf(amax, &ex);
      k = m > 0.75f ? ex - 2 : ex - 3;
    }
    const bool skip = k < -126;
    uint32_t nib[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      int code = 0, neg = 0;
      if (!skip) {
        const float v = fabsf(r[e]) * __int_as_float((127 - k) << 23);  // exact
        code = (v >= 0.25f) + (v >= 0.75f) + (v >= 1.25f) + (v >= 1.75f) + (v >= 2.5f) +
               (v >= 3.5f) + (v >= 5.f);
        neg = (r[e] < 0.f) && code > 0;
        const float mag = code < 5 ? 0.5f * code : (code == 5 ? 3.f : (code == 6 ? 4.f : 6.f));
        const float q = mag * __int_as_float((k + 127) << 23);          // exact
        r[e] = neg ? r[e] + q : r[e] - q;                               // exact
      }
      nib[e] = uint32_t(code | (neg << 3));
    }
    if (store) {
      *reinterpret_cast<uint16_t *>(q_t0 + t * q_step + 2 * l) =
          uint16_t(nib[0] | (nib[2] << 4) | (nib[1] << 8) | (nib[3] << 12));
      if (l == 0) sf_t0[t * sf_step] = skip ? uint8_t(0) : uint8_t(k > 127 ? 254 : k + 127);
    }
  }
}

// The same split with 4 lanes per block: lane s of the group holds elements
// 4s..4s+3 and 4s+16..4s+19 (r[0..3] and r[4..7]) and writes packed bytes
// 4s..4s+3 of each term as one word. Called by the lanes of `mask`, whole
// 4-lane groups (the amax reduction shuffles within each group).
__device__ __forceinline__ void group4_e2m1_terms(float (&r)[8], int sub, unsigned mask,
                                                  uint8_t *q_t0, int64_t q_step, uint8_t *sf_t0,
                                                  int64_t sf_step) {
#pragma unroll
  for (int t = 0; t < kTerms; ++t) {
    float amax = 0.f;
#pragma unroll
    for (int e = 0; e < 8; ++e) amax = fmaxf(amax, fabsf(r[e]));
    amax = fmaxf(amax, __shfl_xor_sync(mask, amax, 1));
    amax = fmaxf(amax, __shfl_xor_sync(mask, amax, 2));
    int k = -127;
    if (amax > 0.f) {
      int ex;
      const float m = frexpf(amax, &ex);
      k = m > 0.75f ? ex - 2 : ex - 3;
    }
    const bool skip = k < -126;
    uint32_t nib[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      int code = 0, neg = 0;
      if (!skip) {
        const float v = fabsf(r[e]) * __int_as_float((127 - k) << 23);  // exact
        code = (v >= 0.25f) + (v >= 0.75f) + (v >= 1.25f) + (v >= 1.75f) + (v >= 2.5f) +
               (v >= 3.5f) + (v >= 5.f);
        neg = (r[e] < 0.f) && code > 0;
        const float mag = code < 5 ? 0.5f * code : (code == 5 ? 3.f : (code == 6 ? 4.f : 6.f));
        const float q = mag * __int_as_float((k + 127) << 23);          // exact
        r[e] = neg ? r[e] + q : r[e] - q;                               // exact
      }
      nib[e] = uint32_t(code | (neg << 3));
    }
    {
      const uint32_t w = (nib[0] | (nib[4] << 4)) | ((nib[1] | (nib[5] << 4)) << 8) |
                         ((nib[2] | (nib[6] << 4)) << 16) | ((nib[3] | (nib[7] << 4)) << 24);
      *reinterpret_cast<uint32_t *>(q_t0 + t * q_step + 4 * sub) = w;
      if (sub == 0) sf_t0[t * sf_step] = skip ? uint8_t(0) : uint8_t(k > 127 ? 254 : k + 127);
    }
  }
}

// Activations of every pair in grouped order into the line layout of
// act_line_off (per chunk of 4 blocks: the blocks' term records, then the
// chunk's scale records, block b's scale in byte b%4). One warp per (pair
// position, chunk); 8 lanes per block.
template <typename T>
__global__ void __launch_bounds__(256) act_terms_kernel(const char *b, int64_t nb1, int64_t nb2,
                                                        int32_t ne1, int32_t top_k,
                                                        const int32_t *rows, int64_t n_pairs,
                                                        int64_t nb, uint8_t *q,
                                                        uint32_t *zero, int64_t zero_n) {
  pdl_wait();
  pdl_trigger();
  grid_zero(zero, zero_n);   // the call's combine counters
  const int lane = threadIdx.x & 31, grp = lane >> 3, l = lane & 7;
  const int64_t nc = (nb + 3) / 4;
  const int64_t item = int64_t(blockIdx.x) * 8 + (threadIdx.x >> 5);
  if (item >= n_pairs * nc) return;   // whole warps only
  const int64_t pos = item / nc, blk = (item % nc) * 4 + grp;
  const bool live = blk < nb;
  const int64_t pair = rows[pos];
  const int64_t tok = pair / top_k, k1 = (pair % top_k) % ne1;
  const T *x = reinterpret_cast<const T *>(b + tok * nb2 + k1 * nb1) + (live ? blk : 0) * 32;
  float r[4];
  const int el[4] = {2 * l, 2 * l + 1, 2 * l + 16, 2 * l + 17};
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    if constexpr (sizeof(T) == 4) r[e] = live ? float(x[el[e]]) : 0.f;
    else r[e] = live ? __bfloat162float(x[el[e]]) : 0.f;
  }
  group_e2m1_terms(r, l, live, q + act_q_off(0, blk, n_pairs, pos), 16,
                   q + act_sf_off(0, blk / 4, n_pairs, pos) + (blk & 3), 16);
}

// Item w of the launch: its active-slot index (cursor, advanced
// monotonically as w grows), slot, pass and tile.
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

// Split over K: the last segment's warp of one 32-row block sums the
// segments' partial results of each of the pass's cc pairs in segment order
// and finishes the epilogue -- the activation and the down projection's
// terms (two views) or the result rows and the combine (one view). Lane =
// row n of block blk; the pairs are at grouped positions pos .. pos + cc - 1.
template <int NV>
__device__ __forceinline__ void split_finish(const Args &a, int split, int64_t pos, int cc,
                                             int64_t blk, int64_t n, int lane) {
  const bool valid = n < a.n_out;
  for (int j = 0; j < cc; ++j) {
    const int64_t p = pos + j;
    const int64_t pair = a.rows[p];
    float g = 0.f, u = 0.f;
    if (valid) {
      for (int sg = 0; sg < split; ++sg) {
        g += __ldcg(a.part + ((int64_t(sg) * NV) * a.a_rows + p) * a.n_out + n);
        if constexpr (NV == 2)
          u += __ldcg(a.part + ((int64_t(sg) * NV + 1) * a.a_rows + p) * a.n_out + n);
      }
      if (const float *br = bias_row(a.bias, 0, pair)) g += br[n];
      if constexpr (NV == 2)
        if (const float *br = bias_row(a.bias, 1, pair)) u += br[n];
    }
    if constexpr (NV == 1) {
      if (valid) out_row(a.out, pair)[n] = g;
    } else {
      const float h = valid ? ffn_act(a.fa, g, u) : 0.f;
      if (a.act && valid) a.act[pair * a.n_out + n] = h;
      if (blk < a.o_nb)
        warp_e2m1_terms(h, lane, a.oq + act_q_off(0, blk, a.a_rows, p), 16,
                        a.oq + act_sf_off(0, blk / 4, a.a_rows, p) + (blk & 3), 16);
    }
  }
  if constexpr (NV == 1) combine_arrive(a.comb, lane < cc ? a.rows[pos + lane] : 0, cc, blk, lane);
}

template <int NV, bool W>
__global__ void __launch_bounds__(Cfg<NV, W>::kThreads, W ? 1 : 2)
    tc_kernel(const __grid_constant__ Args a) {
  using C = Cfg<NV, W>;
  constexpr int kPairs = C::kPairs;
  constexpr int kN = C::kN;
  constexpr int kStages = C::kStages;
  constexpr int kBufs = C::kAccBufs;
  extern __shared__ __align__(1024) uint8_t smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t n_chunks = (a.nb + C::kCh - 1) / C::kCh;   // stages per item

  uint64_t *full = reinterpret_cast<uint64_t *>(smem + C::kBarOff);
  uint64_t *empty = full + kStages;
  uint64_t *acc_full = empty + kStages;   // [2] MMA -> epilogue
  uint64_t *acc_empty = acc_full + 2;     // [2] epilogue -> MMA
  uint64_t *drained = acc_empty + 2;      // MMA issuer's last commit
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(drained + 1);
  int *abort_flag = reinterpret_cast<int *>(tmem_slot + 1);
  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      sm100::mbar_init(&full[s], 1);
      sm100::mbar_init(&empty[s], NV == 2 ? 2 : 1);   // the stage's MMA warps
    }
    for (int b = 0; b < 2; ++b) {
      sm100::mbar_init(&acc_full[b], C::kMma);
      sm100::mbar_init(&acc_empty[b], 4 * C::kEpiSets);   // every epilogue warp
    }
    sm100::mbar_init(drained, C::kMma);
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
  // The prologue above overlaps the previous kernel; the route and the
  // activation terms are read only after it completed.
  pdl_wait();
  pdl_trigger();
  // Work items: (active slot, 128-row tile, pass of up to kPairs pairs), the
  // passes of one tile adjacent so that CTAs running them at the same time
  // share the tile's weights through L2. item0[i] = first item of active
  // slot i (the zero slot has one item per tile: its epilogue writes every
  // pair's zeros).
  int *item0 = reinterpret_cast<int *>(smem + C::kItemOff);
  const int n_active = a.active[0];
  for (int i = threadIdx.x; i < n_active; i += C::kThreads) {
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
  // Split over K (small batches): as many segments as keep every CTA busy,
  // at most split_max, each of at least one chunk per MMA warp. Every CTA
  // computes the same value from the same route.
  int split = 1;
  if (a.split_max > 0) {
    int64_t sp = n_items > 0 ? int64_t(gridDim.x) / n_items : 1;
    const int64_t by_chunks = n_chunks / (NV == 1 ? C::kMma : 1);
    if (sp > a.split_max) sp = a.split_max;
    if (sp > by_chunks) sp = by_chunks;
    split = sp < 1 ? 1 : int(sp);
  }
  const bool split_mode = split > 1;
  const int64_t n_work = n_items * split;

  if (warp == 0) {
    // ---- producer ----
    if (lane == 0) {
      uint32_t fills[C::kRings] = {};   // copies issued into each ring
      int cur = 0;
      for (int64_t w = blockIdx.x; w < n_work && !*abort_v; w += gridDim.x) {
        const int64_t wi = w / split, seg = w - wi * split;
        const Item item = locate(a, item0, wi, cur);
        const int slot = item.slot;
        if (slot == a.zero_slot) continue;
        const int pos = int(a.offsets[slot] + int64_t(item.pass) * kPairs);
        const int64_t lo = seg * n_chunks / split, hi = (seg + 1) * n_chunks / split;
        for (int64_t i = lo; i < hi; ++i) {
          // Chunk i goes to the ring of the MMA warp that reads it.
          const int ring = C::kRings == 1 ? 0 : int(i % C::kRings);
          uint32_t k = 0;   // (selects keep the counters in registers)
#pragma unroll
          for (int r = 0; r < C::kRings; ++r)
            if (r == ring) k = fills[r];
          const int s = ring * C::kRing + int(k % C::kRing);
          if (!sm100::mbar_wait_bounded(&empty[s], ((k / C::kRing) & 1) ^ 1, a.wait_ns)) {
            atomicOr(&g_status, kStatusProducer);
            *abort_v = 1;
            break;
          }
          uint8_t *st = smem + s * C::kStage;
          uint8_t *sA = st, *sSFA = st + C::kA, *sB = sSFA + C::kSFA;
          const int64_t b0 = i * C::kCh;     // first block of the stage
          const int64_t c0 = i * C::kSfc;    // its first scale chunk
          const int64_t nc = (a.nb + 3) / 4;
          const uint32_t sf_bytes = uint32_t(nc - c0 < C::kSfc ? nc - c0 : C::kSfc) * 512;
          // Full boxes are counted (rows or blocks outside the tensors
          // arrive as zeros); the scale records are copied as far as they
          // exist. A window off the tile grid (view 1 only) also takes the
          // next tile's records when the pool has one.
          bool next_sf[NV];
          uint32_t tx = uint32_t(C::kA + C::kB + C::kSfbRec);
          for (int v = 0; v < NV; ++v) {
            const int64_t r0 = a.row0[v] + item.n0;
            next_sf[v] = v == 1 && (r0 & 127) != 0 && (r0 >> 7) + 1 < (a.N[v] + 127) / 128;
            tx += next_sf[v] ? 2 * sf_bytes : sf_bytes;
          }
          sm100::mbar_expect_tx(&full[s], tx);
          for (int v = 0; v < NV; ++v) {
            const int64_t r0 = a.row0[v] + item.n0;
            sm100::tma_3d(sA + v * C::kCh * 2048, &a.tm_w[v], int(r0) * 2, int(b0), slot,
                          &full[s]);
            const uint8_t *slot_base = a.pool[v] + int64_t(slot) * a.slot_stride[v];
            const uint8_t *sf_tile = slot_base + a.nb * a.N[v] * 16 + ((r0 >> 7) * nc + c0) * 512;
            uint8_t *sfa_v = sSFA + (v == 0 ? 0 : C::kSfa0);
            sm100::bulk_g2s(sfa_v, sf_tile, sf_bytes, &full[s]);
            if (next_sf[v]) sm100::bulk_g2s(sfa_v + C::kSfc * 512, sf_tile + nc * 512, sf_bytes, &full[s]);
          }
          // The pass's activation terms and scales of the stage's chunks.
          sm100::tma_3d(sB, &a.tm_aq, pos * 8, 0, int(c0), &full[s]);
#pragma unroll
          for (int r = 0; r < C::kRings; ++r)
            if (r == ring) fills[r] = k + 1;
        }
      }
      // No copy may still be landing in shared memory when the CTA exits
      // (only possible after an abort): wait for each ring's last fills.
#pragma unroll
      for (int ring = 0; ring < C::kRings; ++ring) {
        const uint32_t n = fills[ring];
        for (uint32_t k = n > uint32_t(C::kRing) ? n - C::kRing : 0; k < n; ++k)
          if (!sm100::mbar_wait_bounded(&full[ring * C::kRing + k % C::kRing], (k / C::kRing) & 1,
                                        a.wait_ns))
            atomicOr(&g_status, kStatusDrain);
      }
    }
  } else if (warp <= 3) {
    // ---- scale-factor copies and MMA issue (warps 1-2; warp 3 idles) ----
    // One thread issuing every tcgen05 copy and MMA caps a CTA at ~26 GB/s
    // (about 0.4 us per stage), so several warps issue: with two views each
    // of warps 1-2 takes one (gate, up); with one view they take the chunks
    // in turn (chunk i to warp i % kMma, staged in that warp's ring),
    // each into its own accumulator, added by the epilogue.
    // The whole warp runs the loop (every lane waits on the barriers, so all
    // see the staged bytes); lane 0 issues the tensor-core instructions.
    const int m = warp - 1;
    if (m < C::kMma) {
      uint32_t it = 0, acc = 0;
      // Base descriptors at the shared-memory base: A (2 KB per block of
      // 128 rows), B (the pass's kN rows per block) and the 32-row scale atoms.
      const uint32_t smem_base = sm100::smem_u32(smem);
      const uint64_t desc_a = sm100::smem_desc(smem_base, 2048, 128);
      const uint64_t desc_b = sm100::smem_desc(smem_base, kN * 16, 128);
      const uint64_t desc_sf = sm100::smem_desc(smem_base, 0, 128);
      constexpr uint32_t kIdesc0 = sm100::idesc_mxf4(kN, 0, 0), kIdesc2 = sm100::idesc_mxf4(kN, 2, 2);
      int cur = 0;
      const int v = NV == 2 ? m : 0;
      // Scale rows of a view that starts `shift` 32-row groups into a tile:
      // window row 32q + l is pool tile row 32(shift + q) + l, in the next
      // tile's chunk once shift + q reaches 4.
      const int shift = NV == 2 ? int((a.row0[v] & 127) >> 5) : 0;
      for (int64_t w = blockIdx.x; w < n_work && !__shfl_sync(0xffffffffu, *abort_v, 0);
           w += gridDim.x) {
        const int64_t wi = w / split, seg = w - wi * split;
        const Item item = locate(a, item0, wi, cur);
        if (item.slot == a.zero_slot) continue;
        const int64_t lo = seg * n_chunks / split, hi = (seg + 1) * n_chunks / split;
        const int buf = acc % kBufs;
        if (!__all_sync(0xffffffffu,
                        sm100::mbar_wait_bounded(&acc_empty[buf], ((acc / kBufs) & 1) ^ 1, a.wait_ns))) {
          if (lane == 0) {
            atomicOr(&g_status, kStatusAccEmpty);
            *abort_v = 1;
          }
          break;
        }
        sm100::tc_fence_after();
        const uint32_t d0 = tmem + buf * C::kAccCols + m * kN;
        const int64_t r0 = a.row0[v] + item.n0;
        const bool has_next = (r0 >> 7) + 1 < (a.N[v] + 127) / 128;
        bool first = true;
        for (int64_t i = lo; i < hi; ++i) {
          if (NV == 1 && i % C::kMma != m) continue;   // another warp's chunk
          // This warp's ring (one view) or the shared ring (two views), in
          // the order the producer fills it.
          const uint32_t k = it++;
          const int s = (NV == 1 ? m * C::kRing : 0) + int(k % C::kRing);
          if (!__all_sync(0xffffffffu, sm100::mbar_wait_bounded(&full[s], (k / C::kRing) & 1, a.wait_ns))) {
            if (lane == 0) {
              atomicOr(&g_status, kStatusFull);
              *abort_v = 1;
            }
            break;
          }
          uint8_t *st = smem + s * C::kStage;
          uint8_t *sSFA = st + C::kA, *sB = sSFA + C::kSFA;
          uint8_t *sfa_v = sSFA + (v == 0 ? 0 : C::kSfa0);
          const int kbn = int(a.nb - i * C::kCh < C::kCh ? a.nb - i * C::kCh : C::kCh);
          const int ncs = (kbn + 3) / 4;   // scale chunks with MMAs in this stage
          for (int c = 0; c < ncs; ++c) {
            if (shift) {
              // Reassemble the window's record of chunk c in place: lane l
              // owns 16-byte row l of this tile's and the next tile's
              // records (words = 32-row groups).
              uint8_t *rec = sfa_v + c * 512;
              const uint4 q0 = *reinterpret_cast<const uint4 *>(rec + lane * 16);
              uint4 q1 = make_uint4(0u, 0u, 0u, 0u);   // rows past the pool: scale 2^-127
              if (has_next)
                q1 = *reinterpret_cast<const uint4 *>(rec + C::kSfc * 512 + lane * 16);
              const uint4 o = shift == 1   ? make_uint4(q0.y, q0.z, q0.w, q1.x)
                              : shift == 2 ? make_uint4(q0.z, q0.w, q1.x, q1.y)
                                           : make_uint4(q0.w, q1.x, q1.y, q1.z);
              *reinterpret_cast<uint4 *>(rec + lane * 16) = o;
              sm100::fence_proxy_async_smem();
            }
            if constexpr (W) {
              // Scale atom of chunk c of the pass's 96 B rows: word j of row
              // l is the record of B row 32j + l (rows 96-127 do not exist:
              // scale 0).
              const uint8_t *recs = sB + (c * 5 + 4) * (kN * 16);
              uint8_t *atom = sB + C::kB + C::kSfbRec + (m * C::kSfc + c) * 512;
              const uint4 o = make_uint4(*reinterpret_cast<const uint32_t *>(recs + lane * 16),
                                         *reinterpret_cast<const uint32_t *>(recs + (32 + lane) * 16),
                                         *reinterpret_cast<const uint32_t *>(recs + (64 + lane) * 16),
                                         0u);
              *reinterpret_cast<uint4 *>(atom + lane * 16) = o;
              sm100::fence_proxy_async_smem();
            }
          }
          __syncwarp();
          if (lane == 0) {
            // Byte offsets of the stage's operands from the shared-memory
            // base, added to the base descriptors (the address field holds
            // address / 16 in 14 bits; shared addresses stay below 2^18, so
            // the adds never carry out of it).
            const uint32_t st_off = uint32_t(s) * uint32_t(C::kStage);
            const uint32_t a_off = st_off + uint32_t(v * C::kCh * 2048);
            // B lines per chunk: 4 blocks, then the scale records.
            constexpr uint32_t kLine = uint32_t(kN * 16);
            const uint32_t b_off = st_off + uint32_t(C::kA + C::kSFA);
            const uint32_t sfa_off = st_off + uint32_t(C::kA + (v == 0 ? 0 : C::kSfa0));
            const uint32_t sfb_off = W ? b_off + uint32_t(C::kB + C::kSfbRec + m * C::kSfc * 512)
                                       : b_off + 4 * kLine;
            constexpr uint32_t kSfbStep = W ? 512u : 5 * kLine;
            const uint32_t sf0 = tmem + C::kSfBase + s * C::kSfCols + (NV == 2 ? m * 8 * C::kSfc : 0);
#pragma unroll
            for (int c = 0; c < C::kSfc; ++c) {
              if (c < ncs) {
                // Chunk c: its scale factors into tensor memory, then the
                // MMAs of its two K=64 halves (blocks 4c .. 4c + 3).
                const uint32_t sf_col = sf0 + c * 8;
                sm100::tmem_cp_32x128b_x4(sf_col, desc_sf + ((sfa_off + c * 512) >> 4));
                sm100::tmem_cp_32x128b_x4(sf_col + 4, desc_sf + ((sfb_off + c * kSfbStep) >> 4));
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                  const int j = 2 * c + h;
                  // B: the pass's stacked rows of 16 B per block; K-halves
                  // one block apart. A: 2 KB per block.
                  if (j < kbn / 2)
                    sm100::mma_mxf4(d0, desc_a + ((a_off + j * 4096) >> 4),
                                    desc_b + ((b_off + (c * 5 + 2 * h) * kLine) >> 4),
                                    h ? kIdesc2 : kIdesc0, sf_col | (h ? 2u << 30 : 0u),
                                    (sf_col + 4) | (h ? 2u << 30 : 0u),
                                    (first && j == 0) ? 0u : 1u);
                }
              }
            }
            sm100::tc_commit(&empty[s]);
          }
          __syncwarp();
          first = false;
        }
        if (lane == 0) sm100::tc_commit(&acc_full[buf]);
        ++acc;
      }
      // Every MMA and scale-factor copy is complete before tensor memory is
      // released.
      if (lane == 0) {
        sm100::tc_commit(drained);
        if (!sm100::mbar_wait_bounded(drained, 0, a.wait_ns)) atomicOr(&g_status, kStatusDrain);
      }
    }
  } else {
    // ---- epilogue (warps 4 .. 4 + 4 * kEpiSets - 1) ----
    const int quad = warp & 3;            // TMEM lane quadrant of this warp
    const int set = (warp - 4) >> 2;      // epilogue warp set
    float *sh = reinterpret_cast<float *>(smem + C::kStageHOff) + (warp - 4) * 8 * 32;
    const uint32_t lane_addr = uint32_t(quad * 32) << 16;
    uint32_t acc = 0;
    int cur = 0;
    for (int64_t w = blockIdx.x; w < n_work && !*abort_v; w += gridDim.x) {
      const int64_t wi = w / split, seg = w - wi * split;
      const Item item = locate(a, item0, wi, cur);
      const int slot = item.slot;
      const int64_t n0 = item.n0;
      const int64_t n = n0 + quad * 32 + lane;
      const bool valid = n < a.n_out;
      const int64_t blk = (n0 >> 5) + quad;   // SwiGLU output block of this warp
      const int c_total = a.counts[slot];
      const int64_t pos0 = a.offsets[slot];
      if (slot == a.zero_slot && (seg != 0 || set != 0)) continue;   // written once
      if (slot == a.zero_slot) {
        // Every weight of the zero slot is 0, so the exact result is 0; for
        // the down projection's input, 0 splits into four zero terms with
        // scale byte 0 (stored directly, 8 pairs x 4 terms per warp step).
        for (int j = 0; j < c_total; ++j) {
          const int64_t pair = a.rows[pos0 + j];
          if constexpr (NV == 1) {
            if (valid && !a.out.skip_zero) out_row(a.out, pair)[n] = 0.f;
          } else {
            if (a.act && valid) a.act[pair * a.n_out + n] = 0.f;
          }
        }
        if constexpr (NV == 1) {
          for (int j0 = 0; j0 < c_total; j0 += 32) {
            const int m = min(32, c_total - j0);
            combine_arrive(a.comb, lane < m ? a.rows[pos0 + j0 + lane] : 0, m, blk, lane);
          }
        }
        if constexpr (NV == 2) {
          if (blk < a.o_nb) {
            const int t = lane & 3;
            for (int j = lane >> 2; j < c_total; j += 8) {
              *reinterpret_cast<uint4 *>(a.oq + act_q_off(t, blk, a.a_rows, pos0 + j)) =
                  make_uint4(0u, 0u, 0u, 0u);
              a.oq[act_sf_off(t, blk / 4, a.a_rows, pos0 + j) + (blk & 3)] = 0;
            }
          }
        }
        continue;
      }
      const uint32_t a_i = acc++;
      const int buf = a_i % kBufs;
      // The pass's pairs (lane j holds the j-th), loaded while the MMAs run.
      const int g0 = item.pass * kPairs;
      const int cc = min(kPairs, c_total - g0);
      const int64_t pos = pos0 + g0;
      const int64_t my_pair = lane < cc ? a.rows[pos + lane] : 0;
      if (!sm100::mbar_wait_bounded(&acc_full[buf], (a_i / kBufs) & 1, a.wait_ns)) {
        atomicOr(&g_status, kStatusAccFull);
        *abort_v = 1;
        break;
      }
      sm100::tc_fence_after();
      {
        const uint32_t col = tmem + lane_addr + buf * C::kAccCols;
        const int n_groups = (cc + 7) / 8;   // 8-pair column groups this pass uses
        auto release = [&]() {
          // This warp's accumulators are in registers: count it out of the buffer.
          sm100::tc_fence_before();
          __syncwarp();
          if (lane == 0)
            asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(
                             sm100::smem_u32(&acc_empty[buf]))
                         : "memory");
        };
        if (set >= n_groups) release();   // no group of this pass for this set
        for (int gq = set; gq < n_groups; gq += C::kEpiSets) {
          // Group gq: columns 32 gq .. +31 of each accumulator (column
          // 4j + t of the group holds term t of the group's pair j).
          uint32_t dg[32], du[32];
          sm100::tmem_ld_32cols(col + gq * 32, dg);
          if (NV == 2 || n_chunks > 1) sm100::tmem_ld_32cols(col + kN + gq * 32, du);
          sm100::tmem_ld_wait();
          if constexpr (NV == 1) {
            // The MMA warps' accumulators (chunks i % kMma = 0, 1), added
            // in that order; a warp that had no chunk holds nothing.
            static_assert(C::kMma == 2, "one view: two accumulators");
            if (n_chunks > 1) {
#pragma unroll
              for (int c = 0; c < 32; ++c)
                dg[c] = __float_as_uint(__uint_as_float(dg[c]) + __uint_as_float(du[c]));
            }
          }
          if (gq + C::kEpiSets >= n_groups) release();   // this set's last group
          const int gcc = min(8, cc - gq * 8);
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            if (j >= gcc) break;   // same on every lane
            const int jj = gq * 8 + j;
            const int64_t pair = __shfl_sync(0xffffffffu, my_pair, jj);
            const float gv = (__uint_as_float(dg[4 * j]) + __uint_as_float(dg[4 * j + 1])) +
                             (__uint_as_float(dg[4 * j + 2]) + __uint_as_float(dg[4 * j + 3]));
            float u = 0.f;
            if constexpr (NV == 2)
              u = (__uint_as_float(du[4 * j]) + __uint_as_float(du[4 * j + 1])) +
                  (__uint_as_float(du[4 * j + 2]) + __uint_as_float(du[4 * j + 3]));
            if (split_mode) {
              // This segment's partial sums; the split reduce finishes.
              if (valid) {
                a.part[((seg * NV) * a.a_rows + pos + jj) * a.n_out + n] = gv;
                if constexpr (NV == 2)
                  a.part[((seg * NV + 1) * a.a_rows + pos + jj) * a.n_out + n] = u;
              }
              continue;
            }
            if constexpr (NV == 1) {
              if (valid) {
                const float *br = bias_row(a.bias, 0, pair);
                out_row(a.out, pair)[n] = br ? gv + br[n] : gv;
              }
            } else {
              float gb = gv, ub = u;
              if (valid) {
                if (const float *br = bias_row(a.bias, 0, pair)) gb += br[n];
                if (const float *br = bias_row(a.bias, 1, pair)) ub += br[n];
              }
              const float h = (valid) ? ffn_act(a.fa, gb, ub) : 0.f;
              if (a.act && valid) a.act[pair * a.n_out + n] = h;
              sh[j * 32 + lane] = h;
            }
          }
          if constexpr (NV == 2) {
            if (!split_mode && blk < a.o_nb) {
              // The down projection's terms of this warp's 32-row block for
              // the group's pairs: 4 lanes per pair (lane 4j + s holds
              // elements 4s..4s+3 and 4s+16..4s+19 of pair j).
              __syncwarp();
              const int j = lane >> 2, sub = lane & 3;
              if (j < gcc) {
                const unsigned mask = gcc == 8 ? 0xffffffffu : (1u << (4 * gcc)) - 1u;
                float r[8];
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                  r[e] = sh[j * 32 + 4 * sub + e];
                  r[4 + e] = sh[j * 32 + 16 + 4 * sub + e];
                }
                const int64_t p_row = pos + gq * 8 + j;
                group4_e2m1_terms(r, sub, mask, a.oq + act_q_off(0, blk, a.a_rows, p_row), 16,
                                  a.oq + act_sf_off(0, blk / 4, a.a_rows, p_row) + (blk & 3), 16);
              }
              __syncwarp();
            }
          }
          // The group's rows of this 32-row block are stored: count them.
          if constexpr (NV == 1)
            if (!split_mode)
              combine_arrive(a.comb, __shfl_sync(0xffffffffu, my_pair, (gq * 8 + lane) & 31), gcc,
                             blk, lane);
        }
        if (split_mode) {
          // This segment's partial sums of the 32-row block are stored:
          // count the segment in (the stores are fenced before the count);
          // the warp that completes the count finishes the block's rows.
          __threadfence();
          __syncwarp();
          unsigned old = 0;
          if (lane == 0) {
            old = atomicAdd(a.split_cnt + wi * 4 + quad, 1u);
            __threadfence();
          }
          old = __shfl_sync(0xffffffffu, old, 0);
          __syncwarp();
          if (old == unsigned(split - 1)) split_finish<NV>(a, split, pos, cc, blk, n, lane);
        }
      }
    }
  }

  // Teardown: every role is done issuing; release tensor memory.
  sm100::tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    sm100::tc_fence_after();
    sm100::tmem_dealloc(tmem, C::kTmemCols);
  }
  if (a.out.done && threadIdx.x == 0) {
    // This CTA's rows are stored (the barrier above); the last CTA to count
    // itself done tells the rows' owners, once per launch.
    asm volatile("fence.acq_rel.sys;" ::: "memory");
    if (atomicAdd(a.out.done, 1u) == gridDim.x - 1) {
      *a.out.done = 0;
      asm volatile("fence.acq_rel.sys;" ::: "memory");
      for (int i = 0; i < a.out.n_arrive; ++i)
        asm volatile("red.release.sys.global.add.u32 [%0], 1;" ::"l"(a.out.arrive[i])
                     : "memory");
    }
  }
}

}  // namespace tc

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
// Batches of up to kSplitPairs pairs may split K into up to kSplitMax
// segments (tc_projection). Measured on gpt-oss layers (2880 x 2880): 1
// token x top-4 gains 11 %; at 16 pairs the items alone fill the grid.
constexpr int64_t kSplitPairs = 8;
constexpr int kSplitMax = 4;

// Wide passes: 0 = by batch size (MSB_OPT_WIDE_PASSES), 1 = never, 2 = always.
static int g_wide_policy = 0;
constexpr int64_t kWidePairsPerSlot = 12;

static bool wide_passes_enabled(int64_t n_pairs, int64_t max_active) {
  if (g_wide_policy == 1) return false;
  if (g_wide_policy == 2) return true;
  return n_pairs >= kWidePairsPerSlot * max_active;
}

int set_wide_policy(int v) {
  if (v < 0 || v > 2) return fail(MSB_ERR_INVALID, "msb_set_option: wide passes must be 0, 1 or 2");
  g_wide_policy = v;
  return MSB_OK;
}

// Split scratch: the segment counters of a two-view and of a one-view
// launch (kSplitCntWords each: up to 9 active slots -- 8 pairs and the zero
// slot -- x kSplitMaxTiles tiles x 4 row blocks), then the partial sums.
// The counters must be zero when a launch starts: the activation-terms
// kernel that precedes every launch chain zeroes them
// (tc_split_zero_words).
constexpr int64_t kSplitMaxTiles = 128;
constexpr int64_t kSplitCntWords = (kSplitPairs + 1) * kSplitMaxTiles * 4;

int64_t tc_split_bytes(int64_t n_out_max, int64_t n_pairs) {
  return n_pairs > 0 && n_pairs <= kSplitPairs
             ? 2 * kSplitCntWords * 4 + 2 * kSplitMax * n_pairs * n_out_max * 4
             : 0;
}

int64_t tc_split_zero_words(int64_t n_pairs) {
  return n_pairs > 0 && n_pairs <= kSplitPairs ? 2 * kSplitCntWords : 0;
}

int64_t tc_act_bytes(int64_t nb, int64_t rows) {
  return int64_t(tc::kTerms) * 5 * ((nb + 3) / 4) * rows * 16;   // 5 lines per chunk
}

int tc_supported(const msb_pool_s *p) {
  return p->wtype == MSB_TYPE_MXFP4 && p->nb % 2 == 0;
}

int tc_act_terms(const void *b, int b_type, int64_t ne1, int64_t nb1, int64_t nb2, int32_t top_k,
                 const int32_t *rows, int64_t n_pairs, int64_t nb, uint8_t *ws, cudaStream_t st,
                 uint32_t *zero, int64_t zero_n) {
  if (n_pairs == 0) return MSB_OK;
  uint8_t *q = ws;   // terms and scales, act_q_off / act_sf_off
  const int64_t grid = (n_pairs * ((nb + 3) / 4) + 7) / 8;
  const char *p = static_cast<const char *>(b);
  if (b_type == MSB_TYPE_F32)
    MSB_CUDA_TRY(launch_pdl(tc::act_terms_kernel<float>, dim3(unsigned(grid)), dim3(256), 0, st, p,
                            nb1, nb2, int32_t(ne1), top_k, rows, n_pairs, nb, q, zero, zero_n));
  else if (b_type == MSB_TYPE_BF16)
    MSB_CUDA_TRY(launch_pdl(tc::act_terms_kernel<__nv_bfloat16>, dim3(unsigned(grid)), dim3(256), 0,
                            st, p, nb1, nb2, int32_t(ne1), top_k, rows, n_pairs, nb, q, zero,
                            zero_n));
  else
    return fail(MSB_ERR_INVALID, "activation type %d is not F32 or BF16", b_type);
  count_launch();
  MSB_CUDA_TRY(cudaGetLastError());
  return MSB_OK;
}

template <int NV, bool W>
static int launch_tc_t(const tc::Args &a, int max_active, int64_t n_pairs, cudaStream_t st) {
  using C = tc::Cfg<NV, W>;
  MSB_CUDA_TRY(cudaFuncSetAttribute(tc::tc_kernel<NV, W>,
                                    cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmem));
  // Persistent grid: as many CTAs as fit (shared and tensor memory), never
  // more than the work items the route can produce (each active slot has at
  // most ceil(pairs / kPairs) + 1 passes per tile).
  static int n_sm = 0;
  if (!n_sm) {
    int dev = 0;
    MSB_CUDA_TRY(cudaGetDevice(&dev));
    MSB_CUDA_TRY(cudaDeviceGetAttribute(&n_sm, cudaDevAttrMultiProcessorCount, dev));
  }
  const int64_t passes = int64_t(max_active) + n_pairs / C::kPairs + 1;
  int64_t grid = passes * a.tiles * (a.split_max > 0 ? a.split_max : 1);
  if (grid > int64_t(C::kCtasPerSm) * n_sm) grid = int64_t(C::kCtasPerSm) * n_sm;
  if (grid == 0) return MSB_OK;
  MSB_CUDA_TRY(launch_pdl(tc::tc_kernel<NV, W>, dim3(unsigned(grid)), dim3(C::kThreads), C::kSmem,
                          st, a));
  count_launch();
  MSB_CUDA_TRY(cudaGetLastError());
  return MSB_OK;
}

// One projection over rows [row0[v], row0[v] + n_out) of each view's pool
// (pools[1] is used only when nv == 2). act_in: the pairs' activation terms
// (tc_act_terms); nv == 2 writes the terms of silu(view 0) * view 1 to
// act_out, nv == 1 writes res.
int tc_projection(const msb_pool_s *const *pools, int nv, const int64_t *row0, int64_t n_out,
                  const msb_route_t *route, int64_t n_pairs, const uint8_t *act_in, float *res,
                  uint8_t *act_out, float *act_f32, int max_active, cudaStream_t st,
                  const RowTarget *res_rows, const FfnAct *fa, uint8_t *split_ws,
                  int64_t split_bytes, const FfnBias *bias, const Combine *comb,
                  bool allow_wide) {
  const msb_pool_s *pool = pools[0];
  if (row0[0] % 128 != 0)
    return fail(MSB_ERR_INVALID, "tensor-core path: the first view must start on a 128-row tile");
  // Split over K for small batches, where the items alone leave CTAs idle:
  // up to kSplitMax segments, as many as the caller's scratch holds.
  int64_t split_segs = 0;
  if (split_ws && n_pairs > 0 && n_pairs <= kSplitPairs && !(res_rows && res_rows->done) &&
      (n_out + 127) / 128 <= kSplitMaxTiles) {
    split_segs = (split_bytes - 2 * kSplitCntWords * 4) / (int64_t(nv) * n_pairs * n_out * 4);
    if (split_segs > kSplitMax) split_segs = kSplitMax;
    if (split_segs < 2) split_segs = 0;
  }
  // Wide passes (24 pairs, 8-block stages) for prompt-sized batches: when the
  // pairs would fill at least kWidePairsPerSlot passes-worth per possibly
  // active slot. Not with K split, nor for the expert-parallel exchange
  // (allow_wide false), whose rows are padded and few per expert.
  const bool wide = split_segs == 0 && allow_wide && !res_rows &&
                    wide_passes_enabled(n_pairs, max_active);
  tc::Args a{};
  if (bias) a.bias = *bias;
  if (comb) a.comb = *comb;
  for (int v = 0; v < 2; ++v) {
    const msb_pool_s *p = pools[nv == 2 ? v : 0];
    if (!p->has_tmap) return fail(MSB_ERR_UNSUPPORTED, "tensor-core path: pool has no tensor map");
    a.tm_w[v] = (wide || nv == 1) ? p->tmap_w8 : p->tmap_w;   // the config's kCh blocks
    a.pool[v] = p->data;
    a.slot_stride[v] = p->slot_stride;
    a.N[v] = p->N;
    a.row0[v] = nv == 2 ? row0[v] : row0[0];
  }
  a.nb = pool->nb;
  a.n_out = n_out;
  a.tiles = int((n_out + 127) / 128);
  a.counts = route->counts;
  a.offsets = route->offsets;
  a.rows = route->rows;
  a.active = route->active;
  a.zero_slot = pool->n_slot;
  a.wait_ns = wait_limit_ns();
  if (pool->n_slot + 1 > tc::kMaxActive)
    return fail(MSB_ERR_UNSUPPORTED, "tensor-core path: %d slots exceed %d", pool->n_slot,
                tc::kMaxActive - 1);
  a.aq = act_in;
  a.a_rows = n_pairs;
  if (res_rows) {
    a.out = *res_rows;
  } else {
    a.out.blk[0] = res;
    a.out.cap = n_pairs > 0 ? int32_t(n_pairs) : 1;
    a.out.ld = n_out;
  }
  a.oq = act_out;
  a.o_nb = n_out / 32;
  a.act = act_f32;
  a.fa = fa ? *fa : FfnAct{};
  a.split_max = int(split_segs);
  if (split_segs) {
    a.split_cnt = reinterpret_cast<unsigned *>(split_ws) + (nv == 2 ? 0 : kSplitCntWords);
    a.part = reinterpret_cast<float *>(split_ws + 2 * kSplitCntWords * 4);
  }
  {
    // A pair's four 16-byte term records of one line are 64 contiguous
    // bytes (8 elements of 8 bytes); a box row is the pairs of one pass and
    // line (512 or 1536 contiguous bytes), five lines per chunk. Boxes land
    // as [chunk][4 blocks, scales][pair][term]: B rows 4p + t.
    const int pairs_per_pass = wide ? tc::Cfg<1, true>::kPairs : tc::Cfg<1, false>::kPairs;
    const int chunks_per_stage = nv == 2 ? (wide ? tc::Cfg<2, true>::kSfc : tc::Cfg<2, false>::kSfc)
                                         : (wide ? tc::Cfg<1, true>::kSfc : tc::Cfg<1, false>::kSfc);
    const uint64_t nc = uint64_t((pool->nb + 3) / 4);
    const uint64_t row_u64 = uint64_t(n_pairs) * tc::kTerms * 2;
    const uint64_t dq[3] = {row_u64, 5, nc};
    const uint64_t sq[2] = {row_u64 * 8, row_u64 * 8 * 5};
    const uint32_t bq[3] = {uint32_t(pairs_per_pass * tc::kTerms * 2), 5, uint32_t(chunks_per_stage)};
    if (!encode_tmap_u64_3d(&a.tm_aq, a.aq, dq, sq, bq))
      return fail(MSB_ERR_CUDA, "tensor-core path: activation tensor map could not be encoded");
  }
  if (wide)
    return nv == 2 ? launch_tc_t<2, true>(a, max_active, n_pairs, st)
                   : launch_tc_t<1, true>(a, max_active, n_pairs, st);
  return nv == 2 ? launch_tc_t<2, false>(a, max_active, n_pairs, st)
                 : launch_tc_t<1, false>(a, max_active, n_pairs, st);
}

}  // namespace msb

namespace msb {
// Device address of the status word on the current device, for kernels of
// other translation units (looked up once per device).
int status_word(int **out) {
  static std::mutex mu;
  static int *addr[64] = {};
  int dev = 0;
  MSB_CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) return fail(MSB_ERR_INVALID, "device %d out of range", dev);
  std::lock_guard<std::mutex> lk(mu);
  if (!addr[dev]) {
    void *p = nullptr;
    MSB_CUDA_TRY(cudaGetSymbolAddress(&p, tc::g_status));
    addr[dev] = static_cast<int *>(p);
  }
  *out = addr[dev];
  return MSB_OK;
}
}  // namespace msb

extern "C" int msb_stream_check(void *stream, int32_t clear) {
  MSB_CUDA_TRY(cudaStreamSynchronize(static_cast<cudaStream_t>(stream)));
  int32_t v = 0;
  if (int rc = msb_device_status(&v, clear)) return rc;
  if (v == 0) return MSB_OK;
  static const char *names[] = {"tensor-core producer", "accumulator release", "stage arrival",
                                "accumulator arrival", "teardown drain",
                                "expert-parallel rows", "expert-parallel results"};
  char buf[256];
  int n = 0;
  for (int b = 0; b < 7; ++b)
    if (v & (1 << b))
      n += snprintf(buf + n, sizeof(buf) - size_t(n), "%s%s", n ? ", " : "", names[b]);
  if (n == 0) snprintf(buf, sizeof(buf), "unknown");
  return msb::fail(MSB_ERR_TIMEOUT, "a bounded device wait gave up (status 0x%x: %s)", v, buf);
}

extern "C" int msb_device_status(int32_t *status, int32_t clear) {
  MSB_CHECK_ARG(status, "msb_device_status: null status");
  int v = 0;
  MSB_CUDA_TRY(cudaMemcpyFromSymbol(&v, msb::tc::g_status, sizeof(int)));
  *status = v;
  if (clear && v) {
    const int zero = 0;
    MSB_CUDA_TRY(cudaMemcpyToSymbol(msb::tc::g_status, &zero, sizeof(int)));
  }
  return MSB_OK;
}
