// mul_mat_id over the slot pool, the fused SwiGLU variant, and the MoE FFN
// layer built from them (the router-weighted combine runs in the down
// projection's epilogue: Combine in msb_internal.h).
//
// Operator contract (ggml_mul_mat_id; call sites research/spikes/
// s0_slot_slab/main.c:117-148, s6_arena_mulmatid/main.c:82-134):
//   res[n, k, t] = sum_i dequant(as[:, n, slot(k, t)])[i] * b[i, k % b_ne1, t]
//
// Arithmetic (the form of ggml's CPU vec_dot for IQ4_NL and MXFP4 with q8_0
// activations): each 32-element activation block is quantized to int8 with
// d = amax / 127 (codes from the unrounded d, d stored as fp16); per weight
// block the int8 codes are dotted in int32 (dp4a), scaled by
// d_weight * d_act and accumulated in f32.
//
// Kernel shape (decode GEMV): one CTA per (active slot, 32-row tile); lane =
// output row, the 8 warps split the K blocks. Weights stream from HBM as
// coalesced 128-bit loads of the block-major pool layout; the activations of
// the slot's pairs sit in shared memory and are read as warp-wide broadcasts.
// Pairs beyond kMaxPairs per slot are processed in further passes over the
// same weights.
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <cuda_bf16.h>

#include <atomic>
#include <mutex>

#include "msb_internal.h"
#include "pool.cuh"
#include "quant.cuh"

namespace msb {

// Tensor-core path (mmid_tc.cu).
int64_t tc_act_bytes(int64_t nb, int64_t rows);
// Scratch for the split over K of small batches (0 when the batch is not
// small): partial sums of up to two views with n_out_max rows.
int64_t tc_split_bytes(int64_t n_out_max, int64_t n_pairs);
int64_t tc_split_zero_words(int64_t n_pairs);
int tc_supported(const msb_pool_s *p);
int set_wide_policy(int v);
// IQ4_NL on the tensor cores (mmid_f16.cu).
int64_t f16_act_bytes(int64_t K, int64_t rows);
int f16_supported(const msb_pool_s *p);
int f16_act(const void *b, int b_type, int64_t ne1, int64_t nb1, int64_t nb2, int32_t top_k,
            const int32_t *rows, int64_t n_pairs, int64_t K, void *xo, cudaStream_t st,
            uint32_t *zero, int64_t zero_n);
int f16_projection(const msb_pool_s *const *pools, int nv, const int64_t *row0, int64_t n_out,
                   const msb_route_t *route, int64_t n_pairs, const void *x_in, float *res,
                   void *x_out, float *act_f32, int max_active, cudaStream_t st,
                   const RowTarget *res_rows, const FfnAct *fa, const FfnBias *bias,
                   const Combine *comb);
int tc_act_terms(const void *b, int b_type, int64_t ne1, int64_t nb1, int64_t nb2, int32_t top_k,
                 const int32_t *rows, int64_t n_pairs, int64_t nb, uint8_t *ws, cudaStream_t st,
                 uint32_t *zero = nullptr, int64_t zero_n = 0);
int tc_projection(const msb_pool_s *const *pools, int nv, const int64_t *row0, int64_t n_out,
                  const msb_route_t *route, int64_t n_pairs, const uint8_t *act_in, float *res,
                  uint8_t *act_out, float *act_f32, int max_active, cudaStream_t st,
                  const RowTarget *res_rows = nullptr, const FfnAct *fa = nullptr,
                  uint8_t *split_ws = nullptr, int64_t split_bytes = 0,
                  const FfnBias *bias = nullptr, const Combine *comb = nullptr,
                  bool allow_wide = true);

// MXFP4 arithmetic: 0 = tensor cores where the shapes allow, 1 = CUDA cores
// with int8 activations (ggml's q8_0 form) everywhere.
static int g_mxfp4_path = 0;

// IQ4_NL arithmetic: 0 = tensor cores (f16 dequantization) for prompt-sized
// batches where the shapes allow, CUDA cores otherwise; 1 = CUDA cores
// everywhere; 2 = tensor cores wherever the shapes allow.
static int g_iq4nl_path = 0;
constexpr int64_t kF16PairsPerSlot = 4;

static bool use_f16(int64_t pairs, int max_active) {
  if (g_iq4nl_path == 1) return false;
  if (g_iq4nl_path == 2) return true;
  return pairs >= kF16PairsPerSlot * max_active;
}

// Bound of every device wait, in nanoseconds (MSB_OPT_WAIT_LIMIT_US).
static std::atomic<int64_t> g_wait_ns{1000000000};
int64_t wait_limit_ns() { return g_wait_ns.load(); }

static constexpr int kThreads = 256;
static constexpr int kWarps = kThreads / 32;
static constexpr int kMaxPairs = 8;  // activation rows held per pass
static constexpr int kPrefetch = 4;  // weight blocks in flight per lane and view

// Activations quantized per block, interleaved order (quant.cuh):
// codes at q + (row*nb + b)*32, scale at d[row*nb + b].
struct ActQ8 {
  int8_t *q;
  float *d;
  int64_t nb;
};

__device__ __forceinline__ float round_half_away(float x) { return roundf(x); }

// ---------------------------------------------------------------------------
// Activation quantization: one warp per (row, block); lane j owns element j.
// Row r = t * ne1 + j1 covers b[:, j1, t].
// ---------------------------------------------------------------------------
template <typename T>
__device__ __forceinline__ float load_act(const char *p) {
  if constexpr (sizeof(T) == 4) return *reinterpret_cast<const float *>(p);
  else return __bfloat162float(*reinterpret_cast<const __nv_bfloat16 *>(p));
}

__device__ __forceinline__ void store_q8_block(ActQ8 out, int64_t row, int64_t b, float v,
                                               int lane) {
  float amax = fabsf(v);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  const float d = amax / 127.f;
  const float id = d != 0.f ? 1.f / d : 0.f;
  const int q = int(round_half_away(__fmul_rn(v, id)));
  out.q[(row * out.nb + b) * 32 + interleaved_pos(lane)] = int8_t(q);
  if (lane == 0) out.d[row * out.nb + b] = __half2float(__float2half_rn(d));
}

template <typename T>
__global__ void __launch_bounds__(kThreads) quantize_act_kernel(
    const char *b, int64_t nb1, int64_t nb2, int64_t ne1, int64_t n_rows, ActQ8 out,
    uint32_t *zero, int64_t zero_n) {
  pdl_wait();
  pdl_trigger();
  grid_zero(zero, zero_n);   // the call's combine counters
  const int lane = threadIdx.x & 31;
  const int64_t item = int64_t(blockIdx.x) * kWarps + (threadIdx.x >> 5);
  if (item >= n_rows * out.nb) return;
  const int64_t row = item / out.nb, blk = item % out.nb;
  const int64_t t = row / ne1, j1 = row % ne1;
  const char *p = b + t * nb2 + j1 * nb1 + (blk * 32 + lane) * int64_t(sizeof(T));
  store_q8_block(out, row, blk, load_act<T>(p), lane);
}

// ---------------------------------------------------------------------------
// Grouped GEMV
// ---------------------------------------------------------------------------
struct GemvArgs {
  PoolView w;        // weights (the gate when SWIGLU)
  PoolView w2;       // up weights (SWIGLU only)
  int64_t n_out;     // output rows per view
  int tiles;         // ceil(n_out / 32)
  const int32_t *counts, *offsets, *rows, *active;
  int32_t zero_slot;
  int32_t top_k, b_ne1;
  ActQ8 in;          // activations, nb = w.nb
  float *res;        // plain: res[pair * n_out + n]
  ActQ8 out;         // SWIGLU: quantized silu(g) * u, nb = n_out / 32
  float *act;        // SWIGLU, optional: f32 silu(g) * u [pair * n_out + n]
  FfnAct fa;         // SWIGLU: the activation
  FfnBias bias;      // expert biases (view 0, and view 1 with SWIGLU)
  Combine comb;      // plain: the fused router-weighted combine (optional)
};

template <int WT>
__device__ __forceinline__ Codebook codebook() {
  if constexpr (WT == MSB_TYPE_MXFP4) return codebook_mxfp4();
  else return codebook_iq4nl();
}

// Dot of one weight block (8 code words) with one activation block.
__device__ __forceinline__ int dot_block(const uint32_t (&wq)[8], const int4 *a) {
  const int4 a0 = a[0], a1 = a[1];
  int s = __dp4a(int(wq[0]), a0.x, 0);
  s = __dp4a(int(wq[1]), a0.y, s);
  s = __dp4a(int(wq[2]), a0.z, s);
  s = __dp4a(int(wq[3]), a0.w, s);
  s = __dp4a(int(wq[4]), a1.x, s);
  s = __dp4a(int(wq[5]), a1.y, s);
  s = __dp4a(int(wq[6]), a1.z, s);
  s = __dp4a(int(wq[7]), a1.w, s);
  return s;
}

// Raw weight block of one lane: 16 bytes of nibbles and the scale bits.
struct RawBlock {
  uint4 q;
  uint32_t s;
};

template <int WT>
__device__ __forceinline__ RawBlock load_block(const PoolView &v, int slot, int64_t b, int64_t n,
                                               bool valid) {
  RawBlock r{make_uint4(0, 0, 0, 0), 0u};
  if (valid) {
    const uint8_t *sb = v.base + int64_t(slot) * v.slot_stride;
    const int64_t off = b * v.N + v.row0 + n;
    r.q = __ldg(reinterpret_cast<const uint4 *>(sb + off * 16));
    const uint8_t *sc = sb + v.nb * v.N * 16;
    if constexpr (WT == MSB_TYPE_MXFP4) r.s = __ldg(sc + scale_offset(true, b, v.row0 + n, v.N, v.nb));
    else r.s = __ldg(reinterpret_cast<const unsigned short *>(sc) + off);
  }
  return r;
}

template <int WT>
__device__ __forceinline__ float scale_of(uint32_t s) {
  if constexpr (WT == MSB_TYPE_MXFP4) return e8m0_half(s);
  else return __half2float(__ushort_as_half((unsigned short)s));
}

__device__ __forceinline__ void decode_block(const uint4 &q, const Codebook &cb,
                                             uint32_t (&wq)[8]) {
  decode_nibbles(q.x, cb, wq[0], wq[1]);
  decode_nibbles(q.y, cb, wq[2], wq[3]);
  decode_nibbles(q.z, cb, wq[4], wq[5]);
  decode_nibbles(q.w, cb, wq[6], wq[7]);
}

// K loop of one pass over C activation rows: each warp takes blocks
// b = warp, warp + 8, ...; lane = output row. Partial sums go to s_red.
template <int WT, bool SWIGLU, int C>
__device__ __forceinline__ void k_loop(const GemvArgs &a, int slot, int64_t n, bool valid,
                                       int warp, int lane, const int8_t *s_q, const float *s_d,
                                       float *s_red) {
  constexpr int NV = SWIGLU ? 2 : 1;
  const int nb = int(a.w.nb);
  const Codebook cb = codebook<WT>();
  float acc[NV][C];
#pragma unroll
  for (int v = 0; v < NV; ++v)
#pragma unroll
    for (int r = 0; r < C; ++r) acc[v][r] = 0.f;
  // Rolling prefetch: kPrefetch block loads per view stay in flight; each
  // consumed slot is refilled with the block kPrefetch iterations ahead.
  const int n_iter = nb > warp ? (nb - warp + kWarps - 1) / kWarps : 0;
  RawBlock buf[kPrefetch][NV];
#pragma unroll
  for (int p = 0; p < kPrefetch; ++p) {
    const bool in = p < n_iter;
    buf[p][0] = load_block<WT>(a.w, slot, warp + p * kWarps, n, valid && in);
    if constexpr (SWIGLU) buf[p][NV - 1] = load_block<WT>(a.w2, slot, warp + p * kWarps, n, valid && in);
  }
  for (int base = 0; base < n_iter; base += kPrefetch) {
#pragma unroll
    for (int p = 0; p < kPrefetch; ++p) {
      const int it = base + p;
      if (it < n_iter) {
        const int b = warp + it * kWarps;
        uint32_t wq[NV][8];
        float sw[NV];
#pragma unroll
        for (int v = 0; v < NV; ++v) {
          decode_block(buf[p][v].q, cb, wq[v]);
          sw[v] = scale_of<WT>(buf[p][v].s);
        }
        const int nxt = it + kPrefetch;
        const bool in = nxt < n_iter;
        buf[p][0] = load_block<WT>(a.w, slot, warp + nxt * kWarps, n, valid && in);
        if constexpr (SWIGLU) buf[p][NV - 1] = load_block<WT>(a.w2, slot, warp + nxt * kWarps, n, valid && in);
#pragma unroll
        for (int r = 0; r < C; ++r) {
          const int4 *ap = reinterpret_cast<const int4 *>(s_q + (int64_t(r) * nb + b) * 32);
          const float da = s_d[r * nb + b];
#pragma unroll
          for (int v = 0; v < NV; ++v)
            acc[v][r] += __fmul_rn(sw[v], da) * float(dot_block(wq[v], ap));
        }
      }
    }
  }
#pragma unroll
  for (int v = 0; v < NV; ++v)
#pragma unroll
    for (int r = 0; r < C; ++r) s_red[((warp * NV + v) * kMaxPairs + r) * 32 + lane] = acc[v][r];
}

template <int WT, bool SWIGLU>
__global__ void __launch_bounds__(kThreads, 2) gemv_kernel(GemvArgs a) {
  constexpr int NV = SWIGLU ? 2 : 1;  // weight views per lane
  pdl_wait();
  pdl_trigger();
  extern __shared__ __align__(16) uint8_t smem[];
  const int nb = int(a.w.nb);
  int8_t *s_q = reinterpret_cast<int8_t *>(smem);                           // [kMaxPairs][nb][32]
  float *s_d = reinterpret_cast<float *>(smem + size_t(kMaxPairs) * nb * 32);  // [kMaxPairs][nb]
  float *s_red = s_d + size_t(kMaxPairs) * nb;                              // [kWarps][NV][kMaxPairs][32]

  const int ai = blockIdx.x / a.tiles;
  const int tile = blockIdx.x - ai * a.tiles;
  if (ai >= a.active[0]) return;
  const int slot = a.active[1 + ai];
  const int c_total = a.counts[slot];
  const int32_t *prs = a.rows + a.offsets[slot];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t n0 = int64_t(tile) * 32;
  const int64_t n = n0 + lane;
  const bool valid = n < a.n_out;

  if (slot == a.zero_slot) {
    // Every weight of the zero slot is 0: write the exact result directly.
    for (int r = warp; r < c_total; r += kWarps) {
      const int64_t pair = prs[r];
      if constexpr (SWIGLU) {
        a.out.q[(pair * a.out.nb + tile) * 32 + lane] = 0;
        if (lane == 0) a.out.d[pair * a.out.nb + tile] = 0.f;
        if (a.act && valid) a.act[pair * a.n_out + n] = 0.f;
      } else {
        if (valid) a.res[pair * a.n_out + n] = 0.f;
        combine_arrive(a.comb, pair, 1, tile, lane);
      }
    }
    return;
  }

  for (int c0 = 0; c0 < c_total; c0 += kMaxPairs) {
    const int cc = min(kMaxPairs, c_total - c0);
    __syncthreads();  // shared buffers of the previous pass are consumed
    // Stage the activation blocks of this pass's pairs.
    const int units = cc * nb * 2;  // 16-byte units
    for (int u = threadIdx.x; u < units; u += kThreads) {
      const int r = u / (nb * 2), rem = u - r * nb * 2;
      const int64_t pair = prs[c0 + r];
      const int64_t t = pair / a.top_k, k = pair - t * a.top_k;
      const int64_t arow = t * a.b_ne1 + (k % a.b_ne1);
      reinterpret_cast<int4 *>(s_q)[int64_t(r) * nb * 2 + rem] =
          reinterpret_cast<const int4 *>(a.in.q + arow * a.in.nb * 32)[rem];
    }
    for (int u = threadIdx.x; u < cc * nb; u += kThreads) {
      const int r = u / nb, bb = u - r * nb;
      const int64_t pair = prs[c0 + r];
      const int64_t t = pair / a.top_k, k = pair - t * a.top_k;
      const int64_t arow = t * a.b_ne1 + (k % a.b_ne1);
      s_d[u] = a.in.d[arow * a.in.nb + bb];
    }
    __syncthreads();

    // The K loop is specialized on the pass's pair count, so no instruction
    // is issued for pairs the pass does not have.
    switch (cc) {
      case 1: k_loop<WT, SWIGLU, 1>(a, slot, n, valid, warp, lane, s_q, s_d, s_red); break;
      case 2: k_loop<WT, SWIGLU, 2>(a, slot, n, valid, warp, lane, s_q, s_d, s_red); break;
      case 3: k_loop<WT, SWIGLU, 3>(a, slot, n, valid, warp, lane, s_q, s_d, s_red); break;
      case 4: k_loop<WT, SWIGLU, 4>(a, slot, n, valid, warp, lane, s_q, s_d, s_red); break;
      case 5: k_loop<WT, SWIGLU, 5>(a, slot, n, valid, warp, lane, s_q, s_d, s_red); break;
      case 6: k_loop<WT, SWIGLU, 6>(a, slot, n, valid, warp, lane, s_q, s_d, s_red); break;
      case 7: k_loop<WT, SWIGLU, 7>(a, slot, n, valid, warp, lane, s_q, s_d, s_red); break;
      default: k_loop<WT, SWIGLU, 8>(a, slot, n, valid, warp, lane, s_q, s_d, s_red); break;
    }
    __syncthreads();

    // Reduce over warps in fixed order; warp r finishes pair r of the pass.
    for (int r = warp; r < cc; r += kWarps) {
      float tot[NV];
#pragma unroll
      for (int v = 0; v < NV; ++v) {
        float s = 0.f;
        for (int w = 0; w < kWarps; ++w) s += s_red[((w * NV + v) * kMaxPairs + r) * 32 + lane];
        tot[v] = s;
      }
      const int64_t pair = prs[c0 + r];
      if (valid) {
        if (const float *br = bias_row(a.bias, 0, pair)) tot[0] += br[n];
        if constexpr (SWIGLU)
          if (const float *br = bias_row(a.bias, 1, pair)) tot[NV - 1] += br[n];
      }
      if constexpr (SWIGLU) {
        const float g = tot[0], up = tot[1];
        float h = valid ? ffn_act(a.fa, g, up) : 0.f;
        if (a.act && valid) a.act[pair * a.n_out + n] = h;
        store_q8_block(a.out, pair, tile, h, lane);
      } else {
        if (valid) a.res[pair * a.n_out + n] = tot[0];
        combine_arrive(a.comb, pair, 1, tile, lane);
      }
    }
  }
}

// ---------------------------------------------------------------------------
// Host helpers
// ---------------------------------------------------------------------------
static int64_t align_up(int64_t x, int64_t a) { return (x + a - 1) / a * a; }

// Carves an ActQ8 for n_rows x nb out of the workspace at *off.
static ActQ8 carve_act(uint8_t *ws, int64_t *off, int64_t n_rows, int64_t nb) {
  ActQ8 q;
  q.q = reinterpret_cast<int8_t *>(ws + *off);
  *off = align_up(*off + n_rows * nb * 32, 256);
  q.d = reinterpret_cast<float *>(ws + *off);
  *off = align_up(*off + n_rows * nb * 4, 256);
  q.nb = nb;
  return q;
}

static int quantize_act(const void *b, int b_type, int64_t b_ne1, int64_t b_nb1, int64_t b_nb2,
                        int64_t n_rows, ActQ8 out, cudaStream_t st, uint32_t *zero = nullptr,
                        int64_t zero_n = 0) {
  const int64_t items = n_rows * out.nb;
  if (items == 0) return MSB_OK;
  const int64_t grid = (items + kWarps - 1) / kWarps;
  const char *p = static_cast<const char *>(b);
  if (b_type == MSB_TYPE_F32)
    MSB_CUDA_TRY(launch_pdl(quantize_act_kernel<float>, dim3(unsigned(grid)), dim3(kThreads), 0, st,
                            p, b_nb1, b_nb2, b_ne1, n_rows, out, zero, zero_n));
  else if (b_type == MSB_TYPE_BF16)
    MSB_CUDA_TRY(launch_pdl(quantize_act_kernel<__nv_bfloat16>, dim3(unsigned(grid)), dim3(kThreads),
                            0, st, p, b_nb1, b_nb2, b_ne1, n_rows, out, zero, zero_n));
  else
    return fail(MSB_ERR_INVALID, "activation type %d is not F32 or BF16", b_type);
  count_launch();
  MSB_CUDA_TRY(cudaGetLastError());
  return MSB_OK;
}

// One-shot timing request for the next fused gate/up launch on this thread.
static thread_local cudaEvent_t g_gate_up_start = nullptr, g_gate_up_stop = nullptr;

// Under stream capture the event becomes an external event node of the
// graph, so it is recorded (and timeable) at every replay.
static cudaError_t record_timing_event(cudaEvent_t ev, cudaStream_t st) {
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  if (cudaError_t e = cudaStreamIsCapturing(st, &cs)) return e;
  return cs == cudaStreamCaptureStatusActive ? cudaEventRecordWithFlags(ev, st, cudaEventRecordExternal)
                                             : cudaEventRecord(ev, st);
}

template <int WT, bool SWIGLU>
static int launch_gemv_t(const GemvArgs &a, int max_active, cudaStream_t st) {
  const int NV = SWIGLU ? 2 : 1;
  const size_t smem = size_t(kMaxPairs) * a.w.nb * 36 + size_t(kWarps) * NV * kMaxPairs * 32 * 4;
  if (smem > 48 * 1024)
    MSB_CUDA_TRY(cudaFuncSetAttribute(gemv_kernel<WT, SWIGLU>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)));
  const int64_t grid = int64_t(max_active) * a.tiles;
  if (grid == 0) return MSB_OK;
  const bool timed = SWIGLU && g_gate_up_start && g_gate_up_stop;
  if (timed) MSB_CUDA_TRY(record_timing_event(g_gate_up_start, st));
  MSB_CUDA_TRY(launch_pdl(gemv_kernel<WT, SWIGLU>, dim3(unsigned(grid)), dim3(kThreads), smem, st, a));
  count_launch();
  if (timed) {
    MSB_CUDA_TRY(record_timing_event(g_gate_up_stop, st));
    g_gate_up_start = g_gate_up_stop = nullptr;
  }
  MSB_CUDA_TRY(cudaGetLastError());
  return MSB_OK;
}

static int launch_gemv(int wtype, bool swiglu, const GemvArgs &a, int max_active, cudaStream_t st) {
  if (a.w.nb * 36 * kMaxPairs > 160 * 1024)
    return fail(MSB_ERR_UNSUPPORTED, "K = %lld too large for the staged activations", (long long)(a.w.nb * 32));
  if (wtype == MSB_TYPE_MXFP4)
    return swiglu ? launch_gemv_t<MSB_TYPE_MXFP4, true>(a, max_active, st)
                  : launch_gemv_t<MSB_TYPE_MXFP4, false>(a, max_active, st);
  if (wtype == MSB_TYPE_IQ4_NL)
    return swiglu ? launch_gemv_t<MSB_TYPE_IQ4_NL, true>(a, max_active, st)
                  : launch_gemv_t<MSB_TYPE_IQ4_NL, false>(a, max_active, st);
  return fail(MSB_ERR_INVALID, "weight type %d", wtype);
}

static void set_route(GemvArgs &g, const msb_route_t *r) {
  g.counts = r->counts;
  g.offsets = r->offsets;
  g.rows = r->rows;
  g.active = r->active;
}

}  // namespace msb

using namespace msb;

extern "C" void msb_time_next_gate_up(void *start, void *stop) {
  g_gate_up_start = static_cast<cudaEvent_t>(start);
  g_gate_up_stop = static_cast<cudaEvent_t>(stop);
}

// Words of the fused combine's counters: one per (token, 32-row block of the
// output width).
static int64_t combine_words(int64_t n_tok, int64_t n_out) { return n_tok * ((n_out + 31) / 32); }

extern "C" int64_t msb_workspace_bytes(int64_t K_max, int32_t n_tok, int32_t top_k, int32_t n_slot) {
  (void)n_slot;
  if (K_max <= 0 || K_max % 32 || n_tok < 0 || top_k <= 0) return -1;
  const int64_t nb = K_max / 32, pairs = int64_t(n_tok) * top_k;
  const int64_t cnt = align_up(combine_words(n_tok, K_max) * 4, 256);
  // CUDA-core path: int8 activations in and SwiGLU out, down result, the
  // combine's counters.
  int64_t q8 = 0;
  q8 = align_up(q8 + pairs * nb * 32, 256);
  q8 = align_up(q8 + pairs * nb * 4, 256);
  q8 = align_up(q8 + pairs * nb * 32, 256);
  q8 = align_up(q8 + pairs * nb * 4, 256);
  q8 = align_up(q8 + pairs * K_max * 4, 256);
  q8 += cnt;
  // Tensor-core path: activation terms in and SwiGLU out, down result, the
  // combine's counters.
  int64_t tcb = 0;
  tcb = align_up(tcb + tc_act_bytes(nb, pairs), 256);
  tcb = align_up(tcb + tc_act_bytes(nb, pairs), 256);
  tcb = align_up(tcb + pairs * K_max * 4, 256);
  tcb += cnt;
  // Split over K of small batches: partial sums (the largest projection
  // mul_mat_id serves has 2 K_max rows: a fused gate_up).
  tcb = align_up(tcb + tc_split_bytes(2 * K_max, pairs), 256);
  // IQ4_NL tensor-core path: f16 activations in and SwiGLU out, down result,
  // the combine's counters.
  int64_t f16b = 0;
  f16b = align_up(f16b + f16_act_bytes(K_max, pairs), 256);
  f16b = align_up(f16b + f16_act_bytes(K_max, pairs), 256);
  f16b = align_up(f16b + pairs * K_max * 4, 256);
  f16b += cnt;
  int64_t need = q8 > tcb ? q8 : tcb;
  if (f16b > need) need = f16b;
  return need + 256;
}

extern "C" int msb_set_option(int option, int value) {
  if (option == MSB_OPT_MXFP4_PATH) {
    MSB_CHECK_ARG(value == 0 || value == 1, "msb_set_option: MXFP4 path must be 0 or 1");
    g_mxfp4_path = value;
    return MSB_OK;
  }
  if (option == MSB_OPT_WIDE_PASSES) return set_wide_policy(value);
  if (option == MSB_OPT_IQ4NL_PATH) {
    MSB_CHECK_ARG(value >= 0 && value <= 2, "msb_set_option: IQ4_NL path must be 0, 1 or 2");
    g_iq4nl_path = value;
    return MSB_OK;
  }
  if (option == MSB_OPT_WAIT_LIMIT_US) {
    MSB_CHECK_ARG(value >= 1 && value <= 60000000,
                  "msb_set_option: wait limit must be 1 .. 60000000 microseconds");
    g_wait_ns.store(int64_t(value) * 1000);
    return MSB_OK;
  }
  return fail(MSB_ERR_INVALID, "msb_set_option: unknown option %d", option);
}

extern "C" int msb_mul_mat_id(msb_pool_t pool, const void *b_dev, int b_type, int64_t b_ne1,
                              int64_t b_nb1, int64_t b_nb2, const msb_route_t *route,
                              int32_t top_k, int32_t n_tok, float *res_dev, void *workspace,
                              int64_t workspace_bytes, void *stream) {
  MSB_CHECK_ARG(pool && route && res_dev && workspace, "msb_mul_mat_id: null argument");
  MSB_CHECK_ARG(b_dev || n_tok == 0, "msb_mul_mat_id: null b");
  MSB_CHECK_ARG(top_k > 0 && n_tok >= 0, "msb_mul_mat_id: bad shape");
  MSB_CHECK_ARG(b_ne1 == 1 || b_ne1 == top_k, "msb_mul_mat_id: b_ne1 must be 1 or top_k");
  const int64_t need = msb_workspace_bytes(pool->K, n_tok, top_k, pool->n_slot);
  MSB_CHECK_ARG(workspace_bytes >= need, "msb_mul_mat_id: workspace %lld < %lld bytes",
                (long long)workspace_bytes, (long long)need);
  if (n_tok == 0) return MSB_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  uint8_t *ws = static_cast<uint8_t *>(workspace);
  int64_t off = 0;
  const int64_t pairs = int64_t(n_tok) * top_k;
  const int max_active = int(pairs < pool->n_slot + 1 ? pairs : pool->n_slot + 1);
  if (g_mxfp4_path == 0 && tc_supported(pool)) {
    // Tensor cores: activation terms per pair (grouped order), then one
    // projection writing res directly.
    // The rest of the workspace is the split scratch; its segment counters
    // are zeroed by the activation-terms kernel.
    uint8_t *act = ws;
    const int64_t used = align_up(tc_act_bytes(pool->nb, pairs), 256);
    if (int rc = tc_act_terms(b_dev, b_type, b_ne1, b_nb1, b_nb2, top_k, route->rows, pairs,
                              pool->nb, act, st, reinterpret_cast<uint32_t *>(ws + used),
                              tc_split_zero_words(pairs)))
      return rc;
    const int64_t row0[2] = {0, 0};
    const msb_pool_s *pools[2] = {pool, pool};
    return tc_projection(pools, 1, row0, pool->N, route, pairs, act, res_dev, nullptr, nullptr,
                         max_active, st, nullptr, nullptr, ws + used, workspace_bytes - used);
  }
  if (f16_supported(pool) && use_f16(pairs, max_active)) {
    // Tensor cores: f16 activations per pair (grouped order), then one
    // projection writing res directly.
    if (int rc = f16_act(b_dev, b_type, b_ne1, b_nb1, b_nb2, top_k, route->rows, pairs, pool->K,
                         ws, st, nullptr, 0))
      return rc;
    const int64_t row0[2] = {0, 0};
    const msb_pool_s *pools[2] = {pool, pool};
    return f16_projection(pools, 1, row0, pool->N, route, pairs, ws, res_dev, nullptr, nullptr,
                          max_active, st, nullptr, nullptr, nullptr, nullptr);
  }
  const int64_t n_rows = int64_t(n_tok) * b_ne1;
  ActQ8 in = carve_act(ws, &off, n_rows, pool->nb);
  if (int rc = quantize_act(b_dev, b_type, b_ne1, b_nb1, b_nb2, n_rows, in, st)) return rc;
  GemvArgs g{};
  g.w = view_of(pool);
  g.w2 = g.w;
  g.n_out = pool->N;
  g.tiles = int((pool->N + 31) / 32);
  set_route(g, route);
  g.zero_slot = pool->n_slot;
  g.top_k = top_k;
  g.b_ne1 = int32_t(b_ne1);
  g.in = in;
  g.res = res_dev;
  return launch_gemv(pool->wtype, false, g, max_active, st);
}

// Internal bias views of one FFN call: gate/up (views 0 and 1) and down.
static void split_bias(const msb_ffn_bias_t *b, int32_t top_k, FfnBias *gu, FfnBias *dn) {
  *gu = FfnBias{};
  *dn = FfnBias{};
  if (!b) return;
  FfnBias base;
  base.ids = reinterpret_cast<const char *>(b->ids);
  base.nb0 = b->ids_nb0;
  base.nb1 = b->ids_nb1;
  base.top_k = top_k;
  base.n_expert = b->n_expert;
  *gu = base;
  gu->b[0] = b->gate_b;
  gu->ld[0] = b->gate_ld;
  gu->b[1] = b->up_b;
  gu->ld[1] = b->up_ld;
  *dn = base;
  dn->b[0] = b->down_b;
  dn->ld[0] = b->down_ld;
}

// msb_moe_ffn; with `rows` the down projection stores its result rows there
// instead of y (top_k 1, no weights, tensor-core shapes only).
static int moe_ffn_core(msb_pool_t gate, msb_pool_t up, int64_t up_row0, msb_pool_t down,
                        const void *x_dev, int x_type, int64_t x_nb1, const msb_route_t *route,
                        const float *w_dev, int32_t top_k, int32_t n_tok, float *y_dev,
                        float *act_dev, void *workspace, int64_t workspace_bytes,
                        const RowTarget *rows, void *stream, const FfnAct &fa,
                        const msb_ffn_bias_t *bias, bool accumulate = false) {
  MSB_CHECK_ARG(fa.kind == 0 || (fa.kind == 1 && fa.limit > 0.f),
                "msb_moe_ffn: unknown activation %d (or limit <= 0)", fa.kind);
  MSB_CHECK_ARG(gate && up && down && route && (y_dev || rows) && workspace,
                "msb_moe_ffn: null argument");
  MSB_CHECK_ARG(!rows || (!w_dev && top_k == 1), "msb_moe_ffn: row targets need top_k 1");
  MSB_CHECK_ARG(w_dev || top_k == 1, "msb_moe_ffn: router weights may be omitted only for top_k 1");
  MSB_CHECK_ARG(x_dev || n_tok == 0, "msb_moe_ffn: null x");
  MSB_CHECK_ARG(top_k > 0 && n_tok >= 0, "msb_moe_ffn: bad shape");
  MSB_CHECK_ARG(!accumulate || w_dev, "msb_moe_ffn: accumulating into y needs router weights");
  MSB_CHECK_ARG(!bias || ((bias->ids || n_tok == 0) && bias->n_expert > 0 &&
                          (bias->gate_b || bias->up_b || bias->down_b)),
                "msb_moe_ffn: biases need the router's expert ids, n_expert > 0 and a bias row");
  const int64_t n_ff = down->K;
  MSB_CHECK_ARG(gate->wtype == up->wtype && up->wtype == down->wtype,
                "msb_moe_ffn: gate, up and down must share a weight type");
  MSB_CHECK_ARG(gate->K == up->K && down->N == gate->K,
                "msb_moe_ffn: gate/up input width must equal down output width");
  MSB_CHECK_ARG(gate->n_slot == up->n_slot && up->n_slot == down->n_slot,
                "msb_moe_ffn: pools must have the same slot count");
  MSB_CHECK_ARG(up_row0 >= 0 && up_row0 + n_ff <= up->N && n_ff <= gate->N,
                "msb_moe_ffn: gate/up rows do not cover the down input width %lld", (long long)n_ff);
  MSB_CHECK_ARG(up != gate || up_row0 >= n_ff, "msb_moe_ffn: fused gate_up needs up_row0 >= N_ff");
  const int64_t K = gate->K;
  const int64_t kmax = K > n_ff ? K : n_ff;
  const int64_t need = msb_workspace_bytes(kmax, n_tok, top_k, gate->n_slot);
  MSB_CHECK_ARG(workspace_bytes >= need, "msb_moe_ffn: workspace %lld < %lld bytes",
                (long long)workspace_bytes, (long long)need);
  if (n_tok == 0) return MSB_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  uint8_t *ws = static_cast<uint8_t *>(workspace);
  const int64_t pairs = int64_t(n_tok) * top_k;
  FfnBias bias_gu, bias_dn;
  split_bias(bias, top_k, &bias_gu, &bias_dn);
  const int max_active = int(pairs < gate->n_slot + 1 ? pairs : gate->n_slot + 1);
  const bool tc = g_mxfp4_path == 0 && tc_supported(gate) && tc_supported(up) &&
                  tc_supported(down) && n_ff % 64 == 0 && up_row0 % 32 == 0;
  if (rows && !tc)
    return fail(MSB_ERR_UNSUPPORTED, "msb_moe_ffn: row targets need the tensor-core path");
  // With router weights the down projection's epilogue also combines: its
  // result rows go to the workspace and y is written by the last warp to
  // store each (token, 32-row block); without them (top_k 1) it writes y.
  const int64_t cnt_n = w_dev ? combine_words(n_tok, down->N) : 0;
  Combine comb;
  if (tc) {
    // Tensor cores: x terms per pair -> fused gate/up + SwiGLU writing the
    // down projection's terms -> down projection with the combine.
    int64_t o = 0;
    uint8_t *xa = ws + o;
    o = align_up(o + tc_act_bytes(gate->nb, pairs), 256);
    uint8_t *ha = ws + o;
    o = align_up(o + tc_act_bytes(n_ff / 32, pairs), 256);
    float *rd = w_dev ? reinterpret_cast<float *>(ws + o) : y_dev;
    o = align_up(o + pairs * down->N * 4, 256);
    uint32_t *cnt = reinterpret_cast<uint32_t *>(ws + o);
    o += align_up(cnt_n * 4, 256);
    if (w_dev) {
      comb.w = w_dev;
      comb.y = y_dev;
      comb.r = rd;
      comb.cnt = cnt;
      comb.top_k = top_k;
      comb.n_out = down->N;
      comb.nblk = (down->N + 31) / 32;
      comb.accumulate = accumulate;
    }
    // The rest: scratch for the split over K of small batches (gate/up and
    // down use it one after the other). The activation-terms kernel zeroes
    // the combine's counters and the split's segment counters, which follow
    // them.
    uint8_t *split_ws = ws + o;
    const int64_t split_bytes = workspace_bytes - o;
    const int64_t zero_n = (split_ws - reinterpret_cast<uint8_t *>(cnt)) / 4 + tc_split_zero_words(pairs);
    if (int rc = tc_act_terms(x_dev, x_type, 1, x_nb1, x_nb1, top_k, route->rows, pairs, gate->nb,
                              xa, st, zero_n ? cnt : nullptr, zero_n))
      return rc;
    const int64_t rows_gu[2] = {0, up_row0};
    const msb_pool_s *gu_pools[2] = {gate, up};
    const bool timed = g_gate_up_start && g_gate_up_stop;
    if (timed) MSB_CUDA_TRY(record_timing_event(g_gate_up_start, st));
    // Expert-parallel rows (`rows`) are mostly padding: the pairs per
    // expert stay few, so the passes stay narrow.
    if (int rc = tc_projection(gu_pools, 2, rows_gu, n_ff, route, pairs, xa, nullptr, ha, act_dev,
                               max_active, st, nullptr, &fa, split_ws, split_bytes, &bias_gu,
                               nullptr, rows == nullptr))
      return rc;
    if (timed) {
      MSB_CUDA_TRY(record_timing_event(g_gate_up_stop, st));
      g_gate_up_start = g_gate_up_stop = nullptr;
    }
    const int64_t rows_dn[2] = {0, 0};
    const msb_pool_s *dn_pools[2] = {down, down};
    return tc_projection(dn_pools, 1, rows_dn, down->N, route, pairs, ha, rd, nullptr, nullptr,
                         max_active, st, rows, nullptr, split_ws, split_bytes, &bias_dn, &comb,
                         rows == nullptr);
  }
  const bool f16 = !rows && f16_supported(gate) && f16_supported(up) && f16_supported(down) &&
                   up_row0 % 128 == 0 && use_f16(pairs, max_active);
  if (f16) {
    // Tensor cores with f16 dequantization: x in f16 per pair -> gate/up +
    // activation writing the down projection's f16 input -> down with the
    // combine.
    int64_t o = 0;
    uint8_t *xa = ws + o;
    o = align_up(o + f16_act_bytes(K, pairs), 256);
    uint8_t *ha = ws + o;
    o = align_up(o + f16_act_bytes(n_ff, pairs), 256);
    float *rd = w_dev ? reinterpret_cast<float *>(ws + o) : y_dev;
    o = align_up(o + pairs * down->N * 4, 256);
    uint32_t *cnt = reinterpret_cast<uint32_t *>(ws + o);
    if (w_dev) {
      comb.w = w_dev;
      comb.y = y_dev;
      comb.r = rd;
      comb.cnt = cnt;
      comb.top_k = top_k;
      comb.n_out = down->N;
      comb.nblk = (down->N + 31) / 32;
      comb.accumulate = accumulate;
    }
    if (int rc = f16_act(x_dev, x_type, 1, x_nb1, x_nb1, top_k, route->rows, pairs, K, xa, st,
                         w_dev ? cnt : nullptr, cnt_n))
      return rc;
    const int64_t rows_gu[2] = {0, up_row0};
    const msb_pool_s *gu_pools[2] = {gate, up};
    const bool timed = g_gate_up_start && g_gate_up_stop;
    if (timed) MSB_CUDA_TRY(record_timing_event(g_gate_up_start, st));
    if (int rc = f16_projection(gu_pools, 2, rows_gu, n_ff, route, pairs, xa, nullptr, ha,
                                act_dev, max_active, st, nullptr, &fa, &bias_gu, nullptr))
      return rc;
    if (timed) {
      MSB_CUDA_TRY(record_timing_event(g_gate_up_stop, st));
      g_gate_up_start = g_gate_up_stop = nullptr;
    }
    const int64_t rows_dn[2] = {0, 0};
    const msb_pool_s *dn_pools[2] = {down, down};
    return f16_projection(dn_pools, 1, rows_dn, down->N, route, pairs, ha, rd, nullptr, nullptr,
                          max_active, st, nullptr, nullptr, &bias_dn, &comb);
  }
  int64_t off = 0;
  ActQ8 xq = carve_act(ws, &off, n_tok, gate->nb);
  ActQ8 hq = carve_act(ws, &off, pairs, n_ff / 32);
  float *rdown = w_dev ? reinterpret_cast<float *>(ws + off) : y_dev;
  off = align_up(off + pairs * down->N * 4, 256);
  uint32_t *cnt = reinterpret_cast<uint32_t *>(ws + off);
  if (w_dev) {
    comb.w = w_dev;
    comb.y = y_dev;
    comb.r = rdown;
    comb.cnt = cnt;
    comb.top_k = top_k;
    comb.n_out = down->N;
    comb.nblk = (down->N + 31) / 32;
    comb.accumulate = accumulate;
  }
  if (int rc = quantize_act(x_dev, x_type, 1, x_nb1, x_nb1, n_tok, xq, st, w_dev ? cnt : nullptr,
                            cnt_n))
    return rc;

  GemvArgs g{};
  g.w = view_of(gate, 0);
  g.w2 = view_of(up, up_row0);
  g.n_out = n_ff;
  g.tiles = int((n_ff + 31) / 32);
  set_route(g, route);
  g.zero_slot = gate->n_slot;
  g.top_k = top_k;
  g.b_ne1 = 1;
  g.fa = fa;
  g.in = xq;
  g.out = hq;
  g.act = act_dev;
  g.bias = bias_gu;
  if (int rc = launch_gemv(gate->wtype, true, g, max_active, st)) return rc;

  GemvArgs d{};
  d.w = view_of(down);
  d.w2 = d.w;
  d.n_out = down->N;
  d.tiles = int((down->N + 31) / 32);
  set_route(d, route);
  d.zero_slot = down->n_slot;
  d.top_k = top_k;
  d.b_ne1 = top_k;
  d.in = hq;
  d.res = rdown;
  d.bias = bias_dn;
  d.comb = comb;
  return launch_gemv(down->wtype, false, d, max_active, st);
}

static FfnAct act_of(const msb_ffn_act_t *act) {
  FfnAct fa;
  if (act) {
    fa.kind = act->kind;
    fa.alpha = act->alpha;
    fa.limit = act->limit;
  }
  return fa;
}

extern "C" int msb_moe_ffn(msb_pool_t gate, msb_pool_t up, int64_t up_row0, msb_pool_t down,
                           const void *x_dev, int x_type, int64_t x_nb1, const msb_route_t *route,
                           const float *w_dev, int32_t top_k, int32_t n_tok, float *y_dev,
                           float *act_dev, void *workspace, int64_t workspace_bytes, void *stream) {
  return moe_ffn_core(gate, up, up_row0, down, x_dev, x_type, x_nb1, route, w_dev, top_k, n_tok,
                      y_dev, act_dev, workspace, workspace_bytes, nullptr, stream, FfnAct{},
                      nullptr);
}

extern "C" int msb_moe_ffn_act(msb_pool_t gate, msb_pool_t up, int64_t up_row0, msb_pool_t down,
                               const void *x_dev, int x_type, int64_t x_nb1,
                               const msb_route_t *route, const float *w_dev, int32_t top_k,
                               int32_t n_tok, float *y_dev, float *act_dev,
                               const msb_ffn_act_t *act, void *workspace,
                               int64_t workspace_bytes, void *stream) {
  return moe_ffn_core(gate, up, up_row0, down, x_dev, x_type, x_nb1, route, w_dev, top_k, n_tok,
                      y_dev, act_dev, workspace, workspace_bytes, nullptr, stream, act_of(act),
                      nullptr);
}

extern "C" int msb_moe_ffn_ex(msb_pool_t gate, msb_pool_t up, int64_t up_row0, msb_pool_t down,
                              const void *x_dev, int x_type, int64_t x_nb1,
                              const msb_route_t *route, const float *w_dev, int32_t top_k,
                              int32_t n_tok, float *y_dev, float *act_dev,
                              const msb_ffn_act_t *act, const msb_ffn_bias_t *bias,
                              int32_t accumulate, void *workspace, int64_t workspace_bytes,
                              void *stream) {
  return moe_ffn_core(gate, up, up_row0, down, x_dev, x_type, x_nb1, route, w_dev, top_k, n_tok,
                      y_dev, act_dev, workspace, workspace_bytes, nullptr, stream, act_of(act),
                      bias, accumulate != 0);
}

int msb::moe_ffn_to_rows(msb_pool_t gate, msb_pool_t up, int64_t up_row0, msb_pool_t down,
                         const void *x_dev, int x_type, int64_t x_nb1, const msb_route_t *route,
                         int32_t n_tok, const RowTarget &rows, void *workspace,
                         int64_t workspace_bytes, void *stream, const FfnAct &fa) {
  return moe_ffn_core(gate, up, up_row0, down, x_dev, x_type, x_nb1, route, nullptr, 1, n_tok,
                      nullptr, nullptr, workspace, workspace_bytes, &rows, stream, fa, nullptr);
}

// ---- mul_mat_id without allocation ------------------------------------------
// Some callers cannot call cudaMalloc at all: code that runs inside another
// runtime's allocator or memory-accounting hooks (where re-entering the
// allocator deadlocks or is forbidden), and hosts whose device memory is
// carved up in advance, where a late allocation fails under memory
// pressure. For them, msb_mul_mat_id_noalloc takes its workspace from the
// fixed device array below instead of from the caller.
//
// The array lives in this library's module: every GPU that loads the library
// holds kNoAllocScratchBytes of it until the process exits. Every call on a
// device shares it and finds the previous call's contents there; calls whose
// kernels overlap on the GPU (different streams, no ordering between them)
// race on it.
namespace {
constexpr int64_t kNoAllocScratchBytes = int64_t(8) << 20;   // 8 MiB
static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_noalloc_mu;
void *g_noalloc_ptr[kMaxDevices] = {};

// Device address of the array on `dev` (the current device). The host-side
// symbol is only a stand-in, so the address is looked up once per device
// with that device current; the first call on a device therefore does this
// set-up and should come before any stream capture on that device.
int noalloc_scratch(int dev, void **out) {
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  if (!g_noalloc_ptr[dev]) {
    void *p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess)
      return fail(MSB_ERR_CUDA, "msb_mul_mat_id_noalloc: cudaGetSymbolAddress failed on device %d: %s",
                  dev, cudaGetErrorString(e));
    g_noalloc_ptr[dev] = p;
  }
  *out = g_noalloc_ptr[dev];
  return MSB_OK;
}
}  // namespace

extern "C" int msb_mul_mat_id_noalloc(msb_pool_t pool, const void *b_dev, int b_type,
                                      int64_t b_ne1, int64_t b_nb1, int64_t b_nb2,
                                      const msb_route_t *route, int32_t top_k, int32_t n_tok,
                                      float *res_dev, void *stream) {
  MSB_CHECK_ARG(pool && route && res_dev, "msb_mul_mat_id_noalloc: null argument");
  MSB_CHECK_ARG(top_k > 0 && n_tok >= 0, "msb_mul_mat_id_noalloc: bad shape");
  const int64_t need = msb_workspace_bytes(pool->K, n_tok, top_k, pool->n_slot);
  MSB_CHECK_ARG(need >= 0 && need <= kNoAllocScratchBytes,
                "msb_mul_mat_id_noalloc: K=%lld with %d tokens x top-%d needs %lld workspace "
                "bytes, more than its fixed %lld-byte scratch; use msb_mul_mat_id with a "
                "caller-provided workspace",
                (long long)pool->K, n_tok, top_k, (long long)need,
                (long long)kNoAllocScratchBytes);
  int dev = -1;
  MSB_CUDA_TRY(cudaGetDevice(&dev));
  MSB_CHECK_ARG(dev >= 0 && dev < kMaxDevices, "msb_mul_mat_id_noalloc: device %d out of range",
                dev);
  MSB_CHECK_ARG(dev == pool->device,
                "msb_mul_mat_id_noalloc: current device %d is not the pool's device %d", dev,
                pool->device);
  void *scratch = nullptr;
  if (int rc = noalloc_scratch(dev, &scratch)) return rc;
  // Nothing in the workspace has to start at zero: every byte a call reads
  // is written earlier in the same call.
  return msb_mul_mat_id(pool, b_dev, b_type, b_ne1, b_nb1, b_nb2, route, top_k, n_tok, res_dev,
                        scratch, kNoAllocScratchBytes, stream);
}
