/*
 * msb_oracle.c -- CPU oracle for the expert-indexed matmul path.
 *
 * TEST INFRASTRUCTURE ONLY. Only tests/, __graft_entry__.smoke() and
 * bench.py's CPU-baseline leg may load this library, and only as the checker
 * (or the timed CPU baseline); the product path never calls it.
 *
 * What it restates, and from where:
 *   - block formats IQ4_NL and MXFP4 and their dequantization: ggml's block
 *     layout as published by its Python codec gguf 0.19.0
 *     (gguf/quants.py:656-704 MXFP4, :1330-1349 IQ4_NL; block sizes
 *     gguf/constants.py:4251,4264). ggml itself is a third-party dependency of
 *     the reference that is not vendored (pins: llama.cpp
 *     b0539c43ed13b16bf0d8a0840646faea65469702, Dockerfile:4; ggml
 *     78de606907c364b76601f734021f76bd29ca5637,
 *     research/docker/Dockerfile.dev:10).
 *   - MXFP4 quantization: gguf/quants.py:669-687 (e = floor(log2 amax) - 2 +
 *     127, nearest doubled-e2m1 code, first index on ties). floor(log2) is
 *     taken exactly from the float's exponent.
 *   - IQ4_NL quantization: this project's own deterministic scale search (gguf
 *     has no IQ4_NL quantizer); bit-identical to the device quantizer.
 *   - mul_mat_id: the operator contract of ggml_mul_mat_id as the reference
 *     calls it (research/spikes/s0_slot_slab/main.c:81-95 reference_matmul,
 *     :117-148; research/spikes/s6_arena_mulmatid/main.c:82-134):
 *       res[t][k][n] = sum_i W[slot(k,t)][n][i] * b[t][k % b_ne1][i]
 *     in two modes: "exact" (f64 accumulation of dequantized weights) and
 *     "q8" (ggml's CPU vec_dot form: activations quantized per 32-block to
 *     int8 with d = amax/127 stored as fp16, int32 dot per block, f32
 *     accumulation of d_w * d_a * isum in block order).
 *     A third mode, "e2m1x4", is the activation form of this library's
 *     tensor-core path for MXFP4: each 32-element block of activations is
 *     split into 4 terms, each 32 e2m1 codes with a power-of-two scale; the
 *     sum of the terms replaces the activations, and the products accumulate
 *     in f64. A fourth, "f16", is the form of the IQ4_NL tensor-core path:
 *     every weight d * kv and every activation rounded to fp16 (round to
 *     nearest even), products accumulated in f64.
 *   - MoE FFN: research/spikes/s1_real_expert_stream/main.c:186-209 and
 *     research/spikes/s4_sweep_math/main.c:89-92 (SwiGLU, then down, then the
 *     router-weighted sum over k).
 *
 * Parity pins: dequantization and MXFP4 quantization are checked against
 * golden vectors produced by gguf (tests/golden/make_golden.py). The matmul
 * arithmetic of ggml itself is not available here, so mul_mat_id parity is
 * pinned only through the properties the reference's spikes assert
 * (bit-identity under slot permutation, exact zero from the zero slot,
 * additivity of split expert sets) plus the exact-mode oracle.
 *
 * Build: oracle/Makefile (no floating-point contraction, so every product
 * and difference rounds as written).
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define ORC_IQ4_NL 20
#define ORC_MXFP4 39

static const int8_t KV_IQ4NL[16] = {-127, -104, -83, -65, -49, -35, -22, -10,
                                    1,    13,   25,  38,  53,  69,  89,  113};
static const int8_t KV_MXFP4[16] = {0, 1, 2, 3, 4, 6, 8, 12,
                                    0, -1, -2, -3, -4, -6, -8, -12};

/* ---- fp16 <-> f32 (IEEE binary16, round to nearest even) -------------- */
float orc_f16_to_f32(uint16_t h) {
  const uint32_t sign = (uint32_t)(h >> 15) << 31;
  const uint32_t exp = (h >> 10) & 0x1f, man = h & 0x3ff;
  uint32_t bits;
  if (exp == 0) {
    if (man == 0) {
      bits = sign;
    } else { /* subnormal: normalise */
      int e = -1;
      uint32_t m = man;
      do { m <<= 1; e++; } while (!(m & 0x400));
      bits = sign | ((uint32_t)(127 - 15 - e) << 23) | ((m & 0x3ff) << 13);
    }
  } else if (exp == 31) {
    bits = sign | 0x7f800000u | (man << 13);
  } else {
    bits = sign | ((exp - 15 + 127) << 23) | (man << 13);
  }
  float f;
  memcpy(&f, &bits, 4);
  return f;
}

uint16_t orc_f32_to_f16(float f) {
  uint32_t x;
  memcpy(&x, &f, 4);
  const uint16_t sign = (uint16_t)((x >> 16) & 0x8000);
  const uint32_t ax = x & 0x7fffffffu;
  if (ax >= 0x7f800000u) /* inf or nan */
    return sign | 0x7c00 | (ax > 0x7f800000u ? 0x200 : 0);
  if (ax >= 0x477ff000u) return sign | 0x7c00; /* rounds to >= 65520: inf */
  if (ax < 0x38800000u) {                      /* below fp16 normal range */
    if (ax < 0x33000000u) return sign;         /* < 2^-25 rounds to 0 */
    const uint32_t e = ax >> 23, m = (ax & 0x7fffff) | 0x800000;
    const int s = 126 - (int)e; /* 14..24 mantissa bits dropped */
    uint32_t q = m >> s;
    const uint32_t rem = m & ((1u << s) - 1), half = 1u << (s - 1);
    if (rem > half || (rem == half && (q & 1))) q++;
    return sign | (uint16_t)q;
  }
  uint32_t q = ax - 0x38000000u; /* rebias exponent 127 -> 15 */
  const uint32_t rem = q & 0x1fff;
  q >>= 13;
  if (rem > 0x1000 || (rem == 0x1000 && (q & 1))) q++;
  return sign | (uint16_t)q;
}

/* 2^(e-128): ggml's "e8m0 to fp32 half". */
float orc_e8m0_half(uint8_t e) { return ldexpf(1.0f, (int)e - 128); }

/* ---- dequantization ---------------------------------------------------- */
static int block_bytes(int type) {
  return type == ORC_IQ4_NL ? 18 : type == ORC_MXFP4 ? 17 : -1;
}

int orc_block_bytes(int type) { return block_bytes(type); }

/* One row of K elements (K/32 blocks) from ggml bytes. */
int orc_dequant_row(int type, const uint8_t *src, float *dst, int64_t K) {
  if (K % 32 || block_bytes(type) < 0) return -1;
  for (int64_t b = 0; b < K / 32; ++b) {
    const uint8_t *blk = src + b * block_bytes(type);
    float d;
    const uint8_t *qs;
    const int8_t *kv;
    if (type == ORC_IQ4_NL) {
      uint16_t h;
      memcpy(&h, blk, 2);
      d = orc_f16_to_f32(h);
      qs = blk + 2;
      kv = KV_IQ4NL;
    } else {
      d = orc_e8m0_half(blk[0]);
      qs = blk + 1;
      kv = KV_MXFP4;
    }
    for (int j = 0; j < 16; ++j) {
      dst[b * 32 + j] = d * (float)kv[qs[j] & 15];
      dst[b * 32 + j + 16] = d * (float)kv[qs[j] >> 4];
    }
  }
  return 0;
}

/* ---- quantization ------------------------------------------------------ */
static int nearest_code(float x, float d, const int8_t *kv) {
  int best = 0;
  float best_err = fabsf(d * (float)kv[0] - x);
  for (int i = 1; i < 16; ++i) {
    const float err = fabsf(d * (float)kv[i] - x);
    if (err < best_err) {
      best_err = err;
      best = i;
    }
  }
  return best;
}

static void quantize_block_mxfp4(const float *x, uint8_t *o) {
  float amax = 0.f;
  for (int j = 0; j < 32; ++j) amax = fmaxf(amax, fabsf(x[j]));
  uint8_t e = 0;
  if (amax > 0.f) {
    int ex;
    frexpf(amax, &ex);
    e = (uint8_t)((ex - 1) - 2 + 127);
  }
  const float d = orc_e8m0_half(e);
  o[0] = e;
  for (int j = 0; j < 16; ++j)
    o[1 + j] = (uint8_t)(nearest_code(x[j], d, KV_MXFP4) |
                         (nearest_code(x[j + 16], d, KV_MXFP4) << 4));
}

static float iq4nl_sse(const float *x, float d, uint8_t *idx) {
  float sse = 0.f;
  for (int j = 0; j < 32; ++j) {
    idx[j] = (uint8_t)nearest_code(x[j], d, KV_IQ4NL);
    const float r = x[j] - d * (float)KV_IQ4NL[idx[j]];
    sse = sse + r * r;
  }
  return sse;
}

static void quantize_block_iq4nl(const float *x, uint8_t *o) {
  float amax = 0.f, vmax = 0.f;
  for (int j = 0; j < 32; ++j) {
    const float a = fabsf(x[j]);
    if (a > amax) {
      amax = a;
      vmax = x[j];
    }
  }
  uint8_t idx[32], idx1[32];
  float d;
  if (amax == 0.f) {
    d = 0.f;
    for (int j = 0; j < 32; ++j) idx[j] = 8;
  } else {
    d = orc_f16_to_f32(orc_f32_to_f16(vmax / -127.f));
    const float sse0 = iq4nl_sse(x, d, idx);
    float sxl = 0.f, sll = 0.f;
    for (int j = 0; j < 32; ++j) {
      const float l = (float)KV_IQ4NL[idx[j]];
      sxl = sxl + x[j] * l;
      sll = sll + l * l;
    }
    const float d1 = orc_f16_to_f32(orc_f32_to_f16(sxl / sll));
    const float sse1 = iq4nl_sse(x, d1, idx1);
    if (sse1 < sse0) {
      d = d1;
      memcpy(idx, idx1, 32);
    }
  }
  const uint16_t h = orc_f32_to_f16(d);
  memcpy(o, &h, 2);
  for (int j = 0; j < 16; ++j) o[2 + j] = (uint8_t)(idx[j] | (idx[j + 16] << 4));
}

int orc_quantize_rows(int type, const float *src, int64_t n_rows, int64_t K, uint8_t *dst) {
  if (K % 32 || block_bytes(type) < 0) return -1;
  const int64_t nblk = n_rows * (K / 32);
  for (int64_t b = 0; b < nblk; ++b) {
    if (type == ORC_MXFP4) quantize_block_mxfp4(src + b * 32, dst + b * 17);
    else quantize_block_iq4nl(src + b * 32, dst + b * 18);
  }
  return 0;
}

/* ggml's q8_0 form: d = amax/127, codes round(x * (1/d)) half away from zero,
 * d kept as fp16. */
void orc_quantize_q8(const float *x, int64_t K, int8_t *q, float *d_out) {
  for (int64_t b = 0; b < K / 32; ++b) {
    float amax = 0.f;
    for (int j = 0; j < 32; ++j) amax = fmaxf(amax, fabsf(x[b * 32 + j]));
    const float d = amax / 127.f;
    const float id = d != 0.f ? 1.f / d : 0.f;
    for (int j = 0; j < 32; ++j) q[b * 32 + j] = (int8_t)roundf(x[b * 32 + j] * id);
    d_out[b] = orc_f16_to_f32(orc_f32_to_f16(d));
  }
}

/* ---- e2m1 activation terms (tensor-core form) -------------------------- */
static const float E2M1_MAG[8] = {0.f, 0.5f, 1.f, 1.5f, 2.f, 3.f, 4.f, 6.f};

/* Nearest e2m1 magnitude code of v in [0, 6], ties upward. */
static int e2m1_code(float v) {
  return (v >= 0.25f) + (v >= 0.75f) + (v >= 1.25f) + (v >= 1.75f) + (v >= 2.5f) +
         (v >= 3.5f) + (v >= 5.f);
}

/* Splits each 32-element block of x (n elements) into `terms` e2m1 terms: per
 * term, k = the smallest integer with max|r| <= 6 * 2^k (r the remaining
 * residual; k taken exactly from the float's exponent), codes = nearest e2m1
 * of |r| / 2^k with r's sign, r -= code * 2^k (exact). A term whose k would
 * fall below -126 is skipped (contributes 0). Writes the sum of the terms to
 * approx, and optionally the codes (nibbles, sign in bit 3) and the scale
 * bytes k + 127 per (term, block). */
void orc_e2m1_split(const float *x, int64_t n, int terms, float *approx,
                    uint8_t *codes, uint8_t *exps) {
  const int64_t nb = n / 32;
  for (int64_t b = 0; b < nb; ++b) {
    float r[32];
    for (int j = 0; j < 32; ++j) r[j] = x[b * 32 + j];
    for (int t = 0; t < terms; ++t) {
      float amax = 0.f;
      for (int j = 0; j < 32; ++j) amax = fmaxf(amax, fabsf(r[j]));
      int k = -127;
      if (amax > 0.f) {
        int ex;
        const float m = frexpf(amax, &ex);
        k = m > 0.75f ? ex - 2 : ex - 3;
      }
      const int skip = k < -126;
      if (exps) exps[t * nb + b] = skip ? 0 : (uint8_t)(k > 127 ? 254 : k + 127);
      for (int j = 0; j < 32; ++j) {
        int code = 0, neg = 0;
        if (!skip) {
          const float v = fabsf(r[j]) * ldexpf(1.f, -k);
          code = e2m1_code(v);
          neg = r[j] < 0.f && code > 0;
          const float q = ldexpf(E2M1_MAG[code], k);
          r[j] = neg ? r[j] + q : r[j] - q;
        }
        if (codes) codes[(t * nb + b) * 32 + j] = (uint8_t)(code | (neg << 3));
      }
    }
    for (int j = 0; j < 32; ++j) approx[b * 32 + j] = x[b * 32 + j] - r[j];
  }
}

/* ---- mul_mat_id -------------------------------------------------------- */
typedef struct {
  int type, mode;
  const uint8_t *as;
  int64_t K, N, slot_bytes;
  const float *b;
  int64_t b_ne1;
  const int32_t *ids;
  int top_k, T;
  float *res;
  int64_t lo, hi; /* range of (pair, n) items */
  const int8_t *bq; /* q8 mode: quantized activations [T*b_ne1][K] */
  const float *bd;  /*           scales [T*b_ne1][K/32]               */
  const float *bx;  /* e2m1x4 mode: activations as the sum of 4 terms  */
} mm_job;

static void *mm_worker(void *arg) {
  mm_job *j = (mm_job *)arg;
  const int64_t nb = j->K / 32, bb = block_bytes(j->type);
  float *wrow = (float *)malloc(sizeof(float) * j->K);
  for (int64_t it = j->lo; it < j->hi; ++it) {
    const int64_t pair = it / j->N, n = it % j->N;
    const int64_t t = pair / j->top_k, k = pair % j->top_k;
    const int32_t slot = j->ids[pair];
    const uint8_t *row = j->as + slot * j->slot_bytes + n * nb * bb;
    const int64_t arow = t * j->b_ne1 + (k % j->b_ne1);
    if (j->mode == 0 || j->mode == 2 || j->mode == 3) {
      orc_dequant_row(j->type, row, wrow, j->K);
      if (j->mode == 3) /* f16 form: each weight d * kv rounded once to fp16 */
        for (int64_t i = 0; i < j->K; ++i) wrow[i] = orc_f16_to_f32(orc_f32_to_f16(wrow[i]));
      const float *a = (j->mode == 2 || j->mode == 3 ? j->bx : j->b) + arow * j->K;
      double s = 0.0;
      for (int64_t i = 0; i < j->K; ++i) s += (double)wrow[i] * (double)a[i];
      j->res[pair * j->N + n] = (float)s;
    } else {
      const int8_t *aq = j->bq + arow * j->K;
      const float *ad = j->bd + arow * nb;
      float sumf = 0.f;
      for (int64_t b = 0; b < nb; ++b) {
        const uint8_t *blk = row + b * bb;
        float dw;
        const uint8_t *qs;
        const int8_t *kv;
        if (j->type == ORC_IQ4_NL) {
          uint16_t h;
          memcpy(&h, blk, 2);
          dw = orc_f16_to_f32(h);
          qs = blk + 2;
          kv = KV_IQ4NL;
        } else {
          dw = orc_e8m0_half(blk[0]);
          qs = blk + 1;
          kv = KV_MXFP4;
        }
        int32_t isum = 0;
        for (int i = 0; i < 16; ++i) {
          isum += (int32_t)kv[qs[i] & 15] * aq[b * 32 + i];
          isum += (int32_t)kv[qs[i] >> 4] * aq[b * 32 + i + 16];
        }
        sumf += dw * ad[b] * (float)isum;
      }
      j->res[pair * j->N + n] = sumf;
    }
  }
  free(wrow);
  return NULL;
}

/* as: [n_slots][N][K/32 blocks] ggml bytes; b: f32 [T][b_ne1][K];
 * ids: slot ids [T][top_k]; res: f32 [T][top_k][N]. mode 0 exact, 1 q8, 2 e2m1x4,
 * 3 f16. */
int orc_mul_mat_id(int type, const uint8_t *as, int64_t K, int64_t N, int64_t n_slots,
                   const float *b, int64_t b_ne1, const int32_t *ids, int top_k, int T,
                   int mode, float *res, int nthreads) {
  if (K % 32 || block_bytes(type) < 0 || top_k <= 0 || T < 0) return -1;
  if (b_ne1 != 1 && b_ne1 != top_k) return -1;
  for (int64_t p = 0; p < (int64_t)T * top_k; ++p)
    if (ids[p] < 0 || ids[p] >= n_slots) return -2;
  const int64_t slot_bytes = N * (K / 32) * block_bytes(type);
  int8_t *bq = NULL;
  float *bd = NULL;
  const int64_t rows = (int64_t)T * b_ne1;
  float *bx = NULL;
  if (mode == 1) {
    bq = (int8_t *)malloc((size_t)(rows * K));
    bd = (float *)malloc(sizeof(float) * (size_t)(rows * (K / 32)));
    for (int64_t r = 0; r < rows; ++r) orc_quantize_q8(b + r * K, K, bq + r * K, bd + r * (K / 32));
  } else if (mode == 2) {
    bx = (float *)malloc(sizeof(float) * (size_t)(rows * K));
    for (int64_t r = 0; r < rows; ++r) orc_e2m1_split(b + r * K, K, 4, bx + r * K, NULL, NULL);
  } else if (mode == 3) {
    bx = (float *)malloc(sizeof(float) * (size_t)(rows * K));
    for (int64_t i = 0; i < rows * K; ++i) bx[i] = orc_f16_to_f32(orc_f32_to_f16(b[i]));
  }
  if (nthreads < 1) nthreads = 1;
  const int64_t items = (int64_t)T * top_k * N;
  if (nthreads > items) nthreads = items > 0 ? (int)items : 1;
  pthread_t *th = (pthread_t *)malloc(sizeof(pthread_t) * nthreads);
  mm_job *jobs = (mm_job *)malloc(sizeof(mm_job) * nthreads);
  for (int i = 0; i < nthreads; ++i) {
    mm_job j = {type, mode, as, K, N, slot_bytes, b, b_ne1, ids, top_k, T, res,
                items * i / nthreads, items * (i + 1) / nthreads, bq, bd, bx};
    jobs[i] = j;
    if (nthreads == 1) mm_worker(&jobs[i]);
    else pthread_create(&th[i], NULL, mm_worker, &jobs[i]);
  }
  if (nthreads > 1)
    for (int i = 0; i < nthreads; ++i) pthread_join(th[i], NULL);
  free(th);
  free(jobs);
  free(bq);
  free(bd);
  free(bx);
  return 0;
}

/* MoE FFN over slot ids: h = silu(gate(x)) * up(x) per (t, k) (act 1: the
 * gpt-oss clamped form with alpha and limit), r = down(h),
 * y[t] = sum_k w[t][k] * r[t][k]. gate/up/down: [n_slots][rows][K/32] ggml
 * bytes; up rows start at up_row0 within up (fused gate_up tensors).
 * In q8 mode h is re-quantized before the down projection, as the device
 * path does. x: f32 [T][K]; w: f32 [T][top_k]; y: f32 [T][K]. */
/* Expert biases (gpt-oss; llama.cpp adds them with add_id over the router's
 * expert ids): gate_b / up_b / down_b are f32 rows [n_expert][ld], expert e's
 * row at +e*ld (NULL: none), looked up by eids[t][k] (the expert id of the
 * pair, before the remap); added to the f32 matmul result of every pair not
 * routed to the zero slot (slot n_slots - 1), before the activation (gate,
 * up) or the weighting (down). Ids outside [0, n_expert) add nothing. */
typedef struct {
  const float *gate_b, *up_b, *down_b;
  int64_t gate_ld, up_ld, down_ld;
  const int32_t *eids;
  int n_expert;
} orc_bias;

static void add_bias(float *res, int64_t pairs, int64_t n, const float *b, int64_t ld,
                     const int32_t *eids, int n_expert, const int32_t *ids, int64_t zero_slot) {
  if (!b) return;
  for (int64_t p = 0; p < pairs; ++p) {
    const int32_t e = eids[p];
    if (ids[p] == zero_slot || e < 0 || e >= n_expert) continue;
    for (int64_t i = 0; i < n; ++i) res[p * n + i] += b[(int64_t)e * ld + i];
  }
}

static int moe_ffn_impl(int type, const uint8_t *gate, int64_t gate_rows, const uint8_t *up,
                        int64_t up_rows, int64_t up_row0, const uint8_t *down, int64_t K,
                        int64_t n_ff, int64_t n_slots, const float *x, const int32_t *ids,
                        const float *w, int top_k, int T, int mode, int act, float alpha,
                        float limit, float *y, float *h_out, int nthreads, const orc_bias *bias);

int orc_moe_ffn(int type, const uint8_t *gate, int64_t gate_rows, const uint8_t *up,
                int64_t up_rows, int64_t up_row0, const uint8_t *down, int64_t K, int64_t n_ff,
                int64_t n_slots, const float *x, const int32_t *ids, const float *w, int top_k,
                int T, int mode, int act, float alpha, float limit, float *y, float *h_out,
                int nthreads) {
  return moe_ffn_impl(type, gate, gate_rows, up, up_rows, up_row0, down, K, n_ff, n_slots, x, ids,
                      w, top_k, T, mode, act, alpha, limit, y, h_out, nthreads, NULL);
}

int orc_moe_ffn_bias(int type, const uint8_t *gate, int64_t gate_rows, const uint8_t *up,
                     int64_t up_rows, int64_t up_row0, const uint8_t *down, int64_t K,
                     int64_t n_ff, int64_t n_slots, const float *x, const int32_t *ids,
                     const float *w, int top_k, int T, int mode, int act, float alpha,
                     float limit, float *y, float *h_out, int nthreads, const float *gate_b,
                     const float *up_b, const float *down_b, int64_t gate_ld, int64_t up_ld,
                     int64_t down_ld, const int32_t *eids, int n_expert) {
  const orc_bias b = {gate_b, up_b, down_b, gate_ld, up_ld, down_ld, eids, n_expert};
  return moe_ffn_impl(type, gate, gate_rows, up, up_rows, up_row0, down, K, n_ff, n_slots, x, ids,
                      w, top_k, T, mode, act, alpha, limit, y, h_out, nthreads, &b);
}

static int moe_ffn_impl(int type, const uint8_t *gate, int64_t gate_rows, const uint8_t *up,
                        int64_t up_rows, int64_t up_row0, const uint8_t *down, int64_t K,
                        int64_t n_ff, int64_t n_slots, const float *x, const int32_t *ids,
                        const float *w, int top_k, int T, int mode, int act, float alpha,
                        float limit, float *y, float *h_out, int nthreads, const orc_bias *bias) {
  const int64_t pairs = (int64_t)T * top_k;
  const int64_t bb = block_bytes(type);
  if (bb < 0 || K % 32 || n_ff % 32) return -1;
  float *g = (float *)malloc(sizeof(float) * (size_t)(pairs * n_ff));
  float *u = (float *)malloc(sizeof(float) * (size_t)(pairs * n_ff));
  float *r = (float *)malloc(sizeof(float) * (size_t)(pairs * K));
  /* Views of n_ff rows per slot: gate rows [0, n_ff) of a slot of gate_rows
   * rows, up rows [up_row0, up_row0 + n_ff) of a slot of up_rows rows. */
  const int64_t row_bytes = (K / 32) * bb, view = n_ff * row_bytes;
  uint8_t *gv = (uint8_t *)malloc((size_t)(n_slots * view));
  uint8_t *uv = (uint8_t *)malloc((size_t)(n_slots * view));
  for (int64_t s = 0; s < n_slots; ++s) {
    memcpy(gv + s * view, gate + s * gate_rows * row_bytes, (size_t)view);
    memcpy(uv + s * view, up + s * up_rows * row_bytes + up_row0 * row_bytes, (size_t)view);
  }
  int rc = orc_mul_mat_id(type, gv, K, n_ff, n_slots, x, 1, ids, top_k, T, mode, g, nthreads);
  if (!rc) rc = orc_mul_mat_id(type, uv, K, n_ff, n_slots, x, 1, ids, top_k, T, mode, u, nthreads);
  free(gv);
  free(uv);
  if (!rc && bias) {
    add_bias(g, pairs, n_ff, bias->gate_b, bias->gate_ld, bias->eids, bias->n_expert, ids,
             n_slots - 1);
    add_bias(u, pairs, n_ff, bias->up_b, bias->up_ld, bias->eids, bias->n_expert, ids,
             n_slots - 1);
  }
  if (!rc) {
    float *h = (float *)malloc(sizeof(float) * (size_t)(pairs * n_ff));
    for (int64_t i = 0; i < pairs * n_ff; ++i) {
      if (act == 1) {
        /* gpt-oss: gate clamped above, up clamped both ways and shifted by
         * one, sigmoid with slope alpha (llama.cpp's swiglu_oai). */
        const float xg = g[i] < limit ? g[i] : limit;
        const float yu = u[i] < -limit ? -limit : (u[i] > limit ? limit : u[i]);
        h[i] = xg / (1.f + expf(-alpha * xg)) * (yu + 1.f);
      } else {
        h[i] = g[i] / (1.f + expf(-g[i])) * u[i];
      }
    }
    /* rows of the zero slot are exactly 0 before the down projection */
    if (bias)
      for (int64_t p = 0; p < pairs; ++p)
        if (ids[p] == n_slots - 1)
          for (int64_t i = 0; i < n_ff; ++i) h[p * n_ff + i] = 0.f;
    if (h_out) memcpy(h_out, h, sizeof(float) * (size_t)(pairs * n_ff));
    rc = orc_mul_mat_id(type, down, n_ff, K, n_slots, h, top_k, ids, top_k, T, mode, r, nthreads);
    if (!rc && bias)
      add_bias(r, pairs, K, bias->down_b, bias->down_ld, bias->eids, bias->n_expert, ids,
               n_slots - 1);
    free(h);
  }
  if (!rc) {
    for (int64_t t = 0; t < T; ++t)
      for (int64_t n = 0; n < K; ++n) {
        double s = 0.0;
        for (int k = 0; k < top_k; ++k)
          s += (double)w[t * top_k + k] * (double)r[(t * top_k + k) * K + n];
        y[t * K + n] = (float)s;
      }
  }
  free(g);
  free(u);
  free(r);
  return rc;
}
