/*
 * msb_cpu_fast.c -- the CPU baseline of the MoE FFN path, vectorized.
 *
 * TEST INFRASTRUCTURE ONLY (like msb_oracle.c): bench.py times it as the
 * reference's CPU implementation of the path; tests check it against the
 * scalar oracle. The product never calls it.
 *
 * What it restates: ggml's CPU mul_mat_id for IQ4_NL / MXFP4 weights with
 * q8_0 activations -- the path the reference runs on the host
 * (research/spikes/s1_real_expert_stream/main.c:186-209 composes the FFN from
 * ggml_mul_mat_id calls; ggml itself is a third-party dependency that is not
 * vendored: llama.cpp b0539c43ed13b16bf0d8a0840646faea65469702, ggml
 * 78de606907c364b76601f734021f76bd29ca5637). ggml's published x86 scheme is
 * restated here in this file's own code:
 *   - activations quantized per 32-element block to int8 with d = amax/127
 *     (q8_0, the scale stored as fp16) -- orc_quantize_q8;
 *   - the 4-bit indices of a weight block mapped to int8 codebook values
 *     with a byte shuffle (IQ4_NL kvalues, or MXFP4's doubled e2m1 values);
 *   - int8 x int8 products summed to int32 lanes (VNNI dpbusd, or
 *     maddubs + madd on AVX2) with the sign moved onto the activations so
 *     the weight operand is unsigned;
 *   - the lanes converted to f32 and accumulated with the block's
 *     d_weight * d_act, one horizontal sum per output.
 * Experts are grouped by slot and every weight row is decoded once and dotted
 * with each of the slot's (token, k) rows, as ggml's mul_mat_id groups rows
 * by expert (up to 4 rows straight from the decoded block in registers, more
 * through a decoded copy of the row); threads take (slot, 32-row chunk)
 * items from a shared counter.
 * The f32 lane sums run in another order than the scalar oracle's block
 * order, so results agree with it to ~1e-6 relative, not bit for bit.
 */
#include <immintrin.h>
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define ORC_IQ4_NL 20
#define ORC_MXFP4 39

/* msb_oracle.c */
void orc_quantize_q8(const float *x, int64_t K, int8_t *q, float *d_out);
float orc_f16_to_f32(uint16_t h);
float orc_e8m0_half(uint8_t e);

static const int8_t KV_IQ4NL_F[16] = {-127, -104, -83, -65, -49, -35, -22, -10,
                                      1,    13,   25,  38,  53,  69,  89,  113};
static const int8_t KV_MXFP4_F[16] = {0, 1, 2, 3, 4, 6, 8, 12, 0, -1, -2, -3, -4, -6, -8, -12};

/* ---- instruction set ---------------------------------------------------- */
enum { ISA_SCALAR = 0, ISA_AVX2 = 1, ISA_VNNI = 2 };
static int g_isa = -1;

int orc_fast_isa(void) {
  if (g_isa < 0) {
    __builtin_cpu_init();
    if (__builtin_cpu_supports("avx512vnni") && __builtin_cpu_supports("avx512vl") &&
        __builtin_cpu_supports("avx512bw"))
      g_isa = ISA_VNNI;
    else if (__builtin_cpu_supports("avx2") && __builtin_cpu_supports("fma"))
      g_isa = ISA_AVX2;
    else
      g_isa = ISA_SCALAR;
  }
  return g_isa;
}

/* Forces an instruction set (tests compare them); -1 restores detection. */
void orc_fast_set_isa(int isa) {
  g_isa = -1;
  if (isa >= 0 && isa <= orc_fast_isa()) g_isa = isa;
}

/* ---- one weight row: decode and dot -------------------------------------- */
/* A block's scale without library calls: e8m0 as 2^(e - 128) built from its
 * bits (subnormal for e < 2), fp16 through the F16C conversion. */
static inline float e8m0_half_bits(uint8_t e) {
  const uint32_t bits = e >= 2 ? (uint32_t)(e - 1) << 23 : (e == 1 ? 0x00400000u : 0x00200000u);
  float f;
  memcpy(&f, &bits, 4);
  return f;
}
__attribute__((target("f16c"))) static inline float scale_of_block(int type, const uint8_t *blk) {
  if (type == ORC_IQ4_NL) {
    uint16_t h;
    memcpy(&h, blk, 2);
    return _cvtsh_ss(h);
  }
  return e8m0_half_bits(blk[0]);
}

/* Decodes one row of nb ggml blocks into int8 codebook values (element order)
 * and f32 block scales. */
static void decode_row_scalar(int type, const uint8_t *row, int64_t nb, int8_t *wq, float *ws) {
  const int bb = type == ORC_IQ4_NL ? 18 : 17;
  const int8_t *kv = type == ORC_IQ4_NL ? KV_IQ4NL_F : KV_MXFP4_F;
  for (int64_t b = 0; b < nb; ++b) {
    const uint8_t *blk = row + b * bb;
    const uint8_t *qs;
    if (type == ORC_IQ4_NL) {
      uint16_t h;
      memcpy(&h, blk, 2);
      ws[b] = orc_f16_to_f32(h);
      qs = blk + 2;
    } else {
      ws[b] = orc_e8m0_half(blk[0]);
      qs = blk + 1;
    }
    for (int i = 0; i < 16; ++i) {
      wq[b * 32 + i] = kv[qs[i] & 15];
      wq[b * 32 + 16 + i] = kv[qs[i] >> 4];
    }
  }
}

__attribute__((target("avx2,fma,f16c"))) static void decode_row_avx2(int type, const uint8_t *row,
                                                                 int64_t nb, int8_t *wq,
                                                                 float *ws) {
  const int bb = type == ORC_IQ4_NL ? 18 : 17;
  const int8_t *kv = type == ORC_IQ4_NL ? KV_IQ4NL_F : KV_MXFP4_F;
  const __m128i table = _mm_loadu_si128((const __m128i *)kv);
  const __m128i m4 = _mm_set1_epi8(0x0f);
  for (int64_t b = 0; b < nb; ++b) {
    const uint8_t *blk = row + b * bb;
    const uint8_t *qs;
    ws[b] = scale_of_block(type, blk);
    qs = blk + (type == ORC_IQ4_NL ? 2 : 1);
    const __m128i q = _mm_loadu_si128((const __m128i *)qs);
    const __m128i lo = _mm_shuffle_epi8(table, _mm_and_si128(q, m4));
    const __m128i hi = _mm_shuffle_epi8(table, _mm_and_si128(_mm_srli_epi16(q, 4), m4));
    _mm_storeu_si128((__m128i *)(wq + b * 32), lo);
    _mm_storeu_si128((__m128i *)(wq + b * 32 + 16), hi);
  }
}

static float dot_row_scalar(const int8_t *wq, const float *ws, const int8_t *aq, const float *ad,
                            int64_t nb) {
  float sumf = 0.f;
  for (int64_t b = 0; b < nb; ++b) {
    int32_t s = 0;
    for (int i = 0; i < 32; ++i) s += (int32_t)wq[b * 32 + i] * aq[b * 32 + i];
    sumf += ws[b] * ad[b] * (float)s;
  }
  return sumf;
}

__attribute__((target("avx2,fma,f16c"))) static inline float hsum8(__m256 v) {
  __m128 s = _mm_add_ps(_mm256_castps256_ps128(v), _mm256_extractf128_ps(v, 1));
  s = _mm_add_ps(s, _mm_movehl_ps(s, s));
  s = _mm_add_ss(s, _mm_movehdup_ps(s));
  return _mm_cvtss_f32(s);
}

__attribute__((target("avx2,fma"))) static float dot_row_avx2(const int8_t *wq, const float *ws,
                                                               const int8_t *aq, const float *ad,
                                                               int64_t nb) {
  const __m256i ones = _mm256_set1_epi16(1);
  __m256 acc0 = _mm256_setzero_ps(), acc1 = _mm256_setzero_ps();
  int64_t b = 0;
  for (; b + 1 < nb; b += 2) {
    const __m256i w0 = _mm256_loadu_si256((const __m256i *)(wq + b * 32));
    const __m256i a0 = _mm256_loadu_si256((const __m256i *)(aq + b * 32));
    const __m256i w1 = _mm256_loadu_si256((const __m256i *)(wq + b * 32 + 32));
    const __m256i a1 = _mm256_loadu_si256((const __m256i *)(aq + b * 32 + 32));
    const __m256i p0 = _mm256_madd_epi16(
        _mm256_maddubs_epi16(_mm256_sign_epi8(w0, w0), _mm256_sign_epi8(a0, w0)), ones);
    const __m256i p1 = _mm256_madd_epi16(
        _mm256_maddubs_epi16(_mm256_sign_epi8(w1, w1), _mm256_sign_epi8(a1, w1)), ones);
    acc0 = _mm256_fmadd_ps(_mm256_set1_ps(ws[b] * ad[b]), _mm256_cvtepi32_ps(p0), acc0);
    acc1 = _mm256_fmadd_ps(_mm256_set1_ps(ws[b + 1] * ad[b + 1]), _mm256_cvtepi32_ps(p1), acc1);
  }
  for (; b < nb; ++b) {
    const __m256i w0 = _mm256_loadu_si256((const __m256i *)(wq + b * 32));
    const __m256i a0 = _mm256_loadu_si256((const __m256i *)(aq + b * 32));
    const __m256i p0 = _mm256_madd_epi16(
        _mm256_maddubs_epi16(_mm256_sign_epi8(w0, w0), _mm256_sign_epi8(a0, w0)), ones);
    acc0 = _mm256_fmadd_ps(_mm256_set1_ps(ws[b] * ad[b]), _mm256_cvtepi32_ps(p0), acc0);
  }
  return hsum8(_mm256_add_ps(acc0, acc1));
}

__attribute__((target("avx2,fma,avx512f,avx512bw,avx512vl,avx512vnni"))) static float
dot_row_vnni(const int8_t *wq, const float *ws, const int8_t *aq, const float *ad, int64_t nb) {
  __m256 acc0 = _mm256_setzero_ps(), acc1 = _mm256_setzero_ps();
  const __m256i z = _mm256_setzero_si256();
  int64_t b = 0;
  for (; b + 1 < nb; b += 2) {
    const __m256i w0 = _mm256_loadu_si256((const __m256i *)(wq + b * 32));
    const __m256i a0 = _mm256_loadu_si256((const __m256i *)(aq + b * 32));
    const __m256i w1 = _mm256_loadu_si256((const __m256i *)(wq + b * 32 + 32));
    const __m256i a1 = _mm256_loadu_si256((const __m256i *)(aq + b * 32 + 32));
    const __m256i p0 = _mm256_dpbusd_epi32(z, _mm256_sign_epi8(w0, w0), _mm256_sign_epi8(a0, w0));
    const __m256i p1 = _mm256_dpbusd_epi32(z, _mm256_sign_epi8(w1, w1), _mm256_sign_epi8(a1, w1));
    acc0 = _mm256_fmadd_ps(_mm256_set1_ps(ws[b] * ad[b]), _mm256_cvtepi32_ps(p0), acc0);
    acc1 = _mm256_fmadd_ps(_mm256_set1_ps(ws[b + 1] * ad[b + 1]), _mm256_cvtepi32_ps(p1), acc1);
  }
  for (; b < nb; ++b) {
    const __m256i w0 = _mm256_loadu_si256((const __m256i *)(wq + b * 32));
    const __m256i a0 = _mm256_loadu_si256((const __m256i *)(aq + b * 32));
    const __m256i p0 = _mm256_dpbusd_epi32(z, _mm256_sign_epi8(w0, w0), _mm256_sign_epi8(a0, w0));
    acc0 = _mm256_fmadd_ps(_mm256_set1_ps(ws[b] * ad[b]), _mm256_cvtepi32_ps(p0), acc0);
  }
  return hsum8(_mm256_add_ps(acc0, acc1));
}

/* One weight row against up to 4 activation rows at once: every block is
 * decoded once (byte shuffle of its nibbles) and dotted with each row. */
#define FUSED_MAX 4
#define DEFINE_FUSED(NAME, TARGET, DOT32)                                                   \
  __attribute__((target(TARGET))) static inline void NAME##_p(                             \
      int type, const uint8_t *row, int64_t nb, const int8_t *const *aq,                     \
      const float *const *ad, int P, float *out) {                                          \
    const int bb = type == ORC_IQ4_NL ? 18 : 17, qo = type == ORC_IQ4_NL ? 2 : 1;           \
    const __m128i table =                                                                   \
        _mm_loadu_si128((const __m128i *)(type == ORC_IQ4_NL ? KV_IQ4NL_F : KV_MXFP4_F));   \
    const __m128i m4 = _mm_set1_epi8(0x0f);                                                 \
    __m256 acc[FUSED_MAX];                                                                  \
    for (int p = 0; p < FUSED_MAX; ++p) acc[p] = _mm256_setzero_ps();                       \
    for (int64_t b = 0; b < nb; ++b) {                                                      \
      const uint8_t *blk = row + b * bb;                                                    \
      const float dw = scale_of_block(type, blk);                                           \
      const __m128i q = _mm_loadu_si128((const __m128i *)(blk + qo));                       \
      const __m256i wv = _mm256_set_m128i(                                                  \
          _mm_shuffle_epi8(table, _mm_and_si128(_mm_srli_epi16(q, 4), m4)),                 \
          _mm_shuffle_epi8(table, _mm_and_si128(q, m4)));                                   \
      const __m256i wa = _mm256_sign_epi8(wv, wv);                                          \
      for (int p = 0; p < FUSED_MAX; ++p) {                                                 \
        if (p >= P) break;                                                                  \
        const __m256i av = _mm256_loadu_si256((const __m256i *)(aq[p] + b * 32));           \
        const __m256i prod = DOT32(wa, _mm256_sign_epi8(av, wv));                           \
        acc[p] = _mm256_fmadd_ps(_mm256_set1_ps(dw * ad[p][b]), _mm256_cvtepi32_ps(prod),   \
                                 acc[p]);                                                   \
      }                                                                                     \
    }                                                                                       \
    for (int p = 0; p < P; ++p) out[p] = hsum8(acc[p]);                                     \
  }

__attribute__((target("avx2,fma,f16c"))) static inline __m256i dot32_avx2(__m256i wa, __m256i as) {
  return _mm256_madd_epi16(_mm256_maddubs_epi16(wa, as), _mm256_set1_epi16(1));
}
__attribute__((target("avx2,fma,f16c,avx512f,avx512bw,avx512vl,avx512vnni"))) static inline __m256i
dot32_vnni(__m256i wa, __m256i as) {
  return _mm256_dpbusd_epi32(_mm256_setzero_si256(), wa, as);
}
DEFINE_FUSED(fused_avx2, "avx2,fma,f16c", dot32_avx2)
DEFINE_FUSED(fused_vnni, "avx2,fma,f16c,avx512f,avx512bw,avx512vl,avx512vnni", dot32_vnni)

/* Dots of one weight row (ggml bytes) with P activation rows (q8 codes and
 * scales), P <= FUSED_MAX, into out[0..P-1]; false when no vector unit. */
static int dot_rows_fused(int type, const uint8_t *row, int64_t nb, const int8_t *const *aq,
                          const float *const *ad, int P, float *out) {
  if (g_isa == ISA_VNNI) { fused_vnni_p(type, row, nb, aq, ad, P, out); return 1; }
  if (g_isa == ISA_AVX2) { fused_avx2_p(type, row, nb, aq, ad, P, out); return 1; }
  return 0;
}

static void decode_row(int type, const uint8_t *row, int64_t nb, int8_t *wq, float *ws) {
  if (g_isa >= ISA_AVX2) decode_row_avx2(type, row, nb, wq, ws);
  else decode_row_scalar(type, row, nb, wq, ws);
}

static float dot_row(const int8_t *wq, const float *ws, const int8_t *aq, const float *ad,
                     int64_t nb) {
  if (g_isa == ISA_VNNI) return dot_row_vnni(wq, ws, aq, ad, nb);
  if (g_isa == ISA_AVX2) return dot_row_avx2(wq, ws, aq, ad, nb);
  return dot_row_scalar(wq, ws, aq, ad, nb);
}

/* ---- the FFN, threaded ------------------------------------------------------ */
#define ROW_CHUNK 32

typedef struct {
  int type, act;
  float alpha, limit;
  const uint8_t *gate, *up, *down;
  int64_t gate_rows, up_rows, up_row0, K, n_ff, n_slots;
  const float *x, *w;
  int top_k, T;
  float *y;
  int64_t pairs;
  /* grouping: pairs of each slot, in pair order */
  int32_t *off, *list, *active;
  int n_active;
  /* work */
  int8_t *xq;
  float *xd;
  float *h;
  int8_t *hq;
  float *hd;
  float *r;
  int nthreads;
  pthread_barrier_t bar;
  volatile int64_t next[4];
} ffn_ctx;

static int64_t take(ffn_ctx *c, int phase) {
  return __atomic_fetch_add(&c->next[phase], 1, __ATOMIC_RELAXED);
}

static void *ffn_worker(void *arg) {
  ffn_ctx *c = (ffn_ctx *)arg;
  const int bb = c->type == ORC_IQ4_NL ? 18 : 17;
  const int64_t nb_in = c->K / 32, nb_ff = c->n_ff / 32;
  const int64_t nb_max = nb_in > nb_ff ? nb_in : nb_ff;
  int8_t *wq = (int8_t *)malloc((size_t)(nb_max * 32));
  int8_t *wq2 = (int8_t *)malloc((size_t)(nb_max * 32));
  float *ws = (float *)malloc(sizeof(float) * (size_t)nb_max);
  float *ws2 = (float *)malloc(sizeof(float) * (size_t)nb_max);
  /* phase 0: activations to q8 */
  for (int64_t t; (t = take(c, 0)) < c->T;)
    orc_quantize_q8(c->x + t * c->K, c->K, c->xq + t * c->K, c->xd + t * nb_in);
  pthread_barrier_wait(&c->bar);
  /* phase 1: gate and up rows of every active slot, then the activation */
  const int64_t row_in = nb_in * bb;
  const int64_t chunks_ff = (c->n_ff + ROW_CHUNK - 1) / ROW_CHUNK;
  for (int64_t it; (it = take(c, 1)) < c->n_active * chunks_ff;) {
    const int s = c->active[it / chunks_ff];
    const int64_t n0 = (it % chunks_ff) * ROW_CHUNK;
    const int64_t n1 = n0 + ROW_CHUNK < c->n_ff ? n0 + ROW_CHUNK : c->n_ff;
    const uint8_t *gs = c->gate + (int64_t)s * c->gate_rows * row_in;
    const uint8_t *us = c->up + (int64_t)s * c->up_rows * row_in;
    const int32_t j0 = c->off[s], j1 = c->off[s + 1];
    const int fused = j1 - j0 <= FUSED_MAX;
    const int8_t *aq[FUSED_MAX];
    const float *ad[FUSED_MAX];
    for (int32_t j = j0; j < j1 && j - j0 < FUSED_MAX; ++j) {
      const int64_t t = c->list[j] / c->top_k;
      aq[j - j0] = c->xq + t * c->K;
      ad[j - j0] = c->xd + t * nb_in;
    }
    for (int64_t n = n0; n < n1; ++n) {
      float gf[FUSED_MAX], uf[FUSED_MAX];
      const int use_fused =
          fused &&
          dot_rows_fused(c->type, gs + n * row_in, nb_in, aq, ad, (int)(j1 - j0), gf) &&
          dot_rows_fused(c->type, us + (c->up_row0 + n) * row_in, nb_in, aq, ad, (int)(j1 - j0),
                         uf);
      if (!use_fused) {
        decode_row(c->type, gs + n * row_in, nb_in, wq, ws);
        decode_row(c->type, us + (c->up_row0 + n) * row_in, nb_in, wq2, ws2);
      }
      for (int32_t j = j0; j < j1; ++j) {
        const int64_t p = c->list[j], t = p / c->top_k;
        const float g = use_fused ? gf[j - j0]
                                  : dot_row(wq, ws, c->xq + t * c->K, c->xd + t * nb_in, nb_in);
        const float u = use_fused ? uf[j - j0]
                                  : dot_row(wq2, ws2, c->xq + t * c->K, c->xd + t * nb_in, nb_in);
        float hv;
        if (c->act == 1) {
          const float xg = g < c->limit ? g : c->limit;
          const float yu = u < -c->limit ? -c->limit : (u > c->limit ? c->limit : u);
          hv = xg / (1.f + expf(-c->alpha * xg)) * (yu + 1.f);
        } else {
          hv = g / (1.f + expf(-g)) * u;
        }
        c->h[p * c->n_ff + n] = hv;
      }
    }
  }
  pthread_barrier_wait(&c->bar);
  /* phase 2: the activation rows to q8 */
  for (int64_t p; (p = take(c, 2)) < c->pairs;)
    orc_quantize_q8(c->h + p * c->n_ff, c->n_ff, c->hq + p * c->n_ff, c->hd + p * nb_ff);
  pthread_barrier_wait(&c->bar);
  /* phase 3: down rows */
  const int64_t row_ff = nb_ff * bb;
  const int64_t chunks_k = (c->K + ROW_CHUNK - 1) / ROW_CHUNK;
  for (int64_t it; (it = take(c, 3)) < c->n_active * chunks_k;) {
    const int s = c->active[it / chunks_k];
    const int64_t n0 = (it % chunks_k) * ROW_CHUNK;
    const int64_t n1 = n0 + ROW_CHUNK < c->K ? n0 + ROW_CHUNK : c->K;
    const uint8_t *ds = c->down + (int64_t)s * c->K * row_ff;
    const int32_t j0 = c->off[s], j1 = c->off[s + 1];
    const int8_t *aq[FUSED_MAX];
    const float *ad[FUSED_MAX];
    for (int32_t j = j0; j < j1 && j - j0 < FUSED_MAX; ++j) {
      aq[j - j0] = c->hq + (int64_t)c->list[j] * c->n_ff;
      ad[j - j0] = c->hd + (int64_t)c->list[j] * nb_ff;
    }
    for (int64_t n = n0; n < n1; ++n) {
      float rf[FUSED_MAX];
      if (j1 - j0 <= FUSED_MAX &&
          dot_rows_fused(c->type, ds + n * row_ff, nb_ff, aq, ad, (int)(j1 - j0), rf)) {
        for (int32_t j = j0; j < j1; ++j) c->r[(int64_t)c->list[j] * c->K + n] = rf[j - j0];
        continue;
      }
      decode_row(c->type, ds + n * row_ff, nb_ff, wq, ws);
      for (int32_t j = j0; j < j1; ++j) {
        const int64_t p = c->list[j];
        c->r[p * c->K + n] = dot_row(wq, ws, c->hq + p * c->n_ff, c->hd + p * nb_ff, nb_ff);
      }
    }
  }
  free(wq);
  free(wq2);
  free(ws);
  free(ws2);
  return NULL;
}

/* The MoE FFN of orc_moe_ffn in its q8 form (same arguments and meaning; the
 * slot ids must be < n_slots), vectorized and threaded. y[t] = sum_k w[t][k] *
 * r[t][k] in k order. Returns 0, or -1 for bad shapes. */
int orc_moe_ffn_fast(int type, const uint8_t *gate, int64_t gate_rows, const uint8_t *up,
                     int64_t up_rows, int64_t up_row0, const uint8_t *down, int64_t K,
                     int64_t n_ff, int64_t n_slots, const float *x, const int32_t *ids,
                     const float *w, int top_k, int T, int act, float alpha, float limit, float *y,
                     int nthreads) {
  if ((type != ORC_IQ4_NL && type != ORC_MXFP4) || K % 32 || n_ff % 32 || top_k <= 0 || T < 0)
    return -1;
  orc_fast_isa();
  const int64_t pairs = (int64_t)T * top_k;
  for (int64_t p = 0; p < pairs; ++p)
    if (ids[p] < 0 || ids[p] >= n_slots) return -2;
  ffn_ctx c;
  memset(&c, 0, sizeof(c));
  c.type = type;
  c.act = act;
  c.alpha = alpha;
  c.limit = limit;
  c.gate = gate;
  c.up = up;
  c.down = down;
  c.gate_rows = gate_rows;
  c.up_rows = up_rows;
  c.up_row0 = up_row0;
  c.K = K;
  c.n_ff = n_ff;
  c.n_slots = n_slots;
  c.x = x;
  c.w = w;
  c.top_k = top_k;
  c.T = T;
  c.y = y;
  c.pairs = pairs;
  /* group pairs by slot (counting sort, pair order within a slot) */
  c.off = (int32_t *)calloc((size_t)(n_slots + 1), sizeof(int32_t));
  c.list = (int32_t *)malloc(sizeof(int32_t) * (size_t)(pairs > 0 ? pairs : 1));
  c.active = (int32_t *)malloc(sizeof(int32_t) * (size_t)n_slots);
  for (int64_t p = 0; p < pairs; ++p) c.off[ids[p] + 1]++;
  for (int64_t s = 0; s < n_slots; ++s) {
    if (c.off[s + 1] > 0) c.active[c.n_active++] = (int32_t)s;
    c.off[s + 1] += c.off[s];
  }
  int32_t *fillp = (int32_t *)malloc(sizeof(int32_t) * (size_t)n_slots);
  memcpy(fillp, c.off, sizeof(int32_t) * (size_t)n_slots);
  for (int64_t p = 0; p < pairs; ++p) c.list[fillp[ids[p]]++] = (int32_t)p;
  free(fillp);
  c.xq = (int8_t *)malloc((size_t)(T * K + 1));
  c.xd = (float *)malloc(sizeof(float) * (size_t)(T * (K / 32) + 1));
  c.h = (float *)malloc(sizeof(float) * (size_t)(pairs * n_ff + 1));
  c.hq = (int8_t *)malloc((size_t)(pairs * n_ff + 1));
  c.hd = (float *)malloc(sizeof(float) * (size_t)(pairs * (n_ff / 32) + 1));
  c.r = (float *)malloc(sizeof(float) * (size_t)(pairs * K + 1));
  if (nthreads < 1) nthreads = 1;
  c.nthreads = nthreads;
  pthread_barrier_init(&c.bar, NULL, (unsigned)nthreads);
  pthread_t *th = (pthread_t *)malloc(sizeof(pthread_t) * (size_t)nthreads);
  for (int i = 1; i < nthreads; ++i) pthread_create(&th[i], NULL, ffn_worker, &c);
  ffn_worker(&c);
  for (int i = 1; i < nthreads; ++i) pthread_join(th[i], NULL);
  pthread_barrier_destroy(&c.bar);
  free(th);
  for (int64_t t = 0; t < T; ++t)
    for (int64_t n = 0; n < K; ++n) {
      double s = 0.0;
      for (int k = 0; k < top_k; ++k)
        s += (double)w[t * top_k + k] * (double)c.r[(t * top_k + k) * K + n];
      y[t * K + n] = (float)s;
    }
  free(c.off);
  free(c.list);
  free(c.active);
  free(c.xq);
  free(c.xd);
  free(c.h);
  free(c.hq);
  free(c.hd);
  free(c.r);
  return 0;
}
