/*
 * wg_gen.c — seeded synthetic Whisper decoder models and encoder outputs,
 * quantised with a restatement of the reference quantiser.
 *
 * No Whisper checkpoint exists in the reference tree (models/ holds only
 * tokenizer JSON), so every benchmark and parity run uses models made here:
 *   linear weights and token embedding ~ N(0, 0.02) quantised to the chosen
 *   GGUF type, LayerNorm gamma = 1 / beta = 0, biases 0 (fp32), positional
 *   embedding ~ N(0, 0.01) fp32, encoder outputs ~ N(0, 1) fp32.
 *
 * PRNG: counter-based SplitMix64 -> Box-Muller in double. Value pair j of
 * stream s under seed S uses u1 = U(mix(key + 2j)), u2 = U(mix(key + 2j + 1))
 * with key = mix(S ^ mix(s + golden)), so any tensor (or slice of it) can be
 * generated independently and in parallel with identical results.
 *
 * Quantisers restate internal/gguf/quant.go:99-232 (QuantizeQ4_0 ..
 * QuantizeQ8_0) and float32ToF16 (:11-55) bit for bit: the scale is computed
 * in float32, stored as f16, and the codes use the float32 scale with
 * math.Round (half away from zero) on float64(v/scale). Rows are quantised
 * independently, which is what ml.NewQuantizedMatrix expects
 * (ml/matmul_q8.go:74-87).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#include "../../include/wg_decoder.h"

#define GEN_API __attribute__((visibility("default")))

static inline uint64_t mix64(uint64_t z) {
  z += 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}
static inline double unit(uint64_t x) { /* (0, 1] */
  return ((double)(x >> 11) + 1.0) * (1.0 / 9007199254740992.0);
}

/* out[i] = std * N(0,1) for i in [0, n): elements [offset, offset+n) of stream. */
GEN_API void wg_gen_normal(uint64_t seed, uint64_t stream, int64_t offset, int64_t n, float std, float* out) {
  uint64_t key = mix64(seed ^ mix64(stream + 0x632BE59BD9B4E019ull));
  const double two_pi = 6.283185307179586476925286766559;
#pragma omp parallel for schedule(static) if (n > (1 << 16))
  for (int64_t i = 0; i < n; i++) {
    int64_t e = offset + i, j = e >> 1;
    double u1 = unit(mix64(key + 2 * (uint64_t)j));
    double u2 = unit(mix64(key + 2 * (uint64_t)j + 1));
    double r = sqrt(-2.0 * log(u1));
    double z = (e & 1) ? r * sin(two_pi * u2) : r * cos(two_pi * u2);
    out[i] = (float)(z * (double)std);
  }
}

/* internal/gguf/quant.go:11-55 */
GEN_API uint16_t wg_gen_f32_to_f16(float f) {
  uint32_t bits;
  memcpy(&bits, &f, 4);
  uint16_t sign = (uint16_t)(bits >> 31);
  int exp = (int)((bits >> 23) & 0xFF);
  uint32_t mant = bits & 0x7FFFFF;
  if (exp == 255) return mant ? (uint16_t)(sign << 15 | 0x7E00) : (uint16_t)(sign << 15 | 0x7C00);
  if (exp == 0) return (uint16_t)(sign << 15);
  int exp16 = exp - 127 + 15;
  if (exp16 >= 31) return (uint16_t)(sign << 15 | 0x7C00);
  if (exp16 <= 0) {
    if (exp16 < -10) return (uint16_t)(sign << 15);
    unsigned shift = (unsigned)(1 - exp16);
    return (uint16_t)(sign << 15 | (uint16_t)((mant | 0x800000) >> (13 + shift)));
  }
  uint16_t mant16 = (uint16_t)(mant >> 13);
  if ((mant >> 12) & 1) mant16++;
  if (mant16 >= 0x400) {
    mant16 = 0;
    exp16++;
    if (exp16 >= 31) return (uint16_t)(sign << 15 | 0x7C00);
  }
  return (uint16_t)(sign << 15 | (uint16_t)exp16 << 10 | mant16);
}

static inline void put16(uint8_t* p, float f) {
  uint16_t h = wg_gen_f32_to_f16(f);
  p[0] = (uint8_t)h;
  p[1] = (uint8_t)(h >> 8);
}
static inline int32_t go_round(float x) { return (int32_t)round((double)x); } /* math.Round */

static inline float blk_get(const float* blk, int len, int i) { return i < len ? blk[i] : 0.0f; }

/* One 32-element block (len <= 32 valid values) of each type. */
static void q4_0_block(const float* blk, int len, uint8_t* ob) { /* quant.go:99-120 */
  float absmax = 0;
  for (int i = 0; i < len; i++) { float a = fabsf(blk[i]); if (a > absmax) absmax = a; }
  float scale = absmax / 7.0f;
  put16(ob, scale);
  for (int i = 0; i < 16; i++) {
    int32_t q[2];
    for (int h = 0; h < 2; h++) { /* quantNibble :284-300 */
      float v = blk_get(blk, len, 2 * i + h);
      int32_t qq = 8;
      if (scale != 0) qq = go_round(v / scale) + 8;
      if (qq < 0) qq = 0;
      if (qq > 15) qq = 15;
      q[h] = qq;
    }
    ob[2 + i] = (uint8_t)(q[0] | (q[1] << 4));
  }
}
static void minmax(const float* blk, int len, float* mn, float* mx) { /* quant.go:261-275 */
  if (len == 0) { *mn = *mx = 0; return; }
  *mn = *mx = blk[0];
  for (int i = 1; i < len; i++) { if (blk[i] < *mn) *mn = blk[i]; if (blk[i] > *mx) *mx = blk[i]; }
}
static void q4_1_block(const float* blk, int len, uint8_t* ob) { /* quant.go:124-141 */
  float mn, mx;
  minmax(blk, len, &mn, &mx);
  float scale = (mx - mn) / 15.0f;
  put16(ob, scale);
  put16(ob + 2, mn);
  for (int i = 0; i < 16; i++) {
    int32_t q[2];
    for (int h = 0; h < 2; h++) { /* quantNibbleUnsigned :303-319 */
      float v = blk_get(blk, len, 2 * i + h);
      int32_t qq = 0;
      if (scale != 0) qq = go_round((v - mn) / scale);
      if (qq < 0) qq = 0;
      if (qq > 15) qq = 15;
      q[h] = qq;
    }
    ob[4 + i] = (uint8_t)(q[0] | (q[1] << 4));
  }
}
static void nibble_set(uint8_t* dst, int i, uint8_t v) { /* quant.go:360-366 */
  if (i % 2 == 0) dst[i / 2] = (uint8_t)((dst[i / 2] & 0xF0) | (v & 0xF));
  else dst[i / 2] = (uint8_t)((dst[i / 2] & 0x0F) | ((v & 0xF) << 4));
}
static void q5_0_block(const float* blk, int len, uint8_t* ob) { /* quant.go:145-173 */
  float absmax = 0;
  for (int i = 0; i < len; i++) { float a = fabsf(blk[i]); if (a > absmax) absmax = a; }
  float scale = absmax / 15.0f;
  put16(ob, scale);
  uint32_t qh = 0;
  for (int i = 0; i < 32; i++) { /* quant5Signed :322-338 */
    float v = blk_get(blk, len, i);
    int32_t q = 16;
    if (scale != 0) q = go_round(v / scale) + 16;
    if (q < 0) q = 0;
    if (q > 31) q = 31;
    if ((q >> 4) & 1) qh |= 1u << i;
    nibble_set(ob + 6, i, (uint8_t)(q & 0xF));
  }
  ob[2] = (uint8_t)qh; ob[3] = (uint8_t)(qh >> 8); ob[4] = (uint8_t)(qh >> 16); ob[5] = (uint8_t)(qh >> 24);
}
static void q5_1_block(const float* blk, int len, uint8_t* ob) { /* quant.go:177-201 */
  float mn, mx;
  minmax(blk, len, &mn, &mx);
  float scale = (mx - mn) / 31.0f;
  put16(ob, scale);
  put16(ob + 2, mn);
  uint32_t qh = 0;
  for (int i = 0; i < 32; i++) { /* quant5Unsigned :341-357 */
    float v = blk_get(blk, len, i);
    int32_t q = 0;
    if (scale != 0) q = go_round((v - mn) / scale);
    if (q < 0) q = 0;
    if (q > 31) q = 31;
    if ((q >> 4) & 1) qh |= 1u << i;
    nibble_set(ob + 8, i, (uint8_t)(q & 0xF));
  }
  ob[4] = (uint8_t)qh; ob[5] = (uint8_t)(qh >> 8); ob[6] = (uint8_t)(qh >> 16); ob[7] = (uint8_t)(qh >> 24);
}
static void q8_0_block(const float* blk, int len, uint8_t* ob) { /* quant.go:205-232 */
  float absmax = 0;
  for (int i = 0; i < len; i++) { float a = fabsf(blk[i]); if (a > absmax) absmax = a; }
  float scale = absmax / 127.0f;
  put16(ob, scale);
  for (int i = 0; i < 32; i++) {
    float v = blk_get(blk, len, i);
    int32_t q = 0;
    if (scale != 0) {
      q = go_round(v / scale);
      if (q < -127) q = -127; /* clampI8 :368-376 */
      if (q > 127) q = 127;
    }
    ob[2 + i] = (uint8_t)(int8_t)q;
  }
}

GEN_API int64_t wg_gen_row_bytes(uint32_t qtype, int64_t cols) {
  int64_t blocks = (cols + 31) / 32;
  switch (qtype) {
    case WG_QTYPE_F32: return cols * 4;
    case WG_QTYPE_F16: return cols * 2;
    case WG_QTYPE_Q4_0: return blocks * 18;
    case WG_QTYPE_Q4_1: return blocks * 20;
    case WG_QTYPE_Q5_0: return blocks * 22;
    case WG_QTYPE_Q5_1: return blocks * 24;
    case WG_QTYPE_Q8_0: return blocks * 34;
    default: return -1;
  }
}

/* Quantise n values as one GGUF tensor run (blocks of 32 over the flat
 * data, as QuantizeQ* do). Returns bytes written or -1. */
GEN_API int64_t wg_gen_quantize(uint32_t qtype, const float* data, int64_t n, void* out_) {
  uint8_t* out = (uint8_t*)out_;
  int64_t nb = (n + 31) / 32;
  int64_t bb = wg_gen_row_bytes(qtype, 32);
  if (qtype == WG_QTYPE_F32) { memcpy(out, data, (size_t)n * 4); return n * 4; }
  if (qtype == WG_QTYPE_F16) {
    for (int64_t i = 0; i < n; i++) put16(out + 2 * i, data[i]);
    return n * 2;
  }
  if (bb < 0) return -1;
  for (int64_t b = 0; b < nb; b++) {
    const float* blk = data + b * 32;
    int len = (int)((n - b * 32) < 32 ? (n - b * 32) : 32);
    uint8_t* ob = out + b * bb;
    memset(ob, 0, (size_t)bb);
    switch (qtype) {
      case WG_QTYPE_Q4_0: q4_0_block(blk, len, ob); break;
      case WG_QTYPE_Q4_1: q4_1_block(blk, len, ob); break;
      case WG_QTYPE_Q5_0: q5_0_block(blk, len, ob); break;
      case WG_QTYPE_Q5_1: q5_1_block(blk, len, ob); break;
      case WG_QTYPE_Q8_0: q8_0_block(blk, len, ob); break;
      default: return -1;
    }
  }
  return nb * bb;
}

/* Quantise a [rows, cols] matrix row by row (each row its own block run). */
GEN_API int wg_gen_quantize_matrix(uint32_t qtype, const float* data, int64_t rows, int64_t cols, void* out_) {
  int64_t rb = wg_gen_row_bytes(qtype, cols);
  if (rb < 0) return -1;
  uint8_t* out = (uint8_t*)out_;
  int bad = 0;
#pragma omp parallel for schedule(static) if (rows * cols > (1 << 18))
  for (int64_t r = 0; r < rows; r++)
    if (wg_gen_quantize(qtype, data + r * cols, cols, out + r * rb) < 0) bad = 1;
  return bad ? -1 : 0;
}

/* ---- synthetic model ---------------------------------------------------- */

typedef struct gen_model {
  wg_model_desc desc;      /* must stay first: the handle is a wg_model_desc* */
  wg_layer_desc* layers;
  void** allocs;
  int n_allocs, cap_allocs;
} gen_model;

static void* track(gen_model* g, size_t bytes) {
  void* p = calloc(1, bytes ? bytes : 1);
  if (!p) return NULL;
  if (g->n_allocs == g->cap_allocs) {
    g->cap_allocs = g->cap_allocs ? 2 * g->cap_allocs : 64;
    g->allocs = (void**)realloc(g->allocs, sizeof(void*) * (size_t)g->cap_allocs);
  }
  g->allocs[g->n_allocs++] = p;
  return p;
}

/* stream ids: tensor kind in the low byte, layer above it */
enum { S_TOK = 1, S_POS = 2, S_SQ = 3, S_SK, S_SV, S_SO, S_CQ, S_CK, S_CV, S_CO, S_M0, S_M2 };

static int gen_matrix(gen_model* g, uint64_t seed, uint64_t stream, uint32_t qtype, int rows, int cols,
                      float std, wg_matrix* out) {
  float* tmp = (float*)malloc((size_t)rows * cols * 4);
  if (!tmp) return -1;
  wg_gen_normal(seed, stream, 0, (int64_t)rows * cols, std, tmp);
  int64_t rb = wg_gen_row_bytes(qtype, cols);
  void* data = track(g, (size_t)(rb * rows));
  if (!data) { free(tmp); return -1; }
  int rc = wg_gen_quantize_matrix(qtype, tmp, rows, cols, data);
  free(tmp);
  out->qtype = qtype; out->rows = rows; out->cols = cols; out->data = data;
  return rc;
}

static float* gen_const(gen_model* g, int n, float v) {
  float* p = (float*)track(g, (size_t)n * 4);
  if (p) for (int i = 0; i < n; i++) p[i] = v;
  return p;
}

GEN_API void wg_gen_model_free(wg_model_desc* d) {
  if (!d) return;
  gen_model* g = (gen_model*)d;
  for (int i = 0; i < g->n_allocs; i++) free(g->allocs[i]);
  free(g->allocs);
  free(g->layers);
  free(g);
}

/* Synthetic decoder of the given shape; every weight matrix in qtype. */
GEN_API wg_model_desc* wg_gen_model_create(int n_vocab, int d, int n_head, int n_layer, int n_ctx,
                                           uint32_t qtype, uint64_t seed) {
  gen_model* g = (gen_model*)calloc(1, sizeof(gen_model));
  if (!g) return NULL;
  g->layers = (wg_layer_desc*)calloc((size_t)n_layer, sizeof(wg_layer_desc));
  wg_model_desc* m = &g->desc;
  m->n_vocab = n_vocab; m->n_state = d; m->n_head = n_head; m->n_layer = n_layer;
  m->n_text_ctx = n_ctx; m->eot = 50256; m->layers = g->layers;
  int bad = gen_matrix(g, seed, S_TOK, qtype, n_vocab, d, 0.02f, &m->token_embedding);
  float* pos = (float*)track(g, (size_t)n_ctx * d * 4);
  if (!pos) bad = 1; else wg_gen_normal(seed, S_POS, 0, (int64_t)n_ctx * d, 0.01f, pos);
  m->positional_embedding = pos;
  m->ln_w = gen_const(g, d, 1.0f);
  m->ln_b = gen_const(g, d, 0.0f);
  for (int l = 0; l < n_layer && !bad; l++) {
    wg_layer_desc* L = &g->layers[l];
    uint64_t s = (uint64_t)(l + 1) << 8;
    L->self_ln_w = gen_const(g, d, 1.0f); L->self_ln_b = gen_const(g, d, 0.0f);
    L->cross_ln_w = gen_const(g, d, 1.0f); L->cross_ln_b = gen_const(g, d, 0.0f);
    L->mlp_ln_w = gen_const(g, d, 1.0f); L->mlp_ln_b = gen_const(g, d, 0.0f);
    L->self_q_b = gen_const(g, d, 0.0f); L->self_v_b = gen_const(g, d, 0.0f);
    L->self_o_b = gen_const(g, d, 0.0f);
    L->cross_q_b = gen_const(g, d, 0.0f); L->cross_v_b = gen_const(g, d, 0.0f);
    L->cross_o_b = gen_const(g, d, 0.0f);
    L->mlp0_b = gen_const(g, 4 * d, 0.0f); L->mlp2_b = gen_const(g, d, 0.0f);
    bad |= gen_matrix(g, seed, s | S_SQ, qtype, d, d, 0.02f, &L->self_q);
    bad |= gen_matrix(g, seed, s | S_SK, qtype, d, d, 0.02f, &L->self_k);
    bad |= gen_matrix(g, seed, s | S_SV, qtype, d, d, 0.02f, &L->self_v);
    bad |= gen_matrix(g, seed, s | S_SO, qtype, d, d, 0.02f, &L->self_o);
    bad |= gen_matrix(g, seed, s | S_CQ, qtype, d, d, 0.02f, &L->cross_q);
    bad |= gen_matrix(g, seed, s | S_CK, qtype, d, d, 0.02f, &L->cross_k);
    bad |= gen_matrix(g, seed, s | S_CV, qtype, d, d, 0.02f, &L->cross_v);
    bad |= gen_matrix(g, seed, s | S_CO, qtype, d, d, 0.02f, &L->cross_o);
    bad |= gen_matrix(g, seed, s | S_M0, qtype, 4 * d, d, 0.02f, &L->mlp0);
    bad |= gen_matrix(g, seed, s | S_M2, qtype, d, 4 * d, 0.02f, &L->mlp2);
  }
  if (bad) { wg_gen_model_free(m); return NULL; }
  return m;
}

/* Encoder output of utterance u: [T, d] ~ N(0,1) with seed (seed + u). */
GEN_API void wg_gen_encoder(uint64_t seed, int u, int T, int d, float* out) {
  wg_gen_normal(seed + (uint64_t)u, 0xE4C0DE, 0, (int64_t)T * d, 1.0f, out);
}
