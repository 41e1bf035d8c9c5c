/*
 * oracle.c — CPU restatement of whisper.go's decoder token loop.
 *
 * TEST INFRASTRUCTURE ONLY. This file is the parity checker for the CUDA
 * library and the timed CPU baseline ("port") of bench.py. Nothing in the
 * product path links, loads or calls it.
 *
 * Every function restates one reference function; the citation is the
 * reference file:line (paths inside the wxcdart/whisper.go module). The
 * reference is pure Go and cannot be built here (no Go toolchain; gonum
 * v0.17.0 / purego v0.10.0 / x/sync v0.20.0 / x/sys v0.42.0 are not
 * vendored), so parity is pinned by the reference's own known-answer tests
 * (internal/gguf/gguf_test.go:155-311, quant_test.go, ml/ops_test.go,
 * ml/attention_test.go, ml/matmul_q8_test.go), committed as fixtures under
 * tests/golden/.
 *
 * Build: -O2 -ffp-contract=off (Go never fuses a*b+c on amd64, and the
 * dequantisers d*v+m must round twice), -fopenmp.
 *
 * Known deviation: the dense fp32 dot products inside attention go through
 * gonum's sgemm in the reference (ml/blas.go:47-88); its blocking is not
 * available, so they are plain sequential dot products here. They are
 * pinned only by tolerance (ml/ops_test.go:349-438, attention_test.go:57).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#include <float.h>
#include <omp.h>

#include "../include/wg_decoder.h"

#define OR_API __attribute__((visibility("default")))

/* ------------------------------------------------------------------------ */
/* f16 <-> f32                                                               */
/* ------------------------------------------------------------------------ */

static inline uint32_t f32_bits(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static inline float bits_f32(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }

/* internal/gguf/quant.go:11-55 (float32ToF16): round-half-up on bit 12,
 * f16 subnormals truncated, float32 subnormals flushed to +-0. */
OR_API uint16_t or_f32_to_f16(float f) {
  uint32_t bits = f32_bits(f);
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
    uint16_t mant16 = (uint16_t)((mant | 0x800000) >> (13 + shift));
    return (uint16_t)(sign << 15 | mant16);
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

/* internal/gguf/dequant.go:15-44 (f16ToF32), identical to
 * ml/matmul_q8.go:759-781 (f16ToF32Local). */
OR_API float or_f16_to_f32(uint16_t h) {
  uint32_t s = (uint32_t)(h >> 15) << 31;
  uint32_t e = (h >> 10) & 0x1F;
  uint32_t m = h & 0x3FF;
  if (e == 0) {
    if (m == 0) return bits_f32(s);
    uint32_t k = 1;
    m <<= 1;
    while ((m & 0x400) == 0) { m <<= 1; k++; }
    m &= 0x3FF;
    return bits_f32(s | ((113 - k) << 23) | (m << 13));
  }
  if (e == 31) return bits_f32(s | 0x7F800000 | (m << 13));
  return bits_f32(s | ((e + 112) << 23) | (m << 13));
}

static inline uint16_t rd16(const uint8_t* p) { return (uint16_t)(p[0] | (p[1] << 8)); }
static inline uint32_t rd32(const uint8_t* p) {
  return (uint32_t)p[0] | (uint32_t)p[1] << 8 | (uint32_t)p[2] << 16 | (uint32_t)p[3] << 24;
}

/* ------------------------------------------------------------------------ */
/* block formats                                                             */
/* ------------------------------------------------------------------------ */

/* ml/matmul_q8.go:198-214 (quantRowBytes) plus the dense GGUF types. */
OR_API int64_t or_row_bytes(uint32_t qtype, int64_t cols) {
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

/* internal/gguf/dequant.go:47-81 (dequantize) with the block decoders
 * dequantQ4_0 :92-108, dequantQ4_1 :113-130, dequantQ5_0 :135-156,
 * dequantQ5_1 :161-183, dequantQ8_0 :188-201. Interleaved nibbles: element
 * 2i is the low nibble of qs[i], element 2i+1 the high nibble. */
OR_API int or_dequant(uint32_t qtype, const void* raw_, int64_t n, float* out) {
  const uint8_t* raw = (const uint8_t*)raw_;
  int64_t nb = (n + 31) / 32;
  switch (qtype) {
    case WG_QTYPE_F32:
      memcpy(out, raw, (size_t)n * 4);
      return 0;
    case WG_QTYPE_F16:
      for (int64_t i = 0; i < n; i++) out[i] = or_f16_to_f32(rd16(raw + 2 * i));
      return 0;
    case WG_QTYPE_Q4_0:
      for (int64_t b = 0; b < nb; b++) {
        const uint8_t* blk = raw + b * 18;
        float scale = or_f16_to_f32(rd16(blk));
        const uint8_t* qs = blk + 2;
        int64_t base = b * 32;
        for (int i = 0; i < 16; i++) {
          int64_t j = base + i * 2;
          if (j < n) out[j] = scale * (float)((int32_t)(qs[i] & 0xF) - 8);
          if (j + 1 < n) out[j + 1] = scale * (float)((int32_t)(qs[i] >> 4) - 8);
        }
      }
      return 0;
    case WG_QTYPE_Q4_1:
      for (int64_t b = 0; b < nb; b++) {
        const uint8_t* blk = raw + b * 20;
        float d = or_f16_to_f32(rd16(blk));
        float m = or_f16_to_f32(rd16(blk + 2));
        const uint8_t* qs = blk + 4;
        int64_t base = b * 32;
        for (int i = 0; i < 16; i++) {
          int64_t j = base + i * 2;
          if (j < n) out[j] = d * (float)(qs[i] & 0xF) + m;
          if (j + 1 < n) out[j + 1] = d * (float)(qs[i] >> 4) + m;
        }
      }
      return 0;
    case WG_QTYPE_Q5_0:
      for (int64_t b = 0; b < nb; b++) {
        const uint8_t* blk = raw + b * 22;
        float scale = or_f16_to_f32(rd16(blk));
        uint32_t qh = rd32(blk + 2);
        const uint8_t* qs = blk + 6;
        int64_t base = b * 32;
        for (int i = 0; i < 16; i++) {
          uint32_t hi0 = (qh >> (i * 2)) & 1, hi1 = (qh >> (i * 2 + 1)) & 1;
          int32_t v0 = (int32_t)((uint32_t)(qs[i] & 0xF) | (hi0 << 4)) - 16;
          int32_t v1 = (int32_t)((uint32_t)(qs[i] >> 4) | (hi1 << 4)) - 16;
          int64_t j = base + i * 2;
          if (j < n) out[j] = scale * (float)v0;
          if (j + 1 < n) out[j + 1] = scale * (float)v1;
        }
      }
      return 0;
    case WG_QTYPE_Q5_1:
      for (int64_t b = 0; b < nb; b++) {
        const uint8_t* blk = raw + b * 24;
        float d = or_f16_to_f32(rd16(blk));
        float m = or_f16_to_f32(rd16(blk + 2));
        uint32_t qh = rd32(blk + 4);
        const uint8_t* qs = blk + 8;
        int64_t base = b * 32;
        for (int i = 0; i < 16; i++) {
          uint32_t hi0 = (qh >> (i * 2)) & 1, hi1 = (qh >> (i * 2 + 1)) & 1;
          float v0 = (float)((uint32_t)(qs[i] & 0xF) | (hi0 << 4));
          float v1 = (float)((uint32_t)(qs[i] >> 4) | (hi1 << 4));
          int64_t j = base + i * 2;
          if (j < n) out[j] = d * v0 + m;
          if (j + 1 < n) out[j + 1] = d * v1 + m;
        }
      }
      return 0;
    case WG_QTYPE_Q8_0:
      for (int64_t b = 0; b < nb; b++) {
        const uint8_t* blk = raw + b * 34;
        float scale = or_f16_to_f32(rd16(blk));
        const int8_t* qs = (const int8_t*)(blk + 2);
        int64_t base = b * 32;
        for (int i = 0; i < 32; i++)
          if (base + i < n) out[base + i] = scale * (float)qs[i];
      }
      return 0;
    default:
      return WG_ERR_UNSUPPORTED;
  }
}

/* ------------------------------------------------------------------------ */
/* quantised dot products (the generic kernels)                              */
/* ------------------------------------------------------------------------ */

/* ml/matmul_q8.go:679-692 dotQ8Block32 */
static float dot_q8_block32(float scale, const int8_t* q, const float* f) {
  float s0 = 0, s1 = 0, s2 = 0, s3 = 0;
  for (int i = 0; i < 32; i += 8) {
    s0 += (float)q[i + 0] * f[i + 0];
    s1 += (float)q[i + 1] * f[i + 1];
    s2 += (float)q[i + 2] * f[i + 2];
    s3 += (float)q[i + 3] * f[i + 3];
    s0 += (float)q[i + 4] * f[i + 4];
    s1 += (float)q[i + 5] * f[i + 5];
    s2 += (float)q[i + 6] * f[i + 6];
    s3 += (float)q[i + 7] * f[i + 7];
  }
  return scale * (s0 + s1 + s2 + s3);
}

/* Dot of one stored row with an fp32 vector of length k.
 * Q4_0 ml/matmul_q8.go:237-269 (+dotQ40Block32 :694-703),
 * Q4_1 :275-308 (+dotQ41Block32 :705-714), Q5_0 :314-351 (+:716-729),
 * Q5_1 :357-395 (+:731-744), Q8_0 :403-429 (+:679-692).
 * F32/F16 rows (dense tensors, ml/matmul.go → sgemm) are a sequential dot. */
OR_API float or_dot_row(uint32_t qtype, const void* row_, const float* f, int n) {
  const uint8_t* q = (const uint8_t*)row_;
  int nb = (n + 31) / 32;
  float sum = 0;
  switch (qtype) {
    case WG_QTYPE_F32: {
      const float* w = (const float*)row_;
      for (int i = 0; i < n; i++) sum += f[i] * w[i];
      return sum;
    }
    case WG_QTYPE_F16:
      for (int i = 0; i < n; i++) sum += f[i] * or_f16_to_f32(rd16(q + 2 * i));
      return sum;
    case WG_QTYPE_Q8_0:
      for (int b = 0; b < nb; b++) {
        const uint8_t* blk = q + b * 34;
        float scale = or_f16_to_f32(rd16(blk));
        const int8_t* v = (const int8_t*)(blk + 2);
        int start = b * 32, rem = n - start;
        if (rem >= 32) { sum += dot_q8_block32(scale, v, f + start); continue; }
        for (int i = 0; i < rem; i++) sum += scale * (float)v[i] * f[start + i];
      }
      return sum;
    case WG_QTYPE_Q4_0:
      for (int b = 0; b < nb; b++) {
        const uint8_t* blk = q + b * 18;
        float d = or_f16_to_f32(rd16(blk));
        const uint8_t* qs = blk + 2;
        int base = b * 32, rem = n - base;
        if (rem >= 32) {
          float s = 0;
          for (int i = 0; i < 16; i++) {
            s += (float)((int32_t)(qs[i] & 0xF) - 8) * f[base + 2 * i];
            s += (float)((int32_t)(qs[i] >> 4) - 8) * f[base + 2 * i + 1];
          }
          sum += d * s;
          continue;
        }
        for (int i = 0; i < 16; i++) {
          int j0 = base + i * 2;
          if (j0 < n) sum += d * (float)((int32_t)(qs[i] & 0xF) - 8) * f[j0];
          if (j0 + 1 < n) sum += d * (float)((int32_t)(qs[i] >> 4) - 8) * f[j0 + 1];
        }
      }
      return sum;
    case WG_QTYPE_Q4_1:
      for (int b = 0; b < nb; b++) {
        const uint8_t* blk = q + b * 20;
        float d = or_f16_to_f32(rd16(blk)), m = or_f16_to_f32(rd16(blk + 2));
        const uint8_t* qs = blk + 4;
        int base = b * 32, rem = n - base;
        if (rem >= 32) {
          float s = 0;
          for (int i = 0; i < 16; i++) {
            s += (d * (float)(qs[i] & 0xF) + m) * f[base + 2 * i];
            s += (d * (float)(qs[i] >> 4) + m) * f[base + 2 * i + 1];
          }
          sum += s;
          continue;
        }
        for (int i = 0; i < 16; i++) {
          int j0 = base + i * 2;
          if (j0 < n) sum += (d * (float)(qs[i] & 0xF) + m) * f[j0];
          if (j0 + 1 < n) sum += (d * (float)(qs[i] >> 4) + m) * f[j0 + 1];
        }
      }
      return sum;
    case WG_QTYPE_Q5_0:
      for (int b = 0; b < nb; b++) {
        const uint8_t* blk = q + b * 22;
        float d = or_f16_to_f32(rd16(blk));
        uint32_t qh = rd32(blk + 2);
        const uint8_t* qs = blk + 6;
        int base = b * 32, rem = n - base;
        float s = 0;
        for (int i = 0; i < 16; i++) {
          uint32_t hi0 = (qh >> (i * 2)) & 1, hi1 = (qh >> (i * 2 + 1)) & 1;
          float v0 = (float)((int32_t)((uint32_t)(qs[i] & 0xF) | (hi0 << 4)) - 16);
          float v1 = (float)((int32_t)((uint32_t)(qs[i] >> 4) | (hi1 << 4)) - 16);
          int j0 = base + i * 2;
          if (rem >= 32) {
            s += d * v0 * f[j0];
            s += d * v1 * f[j0 + 1];
          } else {
            if (j0 < n) sum += d * v0 * f[j0];
            if (j0 + 1 < n) sum += d * v1 * f[j0 + 1];
          }
        }
        if (rem >= 32) sum += s;
      }
      return sum;
    case WG_QTYPE_Q5_1:
      for (int b = 0; b < nb; b++) {
        const uint8_t* blk = q + b * 24;
        float d = or_f16_to_f32(rd16(blk)), m = or_f16_to_f32(rd16(blk + 2));
        uint32_t qh = rd32(blk + 4);
        const uint8_t* qs = blk + 8;
        int base = b * 32, rem = n - base;
        float s = 0;
        for (int i = 0; i < 16; i++) {
          uint32_t hi0 = (qh >> (i * 2)) & 1, hi1 = (qh >> (i * 2 + 1)) & 1;
          float v0 = (float)((uint32_t)(qs[i] & 0xF) | (hi0 << 4));
          float v1 = (float)((uint32_t)(qs[i] >> 4) | (hi1 << 4));
          int j0 = base + i * 2;
          if (rem >= 32) {
            s += (d * v0 + m) * f[j0];
            s += (d * v1 + m) * f[j0 + 1];
          } else {
            if (j0 < n) sum += (d * v0 + m) * f[j0];
            if (j0 + 1 < n) sum += (d * v1 + m) * f[j0 + 1];
          }
        }
        if (rem >= 32) sum += s;
      }
      return sum;
    default:
      return NAN;
  }
}

static int g_inner_threads = 1;
/* Threads used inside one GEMV (over output rows). The reference runs the
 * decoder's M=1 GEMVs serially (ml/matmul_q8.go:110-116); parallelising over
 * output rows changes no arithmetic, only the wall time of the tests. */
OR_API void or_set_inner_threads(int n) { g_inner_threads = n < 1 ? 1 : n; }

/* ml/matmul_q8.go:93-196 (MatMulQuantTransBInto): out[i,j] = dot(B row j, A row i). */
OR_API int or_matmul(uint32_t qtype, const void* raw, int rows, int cols,
                     const float* a, int m, float* out) {
  int64_t rb = or_row_bytes(qtype, cols);
  if (rb < 0) return WG_ERR_UNSUPPORTED;
  const uint8_t* w = (const uint8_t*)raw;
  int64_t total = (int64_t)m * rows;
#pragma omp parallel for schedule(static) num_threads(g_inner_threads) if (g_inner_threads > 1 && total >= 512)
  for (int64_t t = 0; t < total; t++) {
    int i = (int)(t / rows), j = (int)(t % rows);
    out[t] = or_dot_row(qtype, w + (int64_t)j * rb, a + (int64_t)i * cols, cols);
  }
  return 0;
}

/* ------------------------------------------------------------------------ */
/* elementwise ops                                                            */
/* ------------------------------------------------------------------------ */

/* ml/ops.go:153-202 (LayerNormInto): 4-way unrolled sums, std via float64
 * sqrt, out = w*(v-mean)/std + b. */
OR_API void or_layernorm(float* dst, const float* src, const float* w, const float* b,
                         int rows, int C, float eps) {
  for (int r = 0; r < rows; r++) {
    const float* s = src + (int64_t)r * C;
    float* d = dst + (int64_t)r * C;
    float mean = 0;
    int i = 0;
    for (; i + 3 < C; i += 4) mean += s[i] + s[i + 1] + s[i + 2] + s[i + 3];
    for (; i < C; i++) mean += s[i];
    mean /= (float)C;
    float vari = 0;
    i = 0;
    for (; i + 3 < C; i += 4) {
      float d0 = s[i] - mean, d1 = s[i + 1] - mean, d2 = s[i + 2] - mean, d3 = s[i + 3] - mean;
      vari += d0 * d0 + d1 * d1 + d2 * d2 + d3 * d3;
    }
    for (; i < C; i++) { float dd = s[i] - mean; vari += dd * dd; }
    vari /= (float)C;
    float std = (float)sqrt((double)(vari + eps));
    for (i = 0; i < C; i++) d[i] = w[i] * (s[i] - mean) / std + b[i];
  }
}

/* ml/ops.go:102-122 (GELUInPlace): tanh form, tanh in float64. */
OR_API void or_gelu_inplace(float* x, int64_t n) {
  const float sqrt2OverPi = (float)0.7978845608028654;
  const float c = (float)0.044715;
  for (int64_t i = 0; i < n; i++) {
    float v = x[i];
    float inner = sqrt2OverPi * (v + c * v * v * v);
    x[i] = v * 0.5f * (float)(1 + tanh((double)inner));
  }
}

/* ml/attention.go:34-61 (fastExpApprox). */
OR_API float or_fast_exp(float x) {
  const float invLn2 = (float)1.4426950408889634;
  const float ln2 = (float)0.6931471805599453;
  if (x <= -20) return 0;
  float y = x * invLn2;
  int k = (int)y;
  if ((float)k > y) k--;
  float r = x - (float)k * ln2;
  float r2 = r * r;
  float r3 = r2 * r;
  float r4 = r3 * r;
  float poly = 1 + r + 0.5f * r2 + (float)(1.0 / 6.0) * r3 + (float)(1.0 / 24.0) * r4;
  if (k < -126) return 0;
  if (k > 127) return FLT_MAX;
  return poly * bits_f32((uint32_t)(k + 127) << 23);
}

/* ml/attention.go:63-91 (rowMaxUnrolled) + attention_simd_kernels.go:24-69
 * (softmaxRowFastInPlaceWide, the amd64/AVX2 dispatch of
 * simd_dispatch_amd64.go). */
OR_API void or_softmax_fast(float* row, int n) {
  float maxv = row[0];
  for (int i = 1; i < n; i++) if (row[i] > maxv) maxv = row[i];
  float sum = 0;
  int i = 0;
  for (; i + 7 < n; i += 8) {
    float x0 = or_fast_exp(row[i] - maxv), x1 = or_fast_exp(row[i + 1] - maxv);
    float x2 = or_fast_exp(row[i + 2] - maxv), x3 = or_fast_exp(row[i + 3] - maxv);
    float x4 = or_fast_exp(row[i + 4] - maxv), x5 = or_fast_exp(row[i + 5] - maxv);
    float x6 = or_fast_exp(row[i + 6] - maxv), x7 = or_fast_exp(row[i + 7] - maxv);
    row[i] = x0; row[i + 1] = x1; row[i + 2] = x2; row[i + 3] = x3;
    row[i + 4] = x4; row[i + 5] = x5; row[i + 6] = x6; row[i + 7] = x7;
    sum += x0 + x1 + x2 + x3 + x4 + x5 + x6 + x7;
  }
  for (; i < n; i++) { float x = or_fast_exp(row[i] - maxv); row[i] = x; sum += x; }
  if (sum == 0) {
    float inv = 1.0f / (float)n;
    for (i = 0; i < n; i++) row[i] = inv;
    return;
  }
  float invSum = 1 / sum;
  for (i = 0; i < n; i++) row[i] *= invSum;
}

/* ml/attention.go:193-317 (ScaledDotProductAttentionInto) for one query
 * block: q [H,Tq,hd], k/v [H,Tk,hd] (head h at k + h*k_head_stride),
 * scores via a plain dot (sgemm), *scale, causal mask j>i, fast softmax,
 * out = P.V. scores: scratch of Tq*Tk floats. */
OR_API void or_attention(const float* q, const float* k, const float* v, int heads, int Tq,
                         int Tk, int hd, int64_t kv_head_stride, int causal, float* out,
                         float* scores) {
  float scale = (float)(1.0 / sqrt((double)hd));
  for (int h = 0; h < heads; h++) {
    const float* qh = q + (int64_t)h * Tq * hd;
    const float* kh = k + (int64_t)h * kv_head_stride;
    const float* vh = v + (int64_t)h * kv_head_stride;
    for (int i = 0; i < Tq; i++)
      for (int j = 0; j < Tk; j++) {
        float s = 0;
        for (int c = 0; c < hd; c++) s += qh[i * hd + c] * kh[(int64_t)j * hd + c];
        scores[i * Tk + j] = s;
      }
    for (int t = 0; t < Tq * Tk; t++) scores[t] *= scale;
    if (causal)
      for (int i = 0; i < Tq; i++)
        for (int j = i + 1; j < Tk; j++) scores[i * Tk + j] = -INFINITY;
    for (int i = 0; i < Tq; i++) or_softmax_fast(scores + i * Tk, Tk);
    float* oh = out + (int64_t)h * Tq * hd;
    for (int i = 0; i < Tq; i++)
      for (int c = 0; c < hd; c++) {
        float s = 0;
        for (int j = 0; j < Tk; j++) s += scores[i * Tk + j] * vh[(int64_t)j * hd + c];
        oh[i * hd + c] = s;
      }
  }
}

/* ------------------------------------------------------------------------ */
/* sampling                                                                  */
/* ------------------------------------------------------------------------ */

/* model/decoder.go:1140-1167 (applyRepetitionPenalty): out[id] -= penalty*count
 * over the last `window` history tokens. Applied in place. */
OR_API void or_apply_penalty(float* logits, int V, const int32_t* hist, int n_hist,
                             float penalty, int window) {
  if (penalty <= 0 || n_hist == 0 || window <= 0) return;
  int start = n_hist > window ? n_hist - window : 0;
  for (int i = start; i < n_hist; i++) {
    int id = hist[i];
    if (id < 0 || id >= V) continue;
    int first = 1;
    for (int j = start; j < i; j++) if (hist[j] == id) { first = 0; break; }
    if (!first) continue;
    int cnt = 0;
    for (int j = i; j < n_hist; j++) if (hist[j] == id) cnt++;
    logits[id] -= penalty * (float)cnt;
  }
}

static float inv_temp(float t) { return t > 0 ? 1 / t : 1.0f; }

/* model/decoder.go:996-1059 (sampleGreedyWithScratch). The top-p fallback
 * (:1036-1056, unseeded math/rand) is rejected by the callers. */
OR_API int or_sample_greedy(const float* logits, int V, int eot, float temperature,
                            int suppress_nst, float no_speech_thold) {
  float it = inv_temp(temperature);
  int maxIdx = 0;
  float maxScaled = logits[0] * it;
  for (int i = 1; i < V; i++) {
    float s = logits[i] * it;
    if (s > maxScaled) { maxScaled = s; maxIdx = i; }
  }
  if (suppress_nst && eot >= 0 && eot < V) {
    if (logits[eot] < -no_speech_thold && maxIdx == eot) {
      maxIdx = -1;
      maxScaled = -INFINITY;
      for (int i = 0; i < V; i++) {
        if (i == eot) continue;
        float s = logits[i] * it;
        if (s > maxScaled) { maxScaled = s; maxIdx = i; }
      }
      if (maxIdx < 0) maxIdx = eot;
    }
  }
  return maxIdx;
}

/* scaled values desc, lower index first on equal values (the reference's
 * sort.Slice is unstable; exactly equal values are measure-zero) */
static const float* g_sort_key;
static int cmp_desc(const void* a, const void* b) {
  int i = *(const int*)a, j = *(const int*)b;
  float x = g_sort_key[i], y = g_sort_key[j];
  if (x > y) return -1;
  if (x < y) return 1;
  return i < j ? -1 : (i > j);
}
static void sort_desc(int* idx, int n, const float* key) {
  /* qsort with a file-scope key: the oracle's decodes are parallel over
   * utterances, so serialise the (rare) fallback sorts */
#pragma omp critical(or_sort)
  {
    g_sort_key = key;
    qsort(idx, (size_t)n, sizeof(int), cmp_desc);
  }
}

/* model/decoder.go:1251-1378 (sampleTopPFromLogitsWithScratch): scaled
 * logits, logZ (float32 sum of float64 exps), the best min(512, V) by a
 * replace-min scan, sorted descending; cumulative float32 probabilities up to
 * topP (a full sort of the row when those 512 do not reach it); then the draw
 * r = u01 * cumSum walks the same cumulative sum. u01 replaces the
 * reference's rand.Float32() (unseeded math/rand): wg_uniform(seed, u, t). */
OR_API int or_sample_topp(const float* logits, int V, float temperature, float topP, float u01) {
  if (V <= 0) return 0;
  float it = inv_temp(temperature);
  float* sc = (float*)malloc((size_t)V * 4);
  int* idx = (int*)malloc((size_t)V * 4);
  float scaledMax = logits[0] * it;
  for (int i = 0; i < V; i++) {
    sc[i] = logits[i] * it;
    idx[i] = i;
    if (sc[i] > scaledMax) scaledMax = sc[i];
  }
  float expSum = 0;
  for (int i = 0; i < V; i++) expSum += (float)exp((double)(sc[i] - scaledMax));
  float logZ = (float)log((double)expSum) + scaledMax;
  int limit = V < 512 ? V : 512;
  int n = 0, minPos = -1;
  float minScore = 0;
  for (int i = 0; i < V; i++) {
    if (n < limit) {
      idx[n++] = i;
      if (minPos < 0 || sc[i] < minScore) { minPos = n - 1; minScore = sc[i]; }
      continue;
    }
    if (sc[i] > minScore) {
      idx[minPos] = i;
      minPos = 0;
      minScore = sc[idx[0]];
      for (int j = 1; j < n; j++)
        if (sc[idx[j]] < minScore) { minScore = sc[idx[j]]; minPos = j; }
    }
  }
  sort_desc(idx, n, sc);
  int topCount = 0;
  float cumSum = 0;
  for (int i = 0; i < n; i++) {
    cumSum += (float)exp((double)(sc[idx[i]] - logZ));
    topCount = i + 1;
    if (cumSum >= topP) break;
  }
  if (cumSum < topP && n < V) { /* full sort */
    for (int i = 0; i < V; i++) idx[i] = i;
    sort_desc(idx, V, sc);
    n = V;
    topCount = 0;
    cumSum = 0;
    for (int i = 0; i < n; i++) {
      cumSum += (float)exp((double)(sc[idx[i]] - logZ));
      topCount = i + 1;
      if (cumSum >= topP) break;
    }
  }
  int tok = idx[topCount > 0 ? topCount - 1 : 0];
  if (topCount > 0) {
    float r = u01 * cumSum, run = 0;
    for (int i = 0; i < topCount; i++) {
      run += (float)exp((double)(sc[idx[i]] - logZ));
      if (run >= r) { tok = idx[i]; break; }
    }
  }
  free(sc);
  free(idx);
  return tok;
}

/* wg_uniform of the ABI header (the seeded top-p draw), for the tests. */
OR_API float or_uniform(uint64_t seed, uint32_t u, uint32_t t) { return wg_uniform(seed, u, t); }

/* The top-p fallback test of sampleGreedyWithScratch (decoder.go:1036-1056):
 * returns 1 when the chosen token's log-prob (at temperature T) is below
 * -logprob_thold, so the step draws from the nucleus instead. */
OR_API int or_topp_fallback(const float* logits, int V, int chosen, float temperature, float logprob_thold) {
  float it = inv_temp(temperature);
  float scaledMax = -INFINITY;
  for (int i = 0; i < V; i++)
    if (logits[i] * it > scaledMax) scaledMax = logits[i] * it;
  float expSum = 0;
  for (int i = 0; i < V; i++) expSum += (float)exp((double)(logits[i] * it - scaledMax));
  float logZ = (float)log((double)expSum) + scaledMax;
  return logits[chosen] * it - logZ < -logprob_thold;
}

/* model/decoder.go:1068-1136 (topKTokensWithScratch): replace-min scan, then
 * logZ = log(sum float32(exp(float64(s - max)))) + max, lp = s - logZ,
 * sorted by lp descending (stable here; Go's sort.Slice is unstable, which
 * only matters for exactly tied log-probs). Returns the count (<= k). */
OR_API int or_topk(const float* logits, int V, int k, float temperature, int32_t* tok, float* lp) {
  if (k <= 0) return 0;
  if (k > V) k = V;
  float it = inv_temp(temperature);
  int n = 0, minPos = -1;
  float minVal = 0, scaledMax = -INFINITY;
  for (int i = 0; i < V; i++) {
    float s = logits[i] * it;
    if (s > scaledMax) scaledMax = s;
    if (n < k) {
      tok[n] = i; lp[n] = s; n++;
      if (minPos < 0 || s < minVal) { minPos = n - 1; minVal = s; }
      continue;
    }
    if (s <= minVal) continue;
    tok[minPos] = i; lp[minPos] = s;
    minPos = 0; minVal = lp[0];
    for (int j = 1; j < n; j++) if (lp[j] < minVal) { minVal = lp[j]; minPos = j; }
  }
  float expSum = 0;
  for (int i = 0; i < V; i++) expSum += (float)exp((double)(logits[i] * it - scaledMax));
  float logZ = (float)log((double)expSum) + scaledMax;
  for (int i = 0; i < n; i++) lp[i] -= logZ;
  for (int i = 1; i < n; i++) { /* stable insertion sort, descending */
    int32_t tt = tok[i]; float vv = lp[i]; int j = i - 1;
    while (j >= 0 && lp[j] < vv) { tok[j + 1] = tok[j]; lp[j + 1] = lp[j]; j--; }
    tok[j + 1] = tt; lp[j + 1] = vv;
  }
  return n;
}

/* ------------------------------------------------------------------------ */
/* decoder model                                                             */
/* ------------------------------------------------------------------------ */

#define LN_EPS 1e-5f /* model/encoder.go:11 layerNormEps */

typedef struct {
  const wg_model_desc* m;
  int d, H, hd, L, V, ctx;
} om;

typedef struct {
  float* kv;       /* [L][2][H][ctx][hd] (decoder.go:346) */
  float *x, *xln, *q, *k, *v, *attn, *out, *mlph, *logits, *scores;
  float* xscores; /* [H][T_enc] cross-attention scores, one row per head (inner threads) */
  int scores_cap;
} ostate;

static void st_init(ostate* s, const om* M, int T_enc) {
  memset(s, 0, sizeof(*s));
  s->kv = (float*)calloc((size_t)M->L * 2 * M->H * M->ctx * M->hd, 4);
  s->x = (float*)calloc(M->d, 4); s->xln = (float*)calloc(M->d, 4);
  s->q = (float*)calloc(M->d, 4); s->k = (float*)calloc(M->d, 4); s->v = (float*)calloc(M->d, 4);
  s->attn = (float*)calloc(M->d, 4); s->out = (float*)calloc(M->d, 4);
  s->mlph = (float*)calloc(4 * M->d, 4);
  s->logits = (float*)calloc(M->V, 4);
  s->scores_cap = (T_enc > M->ctx ? T_enc : M->ctx);
  s->scores = (float*)calloc(s->scores_cap, 4);
  s->xscores = g_inner_threads > 1 ? (float*)calloc((size_t)M->H * T_enc, 4) : NULL;
}
static void st_free(ostate* s) {
  free(s->kv); free(s->x); free(s->xln); free(s->q); free(s->k); free(s->v);
  free(s->attn); free(s->out); free(s->mlph); free(s->logits); free(s->scores); free(s->xscores);
}

static void matvec(const wg_matrix* w, const float* x, float* y) {
  or_matmul(w->qtype, w->data, w->rows, w->cols, x, 1, y);
}

/* Per-utterance cross K/V (decoder.go:923-940): K = E.Wk^T, V = E.Wv^T + vB. */
typedef struct { float *k, *v; } ocross;

static void cross_precompute(const om* M, const float* enc, int T, ocross* cr, int fake) {
  for (int l = 0; l < M->L; l++) {
    const wg_layer_desc* ly = &M->m->layers[l];
    cr[l].k = (float*)malloc((size_t)T * M->d * 4);
    cr[l].v = (float*)malloc((size_t)T * M->d * 4);
    if (fake) { /* timing-only: values are irrelevant to the step loop's cost */
      for (int64_t i = 0; i < (int64_t)T * M->d; i++) {
        cr[l].k[i] = (float)((i * 2654435761u) % 1000) * 1e-3f - 0.5f;
        cr[l].v[i] = (float)((i * 40503u) % 1000) * 1e-3f - 0.5f;
      }
      continue;
    }
    or_matmul(ly->cross_k.qtype, ly->cross_k.data, M->d, M->d, enc, T, cr[l].k);
    or_matmul(ly->cross_v.qtype, ly->cross_v.data, M->d, M->d, enc, T, cr[l].v);
    for (int t = 0; t < T; t++)
      for (int j = 0; j < M->d; j++) cr[l].v[(int64_t)t * M->d + j] += ly->cross_v_b[j];
  }
}
static void cross_free(const om* M, ocross* cr) {
  for (int l = 0; l < M->L; l++) { free(cr[l].k); free(cr[l].v); }
}

/* model/decoder.go:745-833 (forward) for the token at position pos, with the
 * Q1 fix: the embedding row is the dequantised row of the (quantised) token
 * embedding (the reference reads only the dense tokenEmb, :761-766, which is
 * empty whenever the embedding is quantised). mode selects the self-attention
 * semantics (see WG_MODE_*). want_logits=0 skips the logits GEMV (prefill). */
static int forward(const om* M, ostate* s, const ocross* cr, int T_enc, int token, int pos,
                   int mode, int want_logits) {
  int d = M->d, H = M->H, hd = M->hd;
  if (pos >= M->ctx || token < 0 || token >= M->V) return WG_ERR_INVALID;
  const wg_matrix* te = &M->m->token_embedding;
  int64_t rb = or_row_bytes(te->qtype, d);
  or_dequant(te->qtype, (const uint8_t*)te->data + (int64_t)token * rb, d, s->x);
  const float* pe = M->m->positional_embedding + (int64_t)pos * d;
  for (int i = 0; i < d; i++) s->x[i] += pe[i];
  int64_t headBlock = (int64_t)M->ctx * hd;
  for (int l = 0; l < M->L; l++) {
    const wg_layer_desc* ly = &M->m->layers[l];
    /* self-attention (decoder.go:836-908) */
    or_layernorm(s->xln, s->x, ly->self_ln_w, ly->self_ln_b, 1, d, LN_EPS);
    matvec(&ly->self_q, s->xln, s->q);
    for (int i = 0; i < d; i++) s->q[i] += ly->self_q_b[i];
    matvec(&ly->self_k, s->xln, s->k);
    matvec(&ly->self_v, s->xln, s->v);
    for (int i = 0; i < d; i++) s->v[i] += ly->self_v_b[i];
    float* kc = s->kv + (int64_t)l * 2 * H * headBlock;
    float* vc = kc + (int64_t)H * headBlock;
    for (int h = 0; h < H; h++) {
      memcpy(kc + h * headBlock + (int64_t)pos * hd, s->k + h * hd, hd * 4);
      memcpy(vc + h * headBlock + (int64_t)pos * hd, s->v + h * hd, hd * 4);
    }
    /* REF_COMPAT: Tq=1 with causal=true masks every slot j>0 (decoder.go:895,
     * attention.go:250-256). CORRECT: all slots 0..pos. */
    or_attention(s->q, kc, vc, H, 1, pos + 1, hd, headBlock, mode == WG_MODE_REF_COMPAT,
                 s->attn, s->scores);
    matvec(&ly->self_o, s->attn, s->out);
    for (int i = 0; i < d; i++) s->x[i] += s->out[i] + ly->self_o_b[i]; /* :790, :394-398 */
    /* cross-attention (decoder.go:911-971) */
    or_layernorm(s->xln, s->x, ly->cross_ln_w, ly->cross_ln_b, 1, d, LN_EPS);
    matvec(&ly->cross_q, s->xln, s->q);
    for (int i = 0; i < d; i++) s->q[i] += ly->cross_q_b[i];
    /* K_c/V_c [T,d] viewed as [H,T,hd] by reshape (:950-951): head h is the
     * column block h*hd..h*hd+hd-1 of every row, i.e. stride d between rows.
     * or_attention wants [T,hd] per head, so gather per head. */
    /* heads are independent: with inner threads each head has its own
     * scores row (same arithmetic as one thread doing them in turn) */
#pragma omp parallel for schedule(static) num_threads(g_inner_threads) if (s->xscores && H > 1)
    for (int h = 0; h < H; h++) {
      float* sc = s->xscores ? s->xscores + (int64_t)h * T_enc : s->scores;
      /* scores */
      float scale = (float)(1.0 / sqrt((double)hd));
      for (int t = 0; t < T_enc; t++) {
        float acc = 0;
        const float* kr = cr[l].k + (int64_t)t * d + h * hd;
        for (int c = 0; c < hd; c++) acc += s->q[h * hd + c] * kr[c];
        sc[t] = acc;
      }
      for (int t = 0; t < T_enc; t++) sc[t] *= scale;
      or_softmax_fast(sc, T_enc);
      for (int c = 0; c < hd; c++) {
        float acc = 0;
        for (int t = 0; t < T_enc; t++) acc += sc[t] * cr[l].v[(int64_t)t * d + h * hd + c];
        s->attn[h * hd + c] = acc;
      }
    }
    matvec(&ly->cross_o, s->attn, s->out);
    for (int i = 0; i < d; i++) s->x[i] += s->out[i] + ly->cross_o_b[i];
    /* MLP (decoder.go:974-993) */
    or_layernorm(s->xln, s->x, ly->mlp_ln_w, ly->mlp_ln_b, 1, d, LN_EPS);
    matvec(&ly->mlp0, s->xln, s->mlph);
    for (int i = 0; i < 4 * d; i++) s->mlph[i] += ly->mlp0_b[i];
    or_gelu_inplace(s->mlph, 4 * d);
    matvec(&ly->mlp2, s->mlph, s->out);
    for (int i = 0; i < d; i++) s->x[i] += s->out[i] + ly->mlp2_b[i];
  }
  if (!want_logits) return 0;
  or_layernorm(s->x, s->x, M->m->ln_w, M->m->ln_b, 1, d, LN_EPS); /* :818 */
  matvec(te, s->x, s->logits);                                   /* :823 */
  return 0;
}

static int om_init(om* M, const wg_model_desc* m) {
  M->m = m; M->d = m->n_state; M->H = m->n_head; M->L = m->n_layer;
  M->V = m->n_vocab; M->ctx = m->n_text_ctx;
  if (M->H <= 0 || M->d % M->H) return WG_ERR_INVALID;
  M->hd = M->d / M->H;
  return 0;
}

static int max_tokens_for(const om* M, const wg_decode_params* p, int P) {
  /* decoder.go:421-430 */
  int mt = p->max_tokens;
  if (mt <= 0) mt = M->ctx;
  if (M->ctx - P < mt) mt = M->ctx - P;
  if (mt < 0) mt = 0;
  return mt;
}

static float temperature_for(const wg_decode_params* p) {
  float base = p->temperature == 0 ? 1.0f : p->temperature; /* :416-419 */
  return base + (float)p->attempt * 0.2f;                   /* :435 */
}

/* CORRECT-mode prompt prefill: positions 0..P-2 (no logits). */
static int prefill(const om* M, ostate* s, const ocross* cr, int T_enc, const int32_t* prompt, int P) {
  for (int i = 0; i + 1 < P; i++) {
    int rc = forward(M, s, cr, T_enc, prompt[i], i, WG_MODE_CORRECT, 0);
    if (rc) return rc;
  }
  return 0;
}

/* Optional record of a decode for the parity tests: the margin of every
 * step's decision (how far the logits could move before another token or
 * beam order would be chosen) and, for beam search, the beams after every
 * step. Not part of the reference; it only observes the loops below. */
typedef struct {
  float* margin;        /* [max_tokens] */
  int32_t* topp;        /* [max_tokens] 1 where the step drew from the top-p nucleus */
  int32_t* beam_toks;   /* [max_tokens][B][stride] */
  int32_t* beam_lens;   /* [max_tokens][B] */
  float* beam_scores;   /* [max_tokens][B] */
  int stride;           /* P + max_tokens */
  int steps;            /* out: steps executed */
} otrace;

/* Top-2 gap of scaled logits (optionally without one id). */
static float top2_gap(const float* lg, int V, float it, int skip) {
  float a = -INFINITY, b = -INFINITY;
  for (int i = 0; i < V; i++) {
    if (i == skip) continue;
    float s = lg[i] * it;
    if (s > a) { b = a; a = s; }
    else if (s > b) b = s;
  }
  return b == -INFINITY ? FLT_MAX : a - b;
}

/* Decision margin of sampleGreedyWithScratch on one row (decoder.go:1006-1034). */
static float greedy_margin(const float* lg, int V, int eot, float temperature, int suppress_nst, float thold) {
  float it = inv_temp(temperature);
  int arg = or_sample_greedy(lg, V, eot, temperature, 0, 0.f);
  float m;
  if (suppress_nst && eot >= 0 && eot < V && arg == eot) {
    float d = fabsf(lg[eot] + thold); /* the threshold test itself */
    m = lg[eot] < -thold ? top2_gap(lg, V, it, eot) : top2_gap(lg, V, it, -1);
    if (d < m) m = d;
  } else {
    m = top2_gap(lg, V, it, -1);
  }
  return m;
}

/* model/decoder.go:413-525 (decodeGreedy) without a vocabulary (no
 * compression-ratio retry, :490). */
static int decode_greedy(const om* M, const ocross* cr, int T_enc, const int32_t* prompt, int P,
                         const wg_decode_params* p, int32_t* toks, int* len, int max_steps, otrace* tr, int utt) {
  ostate s;
  st_init(&s, M, T_enc);
  int mt = max_tokens_for(M, p, P);
  float temp = temperature_for(p);
  memcpy(toks, prompt, P * 4);
  int n = P, rc = 0;
  if (p->mode == WG_MODE_CORRECT) rc = prefill(M, &s, cr, T_enc, prompt, P);
  int streak = 0, prev = -1, steps = 0;
  float* cur = (float*)malloc((size_t)M->V * 4);
  while (!rc && n < P + mt && steps < max_steps) {
    rc = forward(M, &s, cr, T_enc, toks[n - 1], n - 1, p->mode, 1);
    if (rc) break;
    memcpy(cur, s.logits, (size_t)M->V * 4);
    or_apply_penalty(cur, M->V, toks, n, 2.0f, 128); /* :454-457 */
    if (p->suppress_eot && M->m->eot >= 0 && M->m->eot < M->V) cur[M->m->eot] = -INFINITY;
    int next = or_sample_greedy(cur, M->V, M->m->eot, temp, p->suppress_nst, p->no_speech_thold);
    if (tr) tr->margin[steps] = greedy_margin(cur, M->V, M->m->eot, temp, p->suppress_nst, p->no_speech_thold);
    if (p->logprob_thold > 0 && !p->no_fallback && temp > 0 &&      /* :1036-1056 */
        or_topp_fallback(cur, M->V, next, temp, p->logprob_thold)) {
      next = or_sample_topp(cur, M->V, temp, 0.9f, wg_uniform(p->seed, (uint32_t)utt, (uint32_t)steps));
      if (tr) tr->topp[steps] = 1;
    }
    toks[n++] = next;
    steps++;
    if (next == M->m->eot) break;     /* :470 */
    if (prev == next) streak++;        /* :475-484 */
    else { streak = 1; prev = next; }
    if (streak > 20) break;
  }
  free(cur);
  st_free(&s);
  *len = n;
  if (tr) tr->steps = steps;
  return rc;
}

typedef struct { int parent; float score; int32_t token; float logprob, norm; int carried; } ocand;

/* model/decoder.go:528-726 (decodeBeamSearch) without a vocabulary. */
static int decode_beam(const om* M, const ocross* cr, int T_enc, const int32_t* prompt, int P,
                       const wg_decode_params* p, int32_t* out_toks, int* out_len, float* out_score,
                       int max_steps, otrace* tr) {
  int B = p->beam_size, ctxw = P + max_tokens_for(M, p, P) + 1;
  int mt = max_tokens_for(M, p, P);
  float temp = temperature_for(p);
  int eot = M->m->eot;
  ostate* st = (ostate*)calloc(B, sizeof(ostate));
  ostate* tmpst = (ostate*)calloc(B, sizeof(ostate));
  int32_t* toks = (int32_t*)malloc((size_t)B * ctxw * 4);
  int32_t* ntoks = (int32_t*)calloc((size_t)B * ctxw, 4);
  int* len = (int*)malloc(B * 4);
  int* nlen = (int*)calloc(B, 4);
  float* score = (float*)calloc(B, 4);
  float* nscore = (float*)calloc(B, 4);
  ocand* cands = (ocand*)malloc((size_t)B * 6 * sizeof(ocand));
  float* cur = (float*)malloc((size_t)M->V * 4);
  int rc = 0;
  size_t kv_elems = (size_t)M->L * 2 * M->H * M->ctx * M->hd;
  for (int b = 0; b < B; b++) {
    st_init(&st[b], M, T_enc);
    memcpy(toks + b * ctxw, prompt, P * 4);
    len[b] = P;
    if (p->mode == WG_MODE_CORRECT) {
      if (b == 0) rc = prefill(M, &st[0], cr, T_enc, prompt, P);
      else memcpy(st[b].kv, st[0].kv, kv_elems * 4);
    }
  }
  if (p->mode == WG_MODE_CORRECT)
    for (int b = 0; b < B; b++) tmpst[b].kv = (float*)malloc(kv_elems * 4);
  int step = 0;
  for (step = 0; !rc && step < mt && step < max_steps; step++) {
    int nc = 0;
    float margin = FLT_MAX;
    for (int b = 0; b < B; b++) {
      int32_t* tb = toks + b * ctxw;
      if (len[b] > 0 && tb[len[b] - 1] == eot) { /* :580-591 */
        ocand c = {b, score[b], eot, 0, score[b] / (float)pow((double)len[b], 0.6), 1};
        cands[nc++] = c;
        continue;
      }
      if (p->mode == WG_MODE_REF_COMPAT) {
        /* resetDecoderState (:372-386, called at :593): the whole cache is
         * zeroed; only slot 0 is ever read in this mode, and slots j>0 enter
         * with weight exactly 0, so zeroing slot 0 is equivalent. */
        for (int l = 0; l < M->L; l++)
          for (int kv = 0; kv < 2; kv++)
            for (int h = 0; h < M->H; h++)
              memset(st[b].kv + ((((size_t)l * 2 + kv) * M->H + h) * M->ctx) * M->hd, 0, M->hd * 4);
      }
      rc = forward(M, &st[b], cr, T_enc, tb[len[b] - 1], len[b] - 1, p->mode, 1);
      if (rc) break;
      memcpy(cur, st[b].logits, (size_t)M->V * 4);
      or_apply_penalty(cur, M->V, tb, len[b], 2.0f, 128); /* :600-603 */
      if (p->suppress_eot && eot >= 0 && eot < M->V) cur[eot] = -INFINITY;
      int32_t tk[5]; float lp[5];
      int k = or_topk(cur, M->V, 5, temp, tk, lp); /* :606-608 */
      if (tr) { /* the 5th / 6th boundary of this row's candidates */
        int32_t tk6[6]; float lp6[6];
        if (or_topk(cur, M->V, 6, temp, tk6, lp6) == 6 && lp6[4] - lp6[5] < margin) margin = lp6[4] - lp6[5];
      }
      for (int j = 0; j < k; j++) {                /* :610-622 */
        int newLen = len[b] + 1;
        float ns = score[b] + lp[j];
        ocand c = {b, ns, tk[j], lp[j], ns / (float)pow((double)newLen, 0.6), 0};
        cands[nc++] = c;
      }
    }
    if (rc) break;
    /* sortAndPruneBeams (:1462-1475); stable here */
    for (int i = 1; i < nc; i++) {
      ocand c = cands[i]; int j = i - 1;
      while (j >= 0 && cands[j].norm < c.norm) { cands[j + 1] = cands[j]; j--; }
      cands[j + 1] = c;
    }
    int nb = nc < B ? nc : B;
    if (tr) { /* order of the kept candidates and the kept / dropped boundary */
      int lim = nc < B + 1 ? nc : B + 1;
      for (int i = 0; i + 1 < lim; i++)
        if (cands[i].norm - cands[i + 1].norm < margin) margin = cands[i].norm - cands[i + 1].norm;
      tr->margin[step] = margin;
    }
    /* rebuild beams (:629-660) */
    for (int i = 0; i < nb; i++) {
      const ocand* c = &cands[i];
      int32_t* src = toks + c->parent * ctxw;
      int32_t* dst = ntoks + i * ctxw;
      int pl = len[c->parent];
      memcpy(dst, src, pl * 4);
      if (pl > 0 && src[pl - 1] == eot && c->token == eot && c->logprob == 0) nlen[i] = pl;
      else { dst[pl] = c->token; nlen[i] = pl + 1; }
      nscore[i] = c->score;
      if (p->mode == WG_MODE_CORRECT) memcpy(tmpst[i].kv, st[c->parent].kv, kv_elems * 4);
    }
    if (p->mode == WG_MODE_CORRECT)
      for (int i = 0; i < nb; i++) { float* t = st[i].kv; st[i].kv = tmpst[i].kv; tmpst[i].kv = t; }
    memcpy(toks, ntoks, (size_t)B * ctxw * 4);
    memcpy(len, nlen, (size_t)B * 4);
    memcpy(score, nscore, (size_t)B * 4);
    B = nb; /* beams = nextBeams (len(bestCandidates)) */
    if (tr) {
      const int B0 = p->beam_size;
      for (int b = 0; b < B0; b++) {
        int32_t* dst = tr->beam_toks + ((int64_t)step * B0 + b) * tr->stride;
        memset(dst, 0, (size_t)tr->stride * 4);
        if (b < B) memcpy(dst, toks + b * ctxw, (size_t)(len[b] < tr->stride ? len[b] : tr->stride) * 4);
        tr->beam_lens[step * B0 + b] = b < B ? len[b] : 0;
        tr->beam_scores[step * B0 + b] = b < B ? score[b] : 0.f;
      }
      tr->steps = step + 1;
    }
    int allEOT = 1; /* :662-672 */
    for (int b = 0; b < B; b++) if (len[b] == 0 || toks[b * ctxw + len[b] - 1] != eot) { allEOT = 0; break; }
    if (allEOT) break;
    if (B > 0 && len[0] >= 2) { /* :675-691 */
      int32_t* t0 = toks;
      int32_t last = t0[len[0] - 1];
      int streak = 1, stop = 0;
      for (int i = len[0] - 2; i >= 0 && t0[i] == last; i--) {
        streak++;
        if (streak > 20) { stop = 1; break; }
      }
      if (stop) break;
    }
  }
  if (B > 0) { memcpy(out_toks, toks, len[0] * 4); *out_len = len[0]; *out_score = score[0]; }
  else { *out_len = 0; *out_score = 0; }
  for (int b = 0; b < p->beam_size; b++) {
    st_free(&st[b]);
    if (p->mode == WG_MODE_CORRECT) free(tmpst[b].kv);
  }
  free(st); free(tmpst); free(toks); free(ntoks); free(len); free(nlen);
  free(score); free(nscore); free(cands); free(cur);
  return rc;
}

static int check_params(const om* M, const wg_decode_params* p, int P) {
  if (P <= 0) return WG_ERR_INVALID;
  if (p->mode != WG_MODE_REF_COMPAT && p->mode != WG_MODE_CORRECT) return WG_ERR_INVALID;
  if (P > M->ctx) return WG_ERR_INVALID;
  return 0;
}

/* Decode U utterances (each like one Decode call), utterances in parallel
 * over nthreads host threads. tokens: U x (P + max_tokens). */
static int decode_all(const wg_model_desc* m, const float* const* enc, int U, int T_enc,
                      const int32_t* prompt, int P, const wg_decode_params* p, int32_t* tokens,
                      int32_t* lens, float* scores, int nthreads, otrace* trs);

OR_API int or_decode(const wg_model_desc* m, const float* const* enc, int U, int T_enc,
                     const int32_t* prompt, int P, const wg_decode_params* p, int32_t* tokens,
                     int32_t* lens, float* scores, int nthreads) {
  return decode_all(m, enc, U, T_enc, prompt, P, p, tokens, lens, scores, nthreads, NULL);
}

/* or_decode plus the per-step record of every utterance (otrace): margins
 * [U][max_tokens]; for beam search the beams after each step, tokens
 * [U][max_tokens][B][P + max_tokens], lens and scores [U][max_tokens][B];
 * steps [U] = steps executed. */
OR_API int or_decode_trace(const wg_model_desc* m, const float* const* enc, int U, int T_enc,
                           const int32_t* prompt, int P, const wg_decode_params* p, int32_t* tokens,
                           int32_t* lens, float* scores, int nthreads, float* margins, int32_t* beam_toks,
                           int32_t* beam_lens, float* beam_scores, int32_t* steps, int32_t* topp) {
  om M;
  int rc = om_init(&M, m);
  if (rc) return rc;
  int mt = max_tokens_for(&M, p, P), B = p->beam_size > 1 ? p->beam_size : 1, stride = P + mt;
  otrace* trs = (otrace*)calloc(U, sizeof(otrace));
  for (int u = 0; u < U; u++) {
    trs[u].margin = margins + (int64_t)u * mt;
    trs[u].topp = topp + (int64_t)u * mt;
    for (int i = 0; i < mt; i++) { trs[u].margin[i] = FLT_MAX; trs[u].topp[i] = 0; }
    if (B > 1) {
      trs[u].beam_toks = beam_toks + (int64_t)u * mt * B * stride;
      trs[u].beam_lens = beam_lens + (int64_t)u * mt * B;
      trs[u].beam_scores = beam_scores + (int64_t)u * mt * B;
    }
    trs[u].stride = stride;
  }
  rc = decode_all(m, enc, U, T_enc, prompt, P, p, tokens, lens, scores, nthreads, trs);
  for (int u = 0; u < U; u++) steps[u] = trs[u].steps;
  free(trs);
  return rc;
}

static int decode_all(const wg_model_desc* m, const float* const* enc, int U, int T_enc,
                      const int32_t* prompt, int P, const wg_decode_params* p, int32_t* tokens,
                      int32_t* lens, float* scores, int nthreads, otrace* trs) {
  om M;
  int rc = om_init(&M, m);
  if (rc) return rc;
  if ((rc = check_params(&M, p, P))) return rc;
  int mt = max_tokens_for(&M, p, P);
  int stride = P + mt;
  int err = 0;
#pragma omp parallel for schedule(dynamic, 1) num_threads(nthreads < 1 ? 1 : nthreads)
  for (int u = 0; u < U; u++) {
    ocross* cr = (ocross*)calloc(M.L, sizeof(ocross));
    cross_precompute(&M, enc[u], T_enc, cr, 0);
    int len = 0, r;
    float sc = 0;
    int32_t* buf = (int32_t*)calloc((size_t)stride + 1, 4);
    if (p->beam_size > 1)
      r = decode_beam(&M, cr, T_enc, prompt, P, p, buf, &len, &sc, 1 << 30, trs ? &trs[u] : NULL);
    else
      r = decode_greedy(&M, cr, T_enc, prompt, P, p, buf, &len, 1 << 30, trs ? &trs[u] : NULL, u);
    if (r) {
#pragma omp atomic write
      err = r;
    }
    memset(tokens + (int64_t)u * stride, 0, (size_t)stride * 4);
    memcpy(tokens + (int64_t)u * stride, buf, (size_t)(len < stride ? len : stride) * 4);
    lens[u] = len;
    if (scores) scores[u] = sc;
    free(buf);
    cross_free(&M, cr);
    free(cr);
  }
  return err;
}

/* Teacher forcing through decodeGreedy's forward calls (decoder.go:441-447):
 * step s runs forward on the last token of prompt+forced[0..s) at position
 * P-1+s and stores the raw logits. */
OR_API int or_teacher_forced(const wg_model_desc* m, const float* enc, int T_enc,
                             const int32_t* prompt, int P, const int32_t* forced, int n_forced,
                             int mode, float* logits) {
  om M;
  int rc = om_init(&M, m);
  if (rc) return rc;
  if (P <= 0 || P + n_forced > M.ctx + 1) return WG_ERR_INVALID;
  ocross* cr = (ocross*)calloc(M.L, sizeof(ocross));
  cross_precompute(&M, enc, T_enc, cr, 0);
  ostate s;
  st_init(&s, &M, T_enc);
  if (mode == WG_MODE_CORRECT) rc = prefill(&M, &s, cr, T_enc, prompt, P);
  int32_t* seq = (int32_t*)malloc((size_t)(P + n_forced) * 4);
  memcpy(seq, prompt, P * 4);
  memcpy(seq + P, forced, (size_t)n_forced * 4);
  for (int st = 0; !rc && st < n_forced; st++) {
    int pos = P - 1 + st;
    rc = forward(&M, &s, cr, T_enc, seq[pos], pos, mode, 1);
    if (!rc) memcpy(logits + (int64_t)st * M.V, s.logits, (size_t)M.V * 4);
  }
  free(seq);
  st_free(&s);
  cross_free(&M, cr);
  free(cr);
  return rc;
}

/* CPU baseline timing: U utterances over nthreads threads (one utterance per
 * thread at a time, GEMVs serial as in the reference), n_steps token steps
 * each. The cross K/V precompute is outside the timed region and filled with
 * synthetic values (its values do not change the step loop's cost).
 * Returns the wall seconds of the step loops and the token steps executed. */
OR_API int or_bench_steps(const wg_model_desc* m, int U, int T_enc, const int32_t* prompt, int P,
                          const wg_decode_params* p, int n_steps, int nthreads, double* seconds,
                          int64_t* tokens_done) {
  om M;
  int rc = om_init(&M, m);
  if (rc) return rc;
  if ((rc = check_params(&M, p, P))) return rc;
  int saved_inner = g_inner_threads;
  g_inner_threads = 1;
  ocross** crs = (ocross**)calloc(U, sizeof(ocross*));
  for (int u = 0; u < U; u++) {
    crs[u] = (ocross*)calloc(M.L, sizeof(ocross));
    cross_precompute(&M, NULL, T_enc, crs[u], 1);
  }
  int mt = max_tokens_for(&M, p, P);
  int64_t done = 0;
  double t0 = omp_get_wtime();
#pragma omp parallel for schedule(dynamic, 1) num_threads(nthreads < 1 ? 1 : nthreads) reduction(+ : done)
  for (int u = 0; u < U; u++) {
    int32_t* buf = (int32_t*)calloc((size_t)P + mt + 1, 4);
    int len = 0;
    float sc = 0;
    if (p->beam_size > 1) decode_beam(&M, crs[u], T_enc, prompt, P, p, buf, &len, &sc, n_steps, NULL);
    else decode_greedy(&M, crs[u], T_enc, prompt, P, p, buf, &len, n_steps, NULL, u);
    done += len - P;
    free(buf);
  }
  *seconds = omp_get_wtime() - t0;
  *tokens_done = done;
  for (int u = 0; u < U; u++) { cross_free(&M, crs[u]); free(crs[u]); }
  free(crs);
  g_inner_threads = saved_inner;
  return 0;
}
