// gemv_frag.cuh — mma.m16n8k16 fragments of the dequant GEMV kernels
// (gemm.cu streaming kernels, gemv_bulk.cu): one lane's share of a
// (tile, block) payload in the tile128 layout, its dequantisation into f16 A
// fragments, and the scalar Epi store.
#pragma once

#include "kernels.cuh"

namespace wg {
namespace {

__device__ __forceinline__ void mma16816(float* c, const uint32_t* a, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t h2_as_u32(__half2 h) {
  uint32_t u;
  memcpy(&u, &h, 4);
  return u;
}
__device__ __forceinline__ __half2 u32_as_h2(uint32_t u) {
  __half2 h;
  memcpy(&h, &u, 4);
  return h;
}

// One lane's share of one (tile, block).
struct Pay {
  uint4 q;
  uint32_t hb;
  __half2 d, m;
};

__device__ __forceinline__ uint4 ldg_stream16(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}
__device__ __forceinline__ uint2 ldg_stream8(const void* p) {
  uint2 v;
  asm volatile("ld.global.nc.L1::no_allocate.v2.u32 {%0,%1}, [%2];" : "=r"(v.x), "=r"(v.y) : "l"(p));
  return v;
}

template <uint32_t QT>
__device__ __forceinline__ Pay load_payload(const DMat& W, int64_t slot, int lane) {
  Pay p;
  if (QT == WG_QTYPE_Q8_0) {
    p.q = ldg_stream16(W.qs + (slot * 32 + lane) * 16);
  } else {
    uint2 v = ldg_stream8(W.qs + (slot * 32 + lane) * 8);
    p.q = make_uint4(v.x, v.y, 0, 0);
  }
  p.d = W.dsc[slot * 8 + (lane >> 2)];
  if (QT == WG_QTYPE_Q4_1 || QT == WG_QTYPE_Q5_1) p.m = W.msc[slot * 8 + (lane >> 2)];
  else p.m = __float2half2_rn(0.f);
  if (QT == WG_QTYPE_Q5_0 || QT == WG_QTYPE_Q5_1) p.hb = W.hb[slot * 32 + lane];
  else p.hb = 0;
  return p;
}

// A fragment of mma step s (0/1) of a 32-wide quant block.
// reg 0: row g, k 2t..2t+1; reg 1: row g+8; reg 2: row g, k+8; reg 3: row g+8, k+8.
template <uint32_t QT>
__device__ __forceinline__ void dequant_step(const Pay& p, int s, uint32_t* a) {
  const __half2 dg = __low2half2(p.d), dg8 = __high2half2(p.d);
  if (QT == WG_QTYPE_Q8_0) {
    uint32_t w0 = (s ? p.q.z : p.q.x) ^ 0x80808080u;
    uint32_t w1 = (s ? p.q.w : p.q.y) ^ 0x80808080u;
    const __half2 bias = __float2half2_rn(1152.f);  // 1024 + 128
    __half2 h0 = __hsub2(u32_as_h2(__byte_perm(w0, 0x64, 0x4140)), bias);
    __half2 h1 = __hsub2(u32_as_h2(__byte_perm(w0, 0x64, 0x4342)), bias);
    __half2 h2 = __hsub2(u32_as_h2(__byte_perm(w1, 0x64, 0x4140)), bias);
    __half2 h3 = __hsub2(u32_as_h2(__byte_perm(w1, 0x64, 0x4342)), bias);
    a[0] = h2_as_u32(__hmul2(h0, dg));
    a[1] = h2_as_u32(__hmul2(h1, dg8));
    a[2] = h2_as_u32(__hmul2(h2, dg));
    a[3] = h2_as_u32(__hmul2(h3, dg8));
  } else {
    uint32_t w = s ? p.q.y : p.q.x;
#pragma unroll
    for (int r = 0; r < 4; r++) {
      uint32_t hq = ((w >> (4 * r)) & 0x000F000Fu) | 0x64006400u;
      if (QT == WG_QTYPE_Q5_0 || QT == WG_QTYPE_Q5_1) {
        uint32_t b = (p.hb >> (2 * (4 * s + r))) & 3u;
        hq |= ((b & 1u) << 4) | ((b >> 1) << 20);
      }
      const __half2 d = (r & 1) ? dg8 : dg;
      __half2 v;
      if (QT == WG_QTYPE_Q4_0) v = __hmul2(__hsub2(u32_as_h2(hq), __float2half2_rn(1032.f)), d);
      else if (QT == WG_QTYPE_Q5_0) v = __hmul2(__hsub2(u32_as_h2(hq), __float2half2_rn(1040.f)), d);
      else {
        const __half2 m = (r & 1) ? __high2half2(p.m) : __low2half2(p.m);
        v = __hfma2(__hsub2(u32_as_h2(hq), __float2half2_rn(1024.f)), d, m);
      }
      a[r] = h2_as_u32(v);
    }
  }
}

// Split dequantisation: the weight value v exactly as the reference
// computes it in float32 (d*q, d*(q-8), d*(q-16), or d*q + m with two
// float32 roundings; matmul_q8.go:237-429, dequant.go:92-201) as hi + lo / 2^10
// with hi = f16(v) and lo = f16((v - hi) * 2^10) (scaled, so lo stays a
// normal f16 number for |v| >= 2^-8, and hi * 2^10 stays finite for
// |v| < 64). hi carries v to 11 bits, hi + lo/2^10 to ~22 bits, beyond the
// float32 products' 19 significant bits for Q8_0, so the f16 tensor-core
// products lose nothing against the reference's float32 weights.
constexpr float SPLIT_SCALE = 1024.f, SPLIT_INV = 1.f / 1024.f;
template <uint32_t QT>
__device__ __forceinline__ void dequant_step_split(const Pay& p, int s, uint32_t* a, uint32_t* lo) {
  const __half2 dg = __low2half2(p.d), dg8 = __high2half2(p.d);
  if (QT == WG_QTYPE_Q8_0 || QT == WG_QTYPE_Q4_0 || QT == WG_QTYPE_Q5_0) {
    // q * d is a product of two f16 values: hi = its f16 rounding (one
    // hmul), and (q * d - hi) * 2^10 = fma(q, d * 2^10, -hi * 2^10) in f16
    // (both scalings exact)
    const __half2 sc = __float2half2_rn(SPLIT_SCALE);
    const __half2 dgs = __hmul2(dg, sc), dg8s = __hmul2(dg8, sc);
    __half2 qv[4];
    if (QT == WG_QTYPE_Q8_0) {
      uint32_t w0 = (s ? p.q.z : p.q.x) ^ 0x80808080u;
      uint32_t w1 = (s ? p.q.w : p.q.y) ^ 0x80808080u;
      const __half2 bias = __float2half2_rn(1152.f);
      qv[0] = __hsub2(u32_as_h2(__byte_perm(w0, 0x64, 0x4140)), bias);
      qv[1] = __hsub2(u32_as_h2(__byte_perm(w0, 0x64, 0x4342)), bias);
      qv[2] = __hsub2(u32_as_h2(__byte_perm(w1, 0x64, 0x4140)), bias);
      qv[3] = __hsub2(u32_as_h2(__byte_perm(w1, 0x64, 0x4342)), bias);
    } else {
      uint32_t w = s ? p.q.y : p.q.x;
#pragma unroll
      for (int r = 0; r < 4; r++) {
        uint32_t hq = ((w >> (4 * r)) & 0x000F000Fu) | 0x64006400u;
        if (QT == WG_QTYPE_Q5_0) {
          uint32_t b = (p.hb >> (2 * (4 * s + r))) & 3u;
          hq |= ((b & 1u) << 4) | ((b >> 1) << 20);
        }
        qv[r] = __hsub2(u32_as_h2(hq), __float2half2_rn(QT == WG_QTYPE_Q4_0 ? 1032.f : 1040.f));
      }
    }
#pragma unroll
    for (int r = 0; r < 4; r++) {
      const __half2 d = (r & 1) ? dg8 : dg, ds = (r & 1) ? dg8s : dgs;
      const __half2 hi = __hmul2(qv[r], d);
      a[r] = h2_as_u32(hi);
      lo[r] = h2_as_u32(__hfma2(qv[r], ds, __hneg2(__hmul2(hi, sc))));
    }
  } else {  // Q4_1 / Q5_1: v = float32(float32(d * q) + m), then the split in float32
    uint32_t w = s ? p.q.y : p.q.x;
#pragma unroll
    for (int r = 0; r < 4; r++) {
      uint32_t hq = ((w >> (4 * r)) & 0x000F000Fu) | 0x64006400u;
      if (QT == WG_QTYPE_Q5_1) {
        uint32_t b = (p.hb >> (2 * (4 * s + r))) & 3u;
        hq |= ((b & 1u) << 4) | ((b >> 1) << 20);
      }
      const float2 q = __half22float2(__hsub2(u32_as_h2(hq), __float2half2_rn(1024.f)));
      const float2 d = __half22float2((r & 1) ? dg8 : dg);
      const float2 m = __half22float2((r & 1) ? __high2half2(p.m) : __low2half2(p.m));
      const float v0 = __fadd_rn(__fmul_rn(d.x, q.x), m.x), v1 = __fadd_rn(__fmul_rn(d.y, q.y), m.y);
      const __half2 hi = __floats2half2_rn(v0, v1);
      const float2 h = __half22float2(hi);
      a[r] = h2_as_u32(hi);
      lo[r] = h2_as_u32(__floats2half2_rn(__fmul_rn(__fsub_rn(v0, h.x), SPLIT_SCALE),
                                          __fmul_rn(__fsub_rn(v1, h.y), SPLIT_SCALE)));
    }
  }
}

// Bias added to output column n (model data, never written by the token
// loop, so kernels may read it before their dependency wait).
__device__ __forceinline__ float epi_bias(const Epi& e, int n) {
  switch (e.mode) {
    case EPI_QKV: {
      const int seg = n / e.d, j = n - seg * e.d;
      return seg == 0 ? e.bias_q[j] : (seg == 2 ? e.bias_v[j] : 0.f);
    }
    case EPI_CROSS_KV: {
      const int lk = n / e.d, j = n - lk * e.d;
      return (lk & 1) ? e.bias_v[(int64_t)(lk >> 1) * e.d + j] : 0.f;
    }
    default:
      return e.bias ? e.bias[n] : 0.f;
  }
}

// Stores v (+ bias b of column n) of activation row r; pos is the decode
// position (*e.pos) for the KV-cache scatter of EPI_QKV.
__device__ __forceinline__ void epi_store_b(const Epi& e, int r, int n, float v, float b, int pos) {
  switch (e.mode) {
    case EPI_F32:
      if (e.bias) v = __fadd_rn(v, b);
      e.out[(int64_t)r * e.ldo + n] = v;
      break;
    case EPI_RESID: {
      // x += (acc + b): one writer per element, so the fire-and-forget
      // reduction rounds exactly like load-add-store without waiting on x
      const float add = __fadd_rn(v, b);
      asm volatile("red.global.add.f32 [%0], %1;" ::"l"(e.out + (int64_t)r * e.ldo + n), "f"(add) : "memory");
      break;
    }
    case EPI_GELU_F16:
      if (e.bias) v = __fadd_rn(v, b);
      e.out16[(int64_t)r * e.ldo + n] = __float2half_rn(gelu_f32(v));
      break;
    case EPI_QKV: {
      int seg = n / e.d, j = n - seg * e.d, h = j / e.hd, c = j - h * e.hd;
      if (seg == 0) {
        e.out[(int64_t)r * e.ldo + j] = __fadd_rn(v, b);
      } else {
        if (seg == 2) v = __fadd_rn(v, b);
        e.kv[((((int64_t)r * 2 + (seg - 1)) * e.H + h) * e.T + pos) * e.hd + c] = __float2half_rn(v);
      }
      break;
    }
    case EPI_CROSS_KV: {
      int u = r / e.T, tt = r - u * e.T;
      int lk = n / e.d, j = n - lk * e.d, l = lk >> 1, kv = lk & 1, h = j / e.hd, c = j - h * e.hd;
      if (kv) v = __fadd_rn(v, b);
      e.kv[(((((int64_t)l * e.U + u) * 2 + kv) * e.H + h) * e.T + tt) * e.hd + c] = __float2half_rn(v);
      break;
    }
  }
}

__device__ __forceinline__ void epi_store(const Epi& e, int r, int n, float v) {
  epi_store_b(e, r, n, v, epi_bias(e, n), e.mode == EPI_QKV ? *e.pos : 0);
}

}  // namespace
}  // namespace wg
