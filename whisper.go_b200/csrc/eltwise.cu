// eltwise.cu — embedding gather and LayerNorm of the decoder token loop.
#include "kernels.cuh"

namespace wg {
namespace {

// Exact fp32 dequantisation of element (r, k) of a device matrix
// (internal/gguf/dequant.go:92-201 through the tile128 layout).
__device__ __forceinline__ float dmat_elem(const DMat& m, int r, int k) {
  if (m.qtype == WG_QTYPE_F32) return reinterpret_cast<const float*>(m.qs)[(int64_t)r * m.cols + k];
  if (m.qtype == WG_QTYPE_F16) return __half2float(reinterpret_cast<const __half*>(m.qs)[(int64_t)r * m.cols + k]);
  int tile = r >> 4, gg = r & 15, g = gg & 7, hi = gg >> 3;
  int kb = k >> 5, kk = k & 31, s = kk >> 4, kr = kk & 15;
  int t = kr >> 2, e = kr & 1, reg = (((kr >> 1) & 1) << 1) | hi;
  int lane = g * 4 + t;
  int64_t slot = slot_of(m, tile, kb);
  __half2 dd = m.dsc[slot * 8 + g];
  float d = __half2float(hi ? __high2half(dd) : __low2half(dd));
  if (m.qtype == WG_QTYPE_Q8_0) {
    int8_t q = (int8_t)m.qs[(slot * 32 + lane) * 16 + s * 8 + reg * 2 + e];
    return __fmul_rn(d, (float)q);
  }
  uint2 w2 = reinterpret_cast<const uint2*>(m.qs)[slot * 32 + lane];
  uint32_t w = s ? w2.y : w2.x;
  uint32_t q = (w >> (e ? 16 + 4 * reg : 4 * reg)) & 0xF;
  if (m.hb) q |= (((uint32_t)m.hb[slot * 32 + lane] >> (2 * (4 * s + reg) + e)) & 1u) << 4;
  if (m.qtype == WG_QTYPE_Q4_0) return __fmul_rn(d, (float)((int)q - 8));
  if (m.qtype == WG_QTYPE_Q5_0) return __fmul_rn(d, (float)((int)q - 16));
  __half2 mm = m.msc[slot * 8 + g];
  float mn = __half2float(hi ? __high2half(mm) : __low2half(mm));
  return __fadd_rn(__fmul_rn(d, (float)q), mn);
}

// x[r] = tokEmb[tok[r]] + posEmb[pos] (decoder.go:756-773). The embedding row
// is read from the quantised matrix (the reference reads only the dense
// tensor, which is empty when the embedding is quantised, decoder.go:761-766).
__global__ void embed_kernel(DMat te, const float* __restrict__ pos_emb, const int* __restrict__ tokens,
                             const int* __restrict__ pos, int pos_offset, int d, float* __restrict__ x) {
  pdl_trigger();
  pdl_wait();
  int r = blockIdx.x;
  int tok = tokens[r];
  int p = *pos + pos_offset;
  if (tok < 0 || tok >= te.rows) tok = 0;  // guarded: ids are validated on the host
  for (int i = threadIdx.x; i < d; i += blockDim.x)
    x[(int64_t)r * d + i] = __fadd_rn(dmat_elem(te, tok, i), pos_emb[(int64_t)p * d + i]);
}

// internal/ml/ops.go:153-202 (LayerNormInto): two-pass mean / variance in
// fp32, std = float32(sqrt(float64(var + eps))) (== IEEE sqrtf),
// out = w*(v-mean)/std + b. One warp per row.
__global__ void layernorm_kernel(const float* __restrict__ x, const float* __restrict__ w,
                                 const float* __restrict__ b, int R, int d, __half* __restrict__ out16,
                                 int ld16, float* __restrict__ out32) {
  pdl_trigger();
  pdl_wait();
  int r = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  int lane = threadIdx.x & 31;
  if (r >= R) return;
  const float* xr = x + (int64_t)r * d;
  float s = 0.f;
  for (int i = lane; i < d; i += 32) s += xr[i];
  s = warp_sum(s);
  float mean = __fdiv_rn(s, (float)d);
  float v = 0.f;
  for (int i = lane; i < d; i += 32) {
    float dd = __fsub_rn(xr[i], mean);
    v = __fmaf_rn(dd, dd, v);
  }
  v = warp_sum(v);
  float var = __fdiv_rn(v, (float)d);
  float sd = __fsqrt_rn(__fadd_rn(var, 1e-5f));
  for (int i = lane; i < d; i += 32) {
    float o = __fadd_rn(__fdiv_rn(__fmul_rn(w[i], __fsub_rn(xr[i], mean)), sd), b[i]);
    if (out16) out16[(int64_t)r * ld16 + i] = __float2half_rn(o);
    if (out32) out32[(int64_t)r * d + i] = o;
  }
}

// Same arithmetic with the row held in registers (d == 128 * NV): one read
// of x instead of three dependent passes. gamma and beta are model data,
// never written by the token loop, so each lane loads its share of them
// before the dependency wait and only the read of x follows it.
template <int NV>
__global__ void layernorm_reg_kernel(const float* __restrict__ x, const float* __restrict__ w,
                                     const float* __restrict__ b, int R, __half* __restrict__ out16, int ld16,
                                     float* __restrict__ out32) {
  pdl_trigger();
  constexpr int d = NV * 128;
  const int r = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  const float4* w4 = reinterpret_cast<const float4*>(w);
  const float4* b4 = reinterpret_cast<const float4*>(b);
  float4 wv[NV], bw[NV];
#pragma unroll
  for (int i = 0; i < NV; i++) {
    wv[i] = w4[lane + 32 * i];
    bw[i] = b4[lane + 32 * i];
  }
  pdl_wait();
  if (r >= R) return;
  const float4* xr = reinterpret_cast<const float4*>(x + (int64_t)r * d);
  float4 v[NV];
#pragma unroll
  for (int i = 0; i < NV; i++) v[i] = xr[lane + 32 * i];
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < NV; i++) s += (v[i].x + v[i].y) + (v[i].z + v[i].w);
  s = warp_sum(s);
  const float mean = __fdiv_rn(s, (float)d);
  float q = 0.f;
#pragma unroll
  for (int i = 0; i < NV; i++) {
    float a = __fsub_rn(v[i].x, mean), bb = __fsub_rn(v[i].y, mean), c = __fsub_rn(v[i].z, mean),
          e = __fsub_rn(v[i].w, mean);
    q = __fmaf_rn(a, a, q);
    q = __fmaf_rn(bb, bb, q);
    q = __fmaf_rn(c, c, q);
    q = __fmaf_rn(e, e, q);
  }
  q = warp_sum(q);
  const float sd = __fsqrt_rn(__fadd_rn(__fdiv_rn(q, (float)d), 1e-5f));
#pragma unroll
  for (int i = 0; i < NV; i++) {
    const int c4 = lane + 32 * i;
    const float4 ww = wv[i], bv = bw[i];
    float4 o;
    o.x = __fadd_rn(__fdiv_rn(__fmul_rn(ww.x, __fsub_rn(v[i].x, mean)), sd), bv.x);
    o.y = __fadd_rn(__fdiv_rn(__fmul_rn(ww.y, __fsub_rn(v[i].y, mean)), sd), bv.y);
    o.z = __fadd_rn(__fdiv_rn(__fmul_rn(ww.z, __fsub_rn(v[i].z, mean)), sd), bv.z);
    o.w = __fadd_rn(__fdiv_rn(__fmul_rn(ww.w, __fsub_rn(v[i].w, mean)), sd), bv.w);
    if (out16) {
      __half2 h0 = __floats2half2_rn(o.x, o.y), h1 = __floats2half2_rn(o.z, o.w);
      uint2 u;
      memcpy(&u.x, &h0, 4);
      memcpy(&u.y, &h1, 4);
      *reinterpret_cast<uint2*>(out16 + (int64_t)r * ld16 + 4 * c4) = u;
    }
    if (out32) reinterpret_cast<float4*>(out32 + (int64_t)r * d)[c4] = o;
  }
}

__global__ void f32_to_f16_kernel(const float* __restrict__ in, __half* __restrict__ out, int64_t n) {
  int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (; i < n; i += stride) out[i] = __float2half_rn(in[i]);
}

}  // namespace

int launch_embed(const DMat& te, const float* pos_emb, const int* tokens, const int* pos, int pos_offset, int R,
                 int d, float* x, cudaStream_t st) {
  return launch_check(launch_k(embed_kernel, dim3(R), dim3(256), 0, st, te, pos_emb, tokens, pos, pos_offset, d, x),
                      "embed");
}

bool layernorm_uses_vec(int d) { return d == 384 || d == 512 || d == 768 || d == 1024 || d == 1280; }

int launch_layernorm(const float* x, const float* w, const float* b, int R, int d, __half* out16, float* out32,
                     cudaStream_t st) {
  int ld16 = (d + 7) / 8 * 8;
  const unsigned grid = (R + 7) / 8;
  cudaError_t e;
  switch (d) {
    case 384: e = launch_k(layernorm_reg_kernel<3>, dim3(grid), dim3(256), 0, st, x, w, b, R, out16, ld16, out32); break;
    case 512: e = launch_k(layernorm_reg_kernel<4>, dim3(grid), dim3(256), 0, st, x, w, b, R, out16, ld16, out32); break;
    case 768: e = launch_k(layernorm_reg_kernel<6>, dim3(grid), dim3(256), 0, st, x, w, b, R, out16, ld16, out32); break;
    case 1024: e = launch_k(layernorm_reg_kernel<8>, dim3(grid), dim3(256), 0, st, x, w, b, R, out16, ld16, out32); break;
    case 1280:
      e = launch_k(layernorm_reg_kernel<10>, dim3(grid), dim3(256), 0, st, x, w, b, R, out16, ld16, out32);
      break;
    default: e = launch_k(layernorm_kernel, dim3(grid), dim3(256), 0, st, x, w, b, R, d, out16, ld16, out32);
  }
  return launch_check(e, "layernorm");
}

int launch_f32_to_f16(const float* in, __half* out, int64_t n, cudaStream_t st) {
  int64_t blocks = (n + 255) / 256;
  if (blocks > 148 * 32) blocks = 148 * 32;
  f32_to_f16_kernel<<<(unsigned)blocks, 256, 0, st>>>(in, out, n);
  return launch_status("f32_to_f16");
}

}  // namespace wg
