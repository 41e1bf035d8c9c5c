// weights.cu — upload of raw GGUF tensors into the device "tile16" layout
// (see DMat in common.cuh) and the bit-exact device dequantiser.
//
// Block codecs follow internal/gguf/dequant.go:92-201 and the dot kernels of
// internal/ml/matmul_q8.go:237-429: interleaved nibbles (element 2i = low
// nibble of qs[i], element 2i+1 = high nibble), Q5 fifth bit i = bit i of
// the u32 qh, values d*(q-8) / d*q+m / d*(q5-16) / d*q5+m / d*q.
#include <vector>

#include "common.cuh"
#include "kernels.cuh"

namespace wg {

namespace {

__device__ __forceinline__ uint16_t rd16(const uint8_t* p) { return (uint16_t)(p[0] | (p[1] << 8)); }
__device__ __forceinline__ uint32_t rd32(const uint8_t* p) {
  return (uint32_t)p[0] | (uint32_t)p[1] << 8 | (uint32_t)p[2] << 16 | (uint32_t)p[3] << 24;
}

struct QOff { int qs, qh, m; };  // byte offsets inside one GGUF block (d is at 0)
__device__ __forceinline__ QOff qoff(uint32_t q) {
  switch (q) {
    case WG_QTYPE_Q4_0: return {2, -1, -1};
    case WG_QTYPE_Q4_1: return {4, -1, 2};
    case WG_QTYPE_Q5_0: return {6, 2, -1};
    case WG_QTYPE_Q5_1: return {8, 4, 2};
    default: return {2, -1, -1};  // Q8_0
  }
}

// One thread per (tile, block, lane). raw: rows_part x row_bytes GGUF bytes
// that land at tile offset tile0 of the destination.
__global__ void repack_tile16_kernel(uint32_t qtype, const uint8_t* __restrict__ raw, int rows_part,
                                     int64_t row_bytes, int kblocks, int tile0, int ntiles_part,
                                     DMat dst) {
  int64_t gid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  int64_t total = (int64_t)ntiles_part * kblocks * 32;
  if (gid >= total) return;
  int lane = (int)(gid & 31);
  int64_t tb = gid >> 5;
  int kb = (int)(tb % kblocks);
  int tile = (int)(tb / kblocks);
  int g = lane >> 2, t = lane & 3;
  int r0 = tile * 16 + g, r1 = r0 + 8;
  const int64_t bb = gguf_block_bytes(qtype);
  const QOff off = qoff(qtype);
  const uint8_t* b0 = r0 < rows_part ? raw + (int64_t)r0 * row_bytes + (int64_t)kb * bb : nullptr;
  const uint8_t* b1 = r1 < rows_part ? raw + (int64_t)r1 * row_bytes + (int64_t)kb * bb : nullptr;
  int64_t slot = slot_of(dst, tile0 + tile, kb);
  if (qtype == WG_QTYPE_Q8_0) {
    uint8_t pay[16];
#pragma unroll
    for (int j = 0; j < 16; j++) {
      int s = j >> 3, reg = (j & 7) >> 1, e = j & 1;
      const uint8_t* b = (reg & 1) ? b1 : b0;
      int k = 16 * s + 4 * t + 2 * (reg >> 1) + e;
      pay[j] = b ? b[off.qs + k] : 0;
    }
    uint4 v;
    memcpy(&v, pay, 16);
    reinterpret_cast<uint4*>(dst.qs)[slot * 32 + lane] = v;
  } else {
    uint32_t w[2] = {0, 0};
    uint32_t hbits = 0;
    uint32_t qh0 = (b0 && off.qh >= 0) ? rd32(b0 + off.qh) : 0;
    uint32_t qh1 = (b1 && off.qh >= 0) ? rd32(b1 + off.qh) : 0;
#pragma unroll
    for (int s = 0; s < 2; s++)
#pragma unroll
      for (int p = 0; p < 4; p++) {
        const uint8_t* b = (p & 1) ? b1 : b0;
        int k0 = 16 * s + 4 * t + 2 * (p >> 1);
        uint32_t byte = b ? b[off.qs + k0 / 2] : 0x00;
        w[s] |= (byte & 0xF) << (4 * p);
        w[s] |= (byte >> 4) << (16 + 4 * p);
        uint32_t qh = (p & 1) ? qh1 : qh0;
        int bit = 2 * (4 * s + p);
        hbits |= ((qh >> k0) & 1u) << bit;
        hbits |= ((qh >> (k0 + 1)) & 1u) << (bit + 1);
      }
    reinterpret_cast<uint2*>(dst.qs)[slot * 32 + lane] = make_uint2(w[0], w[1]);
    if (dst.hb) dst.hb[slot * 32 + lane] = (uint16_t)hbits;
  }
  if (t == 0) {
    uint16_t d0 = b0 ? rd16(b0) : 0, d1 = b1 ? rd16(b1) : 0;
    dst.dsc[slot * 8 + g] = __halves2half2(__ushort_as_half(d0), __ushort_as_half(d1));
    if (dst.msc) {
      uint16_t m0 = b0 ? rd16(b0 + off.m) : 0, m1 = b1 ? rd16(b1 + off.m) : 0;
      dst.msc[slot * 8 + g] = __halves2half2(__ushort_as_half(m0), __ushort_as_half(m1));
    }
  }
}

// Reads element (r, k) back out of the tile16 layout and dequantises it in
// fp32 exactly as internal/gguf/dequant.go does (products and the +m rounded
// separately; no fused multiply-add).
__global__ void dequant_tile16_kernel(DMat m, int64_t n_valid, float* __restrict__ out) {
  int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n_valid) return;
  int r = (int)(i / m.cols), k = (int)(i % m.cols);
  int tile = r >> 4, gg = r & 15, g = gg & 7, hi = gg >> 3;
  int kb = k >> 5, kk = k & 31, s = kk >> 4, kr = kk & 15;
  int t = kr >> 2, e = kr & 1, reg = (((kr >> 1) & 1) << 1) | hi;
  int lane = g * 4 + t;
  int64_t slot = slot_of(m, tile, kb);
  __half2 dd = m.dsc[slot * 8 + g];
  float d = __half2float(hi ? __high2half(dd) : __low2half(dd));
  float v;
  if (m.qtype == WG_QTYPE_Q8_0) {
    int8_t q = (int8_t)m.qs[(slot * 32 + lane) * 16 + s * 8 + reg * 2 + e];
    v = __fmul_rn(d, (float)q);
  } else {
    uint32_t w = reinterpret_cast<const uint2*>(m.qs)[slot * 32 + lane].x;
    if (s) w = reinterpret_cast<const uint2*>(m.qs)[slot * 32 + lane].y;
    uint32_t q = (w >> (e ? 16 + 4 * reg : 4 * reg)) & 0xF;
    if (m.hb) q |= (((uint32_t)m.hb[slot * 32 + lane] >> (2 * (4 * s + reg) + e)) & 1u) << 4;
    if (m.qtype == WG_QTYPE_Q4_0) v = __fmul_rn(d, (float)((int)q - 8));
    else if (m.qtype == WG_QTYPE_Q5_0) v = __fmul_rn(d, (float)((int)q - 16));
    else {
      __half2 mm = m.msc[slot * 8 + g];
      float mn = __half2float(hi ? __high2half(mm) : __low2half(mm));
      v = __fadd_rn(__fmul_rn(d, (float)q), mn);
    }
  }
  out[i] = v;
}

__global__ void dequant_dense_kernel(DMat m, int64_t n_valid, float* __restrict__ out) {
  int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n_valid) return;
  if (m.qtype == WG_QTYPE_F32) out[i] = reinterpret_cast<const float*>(m.qs)[i];
  else out[i] = __half2float(reinterpret_cast<const __half*>(m.qs)[i]);
}

}  // namespace

void free_dmat(DMat& m) {
  cudaFree(m.qs);
  cudaFree(m.dsc);
  cudaFree(m.msc);
  cudaFree(m.hb);
  m = DMat{};
}

int64_t dmat_device_bytes(const DMat& m) {
  if (!qtype_is_quant(m.qtype)) return (int64_t)m.rows * m.cols * (m.qtype == WG_QTYPE_F32 ? 4 : 2);
  int64_t slots = dmat_slots(m);
  int64_t b = slots * 32 * qtype_payload_bytes(m.qtype) + slots * 8 * 4;
  if (qtype_has_min(m.qtype)) b += slots * 8 * 4;
  if (qtype_has_hbits(m.qtype)) b += slots * 32 * 2;
  return b;
}

// Uploads the row-wise concatenation of parts (same qtype and cols) as one
// device matrix. Quantised parts other than the last must have rows % 16 == 0.
int upload_matrix(const wg_matrix* const* parts, int nparts, DMat* out, cudaStream_t st) {
  DMat m;
  if (nparts <= 0 || !parts[0]) { set_error("upload_matrix: no parts"); return WG_ERR_INVALID; }
  m.qtype = parts[0]->qtype;
  m.cols = parts[0]->cols;
  int rows = 0;
  for (int i = 0; i < nparts; i++) {
    const wg_matrix* p = parts[i];
    if (!p || !p->data || p->rows <= 0 || p->cols != m.cols || p->qtype != m.qtype) {
      set_error("upload_matrix: part %d has a missing buffer or a shape/type mismatch", i);
      return WG_ERR_INVALID;
    }
    if (qtype_is_quant(m.qtype) && i + 1 < nparts && p->rows % 16) {
      set_error("upload_matrix: concatenated quantised parts need rows %% 16 == 0");
      return WG_ERR_UNSUPPORTED;
    }
    rows += p->rows;
  }
  m.rows = rows;
  if (m.qtype == WG_QTYPE_F32 || m.qtype == WG_QTYPE_F16) {
    size_t esz = m.qtype == WG_QTYPE_F32 ? 4 : 2;
    WG_CHECK_CUDA(cudaMalloc(&m.qs, (size_t)rows * m.cols * esz));
    size_t offb = 0;
    for (int i = 0; i < nparts; i++) {
      size_t nb = (size_t)parts[i]->rows * m.cols * esz;
      WG_CHECK_CUDA(cudaMemcpyAsync(m.qs + offb, parts[i]->data, nb, cudaMemcpyHostToDevice, st));
      offb += nb;
    }
    WG_CHECK_CUDA(cudaStreamSynchronize(st));
    *out = m;
    return WG_OK;
  }
  if (!qtype_is_quant(m.qtype)) {
    set_error("upload_matrix: unsupported tensor type %u", m.qtype);
    return WG_ERR_UNSUPPORTED;
  }
  if (m.cols % 64) {
    set_error("upload_matrix: quantised matrices need cols %% 64 == 0 (got %d)", m.cols);
    return WG_ERR_UNSUPPORTED;
  }
  m.kblocks = m.cols / 32;
  m.ntiles = (rows + 15) / 16;
  int64_t slots = dmat_slots(m);
  int pb = qtype_payload_bytes(m.qtype);
  // padding tiles of the last 128-row group stay zero (scale 0 -> value 0)
  WG_CHECK_CUDA(cudaMalloc(&m.qs, (size_t)slots * 32 * pb));
  WG_CHECK_CUDA(cudaMemsetAsync(m.qs, 0, (size_t)slots * 32 * pb, st));
  WG_CHECK_CUDA(cudaMalloc(&m.dsc, (size_t)slots * 8 * sizeof(__half2)));
  WG_CHECK_CUDA(cudaMemsetAsync(m.dsc, 0, (size_t)slots * 8 * sizeof(__half2), st));
  if (qtype_has_min(m.qtype)) {
    WG_CHECK_CUDA(cudaMalloc(&m.msc, (size_t)slots * 8 * sizeof(__half2)));
    WG_CHECK_CUDA(cudaMemsetAsync(m.msc, 0, (size_t)slots * 8 * sizeof(__half2), st));
  }
  if (qtype_has_hbits(m.qtype)) {
    WG_CHECK_CUDA(cudaMalloc(&m.hb, (size_t)slots * 32 * 2));
    WG_CHECK_CUDA(cudaMemsetAsync(m.hb, 0, (size_t)slots * 32 * 2, st));
  }
  int64_t row_bytes = gguf_row_bytes(m.qtype, m.cols);
  size_t max_part = 0;
  for (int i = 0; i < nparts; i++) max_part = std::max(max_part, (size_t)parts[i]->rows * row_bytes);
  uint8_t* staging = nullptr;
  WG_CHECK_CUDA(cudaMalloc(&staging, max_part));
  int tile0 = 0;
  int rc = WG_OK;
  for (int i = 0; i < nparts && rc == WG_OK; i++) {
    const wg_matrix* p = parts[i];
    size_t nb = (size_t)p->rows * row_bytes;
    cudaError_t e = cudaMemcpyAsync(staging, p->data, nb, cudaMemcpyHostToDevice, st);
    if (e != cudaSuccess) { set_error("upload_matrix: copy: %s", cudaGetErrorString(e)); rc = WG_ERR_CUDA; break; }
    int nt = (p->rows + 15) / 16;
    int64_t threads = (int64_t)nt * m.kblocks * 32;
    repack_tile16_kernel<<<(unsigned)((threads + 255) / 256), 256, 0, st>>>(
        m.qtype, staging, p->rows, row_bytes, m.kblocks, tile0, nt, m);
    rc = launch_status("repack_tile16");
    // the staging buffer is reused by the next part: wait for this one
    e = cudaStreamSynchronize(st);
    if (rc == WG_OK && e != cudaSuccess) { set_error("upload_matrix: %s", cudaGetErrorString(e)); rc = WG_ERR_CUDA; }
    tile0 += nt;
  }
  cudaFree(staging);
  if (rc != WG_OK) { free_dmat(m); return rc; }
  *out = m;
  return WG_OK;
}

int dequant_dmat(const DMat& m, float* d_out, cudaStream_t st) {
  int64_t n = (int64_t)m.rows * m.cols;
  unsigned grid = (unsigned)((n + 255) / 256);
  if (qtype_is_quant(m.qtype)) dequant_tile16_kernel<<<grid, 256, 0, st>>>(m, n, d_out);
  else dequant_dense_kernel<<<grid, 256, 0, st>>>(m, n, d_out);
  return launch_status("dequant");
}

}  // namespace wg
