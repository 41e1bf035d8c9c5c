// gemm.cu — fused dequant GEMV / GEMM: out[r, n] = sum_k X[r, k] * deq(W[n, k]).
//
// Replaces ml.MatMulQuantTransBInto (internal/ml/matmul_q8.go:93-119) and
// its per-type dot kernels (:237-429, the AVX2 routines of
// matmul_q8_kernels_amd64.go and dot_int8_f32_avx2_amd64.s) on the decoder
// token loop, with the bias / residual / GELU / KV-cache writes of
// internal/model/decoder.go fused into the epilogue.
//
// Weights stream from HBM in the tile16 layout (one coalesced 16- or 8-byte
// load per lane per 16x32 tile-block), are dequantised in registers straight
// into mma.m16n8k16 A fragments (f16 = d*q rounded once; f32 accumulation),
// and multiply activation rows staged in shared memory as f16 B fragments.
//   small-R kernel (R <= 16): one 16-row tile per CTA, 8 warps split K,
//     whole activation block resident in shared memory, deterministic
//     shared-memory reduction across warps.
//   large-R kernel (R > 16): 64 weight rows x 64 activation rows per CTA,
//     activation K-slices through a 4-stage cp.async ring.
#include "gemv_frag.cuh"

namespace wg {
namespace {

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem, int src_bytes) {
  uint32_t s = (uint32_t)__cvta_generic_to_shared(smem);
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(s), "l"(gmem), "r"(src_bytes));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N)); }

// Output addressing of one weight row n: element (r, n) lives at
// base + r * row_stride + col_off (CROSS_KV adds the utterance / frame split).
struct EpiRow {
  int64_t col_off, row_stride;
  float bias;
  int kind;  // 0 f32 store, 1 f32 residual add, 2 f16 GELU, 3 f16 store (K/V cache), 4 cross K/V
  bool ok;
};

__device__ __forceinline__ EpiRow epi_row(const Epi& e, int n, int pos) {
  EpiRow er{0, 0, 0.f, 0, n < e.N};
  const int nn = er.ok ? n : 0;
  switch (e.mode) {
    case EPI_F32: er.kind = 0; er.bias = e.bias ? e.bias[nn] : 0.f; er.col_off = nn; er.row_stride = e.ldo; break;
    case EPI_RESID: er.kind = 1; er.bias = e.bias ? e.bias[nn] : 0.f; er.col_off = nn; er.row_stride = e.ldo; break;
    case EPI_GELU_F16: er.kind = 2; er.bias = e.bias ? e.bias[nn] : 0.f; er.col_off = nn; er.row_stride = e.ldo; break;
    case EPI_QKV: {
      const int seg = nn / e.d, j = nn - seg * e.d, h = j / e.hd, c = j - h * e.hd;
      if (seg == 0) { er.kind = 0; er.bias = e.bias_q[j]; er.col_off = j; er.row_stride = e.ldo; }
      else {
        er.kind = 3;
        er.bias = seg == 2 ? e.bias_v[j] : 0.f;
        er.col_off = (((int64_t)(seg - 1) * e.H + h) * e.T + pos) * e.hd + c;
        er.row_stride = (int64_t)2 * e.H * e.T * e.hd;
      }
      break;
    }
    default: {  // EPI_CROSS_KV
      const int lk = nn / e.d, j = nn - lk * e.d, l = lk >> 1, kv = lk & 1, h = j / e.hd, c = j - h * e.hd;
      er.kind = 4;
      er.bias = kv ? e.bias_v[(int64_t)l * e.d + j] : 0.f;
      er.col_off = (((int64_t)l * e.U * 2 + kv) * e.H + h) * (int64_t)e.T * e.hd + c;
    }
  }
  return er;
}

__device__ __forceinline__ int64_t epi_index(const Epi& e, const EpiRow& er, int r) {
  if (er.kind == 4) {
    const int u = r / e.T, tt = r - u * e.T;
    return er.col_off + (int64_t)u * 2 * e.H * e.T * e.hd + (int64_t)tt * e.hd;
  }
  return (int64_t)r * er.row_stride + er.col_off;
}

// The 4*NB accumulators of one thread: rows n0 (c = 0,1) and n0 + 8 (c = 2,3),
// activation rows rbase(nb) + (c & 1). Residual adds are fire-and-forget
// reductions, so no store waits on a load.
template <int NB>
__device__ __forceinline__ void epi_fragments(const Epi& e, int n0, int rbase0, float (&acc)[NB][4]) {
  int pos = 0;
  if (e.mode == EPI_QKV) pos = *e.pos;
  const EpiRow er0 = epi_row(e, n0, pos), er1 = epi_row(e, n0 + 8, pos);
#pragma unroll
  for (int nb = 0; nb < NB; nb++)
#pragma unroll
    for (int c = 0; c < 4; c++) {
      const EpiRow& er = (c >> 1) ? er1 : er0;
      const int r = rbase0 + nb * 8 + (c & 1);
      if (!er.ok || r >= e.R) continue;
      const float v = __fadd_rn(acc[nb][c], er.bias);
      const int64_t idx = epi_index(e, er, r);
      switch (er.kind) {
        case 0: e.out[idx] = v; break;
        case 1:  // x += (acc + b); single writer per element
          asm volatile("red.global.add.f32 [%0], %1;" ::"l"(e.out + idx), "f"(v) : "memory");
          break;
        case 2: e.out16[idx] = __float2half_rn(gelu_f32(v)); break;
        default: e.kv[idx] = __float2half_rn(v); break;
      }
    }
}

// ---- small-R kernel ------------------------------------------------------------------
constexpr int SMALL_WK = 8;  // warps splitting K
constexpr int SMALL_PF = 4;  // blocks in flight per warp

template <uint32_t QT, int NB>
__global__ void __launch_bounds__(SMALL_WK * 32)
    gemv_small_kernel(DMat W, const __half* __restrict__ X, int ldx, Epi e) {
  pdl_trigger();
  pdl_wait();
  extern __shared__ __align__(16) unsigned char smem[];
  constexpr int RC = NB * 8;
  const int K = W.cols, KB = W.kblocks;
  const int xs = K + 16;  // padded row stride in halves: conflict-free 8-byte B-fragment loads
  __half* xsm = reinterpret_cast<__half*>(smem);
  const int tile = blockIdx.x;
  const int r0 = blockIdx.y * RC;
  const int cpr = K / 8;
  for (int i = threadIdx.x; i < RC * cpr; i += blockDim.x) {
    int rr = i / cpr, cc = i - rr * cpr;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (r0 + rr < e.R) v = *reinterpret_cast<const uint4*>(X + (int64_t)(r0 + rr) * ldx + cc * 8);
    *reinterpret_cast<uint4*>(xsm + rr * xs + cc * 8) = v;
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  float acc[NB][4];
#pragma unroll
  for (int nb = 0; nb < NB; nb++)
#pragma unroll
    for (int c = 0; c < 4; c++) acc[nb][c] = 0.f;
  for (int j0 = 0;; j0 += SMALL_PF) {
    const int kbase = warp + SMALL_WK * j0;
    if (kbase >= KB) break;
    Pay p[SMALL_PF];
#pragma unroll
    for (int i = 0; i < SMALL_PF; i++) {
      int kb = kbase + SMALL_WK * i;
      if (kb < KB) p[i] = load_payload<QT>(W, slot_of(W, tile, kb), lane);
    }
#pragma unroll
    for (int i = 0; i < SMALL_PF; i++) {
      int kb = kbase + SMALL_WK * i;
      if (kb < KB) {
#pragma unroll
        for (int s = 0; s < 2; s++) {
          uint32_t a[4];
          dequant_step<QT>(p[i], s, a);
          // the payload's K order within 16 (lane t: k = 4t..4t+3) is the
          // order of the B fragment: one 8-byte load
          const int k0 = kb * 32 + s * 16 + 4 * t;
#pragma unroll
          for (int nb = 0; nb < NB; nb++) {
            const uint2 bb = *reinterpret_cast<const uint2*>(xsm + (nb * 8 + g) * xs + k0);
            mma16816(acc[nb], a, bb.x, bb.y);
          }
        }
      }
    }
  }
  float* red = reinterpret_cast<float*>(smem + (size_t)RC * xs * 2);
#pragma unroll
  for (int nb = 0; nb < NB; nb++)
#pragma unroll
    for (int c = 0; c < 4; c++) red[((warp * NB + nb) * 4 + c) * 32 + lane] = acc[nb][c];
  __syncthreads();
  if (warp != 0) return;
#pragma unroll
  for (int nb = 0; nb < NB; nb++)
#pragma unroll
    for (int c = 0; c < 4; c++)
      for (int w = 1; w < SMALL_WK; w++) acc[nb][c] += red[((w * NB + nb) * 4 + c) * 32 + lane];
  epi_fragments<NB>(e, tile * 16 + g, r0 + 2 * t, acc);
}

// ---- large-R kernel ------------------------------------------------------------------
constexpr int LG_RC = 64, LG_NB = 8, LG_STAGES = 4, LG_XS = 48;  // row stride: conflict-free 8-byte loads

template <uint32_t QT>
__global__ void __launch_bounds__(128) gemm_large_kernel(DMat W, const __half* __restrict__ X, int ldx, Epi e) {
  pdl_trigger();
  pdl_wait();
  __shared__ __align__(16) __half xs[LG_STAGES][LG_RC * LG_XS];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int tile = blockIdx.x * 4 + warp;
  const bool tile_ok = tile < W.ntiles;
  const int r0 = blockIdx.y * LG_RC;
  const int KB = W.kblocks;
  auto load_stage = [&](int kb, int stg) {
#pragma unroll
    for (int c = threadIdx.x; c < LG_RC * 4; c += 128) {
      int rr = c >> 2, cc = c & 3;
      int r = r0 + rr;
      const __half* src = X + (int64_t)(r < e.R ? r : e.R - 1) * ldx + kb * 32 + cc * 8;
      cp_async16(&xs[stg][rr * LG_XS + cc * 8], src, r < e.R ? 16 : 0);
    }
  };
#pragma unroll
  for (int s = 0; s < LG_STAGES - 1; s++) {
    if (s < KB) load_stage(s, s);
    cp_async_commit();
  }
  float acc[LG_NB][4];
#pragma unroll
  for (int nb = 0; nb < LG_NB; nb++)
#pragma unroll
    for (int c = 0; c < 4; c++) acc[nb][c] = 0.f;
  const int wtile = tile_ok ? tile : 0;
  Pay pcur = load_payload<QT>(W, slot_of(W, wtile, 0), lane);
  for (int kb = 0; kb < KB; kb++) {
    cp_async_wait<LG_STAGES - 2>();
    __syncthreads();
    const int nk = kb + LG_STAGES - 1;
    if (nk < KB) load_stage(nk, nk % LG_STAGES);
    cp_async_commit();
    Pay pnext = pcur;
    if (kb + 1 < KB) pnext = load_payload<QT>(W, slot_of(W, wtile, kb + 1), lane);
    const __half* xb = xs[kb % LG_STAGES];
#pragma unroll
    for (int s = 0; s < 2; s++) {
      uint32_t a[4];
      dequant_step<QT>(pcur, s, a);
#pragma unroll
      for (int nb = 0; nb < LG_NB; nb++) {
        const uint2 bb = *reinterpret_cast<const uint2*>(xb + (nb * 8 + g) * LG_XS + s * 16 + 4 * t);
        mma16816(acc[nb], a, bb.x, bb.y);
      }
    }
    pcur = pnext;
  }
  cp_async_wait<0>();
  if (!tile_ok) return;
  epi_fragments<LG_NB>(e, tile * 16 + g, r0 + 2 * t, acc);
}

// ---- dense F32 / F16 weights (test-sized models; any K) ----------------------
template <typename WT>
__global__ void __launch_bounds__(256) gemv_dense_kernel(const WT* __restrict__ W, int N, int K,
                                                          const __half* __restrict__ X, int ldx, Epi e) {
  pdl_trigger();
  pdl_wait();
  int n = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (n >= N) return;
  const WT* w = W + (int64_t)n * K;
  for (int r = 0; r < e.R; r++) {
    const __half* x = X + (int64_t)r * ldx;
    float acc = 0.f;
    for (int k = lane; k < K; k += 32) acc += (float)w[k] * __half2float(x[k]);
    acc = warp_sum(acc);
    if (lane == 0) epi_store(e, r, n, acc);
  }
}

template <uint32_t QT, int NB>
int configure_small_t() {
  cudaError_t e = cudaFuncSetAttribute(gemv_small_kernel<QT, NB>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       227 * 1024);
  if (e != cudaSuccess) {
    set_error("cudaFuncSetAttribute(gemv_small): %s", cudaGetErrorString(e));
    return WG_ERR_CUDA;
  }
  return WG_OK;
}

template <uint32_t QT, int NB>
int launch_small_t(const DMat& W, const __half* X, int ldx, int R, const Epi& e, cudaStream_t st) {
  constexpr int RC = NB * 8;
  size_t smem = (size_t)RC * (W.cols + 16) * 2 + (size_t)SMALL_WK * NB * 4 * 32 * 4;
  if (smem > 227 * 1024) {
    set_error("gemv: K=%d too large for the small-R kernel", W.cols);
    return WG_ERR_UNSUPPORTED;
  }
  dim3 grid(W.ntiles, (R + RC - 1) / RC);
  return launch_check(launch_k(gemv_small_kernel<QT, NB>, grid, dim3(SMALL_WK * 32), smem, st, W, X, ldx, e),
                      "gemv_small");
}

// WG_GEMM_SMALL_PATH=4 keeps rows <= 16 on the streaming kernel (A/B comparisons).
int small_path_override() {
  static int v = -1;
  if (v < 0) {
    const char* s = getenv("WG_GEMM_SMALL_PATH");
    v = (s && *s) ? atoi(s) : 0;
  }
  return v;
}

// WG_GEMM_LARGE_PATH=2 keeps rows > 16 on the mma.sync kernel (A/B comparisons).
int large_path_override() {
  static int v = -1;
  if (v < 0) {
    const char* s = getenv("WG_GEMM_LARGE_PATH");
    v = (s && *s) ? atoi(s) : 0;
  }
  return v;
}

template <uint32_t QT>
int launch_q(const DMat& W, const __half* X, int ldx, int R, const Epi& e, cudaStream_t st, int path) {
  if (path == 0) {
    path = (R <= 16 || gemv_bulk_supported(W, R)) ? 1 : (tc_supported(W) ? 3 : 2);
    if (path == 3 && large_path_override() == 2) path = 2;
  }
  if (path == 1 && gemv_bulk_supported(W, R) && small_path_override() != 4) return launch_gemv_bulk(W, X, ldx, R, e, st);
  if (path == 4) path = 1;
  if (e.ln_x) {
    set_error("launch_matmul: a fused input LayerNorm needs the small-batch GEMV");
    return WG_ERR_INVALID;
  }
  if (path == 3) {
    if (!tc_supported(W)) {
      set_error("tcgen05 path needs a quantised matrix with K %% 64 == 0 (K=%d)", W.cols);
      return WG_ERR_UNSUPPORTED;
    }
    return launch_matmul_tc(W, X, ldx, R, e, st);
  }
  if (path == 1) {
    if (R <= 8) return launch_small_t<QT, 1>(W, X, ldx, R, e, st);
    if (R <= 16) return launch_small_t<QT, 2>(W, X, ldx, R, e, st);
    // small kernel in chunks of 16 rows
    return launch_small_t<QT, 2>(W, X, ldx, R, e, st);
  }
  dim3 grid((W.ntiles + 3) / 4, (R + LG_RC - 1) / LG_RC);
  return launch_check(launch_k(gemm_large_kernel<QT>, grid, dim3(128), 0, st, W, X, ldx, e), "gemm_large");
}

}  // namespace

// Opt the small-R kernels into the full 227 KB of shared memory on the
// current device (called once per device at model creation).
int init_gemm_attributes() {
  int rc = WG_OK;
#define WG_CFG(QT)                                             \
  if (rc == WG_OK) rc = configure_small_t<QT, 1>();            \
  if (rc == WG_OK) rc = configure_small_t<QT, 2>();
  WG_CFG(WG_QTYPE_Q8_0)
  WG_CFG(WG_QTYPE_Q4_0)
  WG_CFG(WG_QTYPE_Q4_1)
  WG_CFG(WG_QTYPE_Q5_0)
  WG_CFG(WG_QTYPE_Q5_1)
#undef WG_CFG
  return rc;
}

bool matmul_fuses_input_ln(const DMat& W, int R) {
  static int v = -1;
  if (v < 0) {
    const char* s = getenv("WG_LN_FUSE");
    v = (s && *s) ? atoi(s) : 1;
  }
  return v != 0 && gemv_bulk_supported(W, R) && small_path_override() != 4;
}

int launch_matmul(const DMat& W, const __half* X, int ldx, int R, const Epi& e_in, cudaStream_t st, int path) {
  if (R <= 0) return WG_OK;
  Epi e = e_in;
  e.R = R;
  if (e.N <= 0) e.N = W.rows;
  if (qtype_is_quant(W.qtype) && (ldx % 8 || (reinterpret_cast<uintptr_t>(X) & 15))) {
    set_error("launch_matmul: activations must be 16-byte aligned rows");
    return WG_ERR_INVALID;
  }
  switch (W.qtype) {
    case WG_QTYPE_Q8_0: return launch_q<WG_QTYPE_Q8_0>(W, X, ldx, R, e, st, path);
    case WG_QTYPE_Q4_0: return launch_q<WG_QTYPE_Q4_0>(W, X, ldx, R, e, st, path);
    case WG_QTYPE_Q4_1: return launch_q<WG_QTYPE_Q4_1>(W, X, ldx, R, e, st, path);
    case WG_QTYPE_Q5_0: return launch_q<WG_QTYPE_Q5_0>(W, X, ldx, R, e, st, path);
    case WG_QTYPE_Q5_1: return launch_q<WG_QTYPE_Q5_1>(W, X, ldx, R, e, st, path);
    case WG_QTYPE_F32:
      return launch_check(launch_k(gemv_dense_kernel<float>, dim3((W.rows + 7) / 8), dim3(256), 0, st,
                                   reinterpret_cast<const float*>(W.qs), W.rows, W.cols, X, ldx, e),
                          "gemv_dense_f32");
    case WG_QTYPE_F16:
      return launch_check(launch_k(gemv_dense_kernel<__half>, dim3((W.rows + 7) / 8), dim3(256), 0, st,
                                   reinterpret_cast<const __half*>(W.qs), W.rows, W.cols, X, ldx, e),
                          "gemv_dense_f16");
    default:
      set_error("launch_matmul: unsupported tensor type %u", W.qtype);
      return WG_ERR_UNSUPPORTED;
  }
}

}  // namespace wg
