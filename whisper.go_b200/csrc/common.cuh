// common.cuh — shared definitions of the B200 decoder library (sm_100a).
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <nvtx3/nvToolsExt.h>

#include <atomic>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <utility>

#include "../../include/wg_decoder.h"

namespace wg {

// ---- host-side errors ------------------------------------------------------
void set_error(const char* fmt, ...) __attribute__((format(printf, 1, 2)));
const char* last_error();

#define WG_CHECK_CUDA(call)                                                                  \
  do {                                                                                       \
    cudaError_t e_ = (call);                                                                 \
    if (e_ != cudaSuccess) {                                                                 \
      ::wg::set_error("%s:%d: %s failed: %s", __FILE__, __LINE__, #call, cudaGetErrorString(e_)); \
      return e_ == cudaErrorMemoryAllocation ? WG_ERR_OOM : WG_ERR_CUDA;                     \
    }                                                                                        \
  } while (0)

#define WG_CHECK(expr)        \
  do {                        \
    int rc_ = (expr);         \
    if (rc_ != WG_OK) return rc_; \
  } while (0)

// Count of our own kernel launches (wg_kernel_launch_count). Graph replays
// add the number of kernel nodes of the graph.
extern std::atomic<int64_t> g_launches;
inline void count_launch(int64_t n = 1) { g_launches.fetch_add(n, std::memory_order_relaxed); }

// Checks the launch that was just enqueued.
inline int launch_status(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_error("launch of %s failed: %s", what, cudaGetErrorString(e));
    return WG_ERR_CUDA;
  }
  count_launch();
  return WG_OK;
}

// ---- programmatic dependent launch ------------------------------------------
// Kernels of the token step are launched with programmatic stream
// serialisation: the next kernel of the stream may be scheduled, and run its
// prologue, while the current one drains. Each such kernel calls pdl_wait()
// before its first access to memory an earlier kernel wrote (it returns once
// every earlier kernel of the stream has completed and its writes are
// visible) and pdl_trigger() to let its own successor be scheduled.
// WG_PDL=0 turns the attribute off (plain stream order).
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
bool pdl_enabled();

// NVTX range for the lifetime of a scope (host side): names the job start,
// every token step and the phases of a step in a profiler's timeline (a few
// nanoseconds when no tool is attached; header-only NVTX v3).
struct NvtxRange {
  explicit NvtxRange(const char* name) { nvtxRangePushA(name); }
  ~NvtxRange() { nvtxRangePop(); }
  NvtxRange(const NvtxRange&) = delete;
  NvtxRange& operator=(const NvtxRange&) = delete;
};

template <typename... KArgs, typename... Args>
inline cudaError_t launch_k(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                            Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// Status of a launch made with launch_k (counts it when it succeeded).
inline int launch_check(cudaError_t e, const char* what) {
  if (e != cudaSuccess) {
    cudaGetLastError();
    set_error("launch of %s failed: %s", what, cudaGetErrorString(e));
    return WG_ERR_CUDA;
  }
  count_launch();
  return WG_OK;
}

// ---- device weight layout ----------------------------------------------------
//
// Quantised matrices [rows, cols] (cols % 64 == 0) are repacked at upload into
// the "tile128" layout consumed by the tensor-core GEMV/GEMM: rows are grouped
// in tiles of 16, columns in quant blocks of 32; for every (tile, block) each
// of the 32 lanes of a warp owns a contiguous payload: for each of the two
// 16-wide K steps, rows g and g+8 at k = 4t..4t+3 (g = lane/4, t = lane%4),
// i.e. the A fragment of mma.m16n8k16 with K permuted inside each 16 (the
// mma kernels permute the B fragment the same way) and exactly the register
// layout of a tcgen05.st.16x256b store of the dequantised tile into tensor
// memory (registers: row g k 4t..4t+1, row g k 4t+2..4t+3, row g+8 ...).
// The (tile, block) "slots" are ordered so
// that the 8 tiles x 2 blocks of one 128-row x 64-column group are one
// contiguous run (one bulk copy per tensor-core pipeline stage):
//   slot(tile, kb) = (((tile/8) * (kb_count/2) + kb/2) * 8 + tile%8) * 2 + kb%2
//   qs : [slot][32][PB] bytes, PB = 16 (Q8_0: int8 codes) or 8 (4/5-bit:
//        nibble pairs, pair p of step s at bits 4p and 16+4p of word s)
//   dsc: [slot][8] half2 = (d[row g], d[row g+8])     (all quant types)
//   msc: [slot][8] half2 = (m[row g], m[row g+8])     (Q4_1, Q5_1)
//   hb : [slot][32] u16 lane payload of 5th bits      (Q5_0, Q5_1)
// Byte count equals the GGUF block bytes (plus the row padding to 128).
// F32 / F16 matrices stay dense row-major in qs.
struct DMat {
  uint32_t qtype = 0;
  int rows = 0, cols = 0;
  int ntiles = 0, kblocks = 0;  // 16-row tiles holding data; allocation covers round_up(ntiles, 8)
  uint8_t* qs = nullptr;
  __half2* dsc = nullptr;
  __half2* msc = nullptr;
  uint16_t* hb = nullptr;
};

__host__ __device__ inline int64_t slot_of(const DMat& m, int tile, int kb) {
  return ((((int64_t)(tile >> 3) * (m.kblocks >> 1) + (kb >> 1)) * 8 + (tile & 7)) << 1) + (kb & 1);
}
__host__ __device__ inline int64_t dmat_slots(const DMat& m) { return (int64_t)((m.ntiles + 7) / 8) * 8 * m.kblocks; }

__host__ __device__ inline bool qtype_is_quant(uint32_t q) {
  return q == WG_QTYPE_Q4_0 || q == WG_QTYPE_Q4_1 || q == WG_QTYPE_Q5_0 || q == WG_QTYPE_Q5_1 ||
         q == WG_QTYPE_Q8_0;
}
__host__ __device__ inline int qtype_payload_bytes(uint32_t q) { return q == WG_QTYPE_Q8_0 ? 16 : 8; }
__host__ __device__ inline bool qtype_has_min(uint32_t q) { return q == WG_QTYPE_Q4_1 || q == WG_QTYPE_Q5_1; }
__host__ __device__ inline bool qtype_has_hbits(uint32_t q) { return q == WG_QTYPE_Q5_0 || q == WG_QTYPE_Q5_1; }
__host__ __device__ inline int64_t gguf_block_bytes(uint32_t q) {
  switch (q) {
    case WG_QTYPE_Q4_0: return 18;
    case WG_QTYPE_Q4_1: return 20;
    case WG_QTYPE_Q5_0: return 22;
    case WG_QTYPE_Q5_1: return 24;
    case WG_QTYPE_Q8_0: return 34;
    default: return 0;
  }
}
inline int64_t gguf_row_bytes(uint32_t q, int64_t cols) {
  if (q == WG_QTYPE_F32) return cols * 4;
  if (q == WG_QTYPE_F16) return cols * 2;
  int64_t bb = gguf_block_bytes(q);
  return bb ? ((cols + 31) / 32) * bb : -1;
}

// ---- device helpers -------------------------------------------------------------

// IEEE half -> float (exact), for raw GGUF f16 fields.
__device__ __forceinline__ float h2f_bits(uint16_t h) { return __half2float(__ushort_as_half(h)); }

// The reference softmax exponential, internal/ml/attention.go:34-61
// (fastExpApprox): k = floor(x/ln2), r = x - k*ln2, 4th-order Taylor
// polynomial of exp(r) times 2^k, 0 for x <= -20. Every product and sum is
// rounded separately, as Go evaluates it.
__device__ __forceinline__ float ref_fast_exp(float x) {
  const float invLn2 = 1.4426950408889634f;
  const float ln2 = 0.6931471805599453f;
  if (x <= -20.0f) return 0.0f;
  float y = __fmul_rn(x, invLn2);
  int k = (int)y;
  if ((float)k > y) k--;
  float r = __fsub_rn(x, __fmul_rn((float)k, ln2));
  float r2 = __fmul_rn(r, r);
  float r3 = __fmul_rn(r2, r);
  float r4 = __fmul_rn(r3, r);
  float poly = __fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(1.0f, r), __fmul_rn(0.5f, r2)),
                                   __fmul_rn((float)(1.0 / 6.0), r3)),
                         __fmul_rn((float)(1.0 / 24.0), r4));
  if (k < -126) return 0.0f;
  if (k > 127) return 3.40282346638528859811704183484516925440e+38f;
  return __fmul_rn(poly, __uint_as_float((uint32_t)(k + 127) << 23));
}

// GELU of internal/ml/ops.go:60-122 (tanh form),
//   x * 0.5 * (1 + tanh(z)),  z = sqrt(2/pi) * (x + 0.044715 x^3),
// evaluated through the identity 0.5 * (1 + tanh(z)) = 1 / (1 + exp(-2z)):
// one exponential and one division instead of a tanh. The reference takes
// tanh in float64 and rounds 1+tanh to float32; the relative difference of
// this form (fast exponential and division) is a few 1e-6, far below the
// float16 rounding of the stored activation, and where exp(-2z) overflows it
// returns a signed zero (the reference value is then below 1e-30).
__device__ __forceinline__ float gelu_f32(float x) {
  const float s2p = 0.7978845608028654f, c = 0.044715f;
  const float z = s2p * fmaf(c * x, x * x, x);
  return __fdividef(x, 1.0f + __expf(-2.0f * z));
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

}  // namespace wg
