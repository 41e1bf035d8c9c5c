// step.cu — the decoder's layers for one token step as ONE persistent kernel
// (small batches: up to 16 rows per step, i.e. up to 3 utterances x beam 5).
//
// At batch 1 a token step of forward (internal/model/decoder.go:745-833) is a
// chain of ~8 dependent operations per layer (LayerNorm + q|k|v matmul,
// self-attention, output matmul, LayerNorm + cross q, cross-attention, output
// matmul, LayerNorm + mlp.0 + GELU, mlp.2), each moving a few MB: as
// separate kernels every one costs a launch plus a pipeline fill, ~5-7 us,
// against ~0.2-1 us of HBM time. This kernel runs all of them for all layers
// with one CTA per SM, the phases separated by a grid-wide barrier
// (co-residency guaranteed by a cooperative launch; every wait bounded):
//
//  matmul phases: the weight matrix is cut into units of one 128-row group x
//    a range of 64-wide K chunks (the tile128 layout makes each unit one
//    contiguous run per plane); each CTA walks its units of the whole step
//    in order and bulk-copies them into a two-slot shared-memory ring ahead
//    of use (weights never depend on activations, so the copy of the next
//    unit overlaps the current phase and the barrier). A unit multiplies its
//    K range of the activations (LayerNorm applied on the fly where one
//    precedes, from the fp32 residual stream) on mma.m16n8k16 with the weights
//    and activations as f16 high + low parts, writes its fp32 partial tile,
//    and the last unit of a group to arrive (an arrival counter) sums the
//    group's K splits in order — deterministic — and applies the epilogue
//    (bias, residual add, GELU, q / K / V with the K and V of this position
//    written to the cache).
//  self-attention: one unit per (row, head) (decoder.go:836-908).
//  cross-attention: units of (utterance, head, frame chunk); the chunks of a
//    head exchange their maxima through global memory (a local bounded wait)
//    so the softmax uses the exact maximum of all 1,500 frames, like the
//    reference; partial sums are combined by the next matmul phase when it
//    stages its activations (decoder.go:911-971, attention.go:193-317).
//
// Arithmetic follows the separate kernels: LayerNorm two-pass in fp32
// (ops.go:153-202), the reference fast exponential, exact maxima, fp32
// accumulation.
#include <cooperative_groups.h>

#include <algorithm>
#include <vector>

#include "async.cuh"
#include "gemv_frag.cuh"

namespace wg {

__device__ int g_step_error;  // first expired wait of the step kernel: (phase << 8) | site

namespace {

constexpr int ST_WARPS = 8;  // one per 16-row tile of a 128-row group
constexpr int ST_THREADS = ST_WARPS * 32;
constexpr int ST_MAX_PAIRS = 6;  // 64-wide K chunks of one matmul unit
constexpr int ST_MAX_ROWS = 16;
constexpr int ST_MAX_CHUNKS = 8;  // frame chunks of one cross-attention head
constexpr int ST_MAX_POS = 448;   // KV positions (n_text_ctx)
constexpr int ST_MAX_FRAMES_CHUNK = 256;
constexpr int ST_MAX_SPLITS = 16;  // K splits of one matmul
constexpr int ST_VBATCH = 8;       // V rows in flight per warp (attention)

// ---------------------------------------------------------------------------
// synchronisation (all waits bounded: 2 s of %globaltimer)
// ---------------------------------------------------------------------------
constexpr uint64_t ST_WAIT_NS = 2000000000ull;

__device__ __forceinline__ unsigned ld_acquire(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void red_release(unsigned* p, unsigned v) {
  asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ void raise_abort(const StepArgs& a, int code) {
  atomicCAS(a.err, 0, code);
  atomicExch(a.sync + 2, 1u);
}

// Spin (thread 0 only) until *p reaches target (wrap-safe), or abort/timeout.
__device__ bool spin_until(const StepArgs& a, const unsigned* p, unsigned target, int code) {
  const uint64_t t0 = global_ns();
  for (uint32_t i = 0;; i++) {
    if ((int)(ld_acquire(p) - target) >= 0) return true;
    if (ld_acquire(a.sync + 2)) return false;
    if ((i & 63) == 63 && global_ns() - t0 > ST_WAIT_NS) {
      raise_abort(a, code);
      return false;
    }
    __nanosleep(64);
  }
}

// Grid-wide barrier: every CTA's writes before it are visible to every CTA after it.
__device__ void grid_barrier(const StepArgs& a, unsigned& target, int code) {
  __syncthreads();
  if (threadIdx.x == 0) {
    target += gridDim.x;
    __threadfence();
    red_release(a.sync, 1u);
    spin_until(a, a.sync, target, code);
    __threadfence();
  }
  __syncthreads();
}

// ---------------------------------------------------------------------------
// weight stream: the CTA's matmul units of the whole step, in order, through
// a two-slot shared-memory ring (one bulk copy per plane per unit)
// ---------------------------------------------------------------------------
struct Ring {
  uint32_t base;           // shared address of slot 0
  uint32_t slot_bytes;
  uint32_t bar;            // two mbarriers
  int issued, consumed;    // units issued / consumed so far
  int total;               // units of this CTA in the step
  int cl, cm, cu;          // issue cursor (thread 0): layer, matmul, unit of the next copy
};

__device__ __forceinline__ int units_of(const MmPlan& p) { return p.groups * p.ks; }

// Moves the cursor to the next unit of this CTA at or after (cl, cm, cu).
__device__ void cursor_fix(const StepArgs& a, Ring& rg) {
  while (rg.cl < a.L && rg.cu >= units_of(a.mm[rg.cm])) {
    if (++rg.cm == 6) {
      rg.cm = 0;
      rg.cl++;
    }
    rg.cu = blockIdx.x;
  }
}

template <uint32_t QT>
__device__ __forceinline__ uint32_t unit_bytes(int np) {
  constexpr uint32_t pb = QT == WG_QTYPE_Q8_0 ? 16 : 8;
  constexpr bool has_m = QT == WG_QTYPE_Q4_1 || QT == WG_QTYPE_Q5_1;
  constexpr bool has_h = QT == WG_QTYPE_Q5_0 || QT == WG_QTYPE_Q5_1;
  return (uint32_t)np * 16 * (32 * pb + 32 + (has_m ? 32 : 0) + (has_h ? 64 : 0));
}

// Issues the copies of the cursor's unit (the CTA's unit number rg.issued)
// into slot issued % 2, which is free, and advances the cursor (thread 0).
template <uint32_t QT>
__device__ void ring_issue(const StepArgs& a, Ring& rg) {
  if (rg.cl >= a.L) return;
  constexpr uint32_t pb = QT == WG_QTYPE_Q8_0 ? 16 : 8;
  constexpr bool has_m = QT == WG_QTYPE_Q4_1 || QT == WG_QTYPE_Q5_1;
  constexpr bool has_h = QT == WG_QTYPE_Q5_0 || QT == WG_QTYPE_Q5_1;
  const MmPlan& pl = a.mm[rg.cm];
  const DMat& W = a.layers[rg.cl].w[rg.cm];
  const int g = rg.cu / pl.ks, kz = rg.cu % pl.ks;
  const int p0 = kz * pl.per, np = min(pl.per, pl.pairs - p0);
  const uint32_t slots = (uint32_t)np * 16;
  const int64_t S0 = ((int64_t)g * pl.pairs + p0) * 16;
  const int k = rg.issued;
  const uint32_t dst = rg.base + (uint32_t)(k & 1) * rg.slot_bytes, bar = rg.bar + 8 * (k & 1);
  const uint32_t qb = slots * 32 * pb;
  mbar_arrive_tx(bar, unit_bytes<QT>(np));
  bulk_g2s(dst, W.qs + S0 * 32 * pb, qb, bar);
  bulk_g2s(dst + qb, W.dsc + S0 * 8, slots * 32, bar);
  uint32_t o = qb + slots * 32;
  if (has_m) {
    bulk_g2s(dst + o, W.msc + S0 * 8, slots * 32, bar);
    o += slots * 32;
  }
  if (has_h) bulk_g2s(dst + o, W.hb + S0 * 32, slots * 64, bar);
  rg.cu += gridDim.x;
  cursor_fix(a, rg);
}

// ---------------------------------------------------------------------------
// activations of a matmul unit
// ---------------------------------------------------------------------------
// Row statistics of LayerNorm (ops.go:153-202) for all rows: mean, std; one
// warp per row held in registers as float4 runs (d = 128 nv, nv <= 10), all
// loads in flight at once (the layernorm_reg_kernel arithmetic).
constexpr int ST_LN_NV = 10;
__device__ void ln_stats(const StepArgs& a, float* stat) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nv = a.d >> 7;
  for (int r = warp; r < a.R; r += ST_WARPS) {
    const float4* x4 = reinterpret_cast<const float4*>(a.x + (int64_t)r * a.d);
    float4 v[ST_LN_NV];
#pragma unroll
    for (int j = 0; j < ST_LN_NV; j++)
      if (j < nv) v[j] = __ldcg(x4 + lane + 32 * j);
    float s = 0.f;
#pragma unroll
    for (int j = 0; j < ST_LN_NV; j++)
      if (j < nv) s += (v[j].x + v[j].y) + (v[j].z + v[j].w);
    s = warp_sum(s);
    const float mean = __fdiv_rn(s, (float)a.d);
    float q = 0.f;
#pragma unroll
    for (int j = 0; j < ST_LN_NV; j++) {
      if (j < nv) {
        const float e0 = __fsub_rn(v[j].x, mean), e1 = __fsub_rn(v[j].y, mean), e2 = __fsub_rn(v[j].z, mean),
                    e3 = __fsub_rn(v[j].w, mean);
        q = __fmaf_rn(e0, e0, q);
        q = __fmaf_rn(e1, e1, q);
        q = __fmaf_rn(e2, e2, q);
        q = __fmaf_rn(e3, e3, q);
      }
    }
    q = warp_sum(q);
    if (lane == 0) {
      stat[2 * r] = mean;
      stat[2 * r + 1] = __fsqrt_rn(__fadd_rn(__fdiv_rn(q, (float)a.d), 1e-5f));
    }
  }
}

enum Src { SRC_LN = 0, SRC_ATT = 1, SRC_CROSS = 2, SRC_H = 3 };

// Stages rows [0, RC) x columns [k0, k0 + kn) of the unit's input as f16
// high + (scaled) low parts: x_hi = f16(v), x_lo = f16((v - x_hi) * 2^10).
// Four adjacent columns per item; the loads of all of a thread's items are
// issued before any is used (a phase is a short, latency-bound step).
constexpr int ST_STAGE_ITEMS = 4;  // items per thread in one batch
__device__ void stage_x(const StepArgs& a, int src, const float* lnw, const float* lnb, const float* stat, int k0,
                        int kn, int RC, int stride, __half* xh, __half* xl) {
  const int kq = kn >> 2, items = a.R * kq;
  for (int base = threadIdx.x; base < items; base += ST_STAGE_ITEMS * blockDim.x) {
    float4 v[ST_STAGE_ITEMS];
#pragma unroll
    for (int it = 0; it < ST_STAGE_ITEMS; it++) {
      const int i = base + it * blockDim.x;
      v[it] = make_float4(0.f, 0.f, 0.f, 0.f);
      if (i >= items) continue;
      const int r = i / kq, k = k0 + 4 * (i - r * kq);
      if (src == SRC_LN || src == SRC_ATT) v[it] = __ldcg(reinterpret_cast<const float4*>((src == SRC_LN ? a.x : a.att) + (int64_t)r * a.d + k));
      else if (src == SRC_H) v[it] = __ldcg(reinterpret_cast<const float4*>(a.h + (int64_t)r * 4 * a.d + k));
    }
    if (src == SRC_CROSS) {  // combine the frame chunks of (row, head): o / l
      for (int it = 0; it < ST_STAGE_ITEMS; it++) {
        const int i = base + it * blockDim.x;
        if (i >= items) continue;
        const int r = i / kq, k = k0 + 4 * (i - r * kq), hh = k >> 6, c = k & 63;
        float4 o[ST_MAX_CHUNKS];
        float l[ST_MAX_CHUNKS];
#pragma unroll
        for (int ch = 0; ch < ST_MAX_CHUNKS; ch++) {
          if (ch < a.xchunks) {
            const float* p = a.xpart + (((int64_t)ch * a.R + r) * a.H + hh) * 68;
            o[ch] = __ldcg(reinterpret_cast<const float4*>(p + c));
            l[ch] = __ldcg(p + 64);
          }
        }
        float4 so = make_float4(0.f, 0.f, 0.f, 0.f);
        float sl = 0.f;
#pragma unroll
        for (int ch = 0; ch < ST_MAX_CHUNKS; ch++) {
          if (ch < a.xchunks) {
            so.x += o[ch].x; so.y += o[ch].y; so.z += o[ch].z; so.w += o[ch].w;
            sl += l[ch];
          }
        }
        const float inv = __fdiv_rn(1.0f, sl);
        v[it] = make_float4(__fmul_rn(so.x, inv), __fmul_rn(so.y, inv), __fmul_rn(so.z, inv), __fmul_rn(so.w, inv));
      }
    }
#pragma unroll
    for (int it = 0; it < ST_STAGE_ITEMS; it++) {
      const int i = base + it * blockDim.x;
      if (i >= items) continue;
      const int r = i / kq, kk = 4 * (i - r * kq), k = k0 + kk;
      float f[4] = {v[it].x, v[it].y, v[it].z, v[it].w};
      if (src == SRC_LN) {
        const float4 w = *reinterpret_cast<const float4*>(lnw + k), b = *reinterpret_cast<const float4*>(lnb + k);
        const float ww[4] = {w.x, w.y, w.z, w.w}, bb[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
        for (int e = 0; e < 4; e++)
          f[e] = __fadd_rn(__fdiv_rn(__fmul_rn(ww[e], __fsub_rn(f[e], stat[2 * r])), stat[2 * r + 1]), bb[e]);
      }
      __half hv[4], lv[4];
#pragma unroll
      for (int e = 0; e < 4; e++) {
        hv[e] = __float2half_rn(f[e]);
        lv[e] = __float2half_rn(__fmul_rn(__fsub_rn(f[e], __half2float(hv[e])), SPLIT_SCALE));
      }
      *reinterpret_cast<uint2*>(xh + r * stride + kk) =
          make_uint2(h2_as_u32(__halves2half2(hv[0], hv[1])), h2_as_u32(__halves2half2(hv[2], hv[3])));
      *reinterpret_cast<uint2*>(xl + r * stride + kk) =
          make_uint2(h2_as_u32(__halves2half2(lv[0], lv[1])), h2_as_u32(__halves2half2(lv[2], lv[3])));
    }
  }
  // rows R..RC-1 of the MMA tile: zero
  for (int i = threadIdx.x; i < (RC - a.R) * (kn >> 2); i += blockDim.x) {
    const int r = a.R + i / (kn >> 2), kk = 4 * (i % (kn >> 2));
    *reinterpret_cast<uint2*>(xh + r * stride + kk) = make_uint2(0, 0);
    *reinterpret_cast<uint2*>(xl + r * stride + kk) = make_uint2(0, 0);
  }
}

// ---------------------------------------------------------------------------
// one matmul unit: partial tile, then (last arriver of its group) the epilogue
// ---------------------------------------------------------------------------
struct UnitRef {
  int l, m, g, kz;
};

template <uint32_t QT, int NB>
__device__ void mm_unit(const StepArgs& a, const UnitRef& ur, const unsigned char* wsm, unsigned char* smem_x,
                        const float* stat) {
  constexpr int RC = NB * 8;
  constexpr int pb = QT == WG_QTYPE_Q8_0 ? 16 : 8;
  constexpr bool has_m = QT == WG_QTYPE_Q4_1 || QT == WG_QTYPE_Q5_1;
  constexpr bool has_h = QT == WG_QTYPE_Q5_0 || QT == WG_QTYPE_Q5_1;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const StepLayer& ly = a.layers[ur.l];
  const MmPlan& pl = a.mm[ur.m];
  const int p0 = ur.kz * pl.per, np = min(pl.per, pl.pairs - p0);
  const int k0 = p0 * 64, kn = np * 64, stride = ST_MAX_PAIRS * 64 + 16;
  __half* xh = reinterpret_cast<__half*>(smem_x);
  __half* xl = xh + RC * stride;
  // input of this matmul
  const int src = ur.m == 0 || ur.m == 2 || ur.m == 4 ? SRC_LN : (ur.m == 1 ? SRC_ATT : (ur.m == 3 ? SRC_CROSS : SRC_H));
  const float* lnw = ur.m == 0 ? ly.sln_w : (ur.m == 2 ? ly.cln_w : ly.mln_w);
  const float* lnb = ur.m == 0 ? ly.sln_b : (ur.m == 2 ? ly.cln_b : ly.mln_b);
  stage_x(a, src, lnw, lnb, stat, k0, kn, RC, stride, xh, xl);
  __syncthreads();
  // warp w: tile w of the group (weights in the ring slot: qs | dsc | msc | hb)
  const uint32_t slots = (uint32_t)np * 16;
  const unsigned char* qsm = wsm;
  const __half2* dsm = reinterpret_cast<const __half2*>(wsm + slots * 32 * pb);
  const __half2* msm = reinterpret_cast<const __half2*>(wsm + slots * 32 * pb + slots * 32);
  const uint16_t* hsm =
      reinterpret_cast<const uint16_t*>(wsm + slots * 32 * pb + slots * 32 + (has_m ? slots * 32 : 0));
  float acc[NB][4], acl[NB][4];
#pragma unroll
  for (int nb = 0; nb < NB; nb++)
#pragma unroll
    for (int c = 0; c < 4; c++) acc[nb][c] = acl[nb][c] = 0.f;
  for (int kb = 0; kb < 2 * np; kb++) {
    const int slot = (kb >> 1) * 16 + warp * 2 + (kb & 1);
    Pay p;
    if (QT == WG_QTYPE_Q8_0) p.q = reinterpret_cast<const uint4*>(qsm)[slot * 32 + lane];
    else {
      const uint2 v = reinterpret_cast<const uint2*>(qsm)[slot * 32 + lane];
      p.q = make_uint4(v.x, v.y, 0, 0);
    }
    p.d = dsm[slot * 8 + g];
    p.m = has_m ? msm[slot * 8 + g] : __float2half2_rn(0.f);
    p.hb = has_h ? hsm[slot * 32 + lane] : 0u;
#pragma unroll
    for (int s = 0; s < 2; s++) {
      uint32_t aw[4], al[4];
      dequant_step_split<QT>(p, s, aw, al);
      const int kk = kb * 32 + s * 16 + 4 * t;
#pragma unroll
      for (int nb = 0; nb < NB; nb++) {
        const uint2 bh = *reinterpret_cast<const uint2*>(xh + (nb * 8 + g) * stride + kk);
        const uint2 bl = *reinterpret_cast<const uint2*>(xl + (nb * 8 + g) * stride + kk);
        mma16816(acc[nb], aw, bh.x, bh.y);
        mma16816(acl[nb], al, bh.x, bh.y);
        mma16816(acl[nb], aw, bl.x, bl.y);
      }
    }
  }
  // partial tile [R][128] of this K split -> global
  float* mine = a.part + ((int64_t)(ur.g * pl.ks + ur.kz)) * a.R * 128;
#pragma unroll
  for (int nb = 0; nb < NB; nb++)
#pragma unroll
    for (int c = 0; c < 4; c++) {
      const int row = warp * 16 + g + 8 * (c >> 1), col = nb * 8 + 2 * t + (c & 1);
      if (col < a.R) mine[col * 128 + row] = __fmaf_rn(acl[nb][c], SPLIT_INV, acc[nb][c]);
    }
  __syncthreads();
  // arrival: the last K split of the group reduces and stores
  __shared__ int last;
  if (threadIdx.x == 0) {
    __threadfence();
    unsigned* cnt = a.sync + 4 + ur.g;
    const unsigned old = atomicAdd(cnt, 1u);
    last = old == (unsigned)(pl.ks - 1);
    if (last) {
      atomicExch(cnt, 0u);  // the next use of the counter is after a grid barrier
      __threadfence();
    }
  }
  __syncthreads();
  if (!last) return;
  const float* base = a.part + (int64_t)ur.g * pl.ks * a.R * 128;
  const int N = a.layers[ur.l].w[ur.m].rows;
  const int pos = *a.pos;
  for (int i = threadIdx.x; i < a.R * 128; i += blockDim.x) {
    const int r = i >> 7, row = i & 127, n = ur.g * 128 + row;
    if (n >= N) continue;
    float pv[ST_MAX_SPLITS];  // every split's partial loaded before the ordered sum
#pragma unroll
    for (int kz = 0; kz < ST_MAX_SPLITS; kz++)
      pv[kz] = kz < pl.ks ? __ldcg(base + ((int64_t)kz * a.R + r) * 128 + row) : 0.f;
    float v = 0.f;
#pragma unroll
    for (int kz = 0; kz < ST_MAX_SPLITS; kz++)
      if (kz < pl.ks) v += pv[kz];  // in split order
    switch (ur.m) {
      case 0: {  // q | k | v (decoder.go:840-870); K and V of this position into the cache
        const int seg = n / a.d, j = n - seg * a.d, hh = j >> 6, c = j & 63;
        if (seg == 0) {
          a.q[(int64_t)r * a.d + j] = __fadd_rn(v, ly.q_b[j]);
        } else {
          if (seg == 2) v = __fadd_rn(v, ly.v_b[j]);
          __half* kv = a.selfkv + (int64_t)ur.l * a.R * 2 * a.H * a.Tmax * 64;
          kv[((((int64_t)r * 2 + (seg - 1)) * a.H + hh) * a.Tmax + pos) * 64 + c] = __float2half_rn(v);
        }
        break;
      }
      case 1: a.x[(int64_t)r * a.d + n] = __fadd_rn(__ldcg(a.x + (int64_t)r * a.d + n), __fadd_rn(v, ly.so_b[n])); break;
      case 2: a.q[(int64_t)r * a.d + n] = __fadd_rn(v, ly.cq_b[n]); break;
      case 3: a.x[(int64_t)r * a.d + n] = __fadd_rn(__ldcg(a.x + (int64_t)r * a.d + n), __fadd_rn(v, ly.co_b[n])); break;
      case 4: a.h[(int64_t)r * 4 * a.d + n] = gelu_f32(__fadd_rn(v, ly.m0_b[n])); break;
      default: a.x[(int64_t)r * a.d + n] = __fadd_rn(__ldcg(a.x + (int64_t)r * a.d + n), __fadd_rn(v, ly.m2_b[n])); break;
    }
  }
}

// All of this CTA's units of matmul m of layer l.
template <uint32_t QT, int NB>
__device__ void mm_phase(const StepArgs& a, Ring& rg, int l, int m, unsigned char* smem_x, float* stat,
                         unsigned char* ring_mem, int phase_code) {
  const MmPlan& pl = a.mm[m];
  const int n = units_of(pl);
  if ((int)blockIdx.x >= n) return;
  if (m == 0 || m == 2 || m == 4) {
    ln_stats(a, stat);
    __syncthreads();
  }
  __shared__ int wok;
  for (int u = blockIdx.x; u < n; u += gridDim.x) {
    const int k = rg.consumed;
    // the unit's weights: wait for the slot's copies
    if (threadIdx.x == 0) {
      wok = mbar_wait(rg.bar + 8 * (k & 1), (uint32_t)(k >> 1) & 1u, reinterpret_cast<volatile int*>(a.sync + 2),
                      (phase_code << 8) | 1, a.err);
      if (!wok) atomicExch(a.sync + 2, 1u);
    }
    __syncthreads();
    if (!wok) return;
    const UnitRef ur{l, m, u / pl.ks, u % pl.ks};
    mm_unit<QT, NB>(a, ur, ring_mem + (uint32_t)(k & 1) * rg.slot_bytes, smem_x, stat);
    __syncthreads();  // every warp is done with the slot: refill it
    rg.consumed++;
    if (rg.issued < rg.total) {
      if (threadIdx.x == 0) ring_issue<QT>(a, rg);
      rg.issued++;
    }
  }
}

// ---------------------------------------------------------------------------
// attention phases
// ---------------------------------------------------------------------------
// Self-attention of (row r, head h) over positions 0..pos (decoder.go:836-908).
__device__ void self_attn_unit(const StepArgs& a, int l, int r, int hh, float* sm) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int pos = *a.pos;
  float* out = a.att + (int64_t)r * a.d + hh * 64;
  if (a.zero_unless_pos0 && pos != 0) {  // slot 0 was reset (decoder.go:593): output exactly 0
    for (int c = threadIdx.x; c < 64; c += blockDim.x) out[c] = 0.f;
    return;
  }
  const int n = a.ref_compat ? 1 : pos + 1;
  float* qs = sm;               // [64]
  float* sc = sm + 64;          // [n]
  float* red = sc + ST_MAX_POS; // [ST_WARPS][64] + [ST_WARPS]
  for (int c = threadIdx.x; c < 64; c += blockDim.x) qs[c] = __ldcg(a.q + (int64_t)r * a.d + hh * 64 + c);
  __syncthreads();
  const __half* kvl = a.selfkv + (int64_t)l * a.R * 2 * a.H * a.Tmax * 64;
  const float scale = 0.125f;  // 1 / sqrt(64)
  auto slab = [&](int tt) -> int64_t {
    const int pr = a.tbl ? __ldcg(a.tbl + (int64_t)r * a.Tmax + tt) : r;
    return (((int64_t)pr * 2) * a.H + hh) * a.Tmax;
  };
  // scores: one position per thread (its K row: eight 16-byte loads)
  for (int tt = threadIdx.x; tt < n; tt += blockDim.x) {
    const uint4* kr = reinterpret_cast<const uint4*>(kvl + (slab(tt) + tt) * 64);
    float s = 0.f;
#pragma unroll
    for (int j = 0; j < 8; j++) {
      const uint4 u = __ldcg(kr + j);
      const __half2* h2 = reinterpret_cast<const __half2*>(&u);
#pragma unroll
      for (int e = 0; e < 4; e++) {
        const float2 f = __half22float2(h2[e]);
        s = fmaf(qs[8 * j + 2 * e], f.x, s);
        s = fmaf(qs[8 * j + 2 * e + 1], f.y, s);
      }
    }
    sc[tt] = __fmul_rn(s, scale);
  }
  __syncthreads();
  float m = -INFINITY;
  for (int tt = threadIdx.x; tt < n; tt += blockDim.x) m = fmaxf(m, sc[tt]);
  m = warp_max(m);
  if (lane == 0) red[ST_WARPS * 64 + warp] = m;
  __syncthreads();
  m = red[ST_WARPS * 64];
  for (int w = 1; w < ST_WARPS; w++) m = fmaxf(m, red[ST_WARPS * 64 + w]);
  __syncthreads();
  float s = 0.f;
  for (int tt = threadIdx.x; tt < n; tt += blockDim.x) {
    const float e = ref_fast_exp(__fsub_rn(sc[tt], m));
    sc[tt] = e;
    s += e;
  }
  s = warp_sum(s);
  if (lane == 0) red[ST_WARPS * 64 + warp] = s;
  __syncthreads();
  s = 0.f;
  for (int w = 0; w < ST_WARPS; w++) s += red[ST_WARPS * 64 + w];
  const float inv = __fdiv_rn(1.0f, s);  // s >= 1: the maximum's weight is exactly 1
  // out = weights . V: warp per position, lane per channel pair, the V rows
  // of ST_VBATCH positions loaded before use
  float o0 = 0.f, o1 = 0.f;
  for (int t0 = warp; t0 < n; t0 += ST_WARPS * ST_VBATCH) {
    __half2 vv[ST_VBATCH];
#pragma unroll
    for (int j = 0; j < ST_VBATCH; j++) {
      const int tt = t0 + j * ST_WARPS;
      vv[j] = tt < n ? __ldcg(reinterpret_cast<const __half2*>(kvl + (slab(tt) + (int64_t)a.H * a.Tmax + tt) * 64) + lane)
                     : __float2half2_rn(0.f);
    }
#pragma unroll
    for (int j = 0; j < ST_VBATCH; j++) {
      const int tt = t0 + j * ST_WARPS;
      if (tt >= n) continue;
      const float w = __fmul_rn(sc[tt], inv);
      const float2 f = __half22float2(vv[j]);
      o0 = fmaf(w, f.x, o0);
      o1 = fmaf(w, f.y, o1);
    }
  }
  red[warp * 64 + 2 * lane] = o0;
  red[warp * 64 + 2 * lane + 1] = o1;
  __syncthreads();
  if (threadIdx.x < 64) {
    float v = 0.f;
    for (int w = 0; w < ST_WARPS; w++) v += red[w * 64 + threadIdx.x];
    out[threadIdx.x] = v;
  }
  __syncthreads();
}

// Cross-attention of utterance u, head hh over frames [t0, t1) for its B
// rows: local maxima exchanged with the head's other chunks, then the
// partial sums (o = sum e v, l = sum e) for the next matmul phase.
__device__ void cross_attn_unit(const StepArgs& a, int l, int u, int hh, int ch, unsigned target, float* sm) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int B = a.B, per = (a.T + a.xchunks - 1) / a.xchunks;
  const int t0 = ch * per, t1 = min(a.T, t0 + per), nt = max(0, t1 - t0);
  float* qs = sm;                    // [B][64]
  float* sc = qs + ST_MAX_ROWS * 64; // [B][ST_MAX_FRAMES_CHUNK]
  float* red = sc + ST_MAX_ROWS * ST_MAX_FRAMES_CHUNK;  // [ST_WARPS][B][64] + [B] maxima
  for (int i = threadIdx.x; i < B * 64; i += blockDim.x)
    qs[i] = __ldcg(a.q + (int64_t)(u * B + i / 64) * a.d + hh * 64 + (i & 63));
  __syncthreads();
  const __half* kb = a.cross + ((((int64_t)l * a.U + u) * 2) * a.H + hh) * (int64_t)a.T * 64;
  const __half* vb = kb + (int64_t)a.H * a.T * 64;
  for (int i = threadIdx.x; i < nt; i += blockDim.x) {
    const uint4* kr = reinterpret_cast<const uint4*>(kb + (int64_t)(t0 + i) * 64);
    uint4 kv[8];
#pragma unroll
    for (int j = 0; j < 8; j++) kv[j] = kr[j];
    for (int b = 0; b < B; b++) {
      float s = 0.f;
#pragma unroll
      for (int j = 0; j < 8; j++) {
        const __half2* h2 = reinterpret_cast<const __half2*>(&kv[j]);
#pragma unroll
        for (int e = 0; e < 4; e++) {
          const float2 f = __half22float2(h2[e]);
          s = fmaf(qs[b * 64 + 8 * j + 2 * e], f.x, s);
          s = fmaf(qs[b * 64 + 8 * j + 2 * e + 1], f.y, s);
        }
      }
      sc[b * ST_MAX_FRAMES_CHUNK + i] = __fmul_rn(s, 0.125f);
    }
  }
  __syncthreads();
  // local maxima -> global scratch; wait for the head's other chunks
  float* mx = red + ST_WARPS * ST_MAX_ROWS * 64;
  for (int b = warp; b < B; b += ST_WARPS) {
    float m = -INFINITY;
    for (int i = lane; i < nt; i += 32) m = fmaxf(m, sc[b * ST_MAX_FRAMES_CHUNK + i]);
    m = warp_max(m);
    if (lane == 0) a.xmax[((int64_t)ch * a.R + u * B + b) * a.H + hh] = m;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    unsigned* cnt = a.sync + 4 + a.max_groups + u * a.H + hh;
    red_release(cnt, 1u);
    spin_until(a, cnt, target, (5 << 8) | 3);
    __threadfence();
  }
  __syncthreads();
  for (int b = threadIdx.x; b < B; b += blockDim.x) {
    float m = -INFINITY;
    for (int c = 0; c < a.xchunks; c++) m = fmaxf(m, __ldcg(a.xmax + ((int64_t)c * a.R + u * B + b) * a.H + hh));
    mx[b] = m;
  }
  __syncthreads();
  for (int i = threadIdx.x; i < B * nt; i += blockDim.x) {
    const int b = i / nt, j = i - b * nt;
    sc[b * ST_MAX_FRAMES_CHUNK + j] = ref_fast_exp(__fsub_rn(sc[b * ST_MAX_FRAMES_CHUNK + j], mx[b]));
  }
  __syncthreads();
  // o[b][c] = sum_t e[b][t] v_t[c]: warp per frame, lane per channel pair
  float o[ST_MAX_ROWS][2];
#pragma unroll
  for (int b = 0; b < ST_MAX_ROWS; b++) o[b][0] = o[b][1] = 0.f;
  for (int i0 = warp; i0 < nt; i0 += ST_WARPS * ST_VBATCH) {
    __half2 vv[ST_VBATCH];
#pragma unroll
    for (int j = 0; j < ST_VBATCH; j++) {
      const int i = i0 + j * ST_WARPS;
      vv[j] = i < nt ? reinterpret_cast<const __half2*>(vb + (int64_t)(t0 + i) * 64)[lane] : __float2half2_rn(0.f);
    }
#pragma unroll
    for (int j = 0; j < ST_VBATCH; j++) {
      const int i = i0 + j * ST_WARPS;
      if (i >= nt) continue;
      const float2 f = __half22float2(vv[j]);
#pragma unroll
      for (int b = 0; b < ST_MAX_ROWS; b++)
        if (b < B) {
          const float e = sc[b * ST_MAX_FRAMES_CHUNK + i];
          o[b][0] = fmaf(e, f.x, o[b][0]);
          o[b][1] = fmaf(e, f.y, o[b][1]);
        }
    }
  }
#pragma unroll
  for (int b = 0; b < ST_MAX_ROWS; b++)
    if (b < B) {
      red[(warp * ST_MAX_ROWS + b) * 64 + 2 * lane] = o[b][0];
      red[(warp * ST_MAX_ROWS + b) * 64 + 2 * lane + 1] = o[b][1];
    }
  __syncthreads();
  for (int i = threadIdx.x; i < B * 64; i += blockDim.x) {
    const int b = i >> 6, c = i & 63;
    float v = 0.f;
#pragma unroll
    for (int w = 0; w < ST_WARPS; w++) v += red[(w * ST_MAX_ROWS + b) * 64 + c];
    a.xpart[(((int64_t)ch * a.R + u * B + b) * a.H + hh) * 68 + c] = v;
  }
  for (int b = warp; b < B; b += ST_WARPS) {  // l = sum of the chunk's weights, one warp per row
    float l = 0.f;
    for (int j = lane; j < nt; j += 32) l += sc[b * ST_MAX_FRAMES_CHUNK + j];
    l = warp_sum(l);
    if (lane == 0) a.xpart[(((int64_t)ch * a.R + u * B + b) * a.H + hh) * 68 + 64] = l;
  }
  __syncthreads();
}

// ---------------------------------------------------------------------------
// the kernel
// ---------------------------------------------------------------------------
template <uint32_t QT, int NB>
__global__ void __launch_bounds__(ST_THREADS, 1) step_kernel(const __grid_constant__ StepArgs a) {
  extern __shared__ __align__(128) unsigned char st_smem[];
  const uint32_t slot_bytes = unit_bytes<QT>(ST_MAX_PAIRS);
  unsigned char* ring_mem = st_smem;                                   // 2 weight slots
  unsigned char* xmem = st_smem + 2 * slot_bytes;                      // activations hi | lo
  const uint32_t xbytes = 2u * ST_MAX_ROWS * (ST_MAX_PAIRS * 64 + 16) * 2;
  float* red = reinterpret_cast<float*>(xmem + xbytes);               // attention / reduction scratch
  float* stat = red + (ST_MAX_ROWS * 64 + ST_MAX_ROWS * ST_MAX_FRAMES_CHUNK + ST_WARPS * ST_MAX_ROWS * 64 + 64);
  uint64_t* bars = reinterpret_cast<uint64_t*>(stat + 2 * ST_MAX_ROWS);
  Ring rg;
  rg.base = smem_u32(ring_mem);
  rg.slot_bytes = slot_bytes;
  rg.bar = smem_u32(bars);
  rg.issued = rg.consumed = 0;
  rg.cl = 0;
  rg.cm = 0;
  rg.cu = blockIdx.x;
  cursor_fix(a, rg);
  {  // units of this CTA in the whole step
    int tot = 0;
    for (int m = 0; m < 6; m++) {
      const int n = units_of(a.mm[m]);
      tot += n > (int)blockIdx.x ? (n - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x : 0;
    }
    rg.total = tot * a.L;
  }
  if (threadIdx.x == 0) {
    mbar_init(rg.bar, 1);
    mbar_init(rg.bar + 8, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  for (int k = 0; k < 2 && rg.issued < rg.total; k++) {
    if (threadIdx.x == 0) ring_issue<QT>(a, rg);
    rg.issued++;
  }
  unsigned target = 0;
  const int G = gridDim.x;
  for (int l = 0; l < a.L; l++) {
    mm_phase<QT, NB>(a, rg, l, 0, xmem, stat, ring_mem, 1);  // LayerNorm + q|k|v
    grid_barrier(a, target, (l << 12) | 0x11);
    for (int w = blockIdx.x; w < a.R * a.H; w += G) self_attn_unit(a, l, w / a.H, w % a.H, red);
    grid_barrier(a, target, (l << 12) | 0x12);
    mm_phase<QT, NB>(a, rg, l, 1, xmem, stat, ring_mem, 2);  // self out + residual
    grid_barrier(a, target, (l << 12) | 0x13);
    mm_phase<QT, NB>(a, rg, l, 2, xmem, stat, ring_mem, 3);  // LayerNorm + cross q
    grid_barrier(a, target, (l << 12) | 0x14);
    // rounds of whole heads: the chunks of a head exchange maxima and wait
    // for one another, so they must all run in the same round (no CTA may
    // wait on a chunk that another CTA only reaches in a later round)
    const int xu = a.U * a.H * a.xchunks, per_round = (G / a.xchunks) * a.xchunks;
    for (int w = blockIdx.x; (int)blockIdx.x < per_round && w < xu; w += per_round) {
      const int ch = w % a.xchunks, uh = w / a.xchunks;
      cross_attn_unit(a, l, uh / a.H, uh % a.H, ch, (unsigned)((l + 1) * a.xchunks), red);
    }
    grid_barrier(a, target, (l << 12) | 0x15);
    mm_phase<QT, NB>(a, rg, l, 3, xmem, stat, ring_mem, 4);  // cross out + residual
    grid_barrier(a, target, (l << 12) | 0x16);
    mm_phase<QT, NB>(a, rg, l, 4, xmem, stat, ring_mem, 5);  // LayerNorm + mlp.0 + GELU
    grid_barrier(a, target, (l << 12) | 0x17);
    mm_phase<QT, NB>(a, rg, l, 5, xmem, stat, ring_mem, 6);  // mlp.2 + residual
    grid_barrier(a, target, (l << 12) | 0x18);
  }
  // copies still in flight (only after an abort) land before the CTA exits
  if (threadIdx.x == 0)
    for (int k = rg.consumed; k < rg.issued; k++) mbar_drain(rg.bar + 8 * (k & 1), (uint32_t)(k >> 1) & 1u);
  __syncthreads();
}

template <uint32_t QT>
size_t step_smem_bytes();

template <uint32_t QT, int NB>
int configure_step_t() {
  cudaError_t e =
      cudaFuncSetAttribute(step_kernel<QT, NB>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)step_smem_bytes<QT>());
  if (e != cudaSuccess) {
    set_error("cudaFuncSetAttribute(step_kernel): %s", cudaGetErrorString(e));
    return WG_ERR_CUDA;
  }
  return WG_OK;
}

template <uint32_t QT>
size_t step_smem_bytes() {
  const size_t slot = (size_t)ST_MAX_PAIRS * 16 *
                      (32 * (QT == WG_QTYPE_Q8_0 ? 16 : 8) + 32 + (qtype_has_min(QT) ? 32 : 0) +
                       (qtype_has_hbits(QT) ? 64 : 0));
  const size_t xbytes = 2u * ST_MAX_ROWS * (ST_MAX_PAIRS * 64 + 16) * 2;
  const size_t redf = ST_MAX_ROWS * 64 + ST_MAX_ROWS * ST_MAX_FRAMES_CHUNK + ST_WARPS * ST_MAX_ROWS * 64 + 64;
  return 2 * slot + xbytes + (redf + 2 * ST_MAX_ROWS) * 4 + 16 + 128;
}

MmPlan plan_of(const DMat& W, int G) {
  MmPlan p;
  p.groups = (W.ntiles + 7) / 8;
  p.pairs = W.kblocks / 2;
  int ks = std::max(1, std::min(std::min(p.pairs, ST_MAX_SPLITS), (G + p.groups / 2) / p.groups));
  p.per = (p.pairs + ks - 1) / ks;
  if (p.per > ST_MAX_PAIRS) p.per = ST_MAX_PAIRS;
  p.ks = (p.pairs + p.per - 1) / p.per;
  return p;  // ks <= ST_MAX_SPLITS: step_supported checks it
}

int xchunks_of(int U, int H, int T, int G) {
  int c = std::max(1, G / std::max(1, U * H));
  c = std::max(c, (T + ST_MAX_FRAMES_CHUNK - 1) / ST_MAX_FRAMES_CHUNK);
  return std::min(c, ST_MAX_CHUNKS);
}

int sm_count() {
  static int n = 0;
  if (!n) {
    int dev = 0;
    cudaGetDevice(&dev);
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
  }
  return n;
}

template <uint32_t QT>
int launch_step_q(const StepArgs& a, cudaStream_t st) {
  const size_t smem = step_smem_bytes<QT>();
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(sm_count(), 1, 1);
  cfg.blockDim = dim3(ST_THREADS, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeCooperative;  // every CTA resident at once: the grid barrier can complete
  at[0].val.cooperative = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  cudaError_t e = a.R <= 8 ? cudaLaunchKernelEx(&cfg, step_kernel<QT, 1>, a) : cudaLaunchKernelEx(&cfg, step_kernel<QT, 2>, a);
  return launch_check(e, "step_kernel");
}

}  // namespace

bool step_supported(const DMat* const w0[6], int R, int hd, int d, int T, int Tmax) {
  static int on = -1;
  if (on < 0) {  // opt-in (WG_STEP_KERNEL=1): measured slower than the kernel chain
    const char* v = getenv("WG_STEP_KERNEL");
    on = v && v[0] == '1';
  }
  if (!on || R < 1 || R > ST_MAX_ROWS || hd != 64 || d % 64 || T < 1 || Tmax > ST_MAX_POS ||
      (T + ST_MAX_FRAMES_CHUNK - 1) / ST_MAX_FRAMES_CHUNK > ST_MAX_CHUNKS || T > 4 * 1024)
    return false;
  if (d % 128 || d / 128 > ST_LN_NV) return false;  // LayerNorm rows in registers
  for (int m = 0; m < 6; m++) {
    if (!qtype_is_quant(w0[m]->qtype) || w0[m]->qtype != w0[0]->qtype || w0[m]->cols % 64) return false;
    if (plan_of(*w0[m], sm_count()).ks > ST_MAX_SPLITS) return false;
  }
  return true;
}

void step_scratch_sizes(const DMat* const w0[6], int R, int U, int H, int T, int64_t* part, int64_t* xpart,
                        int64_t* xmax, int64_t* sync) {
  const int G = sm_count();
  int64_t units = 0, groups = 0;
  for (int m = 0; m < 6; m++) {
    const MmPlan p = plan_of(*w0[m], G);
    units = std::max<int64_t>(units, (int64_t)p.groups * p.ks);
    groups = std::max<int64_t>(groups, p.groups);
  }
  const int xc = xchunks_of(U, H, T, G);
  *part = units * R * 128;
  *xpart = (int64_t)xc * R * H * 68;
  *xmax = (int64_t)xc * R * H;
  *sync = 4 + groups + (int64_t)U * H;
}

int launch_step(StepArgs a, const DMat* const w0[6], cudaStream_t st) {
  const int G = sm_count();
  int groups = 0;
  for (int m = 0; m < 6; m++) {
    a.mm[m] = plan_of(*w0[m], G);
    groups = std::max(groups, a.mm[m].groups);
  }
  a.max_groups = groups;
  a.xchunks = xchunks_of(a.U, a.H, a.T, G);
  int64_t nsync = 4 + groups + (int64_t)a.U * a.H;
  if (cudaMemsetAsync(a.sync, 0, (size_t)nsync * 4, st) != cudaSuccess) {
    set_error("step kernel: clearing the counters failed");
    return WG_ERR_CUDA;
  }
  switch (w0[0]->qtype) {
    case WG_QTYPE_Q8_0: return launch_step_q<WG_QTYPE_Q8_0>(a, st);
    case WG_QTYPE_Q4_0: return launch_step_q<WG_QTYPE_Q4_0>(a, st);
    case WG_QTYPE_Q4_1: return launch_step_q<WG_QTYPE_Q4_1>(a, st);
    case WG_QTYPE_Q5_0: return launch_step_q<WG_QTYPE_Q5_0>(a, st);
    default: return launch_step_q<WG_QTYPE_Q5_1>(a, st);
  }
}

int init_step_attributes() {
  int rc = configure_step_t<WG_QTYPE_Q8_0, 1>();
  if (rc == WG_OK) rc = configure_step_t<WG_QTYPE_Q8_0, 2>();
  if (rc == WG_OK) rc = configure_step_t<WG_QTYPE_Q4_0, 1>();
  if (rc == WG_OK) rc = configure_step_t<WG_QTYPE_Q4_0, 2>();
  if (rc == WG_OK) rc = configure_step_t<WG_QTYPE_Q4_1, 1>();
  if (rc == WG_OK) rc = configure_step_t<WG_QTYPE_Q4_1, 2>();
  if (rc == WG_OK) rc = configure_step_t<WG_QTYPE_Q5_0, 1>();
  if (rc == WG_OK) rc = configure_step_t<WG_QTYPE_Q5_0, 2>();
  if (rc == WG_OK) rc = configure_step_t<WG_QTYPE_Q5_1, 1>();
  if (rc == WG_OK) rc = configure_step_t<WG_QTYPE_Q5_1, 2>();
  return rc;
}

int step_error_word(int* word, bool clear) {
  int v = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, g_step_error, sizeof(int));
  if (e != cudaSuccess) {
    set_error("reading the step kernel error word: %s", cudaGetErrorString(e));
    return WG_ERR_CUDA;
  }
  if (clear && v) {
    int z = 0;
    cudaMemcpyToSymbol(g_step_error, &z, sizeof(int));
  }
  *word = v;
  return WG_OK;
}

int step_error_ptr(int** p) {
  cudaError_t e = cudaGetSymbolAddress((void**)p, g_step_error);
  if (e != cudaSuccess) {
    set_error("step kernel error word: %s", cudaGetErrorString(e));
    return WG_ERR_CUDA;
  }
  return WG_OK;
}

}  // namespace wg
