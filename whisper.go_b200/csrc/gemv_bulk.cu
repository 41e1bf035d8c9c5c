// gemv_bulk.cu — small-batch dequant GEMV (R <= 16 activation rows):
// out[r, n] = sum_k X[r, k] * deq(W[n, k]), the decode-time form of
// ml.MatMulQuantTransBInto (internal/ml/matmul_q8.go:93-119) at batch 1-3.
//
// Each CTA owns one 128-row weight group (8 tiles of 16 rows) and a range of
// 64-wide K chunks. In the tile128 layout that slice of every plane (codes,
// scales, mins, 5th bits) is one contiguous run, so the CTA fetches it into
// shared memory with a few bulk copies, issued before the programmatic
// dependency wait: weights are never written by the token loop, so their
// HBM latency overlaps the previous kernel. After the wait the CTA stages its
// K range of the activation rows, warp w multiplies tile w on mma.m16n8k16
// (f16 A fragments dequantised from shared memory exactly as the streaming
// kernels do, f32 accumulation), and the K ranges of a group — the CTAs of
// one thread-block cluster — are summed in rank order through distributed
// shared memory (deterministic), then stored through the Epi.
#include <cooperative_groups.h>

#include <algorithm>

#include "async.cuh"
#include "gemv_frag.cuh"

namespace cg = cooperative_groups;

namespace wg {

__device__ int g_gemv_error;  // first expired wait (code) of a gemv_bulk kernel

namespace {

constexpr int GB_WARPS = 8;          // one per 16-row tile of the group
constexpr int GB_MAX_PAIRS = 12;     // 64-wide K chunks per CTA (shared memory bound)
constexpr int GB_MAX_NB = 6;         // 8-row activation blocks: up to 48 rows per step
// K chunks per CTA for NB activation blocks: the activation rows (f16 high +
// low parts) grow with NB, so wider batches take shorter K ranges
__host__ __device__ constexpr int gb_max_pairs(int NB) { return NB <= 2 ? GB_MAX_PAIRS : 8; }
constexpr int GB_MAX_CLUSTER = 16;   // K ranges per group (non-portable cluster size)
constexpr int GB_TARGET_CTAS = 444;  // three per SM (measured: +1.7 % at batch 1, large-v3 mlp.0 in 10 K ranges instead of 7)

struct GbLayout {
  uint32_t qs, dsc, msc, hb, xs, xs_lo, red, stat, lnwb, bar, total;
};

// Shared-memory layout for np K chunks and RC activation rows.
__host__ __device__ inline GbLayout gb_layout(uint32_t qt, int np, int RC) {
  const uint32_t slots = (uint32_t)np * 16;
  GbLayout L{};
  L.qs = 0;
  L.dsc = L.qs + slots * 32 * qtype_payload_bytes(qt);
  L.msc = L.dsc + slots * 32;
  L.hb = L.msc + (qtype_has_min(qt) ? slots * 32 : 0);
  L.xs = L.hb + (qtype_has_hbits(qt) ? slots * 64 : 0);
  const uint32_t xs_stride = (uint32_t)np * 64 + 16;  // halves; conflict-free 8-byte B-fragment loads
  // activation rows: f16 hi, then (fused LayerNorm only) the scaled lo part
  L.xs_lo = L.xs + ((uint32_t)RC * xs_stride * 2 + 15) / 16 * 16;
  L.red = L.xs_lo + ((uint32_t)RC * xs_stride * 2 + 15) / 16 * 16;
  L.stat = L.red + 128u * RC * 4;  // [RC][2] LayerNorm mean, std
  L.lnwb = L.stat + (uint32_t)RC * 8;  // LayerNorm gamma, then beta, of the CTA's K range
  L.bar = L.lnwb + (uint32_t)np * 64 * 4 * 2;
  L.total = L.bar + 16;
  return L;
}

constexpr int LN_MAX_NV = 10;  // float4 runs per lane of the vec layout (d <= 1280)

// Mean and standard deviation of a row held in registers in the vec layout
// (float4 runs lane + 32 j, j < nv): the arithmetic of layernorm_reg_kernel.
__device__ __forceinline__ void ln_stats_regs(const float4* v, int nv, int d, float& mean, float& sd) {
  float s = 0.f, q = 0.f;
#pragma unroll
  for (int j = 0; j < LN_MAX_NV; j++)
    if (j < nv) s += (v[j].x + v[j].y) + (v[j].z + v[j].w);
  s = warp_sum(s);
  mean = __fdiv_rn(s, (float)d);
#pragma unroll
  for (int j = 0; j < LN_MAX_NV; j++) {
    if (j < nv) {
      const float a = __fsub_rn(v[j].x, mean), b = __fsub_rn(v[j].y, mean), c = __fsub_rn(v[j].z, mean),
                  e = __fsub_rn(v[j].w, mean);
      q = __fmaf_rn(a, a, q);
      q = __fmaf_rn(b, b, q);
      q = __fmaf_rn(c, c, q);
      q = __fmaf_rn(e, e, q);
    }
  }
  q = warp_sum(q);
  sd = __fsqrt_rn(__fadd_rn(__fdiv_rn(q, (float)d), 1e-5f));
}

// LayerNorm output o as f16 hi + lo / 2^10 (both f16): the products keep
// ~22 bits of the float32 activation. Writes 4 adjacent halves of each part.
__device__ __forceinline__ void ln_store_split(__half* hi, __half* lo, const float* o) {
  const __half2 h0 = __floats2half2_rn(o[0], o[1]), h1 = __floats2half2_rn(o[2], o[3]);
  const float2 f0 = __half22float2(h0), f1 = __half22float2(h1);
  const __half2 l0 = __floats2half2_rn(__fmul_rn(__fsub_rn(o[0], f0.x), SPLIT_SCALE),
                                       __fmul_rn(__fsub_rn(o[1], f0.y), SPLIT_SCALE));
  const __half2 l1 = __floats2half2_rn(__fmul_rn(__fsub_rn(o[2], f1.x), SPLIT_SCALE),
                                       __fmul_rn(__fsub_rn(o[3], f1.y), SPLIT_SCALE));
  *reinterpret_cast<uint2*>(hi) = make_uint2(h2_as_u32(h0), h2_as_u32(h1));
  *reinterpret_cast<uint2*>(lo) = make_uint2(h2_as_u32(l0), h2_as_u32(l1));
}

// Mean and standard deviation of one row of d floats by one warp, with the
// arithmetic of the LayerNorm kernels (internal/ml/ops.go:153-202): vec —
// per-lane float4 runs lane + 32 i (layernorm_reg_kernel), else lane-strided
// scalars (layernorm_kernel); warp tree sums; two passes; sqrt(var + 1e-5).
__device__ __forceinline__ void ln_row_stats(const float* __restrict__ xr, int d, bool vec, int lane, float& mean,
                                             float& sd) {
  float s = 0.f, q = 0.f;
  if (vec) {  // d = 128 nv, nv <= LN_MAX_NV: the row in registers, all loads in flight at once
    const float4* x4 = reinterpret_cast<const float4*>(xr);
    const int nv = d >> 7;
    float4 v[LN_MAX_NV];
#pragma unroll
    for (int j = 0; j < LN_MAX_NV; j++)
      if (j < nv) v[j] = x4[lane + 32 * j];
#pragma unroll
    for (int j = 0; j < LN_MAX_NV; j++)
      if (j < nv) s += (v[j].x + v[j].y) + (v[j].z + v[j].w);
    s = warp_sum(s);
    mean = __fdiv_rn(s, (float)d);
#pragma unroll
    for (int j = 0; j < LN_MAX_NV; j++) {
      if (j < nv) {
        const float a = __fsub_rn(v[j].x, mean), b = __fsub_rn(v[j].y, mean), c = __fsub_rn(v[j].z, mean),
                    e = __fsub_rn(v[j].w, mean);
        q = __fmaf_rn(a, a, q);
        q = __fmaf_rn(b, b, q);
        q = __fmaf_rn(c, c, q);
        q = __fmaf_rn(e, e, q);
      }
    }
  } else {
    for (int i = lane; i < d; i += 32) s += xr[i];
    s = warp_sum(s);
    mean = __fdiv_rn(s, (float)d);
    for (int i = lane; i < d; i += 32) {
      const float dd = __fsub_rn(xr[i], mean);
      q = __fmaf_rn(dd, dd, q);
    }
  }
  q = warp_sum(q);
  sd = __fsqrt_rn(__fadd_rn(__fdiv_rn(q, (float)d), 1e-5f));
}

template <uint32_t QT, int NB>
__global__ void __launch_bounds__(GB_WARPS * 32)
    gemv_bulk_kernel(DMat W, const __half* __restrict__ X, int ldx, int pairs_per, int ln_vec, Epi e) {
  constexpr int RC = NB * 8;
  constexpr int pb = QT == WG_QTYPE_Q8_0 ? 16 : 8;
  constexpr bool has_m = QT == WG_QTYPE_Q4_1 || QT == WG_QTYPE_Q5_1;
  constexpr bool has_h = QT == WG_QTYPE_Q5_0 || QT == WG_QTYPE_Q5_1;
  extern __shared__ __align__(128) unsigned char gb_smem[];
  pdl_trigger();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int group = blockIdx.x;
  const int kc = gridDim.z;
  const int npairs_all = W.kblocks >> 1;
  const int p0 = blockIdx.z * pairs_per;
  const int np = min(pairs_per, npairs_all - p0);  // >= 1 (host choice)
  const GbLayout L = gb_layout(QT, pairs_per, RC);
  const uint32_t base = smem_u32(gb_smem);
  const uint32_t bar = base + L.bar;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(gb_smem + L.bar + 8);

  // ---- weights: contiguous runs of the group's slots [S0, S0 + 16 np) ----
  const int64_t S0 = ((int64_t)group * npairs_all + p0) * 16;
  const uint32_t slots = (uint32_t)np * 16;
  if (warp == 0) {
    if (lane == 0) {
      mbar_init(bar, 1);
      *abort_flag = 0;
      asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
      const uint32_t tx = slots * (32 * pb + 32 + (has_m ? 32 : 0) + (has_h ? 64 : 0));
      mbar_arrive_tx(bar, tx);
    }
    __syncwarp();
    // codes in up to 4 pieces (one per lane: a lane's copies complete in
    // order, so separate lanes keep several in flight), then the scale planes
    const uint32_t qbytes = slots * 32 * pb;
    const uint32_t piece = (uint32_t)((np + 3) / 4) * 16 * 32 * pb;
    if (lane < 4 && lane * piece < qbytes) {
      const uint32_t off = lane * piece, n = min(piece, qbytes - off);
      bulk_g2s(base + L.qs + off, W.qs + S0 * 32 * pb + off, n, bar);
    }
    if (lane == 4) bulk_g2s(base + L.dsc, W.dsc + S0 * 8, slots * 32, bar);
    if (has_m && lane == 5) bulk_g2s(base + L.msc, W.msc + S0 * 8, slots * 32, bar);
    if (has_h && lane == 6) bulk_g2s(base + L.hb, W.hb + S0 * 32, slots * 64, bar);
  }

  const int k0 = p0 * 64, kn = np * 64;
  // the biases of this thread's first outputs (model data) before the wait
  cg::cluster_group cluster = cg::this_cluster();
  const int crank = kc > 1 ? (int)cluster.block_rank() : 0;
  constexpr int GB_PRE_OUT = 2;
  float bpre[GB_PRE_OUT];
#pragma unroll
  for (int j = 0; j < GB_PRE_OUT; j++) {
    const int o = crank * blockDim.x + threadIdx.x + j * kc * blockDim.x;
    const int row = o / RC, col = o - row * RC, n = group * 128 + row;
    bpre[j] = (o < 128 * RC && col < e.R && n < e.N) ? epi_bias(e, n) : 0.f;
  }
  // LayerNorm gamma / beta of this K range: model data, staged before the wait
  float4* lnw = reinterpret_cast<float4*>(gb_smem + L.lnwb);
  float4* lnb = lnw + kn / 4;
  if (e.ln_x) {
    for (int i = threadIdx.x; i < kn / 4; i += blockDim.x) {
      lnw[i] = reinterpret_cast<const float4*>(e.ln_w + k0)[i];
      lnb[i] = reinterpret_cast<const float4*>(e.ln_b + k0)[i];
    }
    // every warp reads elements other threads staged; the barrier sits before
    // the dependency wait, where the CTA waits for its predecessor anyway
    __syncthreads();
  }

  // ---- activations of this K range (written by earlier kernels) ----
  pdl_wait();
  const int pos = e.mode == EPI_QKV ? *e.pos : 0;
  const int xs_stride = pairs_per * 64 + 16;
  __half* xsm = reinterpret_cast<__half*>(gb_smem + L.xs);
  __half* xsm_lo = reinterpret_cast<__half*>(gb_smem + L.xs_lo);
  const bool x_split = e.ln_x != nullptr;  // the activations have a lo part
  if (e.ln_x && ln_vec) {
    // fused LayerNorm, vec layout (d = 128 nv): warp w loads rows w, w + 8,
    // ... into registers (one L2 round trip), takes their statistics and
    // normalises the elements of this CTA's K range straight from the
    // registers, element by element as the LayerNorm kernel does
    const int nv = e.ln_d >> 7;
    for (int rr = warp; rr < RC; rr += GB_WARPS) {
      if (rr < e.R) {
        const float4* x4 = reinterpret_cast<const float4*>(e.ln_x + (int64_t)rr * e.ln_d);
        float4 v[LN_MAX_NV];
#pragma unroll
        for (int j = 0; j < LN_MAX_NV; j++)
          if (j < nv) v[j] = x4[lane + 32 * j];
        float mean, sd;
        ln_stats_regs(v, nv, e.ln_d, mean, sd);
#pragma unroll
        for (int j = 0; j < LN_MAX_NV; j++) {
          const int kk = 4 * (lane + 32 * j) - k0;
          if (j < nv && kk >= 0 && kk < kn) {
            const float4 w = lnw[kk / 4], b = lnb[kk / 4];
            float o[4];
            o[0] = __fadd_rn(__fdiv_rn(__fmul_rn(w.x, __fsub_rn(v[j].x, mean)), sd), b.x);
            o[1] = __fadd_rn(__fdiv_rn(__fmul_rn(w.y, __fsub_rn(v[j].y, mean)), sd), b.y);
            o[2] = __fadd_rn(__fdiv_rn(__fmul_rn(w.z, __fsub_rn(v[j].z, mean)), sd), b.z);
            o[3] = __fadd_rn(__fdiv_rn(__fmul_rn(w.w, __fsub_rn(v[j].w, mean)), sd), b.w);
            ln_store_split(xsm + rr * xs_stride + kk, xsm_lo + rr * xs_stride + kk, o);
          }
        }
      } else {
        const float z[4] = {0.f, 0.f, 0.f, 0.f};
        for (int kk = 4 * lane; kk < kn; kk += 128) ln_store_split(xsm + rr * xs_stride + kk, xsm_lo + rr * xs_stride + kk, z);
      }
    }
  } else if (e.ln_x) {
    // fused LayerNorm, other d: every CTA takes the statistics of the rows
    // and normalises its own K range, element by element as the kernel does
    float* stat = reinterpret_cast<float*>(gb_smem + L.stat);
    for (int rr = warp; rr < e.R; rr += GB_WARPS) {
      float mean, sd;
      ln_row_stats(e.ln_x + (int64_t)rr * e.ln_d, e.ln_d, false, lane, mean, sd);
      if (lane == 0) {
        stat[2 * rr] = mean;
        stat[2 * rr + 1] = sd;
      }
    }
    __syncthreads();
    // four adjacent elements per thread (d and the K range are multiples of 64)
    const int kq = kn / 4;
    for (int i = threadIdx.x; i < RC * kq; i += blockDim.x) {
      const int rr = i / kq, kk = 4 * (i - rr * kq), k = k0 + kk;
      float o[4] = {0.f, 0.f, 0.f, 0.f};
      if (rr < e.R) {
        const float4 x = *reinterpret_cast<const float4*>(e.ln_x + (int64_t)rr * e.ln_d + k);
        const float4 w = lnw[kk / 4];
        const float4 b = lnb[kk / 4];
        const float mean = stat[2 * rr], sd = stat[2 * rr + 1];
        o[0] = __fadd_rn(__fdiv_rn(__fmul_rn(w.x, __fsub_rn(x.x, mean)), sd), b.x);
        o[1] = __fadd_rn(__fdiv_rn(__fmul_rn(w.y, __fsub_rn(x.y, mean)), sd), b.y);
        o[2] = __fadd_rn(__fdiv_rn(__fmul_rn(w.z, __fsub_rn(x.z, mean)), sd), b.z);
        o[3] = __fadd_rn(__fdiv_rn(__fmul_rn(w.w, __fsub_rn(x.w, mean)), sd), b.w);
      }
      ln_store_split(xsm + rr * xs_stride + kk, xsm_lo + rr * xs_stride + kk, o);
    }
  } else {
    const int cpr = kn / 8;
    for (int i = threadIdx.x; i < RC * cpr; i += blockDim.x) {
      const int rr = i / cpr, cc = i - rr * cpr;
      uint4 v = make_uint4(0, 0, 0, 0);
      if (rr < e.R) v = *reinterpret_cast<const uint4*>(X + (int64_t)rr * ldx + k0 + cc * 8);
      *reinterpret_cast<uint4*>(xsm + rr * xs_stride + cc * 8) = v;
    }
  }
  if (threadIdx.x == 0 && !mbar_wait(bar, 0, abort_flag, 1, &g_gemv_error)) mbar_drain(bar, 0);
  __syncthreads();

  // ---- warp w: tile w of the group over the CTA's K range ----
  // acc: hi x hi; acl: the lo corrections (lo_w x hi_x + hi_w x lo_x), scaled by 2^10
  float acc[NB][4], acl[NB][4];
#pragma unroll
  for (int nb = 0; nb < NB; nb++)
#pragma unroll
    for (int c = 0; c < 4; c++) acc[nb][c] = acl[nb][c] = 0.f;
  if (*abort_flag == 0) {
    const unsigned char* qsm = gb_smem + L.qs;
    const __half2* dsm = reinterpret_cast<const __half2*>(gb_smem + L.dsc);
    const __half2* msm = reinterpret_cast<const __half2*>(gb_smem + L.msc);
    const uint16_t* hsm = reinterpret_cast<const uint16_t*>(gb_smem + L.hb);
    for (int kb = 0; kb < 2 * np; kb++) {
      const int slot = (kb >> 1) * 16 + warp * 2 + (kb & 1);  // slot order inside a pair: tile, block
      Pay p;
      if (QT == WG_QTYPE_Q8_0) {
        p.q = reinterpret_cast<const uint4*>(qsm)[slot * 32 + lane];
      } else {
        const uint2 v = reinterpret_cast<const uint2*>(qsm)[slot * 32 + lane];
        p.q = make_uint4(v.x, v.y, 0, 0);
      }
      p.d = dsm[slot * 8 + g];
      p.m = has_m ? msm[slot * 8 + g] : __float2half2_rn(0.f);
      p.hb = has_h ? hsm[slot * 32 + lane] : 0u;
#pragma unroll
      for (int s = 0; s < 2; s++) {
        uint32_t a[4], al[4];
        dequant_step_split<QT>(p, s, a, al);
        const int kk = kb * 32 + s * 16 + 4 * t;  // the payload's K order within 16 is the B fragment's
#pragma unroll
        for (int nb = 0; nb < NB; nb++) {
          const uint2 bb = *reinterpret_cast<const uint2*>(xsm + (nb * 8 + g) * xs_stride + kk);
          mma16816(acc[nb], a, bb.x, bb.y);
          mma16816(acl[nb], al, bb.x, bb.y);
          if (x_split) {
            const uint2 bl = *reinterpret_cast<const uint2*>(xsm_lo + (nb * 8 + g) * xs_stride + kk);
            mma16816(acl[nb], a, bl.x, bl.y);
          }
        }
      }
    }
  }
  // partial tile [128 weight rows][RC activation rows]
  float* red = reinterpret_cast<float*>(gb_smem + L.red);
#pragma unroll
  for (int nb = 0; nb < NB; nb++)
#pragma unroll
    for (int c = 0; c < 4; c++)
      red[(warp * 16 + g + 8 * (c >> 1)) * RC + nb * 8 + 2 * t + (c & 1)] = __fmaf_rn(acl[nb][c], SPLIT_INV, acc[nb][c]);

  // ---- sum the cluster's K ranges in rank order, store ----
  if (kc > 1) cluster.sync();
  else __syncthreads();
  if (*abort_flag == 0) {
    int jo = 0;
    for (int o = crank * blockDim.x + threadIdx.x; o < 128 * RC; o += kc * blockDim.x, jo++) {
      const int row = o / RC, col = o - row * RC;
      const int n = group * 128 + row;
      if (col >= e.R || n >= e.N) continue;
      float v = 0.f;
      if (kc > 1) {
        float part[GB_MAX_CLUSTER];
#pragma unroll
        for (int k = 0; k < GB_MAX_CLUSTER; k++) part[k] = k < kc ? cluster.map_shared_rank(red, k)[o] : 0.f;
#pragma unroll
        for (int k = 0; k < GB_MAX_CLUSTER; k++)
          if (k < kc) v += part[k];
      } else {
        v = red[o];
      }
      float b;
#pragma unroll
      for (int j = 0; j < GB_PRE_OUT; j++)
        if (jo == j) b = bpre[j];
      if (jo >= GB_PRE_OUT) b = epi_bias(e, n);
      epi_store_b(e, col, n, v, b, pos);
    }
  }
  if (kc > 1) cluster.sync();  // peers may still read this CTA's partial tile
}

template <uint32_t QT, int NB>
int launch_gb_t(const DMat& W, const __half* X, int ldx, int R, const Epi& e, cudaStream_t st) {
  const int groups = (W.ntiles + 7) / 8, pairs = W.kblocks / 2;
  // K ranges per group: up to 16 (a non-portable cluster size; measured
  // +3 % at batch 1 against 8: mlp.2 runs 160 CTAs instead of 80);
  // WG_GB_CLUSTER=8 keeps the portable size
  static int max_kc = -1;
  if (max_kc < 0) {
    const char* s = getenv("WG_GB_CLUSTER");
    max_kc = (s && *s) ? atoi(s) : GB_MAX_CLUSTER;
    if (max_kc < 1 || max_kc > GB_MAX_CLUSTER) max_kc = GB_MAX_CLUSTER;
  }
  int kc = std::min(max_kc, std::max(1, (GB_TARGET_CTAS + groups - 1) / groups));
  int per = (pairs + kc - 1) / kc;
  if (per > gb_max_pairs(NB)) per = gb_max_pairs(NB);
  kc = (pairs + per - 1) / per;
  if (kc > max_kc) {
    set_error("gemv_bulk: K=%d needs more than %d K ranges", W.cols, GB_MAX_CLUSTER);
    return WG_ERR_UNSUPPORTED;
  }
  const GbLayout L = gb_layout(QT, per, NB * 8);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(groups, 1, kc);
  cfg.blockDim = dim3(GB_WARPS * 32, 1, 1);
  cfg.dynamicSmemBytes = L.total;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 1;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = kc;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 2 : 1;
  const int ln_vec = e.ln_x && layernorm_uses_vec(e.ln_d) ? 1 : 0;
  return launch_check(cudaLaunchKernelEx(&cfg, gemv_bulk_kernel<QT, NB>, W, X, ldx, per, ln_vec, e), "gemv_bulk");
}

template <uint32_t QT>
int launch_gb_q(const DMat& W, const __half* X, int ldx, int R, const Epi& e, cudaStream_t st) {
  switch ((R + 7) / 8) {
    case 1: return launch_gb_t<QT, 1>(W, X, ldx, R, e, st);
    case 2: return launch_gb_t<QT, 2>(W, X, ldx, R, e, st);
    case 3: return launch_gb_t<QT, 3>(W, X, ldx, R, e, st);
    case 4: return launch_gb_t<QT, 4>(W, X, ldx, R, e, st);
    case 5: return launch_gb_t<QT, 5>(W, X, ldx, R, e, st);
    default: return launch_gb_t<QT, 6>(W, X, ldx, R, e, st);
  }
}

template <uint32_t QT, int NB>
int configure_gb_t() {
  cudaError_t e = cudaFuncSetAttribute(gemv_bulk_kernel<QT, NB>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       227 * 1024);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(gemv_bulk_kernel<QT, NB>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
  if (e != cudaSuccess) {
    set_error("cudaFuncSetAttribute(gemv_bulk): %s", cudaGetErrorString(e));
    return WG_ERR_CUDA;
  }
  return WG_OK;
}

template <uint32_t QT>
int configure_gb_q() {
  int rc = configure_gb_t<QT, 1>();
  if (rc == WG_OK) rc = configure_gb_t<QT, 2>();
  if (rc == WG_OK) rc = configure_gb_t<QT, 3>();
  if (rc == WG_OK) rc = configure_gb_t<QT, 4>();
  if (rc == WG_OK) rc = configure_gb_t<QT, 5>();
  if (rc == WG_OK) rc = configure_gb_t<QT, 6>();
  return rc;
}

}  // namespace

// Rows per step up to which the small-batch GEMV takes a matmul (with its
// fused LayerNorm) instead of the tcgen05 GEMM: WG_GEMV_MAX_ROWS (at most
// 48), default 16. Measured at 40 rows (large-v3, 8 utterances x beam 5):
// 13.4 us per launch against 7.3 us on the tcgen05 GEMM, the three
// mma.sync products of the split operands for 5 row blocks outweighing the
// saved LayerNorm kernels.
int gemv_bulk_max_rows() {
  static int v = -1;
  if (v < 0) {
    const char* s = getenv("WG_GEMV_MAX_ROWS");
    v = (s && *s) ? atoi(s) : 16;
    if (v < 1) v = 1;
    if (v > 8 * GB_MAX_NB) v = 8 * GB_MAX_NB;
  }
  return v;
}

bool gemv_bulk_supported(const DMat& W, int R) {
  const int NB = (R + 7) / 8;
  return R >= 1 && R <= gemv_bulk_max_rows() && qtype_is_quant(W.qtype) && W.cols % 64 == 0 &&
         (W.kblocks / 2 + gb_max_pairs(NB) - 1) / gb_max_pairs(NB) <= GB_MAX_CLUSTER;
}

int launch_gemv_bulk(const DMat& W, const __half* X, int ldx, int R, const Epi& e, cudaStream_t st) {
  if (!gemv_bulk_supported(W, R)) {
    set_error("gemv_bulk: unsupported shape (R=%d, K=%d, type %u)", R, W.cols, W.qtype);
    return WG_ERR_UNSUPPORTED;
  }
  switch (W.qtype) {
    case WG_QTYPE_Q8_0: return launch_gb_q<WG_QTYPE_Q8_0>(W, X, ldx, R, e, st);
    case WG_QTYPE_Q4_0: return launch_gb_q<WG_QTYPE_Q4_0>(W, X, ldx, R, e, st);
    case WG_QTYPE_Q4_1: return launch_gb_q<WG_QTYPE_Q4_1>(W, X, ldx, R, e, st);
    case WG_QTYPE_Q5_0: return launch_gb_q<WG_QTYPE_Q5_0>(W, X, ldx, R, e, st);
    default: return launch_gb_q<WG_QTYPE_Q5_1>(W, X, ldx, R, e, st);
  }
}

int init_gemv_bulk_attributes() {
  int rc = configure_gb_q<WG_QTYPE_Q8_0>();
  if (rc == WG_OK) rc = configure_gb_q<WG_QTYPE_Q4_0>();
  if (rc == WG_OK) rc = configure_gb_q<WG_QTYPE_Q4_1>();
  if (rc == WG_OK) rc = configure_gb_q<WG_QTYPE_Q5_0>();
  if (rc == WG_OK) rc = configure_gb_q<WG_QTYPE_Q5_1>();
  return rc;
}

int gemv_error_word(int* word, bool clear) {
  int v = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, g_gemv_error, sizeof(int));
  if (e != cudaSuccess) {
    set_error("reading the gemv error word: %s", cudaGetErrorString(e));
    return WG_ERR_CUDA;
  }
  if (clear && v) {
    int z = 0;
    cudaMemcpyToSymbol(g_gemv_error, &z, sizeof(int));
  }
  *word = v;
  return WG_OK;
}

}  // namespace wg
