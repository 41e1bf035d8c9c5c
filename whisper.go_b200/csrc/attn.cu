// attn.cu — decoder attention over the KV caches.
//
// Replaces ml.ScaledDotProductAttentionInto (internal/ml/attention.go:193-317)
// as called by runDecoderSelfAttn (internal/model/decoder.go:836-908) and
// runDecoderCrossAttn (:911-971): scores = q.k * 1/sqrt(hd), softmax with the
// reference fast exponential (fastExpApprox, attention.go:34-61) against the
// exact row maximum, weights = e * (1/sum), out = weights . V.
//
//  attn_simt_kernel: one CTA per (row, head); used for self-attention (one
//    query row per KV history) and for cross-attention when hd != 64.
//  cross_attn_mma_kernel: cross-attention where the beams of an utterance
//    share one K/V read. A thread-block cluster splits the 1500 encoder
//    frames; the row maximum and the exponential sum are exchanged through
//    distributed shared memory so the softmax uses the exact global maximum
//    like the reference; Q.K^T and P.V run on mma.m16n8k16 (f16 in, f32
//    accumulate). The exponentials enter P.V unnormalised; the ranks' partial
//    outputs and exponential sums travel in one exchange and the sum of the
//    partials is scaled by 1/sum (two cluster exchanges instead of three).
#include <cooperative_groups.h>

#include "async.cuh"
#include "kernels.cuh"

namespace cg = cooperative_groups;

namespace wg {
namespace {

__device__ int g_attn_error;  // first expired wait of an attention kernel: (chunk << 8) | role

// ---------------------------------------------------------------------------
// SIMT attention
// ---------------------------------------------------------------------------
struct SimtArgs {
  const float* q;
  int ldq;
  const __half* kv;
  int64_t slab_stride;   // elements between KV slabs (rows or utterances)
  int64_t head_stride;   // elements between heads inside a K (or V) block
  int64_t v_off;         // K -> V offset inside a slab
  const int* tbl;        // [R][tbl_ld] slab of each position, or nullptr
  int tbl_ld;
  int rows_per_slab;     // slab = r / rows_per_slab when tbl == nullptr
  int H, hd;
  int n_mode;            // 0: n = *pos + 1; 1: n = 1; 2: n = n_fixed
  int n_fixed;
  const int* pos;
  int zero_unless_pos0;
  __half* out16;
  int ldo;
};

constexpr int SIMT_WARPS = 16;  // most warps per CTA (launch picks 4 or 16)
constexpr int SIMT_UNROLL = 4;  // warp steps whose loads are issued together

// NW warps share the positions, 4 per warp step. NW = 16 (few CTAs in
// flight, latency-bound): when one round of loads covers all n positions
// (n <= 256) each lane's V rows are loaded together with its K rows and kept
// in registers through the softmax, one dependent round of loads instead of
// four. NW = 4 (large batches, where the HBM stream is the limit): K pass,
// then V pass, at the register count that keeps occupancy up.
template <int NW>
__global__ void __launch_bounds__(NW * 32) attn_simt_kernel(SimtArgs a) {
  pdl_trigger();
  pdl_wait();
  extern __shared__ float sm[];  // scores [n] then reduction scratch
  const int r = blockIdx.x, h = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int hd = a.hd;
  const int p = (a.n_mode == 0 || a.zero_unless_pos0) ? *a.pos : 0;
  int n = a.n_mode == 0 ? p + 1 : (a.n_mode == 1 ? 1 : a.n_fixed);
  __half* out = a.out16 + (int64_t)r * a.ldo + h * hd;
  if (a.zero_unless_pos0 && p != 0) {
    // K/V slot 0 was reset to zero (decoder.go:593 -> :372-386): scores are
    // 0, the single weight is 1 and the output is exactly 0.
    for (int c = threadIdx.x; c < hd; c += blockDim.x) out[c] = __float2half_rn(0.f);
    return;
  }
  float* scores = sm;
  float* red = sm + ((n + 3) & ~3);
  __shared__ float qs[64];
  const float* qr = a.q + (int64_t)r * a.ldq + h * hd;
  for (int c = threadIdx.x; c < 64; c += blockDim.x) qs[c] = c < hd ? qr[c] : 0.f;
  // the row's position table staged once, so a K or V load never waits on a
  // table load from global memory
  int* tsm = reinterpret_cast<int*>(red + SIMT_WARPS + SIMT_WARPS * 64);  // [n] (tbl only)
  if (a.tbl)
    for (int t = threadIdx.x; t < n; t += blockDim.x) tsm[t] = a.tbl[(int64_t)r * a.tbl_ld + t];
  __syncthreads();
  const float scale = (float)(1.0 / sqrt((double)hd));
  const int sub = lane >> 3, dl = (lane & 7) * 8;  // 4 positions per warp step, 8 dims per lane
  auto slab_of = [&](int t) -> int64_t {
    return a.tbl ? (int64_t)tsm[t] : (int64_t)(r / a.rows_per_slab);
  };
  // scores: each warp step covers 4 positions (8 lanes x 8 dims each); the
  // table lookups and K rows of SIMT_UNROLL steps are loaded before use
  constexpr int nw = NW;
  const int step = nw * 4;
  const bool one_round = NW == SIMT_WARPS && n <= step * SIMT_UNROLL && hd == 64;
  uint4 vkeep[SIMT_UNROLL];  // one_round: this lane's V rows, loaded with the K rows
  for (int tb = warp * 4; tb < n; tb += step * SIMT_UNROLL) {
    int64_t off[SIMT_UNROLL];
#pragma unroll
    for (int u = 0; u < SIMT_UNROLL; u++) {
      const int t = tb + u * step + sub;
      off[u] = t < n ? slab_of(t) * a.slab_stride + (int64_t)h * a.head_stride + (int64_t)t * hd : -1;
    }
    uint4 kraw[SIMT_UNROLL];
    if (hd == 64) {
#pragma unroll
      for (int u = 0; u < SIMT_UNROLL; u++)
        kraw[u] = off[u] >= 0 ? *reinterpret_cast<const uint4*>(a.kv + off[u] + dl) : make_uint4(0, 0, 0, 0);
      if (one_round) {
#pragma unroll
        for (int u = 0; u < SIMT_UNROLL; u++)
          vkeep[u] = off[u] >= 0 ? *reinterpret_cast<const uint4*>(a.kv + off[u] + a.v_off + dl)
                                 : make_uint4(0, 0, 0, 0);
      }
    }
#pragma unroll
    for (int u = 0; u < SIMT_UNROLL; u++) {
      const int t = tb + u * step + sub;
      float part = 0.f;
      if (off[u] >= 0) {
        if (hd == 64) {
          const __half2* k2 = reinterpret_cast<const __half2*>(&kraw[u]);
#pragma unroll
          for (int e = 0; e < 4; e++) {
            float2 kf = __half22float2(k2[e]);
            part = fmaf(qs[dl + 2 * e], kf.x, part);
            part = fmaf(qs[dl + 2 * e + 1], kf.y, part);
          }
        } else {
          const __half* kr = a.kv + off[u];
          for (int e = 0; e < 8; e++) {
            int c = dl + e;
            if (c < hd) part = fmaf(qs[c], __half2float(kr[c]), part);
          }
        }
      }
      part += __shfl_xor_sync(0xffffffffu, part, 1);
      part += __shfl_xor_sync(0xffffffffu, part, 2);
      part += __shfl_xor_sync(0xffffffffu, part, 4);
      if (t < n && (lane & 7) == 0) scores[t] = __fmul_rn(part, scale);
    }
  }
  __syncthreads();
  // max
  float m = -INFINITY;
  for (int t = threadIdx.x; t < n; t += blockDim.x) m = fmaxf(m, scores[t]);
  m = warp_max(m);
  if (lane == 0) red[warp] = m;
  __syncthreads();
  m = red[0];
  for (int w = 1; w < nw; w++) m = fmaxf(m, red[w]);
  __syncthreads();
  // exp + sum
  float s = 0.f;
  for (int t = threadIdx.x; t < n; t += blockDim.x) {
    float e = ref_fast_exp(__fsub_rn(scores[t], m));
    scores[t] = e;
    s += e;
  }
  s = warp_sum(s);
  if (lane == 0) red[warp] = s;
  __syncthreads();
  s = 0.f;
  for (int w = 0; w < nw; w++) s += red[w];
  const float inv = s == 0.f ? 0.f : __fdiv_rn(1.0f, s);
  const float uni = __fdiv_rn(1.0f, (float)n);
  for (int t = threadIdx.x; t < n; t += blockDim.x) scores[t] = s == 0.f ? uni : __fmul_rn(scores[t], inv);
  __syncthreads();
  // out = weights . V
  float o[8];
#pragma unroll
  for (int e = 0; e < 8; e++) o[e] = 0.f;
  if (one_round) {
    const int tb = warp * 4;
#pragma unroll
    for (int u = 0; u < SIMT_UNROLL; u++) {
      const int t = tb + u * step + sub;
      if (t >= n) continue;
      const float w = scores[t];
      const __half2* v2 = reinterpret_cast<const __half2*>(&vkeep[u]);
#pragma unroll
      for (int e = 0; e < 4; e++) {
        float2 vf = __half22float2(v2[e]);
        o[2 * e] = fmaf(w, vf.x, o[2 * e]);
        o[2 * e + 1] = fmaf(w, vf.y, o[2 * e + 1]);
      }
    }
  }
  for (int tb = warp * 4; !one_round && tb < n; tb += step * SIMT_UNROLL) {
    int64_t off[SIMT_UNROLL];
#pragma unroll
    for (int u = 0; u < SIMT_UNROLL; u++) {
      const int t = tb + u * step + sub;
      off[u] = t < n ? slab_of(t) * a.slab_stride + a.v_off + (int64_t)h * a.head_stride + (int64_t)t * hd : -1;
    }
    uint4 vraw[SIMT_UNROLL];
    if (hd == 64) {
#pragma unroll
      for (int u = 0; u < SIMT_UNROLL; u++)
        vraw[u] = off[u] >= 0 ? *reinterpret_cast<const uint4*>(a.kv + off[u] + dl) : make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int u = 0; u < SIMT_UNROLL; u++) {
      if (off[u] < 0) continue;
      const float w = scores[tb + u * step + sub];
      if (hd == 64) {
        const __half2* v2 = reinterpret_cast<const __half2*>(&vraw[u]);
#pragma unroll
        for (int e = 0; e < 4; e++) {
          float2 vf = __half22float2(v2[e]);
          o[2 * e] = fmaf(w, vf.x, o[2 * e]);
          o[2 * e + 1] = fmaf(w, vf.y, o[2 * e + 1]);
        }
      } else {
        const __half* vr = a.kv + off[u];
        for (int e = 0; e < 8; e++)
          if (dl + e < hd) o[e] = fmaf(w, __half2float(vr[dl + e]), o[e]);
      }
    }
  }
#pragma unroll
  for (int e = 0; e < 8; e++) {
    o[e] += __shfl_xor_sync(0xffffffffu, o[e], 8);
    o[e] += __shfl_xor_sync(0xffffffffu, o[e], 16);
  }
  float* ored = red + SIMT_WARPS;  // [SIMT_WARPS][64]
  if (lane < 8)
#pragma unroll
    for (int e = 0; e < 8; e++) ored[warp * 64 + dl + e] = o[e];
  __syncthreads();
  for (int c = threadIdx.x; c < hd; c += blockDim.x) {
    float v = ored[c];
    for (int w = 1; w < nw; w++) v += ored[w * 64 + c];
    out[c] = __float2half_rn(v);
  }
}

int launch_simt(const SimtArgs& a, int R, int n_max, cudaStream_t st) {
  // scores [n] | warp reduction [SIMT_WARPS] | warp outputs [SIMT_WARPS][64] | position table [n]
  size_t smem = (size_t)(((n_max + 3) & ~3) + SIMT_WARPS + SIMT_WARPS * 64 + (a.tbl ? n_max : 0)) * 4;
  if (smem > 48 * 1024) {
    set_error("attention: %d positions exceed the SIMT kernel's shared memory", n_max);
    return WG_ERR_UNSUPPORTED;
  }
  // 16 warps while few CTAs are in flight (latency-bound), 4 beyond
  static int many = -1;
  if (many < 0) {
    const char* s = getenv("WG_SELF_MANY");
    many = (s && *s) ? atoi(s) : 512;
  }
  if (R * a.H < many)
    return launch_check(launch_k(attn_simt_kernel<SIMT_WARPS>, dim3(R, a.H), dim3(SIMT_WARPS * 32), smem, st, a),
                        "attn_simt");
  return launch_check(launch_k(attn_simt_kernel<4>, dim3(R, a.H), dim3(4 * 32), smem, st, a), "attn_simt");
}

// ---------------------------------------------------------------------------
// Tensor-core cross-attention with a cluster split over encoder frames
// ---------------------------------------------------------------------------
__device__ __forceinline__ void mma16816(float* c, const uint32_t* a, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void ldsm_x4(uint32_t* r, uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t* r, uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void cp_async16(uint32_t s, const void* g, int src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(s), "l"(g), "r"(src_bytes));
}
__device__ __forceinline__ uint32_t pack_h2(float lo, float hi) {
  __half2 h = __floats2half2_rn(lo, hi);
  uint32_t u;
  memcpy(&u, &h, 4);
  return u;
}

constexpr int XA_MAX_WARPS = 4;

// grid (S, H, U), cluster (S, 1, 1); block = 32 * wpc; each warp owns 64
// frames of this CTA's chunk of 64 * wpc frames.
__global__ void __launch_bounds__(XA_MAX_WARPS * 32)
    cross_attn_mma_kernel(const float* __restrict__ q, const __half* __restrict__ kvc, int U, int B, int H, int T,
                          int wpc, __half* __restrict__ out16, int ldo) {
  pdl_trigger();
  extern __shared__ __align__(128) unsigned char smem[];
  cg::cluster_group cluster = cg::this_cluster();
  const int crank = (int)cluster.block_rank();
  const int csize = (int)cluster.num_blocks();
  const int h = blockIdx.y, u = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t4 = lane & 3;
  const int Tc = 64 * wpc;
  const int t_begin = crank * Tc;
  const int d = H * 64;
  unsigned char* ksm = smem;                      // [Tc][64] halves, 16-byte chunks xor-swizzled
  unsigned char* vsm = smem + (size_t)Tc * 128;   // [Tc][64]
  float* stats = reinterpret_cast<float*>(smem + (size_t)Tc * 256);  // [2][16] published to the cluster
  float* wred = stats + 32;                                          // [wpc][16]
  float* opart = wred + XA_MAX_WARPS * 16;  // [1 + wpc][16][64]: CTA partial output, then one slot per warp
  const __half* kbase = kvc + ((int64_t)u * 2 * H + h) * (int64_t)T * 64;
  const __half* vbase = kbase + (int64_t)H * T * 64;
  const uint32_t ks_addr = (uint32_t)__cvta_generic_to_shared(ksm);
  const uint32_t vs_addr = (uint32_t)__cvta_generic_to_shared(vsm);
  // async loads: K chunk (group 0), V chunk (group 1)
  for (int i = threadIdx.x; i < Tc * 8; i += blockDim.x) {
    int row = i >> 3, ch = i & 7;
    int t = t_begin + row;
    int ok = t < T ? 16 : 0;
    int tt = t < T ? t : T - 1;
    cp_async16(ks_addr + row * 128 + ((ch ^ (row & 7)) << 4), kbase + (int64_t)tt * 64 + ch * 8, ok);
  }
  asm volatile("cp.async.commit_group;\n" ::);
  for (int i = threadIdx.x; i < Tc * 8; i += blockDim.x) {
    int row = i >> 3, ch = i & 7;
    int t = t_begin + row;
    int ok = t < T ? 16 : 0;
    int tt = t < T ? t : T - 1;
    cp_async16(vs_addr + row * 128 + ((ch ^ (row & 7)) << 4), vbase + (int64_t)tt * 64 + ch * 8, ok);
  }
  asm volatile("cp.async.commit_group;\n" ::);
  // the cross K/V cache is written once per decode, before the token loop
  // (its precompute is followed by a fully serialised launch), so its loads
  // above overlap the previous kernel; q is written by it
  pdl_wait();
  // Q fragments (rows = beams of utterance u), scaled by 1/sqrt(64) = 2^-3 (exact)
  uint32_t qa[4][4];
  {
    const int rg = g, rg8 = g + 8;
    const float* q0 = q + ((int64_t)u * B + rg) * d + h * 64;
    const float* q1 = q + ((int64_t)u * B + rg8) * d + h * 64;
#pragma unroll
    for (int ks = 0; ks < 4; ks++) {
      int k0 = ks * 16 + 2 * t4;
      float a0 = rg < B ? q0[k0] * 0.125f : 0.f, a1 = rg < B ? q0[k0 + 1] * 0.125f : 0.f;
      float a2 = rg8 < B ? q1[k0] * 0.125f : 0.f, a3 = rg8 < B ? q1[k0 + 1] * 0.125f : 0.f;
      float a4 = rg < B ? q0[k0 + 8] * 0.125f : 0.f, a5 = rg < B ? q0[k0 + 9] * 0.125f : 0.f;
      float a6 = rg8 < B ? q1[k0 + 8] * 0.125f : 0.f, a7 = rg8 < B ? q1[k0 + 9] * 0.125f : 0.f;
      qa[ks][0] = pack_h2(a0, a1);
      qa[ks][1] = pack_h2(a2, a3);
      qa[ks][2] = pack_h2(a4, a5);
      qa[ks][3] = pack_h2(a6, a7);
    }
  }
  asm volatile("cp.async.wait_group 1;\n" ::);
  __syncthreads();
  // S = Q K^T for this warp's 64 frames: 8 blocks of 8 frames
  float sacc[8][4];
#pragma unroll
  for (int nb = 0; nb < 8; nb++)
#pragma unroll
    for (int c = 0; c < 4; c++) sacc[nb][c] = 0.f;
  const int wrow0 = warp * 64;
#pragma unroll
  for (int nb = 0; nb < 8; nb++) {
#pragma unroll
    for (int kp = 0; kp < 2; kp++) {  // pairs of k-steps (32 dims)
      int row = wrow0 + nb * 8 + (lane & 7);
      int ch = kp * 4 + (lane >> 3);
      uint32_t b[4];
      ldsm_x4(b, ks_addr + row * 128 + ((ch ^ (row & 7)) << 4));
      mma16816(sacc[nb], qa[2 * kp], b[0], b[1]);
      mma16816(sacc[nb], qa[2 * kp + 1], b[2], b[3]);
    }
  }
  // mask frames past T; row maxima (rows g and g+8)
  float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
  for (int nb = 0; nb < 8; nb++)
#pragma unroll
    for (int c = 0; c < 4; c++) {
      int t = t_begin + wrow0 + nb * 8 + 2 * t4 + (c & 1);
      if (t >= T) sacc[nb][c] = -INFINITY;
      if (c < 2) mx0 = fmaxf(mx0, sacc[nb][c]);
      else mx1 = fmaxf(mx1, sacc[nb][c]);
    }
  mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
  mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
  mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
  mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
  if (t4 == 0) {
    wred[warp * 16 + g] = mx0;
    wred[warp * 16 + g + 8] = mx1;
  }
  __syncthreads();
  if (threadIdx.x < 16) {
    float m = wred[threadIdx.x];
    for (int w = 1; w < wpc; w++) m = fmaxf(m, wred[w * 16 + threadIdx.x]);
    stats[threadIdx.x] = m;
  }
  cluster.sync();
  float gm0 = -INFINITY, gm1 = -INFINITY;
  for (int rk = 0; rk < csize; rk++) {
    const float* rs = cluster.map_shared_rank(stats, rk);
    gm0 = fmaxf(gm0, rs[g]);
    gm1 = fmaxf(gm1, rs[g + 8]);
  }
  // exponentials against the global maximum, rounded to f16 as the A
  // fragments of P.V, and this warp's partial sums
  float sum0 = 0.f, sum1 = 0.f;
#pragma unroll
  for (int nb = 0; nb < 8; nb++)
#pragma unroll
    for (int c = 0; c < 4; c++) {
      float e = ref_fast_exp(__fsub_rn(sacc[nb][c], c < 2 ? gm0 : gm1));
      sacc[nb][c] = e;
      if (c < 2) sum0 += e;
      else sum1 += e;
    }
  sum0 += __shfl_xor_sync(0xffffffffu, sum0, 1);
  sum0 += __shfl_xor_sync(0xffffffffu, sum0, 2);
  sum1 += __shfl_xor_sync(0xffffffffu, sum1, 1);
  sum1 += __shfl_xor_sync(0xffffffffu, sum1, 2);
  uint32_t pa[4][4];
#pragma unroll
  for (int kk = 0; kk < 4; kk++) {
    pa[kk][0] = pack_h2(sacc[2 * kk][0], sacc[2 * kk][1]);
    pa[kk][1] = pack_h2(sacc[2 * kk][2], sacc[2 * kk][3]);
    pa[kk][2] = pack_h2(sacc[2 * kk + 1][0], sacc[2 * kk + 1][1]);
    pa[kk][3] = pack_h2(sacc[2 * kk + 1][2], sacc[2 * kk + 1][3]);
  }
  asm volatile("cp.async.wait_group 0;\n" ::);
  __syncthreads();  // V in shared memory; every warp is past its reads of wred
  if (t4 == 0) {
    wred[warp * 16 + g] = sum0;
    wred[warp * 16 + g + 8] = sum1;
  }
  // O = P V over this warp's 64 frames: 8 blocks of 8 dims
  float oacc[8][4];
#pragma unroll
  for (int nd = 0; nd < 8; nd++)
#pragma unroll
    for (int c = 0; c < 4; c++) oacc[nd][c] = 0.f;
#pragma unroll
  for (int kk = 0; kk < 4; kk++) {
#pragma unroll
    for (int ndp = 0; ndp < 4; ndp++) {  // pairs of 8-dim blocks
      int mtx = lane >> 3;
      int row = wrow0 + kk * 16 + (mtx & 1) * 8 + (lane & 7);
      int ch = ndp * 2 + (mtx >> 1);
      uint32_t b[4];
      ldsm_x4_t(b, vs_addr + row * 128 + ((ch ^ (row & 7)) << 4));
      mma16816(oacc[2 * ndp], pa[kk], b[0], b[1]);
      mma16816(oacc[2 * ndp + 1], pa[kk], b[2], b[3]);
    }
  }
  // this warp's unnormalised partial output into its slot
  float* oslot = opart + (1 + warp) * 16 * 64;
#pragma unroll
  for (int nd = 0; nd < 8; nd++)
#pragma unroll
    for (int c = 0; c < 4; c++) oslot[(g + ((c >> 1) << 3)) * 64 + nd * 8 + 2 * t4 + (c & 1)] = oacc[nd][c];
  __syncthreads();
  // the CTA's partial output (slot 0) and exponential sums, warps in order
  for (int i = threadIdx.x; i < B * 64; i += blockDim.x) {
    float v = opart[16 * 64 + i];
    for (int w = 1; w < wpc; w++) v += opart[(1 + w) * 16 * 64 + i];
    opart[i] = v;
  }
  if (threadIdx.x < 16) {
    float sm = wred[threadIdx.x];
    for (int w = 1; w < wpc; w++) sm += wred[w * 16 + threadIdx.x];
    stats[16 + threadIdx.x] = sm;
  }
  cluster.sync();
  // every rank takes a share of the outputs: the partial outputs and sums of
  // all ranks added in rank order, then scaled by 1 / sum (the reference
  // scales each weight by the same reciprocal before the product)
  for (int i = crank * blockDim.x + threadIdx.x; i < B * 64; i += csize * blockDim.x) {
    const int row = i >> 6, col = i & 63;
    float pv[8], ps[8];
#pragma unroll
    for (int rk = 0; rk < 8; rk++) {
      pv[rk] = 0.f;
      ps[rk] = 0.f;
      if (rk < csize) {
        const float* rbase = cluster.map_shared_rank(stats, rk);
        pv[rk] = cluster.map_shared_rank(opart, rk)[row * 64 + col];
        ps[rk] = rbase[16 + row];
      }
    }
    float v = 0.f, sm = 0.f;
#pragma unroll
    for (int rk = 0; rk < 8; rk++) {
      if (rk < csize) {
        v += pv[rk];
        sm += ps[rk];
      }
    }
    const float inv = sm == 0.f ? 0.f : __fdiv_rn(1.f, sm);
    out16[((int64_t)u * B + row) * ldo + h * 64 + col] = __float2half_rn(__fmul_rn(v, inv));
  }
  cluster.sync();
}

// ---------------------------------------------------------------------------
// Streaming cross-attention for large batches: one CTA per (head, utterance)
// reads K then V of its encoder frames exactly once. Warp XS_WARPS issues
// one TMA copy per 128-frame chunk (the 128B-swizzled [128][64] f16 box of
// the utterance's K or V slab; frames >= T read as zeros) into a ring of
// XS_NS slots with FULL / EMPTY mbarriers; warps 0..XS_WARPS-1 each own 16
// frames of every chunk:
//   pass 1 (K chunks): scores (q/8).k of the B <= 8 beam rows on
//     mma.m16n8k16, kept in registers (the C fragments of two 8-frame
//     blocks are the A fragment of the P.V product);
//   the exact row maximum and the exponential sums are combined across the
//     warps in shared memory; weights p = e * (1/sum) rounded to f16;
//   pass 2 (V chunks): O += P V on mma; the warps' partial O are summed in
//     warp order at the end.
// ---------------------------------------------------------------------------
constexpr int XS_WARPS = 8, XS_CH = 128, XS_NS = 6, XS_FW = XS_CH / XS_WARPS;  // frames per warp per chunk
constexpr int XS_MAXCH = 12;  // chunks of one pass held in registers: T <= 1536
constexpr int XS_THREADS = (XS_WARPS + 1) * 32;

__global__ void __launch_bounds__(XS_THREADS, 2)
    cross_attn_stream_kernel(const float* __restrict__ q, const __grid_constant__ CUtensorMap kvmap, int B, int H,
                             int T, __half* __restrict__ out16, int ldo) {
  pdl_trigger();
  extern __shared__ __align__(128) unsigned char smem_raw[];
  unsigned char* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  const int h = blockIdx.x, u = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t4 = lane & 3;
  const int d = H * 64;
  const int nch = (T + XS_CH - 1) / XS_CH;  // <= XS_MAXCH (host check)
  const int total = 2 * nch;
  const uint32_t ring = smem_u32(smem);                                       // XS_NS x 16 KB
  float* red = reinterpret_cast<float*>(smem + XS_NS * XS_CH * 128);         // [2][XS_WARPS][8]
  uint64_t* bars = reinterpret_cast<uint64_t*>(red + 2 * XS_WARPS * 8);      // FULL[XS_NS], EMPTY[XS_NS]
  volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + 2 * XS_NS);
  const uint32_t full0 = smem_u32(bars), empty0 = full0 + 8 * XS_NS;
  if (threadIdx.x == 0) {
    for (int s = 0; s < XS_NS; s++) {
      mbar_init(full0 + 8 * s, 1);
      mbar_init(empty0 + 8 * s, XS_WARPS);
    }
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  if (warp == XS_WARPS) {
    // ---------------- producer ----------------
    if (lane == 0) {
      const int kslab = (u * 2) * H + h, vslab = (u * 2 + 1) * H + h;
      int issued = 0;
      for (int c = 0; c < total; c++) {
        const int s = c % XS_NS;
        // slot s is free once chunk c - XS_NS has been consumed by every warp
        if (c >= XS_NS && !mbar_wait(empty0 + 8 * s, (uint32_t)(c / XS_NS - 1) & 1u, abort_flag, (c << 8) | 2,
                                     &g_attn_error))
          break;
        mbar_arrive_tx(full0 + 8 * s, XS_CH * 128);
        tma_3d(ring + s * (XS_CH * 128), &kvmap, 0, (c < nch ? c : c - nch) * XS_CH, c < nch ? kslab : vslab,
               full0 + 8 * s);
        issued = c + 1;
      }
      if (*abort_flag)  // let the copies in flight land before the CTA exits
        for (int c = max(0, issued - XS_NS); c < issued; c++)
          mbar_drain(full0 + 8 * (c % XS_NS), (uint32_t)(c / XS_NS) & 1u);
    }
    return;
  }
  // ---------------- consumers ----------------
  // The producer streams the cross K/V cache, written once per decode before
  // the token loop (its precompute is followed by a fully serialised launch),
  // without waiting for the previous kernel; q is written by it.
  pdl_wait();
  // Q A-fragments (rows 0-7 = beams; rows 8-15 are zero), scaled by 2^-3
  uint32_t qa[4][2];
  {
    const float* q0 = q + ((int64_t)u * B + g) * d + h * 64;
#pragma unroll
    for (int ks = 0; ks < 4; ks++) {
      const int k0 = ks * 16 + 2 * t4;
      const bool ok = g < B;
      qa[ks][0] = pack_h2(ok ? q0[k0] * 0.125f : 0.f, ok ? q0[k0 + 1] * 0.125f : 0.f);
      qa[ks][1] = pack_h2(ok ? q0[k0 + 8] * 0.125f : 0.f, ok ? q0[k0 + 9] * 0.125f : 0.f);
    }
  }
  bool live = true;
  float sc[XS_MAXCH][2][2];  // row g: chunk, 8-frame block, frame pair
  float mx = -INFINITY;
#pragma unroll
  for (int c = 0; c < XS_MAXCH; c++) {
    if (c < nch) {
      const int s = c % XS_NS;
      if (live)
        live = mbar_wait(full0 + 8 * s, (uint32_t)(c / XS_NS) & 1u, abort_flag, (c << 8) | 1, &g_attn_error);
      const uint32_t st = ring + s * (XS_CH * 128);
#pragma unroll
      for (int nb = 0; nb < 2; nb++) {
        float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int kp = 0; kp < 2; kp++) {
          const int row = warp * XS_FW + nb * 8 + (lane & 7);
          const int ch = kp * 4 + (lane >> 3);
          uint32_t b[4];
          ldsm_x4(b, st + row * 128 + ((ch ^ (row & 7)) << 4));
          uint32_t a0[4] = {qa[2 * kp][0], 0u, qa[2 * kp][1], 0u};
          uint32_t a1[4] = {qa[2 * kp + 1][0], 0u, qa[2 * kp + 1][1], 0u};
          mma16816(acc, a0, b[0], b[1]);
          mma16816(acc, a1, b[2], b[3]);
        }
        const int f = c * XS_CH + warp * XS_FW + nb * 8 + 2 * t4;
        sc[c][nb][0] = f < T ? acc[0] : -INFINITY;
        sc[c][nb][1] = f + 1 < T ? acc[1] : -INFINITY;
        mx = fmaxf(mx, fmaxf(sc[c][nb][0], sc[c][nb][1]));
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(empty0 + 8 * s);
    } else {
#pragma unroll
      for (int nb = 0; nb < 2; nb++) sc[c][nb][0] = sc[c][nb][1] = -INFINITY;
    }
  }
  // ---- exact softmax over all frames ----
  mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
  mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
  if (t4 == 0) red[warp * 8 + g] = mx;
  asm volatile("bar.sync 1, %0;" ::"n"(XS_WARPS * 32) : "memory");
  float m = red[g];
  for (int w = 1; w < XS_WARPS; w++) m = fmaxf(m, red[w * 8 + g]);
  float ssum = 0.f;
#pragma unroll
  for (int c = 0; c < XS_MAXCH; c++)
#pragma unroll
    for (int nb = 0; nb < 2; nb++)
#pragma unroll
      for (int i = 0; i < 2; i++) {
        const float e = ref_fast_exp(__fsub_rn(sc[c][nb][i], m));  // 0 for frames >= T
        sc[c][nb][i] = e;
        ssum += e;
      }
  ssum += __shfl_xor_sync(0xffffffffu, ssum, 1);
  ssum += __shfl_xor_sync(0xffffffffu, ssum, 2);
  if (t4 == 0) red[XS_WARPS * 8 + warp * 8 + g] = ssum;
  asm volatile("bar.sync 1, %0;" ::"n"(XS_WARPS * 32) : "memory");
  float tot = 0.f;
  for (int w = 0; w < XS_WARPS; w++) tot += red[XS_WARPS * 8 + w * 8 + g];
  const float inv = tot == 0.f ? 0.f : __fdiv_rn(1.f, tot);
  // ---- O += P V ----
  float oacc[8][4];
#pragma unroll
  for (int nd = 0; nd < 8; nd++)
#pragma unroll
    for (int k = 0; k < 4; k++) oacc[nd][k] = 0.f;
#pragma unroll
  for (int c = 0; c < XS_MAXCH; c++) {
    if (c < nch) {
      const int cc = nch + c, s = cc % XS_NS;
      if (live)
        live = mbar_wait(full0 + 8 * s, (uint32_t)(cc / XS_NS) & 1u, abort_flag, (cc << 8) | 1, &g_attn_error);
      const uint32_t st = ring + s * (XS_CH * 128);
      uint32_t pa[4];
      pa[0] = g < B ? pack_h2(__fmul_rn(sc[c][0][0], inv), __fmul_rn(sc[c][0][1], inv)) : 0u;
      pa[1] = 0u;
      pa[2] = g < B ? pack_h2(__fmul_rn(sc[c][1][0], inv), __fmul_rn(sc[c][1][1], inv)) : 0u;
      pa[3] = 0u;
#pragma unroll
      for (int ndp = 0; ndp < 4; ndp++) {
        const int mtx = lane >> 3;
        const int row = warp * XS_FW + (mtx & 1) * 8 + (lane & 7);
        const int ch = ndp * 2 + (mtx >> 1);
        uint32_t b[4];
        ldsm_x4_t(b, st + row * 128 + ((ch ^ (row & 7)) << 4));
        mma16816(oacc[2 * ndp], pa, b[0], b[1]);
        mma16816(oacc[2 * ndp + 1], pa, b[2], b[3]);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(empty0 + 8 * s);
    }
  }
  // reduce O over the warps (rows g < B), warps in order; the ring is free
  // once every consumer warp has passed its last chunk
  asm volatile("bar.sync 1, %0;" ::"n"(XS_WARPS * 32) : "memory");
  float* ored = reinterpret_cast<float*>(smem);  // [XS_WARPS][8][64]
#pragma unroll
  for (int nd = 0; nd < 8; nd++) {
    ored[(warp * 8 + g) * 64 + nd * 8 + 2 * t4] = oacc[nd][0];
    ored[(warp * 8 + g) * 64 + nd * 8 + 2 * t4 + 1] = oacc[nd][1];
  }
  asm volatile("bar.sync 1, %0;" ::"n"(XS_WARPS * 32) : "memory");
  for (int i = threadIdx.x; i < B * 64; i += XS_WARPS * 32) {
    const int row = i >> 6, col = i & 63;
    float v = ored[row * 64 + col];
    for (int w = 1; w < XS_WARPS; w++) v += ored[(w * 8 + row) * 64 + col];
    out16[((int64_t)u * B + row) * ldo + h * 64 + col] = __float2half_rn(v);
  }
}

size_t xs_smem() { return 1024 + (size_t)XS_NS * XS_CH * 128 + 2 * XS_WARPS * 8 * 4 + 16 * XS_NS + 16; }

}  // namespace

int launch_self_attn(const SelfAttnArgs& s, cudaStream_t st) {
  SimtArgs a{};
  a.q = s.q;
  a.ldq = s.H * s.hd;
  a.kv = s.kv;
  a.slab_stride = (int64_t)2 * s.H * s.Tmax * s.hd;
  a.head_stride = (int64_t)s.Tmax * s.hd;
  a.v_off = (int64_t)s.H * s.Tmax * s.hd;
  a.tbl = s.ref_compat ? nullptr : s.tbl;
  a.tbl_ld = s.Tmax;
  a.rows_per_slab = 1;
  a.H = s.H;
  a.hd = s.hd;
  a.n_mode = s.ref_compat ? 1 : 0;
  a.pos = s.pos;
  a.zero_unless_pos0 = s.zero_unless_pos0;
  a.out16 = s.out16;
  a.ldo = (s.H * s.hd + 7) / 8 * 8;
  return launch_simt(a, s.R, s.Tmax, st);
}

static int cross_wpc(int T) {
  int w = (T + 511) / 512;
  return w < 1 ? 1 : w;
}

int attn_error_word(int* word, bool clear) {
  int v = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, g_attn_error, sizeof(int));
  if (e != cudaSuccess) {
    set_error("reading the attention error word: %s", cudaGetErrorString(e));
    return WG_ERR_CUDA;
  }
  if (clear && v) {
    int z = 0;
    cudaMemcpyToSymbol(g_attn_error, &z, sizeof(int));
  }
  *word = v;
  return WG_OK;
}

int init_attn_attributes() {
  cudaError_t e = cudaFuncSetAttribute(cross_attn_mma_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       XA_MAX_WARPS * 64 * 256 + (32 + XA_MAX_WARPS * 16 + (1 + XA_MAX_WARPS) * 16 * 64) * 4);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(cross_attn_stream_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)xs_smem());
  if (e != cudaSuccess) {
    set_error("cudaFuncSetAttribute(cross_attn): %s", cudaGetErrorString(e));
    return WG_ERR_CUDA;
  }
  return WG_OK;
}

// WG_XATTN=cluster|stream forces a cross-attention kernel (A/B comparisons
// and tests); read at every launch, so it also applies to graphs captured
// while it is set.
static int xattn_override() {
  const char* s = getenv("WG_XATTN");
  return !s ? 0 : (!strcmp(s, "cluster") ? 1 : (!strcmp(s, "stream") ? 2 : 0));
}

int launch_cross_attn(const CrossAttnArgs& c, cudaStream_t st) {
  const int ldo = (c.H * c.hd + 7) / 8 * 8;
  int wpc = cross_wpc(c.T);
  if (c.hd != 64 || c.B > 16 || wpc > XA_MAX_WARPS) {
    SimtArgs a{};
    a.q = c.q;
    a.ldq = c.H * c.hd;
    a.kv = c.kv;
    a.slab_stride = (int64_t)2 * c.H * c.T * c.hd;
    a.head_stride = (int64_t)c.T * c.hd;
    a.v_off = (int64_t)c.H * c.T * c.hd;
    a.tbl = nullptr;
    a.rows_per_slab = c.B;
    a.H = c.H;
    a.hd = c.hd;
    a.n_mode = 2;
    a.n_fixed = c.T;
    a.pos = nullptr;  // not read in n_mode 2
    a.out16 = c.out16;
    a.ldo = ldo;
    return launch_simt(a, c.U * c.B, c.T, st);
  }
  const bool stream_ok = c.B <= 8 && c.T <= XS_MAXCH * XS_CH;
  const int ov = xattn_override();
  // streaming (one CTA per head and utterance) from U * H >= 64 on: measured
  // faster at U * H = 128 (medium, 8 utterances: 16.4 vs ~37 us per launch),
  // 160 and 1280; below, the cluster kernel's 8-way frame split wins
  if (stream_ok && (ov == 2 || (ov == 0 && c.U * c.H >= 64))) {
    // the layer's cache as [U*2*H slabs][T frames][64] f16, box [1][XS_CH][64]
    EncodeTiledFn enc = encode_fn();
    if (!enc) {
      set_error("cuTensorMapEncodeTiled is unavailable");
      return WG_ERR_CUDA;
    }
    CUtensorMap map;
    cuuint64_t dims[3] = {64, (cuuint64_t)c.T, (cuuint64_t)c.U * 2 * c.H};
    cuuint64_t strides[2] = {128, (cuuint64_t)c.T * 128};
    cuuint32_t box[3] = {64, XS_CH, 1};
    cuuint32_t es[3] = {1, 1, 1};
    CUresult cr = enc(&map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<__half*>(c.kv), dims, strides, box, es,
                      CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                      CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (cr != CUDA_SUCCESS) {
      set_error("cuTensorMapEncodeTiled (cross K/V) failed (%d)", (int)cr);
      return WG_ERR_CUDA;
    }
    return launch_check(launch_k(cross_attn_stream_kernel, dim3(c.H, c.U), dim3(XS_THREADS), xs_smem(), st, c.q, map,
                                 c.B, c.H, c.T, c.out16, ldo),
                        "cross_attn_stream");
  }
  int S = (c.T + 64 * wpc - 1) / (64 * wpc);
  size_t smem = (size_t)wpc * 64 * 256 + (32 + XA_MAX_WARPS * 16 + (size_t)(1 + wpc) * 16 * 64) * 4;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(S, c.H, c.U);
  cfg.blockDim = dim3(32 * wpc, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = S;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 2 : 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, cross_attn_mma_kernel, c.q, c.kv, c.U, c.B, c.H, c.T, wpc, c.out16, ldo);
  if (e != cudaSuccess) {
    set_error("launch of cross_attn_mma failed: %s", cudaGetErrorString(e));
    return WG_ERR_CUDA;
  }
  return launch_status("cross_attn_mma");
}

}  // namespace wg
