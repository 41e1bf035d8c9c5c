// gemm_tc.cu — fused dequant GEMM on the 5th-generation tensor cores
// (tcgen05.mma, accumulators in TMEM) for steps with many rows (R > 16):
// beams x utterances in the token loop and U*1500 encoder frames in the
// cross K/V precompute.
//
// Same contract as launch_matmul's other kernels (ml.MatMulQuantTransBInto,
// internal/ml/matmul_q8.go:93-119, with the decoder's epilogues fused):
//   out[r, n] = sum_k X[r, k] * deq(W[n, k])
// computed transposed on the MMA: D[n (TMEM lane), r (TMEM column)] with
// M = 128 weight rows per CTA and N = NR activation rows (<= 256).
//
// Per 64-wide K stage (ring of `stages` buffers, mbarrier handshakes):
//   warp 4 (one thread): cp.async.bulk of the raw quant payloads of the CTA's
//     128 x 64 weight group (one contiguous run per plane in the tile128
//     layout) -> RAW[s]
//   warp 6 (one thread): TMA 2-D tile load of X[NR, 64] (f16, 128B swizzle)
//     -> B[s]
//   warps 0-3: dequantise RAW[s] -> A[s] (f16 = d*q rounded once, 128B
//     swizzled K-major, the same canonical layout TMA writes for B)
//   warp 5 (one thread): 4 x tcgen05.mma.kind::f16 (K=16) into TMEM, then
//     tcgen05.commit frees the stage
//   epilogue: warps 0-3 read their 32 TMEM lanes with tcgen05.ld and apply
//     the Epi store (bias / residual / GELU / KV-cache scatter).
// Every mbarrier wait is bounded; on expiry the kernel records an error
// word, stops waiting and still frees its TMEM.
#include <cuda.h>

#include "kernels.cuh"

namespace wg {
namespace {

constexpr int TC_BM = 128;      // weight rows per CTA (8 tile16 tiles)
constexpr int TC_BK = 64;       // K per stage
constexpr int TC_THREADS = 224; // warps 0-3 dequant + epilogue, 4 weight loader, 5 MMA, 6 activation loader
constexpr uint32_t WAIT_LIMIT = 1u << 22;

__device__ int g_tc_error;  // first expired wait: (stage << 8) | role

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count));
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void mbar_arrive_tx(uint32_t bar, uint32_t tx) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(tx) : "memory");
}
__device__ __forceinline__ bool mbar_try(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait: returns false (and raises the CTA abort flag) on expiry.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, volatile int* abort, int code) {
  for (uint32_t i = 0; i < WAIT_LIMIT; i++) {
    if (mbar_try(bar, parity)) return true;
    if (*abort) return false;
  }
  *abort = 1;
  atomicCAS(&g_tc_error, 0, code);
  return false;
}

__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
               "l"(src), "r"(bytes), "r"(bar)
               : "memory");
}
__device__ __forceinline__ void tma_2d(uint32_t dst, const CUtensorMap* map, int x, int y, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::
          "r"(dst),
      "l"(map), "r"(x), "r"(y), "r"(bar)
      : "memory");
}

// K-major, 128B-swizzled canonical operand (8-row atoms of 1024 B).
__device__ __forceinline__ uint64_t sw128_desc(uint32_t addr) {
  uint64_t d = 0;
  d |= (uint64_t)((addr >> 4) & 0x3FFF);   // start address
  d |= (uint64_t)1 << 16;                   // leading byte offset (unused for swizzled K-major)
  d |= (uint64_t)(1024 >> 4) << 32;         // stride byte offset: 8 rows x 128 B
  d |= (uint64_t)1 << 46;                   // descriptor version (sm100)
  d |= (uint64_t)2 << 61;                   // SWIZZLE_128B
  return d;
}

__device__ __forceinline__ void st_shared_u32(uint32_t addr, uint32_t v) {
  asm volatile("st.shared.u32 [%0], %1;" ::"r"(addr), "r"(v) : "memory");
}

// Byte offset of element (row, k) of a [rows][64] f16 tile in the 128B-swizzled layout.
__device__ __forceinline__ uint32_t sw128_off(int row, int k) {
  return (uint32_t)((row >> 3) * 1024 + (row & 7) * 128 + ((((k >> 3) ^ (row & 7)) & 7) << 4) + (k & 7) * 2);
}

__device__ __forceinline__ uint32_t h2u(__half2 h) {
  uint32_t u;
  memcpy(&u, &h, 4);
  return u;
}
__device__ __forceinline__ __half2 u2h(uint32_t u) {
  __half2 h;
  memcpy(&h, &u, 4);
  return h;
}

// ---- epilogue (shared with gemm.cu's semantics) --------------------------------
__device__ __forceinline__ float tc_gelu(float x) {
  const float s2p = 0.7978845608028654f, c = 0.044715f;
  float inner = __fmul_rn(s2p, __fadd_rn(x, __fmul_rn(__fmul_rn(__fmul_rn(c, x), x), x)));
  float th = (float)(1.0 + tanh((double)inner));
  return __fmul_rn(__fmul_rn(x, 0.5f), th);
}
struct TcLayout {
  int stages;
  uint32_t a_bytes, b_bytes, raw_bytes;
  uint32_t qs_off, d_off, m_off, hb_off;  // inside one RAW stage
  uint32_t a0, b0, raw0, bar0, total;
};

__host__ __device__ inline TcLayout tc_layout(uint32_t qt, int NR) {
  TcLayout L{};
  const int pb = qt == WG_QTYPE_Q8_0 ? 16 : 8;
  L.a_bytes = TC_BM * TC_BK * 2;  // 16 KB
  L.b_bytes = (uint32_t)NR * TC_BK * 2;
  // RAW: the 16 slots (8 tiles x 2 blocks) of one weight group, plane by plane
  L.qs_off = 0;
  L.d_off = 16 * 32 * pb;
  L.m_off = L.d_off + 16 * 8 * 4;
  L.hb_off = L.m_off + 16 * 8 * 4;
  L.raw_bytes = (L.hb_off + 16 * 32 * 2 + 1023) & ~1023u;
  const uint32_t per = L.a_bytes + L.b_bytes + L.raw_bytes;
  L.stages = (int)((220u * 1024u) / per);
  if (L.stages > 6) L.stages = 6;
  L.a0 = 0;
  L.b0 = L.a0 + L.stages * L.a_bytes;
  L.raw0 = L.b0 + L.stages * L.b_bytes;
  L.bar0 = L.raw0 + L.stages * L.raw_bytes;
  L.total = L.bar0 + 8 * (4 * 6 + 1) + 16 + 1024;  // barriers, tmem slot, alignment slack
  return L;
}

template <uint32_t QT>
__global__ void __launch_bounds__(TC_THREADS, 1)
    gemm_tc_kernel(DMat W, const __grid_constant__ CUtensorMap xmap, int R, int NR, Epi e) {
  extern __shared__ __align__(1024) unsigned char tc_smem_raw[];
  // 1024-byte alignment of the swizzled tiles
  unsigned char* sm = tc_smem_raw + ((1024 - (smem_u32(tc_smem_raw) & 1023)) & 1023);
  const TcLayout L = tc_layout(QT, NR);
  const int S = L.stages;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tile0 = blockIdx.x * 8;
  const int r0 = blockIdx.y * NR;
  const int nk = W.cols / TC_BK;
  const uint32_t base = smem_u32(sm);
  const uint32_t bar = base + L.bar0;
  // barrier groups: raw_full[S], raw_empty[S], mma_full[S], ab_empty[S], done
  auto RAW_FULL = [&](int s) { return bar + 8 * s; };
  auto RAW_EMPTY = [&](int s) { return bar + 8 * (6 + s); };
  auto MMA_FULL = [&](int s) { return bar + 8 * (12 + s); };
  auto AB_EMPTY = [&](int s) { return bar + 8 * (18 + s); };
  const uint32_t DONE = bar + 8 * 24;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(sm + L.bar0 + 8 * 25);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sm + L.bar0 + 8 * 25 + 4);
  if (threadIdx.x == 0) {
    for (int s = 0; s < S; s++) {
      mbar_init(RAW_FULL(s), 1);
      mbar_init(RAW_EMPTY(s), 4);
      mbar_init(MMA_FULL(s), 5);
      mbar_init(AB_EMPTY(s), 1);
    }
    mbar_init(DONE, 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  // TMEM: NR fp32 columns (power of two >= 32)
  uint32_t ncols = 32;
  while (ncols < (uint32_t)NR) ncols <<= 1;
  if (warp == 5) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(ncols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = *tmem_slot;
  const int pb = QT == WG_QTYPE_Q8_0 ? 16 : 8;
  const bool has_m = QT == WG_QTYPE_Q4_1 || QT == WG_QTYPE_Q5_1;
  const bool has_h = QT == WG_QTYPE_Q5_0 || QT == WG_QTYPE_Q5_1;

  if (warp == 4) {
    if (lane == 0) {
      // ---------------- weight loader ----------------
      const uint32_t tx = 16 * 32 * pb + 16 * 8 * 4 + (has_m ? 16 * 8 * 4 : 0) + (has_h ? 16 * 32 * 2 : 0);
      for (int k = 0; k < nk; k++) {
        const int s = k % S;
        const uint32_t ph = (uint32_t)(k / S) & 1u;
        if (!mbar_wait(RAW_EMPTY(s), ph ^ 1u, abort_flag, (k << 8) | 1)) break;
        const uint32_t raw = base + L.raw0 + s * L.raw_bytes;
        const int64_t slot = slot_of(W, tile0, 2 * k);  // first of 16 contiguous slots
        mbar_arrive_tx(RAW_FULL(s), tx);
        bulk_g2s(raw + L.qs_off, W.qs + slot * 32 * pb, 16 * 32 * pb, RAW_FULL(s));
        bulk_g2s(raw + L.d_off, W.dsc + slot * 8, 16 * 8 * 4, RAW_FULL(s));
        if (has_m) bulk_g2s(raw + L.m_off, W.msc + slot * 8, 16 * 8 * 4, RAW_FULL(s));
        if (has_h) bulk_g2s(raw + L.hb_off, W.hb + slot * 32, 16 * 32 * 2, RAW_FULL(s));
      }
    }
  } else if (warp == 6) {
    if (lane == 0) {
      // ---------------- activation loader ----------------
      for (int k = 0; k < nk; k++) {
        const int s = k % S;
        const uint32_t ph = (uint32_t)(k / S) & 1u;
        if (!mbar_wait(AB_EMPTY(s), ph ^ 1u, abort_flag, (k << 8) | 2)) break;
        mbar_arrive_tx(MMA_FULL(s), L.b_bytes);
        tma_2d(base + L.b0 + s * L.b_bytes, &xmap, k * TC_BK, r0, MMA_FULL(s));
      }
    }
  } else if (warp == 5) {
    if (lane == 0) {
      // ---------------- MMA issuer ----------------
      const uint32_t idesc = (1u << 4)                       // D format: f32
                             | (0u << 7) | (0u << 10)        // A, B: f16
                             | ((uint32_t)(NR >> 3) << 17)   // N
                             | ((uint32_t)(TC_BM >> 4) << 24);  // M
      for (int k = 0; k < nk; k++) {
        const int s = k % S;
        const uint32_t ph = (uint32_t)(k / S) & 1u;
        if (!mbar_wait(MMA_FULL(s), ph, abort_flag, (k << 8) | 3)) break;
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint64_t ad = sw128_desc(base + L.a0 + s * L.a_bytes);
        const uint64_t bd = sw128_desc(base + L.b0 + s * L.b_bytes);
#pragma unroll
        for (int kk = 0; kk < 4; kk++) {
          const uint32_t acc = (k > 0 || kk > 0) ? 1u : 0u;
          asm volatile(
              "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
              " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(tmem),
              "l"(ad + (uint64_t)(kk * 2)), "l"(bd + (uint64_t)(kk * 2)), "r"(idesc), "r"(acc)
              : "memory");
        }
        asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(AB_EMPTY(s))
                     : "memory");
      }
      asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(DONE)
                   : "memory");
    }
  } else {
    // ---------------- dequantisers (warps 0-3: row tiles 2w, 2w+1) ----------------
    const int g = lane >> 2;
    // stmatrix row addresses (relative to a stage's A tile): lane l writes row
    // (l & 7) of 8x8 matrix l >> 3 = (rows +8 if odd, k +8 if >= 2) of each
    // (tile, block, step) 16x16 fragment, at its 128B-swizzled position
    uint32_t soff[2][2][2];
#pragma unroll
    for (int tt = 0; tt < 2; tt++)
#pragma unroll
      for (int blk = 0; blk < 2; blk++)
#pragma unroll
        for (int st = 0; st < 2; st++) {
          const int mtx = lane >> 3;
          const int row = (warp * 2 + tt) * 16 + (mtx & 1) * 8 + (lane & 7);
          const int kcol = blk * 32 + st * 16 + (mtx >> 1) * 8;
          soff[tt][blk][st] = sw128_off(row, kcol);
        }
    for (int k = 0; k < nk; k++) {
      const int s = k % S;
      const uint32_t ph = (uint32_t)(k / S) & 1u;
      bool ok = mbar_wait(RAW_FULL(s), ph, abort_flag, (k << 8) | 4);
      ok = __all_sync(0xffffffffu, ok);
      if (ok) ok = mbar_wait(AB_EMPTY(s), ph ^ 1u, abort_flag, (k << 8) | 5);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      const unsigned char* raw = sm + L.raw0 + s * L.raw_bytes;
      const uint32_t abase = base + L.a0 + s * L.a_bytes;
#pragma unroll
      for (int tt = 0; tt < 2; tt++) {
        const int tl = warp * 2 + tt;
#pragma unroll
        for (int blk = 0; blk < 2; blk++) {
          const int sl = tl * 2 + blk;
          const __half2 dd = reinterpret_cast<const __half2*>(raw + L.d_off)[sl * 8 + g];
          const __half2 dg = __low2half2(dd), dg8 = __high2half2(dd);
          __half2 mg = __float2half2_rn(0.f), mg8 = mg;
          if (has_m) {
            const __half2 mm = reinterpret_cast<const __half2*>(raw + L.m_off)[sl * 8 + g];
            mg = __low2half2(mm);
            mg8 = __high2half2(mm);
          }
          uint4 q;
          uint32_t hb = 0;
          if (QT == WG_QTYPE_Q8_0) q = reinterpret_cast<const uint4*>(raw + L.qs_off)[sl * 32 + lane];
          else {
            uint2 v = reinterpret_cast<const uint2*>(raw + L.qs_off)[sl * 32 + lane];
            q = make_uint4(v.x, v.y, 0, 0);
          }
          if (has_h) hb = reinterpret_cast<const uint16_t*>(raw + L.hb_off)[sl * 32 + lane];
#pragma unroll
          for (int st = 0; st < 2; st++) {
            uint32_t a[4];
            if (QT == WG_QTYPE_Q8_0) {
              uint32_t w0 = (st ? q.z : q.x) ^ 0x80808080u, w1 = (st ? q.w : q.y) ^ 0x80808080u;
              const __half2 bias = __float2half2_rn(1152.f);
              a[0] = h2u(__hmul2(__hsub2(u2h(__byte_perm(w0, 0x64, 0x4140)), bias), dg));
              a[1] = h2u(__hmul2(__hsub2(u2h(__byte_perm(w0, 0x64, 0x4342)), bias), dg8));
              a[2] = h2u(__hmul2(__hsub2(u2h(__byte_perm(w1, 0x64, 0x4140)), bias), dg));
              a[3] = h2u(__hmul2(__hsub2(u2h(__byte_perm(w1, 0x64, 0x4342)), bias), dg8));
            } else {
              uint32_t w = st ? q.y : q.x;
#pragma unroll
              for (int r = 0; r < 4; r++) {
                uint32_t hq = ((w >> (4 * r)) & 0x000F000Fu) | 0x64006400u;
                if (has_h) {
                  uint32_t b = (hb >> (2 * (4 * st + r))) & 3u;
                  hq |= ((b & 1u) << 4) | ((b >> 1) << 20);
                }
                const __half2 d = (r & 1) ? dg8 : dg;
                __half2 v;
                if (QT == WG_QTYPE_Q4_0) v = __hmul2(__hsub2(u2h(hq), __float2half2_rn(1032.f)), d);
                else if (QT == WG_QTYPE_Q5_0) v = __hmul2(__hsub2(u2h(hq), __float2half2_rn(1040.f)), d);
                else v = __hfma2(__hsub2(u2h(hq), __float2half2_rn(1024.f)), d, (r & 1) ? mg8 : mg);
                a[r] = h2u(v);
              }
            }
            asm volatile("stmatrix.sync.aligned.m8n8.x4.shared.b16 [%0], {%1, %2, %3, %4};" ::"r"(
                             abase + soff[tt][blk][st]),
                         "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3])
                         : "memory");
          }
        }
      }
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(RAW_EMPTY(s));
        mbar_arrive(MMA_FULL(s));
      }
    }
    // ---------------- epilogue: TMEM lanes 32w..32w+31 ----------------
    bool done_ok = mbar_wait(DONE, 0, abort_flag, 6);
    done_ok = __all_sync(0xffffffffu, done_ok);
    if (done_ok) {
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      // Everything the stores need is read before the first store, so no
      // load waits behind a store it cannot be proven not to alias.
      const int n = tile0 * 16 + warp * 32 + lane;
      const bool nok = n < e.N;
      const int nn = nok ? n : 0;
      float bias_n = 0.f;
      int64_t col_off = 0, row_stride = 0;  // output element (r, n) at base + r * row_stride + col_off
      if (e.mode == EPI_F32 || e.mode == EPI_RESID || e.mode == EPI_GELU_F16) {
        bias_n = e.bias ? e.bias[nn] : 0.f;
        col_off = nn;
        row_stride = e.ldo;
      } else if (e.mode == EPI_QKV) {
        const int seg = nn / e.d, j = nn - seg * e.d, h = j / e.hd, c = j - h * e.hd;
        if (seg == 0) {
          bias_n = e.bias_q[j];
          col_off = j;
          row_stride = e.ldo;
        } else {
          bias_n = seg == 2 ? e.bias_v[j] : 0.f;
          const int p = *e.pos;
          col_off = (((int64_t)(seg - 1) * e.H + h) * e.T + p) * e.hd + c;
          row_stride = (int64_t)2 * e.H * e.T * e.hd;
        }
      } else {  // EPI_CROSS_KV: r = u*T + t
        const int lk = nn / e.d, j = nn - lk * e.d, l = lk >> 1, kv = lk & 1, h = j / e.hd, c = j - h * e.hd;
        bias_n = kv ? e.bias_v[(int64_t)l * e.d + j] : 0.f;
        col_off = (((int64_t)l * e.U * 2 + kv) * e.H + h) * (int64_t)e.T * e.hd + c;
      }
      const bool qkv_q = e.mode == EPI_QKV && nn < e.d;
      for (int c0 = 0; c0 < NR; c0 += 16) {
        uint32_t v[16];
        const uint32_t taddr = tmem + ((uint32_t)(warp * 32) << 16) + (uint32_t)c0;
        asm volatile(
            "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
            : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
              "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
            : "r"(taddr));
        asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
        if (!nok) continue;
        const int rb = r0 + c0;
        if (e.mode == EPI_RESID) {
          // x += (acc + b): one writer per element, so the reduction-add is
          // deterministic and rounds exactly like the load-add-store
#pragma unroll
          for (int i = 0; i < 16; i++)
            if (rb + i < R)
              asm volatile("red.global.add.f32 [%0], %1;" ::"l"(e.out + (int64_t)(rb + i) * row_stride + col_off),
                           "f"(__fadd_rn(__uint_as_float(v[i]), bias_n))
                           : "memory");
        } else if (e.mode == EPI_F32 || qkv_q) {
#pragma unroll
          for (int i = 0; i < 16; i++)
            if (rb + i < R) e.out[(int64_t)(rb + i) * row_stride + col_off] = __fadd_rn(__uint_as_float(v[i]), bias_n);
        } else if (e.mode == EPI_GELU_F16) {
#pragma unroll
          for (int i = 0; i < 16; i++)
            if (rb + i < R)
              e.out16[(int64_t)(rb + i) * row_stride + col_off] =
                  __float2half_rn(tc_gelu(__fadd_rn(__uint_as_float(v[i]), bias_n)));
        } else if (e.mode == EPI_QKV) {
#pragma unroll
          for (int i = 0; i < 16; i++)
            if (rb + i < R)
              e.kv[(int64_t)(rb + i) * row_stride + col_off] = __float2half_rn(__fadd_rn(__uint_as_float(v[i]), bias_n));
        } else {  // EPI_CROSS_KV
#pragma unroll
          for (int i = 0; i < 16; i++) {
            const int r = rb + i;
            if (r < R) {
              const int u = r / e.T, tt = r - u * e.T;
              e.kv[col_off + (int64_t)u * 2 * e.H * e.T * e.hd + (int64_t)tt * e.hd] =
                  __float2half_rn(__fadd_rn(__uint_as_float(v[i]), bias_n));
            }
          }
        }
      }
    }
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 5) {
    __syncwarp();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(ncols) : "memory");
  }
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static bool tried = false;
  if (!tried) {
    tried = true;
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

template <uint32_t QT>
int launch_tc_t(const DMat& W, const __half* X, int ldx, int R, const Epi& e, cudaStream_t st) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) {
    set_error("cuTensorMapEncodeTiled is unavailable");
    return WG_ERR_CUDA;
  }
  const int ntiles_r = (R + 255) / 256;
  int NR = (R + ntiles_r - 1) / ntiles_r;
  NR = (NR + 15) / 16 * 16;
  if (NR < 16) NR = 16;
  CUtensorMap map;
  cuuint64_t dims[2] = {(cuuint64_t)W.cols, (cuuint64_t)R};
  cuuint64_t strides[1] = {(cuuint64_t)ldx * 2};
  cuuint32_t box[2] = {(cuuint32_t)TC_BK, (cuuint32_t)NR};
  cuuint32_t estr[2] = {1, 1};
  CUresult cr = enc(&map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<__half*>(X), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (cr != CUDA_SUCCESS) {
    set_error("cuTensorMapEncodeTiled failed (%d)", (int)cr);
    return WG_ERR_CUDA;
  }
  const TcLayout L = tc_layout(QT, NR);
  dim3 grid((W.ntiles + 7) / 8, (R + NR - 1) / NR);
  gemm_tc_kernel<QT><<<grid, TC_THREADS, L.total, st>>>(W, map, R, NR, e);
  return launch_status("gemm_tc");
}

template <uint32_t QT>
int configure_tc_t() {
  cudaError_t e = cudaFuncSetAttribute(gemm_tc_kernel<QT>, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
  if (e != cudaSuccess) {
    set_error("cudaFuncSetAttribute(gemm_tc): %s", cudaGetErrorString(e));
    return WG_ERR_CUDA;
  }
  return WG_OK;
}

}  // namespace

bool tc_supported(const DMat& W) { return qtype_is_quant(W.qtype) && W.cols % TC_BK == 0; }

int init_tc_attributes() {
  int rc = configure_tc_t<WG_QTYPE_Q8_0>();
  if (rc == WG_OK) rc = configure_tc_t<WG_QTYPE_Q4_0>();
  if (rc == WG_OK) rc = configure_tc_t<WG_QTYPE_Q4_1>();
  if (rc == WG_OK) rc = configure_tc_t<WG_QTYPE_Q5_0>();
  if (rc == WG_OK) rc = configure_tc_t<WG_QTYPE_Q5_1>();
  return rc;
}

int tc_error_word(int* word, bool clear) {
  int v = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, g_tc_error, sizeof(int));
  if (e != cudaSuccess) {
    set_error("reading the tcgen05 error word: %s", cudaGetErrorString(e));
    return WG_ERR_CUDA;
  }
  if (clear && v) {
    int z = 0;
    cudaMemcpyToSymbol(g_tc_error, &z, sizeof(int));
  }
  *word = v;
  return WG_OK;
}

int launch_matmul_tc(const DMat& W, const __half* X, int ldx, int R, const Epi& e, cudaStream_t st) {
  switch (W.qtype) {
    case WG_QTYPE_Q8_0: return launch_tc_t<WG_QTYPE_Q8_0>(W, X, ldx, R, e, st);
    case WG_QTYPE_Q4_0: return launch_tc_t<WG_QTYPE_Q4_0>(W, X, ldx, R, e, st);
    case WG_QTYPE_Q4_1: return launch_tc_t<WG_QTYPE_Q4_1>(W, X, ldx, R, e, st);
    case WG_QTYPE_Q5_0: return launch_tc_t<WG_QTYPE_Q5_0>(W, X, ldx, R, e, st);
    case WG_QTYPE_Q5_1: return launch_tc_t<WG_QTYPE_Q5_1>(W, X, ldx, R, e, st);
    default:
      set_error("tcgen05 path: unsupported tensor type %u", W.qtype);
      return WG_ERR_UNSUPPORTED;
  }
}

}  // namespace wg
