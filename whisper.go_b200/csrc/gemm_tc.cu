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
//   warp 18 (one thread): cp.async.bulk of the raw quant payloads of the
//     CTA's 128 x 64 weight group (16 contiguous tile128 slots: one copy per
//     plane) -> RAW[s], a ring of TC_DQ_NS stages
//   warp 17 (one thread): TMA 2-D tile load of X[NR, 64] (f16, 128B swizzle)
//     -> B[s] in shared memory
//   warps 0-15: two groups of 8 on alternating stages; each warp dequantises
//     one row tile of RAW[s] (f16 = d*q rounded once) and stores it into
//     the stage's A tile in tensor memory (tcgen05.st.16x256b)
//   warp 16 (one thread): 4 x tcgen05.mma.kind::f16 (K=16, A from tensor
//     memory, B from shared memory) into the TMEM accumulator, then
//     tcgen05.commit frees the stage
// K may be split over a thread-block cluster of ks CTAs (grid z); the
// epilogue then reduces the partial tiles through distributed shared memory
// in rank order (deterministic), and stores through the Epi (bias /
// residual / GELU / KV-cache scatter) with vector accesses.
// Every mbarrier wait is bounded; on expiry the kernel records an error
// word, stops waiting and still frees its TMEM.
#include <cooperative_groups.h>

#include <algorithm>

#include "async.cuh"
#include "kernels.cuh"

namespace cg = cooperative_groups;

namespace wg {
namespace {

constexpr int TC_BM = 128;      // weight rows per CTA (8 tile16 tiles)
constexpr int TC_BK = 64;       // K per stage
constexpr int TC_DQ_WARPS = 16;   // dequantisers (two groups of 8, alternate stages) and TMEM readers
constexpr int TC_MMA_WARP = 16;   // TMEM owner and MMA issuer
constexpr int TC_XLOAD_WARP = 17; // activation TMA loader
constexpr int TC_WLOAD_WARP = 18; // weight bulk-copy loader
constexpr int TC_THREADS = 19 * 32;
constexpr int TC_DQ_NS = 6;       // weight stages in flight (raw ring depth)
// Lanes issuing copies in each loader warp (stage kl from lane kl % lanes).
// The copies of an SM share its L2 ingest (~110-120 GB/s); with one lane they
// complete in stage order, which is the order the pipeline consumes them,
// while several lanes make the stages in flight share the bandwidth and each
// one land later. Measured: 1 lane is fastest for these GEMMs.
constexpr int TC_LOAD_LANES = 1;
static_assert(TC_LOAD_LANES <= TC_DQ_NS, "a loader lane must never wait for a slot of its own round");
__device__ int g_tc_error;  // first expired wait: (stage << 8) | role

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
// Shared memory: S stages of B (activation tiles), as many as fit in 220 KB
// next to the RAW ring (TC_DQ_NS stages of quant payloads), then the
// mbarriers. The dequantised A tiles live in tensor memory: the accumulator
// at columns 0..NR-1 (NR <= 256), then per stage s the weight tile's f16
// high part (128 lanes x 64 f16 = 32 columns) at tc_a_col(NR) + 64 s and its
// low part (the f16 rounding error of the high part) 32 columns further:
// the MMA adds both, so the weights enter the product with ~22 bits.
constexpr int TC_S_MAX = 8;
constexpr uint32_t TC_TMEM_COLS = 512;
__host__ __device__ inline uint32_t tc_a_col(int NR) { return (uint32_t)(NR + 31) / 32 * 32; }
struct TcLayout {
  int stages;                    // A/B ring depth
  uint32_t b_bytes;
  uint32_t raw_bytes;            // one RAW stage: 16 slots x {32 x pb | d | m | hb}
  uint32_t b0, raw0, bar0, total;
};

__host__ __device__ inline TcLayout tc_layout(uint32_t qt, int NR) {
  TcLayout L{};
  L.b_bytes = (uint32_t)NR * TC_BK * 2;
  // d at 16*32*pb, m at +512, hb at +1024 (the m gap is kept when only hb is present)
  L.raw_bytes = 16 * 32 * qtype_payload_bytes(qt) + 512 + ((qtype_has_min(qt) || qtype_has_hbits(qt)) ? 512 : 0) +
                (qtype_has_hbits(qt) ? 1024 : 0);
  const uint32_t raw = TC_DQ_NS * L.raw_bytes;
  L.stages = (int)((220u * 1024u - raw) / L.b_bytes);
  if (L.stages > TC_S_MAX) L.stages = TC_S_MAX;
  const int a_stages = (int)((TC_TMEM_COLS - tc_a_col(NR)) / 64);  // hi + lo tiles per stage
  if (L.stages > a_stages) L.stages = a_stages;
  L.b0 = 0;
  L.raw0 = L.b0 + L.stages * L.b_bytes;
  L.bar0 = L.raw0 + raw;
  // barriers, abort flag + tmem slot, drain bookkeeping per ring slot, slack
  L.total = L.bar0 + 8 * (2 * TC_S_MAX + 2 * TC_DQ_NS + 1) + 16 + 4 * (2 * TC_S_MAX + TC_DQ_NS) + 1024;
  return L;
}

// Output addressing of weight row n (fixed per thread in the epilogues):
// element (r, n) is at base + r * row_stride + col_off, except CROSS_KV whose
// rows r = u*T + t add u * 2*H*T*hd + t*hd.
struct TcEpiRow {
  int64_t col_off, row_stride;
  float bias;
  bool ok;
};

__device__ __forceinline__ TcEpiRow tc_epi_row(const Epi& e, int n, int pos) {
  TcEpiRow er{0, 0, 0.f, n < e.N};
  const int nn = er.ok ? n : 0;
  if (e.mode == EPI_F32 || e.mode == EPI_RESID || e.mode == EPI_GELU_F16) {
    er.bias = e.bias ? e.bias[nn] : 0.f;
    er.col_off = nn;
    er.row_stride = e.ldo;
  } else if (e.mode == EPI_QKV) {
    const int seg = nn / e.d, j = nn - seg * e.d, h = j / e.hd, c = j - h * e.hd;
    if (seg == 0) {
      er.bias = e.bias_q[j];
      er.col_off = j;
      er.row_stride = e.ldo;
    } else {
      er.bias = seg == 2 ? e.bias_v[j] : 0.f;
      er.col_off = (((int64_t)(seg - 1) * e.H + h) * e.T + pos) * e.hd + c;
      er.row_stride = (int64_t)2 * e.H * e.T * e.hd;
    }
  } else {  // EPI_CROSS_KV
    const int lk = nn / e.d, j = nn - lk * e.d, l = lk >> 1, kv = lk & 1, h = j / e.hd, c = j - h * e.hd;
    er.bias = kv ? e.bias_v[(int64_t)l * e.d + j] : 0.f;
    er.col_off = (((int64_t)l * e.U * 2 + kv) * e.H + h) * (int64_t)e.T * e.hd + c;
  }
  return er;
}

// Bias of weight row n (model data only; no state written by the token loop).
__device__ __forceinline__ float tc_epi_bias(const Epi& e, int n) {
  if (n >= e.N) return 0.f;
  if (e.mode == EPI_F32 || e.mode == EPI_RESID || e.mode == EPI_GELU_F16) return e.bias ? e.bias[n] : 0.f;
  if (e.mode == EPI_QKV) {
    const int seg = n / e.d, j = n - seg * e.d;
    return seg == 0 ? e.bias_q[j] : (seg == 2 ? e.bias_v[j] : 0.f);
  }
  const int lk = n / e.d, j = n - lk * e.d;  // EPI_CROSS_KV
  return (lk & 1) ? e.bias_v[(int64_t)(lk >> 1) * e.d + j] : 0.f;
}

// Stores acc of rows r0, r0+1, ..., r0+cnt-1 (v[i] for row r0+i) of weight row n.
template <int CNT>
__device__ __forceinline__ void tc_epi_store_run(const Epi& e, const TcEpiRow& er, bool qkv_q, int r0, int R,
                                                 const float* v) {
  if (e.mode == EPI_CROSS_KV) {
    int u = r0 / e.T, tt = r0 - u * e.T;  // one division per run
    const int64_t ustride = (int64_t)2 * e.H * e.T * e.hd;
#pragma unroll
    for (int i = 0; i < CNT; i++) {
      if (r0 + i < R)
        e.kv[er.col_off + (int64_t)u * ustride + (int64_t)tt * e.hd] = __float2half_rn(__fadd_rn(v[i], er.bias));
      if (++tt == e.T) { tt = 0; u++; }
    }
    return;
  }
#pragma unroll
  for (int i = 0; i < CNT; i++) {
    if (r0 + i >= R) break;
    const float x = __fadd_rn(v[i], er.bias);
    const int64_t idx = (int64_t)(r0 + i) * er.row_stride + er.col_off;
    if (e.mode == EPI_RESID) {
      // x += (acc + b): one writer per element, so the reduction-add is
      // deterministic and rounds exactly like the load-add-store
      asm volatile("red.global.add.f32 [%0], %1;" ::"l"(e.out + idx), "f"(x) : "memory");
    } else if (e.mode == EPI_F32 || qkv_q) {
      e.out[idx] = x;
    } else if (e.mode == EPI_GELU_F16) {
      e.out16[idx] = __float2half_rn(gelu_f32(x));
    } else {
      e.kv[idx] = __float2half_rn(x);
    }
  }
}

// Stores x[0..cnt) of weight rows n0..n0+cnt-1 of one activation row, which
// sit at idx, idx+1, ... of the output: one vector access when all four are
// valid and the address is aligned. EPI_RESID adds with a vector reduction
// (one writer per element, so it rounds exactly like load-add-store).
__device__ __forceinline__ void tc_store_quad(const Epi& e, bool qkv_q, int64_t idx, const float* x, int cnt) {
  if (e.mode == EPI_RESID || e.mode == EPI_F32 || qkv_q) {
    float* p = e.out + idx;
    if (cnt == 4 && (reinterpret_cast<uintptr_t>(p) & 15) == 0) {
      if (e.mode == EPI_RESID)
        asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(p), "f"(x[0]), "f"(x[1]), "f"(x[2]),
                     "f"(x[3])
                     : "memory");
      else
        *reinterpret_cast<float4*>(p) = make_float4(x[0], x[1], x[2], x[3]);
      return;
    }
    for (int i = 0; i < cnt; i++) {
      if (e.mode == EPI_RESID) asm volatile("red.global.add.f32 [%0], %1;" ::"l"(p + i), "f"(x[i]) : "memory");
      else p[i] = x[i];
    }
    return;
  }
  __half* p = (e.mode == EPI_GELU_F16 ? e.out16 : e.kv) + idx;
  float y[4];
#pragma unroll
  for (int i = 0; i < 4; i++) y[i] = e.mode == EPI_GELU_F16 ? gelu_f32(x[i]) : x[i];
  if (cnt == 4 && (reinterpret_cast<uintptr_t>(p) & 7) == 0) {
    const __half2 h0 = __floats2half2_rn(y[0], y[1]), h1 = __floats2half2_rn(y[2], y[3]);
    *reinterpret_cast<uint2*>(p) = make_uint2(h2u(h0), h2u(h1));
    return;
  }
  for (int i = 0; i < cnt; i++) p[i] = __float2half_rn(y[i]);
}

// grid (weight groups, row tiles, K splits); a K split > 1 runs as a thread
// block cluster along z whose CTAs reduce their partial tiles through
// distributed shared memory in rank order (deterministic).
template <uint32_t QT>
__global__ void __launch_bounds__(TC_THREADS, 1)
    gemm_tc_kernel(DMat W, const __grid_constant__ CUtensorMap xmap, int R, int NR, int ks, Epi e) {
  extern __shared__ __align__(1024) unsigned char tc_smem_raw[];
  unsigned char* sm = tc_smem_raw + ((1024 - (smem_u32(tc_smem_raw) & 1023)) & 1023);
  // the next kernel of the stream may be scheduled now; this one waits for
  // its predecessors (pdl_wait) only where it reads activations or writes
  // outputs: barrier set-up, TMEM allocation and the weight stream (weights
  // are never written by kernels of the token loop) run before that
  pdl_trigger();
  const TcLayout L = tc_layout(QT, NR);
  const int S = L.stages;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int* const errw = e.err_word ? e.err_word : &g_tc_error;
  const uint32_t a_col = tc_a_col(NR);
  const uint64_t wait_ns = e.test_wait_ns ? e.test_wait_ns : WAIT_NS;
  const int tile0 = blockIdx.x * 8;
  const int r0 = blockIdx.y * NR;
  const int nk_all = W.cols / TC_BK;
  const int per = (nk_all + ks - 1) / ks;
  const int kbeg = blockIdx.z * per;
  const int nk = min(nk_all, kbeg + per) - kbeg;  // >= 1 (host choice of ks)
  // CTAs of different weight groups start their K walk at different stages,
  // so the activation panel they all read is not requested from the same L2
  // lines by every SM at once
  const int krot = (int)(blockIdx.x % (unsigned)nk);
  auto kstage = [&](int kl) { const int k = kl + krot; return kbeg + (k >= nk ? k - nk : k); };
  const uint32_t base = smem_u32(sm);
  const uint32_t bar = base + L.bar0;
  constexpr int NBAR = 2 * TC_S_MAX + 2 * TC_DQ_NS;
  // FULL[s]: the stage's dequant group (8 arrivals) + the activation copy
  // (1 arrival + bytes); EMPTY[s]: the MMAs that read the stage completed
  auto FULL = [&](int s) { return bar + 8 * s; };
  auto EMPTY = [&](int s) { return bar + 8 * (TC_S_MAX + s); };
  auto RAW_FULL = [&](int s) { return bar + 8 * (2 * TC_S_MAX + s); };
  auto RAW_EMPTY = [&](int s) { return bar + 8 * (2 * TC_S_MAX + TC_DQ_NS + s); };
  const uint32_t DONE = bar + 8 * NBAR;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(sm + L.bar0 + 8 * (NBAR + 1));
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sm + L.bar0 + 8 * (NBAR + 1) + 4);
  // Drain bookkeeping: last stage whose copy was issued into each activation /
  // weight ring slot (-1: none) and the dequant arrivals made on each FULL[s]
  // so far; after an abort the copies still in flight are waited for.
  volatile int* issued_x = reinterpret_cast<volatile int*>(sm + L.bar0 + 8 * (NBAR + 1) + 16);
  volatile int* issued_w = issued_x + TC_S_MAX;
  int* dq_arrivals = const_cast<int*>(issued_w + TC_DQ_NS);
  constexpr int pb = QT == WG_QTYPE_Q8_0 ? 16 : 8;
  constexpr bool has_m = QT == WG_QTYPE_Q4_1 || QT == WG_QTYPE_Q5_1;
  constexpr bool has_h = QT == WG_QTYPE_Q5_0 || QT == WG_QTYPE_Q5_1;
  // weight stage kl: bulk copies of its 16 contiguous slots into the RAW ring
  // raw ring slot (per stage): qs [16][32][pb] | d [16][8] half2 | m [16][8] half2 | hb [16][32] u16
  auto issue_weights = [&](int kl) {
    constexpr uint32_t qs_b = 16 * 32 * pb;
    constexpr uint32_t tx = qs_b + 512 + (has_m ? 512 : 0) + (has_h ? 1024 : 0);
    const int s = kl % TC_DQ_NS;
    const uint32_t dst = base + L.raw0 + s * L.raw_bytes;
    const int64_t g0 = slot_of(W, tile0, 2 * kstage(kl));  // 16 contiguous slots: tile t, blocks 0/1
    mbar_arrive_tx(RAW_FULL(s), tx);
    bulk_g2s(dst, W.qs + g0 * 32 * pb, qs_b, RAW_FULL(s));
    bulk_g2s(dst + qs_b, W.dsc + g0 * 8, 512, RAW_FULL(s));
    if (has_m) bulk_g2s(dst + qs_b + 512, W.msc + g0 * 8, 512, RAW_FULL(s));
    if (has_h) bulk_g2s(dst + qs_b + 1024, W.hb + g0 * 32, 1024, RAW_FULL(s));
    issued_w[s] = kl;
  };
  // The weight loader initialises the RAW ring's barriers itself and issues
  // the ring's first stages at once (their slots are free), so the weight
  // stream overlaps the TMEM allocation and the block barrier below.
  const int n_pre = min(nk, TC_DQ_NS);
  if (warp == TC_WLOAD_WARP) {
    if (lane == 0) {
      for (int s = 0; s < TC_DQ_NS; s++) {
        mbar_init(RAW_FULL(s), 1);
        mbar_init(RAW_EMPTY(s), 8);
        issued_w[s] = -1;
      }
      asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncwarp();
    if (lane == 0)
      for (int kl = 0; kl < n_pre; kl++) issue_weights(kl);
  }
  if (threadIdx.x == 0) {
    for (int s = 0; s < S; s++) {
      mbar_init(FULL(s), 8 + 1);
      mbar_init(EMPTY(s), 1);
      issued_x[s] = -1;
      dq_arrivals[s] = 0;
    }
    mbar_init(DONE, 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  const uint32_t ncols = TC_TMEM_COLS;
  if (warp == TC_MMA_WARP) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(ncols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = *tmem_slot;

  if (warp == TC_WLOAD_WARP) {
    // ---------------- weight loader: the remaining stages ----------------
    // (TC_LOAD_LANES <= TC_DQ_NS: a lane only waits for slots that stages
    // issued in earlier rounds occupy)
    for (int k0 = n_pre; k0 < nk; k0 += TC_LOAD_LANES) {
      const int kl = k0 + lane;
      bool ok = true;
      if (lane < TC_LOAD_LANES && kl < nk) {
        const int s = kl % TC_DQ_NS;
        const uint32_t ph = (uint32_t)(kl / TC_DQ_NS) & 1u;
        ok = mbar_wait(RAW_EMPTY(s), ph ^ 1u, abort_flag, (kl << 8) | 1, errw, wait_ns);
        if (ok) issue_weights(kl);
      }
      if (!__all_sync(0xffffffffu, ok)) break;
    }
  } else if (warp == TC_XLOAD_WARP) {
    // ---------------- activation loader ----------------
    pdl_wait();
    const int lanes = min(TC_LOAD_LANES, S);
    for (int k0 = 0; k0 < nk; k0 += lanes) {
      const int kl = k0 + lane;
      bool ok = true;
      if (lane < lanes && kl < nk) {
        const int s = kl % S;
        const uint32_t ph = (uint32_t)(kl / S) & 1u;
        ok = mbar_wait(EMPTY(s), ph ^ 1u, abort_flag, (kl << 8) | 2, errw, wait_ns);
        if (ok && !(e.test_stall && kl == 0)) {
          mbar_arrive_tx(FULL(s), L.b_bytes);
          tma_2d(base + L.b0 + s * L.b_bytes, &xmap, kstage(kl) * TC_BK, r0, FULL(s));
          issued_x[s] = kl;
        }
      }
      if (!__all_sync(0xffffffffu, ok)) break;
    }
  } else if (warp == TC_MMA_WARP) {
    if (lane == 0) {
      // ---------------- MMA issuer ----------------
      const uint32_t idesc = (1u << 4)                          // D format: f32
                             | (0u << 7) | (0u << 10)           // A, B: f16
                             | ((uint32_t)(NR >> 3) << 17)      // N
                             | ((uint32_t)(TC_BM >> 4) << 24);  // M
      for (int kl = 0; kl < nk; kl++) {
        const int s = kl % S;
        if (!mbar_wait(FULL(s), (uint32_t)(kl / S) & 1u, abort_flag, (kl << 8) | 3, errw, wait_ns)) break;
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint32_t at = tmem + a_col + 64u * (uint32_t)s;  // A (high, then low part) in tensor memory
        const uint64_t bd = sw128_desc(base + L.b0 + s * L.b_bytes);
#pragma unroll
        for (int kk = 0; kk < 4; kk++) {
#pragma unroll
          for (int part = 0; part < 2; part++) {
            const uint32_t acc = (kl > 0 || kk > 0 || part > 0) ? 1u : 0u;
            asm volatile(
                "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
                " tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n}\n" ::"r"(tmem),
                "r"(at + 32u * part + (uint32_t)(kk * 8)), "l"(bd + (uint64_t)(kk * 2)), "r"(idesc), "r"(acc)
                : "memory");
          }
        }
        asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(EMPTY(s))
                     : "memory");
      }
      asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(DONE)
                   : "memory");
    }
  } else {
    // ---------------- dequantisers ----------------
    // group grp = warp / 8 takes the stages kl = grp (mod 2), so the two
    // groups' wait / dequantise / store chains overlap. Warp w may only
    // address tensor-memory lanes 32(w%4)..32(w%4)+31, so it owns row tile
    // 2(w%4) + (w/4)%2 (rows = TMEM lanes 16*tile..16*tile+15)
    const int g = lane >> 2, grp = warp >> 3, tile = 2 * (warp & 3) + ((warp >> 2) & 1);
    const uint32_t tlane = (uint32_t)(16 * tile) << 16;
    // this warp's two slots (blocks 0/1 of its tile) inside a raw stage
    const uint32_t d_off = 16 * 32 * pb, m_off = d_off + 512, hb_off = m_off + 512;
    const unsigned char* rq = sm + L.raw0 + (2 * tile) * 32 * pb;
    const unsigned char* rd = sm + L.raw0 + d_off + (2 * tile) * 32;
    const unsigned char* rm = sm + L.raw0 + m_off + (2 * tile) * 32;
    const unsigned char* rh = sm + L.raw0 + hb_off + (2 * tile) * 64;
    for (int kl = grp; kl < nk; kl += 2) {
      const int s = kl % S;
      const uint32_t ph = (uint32_t)(kl / S) & 1u;
      const int rs = kl % TC_DQ_NS;
      bool ok = mbar_wait2(RAW_FULL(rs), (uint32_t)(kl / TC_DQ_NS) & 1u, EMPTY(s), ph ^ 1u, abort_flag,
                           (kl << 8) | 4, errw, wait_ns);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      const uint32_t ro = rs * L.raw_bytes;
      // the stage's 16 rows x 64 k in tcgen05.st.16x256b order: the f16 high
      // part of every weight and its low part (the rounding error of the high
      // part, an exact f16 FMA residual; the _1 types split d*q + m computed
      // in float32 like the reference)
      uint32_t tr[16], tl[16];
#pragma unroll
      for (int blk = 0; blk < 2; blk++) {
        const __half2 dd = reinterpret_cast<const __half2*>(rd + ro)[blk * 8 + g];
        const __half2 dg = __low2half2(dd), dg8 = __high2half2(dd);
        __half2 mg = __float2half2_rn(0.f), mg8 = mg;
        if (has_m) {
          const __half2 mm = reinterpret_cast<const __half2*>(rm + ro)[blk * 8 + g];
          mg = __low2half2(mm);
          mg8 = __high2half2(mm);
        }
        uint4 q;
        uint32_t hb = 0;
        if (QT == WG_QTYPE_Q8_0) q = reinterpret_cast<const uint4*>(rq + ro)[blk * 32 + lane];
        else {
          uint2 v = reinterpret_cast<const uint2*>(rq + ro)[blk * 32 + lane];
          q = make_uint4(v.x, v.y, 0, 0);
        }
        if (has_h) hb = reinterpret_cast<const uint16_t*>(rh + ro)[blk * 32 + lane];
#pragma unroll
        for (int st = 0; st < 2; st++) {
          uint32_t a[4], al[4];
          __half2 qv[4];
          if (QT == WG_QTYPE_Q8_0) {
            uint32_t w0 = (st ? q.z : q.x) ^ 0x80808080u, w1 = (st ? q.w : q.y) ^ 0x80808080u;
            const __half2 bias = __float2half2_rn(1152.f);
            qv[0] = __hsub2(u2h(__byte_perm(w0, 0x64, 0x4140)), bias);
            qv[1] = __hsub2(u2h(__byte_perm(w0, 0x64, 0x4342)), bias);
            qv[2] = __hsub2(u2h(__byte_perm(w1, 0x64, 0x4140)), bias);
            qv[3] = __hsub2(u2h(__byte_perm(w1, 0x64, 0x4342)), bias);
          } else {
            uint32_t w = st ? q.y : q.x;
#pragma unroll
            for (int r = 0; r < 4; r++) {
              uint32_t hq = ((w >> (4 * r)) & 0x000F000Fu) | 0x64006400u;
              if (has_h) {
                uint32_t b = (hb >> (2 * (4 * st + r))) & 3u;
                hq |= ((b & 1u) << 4) | ((b >> 1) << 20);
              }
              const float off = QT == WG_QTYPE_Q4_0 ? 1032.f : (QT == WG_QTYPE_Q5_0 ? 1040.f : 1024.f);
              qv[r] = __hsub2(u2h(hq), __float2half2_rn(off));
            }
          }
#pragma unroll
          for (int r = 0; r < 4; r++) {
            const __half2 d = (r & 1) ? dg8 : dg;
            if (has_m) {
              const float2 qf = __half22float2(qv[r]), df = __half22float2(d);
              const float2 mf = __half22float2((r & 1) ? mg8 : mg);
              const float v0 = __fadd_rn(__fmul_rn(df.x, qf.x), mf.x), v1 = __fadd_rn(__fmul_rn(df.y, qf.y), mf.y);
              const __half2 hi = __floats2half2_rn(v0, v1);
              const float2 hf = __half22float2(hi);
              a[r] = h2u(hi);
              al[r] = h2u(__floats2half2_rn(__fsub_rn(v0, hf.x), __fsub_rn(v1, hf.y)));
            } else {
              const __half2 hi = __hmul2(qv[r], d);
              a[r] = h2u(hi);
              al[r] = h2u(__hfma2(qv[r], d, __hneg2(hi)));
            }
          }
          // a: (row g, k 4t..4t+1), (row g+8, same k), (row g, k 4t+2..4t+3), (row g+8, ...);
          // the store wants row g's two 32-bit columns, then row g+8's
          const int o = (blk * 2 + st) * 4;
          tr[o] = a[0];
          tr[o + 1] = a[2];
          tr[o + 2] = a[1];
          tr[o + 3] = a[3];
          tl[o] = al[0];
          tl[o + 1] = al[2];
          tl[o + 2] = al[1];
          tl[o + 3] = al[3];
        }
      }
      const uint32_t ta = tmem + tlane + a_col + 64u * (uint32_t)s;
      asm volatile(
          "tcgen05.st.sync.aligned.16x256b.x4.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::
              "r"(ta),
          "r"(tr[0]), "r"(tr[1]), "r"(tr[2]), "r"(tr[3]), "r"(tr[4]), "r"(tr[5]), "r"(tr[6]), "r"(tr[7]), "r"(tr[8]),
          "r"(tr[9]), "r"(tr[10]), "r"(tr[11]), "r"(tr[12]), "r"(tr[13]), "r"(tr[14]), "r"(tr[15])
          : "memory");
      asm volatile(
          "tcgen05.st.sync.aligned.16x256b.x4.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::
              "r"(ta + 32u),
          "r"(tl[0]), "r"(tl[1]), "r"(tl[2]), "r"(tl[3]), "r"(tl[4]), "r"(tl[5]), "r"(tl[6]), "r"(tl[7]), "r"(tl[8]),
          "r"(tl[9]), "r"(tl[10]), "r"(tl[11]), "r"(tl[12]), "r"(tl[13]), "r"(tl[14]), "r"(tl[15])
          : "memory");
      asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
      asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(RAW_EMPTY(rs));
        mbar_arrive(FULL(s));
        atomicAdd(&dq_arrivals[s], 1);
      }
    }
  }

  // ---------------- epilogue ----------------
  // (1) warps 0-15 move the fp32 accumulator tile out of TMEM (warp w reads
  //     lanes 32(w%4).. = weight rows of this CTA, the four warps of a lane
  //     quarter split the NR columns) into a [NR][128] partial tile: in
  //     shared memory (the stage ring, free once DONE has fired) when K is
  //     not split, else in this CTA's slice of the split-K workspace in
  //     global memory (L2-resident; distributed shared memory moved such
  //     tiles at a fraction of L2's per-SM bandwidth).
  // (2) barrier (CTA, or cluster: release / acquire at cluster scope, so the
  //     partial tiles written to global memory are visible to the cluster).
  // (3) all warps: each cluster rank owns rows_per = ceil(NR / ks) activation
  //     rows, sums them over the K splits in rank order (deterministic) and
  //     applies the Epi store for 4 adjacent weight rows per thread, as one
  //     16- or 8-byte vector where the layout allows.
  // Weight-row constants of the store (biases are model data: read before
  // the dependency wait)
  const int n0 = tile0 * 16 + 4 * lane;  // weight rows n0 .. n0+3
  const int nvalid = max(0, min(4, e.N - n0));
  float b4[4];
#pragma unroll
  for (int i = 0; i < 4; i++) b4[i] = i < nvalid ? tc_epi_bias(e, n0 + i) : 0.f;
  pdl_wait();  // (returned long ago for the activation loader)
  // the decode position of the KV-cache scatter, loaded long before the stores
  const int pos = e.mode == EPI_QKV ? *e.pos : 0;
  cg::cluster_group cluster = cg::this_cluster();
  const int crank = ks > 1 ? (int)cluster.block_rank() : 0;
  const int rows_per = (NR + ks - 1) / ks;
  // partial tiles of this cluster: [ks][NR][128] fp32
  float* part = ks > 1 ? e.split_ws + (size_t)(blockIdx.y * gridDim.x + blockIdx.x) * ks * NR * 128
                       : reinterpret_cast<float*>(sm);
  bool done_ok = true;
  if (warp < TC_DQ_WARPS) {
    done_ok = mbar_wait(DONE, 0, abort_flag, 6, errw, wait_ns);
    done_ok = __all_sync(0xffffffffu, done_ok);
  }
  if (warp < TC_DQ_WARPS && done_ok) {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const int f = (warp & 3) * 32 + lane;
    const int nchunk = NR / 16, qpart = (nchunk + 3) / 4, sub = warp >> 2;
    const int cbeg = min(nchunk, sub * qpart), cend = min(nchunk, cbeg + qpart);
    float* mine = part + (size_t)crank * NR * 128;
    for (int ci = cbeg; ci < cend; ci++) {
      const int c0 = ci * 16;
      uint32_t v[16];
      const uint32_t taddr = tmem + ((uint32_t)((warp & 3) * 32) << 16) + (uint32_t)c0;
      asm volatile(
          "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
          : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
            "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
          : "r"(taddr));
      asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
      for (int i = 0; i < 16; i++) mine[(size_t)(c0 + i) * 128 + f] = __uint_as_float(v[i]);
    }
  }
  if (ks > 1) cluster.sync();
  else __syncthreads();
  if (*abort_flag == 0) {
    const TcEpiRow er = tc_epi_row(e, n0, pos);
    const bool qkv_q = e.mode == EPI_QKV && n0 < e.d;
    // the 4 weight rows are adjacent in the output unless a head of a
    // cache layout ends inside the quad
    const bool contig = (e.mode != EPI_QKV && e.mode != EPI_CROSS_KV) || qkv_q || (e.hd & 3) == 0;
    const int64_t ustride = (int64_t)2 * e.H * e.T * e.hd;
    const int row_lo = crank * rows_per, nrows = min(rows_per, NR - row_lo);
    for (int jr = warp; jr < nrows; jr += TC_THREADS / 32) {
      const int r = r0 + row_lo + jr;
      if (r >= R) break;
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
      if (ks > 1) {
        // the ks (<= 8) partials of the row are loaded together, then
        // summed in rank order
        float4 p4[8];
#pragma unroll
        for (int k = 0; k < 8; k++)
          if (k < ks) p4[k] = __ldcg(reinterpret_cast<const float4*>(part + ((size_t)k * NR + row_lo + jr) * 128) + lane);
#pragma unroll
        for (int k = 0; k < 8; k++) {
          if (k < ks) {
            acc.x += p4[k].x;
            acc.y += p4[k].y;
            acc.z += p4[k].z;
            acc.w += p4[k].w;
          }
        }
      } else {
        acc = reinterpret_cast<const float4*>(part + (size_t)jr * 128)[lane];
      }
      const float a4[4] = {acc.x, acc.y, acc.z, acc.w};
      if (!contig) {
        for (int i = 0; i < nvalid; i++)
          tc_epi_store_run<1>(e, tc_epi_row(e, n0 + i, pos), e.mode == EPI_QKV && n0 + i < e.d, r, R, &a4[i]);
        continue;
      }
      float x[4];
#pragma unroll
      for (int i = 0; i < 4; i++) x[i] = __fadd_rn(a4[i], b4[i]);
      int64_t idx;
      if (e.mode == EPI_CROSS_KV) {
        const int u = r / e.T, tt = r - u * e.T;
        idx = er.col_off + (int64_t)u * ustride + (int64_t)tt * e.hd;
      } else {
        idx = (int64_t)r * er.row_stride + er.col_off;
      }
      tc_store_quad(e, qkv_q, idx, x, nvalid);
    }
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (*abort_flag) {
    // a wait expired: let the copies still in flight land (bounded) before
    // the CTA's shared memory is released; at most one per ring slot, the last
    // activation slot s: the phase of its last copy, p = kl / S, completes
    // once its 8 dequant arrivals and the bytes are in; arrivals the dequant
    // warps did not make (they stopped) are made here, no warp runs any more
    if (warp == TC_XLOAD_WARP && lane < S && issued_x[lane] >= 0) {
      const int p = issued_x[lane] / S;
      for (int i = dq_arrivals[lane] - 8 * p; i < 8; i++) mbar_arrive(FULL(lane));
      mbar_drain(FULL(lane), (uint32_t)p & 1u);
    }
    if (warp == TC_WLOAD_WARP && lane < TC_DQ_NS && issued_w[lane] >= 0)
      mbar_drain(RAW_FULL(lane), (uint32_t)(issued_w[lane] / TC_DQ_NS) & 1u);
  }
  if (warp == TC_MMA_WARP) {
    // after an abort nobody may have waited for DONE: the MMAs issued before
    // it (DONE tracks them all) must finish writing tensor memory before it
    // is released
    if (*abort_flag && lane == 0) mbar_drain(DONE, 0);
    __syncwarp();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(ncols) : "memory");
  }
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
  const int groups = (W.ntiles + 7) / 8, rtiles = (R + NR - 1) / NR, nk = W.cols / TC_BK;
  // split K over a cluster (<= 8 CTAs) when the output tiles cannot fill the GPU
  int ks = 1;
  if (groups * rtiles < 148) {
    ks = std::min(8, std::max(1, 148 / (groups * rtiles)));
    ks = std::min(ks, nk);
    const int per = (nk + ks - 1) / ks;
    ks = (nk + per - 1) / per;  // every split gets >= 1 stage
  }
  if (ks > 1) {
    // keep every cluster of the grid co-resident (one wave)
    static thread_local int cached_dev = -1, cached_nr = -1, cached_ks = -1, cached_max = 0;
    int dev = 0;
    cudaGetDevice(&dev);
    for (; ks > 1; ks--) {
      int per2 = (nk + ks - 1) / ks;
      if ((nk + per2 - 1) / per2 != ks) continue;
      int maxc = 0;
      if (dev == cached_dev && NR == cached_nr && ks == cached_ks) maxc = cached_max;
      else {
        cudaLaunchConfig_t qc = {};
        qc.gridDim = dim3(groups, rtiles, ks);
        qc.blockDim = dim3(TC_THREADS, 1, 1);
        qc.dynamicSmemBytes = L.total;
        cudaLaunchAttribute qa[1];
        qa[0].id = cudaLaunchAttributeClusterDimension;
        qa[0].val.clusterDim.x = 1;
        qa[0].val.clusterDim.y = 1;
        qa[0].val.clusterDim.z = ks;
        qc.attrs = qa;
        qc.numAttrs = 1;
        if (cudaOccupancyMaxActiveClusters(&maxc, gemm_tc_kernel<QT>, &qc) != cudaSuccess) {
          cudaGetLastError();
          maxc = 0;
        }
        cached_dev = dev; cached_nr = NR; cached_ks = ks; cached_max = maxc;
      }
      if (maxc >= groups * rtiles) break;
    }
  }
  if (ks > 1 && (!e.split_ws || (int64_t)groups * rtiles * ks * NR * 128 > e.split_ws_floats)) {
    set_error("tcgen05 GEMM: split-K workspace missing or too small (%lld floats needed)",
              (long long)groups * rtiles * ks * NR * 128);
    return WG_ERR_INVALID;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(groups, rtiles, ks);
  cfg.blockDim = dim3(TC_THREADS, 1, 1);
  cfg.dynamicSmemBytes = L.total;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 1;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = ks;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 2 : 1;
  Epi et = e;
  {  // failure-handling test hooks (unset in normal runs)
    const char* v = getenv("WG_TEST_WAIT_NS");
    et.test_wait_ns = (v && *v) ? strtoull(v, nullptr, 10) : 0;
    v = getenv("WG_TEST_TC_STALL");
    et.test_stall = (v && v[0] == '1') ? 1 : 0;
  }
  cudaError_t err = cudaLaunchKernelEx(&cfg, gemm_tc_kernel<QT>, W, map, R, NR, ks, et);
  if (err != cudaSuccess) {
    set_error("launch of gemm_tc failed: %s", cudaGetErrorString(err));
    return WG_ERR_CUDA;
  }
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
