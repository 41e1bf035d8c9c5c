// sample.cu — on-device token selection of the decoder token loop.
//
//  penalty_row         applyRepetitionPenalty (internal/model/decoder.go:1140-1167),
//                      applied by greedy_kernel / topk_kernel to their row
//  greedy_kernel       sampleGreedyWithScratch (:996-1059) + the greedy loop's
//                      append / EOT / repeat-streak stops (:467-484)
//  topk_kernel         topKTokensWithScratch (:1068-1136), k = 5
//  beam_update_kernel  candidate scoring (:578-623), sortAndPruneBeams
//                      (:1462-1475), beam rebuild (:629-660), all-EOT and
//                      best-beam repeat stops (:662-691); the KV position
//                      table of every beam follows its parent (CORRECT mode)
#include <cooperative_groups.h>

#include <vector>

#include "kernels.cuh"

namespace wg {
namespace {

// ---- repetition penalty: logit[id] -= 2.0 * count(id in last 128 tokens) ----
// One row, by the whole CTA, at the start of the row's sampling kernel: the
// history window is staged in shared memory; the thread holding the first
// occurrence of an id applies its count (decoder.go:1140-1167), then EOT is
// masked when suppress_eot is set. Ends with a CTA barrier, so the row's
// logits are final for every thread afterwards.
constexpr int PEN_WIN = 128;
// ids outside [c0, c1) are left alone (a CTA that scans only that range of the row)
__device__ void penalty_range(const SampleState& s, int r, int c0, int c1) {
  __shared__ int hs[PEN_WIN];
  const int n = s.len[r];
  const int start = n > PEN_WIN ? n - PEN_WIN : 0, cnt = n - start;
  const int* h = s.hist + (int64_t)r * s.Tcap;
  for (int i = threadIdx.x; i < cnt; i += blockDim.x) hs[i] = h[start + i];
  __syncthreads();
  float* lg = s.logits + (int64_t)r * s.V;
  for (int i = threadIdx.x; i < cnt; i += blockDim.x) {
    const int id = hs[i];
    if (id < 0 || id >= s.V || id < c0 || id >= c1) continue;
    bool first = true;
    for (int j = 0; j < i && first; j++) first = hs[j] != id;
    if (!first) continue;
    int c = 0;
    for (int j = i; j < cnt; j++) c += hs[j] == id;
    lg[id] = __fsub_rn(lg[id], __fmul_rn(2.0f, (float)c));
  }
  __syncthreads();
  if (threadIdx.x == 0 && s.suppress_eot && s.eot >= 0 && s.eot < s.V && s.eot >= c0 && s.eot < c1)
    lg[s.eot] = -INFINITY;
  __syncthreads();
}
__device__ void penalty_row(const SampleState& s, int r) { penalty_range(s, r, 0, s.V); }

struct ArgMax {
  float v;
  int i;
};
__device__ __forceinline__ ArgMax better(ArgMax a, ArgMax b) {
  // larger value wins; on ties the lower index (the reference keeps the first maximum)
  if (b.v > a.v || (b.v == a.v && b.i >= 0 && (a.i < 0 || b.i < a.i))) return b;
  return a;
}
__device__ __forceinline__ ArgMax warp_argmax(ArgMax a) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    ArgMax b{__shfl_xor_sync(0xffffffffu, a.v, o), __shfl_xor_sync(0xffffffffu, a.i, o)};
    a = better(a, b);
  }
  return a;
}

// Logit rows are scanned with SCAN_UNROLL independent loads in flight per
// thread (a row is 51,866 floats; one load at a time made the scan latency-bound).
constexpr int SCAN_UNROLL = 8;

__device__ void greedy_finish(const SampleState& s, int r, int u, ArgMax all, ArgMax excl, const float* lg);
__device__ void greedy_commit(const SampleState& s, int r, int u, int tok);

// ---- greedy ----------------------------------------------------------------------
__global__ void __launch_bounds__(1024) greedy_kernel(SampleState s) {
  pdl_trigger();
  pdl_wait();
  const int r = blockIdx.x, u = r;  // B == 1
  if (s.utt_done[u]) return;
  penalty_row(s, r);
  const float* lg = s.logits + (int64_t)r * s.V;
  ArgMax all{-INFINITY, -1}, excl{-INFINITY, -1};
  // each thread visits i = tid, tid + blockDim, ... in increasing order; the
  // loads of SCAN_UNROLL visits are issued before any is used
  const int stride = blockDim.x;
  for (int i0 = threadIdx.x; i0 < s.V; i0 += SCAN_UNROLL * stride) {
    float x[SCAN_UNROLL];
#pragma unroll
    for (int k = 0; k < SCAN_UNROLL; k++) x[k] = i0 + k * stride < s.V ? lg[i0 + k * stride] : 0.f;
#pragma unroll
    for (int k = 0; k < SCAN_UNROLL; k++) {
      const int i = i0 + k * stride;
      if (i < s.V) {
        const float v = __fmul_rn(x[k], s.inv_temp);
        all = better(all, ArgMax{v, i});
        if (i != s.eot) excl = better(excl, ArgMax{v, i});
      }
    }
  }
  __shared__ ArgMax red[2][32];
  all = warp_argmax(all);
  excl = warp_argmax(excl);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) { red[0][warp] = all; red[1][warp] = excl; }
  __syncthreads();
  if (warp != 0) return;
  const int nw = blockDim.x >> 5;
  all = lane < nw ? red[0][lane] : ArgMax{-INFINITY, -1};
  excl = lane < nw ? red[1][lane] : ArgMax{-INFINITY, -1};
  all = warp_argmax(all);
  excl = warp_argmax(excl);
  if (lane != 0) return;
  greedy_finish(s, r, u, all, excl, lg);
}

// The chosen token of row r (all: arg-max of the row, excl: arg-max without
// EOT) -> SuppressNST re-pick, then (one thread) either the commit, or with
// the top-p fallback enabled the pick left for topp_kernel.
__device__ void greedy_finish(const SampleState& s, int r, int u, ArgMax all, ArgMax excl, const float* lg) {
  int tok = all.i < 0 ? 0 : all.i;
  if (s.suppress_nst && s.eot >= 0 && s.eot < s.V) {
    if (lg[s.eot] < -s.no_speech_thold && tok == s.eot) tok = excl.i < 0 ? s.eot : excl.i;
  }
  if (s.topp) s.new_tok[r] = tok;
  else greedy_commit(s, r, u, tok);
}

// History append, next input and the greedy loop's stop rules (decoder.go:467-484).
__device__ void greedy_commit(const SampleState& s, int r, int u, int tok) {
  int* h = s.hist + (int64_t)r * s.Tcap;
  int n = s.len[r];
  h[n] = tok;
  n++;
  s.len[r] = n;
  s.tok_in[r] = tok;
  s.utt_steps[u] += 1;
  bool done = tok == s.eot || n >= s.P + s.max_tokens;
  if (!done) {
    int streak = 0;  // trailing identical generated tokens (prevToken starts at -1)
    for (int i = n - 1; i >= s.P && h[i] == tok; i--) streak++;
    done = streak > 20;
  }
  if (done) {
    s.utt_done[u] = 1;
    atomicAdd(s.n_done, 1);
  }
}

// ---- top-p fallback of greedy steps --------------------------------------------------
// sampleGreedyWithScratch's fallback (decoder.go:1036-1056) and
// sampleTopPFromLogitsWithScratch (:1251-1378), one CTA per row:
//  (1) scaled = logit / T; logZ = log(sum exp(scaled - max)) + max (float32
//      sum of float64 exponentials); the greedy pick stands unless its
//      log-prob is below -LogprobThold;
//  (2) else p_i = exp(scaled_i - logZ) (float64 exponential rounded to
//      float32, as the reference), written over the row; the nucleus is the
//      shortest prefix of the row in descending p (lower index first among
//      equal p) whose mass reaches 0.9, cumSum its mass, and the token is the
//      first element of that order whose running mass reaches u01 * cumSum.
// Both cuts are found without sorting: a radix descent over the 32-bit
// patterns of p (non-negative floats order like their bits), 8 bits per pass,
// with per-digit counts and masses. Masses are fixed point in units of 2^-40
// (exact integer sums, so the result does not depend on summation order);
// the reference sums float32 in sorted order, which differs by rounding only.
constexpr int TOPP_THREADS = 1024;
constexpr double TOPP_ONE = 1099511627776.0;  // 2^40

__device__ __forceinline__ float uniform_dev(uint64_t seed, uint32_t u, uint32_t t) {
  // wg_uniform (include/wg_decoder.h): SplitMix64 output function, top 24 bits
  uint64_t z = seed ^ ((uint64_t)u + 1) * 0x9E3779B97F4A7C15ull ^ ((uint64_t)t + 1) * 0xD1B54A32D192ED03ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  z ^= z >> 31;
  return (float)(z >> 40) * (1.0f / 16777216.0f);
}
__device__ __forceinline__ unsigned long long topp_fixed(float p) { return __double2ull_rn((double)p * TOPP_ONE); }

struct ToppCut {
  uint32_t key;             // bit pattern of p at the cut
  unsigned long long above; // mass of the elements with larger p
  int j;                    // the cut is the j-th (1-based) element with that p, in index order
};

// Cut of row p (n floats >= 0) at cumulative mass `target` (<= the row's
// mass): the first element, in descending p / ascending index order, whose
// running mass reaches target. Every thread of the CTA calls it and gets it.
__device__ ToppCut topp_cut(const float* p, int n, unsigned long long target) {
  __shared__ unsigned int hc[256];
  __shared__ unsigned long long hs[256];
  __shared__ uint32_t prefix_sh, mask_sh;
  __shared__ unsigned long long above_sh;
  __shared__ int eq_sh;
  if (threadIdx.x == 0) { prefix_sh = 0; mask_sh = 0; above_sh = 0; eq_sh = 0; }
  for (int shift = 24; shift >= 0; shift -= 8) {
    for (int i = threadIdx.x; i < 256; i += blockDim.x) { hc[i] = 0; hs[i] = 0; }
    __syncthreads();
    const uint32_t prefix = prefix_sh, mask = mask_sh;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
      const float v = p[i];
      const uint32_t key = __float_as_uint(v);
      if ((key & mask) == prefix) {
        const int dg = (key >> shift) & 255;
        atomicAdd(&hc[dg], 1u);
        atomicAdd(&hs[dg], topp_fixed(v));
      }
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      unsigned long long above = above_sh;
      int sel = -1;
      for (int dg = 255; dg >= 0; dg--) {
        if (!hc[dg]) continue;
        if (above + hs[dg] >= target) { sel = dg; break; }
        above += hs[dg];
      }
      if (sel < 0)  // only by rounding of target: the cut is the row's last element
        for (int dg = 0; dg < 256; dg++)
          if (hc[dg]) { sel = dg; above -= hs[dg]; break; }
      above_sh = above;
      prefix_sh = prefix | ((uint32_t)sel << shift);
      mask_sh = mask | (255u << shift);
      eq_sh = (int)hc[sel];
    }
    __syncthreads();
  }
  ToppCut c;
  c.key = prefix_sh;
  c.above = above_sh;
  const unsigned long long q = topp_fixed(__uint_as_float(c.key));
  const unsigned long long need = target > c.above ? target - c.above : 0;
  long long j = q ? (long long)((need + q - 1) / q) : 1;
  if (j < 1) j = 1;
  if (j > eq_sh) j = eq_sh;
  c.j = (int)j;
  __syncthreads();
  return c;
}

// Index of the j-th (1-based) element of p whose bit pattern is key (index order).
__device__ int topp_nth(const float* p, int n, uint32_t key, int j) {
  __shared__ int cnt[TOPP_THREADS];
  __shared__ int found;
  const int chunk = (n + blockDim.x - 1) / blockDim.x;
  const int beg = threadIdx.x * chunk, end = min(n, beg + chunk);
  int c = 0;
  for (int i = beg; i < end; i++) c += __float_as_uint(p[i]) == key;
  cnt[threadIdx.x] = c;
  if (threadIdx.x == 0) found = -1;
  __syncthreads();
  if (threadIdx.x == 0) {  // exclusive scan (one thread: 1024 entries)
    int acc = 0;
    for (int t = 0; t < (int)blockDim.x; t++) { const int v = cnt[t]; cnt[t] = acc; acc += v; }
  }
  __syncthreads();
  const int before = cnt[threadIdx.x];
  if (c > 0 && before < j && j <= before + c) {
    int k = before;
    for (int i = beg; i < end; i++)
      if (__float_as_uint(p[i]) == key && ++k == j) { found = i; break; }
  }
  __syncthreads();
  return found;
}

__global__ void __launch_bounds__(TOPP_THREADS) topp_kernel(SampleState s) {
  pdl_trigger();
  pdl_wait();
  const int r = blockIdx.x, u = r;  // greedy: B == 1
  if (s.utt_done[u]) return;
  float* lg = s.logits + (int64_t)r * s.V;
  const int pick = s.new_tok[r];
  __shared__ float red[32];
  __shared__ unsigned long long redq[32];
  __shared__ int fb_sh, tok_sh;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  // (1) max and log Z of the scaled row
  float mx = -INFINITY;
  for (int i = threadIdx.x; i < s.V; i += blockDim.x) mx = fmaxf(mx, __fmul_rn(lg[i], s.inv_temp));
  mx = warp_max(mx);
  if (lane == 0) red[warp] = mx;
  __syncthreads();
  if (warp == 0) {
    float m = lane < nw ? red[lane] : -INFINITY;
    m = warp_max(m);
    if (lane == 0) red[0] = m;
  }
  __syncthreads();
  mx = red[0];
  __syncthreads();
  float es = 0.f;
  for (int i = threadIdx.x; i < s.V; i += blockDim.x)
    es += (float)exp((double)__fsub_rn(__fmul_rn(lg[i], s.inv_temp), mx));
  es = warp_sum(es);
  if (lane == 0) red[warp] = es;
  __syncthreads();
  if (threadIdx.x == 0) {
    float tot = 0.f;
    for (int w = 0; w < nw; w++) tot += red[w];
    const float logZ = __fadd_rn((float)log((double)tot), mx);
    red[0] = logZ;
    fb_sh = __fsub_rn(__fmul_rn(lg[pick], s.inv_temp), logZ) < -s.logprob_thold;
    tok_sh = pick;
  }
  __syncthreads();
  if (fb_sh) {
    const float logZ = red[0];
    // (2) probabilities over the row, and its fixed-point mass
    unsigned long long tq = 0;
    for (int i = threadIdx.x; i < s.V; i += blockDim.x) {
      const float p = (float)exp((double)__fsub_rn(__fmul_rn(lg[i], s.inv_temp), logZ));
      lg[i] = p;
      tq += topp_fixed(p);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) tq += __shfl_xor_sync(0xffffffffu, tq, o);
    if (lane == 0) redq[warp] = tq;
    __syncthreads();
    if (threadIdx.x == 0) {
      unsigned long long t = 0;
      for (int w = 0; w < nw; w++) t += redq[w];
      redq[0] = t;
    }
    __syncthreads();
    const unsigned long long total = redq[0];
    unsigned long long t1 = __double2ull_rn((double)0.9f * TOPP_ONE);  // topP = 0.9 (float32), :1037
    if (t1 > total) t1 = total;
    const ToppCut c1 = topp_cut(lg, s.V, t1);
    const unsigned long long cum = c1.above + (unsigned long long)c1.j * topp_fixed(__uint_as_float(c1.key));
    const float u01 = uniform_dev(s.seed, (uint32_t)s.utt_id[u], (uint32_t)s.utt_steps[u]);
    unsigned long long t2 = (unsigned long long)ceil((double)u01 * (double)cum);
    if (t2 > cum) t2 = cum;
    const ToppCut c2 = topp_cut(lg, s.V, t2);
    const int tok = topp_nth(lg, s.V, c2.key, c2.j);
    if (threadIdx.x == 0 && tok >= 0) tok_sh = tok;
    __syncthreads();
  }
  if (threadIdx.x == 0) greedy_commit(s, r, u, tok_sh);
}

// ---- beam: per-row top-5 of log_softmax(logits / T) ----------------------------
constexpr int TOPK = 5;
__device__ void topk_finish(const SampleState& s, int r, const float* lg, float (&fv)[TOPK], int (&fi)[TOPK],
                            float logZ);

__device__ __forceinline__ void top_insert(float (&v)[TOPK], int (&ix)[TOPK], float nv, int ni) {
  // keep v[0..4] sorted: larger first, lower index first on ties. The new
  // entry replaces the last one and bubbles up; every index is a constant,
  // so the list stays in registers.
  if (!(nv > v[TOPK - 1] || (nv == v[TOPK - 1] && ni < ix[TOPK - 1] && ix[TOPK - 1] >= 0))) return;
  v[TOPK - 1] = nv;
  ix[TOPK - 1] = ni;
#pragma unroll
  for (int j = TOPK - 1; j > 0; j--) {
    if (v[j] > v[j - 1] || (v[j] == v[j - 1] && ix[j] < ix[j - 1])) {
      const float tv = v[j];
      const int ti = ix[j];
      v[j] = v[j - 1];
      ix[j] = ix[j - 1];
      v[j - 1] = tv;
      ix[j - 1] = ti;
    }
  }
}
// Drops the head of a sorted list (the rest moves up one place).
__device__ __forceinline__ void top_pop(float (&v)[TOPK], int (&ix)[TOPK]) {
#pragma unroll
  for (int j = 0; j + 1 < TOPK; j++) {
    v[j] = v[j + 1];
    ix[j] = ix[j + 1];
  }
  v[TOPK - 1] = -INFINITY;
  ix[TOPK - 1] = -1;
}

constexpr int TOPK_THREADS = 512;  // one wave of rows (four CTAs per SM)
__global__ void __launch_bounds__(TOPK_THREADS) topk_kernel(SampleState s) {
  pdl_trigger();
  pdl_wait();
  const int r = blockIdx.x, u = r / s.B;
  if (s.utt_done[u]) return;
  const int n = s.len[r];
  const int* h = s.hist + (int64_t)r * s.Tcap;
  if (n > 0 && h[n - 1] == s.eot) return;  // finished hypothesis: carried forward unchanged
  penalty_row(s, r);
  const float* lg = s.logits + (int64_t)r * s.V;
  float tv[TOPK];
  int ti[TOPK];
#pragma unroll
  for (int j = 0; j < TOPK; j++) { tv[j] = -INFINITY; ti[j] = -1; }
  float mx = -INFINITY;
  const int stride = blockDim.x;
  for (int i0 = threadIdx.x; i0 < s.V; i0 += SCAN_UNROLL * stride) {
    float x[SCAN_UNROLL];
#pragma unroll
    for (int k = 0; k < SCAN_UNROLL; k++) x[k] = i0 + k * stride < s.V ? lg[i0 + k * stride] : 0.f;
#pragma unroll
    for (int k = 0; k < SCAN_UNROLL; k++) {
      const int i = i0 + k * stride;
      if (i < s.V) {
        const float v = __fmul_rn(x[k], s.inv_temp);
        mx = fmaxf(mx, v);
        top_insert(tv, ti, v, i);
      }
    }
  }
  __shared__ float cv[32 * TOPK];
  __shared__ int ci[32 * TOPK];
  __shared__ float wsum[32];
  __shared__ float smax;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  // warp merge: 5 rounds of arg-max over the lanes' list heads
  for (int k = 0; k < TOPK; k++) {
    const ArgMax a{tv[0], ti[0]};
    const ArgMax b = warp_argmax(a);
    if (a.i == b.i && b.i >= 0) top_pop(tv, ti);
    if (lane == 0) { cv[warp * TOPK + k] = b.v; ci[warp * TOPK + k] = b.i; }
  }
  float m = warp_max(mx);
  if (lane == 0) wsum[warp] = m;
  __syncthreads();
  if (warp == 0) {
    float mm = lane < nw ? wsum[lane] : -INFINITY;
    mm = warp_max(mm);
    if (lane == 0) smax = mm;
  }
  __syncthreads();
  mx = smax;
  // expSum = sum float32(exp(float64(s - max)))  (decoder.go:1121-1124); the
  // terms in float32 (expf, within 2 ulp of the rounded float64 value: the
  // reference's sequential float32 sum is reordered here anyway)
  float es = 0.f;
  for (int i0 = threadIdx.x; i0 < s.V; i0 += SCAN_UNROLL * stride) {
    float x[SCAN_UNROLL];
#pragma unroll
    for (int k = 0; k < SCAN_UNROLL; k++) x[k] = i0 + k * stride < s.V ? lg[i0 + k * stride] : 0.f;
#pragma unroll
    for (int k = 0; k < SCAN_UNROLL; k++)
      if (i0 + k * stride < s.V) es += expf(__fsub_rn(__fmul_rn(x[k], s.inv_temp), mx));
  }
  es = warp_sum(es);
  __syncthreads();
  if (lane == 0) wsum[warp] = es;
  __syncthreads();
  if (warp != 0) return;
  float tot = 0.f;
  if (lane == 0)
    for (int w = 0; w < nw; w++) tot += wsum[w];
  tot = __shfl_sync(0xffffffffu, tot, 0);
  const float logZ = __fadd_rn((float)log((double)tot), mx);
  // merge the warps' lists (nw * 5 candidates, 5 per lane)
  float lv[TOPK];
  int li[TOPK];
#pragma unroll
  for (int j = 0; j < TOPK; j++) {
    bool ok = lane < nw;
    lv[j] = ok ? cv[lane * TOPK + j] : -INFINITY;
    li[j] = ok ? ci[lane * TOPK + j] : -1;
  }
  float fv[TOPK];
  int fi[TOPK];
#pragma unroll
  for (int k = 0; k < TOPK; k++) {
    const ArgMax a{lv[0], li[0]};
    const ArgMax b = warp_argmax(a);
    if (a.i == b.i && b.i >= 0) top_pop(lv, li);
    fv[k] = b.v;
    fi[k] = b.i;
  }
  if (lane != 0) return;
  topk_finish(s, r, lg, fv, fi, logZ);
}

// Row r's top-5 (fv, fi: value order, lower index first on ties) and log Z ->
// topk_tok / topk_lp (one thread), with the exact-tie rerun of the reference scan.
__device__ void topk_finish(const SampleState& s, int r, const float* lg, float (&fv)[TOPK], int (&fi)[TOPK],
                            float logZ) {
  bool tie = false;
  for (int k = 0; k + 1 < TOPK; k++) tie |= fi[k + 1] >= 0 && fv[k] == fv[k + 1];
  if (tie) {
    // Equal values keep the slot order of the reference's replace-min scan
    // (decoder.go:1087-1119) through its sort (stable for 5 elements):
    // rerun that scan exactly. Only reached when top-5 values tie exactly.
    int n = 0, minPos = -1;
    float minVal = 0.f;
    for (int i = 0; i < s.V; i++) {
      float v = __fmul_rn(lg[i], s.inv_temp);
      if (n < TOPK) {
        fv[n] = v; fi[n] = i; n++;
        if (minPos < 0 || v < minVal) { minPos = n - 1; minVal = v; }
        continue;
      }
      if (v <= minVal) continue;
      fv[minPos] = v; fi[minPos] = i;
      minPos = 0; minVal = fv[0];
      for (int j = 1; j < n; j++) if (fv[j] < minVal) { minVal = fv[j]; minPos = j; }
    }
    for (int a = 1; a < n; a++) {  // stable insertion sort, descending
      float vv = fv[a]; int ii = fi[a]; int b = a - 1;
      while (b >= 0 && fv[b] < vv) { fv[b + 1] = fv[b]; fi[b + 1] = fi[b]; b--; }
      fv[b + 1] = vv; fi[b + 1] = ii;
    }
  }
  for (int k = 0; k < TOPK; k++) {
    s.topk_tok[r * TOPK + k] = fi[k];
    s.topk_lp[r * TOPK + k] = __fsub_rn(fv[k], logZ);
  }
}

// ---- small batches: each row split over a thread-block cluster --------------------
// With a few rows per step one CTA per row leaves the GPU idle (a row is
// V = 51,866 logits); SPLIT CTAs of a cluster each take a contiguous range of
// the row (penalty, scan), push their partial results into rank 0's shared
// memory (max also into every rank's), and rank 0 merges them in rank order,
// which gives the same candidates as one CTA scanning the whole row
// (first maximum / lower index first on ties). The log-sum-exp is summed per
// range against the row maximum and then in rank order.
constexpr int SPLIT = 8;
constexpr int SPLIT_THREADS = 256;

__device__ __forceinline__ void cluster_arrive_relaxed() {
  asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() { asm volatile("barrier.cluster.wait.aligned;" ::: "memory"); }
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.aligned;\nbarrier.cluster.wait.aligned;" ::: "memory");
}
// generic address of `p` (this CTA's shared memory) in cluster rank `rank`
template <typename T>
__device__ __forceinline__ T* cluster_peer(T* p, int rank) {
  return cooperative_groups::this_cluster().map_shared_rank(p, rank);
}
__device__ __forceinline__ int cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return (int)r;
}

// grid (SPLIT, R), cluster (SPLIT, 1, 1)
__global__ void __launch_bounds__(SPLIT_THREADS) greedy_split_kernel(SampleState s) {
  pdl_trigger();
  cluster_arrive_relaxed();  // peers may be written once every rank runs
  pdl_wait();
  const int r = blockIdx.y, u = r;  // B == 1
  const int rank = cluster_rank();
  const int chunk = (s.V + SPLIT - 1) / SPLIT, c0 = rank * chunk, c1 = min(s.V, c0 + chunk);
  __shared__ ArgMax part[2][SPLIT];  // rank 0: every rank's (all, excl)
  __shared__ ArgMax red[2][SPLIT_THREADS / 32];
  const bool live = s.utt_done[u] == 0;  // the same for every rank of the cluster
  ArgMax all{-INFINITY, -1}, excl{-INFINITY, -1};
  const float* lg = s.logits + (int64_t)r * s.V;
  if (live) {
    penalty_range(s, r, c0, c1);
    for (int i0 = c0 + threadIdx.x; i0 < c1; i0 += SCAN_UNROLL * SPLIT_THREADS) {
      float x[SCAN_UNROLL];
#pragma unroll
      for (int k = 0; k < SCAN_UNROLL; k++) x[k] = i0 + k * SPLIT_THREADS < c1 ? lg[i0 + k * SPLIT_THREADS] : 0.f;
#pragma unroll
      for (int k = 0; k < SCAN_UNROLL; k++) {
        const int i = i0 + k * SPLIT_THREADS;
        if (i < c1) {
          const float v = __fmul_rn(x[k], s.inv_temp);
          all = better(all, ArgMax{v, i});
          if (i != s.eot) excl = better(excl, ArgMax{v, i});
        }
      }
    }
    all = warp_argmax(all);
    excl = warp_argmax(excl);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) { red[0][warp] = all; red[1][warp] = excl; }
    __syncthreads();
    if (warp == 0) {
      all = lane < SPLIT_THREADS / 32 ? red[0][lane] : ArgMax{-INFINITY, -1};
      excl = lane < SPLIT_THREADS / 32 ? red[1][lane] : ArgMax{-INFINITY, -1};
      all = warp_argmax(all);
      excl = warp_argmax(excl);
    }
  }
  cluster_wait();
  if (live && threadIdx.x == 0) {
    ArgMax* dst = cluster_peer(&part[0][0], 0);
    dst[rank] = all;
    dst[SPLIT + rank] = excl;
  }
  cluster_sync_all();  // every range's result (and its penalised logits) is in place
  if (!live || rank != 0 || threadIdx.x != 0) return;
  ArgMax ga = part[0][0], ge = part[1][0];
  for (int k = 1; k < SPLIT; k++) {  // rank order = index order: the first maximum wins ties
    ga = better(ga, part[0][k]);
    ge = better(ge, part[1][k]);
  }
  greedy_finish(s, r, u, ga, ge, lg);
}

// grid (SPLIT, R), cluster (SPLIT, 1, 1)
__global__ void __launch_bounds__(SPLIT_THREADS) topk_split_kernel(SampleState s) {
  pdl_trigger();
  cluster_arrive_relaxed();
  pdl_wait();
  const int r = blockIdx.y, u = r / s.B;
  const int rank = cluster_rank();
  const int chunk = (s.V + SPLIT - 1) / SPLIT, c0 = rank * chunk, c1 = min(s.V, c0 + chunk);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = SPLIT_THREADS / 32;
  __shared__ float cand_v[SPLIT * TOPK];  // rank 0: every rank's top-5
  __shared__ int cand_i[SPLIT * TOPK];
  __shared__ float rmax[SPLIT], rsum[SPLIT];  // every rank: all maxima; rank 0: all sums
  __shared__ float cv[32 * TOPK];
  __shared__ int ci[32 * TOPK];
  __shared__ float wred[32];
  const int n = s.len[r];
  // the same for every rank of the cluster: finished utterance or hypothesis
  const bool live = s.utt_done[u] == 0 && !(n > 0 && s.hist[(int64_t)r * s.Tcap + n - 1] == s.eot);
  const float* lg = s.logits + (int64_t)r * s.V;
  float tv[TOPK];
  int ti[TOPK];
#pragma unroll
  for (int j = 0; j < TOPK; j++) { tv[j] = -INFINITY; ti[j] = -1; }
  float mx = -INFINITY;
  if (live) {
    penalty_range(s, r, c0, c1);
    for (int i0 = c0 + threadIdx.x; i0 < c1; i0 += SCAN_UNROLL * SPLIT_THREADS) {
      float x[SCAN_UNROLL];
#pragma unroll
      for (int k = 0; k < SCAN_UNROLL; k++) x[k] = i0 + k * SPLIT_THREADS < c1 ? lg[i0 + k * SPLIT_THREADS] : 0.f;
#pragma unroll
      for (int k = 0; k < SCAN_UNROLL; k++) {
        const int i = i0 + k * SPLIT_THREADS;
        if (i < c1) {
          const float v = __fmul_rn(x[k], s.inv_temp);
          mx = fmaxf(mx, v);
          top_insert(tv, ti, v, i);
        }
      }
    }
    // CTA top-5: warps, then warp 0 over the warps' lists
    for (int k = 0; k < TOPK; k++) {
      const ArgMax a{tv[0], ti[0]};
      const ArgMax b = warp_argmax(a);
      if (a.i == b.i && b.i >= 0) top_pop(tv, ti);
      if (lane == 0) { cv[warp * TOPK + k] = b.v; ci[warp * TOPK + k] = b.i; }
    }
    const float m = warp_max(mx);
    if (lane == 0) wred[warp] = m;
    __syncthreads();
    if (warp == 0) {
      float mm = lane < nw ? wred[lane] : -INFINITY;
      mx = warp_max(mm);
      float lv[TOPK];
      int li[TOPK];
#pragma unroll
      for (int j = 0; j < TOPK; j++) {
        const bool ok = lane < nw;
        lv[j] = ok ? cv[lane * TOPK + j] : -INFINITY;
        li[j] = ok ? ci[lane * TOPK + j] : -1;
      }
#pragma unroll
      for (int k = 0; k < TOPK; k++) {
        const ArgMax a{lv[0], li[0]};
        const ArgMax b = warp_argmax(a);
        if (a.i == b.i && b.i >= 0) top_pop(lv, li);
        tv[k] = b.v;
        ti[k] = b.i;
      }
    }
  }
  cluster_wait();
  if (live && threadIdx.x == 0) {
    float* cvd = cluster_peer(cand_v, 0);
    int* cid = cluster_peer(cand_i, 0);
    for (int k = 0; k < TOPK; k++) { cvd[rank * TOPK + k] = tv[k]; cid[rank * TOPK + k] = ti[k]; }
    for (int q = 0; q < SPLIT; q++) cluster_peer(rmax, q)[rank] = mx;
  }
  cluster_sync_all();  // every rank's maximum is in its own shared memory
  float es = 0.f;
  float gmax = -INFINITY;
  if (live) {
    for (int q = 0; q < SPLIT; q++) gmax = fmaxf(gmax, rmax[q]);
    // terms in float32 (expf, within 2 ulp of the rounded float64 value of
    // decoder.go:1121-1124); per range, then in rank order
    for (int i0 = c0 + threadIdx.x; i0 < c1; i0 += SCAN_UNROLL * SPLIT_THREADS) {
      float x[SCAN_UNROLL];
#pragma unroll
      for (int k = 0; k < SCAN_UNROLL; k++) x[k] = i0 + k * SPLIT_THREADS < c1 ? lg[i0 + k * SPLIT_THREADS] : 0.f;
#pragma unroll
      for (int k = 0; k < SCAN_UNROLL; k++)
        if (i0 + k * SPLIT_THREADS < c1) es += expf(__fsub_rn(__fmul_rn(x[k], s.inv_temp), gmax));
    }
    es = warp_sum(es);
    __syncthreads();
    if (lane == 0) wred[warp] = es;
    __syncthreads();
    if (threadIdx.x == 0) {
      float tot = 0.f;
      for (int w = 0; w < nw; w++) tot += wred[w];
      cluster_peer(rsum, 0)[rank] = tot;
    }
  }
  cluster_sync_all();
  if (!live || rank != 0 || threadIdx.x != 0) return;
  float tot = 0.f;
  for (int q = 0; q < SPLIT; q++) tot += rsum[q];
  const float logZ = __fadd_rn((float)log((double)tot), gmax);
  // merge the ranks' lists: repeatedly take the best head (value, then lower index)
  int head[SPLIT];
  for (int q = 0; q < SPLIT; q++) head[q] = 0;
  float fv[TOPK];
  int fi[TOPK];
  for (int k = 0; k < TOPK; k++) {
    int bq = -1;
    ArgMax b{-INFINITY, -1};
    for (int q = 0; q < SPLIT; q++) {
      if (head[q] >= TOPK) continue;
      const ArgMax c{cand_v[q * TOPK + head[q]], cand_i[q * TOPK + head[q]]};
      if (c.i < 0) continue;
      if (bq < 0 || c.v > b.v || (c.v == b.v && c.i < b.i)) { b = c; bq = q; }
    }
    if (bq >= 0) head[bq]++;
    fv[k] = b.v;
    fi[k] = b.i;
  }
  topk_finish(s, r, lg, fv, fi, logZ);
}

// ---- beam: candidates, prune, rebuild, stops (one CTA per utterance) -------------
constexpr int MAXB = 16;

__global__ void __launch_bounds__(128) beam_update_kernel(SampleState s) {
  pdl_trigger();
  pdl_wait();
  const int u = blockIdx.x;
  if (s.utt_done[u]) return;
  const int B = s.B;
  __shared__ float c_norm[MAXB * TOPK], c_score[MAXB * TOPK], c_lp[MAXB * TOPK];
  __shared__ int c_parent[MAXB * TOPK], c_tok[MAXB * TOPK];
  __shared__ int nc_sh;
  __shared__ int sel[MAXB];
  __shared__ int b_cnt[MAXB];
  // candidates of beam b (thread b, all beams at once) into slots
  // b*TOPK .. b*TOPK+TOPK-1, then compacted in beam order by one thread
  if (threadIdx.x < B) {
    const int b = threadIdx.x, r = u * B + b, base = b * TOPK;
    const int n = s.len[r];
    const int* h = s.hist + (int64_t)r * s.Tcap;
    const float sc = s.score[r];
    int k = 0;
    if (n > 0 && h[n - 1] == s.eot) {
      c_parent[base] = b; c_score[base] = sc; c_tok[base] = s.eot; c_lp[base] = 0.f;
      c_norm[base] = __fdiv_rn(sc, (float)pow((double)n, 0.6));
      k = 1;
    } else {
      const float den = (float)pow((double)(n + 1), 0.6);
      for (int jj = 0; jj < TOPK; jj++) {
        const int tk = s.topk_tok[r * TOPK + jj];
        if (tk < 0) continue;
        const float lp = s.topk_lp[r * TOPK + jj];
        const float ns = __fadd_rn(sc, lp);
        c_parent[base + k] = b; c_score[base + k] = ns; c_tok[base + k] = tk; c_lp[base + k] = lp;
        c_norm[base + k] = __fdiv_rn(ns, den);
        k++;
      }
    }
    b_cnt[b] = k;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    int nc = 0;  // in place: a candidate only moves to a lower slot
    for (int b = 0; b < B; b++)
      for (int k = 0; k < b_cnt[b]; k++, nc++) {
        const int src = b * TOPK + k;
        if (src == nc) continue;
        c_parent[nc] = c_parent[src]; c_score[nc] = c_score[src]; c_tok[nc] = c_tok[src];
        c_lp[nc] = c_lp[src]; c_norm[nc] = c_norm[src];
      }
    nc_sh = nc;
  }
  __syncthreads();
  const int nc = nc_sh;
  // stable rank by normScore (descending). A NaN score ranks as -inf, so the
  // ranks are a permutation of the candidates whatever the values (with NaN
  // left in, every NaN candidate would rank first and ranks would go unset).
  for (int i = threadIdx.x; i < nc; i += blockDim.x)
    if (c_norm[i] != c_norm[i]) c_norm[i] = -INFINITY;
  __syncthreads();
  for (int i = threadIdx.x; i < nc; i += blockDim.x) {
    int rank = 0;
    for (int j = 0; j < nc; j++) rank += (c_norm[j] > c_norm[i]) || (c_norm[j] == c_norm[i] && j < i);
    if (rank < B) sel[rank] = i;
  }
  __syncthreads();
  const int nb = nc < B ? nc : B;
  // rebuild: token histories (and KV tables) from the parents, via shared memory
  extern __shared__ int dyn[];
  int* th = dyn;                      // [B][Tcap]
  int* tt = dyn + B * s.Tcap;         // [B][Tmax]
  __shared__ int nlen[MAXB];
  const int pos = *s.pos;
  for (int b = 0; b < nb; b++) {
    int ci_ = sel[b];
    int pr = u * B + c_parent[ci_];
    int pl = s.len[pr];
    const int* ph = s.hist + (int64_t)pr * s.Tcap;
    for (int i = threadIdx.x; i < pl; i += blockDim.x) th[b * s.Tcap + i] = ph[i];
    if (s.correct_mode) {
      const int* pt = s.tbl + (int64_t)pr * s.Tmax;
      for (int i = threadIdx.x; i <= pos && i < s.Tmax; i += blockDim.x) tt[b * s.Tmax + i] = pt[i];
    }
    if (threadIdx.x == 0) {
      bool carried = pl > 0 && ph[pl - 1] == s.eot && c_tok[ci_] == s.eot && c_lp[ci_] == 0.f;
      if (carried) nlen[b] = pl;
      else { th[b * s.Tcap + pl] = c_tok[ci_]; nlen[b] = pl + 1; }
    }
  }
  __syncthreads();
  for (int b = 0; b < nb; b++) {
    int r = u * B + b;
    int* dh = s.hist + (int64_t)r * s.Tcap;
    for (int i = threadIdx.x; i < nlen[b]; i += blockDim.x) dh[i] = th[b * s.Tcap + i];
    if (s.correct_mode) {
      int* dt = s.tbl + (int64_t)r * s.Tmax;
      for (int i = threadIdx.x; i <= pos && i < s.Tmax; i += blockDim.x) dt[i] = tt[b * s.Tmax + i];
      if (threadIdx.x == 0 && pos + 1 < s.Tmax) dt[pos + 1] = r;  // the next step writes here
    }
    if (threadIdx.x == 0) {
      s.len[r] = nlen[b];
      s.score[r] = c_score[sel[b]];
      s.tok_in[r] = th[b * s.Tcap + nlen[b] - 1];
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    s.utt_steps[u] += 1;
    bool all_eot = true;  // decoder.go:662-672
    for (int b = 0; b < nb; b++) {
      int r = u * B + b;
      if (s.len[r] == 0 || s.hist[(int64_t)r * s.Tcap + s.len[r] - 1] != s.eot) { all_eot = false; break; }
    }
    bool stop = all_eot;
    if (!stop && nb > 0) {  // best beam repeats > 20 (decoder.go:675-691)
      int r = u * B;
      const int* h = s.hist + (int64_t)r * s.Tcap;
      int n = s.len[r];
      if (n >= 2) {
        int last = h[n - 1], streak = 1;
        for (int i = n - 2; i >= 0 && h[i] == last; i--) {
          streak++;
          if (streak > 20) { stop = true; break; }
        }
      }
    }
    if (s.utt_steps[u] >= s.max_tokens) stop = true;
    if (stop) {
      s.utt_done[u] = 1;
      atomicAdd(s.n_done, 1);
    }
  }
}

__global__ void pos_inc_kernel(int* pos, int* step) {
  pdl_trigger();
  pdl_wait();
  *pos += 1;
  if (step) *step += 1;
}

__global__ void forced_kernel(SampleState s) {
  pdl_trigger();
  pdl_wait();
  const int r = blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= s.R) return;
  const int tok = s.forced[(int64_t)(*s.step) * s.R + r];
  int n = s.len[r];
  if (n < s.Tcap) s.hist[(int64_t)r * s.Tcap + n] = tok;
  s.len[r] = n + 1;
  s.tok_in[r] = tok;
}

__global__ void reset_kernel(SampleState s, const int* __restrict__ prompt) {
  pdl_trigger();
  pdl_wait();
  const int r = blockIdx.x;
  int* h = s.hist + (int64_t)r * s.Tcap;
  for (int i = threadIdx.x; i < s.P; i += blockDim.x) h[i] = prompt[i];
  int* t = s.tbl + (int64_t)r * s.Tmax;
  for (int i = threadIdx.x; i < s.Tmax; i += blockDim.x) t[i] = r;
  if (threadIdx.x == 0) {
    s.len[r] = s.P;
    s.score[r] = 0.f;
    s.tok_in[r] = prompt[s.P - 1];
    if (r % s.B == 0) {
      s.utt_done[r / s.B] = 0;
      s.utt_steps[r / s.B] = 0;
    }
    if (r == 0) {
      *s.n_done = 0;
      *s.pos = s.correct_mode ? 0 : s.P - 1;
      *s.step = 0;
    }
  }
}

}  // namespace

// A launch of grid (SPLIT, R) in clusters of SPLIT CTAs (programmatic
// serialisation as launch_k).
cudaError_t launch_split(void (*kernel)(SampleState), int R, cudaStream_t st, const SampleState& s) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(SPLIT, R, 1);
  cfg.blockDim = dim3(SPLIT_THREADS, 1, 1);
  cfg.stream = st;
  cudaLaunchAttribute at[2];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = SPLIT;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  at[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = pdl_enabled() ? 2 : 1;
  return cudaLaunchKernelEx(&cfg, kernel, s);
}

// rows per step up to which a row is split over a cluster (WG_SAMPLE_SPLIT):
// measured faster at 1-40 rows (40 rows: +1.2 % per step), equal at 320
int sample_split_rows() {
  static int v = -1;
  if (v < 0) {
    const char* e = getenv("WG_SAMPLE_SPLIT");
    v = (e && *e) ? atoi(e) : 64;
  }
  return v;
}

int launch_sample_step(const SampleState& s, cudaStream_t st) {
  const bool split = s.R <= sample_split_rows();
  if (s.B <= 1) {
    if (split) WG_CHECK(launch_check(launch_split(greedy_split_kernel, s.R, st, s), "greedy_split"));
    else WG_CHECK(launch_check(launch_k(greedy_kernel, dim3(s.R), dim3(1024), 0, st, s), "greedy"));
    if (s.topp) WG_CHECK(launch_check(launch_k(topp_kernel, dim3(s.R), dim3(TOPP_THREADS), 0, st, s), "topp"));
  } else {
    if (split) WG_CHECK(launch_check(launch_split(topk_split_kernel, s.R, st, s), "topk_split"));
    else WG_CHECK(launch_check(launch_k(topk_kernel, dim3(s.R), dim3(TOPK_THREADS), 0, st, s), "topk"));
    size_t dyn = (size_t)s.B * (s.Tcap + s.Tmax) * sizeof(int);
    WG_CHECK(launch_check(launch_k(beam_update_kernel, dim3(s.U), dim3(128), dyn, st, s), "beam_update"));
  }
  return launch_check(launch_k(pos_inc_kernel, dim3(1), dim3(1), 0, st, s.pos, s.step), "pos_inc");
}

int launch_forced_step(const SampleState& s, cudaStream_t st) {
  WG_CHECK(launch_check(launch_k(forced_kernel, dim3((s.R + 127) / 128), dim3(128), 0, st, s), "forced"));
  return launch_check(launch_k(pos_inc_kernel, dim3(1), dim3(1), 0, st, s.pos, s.step), "pos_inc");
}

// Kernel-level sampling test (wg_sample_test): the token-selection kernels
// of one step on given logits, with each row its own utterance.
int sample_test(const float* logits, int R, int V, const int32_t* hist, int n_hist, int eot,
                const wg_decode_params* p, int step, int32_t* out_tok, float* out_lp) {
  const bool beam = p->beam_size > 1;
  const int Tcap = n_hist + 2;
  cudaStream_t st = nullptr;
  WG_CHECK_CUDA(cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking));
  float *d_lg = nullptr, *d_f = nullptr;
  int* d_i = nullptr;
  const size_t n_i = (size_t)R * Tcap + (size_t)R * 12 + 8;
  int rc = WG_OK;
  if (cudaMalloc(&d_lg, (size_t)R * V * 4) != cudaSuccess || cudaMalloc(&d_f, (size_t)R * 8 * 4) != cudaSuccess ||
      cudaMalloc(&d_i, n_i * 4) != cudaSuccess) {
    set_error("wg_sample_test: cudaMalloc failed");
    rc = WG_ERR_OOM;
  }
  SampleState s{};
  if (rc == WG_OK) {
    s.R = R; s.B = 1; s.U = R; s.V = V; s.eot = eot; s.Tcap = Tcap; s.P = n_hist; s.max_tokens = 1 << 20;
    s.Tmax = 1;
    const float base = p->temperature == 0.f ? 1.0f : p->temperature;
    const float temp = base + (float)p->attempt * 0.2f;
    s.inv_temp = temp > 0.f ? 1.0f / temp : 1.0f;
    s.suppress_nst = p->suppress_nst;
    s.no_speech_thold = p->no_speech_thold;
    s.suppress_eot = p->suppress_eot;
    s.topp = !beam && p->logprob_thold > 0.f && !p->no_fallback && temp > 0.f;
    s.logprob_thold = p->logprob_thold;
    s.seed = p->seed;
    int* ip = d_i;
    s.hist = ip; ip += (size_t)R * Tcap;
    s.len = ip; ip += R;
    s.tok_in = ip; ip += R;
    s.new_tok = ip; ip += R;
    s.utt_done = ip; ip += R;
    s.utt_steps = ip; ip += R;
    int* uid = ip; ip += R;
    s.utt_id = uid;
    s.topk_tok = ip; ip += (size_t)R * 5;
    s.n_done = ip; ip += 1;
    s.logits = d_lg;
    s.topk_lp = d_f;
    std::vector<int> h((size_t)R * Tcap, 0), ln(R, n_hist), z(R, 0), stp(R, step), ids(R);
    for (int r = 0; r < R; r++) {
      ids[r] = r;
      for (int i = 0; i < n_hist; i++) h[(size_t)r * Tcap + i] = hist[(size_t)r * n_hist + i];
    }
    if (cudaMemcpyAsync(d_lg, logits, (size_t)R * V * 4, cudaMemcpyHostToDevice, st) != cudaSuccess ||
        cudaMemcpyAsync(s.hist, h.data(), h.size() * 4, cudaMemcpyHostToDevice, st) != cudaSuccess ||
        cudaMemcpyAsync(s.len, ln.data(), (size_t)R * 4, cudaMemcpyHostToDevice, st) != cudaSuccess ||
        cudaMemcpyAsync(s.utt_done, z.data(), (size_t)R * 4, cudaMemcpyHostToDevice, st) != cudaSuccess ||
        cudaMemcpyAsync(s.utt_steps, stp.data(), (size_t)R * 4, cudaMemcpyHostToDevice, st) != cudaSuccess ||
        cudaMemcpyAsync(uid, ids.data(), (size_t)R * 4, cudaMemcpyHostToDevice, st) != cudaSuccess ||
        cudaMemsetAsync(s.n_done, 0, 4, st) != cudaSuccess) {
      set_error("wg_sample_test: copy failed");
      rc = WG_ERR_CUDA;
    }
  }
  if (rc == WG_OK) {
    const bool split = R <= sample_split_rows();
    if (!beam) {
      rc = split ? launch_check(launch_split(greedy_split_kernel, R, st, s), "greedy_split")
                 : launch_check(launch_k(greedy_kernel, dim3(R), dim3(1024), 0, st, s), "greedy");
      if (rc == WG_OK && s.topp) rc = launch_check(launch_k(topp_kernel, dim3(R), dim3(TOPP_THREADS), 0, st, s), "topp");
    } else {
      rc = split ? launch_check(launch_split(topk_split_kernel, R, st, s), "topk_split")
                 : launch_check(launch_k(topk_kernel, dim3(R), dim3(TOPK_THREADS), 0, st, s), "topk");
    }
  }
  if (rc == WG_OK) {
    cudaError_t e;
    if (!beam) {
      std::vector<int> h((size_t)R * Tcap);
      e = cudaMemcpyAsync(h.data(), s.hist, h.size() * 4, cudaMemcpyDeviceToHost, st);
      if (e == cudaSuccess) e = cudaStreamSynchronize(st);
      for (int r = 0; r < R && e == cudaSuccess; r++) out_tok[r] = h[(size_t)r * Tcap + n_hist];
    } else {
      e = cudaMemcpyAsync(out_tok, s.topk_tok, (size_t)R * 5 * 4, cudaMemcpyDeviceToHost, st);
      if (e == cudaSuccess && out_lp) e = cudaMemcpyAsync(out_lp, s.topk_lp, (size_t)R * 5 * 4, cudaMemcpyDeviceToHost, st);
      if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    }
    if (e != cudaSuccess) {
      set_error("wg_sample_test: %s", cudaGetErrorString(e));
      rc = WG_ERR_CUDA;
    }
  }
  cudaStreamSynchronize(st);
  cudaFree(d_lg); cudaFree(d_f); cudaFree(d_i);
  cudaStreamDestroy(st);
  return rc;
}

int launch_pos_inc(const SampleState& s, cudaStream_t st) {
  return launch_check(launch_k(pos_inc_kernel, dim3(1), dim3(1), 0, st, s.pos, (int*)nullptr), "pos_inc");
}

// Launched without programmatic serialisation: it starts only once every
// earlier kernel of the stream (the cross K/V precompute) has completed, and
// no later kernel can start before it, so the token loop's kernels may read
// the cross K/V cache before their dependency wait.
int launch_sample_reset(const SampleState& s, const int* prompt_dev, cudaStream_t st) {
  reset_kernel<<<s.R, 128, 0, st>>>(s, prompt_dev);
  return launch_status("sample_reset");
}

}  // namespace wg
