// kernels.cuh — launch interfaces of the decoder kernels (one per reference
// function on the token loop) shared by the C-ABI driver.
#pragma once

#include "common.cuh"

namespace wg {

// ---- weights (weights.cu) ---------------------------------------------------
int upload_matrix(const wg_matrix* const* parts, int nparts, DMat* out, cudaStream_t st);
void free_dmat(DMat& m);
int dequant_dmat(const DMat& m, float* d_out, cudaStream_t st);
int64_t dmat_device_bytes(const DMat& m);

// ---- GEMV / GEMM epilogues (gemm.cu) --------------------------------------------
enum EpiMode {
  EPI_F32 = 0,       // out[r*ldo + n] = acc (+ bias[n])                   (cross q, logits)
  EPI_RESID = 1,     // out[r*ldo + n] += acc + bias[n]                    (residual adds, decoder.go:394-398)
  EPI_GELU_F16 = 2,  // out16[r*ldo + n] = half(GELU(acc + bias[n]))       (mlp.0, decoder.go:981-985)
  EPI_QKV = 3,       // n in [0,d): q; [d,2d): K -> cache slot pos; [2d,3d): V + bias -> cache
  EPI_CROSS_KV = 4   // rows r = u*T + t, cols n = (l*2 + kv)*d + j -> cross K/V cache (+ V bias)
};

struct Epi {
  int mode = EPI_F32;
  int R = 0, N = 0;            // valid activation rows / weight rows
  const float* bias = nullptr; // [N]
  float* out = nullptr;        // fp32 output (EPI_F32, EPI_RESID, q of EPI_QKV)
  __half* out16 = nullptr;     // EPI_GELU_F16
  int ldo = 0;
  // EPI_QKV / EPI_CROSS_KV
  int d = 0, H = 0, hd = 64, T = 0;  // T: positions per (row, head) slab (Tmax or T_enc)
  const int* pos = nullptr;          // device scalar: slot written by EPI_QKV
  __half* kv = nullptr;              // QKV: this layer's cache base; CROSS: whole cross cache
  const float* bias_q = nullptr;     // QKV q bias [d]
  const float* bias_v = nullptr;     // QKV v bias [d]; CROSS: [L][d]
  int U = 0;                         // CROSS: utterances
  // tcgen05 path with K split over a cluster: partial tiles of the splits,
  // device memory of at least TC_SPLIT_WS_FLOATS floats, owned by the stream
  // (no other launch may use it concurrently); contents need no initialisation
  float* split_ws = nullptr;
  int64_t split_ws_floats = 0;
  // tcgen05 path: the word an expired bounded wait records its code in
  // (device memory; nullptr: the tcgen05 kernels' shared word, tc_error_word)
  int* err_word = nullptr;
  // tcgen05 path, set by its launcher from the environment for the
  // failure-handling tests only: WG_TEST_WAIT_NS bounds every wait of the
  // kernel (0: the default 2 s); WG_TEST_TC_STALL=1 makes the activation
  // loader leave its first stage's copy out, so the MMA issuer's wait for it
  // can only expire (the flag that nothing sets) and the abort path runs.
  uint64_t test_wait_ns = 0;
  int test_stall = 0;
  // Small-batch path only (matmul_fuses_input_ln): the activations are
  // LayerNorm(ln_x) of ln_d-wide fp32 rows, normalised inside the GEMV with
  // the LayerNorm kernel's arithmetic (X is not read).
  const float* ln_x = nullptr;
  const float* ln_w = nullptr;
  const float* ln_b = nullptr;
  int ln_d = 0;
};

// Upper bound of the split-K workspace: at most one wave of 148 CTAs, each
// with a 128 x 256 fp32 partial tile (19.4 MB).
constexpr int64_t TC_SPLIT_WS_FLOATS = 148LL * 256 * 128;

// path: 0 auto, 1 small-R kernel (R <= 16: the bulk-copy GEMV where it
// applies, else the streaming one), 2 large-R mma.sync kernel, 3 tcgen05
// tensor-core kernel (quantised weights, K % 64 == 0), 4 streaming small-R
// kernel.
int init_gemm_attributes();
int init_tc_attributes();
bool tc_supported(const DMat& W);
int launch_matmul_tc(const DMat& W, const __half* X, int ldx, int R, const Epi& e, cudaStream_t st);
// First expired bounded wait of a tcgen05 kernel on the current device (0: none).
int tc_error_word(int* word, bool clear);
int launch_matmul(const DMat& W, const __half* X, int ldx, int R, const Epi& e, cudaStream_t st,
                  int path = 0);
// True when launch_matmul(path 0) of W x [R rows] honours Epi.ln_x, i.e. the
// LayerNorm before the matmul can be left to the GEMV (WG_LN_FUSE=0: never).
bool matmul_fuses_input_ln(const DMat& W, int R);
// small-batch GEMV with bulk-copied weight slices (gemv_bulk.cu), R <= 16
bool gemv_bulk_supported(const DMat& W, int R);
int launch_gemv_bulk(const DMat& W, const __half* X, int ldx, int R, const Epi& e, cudaStream_t st);
int init_gemv_bulk_attributes();
// First expired bounded wait of a gemv_bulk kernel on the current device (0: none).
int gemv_error_word(int* word, bool clear);

// ---- elementwise (eltwise.cu) -----------------------------------------------------
// x[r] = dequant(tok_emb row tok[r]) + pos_emb[pos]   (decoder.go:756-773, Q1 fix)
int launch_embed(const DMat& tok_emb, const float* pos_emb, const int* tokens, const int* pos,
                 int pos_offset, int R, int d, float* x, cudaStream_t st);
// out16[r] = half(LayerNorm(x[r]))  (ml/ops.go:153-202); optional fp32 copy
int launch_layernorm(const float* x, const float* w, const float* b, int R, int d, __half* out16,
                     float* out32, cudaStream_t st);
// True when launch_layernorm sums a row as per-lane float4 runs (the register
// kernel) rather than lane-strided scalars.
bool layernorm_uses_vec(int d);
int launch_f32_to_f16(const float* in, __half* out, int64_t n, cudaStream_t st);

// ---- attention (attn.cu) ------------------------------------------------------------
struct SelfAttnArgs {
  const float* q;          // [R][d] (unscaled, bias added)
  const __half* kv;        // this layer's cache base [Rphys][2][H][Tmax][hd]
  const int* tbl;          // [R][Tmax] physical row of each position (nullptr: own row)
  const int* pos;          // device scalar: current position
  int R, H, hd, Tmax;
  int ref_compat;          // 1: only slot 0 is visible (attention.go:250-256 with Tq=1)
  int zero_unless_pos0;    // 1: slot 0 is zero unless pos == 0 (beam reset, decoder.go:593)
  __half* out16;           // [R][d]
};
int launch_self_attn(const SelfAttnArgs& a, cudaStream_t st);

struct CrossAttnArgs {
  const float* q;          // [U*B][d]
  const __half* kv;        // this layer's cross cache [U][2][H][T][hd]
  int U, B, H, hd, T;
  __half* out16;           // [U*B][d]
};
int launch_cross_attn(const CrossAttnArgs& a, cudaStream_t st);
// First expired bounded wait of an attention kernel on the current device (0: none).
int attn_error_word(int* word, bool clear);
int init_attn_attributes();

// ---- the persistent token-step kernel (step.cu) --------------------------------------
// Layer weights and vectors as the step kernel reads them (device array, one per layer).
struct StepLayer {
  DMat w[6];  // q|k|v, self out, cross q, cross out, mlp.0, mlp.2
  const float *sln_w, *sln_b, *cln_w, *cln_b, *mln_w, *mln_b;
  const float *q_b, *v_b, *so_b, *cq_b, *co_b, *m0_b, *m2_b;
};
// One matmul of the step: 128-row groups, 64-wide K pairs, K splits, pairs per split.
struct MmPlan {
  int groups, pairs, ks, per;
};
struct StepArgs {
  const StepLayer* layers;
  int L, R, U, B, d, H, T, Tmax;
  MmPlan mm[6];
  int xchunks;                 // frame chunks per cross-attention head
  const int* pos;              // device scalar
  const int* tbl;              // [R][Tmax] physical row of each position (beams, CORRECT) or nullptr
  int ref_compat, zero_unless_pos0;
  float* x;                    // [R][d] residual stream (embedding already added)
  float* q;                    // [R][d] self-attention q, then cross-attention q
  float* att;                  // [R][d] self-attention output
  float* h;                    // [R][4d] GELU(mlp.0)
  __half* selfkv;              // [L][R][2][H][Tmax][64]
  const __half* cross;         // [L][U][2][H][T][64]
  float* part;                 // matmul partial tiles [group * ks + split][R][128]
  float* xpart;                // cross-attention partials [chunk][R][H][65] (o[64], l)
  float* xmax;                 // [chunk][R][H] per-chunk maxima
  unsigned* sync;              // [0] barrier, [1] unused, [2] abort, [4, 4 + max_groups) group counters,
                               // then [U * H] head counters; zero before every launch
  int max_groups;
  int* err;                    // the step kernel's error word (step_error_word)
};
// Whether the step kernel can run this model at R rows (weights of one
// quantised type, K % 64 == 0, head dim 64, R <= 16) and is switched on
// (WG_STEP_KERNEL=1; off by default: measured slower than the kernel chain).
bool step_supported(const DMat* const w0[6], int R, int hd, int d, int T, int Tmax);
// Scratch of a job using the step kernel: floats of part / xpart / xmax and
// unsigned of sync.
void step_scratch_sizes(const DMat* const w0[6], int R, int U, int H, int T, int64_t* part, int64_t* xpart,
                        int64_t* xmax, int64_t* sync);
// Plans (matmul splits, frame chunks) and the cooperative launch on st; the
// caller fills every other field of a.
int launch_step(StepArgs a, const DMat* const w0[6], cudaStream_t st);
int init_step_attributes();
int step_error_word(int* word, bool clear);
// Device address of the step kernel's error word (current device).
int step_error_ptr(int** p);

// ---- sampling (sample.cu) ----------------------------------------------------------
struct SampleState {
  int R, B, U;             // rows, beam width (1 = greedy), utterances
  int V, eot, Tcap;        // vocab, EOT id, token-history capacity per row
  int P, max_tokens;       // prompt length, token budget
  float inv_temp;          // 1/T (decoder.go:1001-1004)
  int suppress_nst;        // decoder.go:1016-1034
  float no_speech_thold;
  int suppress_eot;        // build switch: EOT never selected
  int correct_mode;        // 1: KV tables are reordered with the beams
  int Tmax;                // KV positions per row
  // device state
  float* logits;           // [R][V] (penalised in place)
  int* hist;               // [R][Tcap] token history (prompt included)
  int* hist_tmp;           // [R][Tcap]
  int* len;                // [R]
  float* score;            // [R] beam log-prob sums
  int* tok_in;             // [R] token fed to the next forward
  int* tbl;                // [R][Tmax] KV position -> physical row (CORRECT beams)
  int* tbl_tmp;
  int* utt_done;           // [U]
  int* utt_steps;          // [U] token steps executed
  int* n_done;             // device scalar: finished utterances
  int* pos;                // device scalar
  int* topk_tok;           // [R][5]
  float* topk_lp;          // [R][5]
  int* parent;             // [R]
  int* new_tok;            // [R]
  float* new_score;        // [R]
  int* new_len;            // [R]
  int* carried;            // [R]
  const int* forced;       // teacher forcing: [n][R] tokens or nullptr
  int* step;               // device scalar: steps taken
  // top-p fallback of greedy steps (decoder.go:1036-1056): enabled when
  // LogprobThold > 0, !NoFallback and the temperature is > 0; the greedy
  // kernels then leave their pick in new_tok and topp_kernel decides
  int topp;
  float logprob_thold;
  uint64_t seed;           // draws wg_uniform(seed, utt_id[u], utt_steps[u])
  const int* utt_id;       // [U] the job's utterance index of each local utterance
};
// One token step of sampling: penalty, greedy argmax or beam top-5 + merge,
// history/KV-table reorder, pos += 1.
int launch_sample_step(const SampleState& s, cudaStream_t st);
// Teacher forcing: append forced[step][r] to every row r, pos += 1.
int launch_forced_step(const SampleState& s, cudaStream_t st);
// pos += 1 (prompt prefill passes).
int launch_pos_inc(const SampleState& s, cudaStream_t st);
// Kernel-level test of the token selection (wg_sample_test).
int sample_test(const float* logits, int R, int V, const int32_t* hist, int n_hist, int eot,
                const wg_decode_params* p, int step, int32_t* out_tok, float* out_lp);
// Reset of the per-job state before a decode.
int launch_sample_reset(const SampleState& s, const int* prompt_dev, cudaStream_t st);

}  // namespace wg
