/*
 * wg_decoder.h — C ABI of the B200 (sm_100a) Whisper decoder token loop.
 *
 * This library replaces, below the Go interface
 *     model.Decoder.Decode(ctx, encoderOut ml.Tensor, params DecoderParams)
 *         (internal/model/interfaces.go:22-25)
 * the CPU implementation in internal/model/decoder.go (WhisperDecoder,
 * decoder.go:61-82) and the tensor ops it calls (internal/ml/matmul_q8.go,
 * attention.go, ops.go). A cgo package (go/internal/cuda in this
 * repository) binds these symbols behind model.Decoder.
 *
 * Conventions
 *  - Every function returns an int status (WG_OK == 0). No C++ exception
 *    crosses this boundary. wg_last_error() returns the text of the last
 *    error raised on the calling thread.
 *  - All pointers in descriptors are HOST pointers and are borrowed: the
 *    library copies what it needs before the call returns.
 *  - Matrices are passed exactly as gguf.FileLike.TensorRaw returns them
 *    (internal/gguf/gguf.go:228-246): raw little-endian GGUF block bytes,
 *    shape[0] = rows (output features), shape[1] = cols (input features).
 *  - A wg_job is not re-entrant; distinct jobs may run concurrently.
 */
#ifndef WG_DECODER_H
#define WG_DECODER_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ------------------------------------------------------ */
enum {
  WG_OK = 0,
  WG_ERR_INVALID = 1,     /* bad argument / shape (reference: ErrShapeMismatch, fmt.Errorf) */
  WG_ERR_CUDA = 2,        /* CUDA runtime error */
  WG_ERR_OOM = 3,         /* device allocation failed */
  WG_ERR_UNSUPPORTED = 4, /* feature of DecoderParams not implemented on the device */
  WG_ERR_CANCELLED = 5,   /* wg_job_cancel() was called (context.Canceled) */
  WG_ERR_TIMEOUT = 6,     /* host watchdog deadline passed */
  WG_ERR_INJECTED = 7,    /* host-side fault injection (WG_FAULT_INJECT) */
  WG_ERR_NO_DEVICE = 8,   /* no CUDA device / library built without one */
  WG_ERR_DEVICE_FLAG = 9  /* a kernel's bounded wait expired and set the error word */
};

/* ---- GGUF tensor types (internal/gguf/gguf.go dtype ids; ml/matmul_q8.go:15-32) */
enum {
  WG_QTYPE_F32 = 0,
  WG_QTYPE_F16 = 1,
  WG_QTYPE_Q4_0 = 2,
  WG_QTYPE_Q4_1 = 3,
  WG_QTYPE_Q5_0 = 6,
  WG_QTYPE_Q5_1 = 7,
  WG_QTYPE_Q8_0 = 8
};

/* ---- decode semantics -------------------------------------------------- */
enum {
  /* The reference's literal behaviour (internal/model/decoder.go):
   * forward() processes only the last token (decoder.go:750-757, no prompt
   * prefill), and the Tq=1 causal mask leaves only KV slot 0 visible
   * (ml/attention.go:250-256). Beam hypotheses reset their KV cache every
   * step (decoder.go:593, resetDecoderState :372-386). */
  WG_MODE_REF_COMPAT = 0,
  /* Standard Whisper decoding: the prompt is prefilled and self-attention
   * covers positions 0..pos; beam hypotheses keep their KV history. */
  WG_MODE_CORRECT = 1
};

/* One weight matrix, as TensorRaw returns it. */
typedef struct wg_matrix {
  uint32_t qtype;   /* WG_QTYPE_* */
  int32_t rows;     /* output features (TensorRaw shape[0]) */
  int32_t cols;     /* input features  (TensorRaw shape[1]) */
  const void* data; /* rows * row_bytes(qtype, cols) bytes */
} wg_matrix;

/* One decoder block (decoderBlock, decoder.go:43-58; loaded at :203-292). */
typedef struct wg_layer_desc {
  const float* self_ln_w;  const float* self_ln_b;      /* [d] */
  wg_matrix self_q;  const float* self_q_b;             /* [d,d], [d] */
  wg_matrix self_k;                                     /* [d,d] no bias */
  wg_matrix self_v;  const float* self_v_b;
  wg_matrix self_o;  const float* self_o_b;
  const float* cross_ln_w; const float* cross_ln_b;
  wg_matrix cross_q; const float* cross_q_b;
  wg_matrix cross_k;                                    /* no bias */
  wg_matrix cross_v; const float* cross_v_b;
  wg_matrix cross_o; const float* cross_o_b;
  const float* mlp_ln_w;   const float* mlp_ln_b;
  wg_matrix mlp0;    const float* mlp0_b;               /* [4d,d], [4d] */
  wg_matrix mlp2;    const float* mlp2_b;               /* [d,4d], [d] */
} wg_layer_desc;

/* Decoder hyper-parameters and weights (WhisperDecoder, decoder.go:61-82;
 * hyper-parameters from metadata keys read at decoder.go:101-105). */
typedef struct wg_model_desc {
  int32_t n_vocab;     /* whisper.vocab.size */
  int32_t n_state;     /* whisper.decoder.embedding_length (d) */
  int32_t n_head;      /* whisper.decoder.attention.head_count */
  int32_t n_layer;     /* whisper.decoder.layer_count */
  int32_t n_text_ctx;  /* whisper.decoder.context_length */
  int32_t eot;         /* end-of-text id; 50256 without a vocabulary (decoder.go:173) */
  wg_matrix token_embedding;          /* [n_vocab, d]; tied with the logits projection */
  const float* positional_embedding;  /* [n_text_ctx, d] fp32 */
  const float* ln_w;  const float* ln_b;  /* final LayerNorm [d] */
  const wg_layer_desc* layers;        /* n_layer entries */
} wg_model_desc;

/* The DecoderParams fields the reference decoder reads
 * (internal/model/interfaces.go:75-90), plus switches of this build. */
typedef struct wg_decode_params {
  int32_t beam_size;        /* <= 1: greedy (decoder.go:406) */
  float temperature;        /* 0 means 1.0 (decoder.go:416-419, :530-533) */
  int32_t attempt;          /* temperature-schedule attempt: T += 0.2*attempt (decoder.go:435,:537) */
  float logprob_thold;      /* > 0 with !no_fallback: greedy steps whose best log-prob is below
                               -logprob_thold draw from the top-p (0.9) nucleus instead
                               (decoder.go:1036-1056, sampler :1251-1378) */
  float no_speech_thold;    /* used by suppress_nst (decoder.go:1016-1034) */
  int32_t no_fallback;
  int32_t max_tokens;       /* <= 0: n_text_ctx; capped at n_text_ctx - P (decoder.go:421-430) */
  int32_t suppress_nst;
  int32_t mode;             /* WG_MODE_REF_COMPAT or WG_MODE_CORRECT */
  int32_t suppress_eot;     /* 1: EOT never selected (fixed-length benchmark runs); 0: reference */
  /* Seed of the top-p draws. The reference draws rand.Float32() from Go's
   * unseeded global source; here the draw of utterance u (its index in the
   * job) at its generated-token step t is wg_uniform(seed, u, t), so a
   * decode is reproducible and the CPU oracle makes the same draws. */
  uint64_t seed;
} wg_decode_params;

/* The top-p draw: SplitMix64's output function (Steele, Lea & Flood 2014) of
 * seed ^ (u + 1) * 0x9E3779B97F4A7C15 ^ (t + 1) * 0xD1B54A32D192ED03, its top
 * 24 bits scaled to [0, 1) (the 24-bit resolution of Go's Float32). */
static inline float wg_uniform(uint64_t seed, uint32_t u, uint32_t t) {
  uint64_t z = seed ^ ((uint64_t)u + 1) * 0x9E3779B97F4A7C15ull ^ ((uint64_t)t + 1) * 0xD1B54A32D192ED03ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  z ^= z >> 31;
  return (float)(z >> 40) * (1.0f / 16777216.0f);
}

typedef struct wg_model wg_model;
typedef struct wg_job wg_job;

/* ---- library / errors -------------------------------------------------- */
int wg_last_error(char* buf, size_t len);
int wg_device_count(int* n);
/* Number of our own kernels launched by this process so far (all devices). */
int wg_kernel_launch_count(int64_t* n);

/* ---- model ------------------------------------------------------------- */
/* Replaces model.NewDecoder (internal/model/decoder.go:97-303): uploads one
 * replica of the weights to each listed device (n_dev >= 1). */
int wg_model_create(const wg_model_desc* desc, const int* devices, int n_dev, wg_model** out);
/* Replaces gguf.Open + model.NewDecoder for a model file (internal/gguf/
 * gguf.go:52-134, internal/model/decoder.go:97-303): maps the GGUF v2/v3 file
 * read-only, resolves the decoder tensors under their whisper.cpp or
 * Hugging Face names (internal/model/compat.go:31-148), infers the
 * hyper-parameters the way NewDecoder does, and uploads the quantised blocks
 * from the mapping to each listed device (no host copy; F16 vectors and
 * transposed dense matrices are converted). EOT is 50256 until
 * wg_model_set_eot. Errors: WG_ERR_INVALID with the reference's
 * "gguf: ..." / "model: ..." texts. */
int wg_model_create_from_gguf(const char* path, const int* devices, int n_dev, wg_model** out);
int wg_model_destroy(wg_model* m);
/* Hyper-parameters of a created model (any pointer may be NULL). */
int wg_model_info(const wg_model* m, int* n_vocab, int* n_state, int* n_head, int* n_layer, int* n_text_ctx);
/* The vocabulary's end-of-text id (SetVocabulary, decoder.go:85-95); jobs
 * created afterwards stop on it. */
int wg_model_set_eot(wg_model* m, int eot);
/* Device bytes of one replica's weights (quant blocks as uploaded). */
int wg_model_weight_bytes(const wg_model* m, int64_t* bytes);

/* ---- decode jobs (replaces WhisperDecoder.Decode, decoder.go:401-410) --- */
/* Allocates device state for U utterances of T_enc encoder frames with a
 * prompt of P tokens shared by every utterance. Utterances are sharded
 * round-robin over the model's devices. */
int wg_job_create(wg_model* m, int U, int T_enc, const int32_t* prompt, int P,
                  const wg_decode_params* params, wg_job** out);
/* Host -> device copy of U encoder outputs, each [T_enc, d] fp32 row-major
 * (enc[u] points at utterance u). */
int wg_job_upload_encoder(wg_job* j, const float* const* enc);
/* Host -> device copy of utterance u's encoder output only (for callers,
 * like cgo, that may pass one buffer per call but no array of pointers to
 * their own memory); returns once the copy is done. */
int wg_job_upload_encoder_one(wg_job* j, int u, const float* enc);
/* Device of utterance u (the device whose memory wg_job_upload_encoder_device
 * expects its encoder output in). */
int wg_job_utterance_device(const wg_job* j, int u, int* device);
/* Encoder -> decoder hand-off on the device (the encoder output that
 * internal/model/encoder.go:265-332 returns, left on the GPU by a GPU
 * encoder): enc[u] is DEVICE memory [T_enc, d] fp32 on utterance u's device.
 * The job's stream first waits for everything enqueued so far on `stream`
 * (a cudaStream_t of the encoder; NULL: the legacy default stream is
 * synchronised), then copies device to device; the call returns without
 * waiting for the copies, and the encoder buffers must stay valid until
 * wg_job_start returns. Replaces wg_job_upload_encoder for that case. */
int wg_job_upload_encoder_device(wg_job* j, const float* const* enc, void* stream);
/* Cross K/V precompute for every layer, prompt prefill (CORRECT mode) and
 * reset of the beam / token state. Must follow an upload. */
int wg_job_start(wg_job* j);
/* Runs up to max_steps token steps on all devices (CUDA-graph replays).
 * *done = 1 when every utterance has finished. Returns WG_ERR_CANCELLED if
 * wg_job_cancel was called before or during the call. */
int wg_job_step(wg_job* j, int max_steps, int* done);
/* tokens: U x (P + max_tokens) int32 (prompt included, like the reference's
 * final token slice), lens: U, scores: U (beam log-prob sum; 0 for greedy). */
int wg_job_result(wg_job* j, int32_t* tokens, int32_t* lens, float* scores);
/* Every hypothesis of every utterance as it stands after the steps run so
 * far (the beams slice of decodeBeamSearch, decoder.go:545-552 and :629-660,
 * in its order: beams[0] is the best). tokens: U x B x (P + max_tokens),
 * lens and scores: U x B (B = 1 for greedy). */
int wg_job_beams(wg_job* j, int32_t* tokens, int32_t* lens, float* scores);
int wg_job_cancel(wg_job* j);
/* Device timer on the job's own stream(s): which = 0 records the start
 * event, which = 1 records the stop event, waits, and returns in *ms the
 * elapsed device time (max over the job's devices). */
int wg_job_timer(wg_job* j, int which, double* ms);
int wg_job_destroy(wg_job* j);
/* Token steps executed so far (max over utterances) and rows per step. */
int wg_job_stats(const wg_job* j, int* steps_done, int* rows, int* max_tokens);
/* 1 when the job's layers run as the persistent step kernel (<= 16 rows). */
int wg_job_uses_step_kernel(const wg_job* j, int* on);

/* One call = the whole Decode for U utterances: create, upload, start,
 * step to completion, result, destroy. */
int wg_decode(wg_model* m, const float* const* enc, int U, int T_enc,
              const int32_t* prompt, int P, const wg_decode_params* params,
              int32_t* tokens, int32_t* lens, float* scores);

/* Teacher-forced logits for U utterances (one row each): step s processes
 * the last token of prompt+forced[u][0..s) exactly as decodeGreedy's forward
 * calls do (decoder.go:441-447) and writes logits[(s*U + u)*n_vocab ...]
 * (before the repetition penalty). forced: U x n_forced. mode: WG_MODE_*. */
int wg_teacher_forced_logits(wg_model* m, const float* const* enc, int U, int T_enc,
                             const int32_t* prompt, int P,
                             const int32_t* forced, int n_forced, int mode,
                             float* logits);

/* ---- pipeline batching (internal/model/pipeline.go:90-193) --------------
 * The reference decodes one 30-s chunk per Decode call: the chunks of a file
 * in turn, and every concurrent Transcribe (whisper.go:24) on its own
 * goroutine. A batcher gathers such single-utterance calls into shared jobs:
 * requests that arrive within window_us of the oldest waiting one and have
 * the same prompt, encoder length and parameters are decoded together, up to
 * max_utterances per job (more rows per token step for the same weight
 * stream). One worker thread per batcher; wg_batcher_decode blocks the
 * calling thread until its utterance is decoded and is safe to call from
 * many threads at once. */
typedef struct wg_batcher wg_batcher;
int wg_batcher_create(wg_model* m, int max_utterances, int window_us, wg_batcher** out);
/* One utterance: enc is HOST [T_enc, d] fp32 and must stay valid until the
 * call returns; cancel (may be NULL) is polled between token steps, and a
 * job stops early once every one of its requests is cancelled
 * (WG_ERR_CANCELLED). tokens receives prompt + generated tokens (at most
 * tokens_cap), *len their count, *score the beam score (0 for greedy). */
int wg_batcher_decode(wg_batcher* b, const float* enc, int T_enc, const int32_t* prompt, int P,
                      const wg_decode_params* params, const volatile int* cancel, int32_t* tokens, int tokens_cap,
                      int32_t* len, float* score);
/* Jobs run and utterances decoded so far. */
int wg_batcher_stats(const wg_batcher* b, int64_t* jobs, int64_t* utterances);
/* Decodes what is queued, then stops the worker. */
int wg_batcher_destroy(wg_batcher* b);

/* ---- unit entry points (kernel-level parity) ---------------------------- */
/* Device dequantisation of raw GGUF blocks through the device weight layout
 * (gguf/dequant.go:92-201). out: n fp32 values. Bit-exact with the reference. */
int wg_dequant_test(uint32_t qtype, const void* raw, int64_t n, float* out);
/* out[m, rows] = x[m, cols] * dequant(W[rows, cols])^T with the device GEMV
 * (path 0: auto, 1: small-batch mma.sync GEMV, 2: mma.sync tiles,
 * 3: tcgen05 tensor-core kernel). x is rounded to f16 on the device first.
 * Replaces ml.MatMulQuantTransBInto (ml/matmul_q8.go:93-119). */
int wg_matmul_test(uint32_t qtype, const void* raw, int rows, int cols,
                   const float* x, int m, float* out, int path);

/* The token-selection kernels of one step on given logits (kernel-level
 * parity): R rows of V fp32 logits, each row an utterance whose history is
 * hist[r][0..n_hist) (prompt included; the repetition penalty reads it,
 * decoder.go:1140-1167). Greedy (params->beam_size <= 1): out_tok[r] =
 * sampleGreedyWithScratch's token (decoder.go:996-1059) with the top-p
 * fallback when params enable it, drawing wg_uniform(seed, r, step).
 * Beam: out_tok[r*5 + k], out_lp[r*5 + k] = topKTokensWithScratch's five
 * (decoder.go:1068-1136). */
int wg_sample_test(const float* logits, int R, int V, const int32_t* hist, int n_hist, int eot,
                   const wg_decode_params* params, int step, int32_t* out_tok, float* out_lp);

/* ---- allocation-free matmul (no reference counterpart) --------------------
 * For callers that may not allocate device memory once they are running
 * (their own pool owns the device, or an allocation would stall a
 * latency-critical path): out[r][n] = sum_k W[n][k] * x16[r][k] for one
 * uploaded weight matrix of replica `replica` of m, on the tcgen05 tensor-core
 * kernel, enqueued on `stream` (a cudaStream_t; NULL is the default stream).
 * No bias is added. This call allocates no device memory: when the kernel
 * splits K over a cluster, its partial tiles go to a fixed scratch array that
 * is part of the library's device image (WG_NOALLOC_SCRATCH_FLOATS floats,
 * 8 MiB, per device); a shape that needs more is rejected with
 * WG_ERR_INVALID and the error text gives the floats it needs. Nothing in
 * the scratch has to start at zero.
 *   which : 0 self-attention q|k|v (N = 3d, K = d), 1 self-attention out,
 *           2 cross-attention q, 3 cross-attention out (N = K = d),
 *           4 mlp.0 (N = 4d, K = d), 5 mlp.2 (N = d, K = 4d)
 *   x16   : device f16 [rows][ldx], 16-byte aligned, ldx % 8 == 0, ldx >= K
 *   out   : device fp32 [rows][ldo], ldo >= N
 *   wait  : nonzero: wait for the stream and report a CUDA error or an
 *           expired device-side wait (WG_ERR_DEVICE_FLAG) before returning;
 *           zero: return once the kernel is enqueued (an expired wait is
 *           then reported by the next call on the device with wait != 0:
 *           these calls keep their own error word, apart from decode jobs).
 * The first call on a device also does set-up (it looks up the scratch
 * array's device address with that device current), so make it before any
 * stream capture begins; the set-up is repeated only if the device's CUDA
 * context was destroyed and created again. All calls on one device share
 * the scratch: calls
 * whose kernels can overlap in time (different streams or host threads)
 * race and give wrong results; issue them in one stream or one at a time.
 * The caller's current device is restored before returning. */
#define WG_NOALLOC_SCRATCH_FLOATS (2LL * 1024 * 1024)
int wg_model_matmul_noalloc(wg_model* m, int replica, int layer, int which,
                            const void* x16, int ldx, int rows, float* out, int ldo,
                            void* stream, int wait);

/* ---- measurement hooks used by bench.py ---------------------------------- */
enum {
  WG_KCLASS_GEMV = 0,        /* the 6 weight matmuls of every layer */
  WG_KCLASS_SELF_ATTN = 1,
  WG_KCLASS_CROSS_ATTN = 2,
  WG_KCLASS_LOGITS = 3,
  WG_KCLASS_PRECOMPUTE = 4,  /* cross K/V projection of all layers (once per decode) */
  WG_KCLASS_STEP = 5,        /* the persistent kernel of all layers (jobs of <= 16 rows) */
  WG_KCLASS_MATMUL0 = 10     /* + k: only matmul k of {qkv, self out, cross q, cross out, mlp0, mlp2} */
};
/* Re-launches one kernel class over all layers of one step on the job's own
 * stream (device 0), iters times, between two CUDA events; *ms = mean time
 * of one launch, *bytes = algorithmic bytes of one launch. Call after
 * wg_job_start. */
int wg_job_time_kernel(wg_job* j, int kclass, int iters, double* ms, double* bytes);

#ifdef __cplusplus
}
#endif
#endif /* WG_DECODER_H */
