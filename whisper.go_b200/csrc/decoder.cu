// decoder.cu — model / job management and the C ABI (include/wg_decoder.h).
//
// The host side replaces WhisperDecoder (internal/model/decoder.go:61-82):
//   wg_model_create   NewDecoder (:97-303): one weight replica per device
//   wg_job_*          Decode (:401-410) for U utterances at once; the greedy
//                     (:413-525) and beam (:528-726) loops run on the device,
//                     one CUDA-graph replay per token step
//   forward_step      forward (:745-833) for every row of the job
#include <cuda.h>

#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdarg>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

#include "kernels.cuh"

namespace wg {

std::atomic<int64_t> g_launches{0};

bool pdl_enabled() {
  static const bool on = [] {
    const char* v = getenv("WG_PDL");
    return !(v && v[0] == '0');
  }();
  return on;
}
static thread_local std::string t_error;

void set_error(const char* fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  t_error = buf;
}
const char* last_error() { return t_error.c_str(); }

int init_attn_attributes();
int init_gemm_attributes();

namespace {

inline int round8(int x) { return (x + 7) / 8 * 8; }

struct DevLayer {
  const float *sln_w, *sln_b, *cln_w, *cln_b, *mln_w, *mln_b;
  DMat qkv, so, cq, co, m0, m2;
  const float *q_b, *v_b, *so_b, *cq_b, *co_b, *m0_b, *m2_b;
};

struct DevModel {
  int dev = 0;
  cudaStream_t st = nullptr;
  DMat tok;
  DMat cross_kv;  // all layers' cross K and V weights: [(l*2 + kv)*d + j][d]
  std::vector<DevLayer> layers;
  float* vec = nullptr;  // all fp32 vectors (LN, biases, positional embedding)
  const float *pos_emb = nullptr, *ln_w = nullptr, *ln_b = nullptr, *cross_vb = nullptr;
  int64_t weight_bytes = 0;
  StepLayer* step_layers = nullptr;  // device copy of every layer's weights and vectors (step kernel)
};

}  // namespace
}  // namespace wg

struct wg_model {
  int d = 0, H = 0, hd = 0, L = 0, V = 0, ctx = 0, eot = 0;
  std::vector<wg::DevModel*> devs;
};

namespace wg {
namespace {

struct DevJob {
  DevModel* dm = nullptr;
  int dev = 0;
  cudaStream_t st = nullptr;
  int U = 0, B = 1, R = 0, T = 0, P = 0, Tmax = 0, Tcap = 0, max_tokens = 0;
  int ldd = 0, ld4 = 0;
  std::vector<int> utt;  // global utterance ids
  float* enc32 = nullptr;
  __half* enc16 = nullptr;
  __half* cross = nullptr;
  __half* selfkv = nullptr;
  float *x = nullptr, *q = nullptr, *logits = nullptr;
  __half *xln16 = nullptr, *attn16 = nullptr, *h16 = nullptr;
  int* ptok = nullptr;  // [P][R] prompt tokens for the prefill passes
  int* prompt_dev = nullptr;
  int* forced_dev = nullptr;
  int* ints = nullptr;
  float* floats = nullptr;
  float* split_ws = nullptr;  // tcgen05 split-K partial tiles (TC_SPLIT_WS_FLOATS)
  // persistent step kernel (R <= 16): fp32 attention / MLP activations and scratch
  bool use_step = false;
  float *st_att = nullptr, *st_h = nullptr, *st_part = nullptr, *st_xpart = nullptr, *st_xmax = nullptr;
  unsigned* st_sync = nullptr;
  int* st_err = nullptr;
  SampleState ss{};
  int* host_done = nullptr;  // pinned
  cudaGraphExec_t graph = nullptr;
  int64_t graph_kernels = 0;
  bool started = false;
  cudaEvent_t ev[2] = {nullptr, nullptr};
};

// An epilogue descriptor carrying the job's split-K workspace.
inline Epi job_epi(const DevJob& j) {
  Epi e;
  e.split_ws = j.split_ws;
  e.split_ws_floats = TC_SPLIT_WS_FLOATS;
  return e;
}

}  // namespace
}  // namespace wg

struct wg_job {
  wg_model* m = nullptr;
  std::vector<wg::DevJob*> dj;
  int U = 0, B = 1, T = 0, P = 0, max_tokens = 0, mode = 0;
  std::vector<int32_t> prompt;
  wg_decode_params params{};
  int steps_done = 0;
  bool all_done = false;
  std::atomic<int> cancel{0};
  int fault_step = -1, fault_device = -1;
};

namespace wg {
namespace {

int64_t env_i64(const char* name, int64_t dflt) {
  const char* v = getenv(name);
  if (!v || !*v) return dflt;
  return strtoll(v, nullptr, 10);
}

// WG_STEP_KERNEL=1 runs the layers of small-batch jobs as the persistent
// step kernel (step.cu); read at job creation and at every forward pass.
bool env_step_enabled() {
  const char* v = getenv("WG_STEP_KERNEL");
  return v && v[0] == '1';
}

// Waits for a stream with the host watchdog deadline (WG_TIMEOUT_MS).
// Error words of the kernels with bounded waits (current device): a wait
// that expired means a copy or a peer never arrived; the step's results are
// not trusted.
static int check_wait_flags() {
  int w = 0;
  WG_CHECK(tc_error_word(&w, true));
  if (w) {
    set_error("a tcgen05 kernel's bounded wait expired (code 0x%x)", w);
    return WG_ERR_DEVICE_FLAG;
  }
  WG_CHECK(attn_error_word(&w, true));
  if (w) {
    set_error("an attention kernel's bounded wait expired (code 0x%x)", w);
    return WG_ERR_DEVICE_FLAG;
  }
  WG_CHECK(gemv_error_word(&w, true));
  if (w) {
    set_error("a GEMV kernel's bounded wait expired (code 0x%x)", w);
    return WG_ERR_DEVICE_FLAG;
  }
  WG_CHECK(step_error_word(&w, true));
  if (w) {
    set_error("the step kernel's bounded wait expired (code 0x%x)", w);
    return WG_ERR_DEVICE_FLAG;
  }
  return WG_OK;
}

int wait_stream(cudaStream_t st) {
  const int64_t limit_ms = env_i64("WG_TIMEOUT_MS", 600000);
  auto t0 = std::chrono::steady_clock::now();
  for (;;) {
    cudaError_t e = cudaStreamQuery(st);
    if (e == cudaSuccess) return WG_OK;
    if (e != cudaErrorNotReady) {
      set_error("device error: %s", cudaGetErrorString(e));
      return WG_ERR_CUDA;
    }
    auto el = std::chrono::duration_cast<std::chrono::milliseconds>(std::chrono::steady_clock::now() - t0).count();
    if (el > limit_ms) {
      set_error("watchdog: device work did not finish within %lld ms", (long long)limit_ms);
      return WG_ERR_TIMEOUT;
    }
    std::this_thread::sleep_for(std::chrono::microseconds(50));
  }
}

bool mat_ok(const wg_matrix& m, int rows, int cols) { return m.data && m.rows == rows && m.cols == cols; }

void free_devmodel(DevModel* d) {
  if (!d) return;
  cudaSetDevice(d->dev);
  free_dmat(d->tok);
  free_dmat(d->cross_kv);
  for (auto& l : d->layers) {
    free_dmat(l.qkv); free_dmat(l.so); free_dmat(l.cq); free_dmat(l.co); free_dmat(l.m0); free_dmat(l.m2);
  }
  cudaFree(d->vec);
  cudaFree(d->step_layers);
  if (d->st) cudaStreamDestroy(d->st);
  delete d;
}

int build_devmodel(const wg_model_desc* md, int dev, DevModel** out) {
  WG_CHECK_CUDA(cudaSetDevice(dev));
  DevModel* dm = new DevModel();
  dm->dev = dev;
  int rc = WG_OK;
  auto fail = [&](int r) { free_devmodel(dm); return r; };
  if (cudaStreamCreateWithFlags(&dm->st, cudaStreamNonBlocking) != cudaSuccess) return fail(WG_ERR_CUDA);
  if ((rc = init_gemm_attributes()) != WG_OK) return fail(rc);
  if ((rc = init_attn_attributes()) != WG_OK) return fail(rc);
  if ((rc = init_tc_attributes()) != WG_OK) return fail(rc);
  if ((rc = init_gemv_bulk_attributes()) != WG_OK) return fail(rc);
  if ((rc = init_step_attributes()) != WG_OK) return fail(rc);
  const int d = md->n_state, L = md->n_layer, ctx = md->n_text_ctx;
  // fp32 vectors: 6 LN + 7 biases (d or 4d) per layer, final LN, pos emb, cross V bias
  std::vector<float> host;
  std::vector<std::pair<const float**, size_t>> fix;
  auto put = [&](const float* src, size_t n, const float** dst) {
    size_t off = host.size();
    host.insert(host.end(), src, src + n);
    host.resize((host.size() + 3) / 4 * 4, 0.f);  // 16-byte aligned slices
    fix.push_back({dst, off});
  };
  dm->layers.resize(L);
  put(md->positional_embedding, (size_t)ctx * d, &dm->pos_emb);
  put(md->ln_w, d, &dm->ln_w);
  put(md->ln_b, d, &dm->ln_b);
  size_t cvb_off = host.size();
  for (int l = 0; l < L; l++) {
    host.insert(host.end(), md->layers[l].cross_v_b, md->layers[l].cross_v_b + d);
  }
  host.resize((host.size() + 3) / 4 * 4, 0.f);
  fix.push_back({&dm->cross_vb, cvb_off});
  for (int l = 0; l < L; l++) {
    const wg_layer_desc& s = md->layers[l];
    DevLayer& o = dm->layers[l];
    put(s.self_ln_w, d, &o.sln_w); put(s.self_ln_b, d, &o.sln_b);
    put(s.cross_ln_w, d, &o.cln_w); put(s.cross_ln_b, d, &o.cln_b);
    put(s.mlp_ln_w, d, &o.mln_w); put(s.mlp_ln_b, d, &o.mln_b);
    put(s.self_q_b, d, &o.q_b); put(s.self_v_b, d, &o.v_b); put(s.self_o_b, d, &o.so_b);
    put(s.cross_q_b, d, &o.cq_b); put(s.cross_o_b, d, &o.co_b);
    put(s.mlp0_b, (size_t)4 * d, &o.m0_b); put(s.mlp2_b, d, &o.m2_b);
  }
  if (cudaMalloc(&dm->vec, host.size() * 4) != cudaSuccess) { set_error("cudaMalloc(vectors) failed"); return fail(WG_ERR_OOM); }
  if (cudaMemcpy(dm->vec, host.data(), host.size() * 4, cudaMemcpyHostToDevice) != cudaSuccess) return fail(WG_ERR_CUDA);
  for (auto& f : fix) *f.first = dm->vec + f.second;
  // matrices
  {
    const wg_matrix* p[1] = {&md->token_embedding};
    if ((rc = upload_matrix(p, 1, &dm->tok, dm->st)) != WG_OK) return fail(rc);
  }
  std::vector<const wg_matrix*> ckv;
  for (int l = 0; l < L; l++) {
    const wg_layer_desc& s = md->layers[l];
    DevLayer& o = dm->layers[l];
    const wg_matrix* qkv[3] = {&s.self_q, &s.self_k, &s.self_v};
    if ((rc = upload_matrix(qkv, 3, &o.qkv, dm->st)) != WG_OK) return fail(rc);
    const wg_matrix* one[1];
    one[0] = &s.self_o; if ((rc = upload_matrix(one, 1, &o.so, dm->st)) != WG_OK) return fail(rc);
    one[0] = &s.cross_q; if ((rc = upload_matrix(one, 1, &o.cq, dm->st)) != WG_OK) return fail(rc);
    one[0] = &s.cross_o; if ((rc = upload_matrix(one, 1, &o.co, dm->st)) != WG_OK) return fail(rc);
    one[0] = &s.mlp0; if ((rc = upload_matrix(one, 1, &o.m0, dm->st)) != WG_OK) return fail(rc);
    one[0] = &s.mlp2; if ((rc = upload_matrix(one, 1, &o.m2, dm->st)) != WG_OK) return fail(rc);
    ckv.push_back(&s.cross_k);
    ckv.push_back(&s.cross_v);
  }
  if ((rc = upload_matrix(ckv.data(), (int)ckv.size(), &dm->cross_kv, dm->st)) != WG_OK) return fail(rc);
  {  // the layers as the step kernel reads them
    std::vector<StepLayer> sl(L);
    for (int l = 0; l < L; l++) {
      const DevLayer& o = dm->layers[l];
      StepLayer& t = sl[l];
      t.w[0] = o.qkv; t.w[1] = o.so; t.w[2] = o.cq; t.w[3] = o.co; t.w[4] = o.m0; t.w[5] = o.m2;
      t.sln_w = o.sln_w; t.sln_b = o.sln_b; t.cln_w = o.cln_w; t.cln_b = o.cln_b; t.mln_w = o.mln_w; t.mln_b = o.mln_b;
      t.q_b = o.q_b; t.v_b = o.v_b; t.so_b = o.so_b; t.cq_b = o.cq_b; t.co_b = o.co_b; t.m0_b = o.m0_b; t.m2_b = o.m2_b;
    }
    if (cudaMalloc(&dm->step_layers, sl.size() * sizeof(StepLayer)) != cudaSuccess ||
        cudaMemcpy(dm->step_layers, sl.data(), sl.size() * sizeof(StepLayer), cudaMemcpyHostToDevice) != cudaSuccess) {
      set_error("model upload: step layer table failed");
      return fail(WG_ERR_OOM);
    }
  }
  int64_t wb = dmat_device_bytes(dm->tok) + dmat_device_bytes(dm->cross_kv);
  for (auto& l : dm->layers)
    wb += dmat_device_bytes(l.qkv) + dmat_device_bytes(l.so) + dmat_device_bytes(l.cq) + dmat_device_bytes(l.co) +
          dmat_device_bytes(l.m0) + dmat_device_bytes(l.m2);
  dm->weight_bytes = wb;
  *out = dm;
  return WG_OK;
}

// The persistent step kernel over all layers of a job's rows (step.cu).
int launch_step_job(wg_model* m, DevJob& j, int mode) {
  DevModel& dm = *j.dm;
  const DevLayer& l0 = dm.layers[0];
  const DMat* w0[6] = {&l0.qkv, &l0.so, &l0.cq, &l0.co, &l0.m0, &l0.m2};
  StepArgs a{};
  a.layers = dm.step_layers;
  a.L = m->L; a.R = j.R; a.U = j.U; a.B = j.B; a.d = m->d; a.H = m->H; a.T = j.T; a.Tmax = j.Tmax;
  a.pos = j.ss.pos;
  const bool ref = mode == WG_MODE_REF_COMPAT;
  a.tbl = (!ref && j.B > 1) ? j.ss.tbl : nullptr;
  a.ref_compat = ref;
  a.zero_unless_pos0 = ref && j.B > 1;
  a.x = j.x; a.q = j.q; a.att = j.st_att; a.h = j.st_h;
  a.selfkv = j.selfkv; a.cross = j.cross;
  a.part = j.st_part; a.xpart = j.st_xpart; a.xmax = j.st_xmax; a.sync = j.st_sync; a.err = j.st_err;
  return launch_step(a, w0, j.st);
}

// ---- one forward pass over all rows of a device job (decoder.go:745-833) ----
int forward_step(wg_model* m, DevJob& j, const int* tokens, bool want_logits, int mode) {
  DevModel& dm = *j.dm;
  cudaStream_t st = j.st;
  const int d = m->d, H = m->H, hd = m->hd, R = j.R;
  WG_CHECK(launch_embed(dm.tok, dm.pos_emb, tokens, j.ss.pos, 0, R, d, j.x, st));
  if (j.use_step && env_step_enabled()) {
    // every layer in one persistent kernel (small batches)
    WG_CHECK(launch_step_job(m, j, mode));
    if (!want_logits) return WG_OK;
    Epi e = job_epi(j);
    if (matmul_fuses_input_ln(dm.tok, R)) {
      e.ln_x = j.x; e.ln_w = dm.ln_w; e.ln_b = dm.ln_b; e.ln_d = d;
    } else {
      WG_CHECK(launch_layernorm(j.x, dm.ln_w, dm.ln_b, R, d, j.xln16, nullptr, st));
    }
    e.mode = EPI_F32; e.out = j.logits; e.ldo = m->V; e.N = m->V;
    return launch_matmul(dm.tok, j.xln16, j.ldd, R, e, st);
  }
  const int64_t layer_kv = (int64_t)R * 2 * H * j.Tmax * hd;
  const int64_t layer_cross = (int64_t)j.U * 2 * H * j.T * hd;
  const bool ref = mode == WG_MODE_REF_COMPAT;
  // LayerNorm of x feeding matmul W: left to the small-batch GEMV where it
  // can take it (no separate kernel), else a LayerNorm kernel into xln16
  auto norm_for = [&](const DMat& W, const float* w, const float* b, Epi& e) -> int {
    if (matmul_fuses_input_ln(W, R)) {
      e.ln_x = j.x;
      e.ln_w = w;
      e.ln_b = b;
      e.ln_d = d;
      return WG_OK;
    }
    return launch_layernorm(j.x, w, b, R, d, j.xln16, nullptr, st);
  };
  for (int l = 0; l < m->L; l++) {
    const DevLayer& ly = dm.layers[l];
    __half* kv = j.selfkv + l * layer_kv;
    NvtxRange layer_range("decoder layer");
    // self-attention (decoder.go:836-908)
    Epi e = job_epi(j);
    WG_CHECK(norm_for(ly.qkv, ly.sln_w, ly.sln_b, e));
    e.mode = EPI_QKV; e.out = j.q; e.ldo = d; e.d = d; e.H = H; e.hd = hd; e.T = j.Tmax; e.pos = j.ss.pos;
    e.kv = kv; e.bias_q = ly.q_b; e.bias_v = ly.v_b; e.N = 3 * d;
    WG_CHECK(launch_matmul(ly.qkv, j.xln16, j.ldd, R, e, st));
    SelfAttnArgs sa{};
    sa.q = j.q; sa.kv = kv; sa.tbl = (!ref && j.B > 1) ? j.ss.tbl : nullptr; sa.pos = j.ss.pos;
    sa.R = R; sa.H = H; sa.hd = hd; sa.Tmax = j.Tmax; sa.ref_compat = ref; sa.zero_unless_pos0 = ref && j.B > 1;
    sa.out16 = j.attn16;
    WG_CHECK(launch_self_attn(sa, st));
    e = job_epi(j); e.mode = EPI_RESID; e.out = j.x; e.ldo = d; e.bias = ly.so_b; e.N = d;
    WG_CHECK(launch_matmul(ly.so, j.attn16, j.ldd, R, e, st));
    // cross-attention (decoder.go:911-971)
    e = job_epi(j);
    WG_CHECK(norm_for(ly.cq, ly.cln_w, ly.cln_b, e));
    e.mode = EPI_F32; e.out = j.q; e.ldo = d; e.bias = ly.cq_b; e.N = d;
    WG_CHECK(launch_matmul(ly.cq, j.xln16, j.ldd, R, e, st));
    CrossAttnArgs ca{};
    ca.q = j.q; ca.kv = j.cross + l * layer_cross; ca.U = j.U; ca.B = j.B; ca.H = H; ca.hd = hd; ca.T = j.T;
    ca.out16 = j.attn16;
    WG_CHECK(launch_cross_attn(ca, st));
    e = job_epi(j); e.mode = EPI_RESID; e.out = j.x; e.ldo = d; e.bias = ly.co_b; e.N = d;
    WG_CHECK(launch_matmul(ly.co, j.attn16, j.ldd, R, e, st));
    // MLP (decoder.go:974-993)
    e = job_epi(j);
    WG_CHECK(norm_for(ly.m0, ly.mln_w, ly.mln_b, e));
    e.mode = EPI_GELU_F16; e.out16 = j.h16; e.ldo = j.ld4; e.bias = ly.m0_b; e.N = 4 * d;
    WG_CHECK(launch_matmul(ly.m0, j.xln16, j.ldd, R, e, st));
    e = job_epi(j); e.mode = EPI_RESID; e.out = j.x; e.ldo = d; e.bias = ly.m2_b; e.N = d;
    WG_CHECK(launch_matmul(ly.m2, j.h16, j.ld4, R, e, st));
  }
  if (!want_logits) return WG_OK;
  NvtxRange logits_range("final LayerNorm + logits");
  Epi e = job_epi(j);
  WG_CHECK(norm_for(dm.tok, dm.ln_w, dm.ln_b, e));  // decoder.go:818
  e.mode = EPI_F32; e.out = j.logits; e.ldo = m->V; e.N = m->V;
  return launch_matmul(dm.tok, j.xln16, j.ldd, R, e, st);  // decoder.go:823 (tied embedding)
}

__global__ void zero_slot0_kernel(__half* kv, int64_t nslabs, int Tmax, int hd) {
  int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= nslabs * hd) return;
  int64_t s = i / hd;
  kv[s * Tmax * hd + (i % hd)] = __float2half_rn(0.f);
}

void free_devjob(DevJob* j) {
  if (!j) return;
  cudaSetDevice(j->dev);
  if (j->graph) cudaGraphExecDestroy(j->graph);
  cudaFree(j->enc32); cudaFree(j->enc16); cudaFree(j->cross); cudaFree(j->selfkv);
  cudaFree(j->x); cudaFree(j->q); cudaFree(j->logits); cudaFree(j->xln16); cudaFree(j->attn16); cudaFree(j->h16);
  cudaFree(j->ptok); cudaFree(j->prompt_dev); cudaFree(j->forced_dev); cudaFree(j->ints); cudaFree(j->floats);
  cudaFree(j->split_ws);
  cudaFree(j->st_att); cudaFree(j->st_h); cudaFree(j->st_part); cudaFree(j->st_xpart); cudaFree(j->st_xmax);
  cudaFree(j->st_sync);
  if (j->host_done) cudaFreeHost(j->host_done);
  for (auto& e : j->ev)
    if (e) cudaEventDestroy(e);
  if (j->st) cudaStreamDestroy(j->st);
  delete j;
}

template <typename T>
int dalloc(T** p, size_t n) {
  cudaError_t e = cudaMalloc(reinterpret_cast<void**>(p), std::max<size_t>(n, 1) * sizeof(T));
  if (e != cudaSuccess) {
    set_error("cudaMalloc(%zu bytes): %s", n * sizeof(T), cudaGetErrorString(e));
    return WG_ERR_OOM;
  }
  return WG_OK;
}

int build_devjob(wg_job* J, DevModel* dm, const std::vector<int>& utt, DevJob** out) {
  wg_model* m = J->m;
  WG_CHECK_CUDA(cudaSetDevice(dm->dev));
  DevJob* j = new DevJob();
  j->dm = dm;
  j->dev = dm->dev;
  j->utt = utt;
  j->U = (int)utt.size();
  j->B = J->B;
  j->R = j->U * j->B;
  j->T = J->T;
  j->P = J->P;
  j->max_tokens = J->max_tokens;
  j->Tmax = std::min(m->ctx, J->P + J->max_tokens);
  if (j->Tmax < 1) j->Tmax = 1;
  j->Tcap = J->P + J->max_tokens + 1;
  j->ldd = round8(m->d);
  j->ld4 = round8(4 * m->d);
  int rc = WG_OK;
  auto fail = [&](int r) { free_devjob(j); return r; };
  if (cudaStreamCreateWithFlags(&j->st, cudaStreamNonBlocking) != cudaSuccess) return fail(WG_ERR_CUDA);
  const int d = m->d, H = m->H, hd = m->hd, L = m->L, R = j->R, U = j->U, T = j->T;
  if ((rc = dalloc(&j->enc32, (size_t)U * T * d)) ||
      (rc = dalloc(&j->enc16, (size_t)U * T * j->ldd)) ||
      (rc = dalloc(&j->cross, (size_t)L * U * 2 * H * T * hd)) ||
      (rc = dalloc(&j->selfkv, (size_t)L * R * 2 * H * j->Tmax * hd)) ||
      (rc = dalloc(&j->x, (size_t)R * d)) || (rc = dalloc(&j->q, (size_t)R * d)) ||
      (rc = dalloc(&j->logits, (size_t)R * m->V)) ||
      (rc = dalloc(&j->xln16, (size_t)R * j->ldd)) || (rc = dalloc(&j->attn16, (size_t)R * j->ldd)) ||
      (rc = dalloc(&j->h16, (size_t)R * j->ld4)) ||
      (rc = dalloc(&j->ptok, (size_t)std::max(1, J->P) * R)) || (rc = dalloc(&j->prompt_dev, (size_t)J->P)) ||
      (rc = dalloc(&j->forced_dev, (size_t)(m->ctx + 1) * R)))
    return fail(rc);
  // zero activations once (padding columns stay zero)
  cudaMemsetAsync(j->xln16, 0, (size_t)R * j->ldd * 2, j->st);
  cudaMemsetAsync(j->attn16, 0, (size_t)R * j->ldd * 2, j->st);
  cudaMemsetAsync(j->h16, 0, (size_t)R * j->ld4 * 2, j->st);
  if (j->ldd != d) cudaMemsetAsync(j->enc16, 0, (size_t)U * T * j->ldd * 2, j->st);
  // integer / float state
  const size_t n_ints = (size_t)R * j->Tcap * 2 + (size_t)R * j->Tmax * 2 + (size_t)R * 16 + (size_t)U * 3 + 8;
  const size_t n_floats = (size_t)R * 8;
  if ((rc = dalloc(&j->ints, n_ints)) || (rc = dalloc(&j->floats, n_floats)) ||
      (rc = dalloc(&j->split_ws, (size_t)TC_SPLIT_WS_FLOATS)))
    return fail(rc);
  {
    const DevLayer& l0 = dm->layers[0];
    const DMat* w0[6] = {&l0.qkv, &l0.so, &l0.cq, &l0.co, &l0.m0, &l0.m2};
    if (step_supported(w0, R, hd, d, T, j->Tmax)) {
      int64_t np = 0, nx = 0, nm = 0, ns = 0;
      step_scratch_sizes(w0, R, U, H, T, &np, &nx, &nm, &ns);
      if ((rc = dalloc(&j->st_att, (size_t)R * d)) || (rc = dalloc(&j->st_h, (size_t)R * 4 * d)) ||
          (rc = dalloc(&j->st_part, (size_t)np)) || (rc = dalloc(&j->st_xpart, (size_t)nx)) ||
          (rc = dalloc(&j->st_xmax, (size_t)nm)) || (rc = dalloc(&j->st_sync, (size_t)ns)) ||
          (rc = step_error_ptr(&j->st_err)))
        return fail(rc);
      j->use_step = true;
    }
  }
  int* ip = j->ints;
  auto take = [&](size_t n) {
    int* p = ip;
    ip += n;
    return p;
  };
  SampleState& s = j->ss;
  s.R = R; s.B = j->B; s.U = U; s.V = m->V; s.eot = m->eot; s.Tcap = j->Tcap; s.P = J->P;
  s.max_tokens = J->max_tokens; s.Tmax = j->Tmax;
  {
    const wg_decode_params& p = J->params;
    float base = p.temperature == 0.f ? 1.0f : p.temperature;  // decoder.go:416-419
    float temp = base + (float)p.attempt * 0.2f;               // :435, :537
    s.inv_temp = temp > 0.f ? 1.0f / temp : 1.0f;               // :1001-1004
    s.suppress_nst = p.suppress_nst;
    s.no_speech_thold = p.no_speech_thold;
    s.suppress_eot = p.suppress_eot;
    // top-p fallback of greedy steps (decoder.go:1036-1037): LogprobThold > 0,
    // !NoFallback, temperature > 0; beam search never falls back
    s.topp = j->B <= 1 && p.logprob_thold > 0.f && !p.no_fallback && temp > 0.f;
    s.logprob_thold = p.logprob_thold;
    s.seed = p.seed;
  }
  s.correct_mode = J->mode == WG_MODE_CORRECT;
  s.hist = take((size_t)R * j->Tcap);
  s.hist_tmp = take((size_t)R * j->Tcap);
  s.tbl = take((size_t)R * j->Tmax);
  s.tbl_tmp = take((size_t)R * j->Tmax);
  s.len = take(R);
  s.tok_in = take(R);
  s.parent = take(R);
  s.new_tok = take(R);
  s.new_len = take(R);
  s.carried = take(R);
  s.topk_tok = take((size_t)R * 5);
  s.utt_done = take(U);
  s.utt_steps = take(U);
  int* utt_id = take(U);
  s.utt_id = utt_id;
  s.n_done = take(1);
  s.pos = take(1);
  s.step = take(1);
  s.score = j->floats;
  s.new_score = j->floats + R;
  s.topk_lp = j->floats + 2 * R;
  s.logits = j->logits;
  s.forced = j->forced_dev;
  std::vector<int> pt((size_t)J->P * R);
  for (int i = 0; i < J->P; i++)
    for (int r = 0; r < R; r++) pt[(size_t)i * R + r] = J->prompt[i];
  if (cudaMemcpyAsync(utt_id, j->utt.data(), (size_t)U * 4, cudaMemcpyHostToDevice, j->st) != cudaSuccess ||
      cudaMemcpyAsync(j->ptok, pt.data(), pt.size() * 4, cudaMemcpyHostToDevice, j->st) != cudaSuccess ||
      cudaMemcpyAsync(j->prompt_dev, J->prompt.data(), (size_t)J->P * 4, cudaMemcpyHostToDevice, j->st) !=
          cudaSuccess) {
    set_error("job setup: prompt copy failed");
    return fail(WG_ERR_CUDA);
  }
  if (cudaMallocHost(&j->host_done, 16) != cudaSuccess) {
    set_error("job setup: cudaMallocHost failed");
    return fail(WG_ERR_OOM);
  }
  cudaError_t e = cudaStreamSynchronize(j->st);
  if (e != cudaSuccess) {
    set_error("job setup: %s", cudaGetErrorString(e));
    return fail(WG_ERR_CUDA);
  }
  *out = j;
  return WG_OK;
}

// Cross K/V precompute + state reset + (CORRECT) prompt prefill.
int start_devjob(wg_job* J, DevJob& j) {
  wg_model* m = J->m;
  WG_CHECK_CUDA(cudaSetDevice(j.dev));
  const int d = m->d;
  if (j.ldd == d) {
    WG_CHECK(launch_f32_to_f16(j.enc32, j.enc16, (int64_t)j.U * j.T * d, j.st));
  } else {
    for (int64_t r = 0; r < (int64_t)j.U * j.T; r++)  // test-sized models (d % 8 != 0) only
      WG_CHECK(launch_f32_to_f16(j.enc32 + r * d, j.enc16 + r * j.ldd, d, j.st));
  }
  // K_c = E Wk^T, V_c = E Wv^T + vB for all layers at once (decoder.go:923-940)
  Epi e = job_epi(j);
  e.mode = EPI_CROSS_KV; e.kv = j.cross; e.d = d; e.H = m->H; e.hd = m->hd; e.T = j.T; e.U = j.U;
  e.bias_v = j.dm->cross_vb; e.N = 2 * m->L * d;
  WG_CHECK(launch_matmul(j.dm->cross_kv, j.enc16, j.ldd, j.U * j.T, e, j.st));
  WG_CHECK(launch_sample_reset(j.ss, j.prompt_dev, j.st));
  if (J->mode == WG_MODE_REF_COMPAT) {
    // slot 0 of every (layer, row, k/v, head) starts at zero (decoder.go:346)
    int64_t nslabs = (int64_t)m->L * j.R * 2 * m->H;
    zero_slot0_kernel<<<(unsigned)((nslabs * m->hd + 255) / 256), 256, 0, j.st>>>(j.selfkv, nslabs, j.Tmax, m->hd);
    WG_CHECK(launch_status("zero_slot0"));
  } else {
    for (int i = 0; i + 1 < J->P; i++) {  // prompt prefill, positions 0..P-2
      WG_CHECK(forward_step(m, j, j.ptok + (size_t)i * j.R, false, J->mode));
      WG_CHECK(launch_pos_inc(j.ss, j.st));
    }
  }
  j.started = true;
  return WG_OK;
}

int step_eager(wg_job* J, DevJob& j) {
  WG_CHECK(forward_step(J->m, j, j.ss.tok_in, true, J->mode));
  NvtxRange sample_range("sampling");
  return launch_sample_step(j.ss, j.st);
}

// One token step as a CUDA graph (built on the first decode of the job).
int ensure_graph(wg_job* J, DevJob& j) {
  if (j.graph || env_i64("WG_NO_GRAPH", 0)) return WG_OK;
  WG_CHECK_CUDA(cudaSetDevice(j.dev));
  WG_CHECK(wait_stream(j.st));
  const int64_t before = g_launches.load();
  cudaGraph_t g = nullptr;
  WG_CHECK_CUDA(cudaStreamBeginCapture(j.st, cudaStreamCaptureModeThreadLocal));
  int rc = step_eager(J, j);
  cudaError_t e = cudaStreamEndCapture(j.st, &g);
  g_launches.store(before);
  if (rc != WG_OK || e != cudaSuccess) {
    if (g) cudaGraphDestroy(g);
    if (j.use_step) {
      // a runtime that cannot capture the cooperative step kernel: replay the
      // step eagerly (a handful of launches per token step)
      cudaGetLastError();
      j.graph = nullptr;
      return WG_OK;
    }
    if (rc == WG_OK) set_error("graph capture failed: %s", cudaGetErrorString(e));
    return rc == WG_OK ? WG_ERR_CUDA : rc;
  }
  size_t n = 0;
  cudaGraphGetNodes(g, nullptr, &n);
  e = cudaGraphInstantiate(&j.graph, g, 0);
  cudaGraphDestroy(g);
  if (e != cudaSuccess) {
    j.graph = nullptr;
    if (j.use_step) {  // as above: eager replay
      cudaGetLastError();
      return WG_OK;
    }
    set_error("cudaGraphInstantiate: %s", cudaGetErrorString(e));
    return WG_ERR_CUDA;
  }
  j.graph_kernels = (int64_t)n;
  return WG_OK;
}

int parse_fault(const char* key) {
  const char* v = getenv("WG_FAULT_INJECT");
  if (!v) return -1;
  const char* p = strstr(v, key);
  if (!p) return -1;
  p += strlen(key);
  if (*p != ':' && *p != '=') return -1;
  return atoi(p + 1);
}

}  // namespace
}  // namespace wg

using namespace wg;

// ============================================================================
// C ABI
// ============================================================================
extern "C" {

int wg_last_error(char* buf, size_t len) {
  if (buf && len) snprintf(buf, len, "%s", last_error());
  return WG_OK;
}

int wg_device_count(int* n) {
  int c = 0;
  if (cudaGetDeviceCount(&c) != cudaSuccess) c = 0;
  cudaGetLastError();
  if (n) *n = c;
  return WG_OK;
}

int wg_kernel_launch_count(int64_t* n) {
  if (n) *n = g_launches.load();
  return WG_OK;
}

int wg_model_create(const wg_model_desc* md, const int* devices, int n_dev, wg_model** out) {
  if (!md || !out) { set_error("wg_model_create: null argument"); return WG_ERR_INVALID; }
  *out = nullptr;
  const int d = md->n_state, H = md->n_head, L = md->n_layer, V = md->n_vocab, ctx = md->n_text_ctx;
  if (d <= 0 || H <= 0 || L <= 0 || V <= 0 || ctx <= 0 || d % H || !md->layers || !md->positional_embedding ||
      !md->ln_w || !md->ln_b) {
    set_error("model: decoder: invalid hyper-parameters d=%d heads=%d layers=%d vocab=%d ctx=%d", d, H, L, V, ctx);
    return WG_ERR_INVALID;
  }
  if (d / H > 64) {
    set_error("model: decoder: head dim %d > 64 is not supported", d / H);
    return WG_ERR_UNSUPPORTED;
  }
  if (!mat_ok(md->token_embedding, V, d)) {
    set_error("model: decoder: token embedding must be [%d, %d]", V, d);
    return WG_ERR_INVALID;
  }
  for (int l = 0; l < L; l++) {
    const wg_layer_desc& s = md->layers[l];
    bool ok = mat_ok(s.self_q, d, d) && mat_ok(s.self_k, d, d) && mat_ok(s.self_v, d, d) && mat_ok(s.self_o, d, d) &&
              mat_ok(s.cross_q, d, d) && mat_ok(s.cross_k, d, d) && mat_ok(s.cross_v, d, d) &&
              mat_ok(s.cross_o, d, d) && mat_ok(s.mlp0, 4 * d, d) && mat_ok(s.mlp2, d, 4 * d) && s.self_ln_w &&
              s.self_ln_b && s.cross_ln_w && s.cross_ln_b && s.mlp_ln_w && s.mlp_ln_b && s.self_q_b && s.self_v_b &&
              s.self_o_b && s.cross_q_b && s.cross_v_b && s.cross_o_b && s.mlp0_b && s.mlp2_b;
    if (!ok) {
      set_error("model: decoder: block %d has a missing tensor or a wrong shape", l);
      return WG_ERR_INVALID;
    }
  }
  int ndev = 0;
  if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev == 0) {
    cudaGetLastError();
    set_error("no CUDA device is available");
    return WG_ERR_NO_DEVICE;
  }
  std::vector<int> devs;
  if (!devices || n_dev <= 0) devs.push_back(0);
  else
    for (int i = 0; i < n_dev; i++) {
      if (devices[i] < 0 || devices[i] >= ndev) {
        set_error("wg_model_create: device %d does not exist (%d visible)", devices[i], ndev);
        return WG_ERR_INVALID;
      }
      devs.push_back(devices[i]);
    }
  wg_model* m = new wg_model();
  m->d = d; m->H = H; m->hd = d / H; m->L = L; m->V = V; m->ctx = ctx; m->eot = md->eot;
  for (int dv : devs) {
    DevModel* dm = nullptr;
    int rc = build_devmodel(md, dv, &dm);
    if (rc != WG_OK) {
      wg_model_destroy(m);
      return rc;
    }
    m->devs.push_back(dm);
  }
  *out = m;
  return WG_OK;
}

int wg_model_destroy(wg_model* m) {
  if (!m) return WG_OK;
  for (auto* d : m->devs) free_devmodel(d);
  delete m;
  return WG_OK;
}

int wg_model_info(const wg_model* m, int* n_vocab, int* n_state, int* n_head, int* n_layer, int* n_text_ctx) {
  if (!m) { set_error("wg_model_info: null model"); return WG_ERR_INVALID; }
  if (n_vocab) *n_vocab = m->V;
  if (n_state) *n_state = m->d;
  if (n_head) *n_head = m->H;
  if (n_layer) *n_layer = m->L;
  if (n_text_ctx) *n_text_ctx = m->ctx;
  return WG_OK;
}

int wg_model_set_eot(wg_model* m, int eot) {
  if (!m) { set_error("wg_model_set_eot: null model"); return WG_ERR_INVALID; }
  m->eot = eot;
  return WG_OK;
}

int wg_model_weight_bytes(const wg_model* m, int64_t* bytes) {
  if (!m || !bytes || m->devs.empty()) return WG_ERR_INVALID;
  *bytes = m->devs[0]->weight_bytes;
  return WG_OK;
}

int wg_job_create(wg_model* m, int U, int T_enc, const int32_t* prompt, int P, const wg_decode_params* params,
                  wg_job** out) {
  if (!m || !out || !params || !prompt) { set_error("wg_job_create: null argument"); return WG_ERR_INVALID; }
  *out = nullptr;
  if (U <= 0 || T_enc <= 0) { set_error("model: decoder: encoder output must be [T, %d]", m->d); return WG_ERR_INVALID; }
  if (P <= 0) { set_error("model: decode: forward: no tokens in state"); return WG_ERR_INVALID; }
  if (P > m->ctx) { set_error("model: decode: forward: position %d >= context length %d", P - 1, m->ctx); return WG_ERR_INVALID; }
  for (int i = 0; i < P; i++)
    if (prompt[i] < 0 || prompt[i] >= m->V) {
      set_error("model: decode: forward: invalid token ID %d", prompt[i]);
      return WG_ERR_INVALID;
    }
  if (params->mode != WG_MODE_REF_COMPAT && params->mode != WG_MODE_CORRECT) {
    set_error("wg_job_create: unknown mode %d", params->mode);
    return WG_ERR_INVALID;
  }
  int B = params->beam_size > 1 ? params->beam_size : 1;
  if (B > 16) { set_error("model: decode: beam size %d > 16 is not supported", B); return WG_ERR_UNSUPPORTED; }
  int mt = params->max_tokens;  // decoder.go:421-430
  if (mt <= 0) mt = m->ctx;
  if (m->ctx - P < mt) mt = m->ctx - P;
  if (mt < 0) mt = 0;
  wg_job* J = new wg_job();
  J->m = m; J->U = U; J->B = B; J->T = T_enc; J->P = P; J->max_tokens = mt; J->mode = params->mode;
  J->prompt.assign(prompt, prompt + P);
  J->params = *params;
  J->fault_step = parse_fault("step");
  J->fault_device = parse_fault("device");
  const int nd = (int)m->devs.size();
  for (int k = 0; k < nd; k++) {
    std::vector<int> utt;
    for (int u = k; u < U; u += nd) utt.push_back(u);
    if (utt.empty()) continue;
    DevJob* dj = nullptr;
    int rc = build_devjob(J, m->devs[k], utt, &dj);
    if (rc != WG_OK) { wg_job_destroy(J); return rc; }
    J->dj.push_back(dj);
  }
  *out = J;
  return WG_OK;
}

int wg_job_upload_encoder(wg_job* J, const float* const* enc) {
  if (!J || !enc) { set_error("wg_job_upload_encoder: null argument"); return WG_ERR_INVALID; }
  const size_t per = (size_t)J->T * J->m->d;
  for (DevJob* j : J->dj) {
    WG_CHECK_CUDA(cudaSetDevice(j->dev));
    for (size_t i = 0; i < j->utt.size(); i++) {
      if (!enc[j->utt[i]]) { set_error("wg_job_upload_encoder: utterance %d is null", j->utt[i]); return WG_ERR_INVALID; }
      WG_CHECK_CUDA(cudaMemcpyAsync(j->enc32 + i * per, enc[j->utt[i]], per * 4, cudaMemcpyHostToDevice, j->st));
    }
  }
  for (DevJob* j : J->dj) {
    cudaSetDevice(j->dev);
    WG_CHECK(wait_stream(j->st));
  }
  return WG_OK;
}

int wg_job_upload_encoder_one(wg_job* J, int u, const float* enc) {
  if (!J || !enc || u < 0 || u >= J->U) { set_error("wg_job_upload_encoder_one: bad argument"); return WG_ERR_INVALID; }
  const size_t per = (size_t)J->T * J->m->d;
  for (DevJob* j : J->dj)
    for (size_t i = 0; i < j->utt.size(); i++)
      if (j->utt[i] == u) {
        WG_CHECK_CUDA(cudaSetDevice(j->dev));
        WG_CHECK_CUDA(cudaMemcpyAsync(j->enc32 + i * per, enc, per * 4, cudaMemcpyHostToDevice, j->st));
        return wait_stream(j->st);  // the caller's buffer may be reused on return
      }
  set_error("wg_job_upload_encoder_one: utterance %d has no device", u);
  return WG_ERR_INVALID;
}

int wg_job_utterance_device(const wg_job* J, int u, int* device) {
  if (!J || !device || u < 0 || u >= J->U) { set_error("wg_job_utterance_device: bad argument"); return WG_ERR_INVALID; }
  for (const DevJob* j : J->dj)
    for (int v : j->utt)
      if (v == u) {
        *device = j->dev;
        return WG_OK;
      }
  set_error("wg_job_utterance_device: utterance %d has no device", u);
  return WG_ERR_INVALID;
}

int wg_job_upload_encoder_device(wg_job* J, const float* const* enc, void* stream) {
  if (!J || !enc) { set_error("wg_job_upload_encoder_device: null argument"); return WG_ERR_INVALID; }
  const size_t per = (size_t)J->T * J->m->d;
  cudaStream_t cs = reinterpret_cast<cudaStream_t>(stream);
  int prev = -1;
  WG_CHECK_CUDA(cudaGetDevice(&prev));
  int rc = WG_OK;
  for (DevJob* j : J->dj) {
    if ((rc = cudaSetDevice(j->dev) == cudaSuccess ? WG_OK : WG_ERR_CUDA) != WG_OK) break;
    for (size_t i = 0; i < j->utt.size() && rc == WG_OK; i++) {
      const float* src = enc[j->utt[i]];
      cudaPointerAttributes pa;
      if (!src || cudaPointerGetAttributes(&pa, src) != cudaSuccess || pa.type != cudaMemoryTypeDevice ||
          pa.device != j->dev) {
        cudaGetLastError();
        set_error("wg_job_upload_encoder_device: utterance %d must be device memory on device %d", j->utt[i],
                  j->dev);
        rc = WG_ERR_INVALID;
      }
    }
    if (rc != WG_OK) break;
    // the job's stream waits for the encoder's stream (its last writes of
    // the encoder outputs), then copies them device to device
    cudaEvent_t ev = nullptr;
    if (cs) {
      if (cudaEventCreateWithFlags(&ev, cudaEventDisableTiming) != cudaSuccess || cudaEventRecord(ev, cs) != cudaSuccess ||
          cudaStreamWaitEvent(j->st, ev, 0) != cudaSuccess) {
        set_error("wg_job_upload_encoder_device: stream ordering failed: %s", cudaGetErrorString(cudaGetLastError()));
        rc = WG_ERR_CUDA;
      }
    } else if (cudaStreamSynchronize(nullptr) != cudaSuccess) {  // legacy default stream
      set_error("wg_job_upload_encoder_device: default stream failed");
      rc = WG_ERR_CUDA;
    }
    for (size_t i = 0; i < j->utt.size() && rc == WG_OK; i++)
      if (cudaMemcpyAsync(j->enc32 + i * per, enc[j->utt[i]], per * 4, cudaMemcpyDeviceToDevice, j->st) !=
          cudaSuccess) {
        set_error("wg_job_upload_encoder_device: copy failed");
        rc = WG_ERR_CUDA;
      }
    if (ev) cudaEventDestroy(ev);
  }
  cudaSetDevice(prev);
  return rc;
}

int wg_job_start(wg_job* J) {
  if (!J) return WG_ERR_INVALID;
  if (J->cancel.load()) { set_error("model: decode: cancelled: context canceled"); return WG_ERR_CANCELLED; }
  for (size_t k = 0; k < J->dj.size(); k++) {
    DevJob& j = *J->dj[k];
    if (J->fault_device >= 0 && j.dev == J->fault_device) {
      set_error("model: decode: injected fault on device %d", j.dev);
      return WG_ERR_INJECTED;
    }
    {
      NvtxRange r("job start: encoder f16, cross K/V precompute, prompt prefill");
      WG_CHECK(start_devjob(J, j));
    }
    NvtxRange r("token-step graph capture");
    WG_CHECK(ensure_graph(J, j));
  }
  for (DevJob* j : J->dj) {
    cudaSetDevice(j->dev);
    WG_CHECK(wait_stream(j->st));
  }
  J->steps_done = 0;
  J->all_done = J->max_tokens == 0;
  return WG_OK;
}

static int poll_done(wg_job* J) {
  int total = 0;
  for (DevJob* j : J->dj) {
    WG_CHECK_CUDA(cudaSetDevice(j->dev));
    WG_CHECK_CUDA(cudaMemcpyAsync(j->host_done, j->ss.n_done, 4, cudaMemcpyDeviceToHost, j->st));
  }
  for (DevJob* j : J->dj) {
    cudaSetDevice(j->dev);
    WG_CHECK(wait_stream(j->st));
    total += *j->host_done;
  }
  if (total >= J->U) J->all_done = true;
  for (DevJob* j : J->dj) {
    cudaSetDevice(j->dev);
    WG_CHECK(check_wait_flags());
  }
  return WG_OK;
}

int wg_job_step(wg_job* J, int max_steps, int* done) {
  if (!J) return WG_ERR_INVALID;
  for (DevJob* j : J->dj)
    if (!j->started) { set_error("wg_job_step: wg_job_start was not called"); return WG_ERR_INVALID; }
  for (int s = 0; s < max_steps; s++) {
    if (J->all_done || J->steps_done >= J->max_tokens) break;
    if (J->cancel.load()) { set_error("model: decode: cancelled: context canceled"); return WG_ERR_CANCELLED; }
    if (J->fault_step >= 0 && J->steps_done == J->fault_step) {
      set_error("model: decode: injected fault at step %d", J->steps_done);
      return WG_ERR_INJECTED;
    }
    NvtxRange step_range("token step");
    for (DevJob* j : J->dj) {
      WG_CHECK_CUDA(cudaSetDevice(j->dev));
      if (j->graph) {
        WG_CHECK_CUDA(cudaGraphLaunch(j->graph, j->st));
        count_launch(j->graph_kernels);
      } else {
        WG_CHECK(step_eager(J, *j));
      }
    }
    J->steps_done++;
    if (J->steps_done % 32 == 0) WG_CHECK(poll_done(J));
  }
  WG_CHECK(poll_done(J));
  if (done) *done = (J->all_done || J->steps_done >= J->max_tokens) ? 1 : 0;
  return WG_OK;
}

int wg_job_result(wg_job* J, int32_t* tokens, int32_t* lens, float* scores) {
  if (!J || !tokens || !lens) { set_error("wg_job_result: null argument"); return WG_ERR_INVALID; }
  const int stride = J->P + J->max_tokens;
  for (DevJob* j : J->dj) {
    WG_CHECK_CUDA(cudaSetDevice(j->dev));
    std::vector<int> hist((size_t)j->R * j->Tcap), len(j->R);
    std::vector<float> sc(j->R);
    WG_CHECK_CUDA(cudaMemcpyAsync(hist.data(), j->ss.hist, hist.size() * 4, cudaMemcpyDeviceToHost, j->st));
    WG_CHECK_CUDA(cudaMemcpyAsync(len.data(), j->ss.len, (size_t)j->R * 4, cudaMemcpyDeviceToHost, j->st));
    WG_CHECK_CUDA(cudaMemcpyAsync(sc.data(), j->ss.score, (size_t)j->R * 4, cudaMemcpyDeviceToHost, j->st));
    WG_CHECK(wait_stream(j->st));
    for (size_t i = 0; i < j->utt.size(); i++) {
      int u = j->utt[i], row = (int)i * j->B;  // beams[0] is the best hypothesis (decoder.go:698)
      int n = std::min(len[row], stride);
      int32_t* dst = tokens + (size_t)u * stride;
      memset(dst, 0, (size_t)stride * 4);
      memcpy(dst, hist.data() + (size_t)row * j->Tcap, (size_t)n * 4);
      lens[u] = n;
      if (scores) scores[u] = J->B > 1 ? sc[row] : 0.f;
    }
  }
  return WG_OK;
}

int wg_job_beams(wg_job* J, int32_t* tokens, int32_t* lens, float* scores) {
  if (!J || !tokens || !lens) { set_error("wg_job_beams: null argument"); return WG_ERR_INVALID; }
  const int stride = J->P + J->max_tokens;
  for (DevJob* j : J->dj) {
    WG_CHECK_CUDA(cudaSetDevice(j->dev));
    std::vector<int> hist((size_t)j->R * j->Tcap), len(j->R);
    std::vector<float> sc(j->R);
    WG_CHECK_CUDA(cudaMemcpyAsync(hist.data(), j->ss.hist, hist.size() * 4, cudaMemcpyDeviceToHost, j->st));
    WG_CHECK_CUDA(cudaMemcpyAsync(len.data(), j->ss.len, (size_t)j->R * 4, cudaMemcpyDeviceToHost, j->st));
    WG_CHECK_CUDA(cudaMemcpyAsync(sc.data(), j->ss.score, (size_t)j->R * 4, cudaMemcpyDeviceToHost, j->st));
    WG_CHECK(wait_stream(j->st));
    for (size_t i = 0; i < j->utt.size(); i++)
      for (int b = 0; b < J->B; b++) {
        const int u = j->utt[i], row = (int)i * J->B + b;
        const size_t o = (size_t)u * J->B + b;
        const int n = std::min(len[row], stride);
        int32_t* dst = tokens + o * stride;
        memset(dst, 0, (size_t)stride * 4);
        memcpy(dst, hist.data() + (size_t)row * j->Tcap, (size_t)n * 4);
        lens[o] = n;
        if (scores) scores[o] = sc[row];
      }
  }
  return WG_OK;
}

int wg_job_timer(wg_job* J, int which, double* ms) {
  if (!J || (which != 0 && which != 1)) return WG_ERR_INVALID;
  double worst = 0.0;
  for (DevJob* j : J->dj) {
    WG_CHECK_CUDA(cudaSetDevice(j->dev));
    if (!j->ev[0]) {
      WG_CHECK_CUDA(cudaEventCreate(&j->ev[0]));
      WG_CHECK_CUDA(cudaEventCreate(&j->ev[1]));
    }
    WG_CHECK_CUDA(cudaEventRecord(j->ev[which], j->st));
  }
  if (which == 1) {
    for (DevJob* j : J->dj) {
      cudaSetDevice(j->dev);
      WG_CHECK(wait_stream(j->st));
      float el = 0.f;
      WG_CHECK_CUDA(cudaEventElapsedTime(&el, j->ev[0], j->ev[1]));
      worst = std::max(worst, (double)el);
    }
    if (ms) *ms = worst;
  }
  return WG_OK;
}

int wg_job_cancel(wg_job* J) {
  if (!J) return WG_ERR_INVALID;
  J->cancel.store(1);
  return WG_OK;
}

int wg_job_destroy(wg_job* J) {
  if (!J) return WG_OK;
  for (DevJob* j : J->dj) free_devjob(j);
  delete J;
  return WG_OK;
}

int wg_job_uses_step_kernel(const wg_job* J, int* on) {
  if (!J || !on) return WG_ERR_INVALID;
  *on = !J->dj.empty() && J->dj[0]->use_step && env_step_enabled();
  return WG_OK;
}

int wg_job_stats(const wg_job* J, int* steps_done, int* rows, int* max_tokens) {
  if (!J) return WG_ERR_INVALID;
  if (steps_done) *steps_done = J->steps_done;
  if (rows) *rows = J->U * J->B;
  if (max_tokens) *max_tokens = J->max_tokens;
  return WG_OK;
}

int wg_decode(wg_model* m, const float* const* enc, int U, int T_enc, const int32_t* prompt, int P,
              const wg_decode_params* params, int32_t* tokens, int32_t* lens, float* scores) {
  wg_job* J = nullptr;
  WG_CHECK(wg_job_create(m, U, T_enc, prompt, P, params, &J));
  int rc = wg_job_upload_encoder(J, enc);
  if (rc == WG_OK) rc = wg_job_start(J);
  int done = 0;
  while (rc == WG_OK && !done) rc = wg_job_step(J, 64, &done);
  if (rc == WG_OK) rc = wg_job_result(J, tokens, lens, scores);
  wg_job_destroy(J);
  return rc;
}

int wg_teacher_forced_logits(wg_model* m, const float* const* enc, int U, int T_enc, const int32_t* prompt, int P,
                             const int32_t* forced, int n_forced, int mode, float* logits) {
  if (!m || !enc || !prompt || !logits || U <= 0 || (n_forced > 0 && !forced)) {
    set_error("wg_teacher_forced_logits: bad argument");
    return WG_ERR_INVALID;
  }
  if (n_forced <= 0) return WG_OK;
  if (P + n_forced - 1 > m->ctx) {
    set_error("model: decode: forward: position %d >= context length %d", P + n_forced - 2, m->ctx);
    return WG_ERR_INVALID;
  }
  for (int64_t i = 0; i < (int64_t)U * n_forced; i++)
    if (forced[i] < 0 || forced[i] >= m->V) {
      set_error("model: decode: forward: invalid token ID %d", forced[i]);
      return WG_ERR_INVALID;
    }
  wg_decode_params p{};
  p.beam_size = 1;
  p.mode = mode;
  p.max_tokens = n_forced;
  p.no_fallback = 1;
  wg_job* J = nullptr;
  // a single-device job on the model's first device
  std::vector<DevModel*> saved = m->devs;
  m->devs.resize(1);
  int rc = wg_job_create(m, U, T_enc, prompt, P, &p, &J);
  m->devs = saved;
  if (rc != WG_OK) return rc;
  J->max_tokens = n_forced;
  rc = wg_job_upload_encoder(J, enc);
  DevJob& j = *J->dj[0];
  if (rc == WG_OK) {
    cudaSetDevice(j.dev);
    rc = start_devjob(J, j);
  }
  // forced tokens, step-major: [s][u]
  std::vector<int32_t> fs((size_t)n_forced * U);
  for (int u = 0; u < U; u++)
    for (int s = 0; s < n_forced; s++) fs[(size_t)s * U + u] = forced[(size_t)u * n_forced + s];
  if (rc == WG_OK && cudaMemcpyAsync(j.forced_dev, fs.data(), fs.size() * 4, cudaMemcpyHostToDevice, j.st) !=
                         cudaSuccess) {
    set_error("teacher forcing: copy failed");
    rc = WG_ERR_CUDA;
  }
  if (rc == WG_OK) rc = wait_stream(j.st);
  for (int s = 0; rc == WG_OK && s < n_forced; s++) {
    rc = forward_step(m, j, j.ss.tok_in, true, mode);
    if (rc == WG_OK && cudaMemcpyAsync(logits + (size_t)s * U * m->V, j.logits, (size_t)U * m->V * 4,
                                       cudaMemcpyDeviceToHost, j.st) != cudaSuccess) {
      set_error("teacher forcing: logits copy failed");
      rc = WG_ERR_CUDA;
    }
    if (rc == WG_OK) rc = launch_forced_step(j.ss, j.st);
    if (rc == WG_OK) rc = wait_stream(j.st);
    if (rc == WG_OK) rc = check_wait_flags();
  }
  wg_job_destroy(J);
  return rc;
}

int wg_dequant_test(uint32_t qtype, const void* raw, int64_t n, float* out) {
  if (!raw || !out || n <= 0) { set_error("wg_dequant_test: bad argument"); return WG_ERR_INVALID; }
  int ndev = 0;
  if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev == 0) {
    cudaGetLastError();
    set_error("no CUDA device is available");
    return WG_ERR_NO_DEVICE;
  }
  WG_CHECK_CUDA(cudaSetDevice(0));
  wg_matrix wm{};
  wm.qtype = qtype;
  wm.data = raw;
  std::vector<uint8_t> padded;
  if (qtype_is_quant(qtype)) {
    // rows of two quant blocks (the device layout needs cols % 64 == 0); an
    // odd trailing block is padded with a zero block
    const int64_t nb = (n + 31) / 32, bb = gguf_block_bytes(qtype);
    wm.cols = 64;
    wm.rows = (int)((nb + 1) / 2);
    if (nb % 2) {
      padded.assign((size_t)(nb + 1) * bb, 0);
      memcpy(padded.data(), raw, (size_t)nb * bb);
      wm.data = padded.data();
    }
  } else {
    wm.cols = (int)n;
    wm.rows = 1;
  }
  const wg_matrix* parts[1] = {&wm};
  DMat dm;
  cudaStream_t st = nullptr;
  WG_CHECK_CUDA(cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking));
  int rc = upload_matrix(parts, 1, &dm, st);
  float* d_out = nullptr;
  if (rc == WG_OK) rc = dalloc(&d_out, (size_t)wm.rows * wm.cols);
  if (rc == WG_OK) rc = dequant_dmat(dm, d_out, st);
  if (rc == WG_OK && cudaMemcpyAsync(out, d_out, (size_t)n * 4, cudaMemcpyDeviceToHost, st) != cudaSuccess) {
    set_error("wg_dequant_test: copy failed");
    rc = WG_ERR_CUDA;
  }
  if (rc == WG_OK) rc = wait_stream(st);
  cudaFree(d_out);
  free_dmat(dm);
  cudaStreamDestroy(st);
  return rc;
}

int wg_matmul_test(uint32_t qtype, const void* raw, int rows, int cols, const float* x, int M, float* out, int path) {
  if (!raw || !x || !out || rows <= 0 || cols <= 0 || M <= 0) {
    set_error("wg_matmul_test: bad argument");
    return WG_ERR_INVALID;
  }
  int ndev = 0;
  if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev == 0) {
    cudaGetLastError();
    set_error("no CUDA device is available");
    return WG_ERR_NO_DEVICE;
  }
  WG_CHECK_CUDA(cudaSetDevice(0));
  WG_CHECK(init_gemm_attributes());
  WG_CHECK(init_tc_attributes());
  WG_CHECK(init_gemv_bulk_attributes());
  cudaStream_t st = nullptr;
  WG_CHECK_CUDA(cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking));
  wg_matrix wm{qtype, rows, cols, raw};
  const wg_matrix* parts[1] = {&wm};
  DMat dm;
  int rc = upload_matrix(parts, 1, &dm, st);
  const int ld = round8(cols);
  float *dx = nullptr, *dout = nullptr, *ws = nullptr;
  __half* dx16 = nullptr;
  if (rc == WG_OK) rc = dalloc(&ws, (size_t)TC_SPLIT_WS_FLOATS);
  if (rc == WG_OK) rc = dalloc(&dx, (size_t)M * cols);
  if (rc == WG_OK) rc = dalloc(&dx16, (size_t)M * ld);
  if (rc == WG_OK) rc = dalloc(&dout, (size_t)M * rows);
  if (rc == WG_OK) {
    cudaMemsetAsync(dx16, 0, (size_t)M * ld * 2, st);
    cudaMemcpyAsync(dx, x, (size_t)M * cols * 4, cudaMemcpyHostToDevice, st);
    for (int r = 0; r < M && rc == WG_OK; r++) rc = launch_f32_to_f16(dx + (size_t)r * cols, dx16 + (size_t)r * ld, cols, st);
  }
  if (rc == WG_OK) {
    Epi e;
    e.mode = EPI_F32; e.out = dout; e.ldo = rows; e.N = rows;
    e.split_ws = ws; e.split_ws_floats = TC_SPLIT_WS_FLOATS;
    rc = launch_matmul(dm, dx16, ld, M, e, st, path);
  }
  if (rc == WG_OK && cudaMemcpyAsync(out, dout, (size_t)M * rows * 4, cudaMemcpyDeviceToHost, st) != cudaSuccess) {
    set_error("wg_matmul_test: copy failed");
    rc = WG_ERR_CUDA;
  }
  if (rc == WG_OK) rc = wait_stream(st);
  if (rc == WG_OK) {
    rc = check_wait_flags();
  }
  cudaFree(dx); cudaFree(dx16); cudaFree(dout); cudaFree(ws);
  free_dmat(dm);
  cudaStreamDestroy(st);
  return rc;
}

int wg_sample_test(const float* logits, int R, int V, const int32_t* hist, int n_hist, int eot,
                   const wg_decode_params* params, int step, int32_t* out_tok, float* out_lp) {
  if (!logits || R <= 0 || V <= 0 || n_hist < 0 || (n_hist > 0 && !hist) || !params || !out_tok || step < 0) {
    set_error("wg_sample_test: bad argument");
    return WG_ERR_INVALID;
  }
  int ndev = 0;
  if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev == 0) {
    cudaGetLastError();
    set_error("no CUDA device is available");
    return WG_ERR_NO_DEVICE;
  }
  WG_CHECK_CUDA(cudaSetDevice(0));
  return sample_test(logits, R, V, hist, n_hist, eot, params, step, out_tok, out_lp);
}

int wg_job_time_kernel(wg_job* J, int kclass, int iters, double* ms, double* bytes) {
  if (!J || J->dj.empty() || !ms || !bytes || iters <= 0) return WG_ERR_INVALID;
  DevJob& j = *J->dj[0];
  wg_model* m = J->m;
  DevModel& dm = *j.dm;
  WG_CHECK_CUDA(cudaSetDevice(j.dev));
  int pos_h = 0;
  WG_CHECK_CUDA(cudaMemcpy(&pos_h, j.ss.pos, 4, cudaMemcpyDeviceToHost));
  if (pos_h >= j.Tmax) pos_h = j.Tmax - 1;
  WG_CHECK_CUDA(cudaMemcpy(j.ss.pos, &pos_h, 4, cudaMemcpyHostToDevice));
  const int d = m->d, H = m->H, hd = m->hd, R = j.R, L = m->L;
  const bool ref = J->mode == WG_MODE_REF_COMPAT;
  const int64_t layer_kv = (int64_t)R * 2 * H * j.Tmax * hd;
  const int64_t layer_cross = (int64_t)j.U * 2 * H * j.T * hd;
  double b = 0;
  int launches = 0;
  auto run = [&](bool count) -> int {
    for (int l = 0; l < L; l++) {
      const DevLayer& ly = dm.layers[l];
      if (kclass == WG_KCLASS_GEMV || (kclass >= WG_KCLASS_MATMUL0 && kclass < WG_KCLASS_MATMUL0 + 6)) {
        const DMat* mats[6] = {&ly.qkv, &ly.so, &ly.cq, &ly.co, &ly.m0, &ly.m2};
        for (int k = 0; k < 6; k++) {
          if (kclass != WG_KCLASS_GEMV && k != kclass - WG_KCLASS_MATMUL0) continue;
          Epi e = job_epi(j);
          const __half* xin = k == 5 ? j.h16 : (k == 1 || k == 3 ? j.attn16 : j.xln16);
          int ldx = k == 5 ? j.ld4 : j.ldd;
          if (k == 4) { e.mode = EPI_GELU_F16; e.out16 = j.h16; e.ldo = j.ld4; e.bias = ly.m0_b; }
          else { e.mode = EPI_F32; e.out = j.logits; e.ldo = mats[k]->rows; }
          WG_CHECK(launch_matmul(*mats[k], xin, ldx, R, e, j.st));
          if (count) {
            b += (double)dmat_device_bytes(*mats[k]) + (double)R * mats[k]->cols * 2 +
                 (double)R * mats[k]->rows * (k == 4 ? 2 : 4);
            launches++;
          }
        }
      } else if (kclass == WG_KCLASS_SELF_ATTN) {
        SelfAttnArgs sa{};
        sa.q = j.q; sa.kv = j.selfkv + l * layer_kv; sa.tbl = (!ref && j.B > 1) ? j.ss.tbl : nullptr;
        sa.pos = j.ss.pos; sa.R = R; sa.H = H; sa.hd = hd; sa.Tmax = j.Tmax; sa.ref_compat = ref;
        sa.zero_unless_pos0 = 0; sa.out16 = j.attn16;
        WG_CHECK(launch_self_attn(sa, j.st));
        if (count) {
          int n_att = ref ? 1 : pos_h + 1;
          b += (double)R * n_att * H * hd * 2 * 2 + (double)R * d * 4 + (double)R * d * 2;
          launches++;
        }
      } else if (kclass == WG_KCLASS_CROSS_ATTN) {
        CrossAttnArgs ca{};
        ca.q = j.q; ca.kv = j.cross + l * layer_cross; ca.U = j.U; ca.B = j.B; ca.H = H; ca.hd = hd; ca.T = j.T;
        ca.out16 = j.attn16;
        WG_CHECK(launch_cross_attn(ca, j.st));
        if (count) {
          b += (double)j.U * 2 * j.T * d * 2 + (double)R * d * 4 + (double)R * d * 2;
          launches++;
        }
      } else if (kclass == WG_KCLASS_PRECOMPUTE) {
        if (l > 0) break;
        Epi e = job_epi(j);
        e.mode = EPI_CROSS_KV; e.kv = j.cross; e.d = d; e.H = H; e.hd = hd; e.T = j.T; e.U = j.U;
        e.bias_v = dm.cross_vb; e.N = 2 * L * d;
        WG_CHECK(launch_matmul(dm.cross_kv, j.enc16, j.ldd, j.U * j.T, e, j.st));
        if (count) {
          b += (double)dmat_device_bytes(dm.cross_kv) + (double)j.U * j.T * d * 2 + (double)j.U * j.T * 2 * L * d * 2;
          launches++;
        }
      } else if (kclass == WG_KCLASS_STEP) {
        if (l > 0) break;
        if (!j.use_step) {
          set_error("wg_job_time_kernel: this job does not use the step kernel");
          return WG_ERR_INVALID;
        }
        WG_CHECK(launch_step_job(m, j, J->mode));
        if (count) {
          for (const DevLayer& ly : dm.layers)
            b += (double)dmat_device_bytes(ly.qkv) + dmat_device_bytes(ly.so) + dmat_device_bytes(ly.cq) +
                 dmat_device_bytes(ly.co) + dmat_device_bytes(ly.m0) + dmat_device_bytes(ly.m2);
          const int n_att = ref ? 1 : pos_h + 1;
          b += (double)R * L * n_att * H * hd * 2 * 2 + (double)j.U * L * 2 * j.T * d * 2;
          launches++;
        }
      } else if (kclass == WG_KCLASS_LOGITS) {
        if (l > 0) break;
        Epi e = job_epi(j);
        e.mode = EPI_F32; e.out = j.logits; e.ldo = m->V; e.N = m->V;
        WG_CHECK(launch_matmul(dm.tok, j.xln16, j.ldd, R, e, j.st));
        if (count) {
          b += (double)dmat_device_bytes(dm.tok) + (double)R * d * 2 + (double)R * m->V * 4;
          launches++;
        }
      } else {
        set_error("wg_job_time_kernel: unknown kernel class %d", kclass);
        return WG_ERR_INVALID;
      }
    }
    return WG_OK;
  };
  WG_CHECK(run(false));  // warm-up
  cudaEvent_t e0, e1;
  WG_CHECK_CUDA(cudaEventCreate(&e0));
  WG_CHECK_CUDA(cudaEventCreate(&e1));
  WG_CHECK_CUDA(cudaEventRecord(e0, j.st));
  for (int i = 0; i < iters; i++) WG_CHECK(run(i == 0));
  WG_CHECK_CUDA(cudaEventRecord(e1, j.st));
  WG_CHECK(wait_stream(j.st));
  float el = 0.f;
  cudaEventElapsedTime(&el, e0, e1);
  cudaEventDestroy(e0);
  cudaEventDestroy(e1);
  *ms = launches ? (double)el / ((double)iters * launches) : 0.0;
  *bytes = launches ? b / launches : 0.0;
  return WG_OK;
}

}  // extern "C"

// ---- allocation-free matmul ------------------------------------------------------
// wg_model_matmul_noalloc runs the tcgen05 GEMM on a model's uploaded weights
// with caller-owned activations and outputs, and takes the split-K scratch
// from this fixed array instead of allocating a workspace: it exists for
// callers that may not allocate device memory while they run. The array is
// part of the module's device image (one copy per device); its address is
// looked up with the device current on the first call in each CUDA context
// of a device (again only if that context was destroyed and recreated).
// Every call on a device shares it, so calls whose kernels overlap in time
// race. Expired waits of these calls are recorded in their own error word,
// not in the one the decode jobs share.
namespace wg {
static __device__ __align__(256) float g_noalloc_scratch[WG_NOALLOC_SCRATCH_FLOATS];
static __device__ int g_noalloc_error;
namespace {
constexpr int NOALLOC_MAX_DEV = 64;
std::mutex g_noalloc_mu;
struct NoallocDev {
  void* ctx = nullptr;  // CUDA context the addresses belong to
  float* scratch = nullptr;
  int* err = nullptr;
};
NoallocDev g_noalloc[NOALLOC_MAX_DEV];

typedef CUresult (*CtxGetCurrentFn)(CUcontext*);
CtxGetCurrentFn ctx_get_current_fn() {
  static CtxGetCurrentFn fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      return reinterpret_cast<CtxGetCurrentFn>(p);
    return (CtxGetCurrentFn) nullptr;
  }();
  return fn;
}

// Device addresses of the scratch array and the error word on device dev
// (which must be current).
int noalloc_symbols(int dev, NoallocDev* out) {
  if (dev < 0 || dev >= NOALLOC_MAX_DEV) {
    set_error("wg_model_matmul_noalloc: device %d out of range", dev);
    return WG_ERR_INVALID;
  }
  CUcontext ctx = nullptr;
  CtxGetCurrentFn get = ctx_get_current_fn();
  if (!get || get(&ctx) != CUDA_SUCCESS || !ctx) {
    set_error("wg_model_matmul_noalloc: no current CUDA context on device %d", dev);
    return WG_ERR_CUDA;
  }
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  NoallocDev& nd = g_noalloc[dev];
  if (nd.ctx != (void*)ctx || !nd.scratch || !nd.err) {
    float* p = nullptr;
    int* w = nullptr;
    cudaError_t e = cudaGetSymbolAddress((void**)&p, g_noalloc_scratch);
    if (e == cudaSuccess) e = cudaGetSymbolAddress((void**)&w, g_noalloc_error);
    if (e != cudaSuccess || !p || !w) {
      set_error("wg_model_matmul_noalloc: cudaGetSymbolAddress of the scratch array failed: %s",
                cudaGetErrorString(e));
      return WG_ERR_CUDA;
    }
    nd.ctx = (void*)ctx;
    nd.scratch = p;
    nd.err = w;
  }
  *out = nd;
  return WG_OK;
}
}  // namespace
}  // namespace wg

extern "C" int wg_model_matmul_noalloc(wg_model* m, int replica, int layer, int which, const void* x16, int ldx,
                                       int rows, float* out, int ldo, void* stream, int wait) {
  using namespace wg;
  if (!m || replica < 0 || replica >= (int)m->devs.size() || layer < 0 || layer >= m->L || which < 0 ||
      which > 5 || !x16 || !out || rows <= 0) {
    set_error("wg_model_matmul_noalloc: bad argument");
    return WG_ERR_INVALID;
  }
  DevModel& dm = *m->devs[replica];
  const DevLayer& ly = dm.layers[layer];
  const DMat* mats[6] = {&ly.qkv, &ly.so, &ly.cq, &ly.co, &ly.m0, &ly.m2};
  const DMat& W = *mats[which];
  if (!tc_supported(W)) {
    set_error("wg_model_matmul_noalloc: the tensor-core kernel needs a quantised matrix with K %% 64 == 0");
    return WG_ERR_UNSUPPORTED;
  }
  if (ldx < W.cols || ldx % 8 || (reinterpret_cast<uintptr_t>(x16) & 15) || ldo < W.rows) {
    set_error("wg_model_matmul_noalloc: x16 needs 16-byte aligned rows of ldx >= %d (ldx %% 8 == 0), out ldo >= %d",
              W.cols, W.rows);
    return WG_ERR_INVALID;
  }
  int prev = -1;
  WG_CHECK_CUDA(cudaGetDevice(&prev));
  WG_CHECK_CUDA(cudaSetDevice(dm.dev));
  NoallocDev sym;
  int rc = noalloc_symbols(dm.dev, &sym);
  if (rc == WG_OK) {
    Epi e;
    e.mode = EPI_F32;
    e.out = out;
    e.ldo = ldo;
    e.N = W.rows;
    e.split_ws = sym.scratch;
    e.split_ws_floats = WG_NOALLOC_SCRATCH_FLOATS;
    e.err_word = sym.err;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    rc = launch_matmul(W, reinterpret_cast<const __half*>(x16), ldx, rows, e, st, 3);
    if (rc == WG_ERR_INVALID) {
      const std::string why = last_error();
      set_error("wg_model_matmul_noalloc: %s; the static scratch holds %lld floats", why.c_str(),
                (long long)WG_NOALLOC_SCRATCH_FLOATS);
    }
    if (rc == WG_OK && wait) {
      rc = wait_stream(st);
      int w = 0;
      if (rc == WG_OK && cudaMemcpyFromSymbol(&w, g_noalloc_error, sizeof(int)) != cudaSuccess) {
        set_error("wg_model_matmul_noalloc: reading the error word failed");
        rc = WG_ERR_CUDA;
      }
      if (rc == WG_OK && w) {
        const int z = 0;
        cudaMemcpyToSymbol(g_noalloc_error, &z, sizeof(int));
        set_error("wg_model_matmul_noalloc: a bounded wait of the tcgen05 kernel expired (code 0x%x)", w);
        rc = WG_ERR_DEVICE_FLAG;
      }
    }
  }
  cudaSetDevice(prev);
  return rc;
}
