// batcher.cu — pipeline batching: concurrent single-utterance Decode calls
// gathered into shared decode jobs.
//
// whisper.go decodes one 30-s chunk per Decoder.Decode call
// (internal/model/pipeline.go:90-193: the chunks of a file one after
// another, and every concurrent Context.Transcribe on its own goroutine,
// whisper.go:24). One utterance gives 1-5 rows per token step; the GPU's
// weight stream per step costs the same for 1 row or 40, so the batcher
// makes one job of every request that arrives within a collection window and
// shares the prompt, the encoder length and the decode parameters (requests
// that differ wait for a later job). A single worker thread per batcher runs
// the jobs (wg_job_create / upload / start / step / result); callers block
// on their own request until its results are in.
#include <atomic>
#include <chrono>
#include <condition_variable>
#include <cstring>
#include <deque>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

#include "kernels.cuh"

namespace {

struct Request {
  const float* enc = nullptr;
  int T = 0;
  std::vector<int32_t> prompt;
  wg_decode_params params{};
  const volatile int* cancel = nullptr;
  // results
  std::vector<int32_t> tokens;
  int32_t len = 0;
  float score = 0.f;
  int rc = WG_OK;
  std::string err;
  bool done = false;
};

bool same_params(const wg_decode_params& a, const wg_decode_params& b) {
  return a.beam_size == b.beam_size && a.temperature == b.temperature && a.attempt == b.attempt &&
         a.logprob_thold == b.logprob_thold && a.no_speech_thold == b.no_speech_thold &&
         a.no_fallback == b.no_fallback && a.max_tokens == b.max_tokens && a.suppress_nst == b.suppress_nst &&
         a.mode == b.mode && a.suppress_eot == b.suppress_eot && a.seed == b.seed;
}
bool compatible(const Request& a, const Request& b) {
  return a.T == b.T && a.prompt == b.prompt && same_params(a.params, b.params);
}

}  // namespace

struct wg_batcher {
  wg_model* m = nullptr;
  int max_utt = 1;
  std::chrono::microseconds window{0};
  std::mutex mu;
  std::condition_variable cv_work, cv_done;
  std::deque<Request*> queue;
  bool stop = false;
  std::thread worker;
  std::atomic<int64_t> jobs{0}, utterances{0};

  void run() {
    std::unique_lock<std::mutex> lk(mu);
    for (;;) {
      cv_work.wait(lk, [&] { return stop || !queue.empty(); });
      if (queue.empty()) return;  // stop requested and nothing left
      // collection window from the oldest request's arrival at the worker
      const auto until = std::chrono::steady_clock::now() + window;
      auto count_compat = [&] {
        int n = 0;
        for (Request* r : queue) n += compatible(*r, *queue.front());
        return n;
      };
      while (!stop && count_compat() < max_utt && std::chrono::steady_clock::now() < until)
        cv_work.wait_until(lk, until);
      std::vector<Request*> batch;
      Request* head = queue.front();
      for (auto it = queue.begin(); it != queue.end() && (int)batch.size() < max_utt;) {
        if (compatible(**it, *head)) {
          batch.push_back(*it);
          it = queue.erase(it);
        } else {
          ++it;
        }
      }
      lk.unlock();
      decode(batch);
      lk.lock();
      for (Request* r : batch) r->done = true;
      cv_done.notify_all();
    }
  }

  void decode(std::vector<Request*>& batch) {
    const Request& h = *batch.front();
    const int U = (int)batch.size(), P = (int)h.prompt.size();
    std::vector<const float*> encs(U);
    for (int u = 0; u < U; u++) encs[u] = batch[u]->enc;
    wg_job* J = nullptr;
    int rc = wg_job_create(m, U, h.T, h.prompt.data(), P, &h.params, &J);
    if (rc == WG_OK) rc = wg_job_upload_encoder(J, encs.data());
    if (rc == WG_OK) rc = wg_job_start(J);
    int done = 0, steps = 0, maxt = 0;
    if (J) wg_job_stats(J, &steps, nullptr, &maxt);
    while (rc == WG_OK && !done) {
      bool all_cancelled = true;
      for (Request* r : batch) all_cancelled = all_cancelled && r->cancel && *r->cancel;
      if (all_cancelled) wg_job_cancel(J);
      rc = wg_job_step(J, 16, &done);
    }
    std::vector<int32_t> toks, lens(U);
    std::vector<float> scores(U);
    const int stride = P + maxt;
    if (rc == WG_OK) {
      toks.resize((size_t)U * stride);
      rc = wg_job_result(J, toks.data(), lens.data(), scores.data());
    }
    const std::string err = rc == WG_OK ? "" : wg::last_error();
    if (J) wg_job_destroy(J);
    jobs++;
    utterances += U;
    for (int u = 0; u < U; u++) {
      Request& r = *batch[u];
      r.rc = rc;
      r.err = err;
      if (rc == WG_OK) {
        r.tokens.assign(toks.begin() + (size_t)u * stride, toks.begin() + (size_t)(u + 1) * stride);
        r.len = lens[u];
        r.score = scores[u];
        if (r.cancel && *r.cancel) {
          r.rc = WG_ERR_CANCELLED;
          r.err = "model: decode: cancelled: context canceled";
        }
      }
    }
  }
};

extern "C" {

int wg_batcher_create(wg_model* m, int max_utterances, int window_us, wg_batcher** out) {
  if (!m || !out || max_utterances < 1 || window_us < 0) {
    wg::set_error("wg_batcher_create: bad argument");
    return WG_ERR_INVALID;
  }
  wg_batcher* b = new wg_batcher();
  b->m = m;
  b->max_utt = max_utterances;
  b->window = std::chrono::microseconds(window_us);
  b->worker = std::thread([b] { b->run(); });
  *out = b;
  return WG_OK;
}

int wg_batcher_decode(wg_batcher* b, const float* enc, int T_enc, const int32_t* prompt, int P,
                      const wg_decode_params* params, const volatile int* cancel, int32_t* tokens, int tokens_cap,
                      int32_t* len, float* score) {
  if (!b || !enc || T_enc <= 0 || !prompt || P <= 0 || !params || !tokens || tokens_cap <= 0 || !len) {
    wg::set_error("wg_batcher_decode: bad argument");
    return WG_ERR_INVALID;
  }
  Request r;
  r.enc = enc;
  r.T = T_enc;
  r.prompt.assign(prompt, prompt + P);
  r.params = *params;
  r.cancel = cancel;
  {
    std::unique_lock<std::mutex> lk(b->mu);
    if (b->stop) {
      wg::set_error("wg_batcher_decode: the batcher is closed");
      return WG_ERR_INVALID;
    }
    b->queue.push_back(&r);
    b->cv_work.notify_one();
    b->cv_done.wait(lk, [&] { return r.done; });
  }
  if (r.rc != WG_OK) {
    wg::set_error("%s", r.err.c_str());
    return r.rc;
  }
  const int n = std::min<int>(r.len, tokens_cap);
  memcpy(tokens, r.tokens.data(), (size_t)n * 4);
  *len = n;
  if (score) *score = r.score;
  return WG_OK;
}

int wg_batcher_stats(const wg_batcher* b, int64_t* jobs, int64_t* utterances) {
  if (!b) return WG_ERR_INVALID;
  if (jobs) *jobs = b->jobs.load();
  if (utterances) *utterances = b->utterances.load();
  return WG_OK;
}

int wg_batcher_destroy(wg_batcher* b) {
  if (!b) return WG_OK;
  {
    std::lock_guard<std::mutex> lk(b->mu);
    b->stop = true;
  }
  b->cv_work.notify_all();
  if (b->worker.joinable()) b->worker.join();  // requests already queued are decoded first
  delete b;
  return WG_OK;
}

}  // extern "C"
