// Multi-GPU pool behind the C ABI: one engine per GPU, each driven by its own worker
// thread, so a C / Rust / JNI caller of the drop-in library can use every GPU of a box
// without torch.distributed.
//
// The reference transcribes the segments of `-S` mode one after another on one context
// (crates/qwen-asr/src/transcribe.rs:328-423). With past-text conditioning off (the
// default, context.rs:150) the segments are independent, so the pool computes the split
// points on the host (bit-exact, transcribe.rs:253-278), assigns segments to GPUs longest
// first, lets every worker transcribe its segments with batched decode, and joins the texts
// in segment order with the reference's boundary-space rule (transcribe.rs:280-286,
// 401-422). Concurrent streams are sharded the same way (stream i on worker i mod n). No
// data crosses GPUs; nothing but host strings is gathered.
#include <algorithm>
#include <condition_variable>
#include <cstring>
#include <functional>
#include <memory>
#include <mutex>
#include <numeric>
#include <string>
#include <thread>
#include <vector>

#include "../../include/qwen_asr_ext.h"
#include "c_api_types.h"
#include "common.h"
#include "host.h"
#include "transcribe.h"

namespace qasr {

// Longest-processing-time-first: segments in decreasing length (ties: lower index first),
// each to the worker with the least assigned samples (ties: lower worker). Deterministic.
std::vector<int> assign_longest_first(const std::vector<long long>& lengths, int workers) {
  std::vector<int> order(lengths.size()), out(lengths.size(), 0);
  std::iota(order.begin(), order.end(), 0);
  std::stable_sort(order.begin(), order.end(), [&](int a, int b) { return lengths[a] > lengths[b]; });
  std::vector<long long> load(std::max(1, workers), 0);
  for (int i : order) {
    int w = (int)(std::min_element(load.begin(), load.end()) - load.begin());
    out[i] = w;
    load[w] += lengths[i];
  }
  return out;
}

namespace {

// A worker thread that owns one engine and runs one task at a time.
class Worker {
 public:
  explicit Worker(int device) : device_(device), th_([this] { loop(); }) {}
  ~Worker() {
    {
      std::lock_guard<std::mutex> lk(mu_);
      stop_ = true;
    }
    cv_.notify_all();
    th_.join();
  }
  void post(std::function<void()> fn) {
    std::lock_guard<std::mutex> lk(mu_);
    task_ = std::move(fn);
    busy_ = true;
    cv_.notify_all();
  }
  void wait() {
    std::unique_lock<std::mutex> lk(mu_);
    cv_.wait(lk, [&] { return !busy_; });
  }
  int device() const { return device_; }
  std::unique_ptr<QwenAsrEngine> eng;

 private:
  void loop() {
    for (;;) {
      std::function<void()> fn;
      {
        std::unique_lock<std::mutex> lk(mu_);
        cv_.wait(lk, [&] { return stop_ || busy_; });
        if (stop_) return;
        fn = std::move(task_);
      }
      cudaSetDevice(device_);
      fn();
      {
        std::lock_guard<std::mutex> lk(mu_);
        busy_ = false;
      }
      cv_.notify_all();
    }
  }
  int device_;
  std::mutex mu_;
  std::condition_variable cv_;
  std::function<void()> task_;
  bool busy_ = false, stop_ = false;
  std::thread th_;
};

}  // namespace
}  // namespace qasr

struct QwenAsrPool {
  std::vector<std::unique_ptr<qasr::Worker>> workers;
  // Runs fn(i, ctx) on every worker in parallel and waits; false if any returned false (the
  // first failure's message becomes the last error).
  bool run_all(const std::function<bool(int, qasr::Ctx&)>& fn, const std::vector<int>* which = nullptr) {
    const int n = (int)workers.size();
    std::vector<char> ok(n, 1);
    std::vector<std::string> err(n);
    std::vector<int> idx;
    if (which) {
      idx = *which;
    } else {
      idx.resize(n);
      std::iota(idx.begin(), idx.end(), 0);
    }
    for (int i : idx)
      workers[i]->post([&, i] {
        try {
          ok[i] = fn(i, workers[i]->eng->ctx) ? 1 : 0;
        } catch (const std::exception& ex) {
          ok[i] = 0;
          qasr::set_error(ex.what());
        }
        if (!ok[i]) err[i] = qasr::last_error();
      });
    for (int i : idx) workers[i]->wait();
    for (int i : idx)
      if (!ok[i]) {
        qasr::set_error("pool worker " + std::to_string(i) + " (device " + std::to_string(workers[i]->device()) +
                        "): " + err[i]);
        return false;
      }
    return true;
  }
};

namespace {
char* dup_c(const std::string& s) {
  if (memchr(s.data(), 0, s.size())) return nullptr;
  char* out = (char*)malloc(s.size() + 1);
  if (out) memcpy(out, s.data(), s.size() + 1);
  return out;
}
}  // namespace

extern "C" {

QwenAsrPool* qwen_asr_pool_new(const char* model_dir, const int32_t* devices, int32_t n_devices, int32_t verbosity) {
  if (!model_dir || n_devices < 0 || (n_devices > 0 && !devices)) return nullptr;
  qasr::g_verbose = verbosity;
  std::vector<int> devs;
  if (n_devices == 0) {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || n <= 0) {
      qasr::set_error("pool: no CUDA device");
      return nullptr;
    }
    for (int i = 0; i < n; ++i) devs.push_back(i);
  } else {
    devs.assign(devices, devices + n_devices);
  }
  auto* p = new (std::nothrow) QwenAsrPool();
  if (!p) return nullptr;
  for (int d : devs) {
    p->workers.emplace_back(new qasr::Worker(d));
    p->workers.back()->eng.reset(new QwenAsrEngine());
  }
  const std::string dir(model_dir);
  if (!p->run_all([&](int i, qasr::Ctx& c) { return c.load(dir, p->workers[i]->device()); })) {
    delete p;
    return nullptr;
  }
  return p;
}

void qwen_asr_pool_free(QwenAsrPool* p) { delete p; }

int32_t qwen_asr_pool_size(const QwenAsrPool* p) { return p ? (int32_t)p->workers.size() : 0; }

QwenAsrEngine* qwen_asr_pool_engine(QwenAsrPool* p, int32_t i) {
  if (!p || i < 0 || i >= (int32_t)p->workers.size()) return nullptr;
  return p->workers[i]->eng.get();
}

void qwen_asr_pool_set_segment_sec(QwenAsrPool* p, float sec) {
  if (!p) return;
  for (auto& w : p->workers) w->eng->ctx.segment_sec = sec;
}

int32_t qwen_asr_pool_set_language(QwenAsrPool* p, const char* language) {
  if (!p || !language) return -1;
  for (auto& w : p->workers)
    if (!w->eng->ctx.set_force_language(language)) return -1;
  return 0;
}

void qwen_asr_pool_set_decode_mode(QwenAsrPool* p, int32_t mode) {
  if (!p) return;
  for (auto& w : p->workers) w->eng->ctx.eng.set_decode_mode(mode == 1 ? qasr::DECODE_BF16 : qasr::DECODE_INT8);
}

void qwen_asr_pool_set_force_n_tokens(QwenAsrPool* p, int32_t n) {
  if (!p) return;
  for (auto& w : p->workers) w->eng->ctx.force_n_tokens = n > 0 ? n : 0;
}

void qwen_asr_pool_stream_set_max_new_tokens(QwenAsrPool* p, int32_t n) {
  if (!p || n <= 0) return;
  for (auto& w : p->workers) w->eng->ctx.stream_max_new_tokens = n;
}

char* qwen_asr_pool_transcribe_pcm(QwenAsrPool* p, const float* samples, int32_t n_samples) {
  if (!p || p->workers.empty() || !samples || n_samples <= 0) return nullptr;
  qasr::Ctx& c0 = p->workers[0]->eng->ctx;
  std::vector<float> in(samples, samples + n_samples);
  std::string result;
  // one segment, or segments that depend on each other (past-text conditioning): worker 0
  std::vector<float> audio;
  if (!c0.skip_silence) audio = in;
  else if (!c0.eng.compact_silence(in.data(), (long)in.size(), audio)) return nullptr;
  std::vector<size_t> splits = qasr::split_points(audio, c0.segment_sec, c0.search_sec);
  if (splits.size() <= 1 || c0.past_text_conditioning || p->workers.size() == 1) {
    const std::vector<int> first{0};
    const bool ok = p->run_all([&](int, qasr::Ctx& c) { return c.transcribe_audio(in, result); }, &first);
    return ok ? dup_c(result) : nullptr;
  }
  std::vector<std::pair<size_t, size_t>> bounds;
  std::vector<long long> lens;
  for (size_t s = 0; s < splits.size(); ++s) {
    bounds.emplace_back(splits[s], s + 1 < splits.size() ? splits[s + 1] : audio.size());
    lens.push_back((long long)(bounds.back().second - bounds.back().first));
  }
  const int nw = (int)p->workers.size();
  const std::vector<int> who = qasr::assign_longest_first(lens, nw);
  std::vector<std::vector<int>> mine(nw);
  for (size_t s = 0; s < who.size(); ++s) mine[who[s]].push_back((int)s);
  std::vector<std::vector<std::string>> texts(nw);
  const bool ok = p->run_all([&](int i, qasr::Ctx& c) {
    if (mine[i].empty()) return true;
    std::vector<std::pair<size_t, size_t>> b;
    for (int s : mine[i]) b.push_back(bounds[s]);
    c.reset_perf();
    return c.transcribe_segment_list(audio.data(), audio.size(), b, texts[i]);
  });
  if (!ok) return nullptr;
  std::vector<std::string> ordered(bounds.size());
  for (int i = 0; i < nw; ++i)
    for (size_t k = 0; k < mine[i].size(); ++k) ordered[mine[i][k]] = texts[i][k];
  for (const std::string& st : ordered) {
    if (st.empty()) continue;
    if (!result.empty() && qasr::should_insert_boundary_space((uint8_t)result.back(), (uint8_t)st[0])) result += ' ';
    result += st;
  }
  return dup_c(result);
}

int32_t qwen_asr_pool_stream_push_many(QwenAsrPool* p, QwenAsrStreamState* const* states,
                                       const float* const* samples, const int32_t* n_samples, int32_t count,
                                       int32_t finalize, char** deltas_out) {
  if (!p || p->workers.empty() || count < 0 || (count > 0 && (!states || !deltas_out))) return -1;
  for (int32_t i = 0; i < count; ++i) {
    if (!states[i]) {
      qasr::set_error("pool_stream_push_many: a null stream");
      return -1;
    }
    for (int32_t j = 0; j < i; ++j)
      if (states[j] == states[i]) {
        qasr::set_error("pool_stream_push_many: a stream appears twice");
        return -1;
      }
  }
  for (int32_t i = 0; i < count; ++i)
    if (samples && samples[i] && n_samples && n_samples[i] > 0)
      states[i]->audio_buf.insert(states[i]->audio_buf.end(), samples[i], samples[i] + n_samples[i]);
  const int nw = (int)p->workers.size();
  std::vector<std::vector<int>> mine(nw);
  for (int32_t i = 0; i < count; ++i) mine[i % nw].push_back(i);
  std::vector<std::vector<std::string>> deltas(nw);
  const bool ok = p->run_all([&](int w, qasr::Ctx& c) {
    if (mine[w].empty()) return true;
    std::vector<const std::vector<float>*> bufs;
    std::vector<qasr::StreamState*> sts;
    for (int i : mine[w]) {
      bufs.push_back(&states[i]->audio_buf);
      sts.push_back(&states[i]->state);
    }
    return c.stream_push_many(bufs, sts, finalize != 0, deltas[w]);
  });
  if (!ok) return -1;
  for (int w = 0; w < nw; ++w)
    for (size_t k = 0; k < mine[w].size(); ++k) {
      std::string txt = qasr::utf8_lossy(deltas[w][k]);
      deltas_out[mine[w][k]] = txt.empty() ? nullptr : dup_c(txt);
    }
  return 0;
}

int32_t qwen_asr_debug_assign_longest_first(const int64_t* lengths, int32_t n, int32_t workers, int32_t* worker_of) {
  if (n < 0 || workers <= 0 || (n > 0 && (!lengths || !worker_of))) return -1;
  std::vector<long long> l(lengths, lengths + n);
  std::vector<int> w = qasr::assign_longest_first(l, workers);
  for (int32_t i = 0; i < n; ++i) worker_of[i] = w[i];
  return 0;
}

}  // extern "C"
