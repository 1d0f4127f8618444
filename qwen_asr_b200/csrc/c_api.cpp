// C ABI of libqwen_asr: the 17 exports of crates/qwen-asr/src/c_api.rs with the same
// names, argument meaning and error convention (NULL / -1, never an exception), plus
// the clearly separated extensions declared in include/qwen_asr_ext.h.
#include <cstdlib>
#include <algorithm>
#include <cstring>
#include <fstream>
#include <mutex>
#include <new>
#include <sstream>

#include "../../include/qwen_asr.h"
#include "../../include/qwen_asr_ext.h"
#include "transcribe.h"

#include "c_api_types.h"

namespace {
// Returns a malloc'ed copy, or NULL when the text holds an interior NUL (CString::new).
char* to_c_string(const std::string& s) {
  if (memchr(s.data(), 0, s.size())) return nullptr;
  char* out = (char*)malloc(s.size() + 1);
  if (!out) return nullptr;
  memcpy(out, s.data(), s.size() + 1);
  return out;
}

// Strict UTF-8 as Rust's CStr::to_str accepts it (no overlong forms, no surrogates, at most
// U+10FFFF): the reference returns NULL / -1 for paths and languages that fail it
// (c_api.rs:28-31, 59-62, 141-144).
bool valid_utf8(const char* z) {
  const unsigned char* s = (const unsigned char*)z;
  while (*s) {
    const unsigned c = *s;
    int n;
    unsigned cp;
    if (c < 0x80) {
      ++s;
      continue;
    } else if (c >= 0xC2 && c <= 0xDF) {
      n = 1; cp = c & 0x1F;
    } else if (c >= 0xE0 && c <= 0xEF) {
      n = 2; cp = c & 0x0F;
    } else if (c >= 0xF0 && c <= 0xF4) {
      n = 3; cp = c & 0x07;
    } else {
      return false;
    }
    for (int i = 1; i <= n; ++i) {
      if ((s[i] & 0xC0) != 0x80) return false;
      cp = (cp << 6) | (s[i] & 0x3F);
    }
    if ((n == 2 && (cp < 0x800 || (cp >= 0xD800 && cp <= 0xDFFF))) || (n == 3 && (cp < 0x10000 || cp > 0x10FFFF)))
      return false;
    s += n + 1;
  }
  return true;
}

bool utf8_arg(const char* z, const char* what) {
  if (valid_utf8(z)) return true;
  qasr::set_error(std::string(what) + " is not valid UTF-8");
  return false;
}

int pick_device() {
  if (const char* d = getenv("QASR_DEVICE")) return atoi(d);
  int dev = 0;
  cudaGetDevice(&dev);
  return dev;
}

char* run_transcribe(QwenAsrEngine* e, const std::vector<float>& samples) {
  std::string out;
  try {
    if (!e->ctx.transcribe_audio(samples, out)) return nullptr;
  } catch (const std::exception& ex) {
    qasr::set_error(std::string("transcribe: ") + ex.what());
    return nullptr;
  }
  return to_c_string(out);
}
// A parsed WAV file: 16 kHz input goes straight to the transcriber; any other rate is
// resampled on the GPU (audio.rs:133-196) and, when neither segmentation nor silence
// compaction needs the samples on the host, transcribed from device memory.
char* run_transcribe_native(QwenAsrEngine* e, const std::vector<float>& samples, int rate) {
  if (rate == qasr::kSampleRate) return run_transcribe(e, samples);
  std::string out;
  try {
    long n = 0;
    const float* d = e->ctx.eng.resample_to_device(samples.data(), (long)samples.size(), rate, &n);
    if (!d) return nullptr;
    if (e->ctx.segment_sec <= 0.0f && !e->ctx.skip_silence) {
      if (!e->ctx.transcribe_device(d, (size_t)n, out)) return nullptr;
    } else {
      std::vector<float> h(n);
      if (cudaMemcpyAsync(h.data(), d, (size_t)n * 4, cudaMemcpyDeviceToHost, e->ctx.eng.stream()) != cudaSuccess ||
          cudaStreamSynchronize(e->ctx.eng.stream()) != cudaSuccess) {
        qasr::set_error("resample: device-to-host copy failed");
        return nullptr;
      }
      if (!e->ctx.transcribe_audio(h, out)) return nullptr;
    }
  } catch (const std::exception& ex) {
    qasr::set_error(std::string("transcribe: ") + ex.what());
    return nullptr;
  }
  return to_c_string(out);
}

}  // namespace

extern "C" {

QwenAsrEngine* qwen_asr_load_model(const char* model_dir, int32_t n_threads, int32_t verbosity) {
  (void)n_threads;  // the CPU thread count has no meaning here: all math runs on the GPU
  return qwen_asr_load_model_on_device(model_dir, -1, verbosity);
}

QwenAsrEngine* qwen_asr_load_model_on_device(const char* model_dir, int32_t device, int32_t verbosity) {
  if (!model_dir || !utf8_arg(model_dir, "model_dir")) return nullptr;
  qasr::g_verbose = verbosity;
  QwenAsrEngine* e = new (std::nothrow) QwenAsrEngine();
  if (!e) return nullptr;
  try {
    if (!e->ctx.load(model_dir, device >= 0 ? device : pick_device())) {
      delete e;
      return nullptr;
    }
  } catch (const std::exception& ex) {
    qasr::set_error(std::string("load: ") + ex.what());
    delete e;
    return nullptr;
  }
  return e;
}

char* qwen_asr_transcribe_file(QwenAsrEngine* e, const char* wav_path) {
  if (!e || !wav_path || !utf8_arg(wav_path, "wav_path")) return nullptr;
  std::ifstream f(wav_path, std::ios::binary);
  if (!f) {
    qasr::set_error(std::string("cannot read ") + wav_path);
    return nullptr;
  }
  std::stringstream ss;
  ss << f.rdbuf();
  std::string data = ss.str();
  std::vector<float> samples;
  int rate = 0;
  if (!qasr::parse_wav_native((const uint8_t*)data.data(), data.size(), samples, rate)) return nullptr;
  return run_transcribe_native(e, samples, rate);
}

char* qwen_asr_transcribe_pcm(QwenAsrEngine* e, const float* samples, int32_t n_samples) {
  if (!e || !samples || n_samples <= 0) return nullptr;
  return run_transcribe(e, std::vector<float>(samples, samples + n_samples));
}

char* qwen_asr_transcribe_wav_buffer(QwenAsrEngine* e, const uint8_t* wav_data, int32_t wav_len) {
  if (!e || !wav_data || wav_len <= 0) return nullptr;
  std::vector<float> samples;
  int rate = 0;
  if (!qasr::parse_wav_native(wav_data, (size_t)wav_len, samples, rate)) return nullptr;
  return run_transcribe_native(e, samples, rate);
}

void qwen_asr_set_segment_sec(QwenAsrEngine* e, float sec) {
  if (e) e->ctx.segment_sec = sec;
}

int32_t qwen_asr_set_language(QwenAsrEngine* e, const char* language) {
  if (!e || !language || !utf8_arg(language, "language")) return -1;
  return e->ctx.set_force_language(language) ? 0 : -1;
}

void qwen_asr_free_string(char* s) { free(s); }

void qwen_asr_free(QwenAsrEngine* e) { delete e; }

QwenAsrStreamState* qwen_asr_stream_new(void) { return new (std::nothrow) QwenAsrStreamState(); }

void qwen_asr_stream_free(QwenAsrStreamState* s) { delete s; }

void qwen_asr_stream_reset(QwenAsrStreamState* s) {
  if (!s) return;
  s->state.reset();
  s->audio_buf.clear();
}

char* qwen_asr_stream_push(QwenAsrEngine* e, QwenAsrStreamState* s, const float* samples, int32_t n_samples,
                           int32_t finalize) {
  if (!e || !s) return nullptr;
  if (samples && n_samples > 0) s->audio_buf.insert(s->audio_buf.end(), samples, samples + n_samples);
  std::string delta;
  try {
    if (!e->ctx.stream_push_audio(s->audio_buf, s->state, finalize != 0, delta)) return nullptr;
  } catch (const std::exception& ex) {
    qasr::set_error(std::string("stream: ") + ex.what());
    return nullptr;
  }
  std::string txt = qasr::utf8_lossy(delta);
  if (txt.empty()) return nullptr;
  return to_c_string(txt);
}

int32_t qwen_asr_stream_push_many(QwenAsrEngine* e, QwenAsrStreamState* const* states, const float* const* samples,
                                  const int32_t* n_samples, int32_t count, int32_t finalize, char** deltas_out) {
  if (!e || count < 0 || (count > 0 && (!states || !deltas_out))) return -1;
  std::vector<const std::vector<float>*> bufs;
  std::vector<qasr::StreamState*> sts;
  // validate the whole list before any stream takes new audio, so a rejected call changes nothing
  for (int32_t i = 0; i < count; ++i) {
    if (!states[i]) {
      qasr::set_error("stream_push_many: a null stream");
      return -1;
    }
    for (int32_t j = 0; j < i; ++j)
      if (states[j] == states[i]) {
        qasr::set_error("stream_push_many: a stream appears twice");
        return -1;
      }
  }
  for (int32_t i = 0; i < count; ++i) {
    if (samples && samples[i] && n_samples && n_samples[i] > 0)
      states[i]->audio_buf.insert(states[i]->audio_buf.end(), samples[i], samples[i] + n_samples[i]);
    bufs.push_back(&states[i]->audio_buf);
    sts.push_back(&states[i]->state);
  }
  std::vector<std::string> deltas;
  try {
    if (!e->ctx.stream_push_many(bufs, sts, finalize != 0, deltas)) return -1;
  } catch (const std::exception& ex) {
    qasr::set_error(std::string("stream: ") + ex.what());
    return -1;
  }
  for (int32_t i = 0; i < count; ++i) {
    std::string txt = qasr::utf8_lossy(deltas[i]);
    deltas_out[i] = txt.empty() ? nullptr : to_c_string(txt);
  }
  return 0;
}

char* qwen_asr_stream_get_result(QwenAsrStreamState* s) {
  if (!s) return nullptr;
  std::string txt = qasr::utf8_lossy(s->state.result_bytes);
  if (txt.empty()) return nullptr;
  return to_c_string(txt);
}

void qwen_asr_stream_set_chunk_sec(QwenAsrEngine* e, float sec) {
  if (e && sec > 0.0f) e->ctx.stream_chunk_sec = sec;
}
void qwen_asr_stream_set_rollback(QwenAsrEngine* e, int32_t tokens) {
  if (e && tokens >= 0) e->ctx.stream_rollback = tokens;
}
void qwen_asr_stream_set_unfixed_chunks(QwenAsrEngine* e, int32_t chunks) {
  if (e && chunks >= 0) e->ctx.stream_unfixed_chunks = chunks;
}
void qwen_asr_stream_set_max_new_tokens(QwenAsrEngine* e, int32_t tokens) {
  if (e && tokens > 0) e->ctx.stream_max_new_tokens = tokens;
}

// ------------------------------------------------------------------ extensions
const char* qwen_asr_last_error(void) {
  static thread_local std::string s;
  s = qasr::last_error();
  return s.c_str();
}

int32_t qwen_asr_set_prompt(QwenAsrEngine* e, const char* prompt) {
  if (!e || !prompt) return -1;
  e->ctx.set_prompt(prompt);
  return 0;
}
void qwen_asr_set_past_text(QwenAsrEngine* e, int32_t on) {
  if (e) e->ctx.past_text_conditioning = on != 0;
}
void qwen_asr_set_skip_silence(QwenAsrEngine* e, int32_t on) {
  if (e) e->ctx.skip_silence = on != 0;
}
int32_t qwen_asr_set_decode_mode(QwenAsrEngine* e, int32_t mode) {
  if (!e || (mode != 0 && mode != 1)) return -1;
  e->ctx.eng.set_decode_mode(mode == 0 ? qasr::DECODE_INT8 : qasr::DECODE_BF16);
  return 0;
}
void qwen_asr_set_force_n_tokens(QwenAsrEngine* e, int32_t n) {
  if (e) e->ctx.force_n_tokens = n > 0 ? n : 0;
}
int32_t qwen_asr_transcribe_segments(QwenAsrEngine* e, const float* samples, int64_t n_samples, const int64_t* starts,
                                     const int64_t* ends, int32_t count, char** texts_out) {
  if (!e || !samples || n_samples <= 0 || !starts || !ends || count < 0 || (count > 0 && !texts_out)) return -1;
  std::vector<std::pair<size_t, size_t>> bounds;
  for (int32_t i = 0; i < count; ++i) {
    if (starts[i] < 0 || ends[i] < starts[i] || ends[i] > n_samples) {
      qasr::set_error("transcribe_segments: segment " + std::to_string(i) + " is out of range");
      return -1;
    }
    bounds.emplace_back((size_t)starts[i], (size_t)ends[i]);
  }
  std::vector<std::string> texts;
  try {
    e->ctx.reset_perf();
    e->ctx.last_tokens.clear();
    e->ctx.perf_audio_ms = 1000.0 * (double)n_samples / qasr::kSampleRate;
    if (!e->ctx.transcribe_segment_list(samples, (size_t)n_samples, bounds, texts)) return -1;
  } catch (const std::exception& ex) {
    qasr::set_error(std::string("transcribe_segments: ") + ex.what());
    return -1;
  }
  for (int32_t i = 0; i < count; ++i) texts_out[i] = to_c_string(texts[i]);
  return 0;
}

int32_t qwen_asr_set_decode_batch(QwenAsrEngine* e, int32_t n) {
  if (!e) return 0;
  e->ctx.decode_batch = n > 0 ? n : 0;
  const int lim = e->ctx.eng.max_decode_batch();
  return n > 0 ? std::min<int32_t>(n, lim) : lim;
}
void qwen_asr_set_use_graph(QwenAsrEngine* e, int32_t on) {
  if (e) e->ctx.eng.use_graph = on != 0;
}

void qwen_asr_set_record_logits(QwenAsrEngine* e, int32_t on) {
  if (!e) return;
  e->ctx.eng.record_logits = on != 0;
  e->ctx.eng.recorded_logits.clear();
}

int64_t qwen_asr_recorded_logits(QwenAsrEngine* e, float* out, int64_t cap) {
  if (!e) return -1;
  const auto& r = e->ctx.eng.recorded_logits;
  if (out) memcpy(out, r.data(), std::min<size_t>(r.size(), cap > 0 ? (size_t)cap : 0) * 4);
  return (int64_t)r.size();
}

void qwen_asr_set_profile(QwenAsrEngine* e, int32_t on) {
  if (!e) return;
  e->ctx.eng.profile = on != 0;
  for (int i = 0; i < 6; ++i) {
    e->ctx.eng.prof_ms[i] = 0;
    e->ctx.eng.prof_n[i] = 0;
  }
}

int32_t qwen_asr_profile_report(QwenAsrEngine* e, double* ms, int64_t* counts, int32_t cap) {
  if (!e) return -1;
  for (int i = 0; i < 6 && i < cap; ++i) {
    if (ms) ms[i] = e->ctx.eng.prof_ms[i];
    if (counts) counts[i] = e->ctx.eng.prof_n[i];
  }
  return 6;
}

char* qwen_asr_transcribe_device(QwenAsrEngine* e, const float* d_samples, int32_t n_samples) {
  if (!e || !d_samples || n_samples <= 0) return nullptr;
  std::string out;
  try {
    if (!e->ctx.transcribe_device(d_samples, (size_t)n_samples, out)) return nullptr;
  } catch (const std::exception& ex) {
    qasr::set_error(std::string("transcribe: ") + ex.what());
    return nullptr;
  }
  return to_c_string(out);
}

void* qwen_asr_cuda_stream(QwenAsrEngine* e) { return e ? (void*)e->ctx.eng.stream() : nullptr; }

int64_t qwen_asr_launch_count(QwenAsrEngine* e) { return e ? (int64_t)e->ctx.eng.launches : -1; }

void qwen_asr_set_timeline(QwenAsrEngine* e, int32_t on) {
  if (e) e->ctx.eng.set_timeline(on != 0);
}

int64_t qwen_asr_get_timeline(QwenAsrEngine* e, uint64_t* out, int64_t cap) {
  if (!e) return -1;
  const auto& t = e->ctx.eng.last_timeline;
  if (out)
    for (int64_t i = 0; i < (int64_t)t.size() && i < cap; ++i) out[i] = t[i];
  return (int64_t)t.size();
}

int32_t qwen_asr_last_tokens(QwenAsrEngine* e, int32_t segment, int32_t* out, int32_t cap) {
  if (!e || segment < 0 || segment >= (int)e->ctx.last_tokens.size()) return -1;
  const auto& v = e->ctx.last_tokens[segment];
  if (out)
    for (int i = 0; i < (int)v.size() && i < cap; ++i) out[i] = v[i];
  return (int32_t)v.size();
}
int32_t qwen_asr_last_segments(QwenAsrEngine* e) { return e ? (int32_t)e->ctx.last_tokens.size() : -1; }

int32_t qwen_asr_get_perf(QwenAsrEngine* e, double* out, int32_t cap) {
  if (!e || !out) return -1;
  const auto& c = e->ctx;
  double v[] = {c.perf_total_ms, c.perf_audio_ms, c.perf_encode_ms, c.perf_decode_ms, (double)c.perf_text_tokens,
                c.eng.perf.mel_ms, c.eng.perf.enc_ms, c.eng.perf.prefill_ms, c.eng.perf.decode_ms,
                (double)c.eng.perf.decode_steps};
  int n = (int)(sizeof(v) / sizeof(v[0]));
  for (int i = 0; i < n && i < cap; ++i) out[i] = v[i];
  return n;
}

int32_t qwen_asr_model_info(QwenAsrEngine* e, int32_t* out, int32_t cap) {
  if (!e || !out) return -1;
  const auto& c = e->ctx.eng.cfg();
  int v[] = {c.enc_d_model, c.enc_layers, c.enc_heads, c.enc_ffn_dim, c.dec_hidden, c.dec_layers, c.dec_heads,
             c.dec_kv_heads, c.dec_intermediate, c.vocab_size, e->ctx.eng.device()};
  int n = (int)(sizeof(v) / sizeof(v[0]));
  for (int i = 0; i < n && i < cap; ++i) out[i] = v[i];
  return n;
}

int32_t qwen_asr_debug_mel(QwenAsrEngine* e, const float* samples, int32_t n, float* out, int64_t cap) {
  if (!e || !samples || n <= 0) return -1;
  int F = e->ctx.eng.mel(samples, n, false);
  if (F <= 0) return -1;
  if (out) {
    if ((int64_t)F * 128 > cap) return -1;
    if (cudaMemcpy(out, e->ctx.eng.mel_buf(), (size_t)F * 128 * 4, cudaMemcpyDeviceToHost) != cudaSuccess) return -1;
  }
  return F;
}

int32_t qwen_asr_debug_encode(QwenAsrEngine* e, const float* mel, int32_t n_frames, float* out, int64_t cap) {
  if (!e || !mel || n_frames <= 0) return -1;
  qasr::DevBuf<float> d;
  if (!d.alloc((size_t)n_frames * 128)) return -1;
  if (cudaMemcpy(d.p, mel, (size_t)n_frames * 128 * 4, cudaMemcpyHostToDevice) != cudaSuccess) return -1;
  int T = e->ctx.eng.encode(d.p, n_frames);
  if (T <= 0) return -1;
  size_t n = (size_t)T * e->ctx.eng.cfg().dec_hidden;
  if (out) {
    if ((int64_t)n > cap) return -1;
    if (cudaMemcpy(out, e->ctx.eng.enc_out(), n * 4, cudaMemcpyDeviceToHost) != cudaSuccess) return -1;
  }
  return T;
}

int32_t qwen_asr_debug_decode(QwenAsrEngine* e, const float* rows, int32_t n_rows, const int32_t* forced,
                              int32_t n_steps, int32_t* out_ids, float* out_logits, float* out_hidden) {
  if (!e || !rows || n_rows <= 0 || n_steps < 0) return -1;
  auto& eng = e->ctx.eng;
  if (!eng.prefill_rows(rows, n_rows, 0)) return -1;
  if (out_hidden) {
    std::vector<float> h;
    if (!eng.copy_prefill_hidden(h, n_rows)) return -1;
    memcpy(out_hidden, h.data(), h.size() * 4);
  }
  std::vector<int> f, ids;
  std::vector<float> lg;
  if (forced) f.assign(forced, forced + n_steps);
  if (!eng.decode(n_steps, false, ids, forced ? &f : nullptr, out_logits ? &lg : nullptr)) return -1;
  if (out_ids)
    for (int i = 0; i < (int)ids.size(); ++i) out_ids[i] = ids[i];
  if (out_logits) memcpy(out_logits, lg.data(), lg.size() * 4);
  return (int32_t)ids.size();
}

int64_t qwen_asr_debug_resample(QwenAsrEngine* e, const float* in, int64_t n, int32_t from_rate, float* out,
                                int64_t cap) {
  if (!e || !in || n <= 0 || from_rate <= 0) return -1;
  long m = 0;
  const float* d = e->ctx.eng.resample_to_device(in, (long)n, from_rate, &m);
  if (!d) return -1;
  if (out && m <= cap) {
    // the engine's stream does not synchronise with the default stream: copy on it
    cudaStream_t s = e->ctx.eng.stream();
    if (cudaMemcpyAsync(out, d, (size_t)m * 4, cudaMemcpyDeviceToHost, s) != cudaSuccess ||
        cudaStreamSynchronize(s) != cudaSuccess)
      return -1;
  }
  return m;
}

int32_t qwen_asr_debug_valid_utf8(const char* s) { return s && valid_utf8(s) ? 1 : 0; }

int64_t qwen_asr_gemm_fallbacks(void) { return qasr::gemm_tc_fallbacks(); }

int32_t qwen_asr_debug_kv(QwenAsrEngine* e, int32_t slot, int32_t layer, int32_t n_pos, float* k, float* v) {
  if (!e || !k || !v) return -1;
  return e->ctx.eng.copy_kv(slot, layer, n_pos, k, v) ? 0 : -1;
}

int32_t qwen_asr_debug_kv_capacity(QwenAsrEngine* e) { return e ? e->ctx.eng.kv_capacity() : -1; }

int32_t qwen_asr_debug_grow_kv(QwenAsrEngine* e, int32_t needed) {
  if (!e || needed <= 0) return -1;
  return e->ctx.eng.grow_kv(needed) ? e->ctx.eng.kv_capacity() : -1;
}

int64_t qwen_asr_debug_quant(QwenAsrEngine* e, int32_t layer, int32_t which, int8_t* q, float* s, int64_t cap_rows) {
  if (!e || (cap_rows > 0 && (!q || !s))) return -1;
  return e->ctx.eng.copy_quant(layer, which, q, s, cap_rows);
}

int32_t qwen_asr_debug_gemm_timed(int32_t M, int32_t N, int32_t K, int32_t epi, int32_t reps, float* ms,
                                  uint64_t* timeline) {
  // Times `reps` back-to-back tensor-core GEMMs of random operands on the current device
  // (CUDA events); timeline (optional, 148 x 8 stamps) records the last launch.
  if (M <= 0 || N <= 0 || K <= 0 || reps <= 0 || !ms) return -1;
  const int ncols = epi == qasr::EPI_SWIGLU ? N / 2 : N;
  qasr::DevBuf<float> dA, dC, db;
  qasr::DevBuf<uint16_t> dB;
  qasr::DevBuf<unsigned long long> dtl;
  if (!dA.alloc((size_t)M * K) || !dB.alloc((size_t)N * K) || !dC.alloc((size_t)M * ncols) || !db.alloc(N) ||
      !dtl.alloc(148 * 8))
    return -1;
  cudaMemset(dA.p, 0, (size_t)M * K * 4);
  cudaMemset(dB.p, 0, (size_t)N * K * 2);
  cudaMemset(db.p, 0, (size_t)N * 4);
  cudaMemset(dC.p, 0, (size_t)M * ncols * 4);
  cudaMemset(dtl.p, 0, 148 * 8 * 8);
  qasr::GemmArgs g;
  g.M = M; g.N = N; g.K = K; g.A = dA.p; g.lda = K; g.B = dB.p; g.ldb = K; g.C = dC.p; g.ldc = ncols; g.epi = epi;
  g.bias = db.p; g.resid = dC.p; g.ldr = ncols;
  cudaEvent_t e0, e1;
  cudaEventCreate(&e0);
  cudaEventCreate(&e1);
  if (!qasr::gemm_tc(g, 0)) return -2;  // warm-up (tensor maps, scratch)
  cudaEventRecord(e0, 0);
  for (int i = 0; i < reps; ++i) {
    if (timeline && i == reps - 1) qasr::gemm_tc_set_timeline(dtl.p);
    qasr::gemm_tc(g, 0);
  }
  cudaEventRecord(e1, 0);
  qasr::gemm_tc_set_timeline(nullptr);
  if (cudaEventSynchronize(e1) != cudaSuccess) return -3;
  cudaEventElapsedTime(ms, e0, e1);
  *ms /= reps;
  cudaEventDestroy(e0);
  cudaEventDestroy(e1);
  if (timeline) cudaMemcpy(timeline, dtl.p, 148 * 8 * 8, cudaMemcpyDeviceToHost);
  return qasr::gemm_tc_error() ? -4 : 0;
}

int32_t qwen_asr_debug_attn_timeline(uint64_t* dev_buf) {
  // Points the attention kernels' debug timeline at a device buffer of 64 u64 (NULL: off).
  qasr::attn_tc_set_timeline((unsigned long long*)dev_buf);
  return 0;
}

int32_t qwen_asr_debug_gemm(int32_t M, int32_t N, int32_t K, const float* A, const uint16_t* B, const float* bias,
                            const float* resid, int32_t epi, int32_t impl, float* C) {
  if (M <= 0 || N <= 0 || K <= 0 || !A || !B || !C) return -1;
  int ncols = epi == qasr::EPI_SWIGLU ? N / 2 : N;
  qasr::DevBuf<float> dA, dC, dbias, dres;
  qasr::DevBuf<uint16_t> dB;
  qasr::DevBuf<int> dg;
  if (!dA.upload(A, (size_t)M * K) || !dB.upload(B, (size_t)N * K) || !dC.alloc((size_t)M * ncols) || !dg.alloc(1))
    return -1;
  qasr::GemmArgs g;
  g.M = M; g.N = N; g.K = K; g.A = dA.p; g.lda = K; g.B = dB.p; g.ldb = K; g.C = dC.p; g.ldc = ncols; g.epi = epi;
  if (bias) {
    if (!dbias.upload(bias, N)) return -1;
    g.bias = dbias.p;
  }
  if (resid) {
    if (!dres.upload(resid, (size_t)M * N)) return -1;
    if (cudaMemcpy(dC.p, resid, (size_t)M * N * 4, cudaMemcpyHostToDevice) != cudaSuccess) return -1;
    g.resid = dC.p; g.ldr = N;
  }
  g.gmax = dg.p;
  cudaDeviceSynchronize();
  if (impl == 1) {
    if (!qasr::gemm_tc(g, 0)) return -2;
  } else {
    qasr::gemm_simt(g, 0);
  }
  if (cudaDeviceSynchronize() != cudaSuccess || cudaGetLastError() != cudaSuccess) return -3;
  if (qasr::gemm_tc_error()) return -4;
  if (cudaMemcpy(C, dC.p, (size_t)M * ncols * 4, cudaMemcpyDeviceToHost) != cudaSuccess) return -1;
  return 0;
}

// ---- host-only hooks (no GPU needed): tokenizer, WAV, segmentation, text handling ----
int32_t qwen_asr_debug_tokenize(const char* model_dir, const char* text, int32_t* out, int32_t cap) {
  if (!model_dir || !text) return -1;
  qasr::Tokenizer t;
  if (!t.load(model_dir)) return -1;
  std::vector<int> ids;
  if (!t.encode(text, ids)) return -2;
  for (int i = 0; i < (int)ids.size() && i < cap; ++i) out[i] = ids[i];
  return (int32_t)ids.size();
}

int32_t qwen_asr_debug_detokenize(const char* model_dir, const int32_t* ids, int32_t n, char* out, int32_t cap) {
  if (!model_dir || !ids || n < 0) return -1;
  qasr::Tokenizer t;
  if (!t.load(model_dir)) return -1;
  std::string b;
  for (int i = 0; i < n; ++i) b += t.decode_bytes(ids[i]);
  if ((int)b.size() > cap) return -1;
  memcpy(out, b.data(), b.size());
  return (int32_t)b.size();
}

int64_t qwen_asr_debug_parse_wav(const uint8_t* data, int64_t len, float* out, int64_t cap) {
  if (!data || len <= 0) return -1;
  std::vector<float> s;
  if (!qasr::parse_wav_buffer(data, (size_t)len, s)) return -1;
  if (out) {
    if ((int64_t)s.size() > cap) return -1;
    memcpy(out, s.data(), s.size() * 4);
  }
  return (int64_t)s.size();
}

int32_t qwen_asr_debug_split_points(const float* samples, int64_t n, float segment_sec, float search_sec,
                                    int64_t* out, int32_t cap) {
  if (!samples || n < 0) return -1;
  std::vector<float> x(samples, samples + n);
  auto sp = qasr::split_points(x, segment_sec, search_sec);
  for (int i = 0; i < (int)sp.size() && i < cap; ++i) out[i] = (int64_t)sp[i];
  return (int32_t)sp.size();
}

int64_t qwen_asr_debug_compact_silence_gpu(QwenAsrEngine* e, const float* samples, int64_t n, float* out,
                                           int64_t cap) {
  if (!e || !samples || n < 0) return -1;
  std::vector<float> r;
  if (!e->ctx.eng.compact_silence(samples, (long)n, r)) return -1;
  if (out) {
    if ((int64_t)r.size() > cap) return -1;
    memcpy(out, r.data(), r.size() * 4);
  }
  return (int64_t)r.size();
}

int64_t qwen_asr_debug_compact_silence(const float* samples, int64_t n, float* out, int64_t cap) {
  if (!samples || n < 0) return -1;
  auto r = qasr::compact_silence(std::vector<float>(samples, samples + n));
  if (out) {
    if ((int64_t)r.size() > cap) return -1;
    memcpy(out, r.data(), r.size() * 4);
  }
  return (int64_t)r.size();
}

int32_t qwen_asr_debug_lossy_trim(const char* bytes, int32_t n, char* out, int32_t cap) {
  if (!bytes || n < 0) return -1;
  std::string r = qasr::rust_trim(qasr::utf8_lossy(std::string(bytes, bytes + n)));
  if ((int)r.size() > cap) return -1;
  memcpy(out, r.data(), r.size());
  return (int32_t)r.size();
}

char* qwen_asr_forced_align(QwenAsrEngine* e, const float* samples, int64_t n_samples, const char* text,
                            const char* language) {
  if (!e || !samples || n_samples <= 0 || !text) {
    qasr::set_error("forced_align: invalid arguments");
    return nullptr;
  }
  std::string lang = language ? language : "";
  if (!lang.empty()) {
    const std::string norm = qasr::normalize_language(lang);
    if (!norm.empty()) lang = norm;
  }
  std::vector<qasr::Ctx::AlignItem> items;
  try {
    if (!e->ctx.forced_align(samples, (size_t)n_samples, text, lang, items)) return nullptr;
  } catch (const std::exception& ex) {
    qasr::set_error(std::string("forced_align: ") + ex.what());
    return nullptr;
  }
  auto esc = [](const std::string& s) {
    std::string o;
    for (unsigned char ch : s) {
      if (ch == '"' || ch == '\\') {
        o += '\\';
        o += (char)ch;
      } else if (ch < 0x20) {
        char b[8];
        snprintf(b, sizeof b, "\\u%04x", ch);
        o += b;
      } else {
        o += (char)ch;
      }
    }
    return o;
  };
  std::string js = "[";
  for (size_t i = 0; i < items.size(); ++i) {
    char b[96];
    snprintf(b, sizeof b, "\",\"start_ms\":%.9g,\"end_ms\":%.9g}", items[i].start_ms, items[i].end_ms);
    js += (i ? ",{\"text\":\"" : "{\"text\":\"") + esc(items[i].text) + b;
  }
  js += "]";
  return to_c_string(js);
}

int32_t qwen_asr_debug_align_words(const char* text, const char* language, char* out, int32_t cap) {
  if (!text || !language) return -1;
  std::vector<std::string> words;
  if (!qasr::align_split_words(text, language, words)) return -1;
  std::string r;
  for (size_t i = 0; i < words.size(); ++i) r += (i ? "\n" : "") + words[i];
  if ((int)r.size() + 1 > cap) return -1;
  memcpy(out, r.c_str(), r.size() + 1);
  return (int32_t)words.size();
}

void qwen_asr_debug_fix_timestamps(float* ts, int32_t n) {
  if (!ts || n <= 0) return;
  std::vector<float> v(ts, ts + n);
  qasr::fix_timestamps(v);
  memcpy(ts, v.data(), (size_t)n * 4);
}

int32_t qwen_asr_debug_normalize_language(const char* lang, char* out, int32_t cap) {
  if (!lang) return -1;
  std::string r = qasr::normalize_language(lang);
  if ((int)r.size() + 1 > cap) return -1;
  memcpy(out, r.c_str(), r.size() + 1);
  return (int32_t)r.size();
}

}  // extern "C"
