// Transcription orchestration (crates/qwen-asr/src/transcribe.rs), host side. All model
// math runs on the GPU through Engine; this file only holds the control flow, prompt
// layout and text handling, which must follow the reference exactly.
#include "transcribe.h"

#include <algorithm>
#include <cstdio>
#include <cstdlib>
#include <atomic>
#include <chrono>
#include <cstring>

namespace qasr {

// transcribe.rs:13-23
static const int kPrefixHead[] = {151644, 8948, 198};
static const int kPrefixTail[] = {151645, 198, 151644, 872, 198, 151669};
static const int kSuffixBase[] = {151670, 151645, 198, 151644, 77091, 198};
static const int kDegenMaxPeriod = 6, kDegenMinRepeats = 4, kStaleChunks = 4, kResetInterval = 45;
static const size_t kResetCarry = 24, kMaxEncWindows = 4;

static double now_ms() {
  using namespace std::chrono;
  return duration<double, std::milli>(steady_clock::now().time_since_epoch()).count();
}

uint64_t StreamState::next_uid() {
  static std::atomic<uint64_t> counter{1};
  return counter.fetch_add(1);
}

void StreamState::reset() {
  bool keep = prompt_prepared;
  *this = StreamState();
  prompt_prepared = keep;
}

int Ctx::stream_slot(StreamState& st, bool& owned) {
  const int first = kDecodeMaxBatch, n = stream_slot_count();
  if ((int)slot_uid.size() < first + n) {
    slot_uid.resize(first + n, 0);
    slot_used.resize(first + n, 0);
  }
  ++slot_tick;
  if (st.slot >= first && st.slot < first + n && slot_uid[st.slot] == st.uid) {
    owned = true;
    slot_used[st.slot] = slot_tick;
    return st.slot;
  }
  int pick = first;  // a free slot, else the least recently used one
  for (int s = first; s < first + n; ++s) {
    if (slot_uid[s] == 0) {
      pick = s;
      break;
    }
    if (slot_used[s] < slot_used[pick]) pick = s;
  }
  slot_uid[pick] = st.uid;
  slot_used[pick] = slot_tick;
  st.slot = pick;
  owned = false;
  return pick;
}

bool Ctx::load(const std::string& dir, int device) {
  model_dir = dir;
  const char* q = getenv("QASR_WEIGHT_QUANT");
  bool trunc = !(q && std::string(q) == "round");
  if (!eng.load(dir, device, trunc)) return false;
  if (!tok.load(dir)) return false;
  return true;
}

void Ctx::reset_perf() {
  perf_total_ms = perf_audio_ms = perf_encode_ms = perf_decode_ms = 0;
  perf_text_tokens = 0;
  eng.perf = StagePerf();
}

bool Ctx::set_force_language(const std::string& lang) {
  if (lang.empty()) {
    force_language.clear();
    prompt_tokens_ready = false;
    return true;
  }
  std::string n = normalize_language(lang);
  if (n.empty()) return false;
  force_language = n;
  prompt_tokens_ready = false;
  return true;
}

bool Ctx::prepare_prompt_tokens() {  // context.rs:197-231
  if (prompt_tokens_ready) return true;
  has_prompt_tokens = has_force_tokens = false;
  prompt_tokens.clear();
  force_prompt_tokens.clear();
  if (!prompt.empty()) {
    if (!tok.encode(prompt, prompt_tokens)) {
      set_error("qwen: failed to encode --prompt text");
      return false;
    }
    has_prompt_tokens = true;
  }
  if (!force_language.empty()) {
    if (!tok.encode("language " + force_language, force_prompt_tokens)) {
      set_error("qwen: failed to encode --language text");
      return false;
    }
    force_prompt_tokens.push_back(kTokAsrText);
    has_force_tokens = true;
  }
  prompt_tokens_ready = true;
  return true;
}

bool Ctx::encode_window(const float* samples, size_t n, std::vector<float>& enc, int& seq) {
  int F = eng.mel(samples, (int)n, false);
  if (F <= 0) return false;
  seq = eng.encode(eng.mel_buf(), F);
  if (seq <= 0) return false;
  enc.resize((size_t)seq * eng.cfg().dec_hidden);
  return cudaMemcpy(enc.data(), eng.enc_out(), enc.size() * 4, cudaMemcpyDeviceToHost) == cudaSuccess;
}

std::vector<int> Ctx::segment_ids(int T, const std::vector<int>* past) const {
  std::vector<int> ids;
  ids.insert(ids.end(), std::begin(kPrefixHead), std::end(kPrefixHead));
  if (has_prompt_tokens) ids.insert(ids.end(), prompt_tokens.begin(), prompt_tokens.end());
  ids.insert(ids.end(), std::begin(kPrefixTail), std::end(kPrefixTail));
  for (int i = 0; i < T; ++i) ids.push_back(-(i + 1));
  ids.insert(ids.end(), std::begin(kSuffixBase), std::end(kSuffixBase));
  if (has_force_tokens) ids.insert(ids.end(), force_prompt_tokens.begin(), force_prompt_tokens.end());
  if (past && !past->empty()) {
    ids.insert(ids.end(), past->begin(), past->end());
    ids.push_back(kTokAsrText);
  }
  return ids;
}

int Ctx::segment_text(const std::vector<int>& gen, bool has_past, std::string& text) const {
  const int limit = force_n_tokens > 0 ? force_n_tokens : 2048;
  bool past_asr = has_force_tokens || has_past;
  std::string bytes;
  int processed = 0, n_text = 0;
  for (int t : gen) {
    if (processed >= limit) break;
    ++processed;
    if (force_n_tokens <= 0 && (t == kTokEndOfText || t == kTokImEnd)) break;
    if (t == kTokAsrText) {
      past_asr = true;
    } else if (past_asr) {
      bytes += tok.decode_bytes(t);
      ++n_text;
    }
  }
  text = rust_trim(utf8_lossy(bytes));
  return n_text;
}

// transcribe.rs:63-247
bool Ctx::transcribe_segment(const float* samples, size_t n, const std::vector<int>* past, std::string& text,
                             int& n_text, bool on_device) {
  double t0 = now_ms();
  n_text = 0;
  StagePerf before = eng.perf;
  int F = eng.mel(samples, (int)n, on_device);
  if (F <= 0) return false;
  int T = eng.encode(eng.mel_buf(), F);
  if (T <= 0) return false;
  if (!prepare_prompt_tokens()) return false;
  const bool has_past = past && !past->empty();
  if (!eng.prefill_ids(segment_ids(T, past), eng.enc_out(), 0)) return false;
  std::vector<int> gen;
  const int limit = force_n_tokens > 0 ? force_n_tokens : 2048;
  if (!eng.decode(limit, force_n_tokens <= 0, gen)) return false;
  n_text = segment_text(gen, has_past, text);
  last_tokens.push_back(gen);
  perf_total_ms += now_ms() - t0;
  perf_text_tokens += n_text;
  perf_encode_ms += (eng.perf.mel_ms - before.mel_ms) + (eng.perf.enc_ms - before.enc_ms);
  perf_decode_ms += (eng.perf.prefill_ms - before.prefill_ms) + (eng.perf.decode_ms - before.decode_ms);
  return true;
}

// Independent segments decoded as one batch: each segment's mel, encoder and prefill run
// into its own KV slot, then one batched greedy decode serves all of them. A segment whose
// mel or encoder yields nothing gets an empty text, as transcribe_segment's failure does
// in the sequential loop (transcribe.rs:386-398 skips it).
bool Ctx::transcribe_segments_batched(const std::vector<std::vector<float>>& segs, std::vector<std::string>& texts) {
  double t0 = now_ms();
  StagePerf before = eng.perf;
  texts.assign(segs.size(), std::string());
  std::vector<int> slot_of(segs.size(), -1);
  // one encoder pass and one prefill pass for the whole group
  std::vector<const float*> smp;
  std::vector<size_t> n;
  for (auto& s : segs) {
    smp.push_back(s.data());
    n.push_back(s.size());
  }
  std::vector<int> seq;
  if (!encode_inputs(smp, n, seq)) return false;
  std::vector<std::vector<int>> ids;
  ids.reserve(segs.size());
  std::vector<Engine::PrefillJob> jobs;
  int B = 0, base = 0;
  for (size_t i = 0; i < segs.size(); ++i) {
    if (seq[i] <= 0) continue;
    ids.push_back(segment_ids(seq[i], nullptr));
    for (int& id : ids.back())
      if (id < 0) id -= base;
    base += seq[i];
    jobs.push_back({&ids.back(), 0, B});
    slot_of[i] = B++;
  }
  if (!jobs.empty() && !eng.prefill_many(jobs, eng.enc_out())) return false;
  std::vector<std::vector<int>> gen;
  const int limit = force_n_tokens > 0 ? force_n_tokens : 2048;
  if (B > 0 && !eng.decode_batch(B, limit, force_n_tokens <= 0, gen)) return false;
  for (size_t i = 0; i < segs.size(); ++i) {
    if (slot_of[i] < 0) continue;
    perf_text_tokens += segment_text(gen[slot_of[i]], false, texts[i]);
    last_tokens.push_back(gen[slot_of[i]]);
  }
  perf_total_ms += now_ms() - t0;
  perf_encode_ms += (eng.perf.mel_ms - before.mel_ms) + (eng.perf.enc_ms - before.enc_ms);
  perf_decode_ms += (eng.perf.prefill_ms - before.prefill_ms) + (eng.perf.decode_ms - before.decode_ms);
  return true;
}

// transcribe.rs:297-426
bool Ctx::transcribe_audio(const std::vector<float>& in, std::string& result) {
  reset_perf();
  last_tokens.clear();
  perf_audio_ms = 1000.0 * (double)in.size() / kSampleRate;
  std::vector<float> audio;
  if (!skip_silence) audio = in;
  else if (!eng.compact_silence(in.data(), (long)in.size(), audio)) return false;
  if (!prepare_prompt_tokens()) return false;
  std::vector<size_t> splits = split_points(audio, segment_sec, search_sec);
  result.clear();
  if (splits.size() == 1) {
    int nt;
    return transcribe_segment(audio.data(), audio.size(), nullptr, result, nt);
  }
  const size_t min_samples = kSampleRate / 2;
  if (!past_text_conditioning && (decode_batch == 0 || decode_batch > 1)) {
    std::vector<std::pair<size_t, size_t>> bounds;
    for (size_t s = 0; s < splits.size(); ++s)
      bounds.emplace_back(splits[s], s + 1 < splits.size() ? splits[s + 1] : audio.size());
    std::vector<std::string> texts;
    if (!transcribe_segment_list(audio.data(), audio.size(), bounds, texts)) return false;
    for (const std::string& st : texts) {
      if (st.empty()) continue;
      if (!result.empty() && should_insert_boundary_space((uint8_t)result.back(), (uint8_t)st[0])) result += ' ';
      result += st;
    }
    return true;
  }
  for (size_t s = 0; s < splits.size(); ++s) {
    size_t a = splits[s], b = s + 1 < splits.size() ? splits[s + 1] : audio.size();
    std::vector<float> seg(audio.begin() + a, audio.begin() + b);
    if (seg.size() < min_samples) seg.resize(min_samples, 0.f);
    std::vector<int> past;
    bool use_past = false;
    if (past_text_conditioning && !result.empty()) use_past = tok.encode(result, past);
    std::string st;
    int nt;
    if (!transcribe_segment(seg.data(), seg.size(), use_past ? &past : nullptr, st, nt)) continue;
    if (st.empty()) continue;
    if (!result.empty() && should_insert_boundary_space((uint8_t)result.back(), (uint8_t)st[0])) result += ' ';
    result += st;
  }
  return true;
}

bool Ctx::transcribe_segment_list(const float* samples, size_t n, const std::vector<std::pair<size_t, size_t>>& bounds,
                                  std::vector<std::string>& texts) {
  if (!prepare_prompt_tokens()) return false;
  const size_t min_samples = kSampleRate / 2;
  const int batch = std::max(1, decode_batch > 0 ? std::min(decode_batch, eng.max_decode_batch()) : eng.max_decode_batch());
  texts.clear();
  for (size_t g = 0; g < bounds.size(); g += batch) {
    std::vector<std::vector<float>> group;
    for (size_t s = g; s < std::min(bounds.size(), g + batch); ++s) {
      size_t a = std::min(bounds[s].first, n), b = std::min(std::max(bounds[s].second, a), n);
      group.emplace_back(samples + a, samples + b);
      if (group.back().size() < min_samples) group.back().resize(min_samples, 0.f);
    }
    std::vector<std::string> part;
    if (!transcribe_segments_batched(group, part)) return false;
    texts.insert(texts.end(), part.begin(), part.end());
  }
  return true;
}

bool Ctx::transcribe_device(const float* d_samples, size_t n, std::string& out) {
  if (segment_sec > 0.0f || skip_silence) {
    // Segmentation and silence compaction are host algorithms: bring the samples back.
    std::vector<float> h(n);
    if (cudaMemcpy(h.data(), d_samples, n * 4, cudaMemcpyDeviceToHost) != cudaSuccess) return false;
    return transcribe_audio(h, out);
  }
  reset_perf();
  last_tokens.clear();
  perf_audio_ms = 1000.0 * (double)n / kSampleRate;
  if (!prepare_prompt_tokens()) return false;
  int nt;
  return transcribe_segment(d_samples, n, nullptr, out, nt, true);
}

// Streaming tail-repetition detector (transcribe.rs:36-55).
static std::pair<size_t, size_t> tail_repeat_blocks(const std::vector<int>& t, size_t max_period) {
  size_t n = t.size();
  if (n < 2) return {1, 0};
  size_t cap = std::min(n / 2, max_period > 0 ? max_period : n / 2);
  size_t best_reps = 1, best_p = 0;
  for (size_t p = 1; p <= cap; ++p) {
    size_t reps = 1;
    while ((reps + 1) * p <= n) {
      bool eq = std::equal(t.begin() + (n - (reps + 1) * p), t.begin() + (n - reps * p), t.begin() + (n - reps * p));
      if (!eq) break;
      ++reps;
    }
    if (reps > best_reps) {
      best_reps = reps;
      best_p = p;
    }
  }
  return {best_reps, best_p};
}

// stream_push_audio (transcribe.rs:902-1304). `samples` is the full audio so far.
// One chunk of stream_push_audio's loop (transcribe.rs:944-1304), split so that several
// streams can share one batched decode: stream_chunk_prepare does the window encodes, the
// prompt assembly, the LCP reuse and the prefill into the stream's KV slot (or, with
// defer_prefill, leaves the prefill job in `w`); the caller decodes max_new tokens in that
// slot; stream_chunk_finish turns them into the delta.
bool Ctx::stream_chunk_prepare(const std::vector<float>& samples, StreamState& st, bool finalize, StreamChunk& w,
                               bool defer_prefill) {
  if (!stream_chunk_begin(samples, st, finalize, w)) return false;
  if (!w.pending) return true;
  std::vector<EncJob*> jobs;
  for (auto& j : w.enc_jobs) jobs.push_back(&j);
  if (!run_enc_jobs(jobs)) return false;
  return stream_chunk_assemble(samples, st, w, defer_prefill);
}

// Host audio inputs through the encoder in one pass (mel per input, then encode_many):
// seq[i] = the encoder rows of input i (0 when it is too short for one mel frame or the
// encode failed); the rows of the inputs with seq > 0 follow each other in eng.enc_out().
bool Ctx::encode_inputs(const std::vector<const float*>& samples, const std::vector<size_t>& n,
                        std::vector<int>& seq) {
  seq.assign(samples.size(), 0);
  size_t frames = 0;
  for (size_t x : n) frames += x / kHop;
  if (frames == 0) return true;
  float* keep = eng.mel_scratch(frames * kMelBins);
  if (!keep) return false;
  std::vector<Engine::EncInput> in;
  std::vector<size_t> which;
  size_t off = 0;
  for (size_t i = 0; i < samples.size(); ++i) {
    if (n[i] / kHop == 0) continue;
    const int F = eng.mel(samples[i], (int)n[i], false);
    if (F <= 0) continue;
    if (cudaMemcpyAsync(keep + off, eng.mel_buf(), (size_t)F * kMelBins * 4, cudaMemcpyDeviceToDevice,
                        eng.stream()) != cudaSuccess)
      return false;
    in.push_back({keep + off, F});
    which.push_back(i);
    off += (size_t)F * kMelBins;
  }
  if (in.empty()) return true;
  std::vector<int> s;
  if (eng.encode_many(in, s) <= 0) return true;  // as failed encodes: every input falls back
  for (size_t k = 0; k < which.size(); ++k) seq[which[k]] = s[k];
  return true;
}

// Encodes the jobs' audio windows in one encoder pass; a window too short for one mel
// frame is marked failed, as encode_window fails on it.
bool Ctx::run_enc_jobs(const std::vector<EncJob*>& jobs) {
  if (jobs.empty()) return true;
  const int dim = eng.cfg().dec_hidden;
  std::vector<const float*> smp;
  std::vector<size_t> n;
  for (EncJob* j : jobs) {
    smp.push_back(j->samples);
    n.push_back(j->n);
  }
  std::vector<int> seq;
  if (!encode_inputs(smp, n, seq)) return false;
  size_t T = 0;
  for (int s : seq) T += s;
  std::vector<float> all(T * dim);
  if (T > 0 && cudaMemcpy(all.data(), eng.enc_out(), all.size() * 4, cudaMemcpyDeviceToHost) != cudaSuccess)
    return false;
  size_t row = 0;
  for (size_t i = 0; i < jobs.size(); ++i) {
    EncJob* j = jobs[i];
    j->seq = seq[i];
    j->ok = seq[i] > 0;
    j->enc.assign(all.begin() + row * dim, all.begin() + (row + seq[i]) * dim);
    row += seq[i];
  }
  return true;
}

// The part of a chunk before its window encodes: advances the audio cursor and lists the
// windows to encode (full windows the cursor crossed, then the partial window when it is
// due) in w.enc_jobs; w.pending is false when the stream has no chunk to run.
bool Ctx::stream_chunk_begin(const std::vector<float>& samples, StreamState& st, bool finalize, StreamChunk& w) {
  w = StreamChunk();
  const size_t chunk_samples = (size_t)(stream_chunk_sec * (float)kSampleRate);
  if (!st.prompt_prepared) {
    if (!prepare_prompt_tokens()) return false;
    st.prompt_prepared = true;
  }
  if (st.audio_cursor >= samples.size()) return true;
  const size_t remaining = samples.size() - st.audio_cursor;
  if (remaining < chunk_samples && !finalize) return true;
  const size_t enc_window_frames = (size_t)std::min(std::max(eng.cfg().enc_n_window_infer, 100), 800);
  const size_t enc_window_samples = enc_window_frames * kHop;

  w.pending = true;
  w.t0 = now_ms();
  st.audio_cursor = std::min(st.audio_cursor + chunk_samples, samples.size());
  w.is_final = finalize && st.audio_cursor >= samples.size();
  w.before = eng.perf;

  w.full_end = (st.audio_cursor / enc_window_samples) * enc_window_samples;
  for (size_t k = st.enc_cache_base_windows + st.enc_cache.size(); k * enc_window_samples < w.full_end; ++k) {
    EncJob j;
    j.samples = samples.data() + k * enc_window_samples;
    j.n = enc_window_samples;
    w.enc_jobs.push_back(std::move(j));
  }
  const size_t enc_update_threshold = chunk_samples * 2;
  const size_t partial_age = st.audio_cursor > st.last_partial_cursor ? st.audio_cursor - st.last_partial_cursor : 0;
  const bool need_encode = st.last_partial_cursor == 0 || partial_age >= enc_update_threshold || w.is_final;
  w.need_partial = need_encode && w.full_end < st.audio_cursor;
  if (w.need_partial) {
    EncJob j;
    j.samples = samples.data() + w.full_end;
    j.n = st.audio_cursor - w.full_end;
    w.enc_jobs.push_back(std::move(j));
  }
  return true;
}

// The rest of a chunk once its windows are encoded: caches the window outputs, assembles
// the prompt, finds the reusable prefix and prefills (or leaves the prefill job in `w`).
bool Ctx::stream_chunk_assemble(const std::vector<float>& samples, StreamState& st, StreamChunk& w,
                                bool defer_prefill) {
  const int rollback = stream_rollback, unfixed = stream_unfixed_chunks;
  const int dim = eng.cfg().dec_hidden;
  static const bool timing = getenv("QASR_STREAM_TIMING") != nullptr;  // debugging aid
  double tm[5] = {w.t0, 0, 0, 0, 0};
  (void)samples;
  size_t k = 0;
  const size_t n_full = w.enc_jobs.size() - (w.need_partial ? 1 : 0);
  for (; k < n_full; ++k) {
    EncJob& j = w.enc_jobs[k];
    if (!j.ok) {
      set_error("stream: encoding a full window failed");
      return false;
    }
    StreamState::EncWindow ew;
    ew.enc = std::move(j.enc);
    ew.seq_len = j.seq;
    st.enc_cached_seq_total += ew.seq_len;
    st.enc_cache.push_back(std::move(ew));
  }
  int partial_seq = 0;
  const std::vector<float>* partial_enc = nullptr;
  if (w.need_partial) {
    EncJob& j = w.enc_jobs[k];
    if (j.ok) {
      st.last_partial_cursor = st.audio_cursor;
      st.last_partial_enc = std::move(j.enc);
      st.last_partial_seq = j.seq;
    }
    partial_seq = st.last_partial_seq;
    partial_enc = &st.last_partial_enc;
  } else if (w.full_end < st.audio_cursor) {
    partial_seq = st.last_partial_seq;
    partial_enc = &st.last_partial_enc;
  }
  size_t enc_seq_len = st.enc_cached_seq_total + partial_seq;
  tm[1] = now_ms();
  if (enc_seq_len == 0) {  // the reference returns an empty delta here (transcribe.rs:1004-1007)
    st.chunk_idx += 1;
    w.empty_stop = true;
    return true;
  }
  std::vector<float> enc_output(enc_seq_len * dim);
  size_t off = 0;
  for (auto& ew : st.enc_cache) {
    memcpy(enc_output.data() + off * dim, ew.enc.data(), (size_t)ew.seq_len * dim * 4);
    off += ew.seq_len;
  }
  if (partial_seq > 0) memcpy(enc_output.data() + off * dim, partial_enc->data(), (size_t)partial_seq * dim * 4);

  w.n_prefix = 0;
  if (past_text_conditioning && st.chunk_idx >= unfixed && !st.raw_tokens.empty())
    w.n_prefix = (size_t)std::max((int)st.raw_tokens.size() - rollback, 0);

  std::vector<int> ids;
  ids.insert(ids.end(), std::begin(kPrefixHead), std::end(kPrefixHead));
  if (has_prompt_tokens) ids.insert(ids.end(), prompt_tokens.begin(), prompt_tokens.end());
  ids.insert(ids.end(), std::begin(kPrefixTail), std::end(kPrefixTail));
  for (size_t i = 0; i < enc_seq_len; ++i) ids.push_back(-(int)(i + 1));
  ids.insert(ids.end(), std::begin(kSuffixBase), std::end(kSuffixBase));
  if (has_force_tokens) ids.insert(ids.end(), force_prompt_tokens.begin(), force_prompt_tokens.end());
  for (size_t i = 0; i < w.n_prefix; ++i) ids.push_back(st.raw_tokens[i]);
  const size_t total_seq = ids.size(), prefill_len = total_seq - 1;

  // LCP reuse: rows equal as f32 vectors (transcribe.rs:1095-1106). Token rows compare
  // by id; encoder rows compare element-wise; a token row never equals an encoder row.
  size_t reused = 0;
  bool owned = false;
  w.slot = stream_slot(st, owned);
  if (!owned) {  // the slot's rows belong to no earlier chunk of this stream
    st.prev_ids.clear();
    st.prev_prefill_len = 0;
  }
  if (!st.prev_ids.empty() && st.prev_prefill_len > 0) {
    size_t cmp = std::min(prefill_len, st.prev_prefill_len);
    while (reused < cmp) {
      int a = st.prev_ids[reused], b = ids[reused];
      bool eq;
      if (a >= 0 || b >= 0) {
        eq = a == b;
      } else {
        const float* ra = st.prev_enc.data() + (size_t)(-a - 1) * dim;
        const float* rb = enc_output.data() + (size_t)(-b - 1) * dim;
        eq = true;
        for (int k = 0; k < dim; ++k)
          if (!(ra[k] == rb[k])) {
            eq = false;
            break;
          }
      }
      if (!eq) break;
      ++reused;
    }
  }
  tm[2] = now_ms();
  if (defer_prefill) {
    w.ids = ids;
    w.reused = (int)reused;
  } else {
    // Device copy of the assembled encoder rows for the prompt gather (grow-only buffer: a
    // free per chunk would synchronise the device).
    if (!stream_enc_dev.alloc(enc_output.size())) return false;
    if (cudaMemcpyAsync(stream_enc_dev.p, enc_output.data(), enc_output.size() * 4, cudaMemcpyHostToDevice,
                        eng.stream()) != cudaSuccess)
      return false;
    if (!eng.prefill_ids(ids, stream_enc_dev.p, (int)reused, w.slot)) return false;
  }
  tm[3] = now_ms();
  st.prev_ids.assign(ids.begin(), ids.begin() + prefill_len);
  st.prev_enc = std::move(enc_output);
  st.prev_prefill_len = prefill_len;
  w.enc = &st.prev_enc;
  tm[4] = now_ms();
  if (timing)
    fprintf(stderr, "stream chunk %d: encode %.2f ms, assemble+lcp %.2f ms, upload+prefill %.2f ms (%zu rows, %zu reused), "
            "keep %.2f ms\n", st.chunk_idx, tm[1] - tm[0], tm[2] - tm[1], tm[3] - tm[2], prefill_len, reused,
            tm[4] - tm[3]);
  w.active = true;
  return true;
}

// Returns true when the stream's loop stops after this chunk (speech ended).
bool Ctx::stream_chunk_finish(StreamState& st, StreamChunk& w, std::string& delta) {
  const int rollback = stream_rollback, unfixed = stream_unfixed_chunks;
  const int max_new = stream_max_new_tokens > 0 ? stream_max_new_tokens : 32;
  const std::vector<int>& gen = w.gen;
  const size_t n_prefix = w.n_prefix;
  const bool is_final = w.is_final;
  last_tokens.push_back(gen);
  std::vector<int> chunk_tokens;
  {
    int token_i = 0, n_generated = 0;
    while (n_generated < max_new && token_i < (int)gen.size()) {
      ++n_generated;
      int t = gen[token_i++];
      if (t == kTokEndOfText || t == kTokImEnd) break;
      chunk_tokens.push_back(t);
    }
  }

  bool speech_ended = chunk_tokens.empty() && !st.raw_tokens.empty() && st.chunk_idx >= unfixed;
  auto text_start_of = [&](const std::vector<int>& rt) -> size_t {
    if (has_force_tokens) return 0;
    auto it = std::find(rt.begin(), rt.end(), kTokAsrText);
    return it == rt.end() ? 0 : (size_t)(it - rt.begin()) + 1;
  };
  auto emit = [&](const std::vector<int>& cand, size_t from, size_t to) {
    for (size_t i = from; i < to; ++i) {
      if (i < cand.size()) {
        if (i >= st.stable_text_tokens.size()) st.stable_text_tokens.push_back(cand[i]);
        const std::string& pb = tok.decode_bytes(cand[i]);
        perf_text_tokens += 1;
        st.result_bytes += pb;
        delta += pb;
      }
    }
  };
  if (speech_ended) {
    size_t ts = text_start_of(st.raw_tokens);
    std::vector<int> cand(st.raw_tokens.begin() + ts, st.raw_tokens.end());
    emit(cand, st.stable_text_tokens.size(), cand.size());
  }
  st.raw_tokens.resize(std::min(st.raw_tokens.size(), n_prefix));
  st.raw_tokens.insert(st.raw_tokens.end(), chunk_tokens.begin(), chunk_tokens.end());

  auto reset_context = [&]() {
    size_t carry = std::min(st.stable_text_tokens.size(), kResetCarry);
    size_t cs = st.stable_text_tokens.size() - carry;
    st.raw_tokens.clear();
    if (carry > 0) {
      st.raw_tokens.push_back(kTokAsrText);
      st.raw_tokens.insert(st.raw_tokens.end(), st.stable_text_tokens.begin() + cs, st.stable_text_tokens.end());
    }
    st.prev_ids.clear();
    st.prev_enc.clear();
    st.prev_prefill_len = 0;
    st.stale_count = 0;
    st.prev_tail_snapshot.clear();
    if (st.enc_cache.size() >= kMaxEncWindows) {
      st.enc_cache_base_windows += st.enc_cache.size();
      st.enc_cache.clear();
      st.enc_cached_seq_total = 0;
    }
  };
  if (!speech_ended) {
    if (st.raw_tokens == st.prev_tail_snapshot) {
      st.stale_count += 1;
    } else {
      st.stale_count = 0;
      st.prev_tail_snapshot = st.raw_tokens;
    }
    auto rep = tail_repeat_blocks(st.raw_tokens, kDegenMaxPeriod);
    bool is_degen = st.stale_count >= kStaleChunks || rep.first >= (size_t)kDegenMinRepeats;
    if (is_degen) reset_context();
    if (st.chunk_idx > 0 && st.chunk_idx % kResetInterval == 0) reset_context();

    size_t ts = text_start_of(st.raw_tokens);
    size_t n_text_tokens = st.raw_tokens.size() > ts ? st.raw_tokens.size() - ts : 0;
    size_t candidate_len;
    if (is_final) candidate_len = n_text_tokens;
    else if (st.chunk_idx >= unfixed) candidate_len = (size_t)std::max((int)n_text_tokens - rollback, 0);
    else candidate_len = 0;
    std::vector<int> cand(st.raw_tokens.begin() + std::min(ts, st.raw_tokens.size()), st.raw_tokens.end());
    size_t from = st.stable_text_tokens.size();
    emit(cand, from, std::max(candidate_len, from));
  }
  perf_encode_ms += (eng.perf.mel_ms - w.before.mel_ms) + (eng.perf.enc_ms - w.before.enc_ms);
  perf_decode_ms += (eng.perf.prefill_ms - w.before.prefill_ms) + (eng.perf.decode_ms - w.before.decode_ms);
  perf_total_ms += now_ms() - w.t0;
  st.chunk_idx += 1;
  return speech_ended;
}

bool Ctx::stream_push_audio(const std::vector<float>& samples, StreamState& st, bool finalize, std::string& delta) {
  delta.clear();
  const int max_new = stream_max_new_tokens > 0 ? stream_max_new_tokens : 32;
  for (;;) {
    StreamChunk w;
    if (!stream_chunk_prepare(samples, st, finalize, w)) return false;
    if (w.empty_stop) {
      delta.clear();
      return true;
    }
    if (!w.active) return true;
    if (!eng.decode(max_new, true, w.gen, nullptr, nullptr, w.slot)) return false;
    if (stream_chunk_finish(st, w, delta)) break;
  }
  return true;
}

// Several streams advance together: every round, each stream with a pending chunk runs
// its prepare step, the chunks whose KV slots are contiguous decode as one batch (weights
// read once per step for all of them), then each finishes its delta. A stream's deltas
// are the ones stream_push_audio gives it alone (same prompts, same per-sequence decode).
int Ctx::stream_slot_count() const { return std::max(1, std::min(max_stream_slots, kMaxSlots - kDecodeMaxBatch)); }

// Streams beyond the number of KV slots are pushed in groups of at most that many: within a
// group every stream holds its own slot for the whole round (a slot is only ever reassigned
// to a stream of a later group), so no stream's prefill can overwrite another's rows.
bool Ctx::stream_push_many(const std::vector<const std::vector<float>*>& samples, const std::vector<StreamState*>& sts,
                           bool finalize, std::vector<std::string>& deltas) {
  const size_t n = sts.size(), g = (size_t)stream_slot_count();
  if (n <= g) return stream_push_group(samples, sts, finalize, deltas);
  deltas.assign(n, std::string());
  for (size_t i0 = 0; i0 < n; i0 += g) {
    const size_t i1 = std::min(n, i0 + g);
    std::vector<const std::vector<float>*> gs(samples.begin() + i0, samples.begin() + i1);
    std::vector<StreamState*> gt(sts.begin() + i0, sts.begin() + i1);
    std::vector<std::string> gd;
    if (!stream_push_group(gs, gt, finalize, gd)) return false;
    for (size_t i = i0; i < i1; ++i) deltas[i] = gd[i - i0];
  }
  return true;
}

bool Ctx::stream_push_group(const std::vector<const std::vector<float>*>& samples, const std::vector<StreamState*>& sts,
                            bool finalize, std::vector<std::string>& deltas) {
  const size_t n = sts.size();
  deltas.assign(n, std::string());
  const int max_new = stream_max_new_tokens > 0 ? stream_max_new_tokens : 32;
  std::vector<char> done(n, 0);
  const int max_b = std::max(1, std::min(decode_batch > 0 ? decode_batch : kDecodeMaxBatch, eng.max_decode_batch()));
  for (;;) {
    std::vector<StreamChunk> work(n);
    std::vector<size_t> act;
    // every stream's window encodes of this round in one encoder pass
    std::vector<EncJob*> jobs;
    for (size_t i = 0; i < n; ++i) {
      if (done[i]) continue;
      if (!stream_chunk_begin(*samples[i], *sts[i], finalize, work[i])) return false;
      for (auto& j : work[i].enc_jobs) jobs.push_back(&j);
    }
    if (!run_enc_jobs(jobs)) return false;
    for (size_t i = 0; i < n; ++i) {
      if (done[i]) continue;
      if (work[i].pending && !stream_chunk_assemble(*samples[i], *sts[i], work[i], true)) return false;
      if (work[i].empty_stop) {
        deltas[i].clear();
        done[i] = 1;
      } else if (!work[i].active) {
        done[i] = 1;
      } else {
        act.push_back(i);
      }
    }
    if (act.empty()) break;
    // one prefill pass for every active chunk: their encoder rows go up as one buffer and
    // each chunk's encoder ids are offset into it
    {
      size_t rows = 0;
      const int dim = eng.cfg().dec_hidden;
      for (size_t i : act) rows += work[i].enc->size() / dim;
      if (!stream_enc_dev.alloc(std::max<size_t>(rows, 1) * dim)) return false;
      std::vector<Engine::PrefillJob> jobs;
      size_t base = 0;
      for (size_t i : act) {
        StreamChunk& w = work[i];
        const size_t r = w.enc->size() / dim;
        if (r > 0 && cudaMemcpyAsync(stream_enc_dev.p + base * dim, w.enc->data(), w.enc->size() * 4,
                                     cudaMemcpyHostToDevice, eng.stream()) != cudaSuccess)
          return false;
        for (int& id : w.ids)
          if (id < 0) id -= (int)base;
        jobs.push_back({&w.ids, w.reused, w.slot});
        base += r;
      }
      if (!eng.prefill_many(jobs, stream_enc_dev.p)) return false;
    }
    std::sort(act.begin(), act.end(), [&](size_t a, size_t b) { return work[a].slot < work[b].slot; });
    for (size_t k = 0; k < act.size();) {
      size_t e = k + 1;  // a run of contiguous slots, at most max_b long
      while (e < act.size() && (int)(e - k) < max_b && work[act[e]].slot == work[act[e - 1]].slot + 1) ++e;
      const int B = (int)(e - k);
      if (B == 1) {
        if (!eng.decode(max_new, true, work[act[k]].gen, nullptr, nullptr, work[act[k]].slot)) return false;
      } else {
        std::vector<std::vector<int>> gen;
        if (!eng.decode_batch(B, max_new, true, gen, work[act[k]].slot)) return false;
        for (int b = 0; b < B; ++b) work[act[k + b]].gen = std::move(gen[b]);
      }
      k = e;
    }
    for (size_t i : act)
      if (stream_chunk_finish(*sts[i], work[i], deltas[i])) done[i] = 1;
  }
  return true;
}

// align.rs:207-351. The prompt is the transcription prompt without prompt or language
// tokens, followed by every word's tokens and two <timestamp> tokens after each word; one
// prefill gives the classify-head argmax at every <timestamp> row (align.rs:275-301).
bool Ctx::forced_align(const float* samples, size_t n, const std::string& text, const std::string& language,
                       std::vector<AlignItem>& out) {
  out.clear();
  const Config& c = eng.cfg();
  if (c.classify_num <= 0) {
    set_error("align: model is not a forced aligner (classify_num=0)");
    return false;
  }
  reset_perf();
  perf_audio_ms = 1000.0 * (double)n / kSampleRate;
  const double t0 = now_ms();
  std::vector<std::string> words;
  if (!align_split_words(text, language, words) || words.empty()) {
    set_error("align: the text has no words");
    return false;
  }
  std::vector<int> text_tokens;  // encode_timestamp (align.rs:66-93)
  for (size_t i = 0; i < words.size(); ++i) {
    std::vector<int> wt;
    if (!tok.encode(words[i], wt)) {
      set_error("align: cannot tokenize \"" + words[i] + "\"");
      return false;
    }
    text_tokens.insert(text_tokens.end(), wt.begin(), wt.end());
    text_tokens.push_back(kTokTimestamp);
    text_tokens.push_back(kTokTimestamp);
    if (i == 0 && wt.empty()) {
      set_error("align: the first word yields no tokens");
      return false;
    }
  }
  StagePerf before = eng.perf;
  const int F = eng.mel(samples, (int)n, false);
  if (F <= 0) return false;
  const int T = eng.encode(eng.mel_buf(), F);
  if (T <= 0) return false;
  std::vector<int> ids;
  ids.insert(ids.end(), std::begin(kPrefixHead), std::end(kPrefixHead));
  ids.insert(ids.end(), std::begin(kPrefixTail), std::end(kPrefixTail));
  for (int i = 0; i < T; ++i) ids.push_back(-(i + 1));
  ids.insert(ids.end(), std::begin(kSuffixBase), std::end(kSuffixBase));
  const int text_off = (int)ids.size();
  ids.insert(ids.end(), text_tokens.begin(), text_tokens.end());
  std::vector<int> rows;
  for (size_t i = 0; i < text_tokens.size(); ++i)
    if (text_tokens[i] == kTokTimestamp) rows.push_back(text_off + (int)i);
  std::vector<int> cls;
  if (!eng.prefill_classify(ids, eng.enc_out(), rows, cls)) return false;
  const float seg_time = 80.0f;  // timestamp_segment_time (config.rs:150)
  std::vector<float> ts(cls.size());
  for (size_t i = 0; i < cls.size(); ++i) ts[i] = (float)cls[i] * seg_time;
  fix_timestamps(ts);
  for (size_t i = 0; i < words.size(); ++i) {
    const float s = 2 * i < ts.size() ? ts[2 * i] : 0.0f;
    const float e = 2 * i + 1 < ts.size() ? ts[2 * i + 1] : s;
    out.push_back({words[i], s, e});
  }
  perf_total_ms += now_ms() - t0;
  perf_encode_ms += (eng.perf.mel_ms - before.mel_ms) + (eng.perf.enc_ms - before.enc_ms);
  perf_decode_ms += eng.perf.prefill_ms - before.prefill_ms;
  return true;
}

}  // namespace qasr
