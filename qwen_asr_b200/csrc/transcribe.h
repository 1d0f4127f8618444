// Transcription orchestration over one Engine: the QwenCtx settings
// (crates/qwen-asr/src/context.rs:26-162) and transcribe.rs's offline, segmented and
// streaming algorithms.
#pragma once
#include <memory>
#include <string>
#include <vector>

#include "engine.h"
#include "host.h"

namespace qasr {

struct StreamState {  // transcribe.rs:801-893
  struct EncWindow {
    int seq_len;
    std::vector<float> enc;
  };
  std::vector<EncWindow> enc_cache;
  size_t enc_cached_seq_total = 0, enc_cache_base_windows = 0;
  std::vector<int> raw_tokens, stable_text_tokens;
  std::string result_bytes;
  // previous prefill rows: token id (>= 0) or encoder row (< 0 -> index into prev_enc)
  std::vector<int> prev_ids;
  std::vector<float> prev_enc;
  size_t prev_prefill_len = 0;
  std::vector<int> prev_tail_snapshot;
  int stale_count = 0;
  size_t last_partial_cursor = 0;
  std::vector<float> last_partial_enc;
  int last_partial_seq = 0;
  size_t audio_cursor = 0;
  int chunk_idx = 0;
  bool prompt_prepared = false;
  // Device KV slot of this stream (assigned by the engine context on first use) and a
  // process-unique id that proves ownership of it: a reset or a new stream gets a new id.
  int slot = -1;
  uint64_t uid = next_uid();
  void reset();
  static uint64_t next_uid();
};

// One chunk of a stream in flight between its prepare and finish steps.
// One audio window of a stream chunk to encode (host samples), and its encoder output.
struct EncJob {
  const float* samples = nullptr;
  size_t n = 0;
  bool ok = false;
  int seq = 0;
  std::vector<float> enc;
};

struct StreamChunk {
  bool active = false;      // prefilled, waiting for its decode
  bool empty_stop = false;  // nothing encoded yet: the push ends with an empty delta
  bool is_final = false;
  int slot = -1;
  size_t n_prefix = 0;
  double t0 = 0;
  StagePerf before;
  std::vector<int> gen;
  // deferred prefill (stream_push_many prefills all streams' chunks in one pass): the
  // prompt ids (encoder rows as -(r+1) into *enc), the reused LCP length
  std::vector<int> ids;
  int reused = 0;
  const std::vector<float>* enc = nullptr;  // window encodes of the chunk (full windows, then the partial window when due)
  bool pending = false;
  bool need_partial = false;
  size_t full_end = 0;
  std::vector<EncJob> enc_jobs;
};

class Ctx {
 public:
  Engine eng;
  std::string model_dir;
  Tokenizer tok;
  // settings (context.rs:133-162)
  float segment_sec = 0.0f, search_sec = 3.0f;
  float stream_chunk_sec = 2.0f;
  int stream_rollback = 5, stream_unfixed_chunks = 2, stream_max_new_tokens = 32;
  bool past_text_conditioning = false, skip_silence = false;
  std::string prompt, force_language;
  int force_n_tokens = 0;          // benchmark extension: exactly N decode steps, EOS ignored
  // Segments of one transcribe_audio call decoded together (one weight read per step for
  // all of them); 0 = the engine's largest batch, 1 = one segment at a time. Only used
  // when past-text conditioning is off (the segments are then independent).
  int decode_batch = 0;
  // Streams keep their prompt rows in their own KV slots (kDecodeMaxBatch..): slot_uid[s]
  // is the id of the stream whose rows slot s holds, slot_used[s] its last-use tick (LRU).
  int max_stream_slots = 32;
  DevBuf<float> stream_enc_dev;  // encoder rows of the chunk being prefilled
  std::vector<uint64_t> slot_uid, slot_used;
  uint64_t slot_tick = 0;
  // Returns the stream's slot; `owned` is false when the slot was (re)assigned, so its KV
  // rows are not the stream's and the prefill starts from scratch.
  int stream_slot(StreamState& st, bool& owned);
  // prompt tokens
  std::vector<int> prompt_tokens, force_prompt_tokens;
  bool has_prompt_tokens = false, has_force_tokens = false, prompt_tokens_ready = false;
  // perf (context.rs:67-73)
  double perf_total_ms = 0, perf_audio_ms = 0, perf_encode_ms = 0, perf_decode_ms = 0;
  int perf_text_tokens = 0;
  std::vector<std::vector<int>> last_tokens;  // generated ids per segment / chunk of the last call

  bool load(const std::string& dir, int device);
  bool set_force_language(const std::string& lang);
  void set_prompt(const std::string& p) {
    prompt = p;
    prompt_tokens_ready = false;
  }
  bool prepare_prompt_tokens();
  bool transcribe_audio(const std::vector<float>& samples, std::string& out);
  // Offline transcription of samples already resident in device memory.
  bool transcribe_device(const float* d_samples, size_t n, std::string& out);
  bool transcribe_segment(const float* samples, size_t n, const std::vector<int>* past, std::string& text,
                          int& n_text, bool on_device = false);
  bool stream_push_audio(const std::vector<float>& samples, StreamState& st, bool finalize, std::string& delta);
  bool stream_push_many(const std::vector<const std::vector<float>*>& samples, const std::vector<StreamState*>& sts,
                        bool finalize, std::vector<std::string>& deltas);
  // Streams whose KV slots can be held at once (slots kDecodeMaxBatch.. of the engine).
  int stream_slot_count() const;
  bool stream_push_group(const std::vector<const std::vector<float>*>& samples, const std::vector<StreamState*>& sts,
                         bool finalize, std::vector<std::string>& deltas);
  bool stream_chunk_prepare(const std::vector<float>& samples, StreamState& st, bool finalize, StreamChunk& w,
                            bool defer_prefill = false);
  bool stream_chunk_begin(const std::vector<float>& samples, StreamState& st, bool finalize, StreamChunk& w);
  bool encode_inputs(const std::vector<const float*>& samples, const std::vector<size_t>& n, std::vector<int>& seq);
  bool run_enc_jobs(const std::vector<EncJob*>& jobs);
  bool stream_chunk_assemble(const std::vector<float>& samples, StreamState& st, StreamChunk& w, bool defer_prefill);
  bool stream_chunk_finish(StreamState& st, StreamChunk& w, std::string& delta);
  void reset_perf();
  // Forced alignment (align.rs:207-351): one unit (word, or character for CJK languages) per
  // entry with its start/end in ms; false (with the error set) when the model is not an
  // aligner, the text has no unit or encoding fails.
  struct AlignItem {
    std::string text;
    float start_ms, end_ms;
  };
  bool forced_align(const float* samples, size_t n, const std::string& text, const std::string& language,
                    std::vector<AlignItem>& out);
  // Transcribes the independent segments [starts[i], ends[i]) of `samples` (each padded to
  // 0.5 s as transcribe.rs:374-384 does), batching their decodes; texts[i] per segment.
  bool transcribe_segment_list(const float* samples, size_t n, const std::vector<std::pair<size_t, size_t>>& bounds,
                               std::vector<std::string>& texts);

 private:
  bool encode_window(const float* samples, size_t n, std::vector<float>& enc, int& seq);
  // Prompt ids of one segment (transcribe.rs:110-150): chat prefix, optional user prompt,
  // T encoder rows (ids -1..-T), assistant prefix, forced language, past text.
  std::vector<int> segment_ids(int T, const std::vector<int>* past) const;
  // Generated ids -> text (transcribe.rs:194-247); returns the text-token count.
  int segment_text(const std::vector<int>& gen, bool has_past, std::string& text) const;
  bool transcribe_segments_batched(const std::vector<std::vector<float>>& segs, std::vector<std::string>& texts);
};

}  // namespace qasr
