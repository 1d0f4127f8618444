// Host-side modules: safetensors reader, model config, tokenizer, audio front end and
// segmentation helpers. Pure C++17; no CUDA types.
#pragma once
#include <cstdint>
#include <map>
#include <string>
#include <unordered_map>
#include <vector>

namespace qasr {

// ---------------------------------------------------------------- safetensors
// mmap reader with multi-shard lookup (crates/qwen-asr/src/safetensors.rs:72-281).
struct TensorInfo {
  std::string dtype;  // "BF16", "F32", ...
  std::vector<int64_t> shape;
  const uint8_t* data = nullptr;
  size_t nbytes = 0;
  size_t numel() const {
    size_t n = 1;
    for (auto d : shape) n *= (size_t)d;
    return n;
  }
};

class SafeTensors {
 public:
  ~SafeTensors();
  // Opens <dir>/model.safetensors, else every <dir>/model-*.safetensors in sorted order.
  bool open(const std::string& dir);
  const TensorInfo* find(const std::string& name) const;
  bool has(const std::string& name) const { return find(name) != nullptr; }

 private:
  struct Map {
    void* base = nullptr;
    size_t size = 0;
  };
  std::vector<Map> maps_;
  std::vector<std::unordered_map<std::string, TensorInfo>> shards_;
  bool open_file(const std::string& path);
};

// Parses a safetensors JSON header into `out` (exposed for tests of malformed input).
bool parse_safetensors_header(const char* json, size_t len, const uint8_t* data_base, size_t data_size,
                              std::unordered_map<std::string, TensorInfo>& out);

// ---------------------------------------------------------------- config
// QwenConfig (config.rs:27-157) plus shape inference for non-published sizes.
struct Config {
  int enc_d_model = 0, enc_layers = 0, enc_heads = 0, enc_head_dim = 64, enc_ffn_dim = 0;
  int enc_output_dim = 0, enc_n_window = 50, enc_n_window_infer = 800, enc_chunk_size = 100;
  int dec_hidden = 0, dec_layers = 28, dec_heads = 16, dec_kv_heads = 8, dec_head_dim = 128;
  int dec_intermediate = 0, vocab_size = 151936;
  float dec_rms_norm_eps = 1e-6f, dec_rope_theta = 1e6f;
  int classify_num = 0;
};
bool detect_config(const SafeTensors& st, Config& cfg);
// config.rs:167-182: returns "" when unsupported.
std::string normalize_language(const std::string& lang);

// ---------------------------------------------------------------- tokenizer
// GPT-2 byte-level BPE (tokenizer.rs).
class Tokenizer {
 public:
  bool load(const std::string& model_dir);
  const std::string& decode_bytes(int id) const;  // raw bytes, possibly partial UTF-8
  // Whole-string BPE; returns false when a symbol is missing (tokenizer.rs:227-279).
  bool encode(const std::string& text, std::vector<int>& ids) const;
  int vocab_size() const { return (int)id_bytes_.size(); }

 private:
  std::vector<std::string> id_bytes_;
  std::unordered_map<std::string, int> vocab_;
  std::unordered_map<std::string, int> merges_;
  int byte_to_cp_[256];
  std::string empty_;
};

// ---------------------------------------------------------------- audio
bool parse_wav_buffer(const uint8_t* data, size_t len, std::vector<float>& out);
// The same parse without the resampling step: mono samples at the file's own rate.
bool parse_wav_native(const uint8_t* data, size_t len, std::vector<float>& out, int& rate);
std::vector<float> resample(const std::vector<float>& in, int from_rate, int to_rate);
std::vector<float> compact_silence(const std::vector<float>& in);
// Segment start offsets of transcribe_audio (transcribe.rs:328-346); {0} when unsplit.
std::vector<size_t> split_points(const std::vector<float>& samples, float segment_sec, float search_sec);
size_t find_split_point(const float* samples, size_t n, size_t target, float search_sec);
bool should_insert_boundary_space(uint8_t prev, uint8_t next);
// Rust str::trim (Unicode White_Space) and String::from_utf8_lossy.
std::string utf8_lossy(const std::string& bytes);
std::string rust_trim(const std::string& s);
// Forced-aligner host steps (align.rs:44-61, 96-189): the units of `text` (CJK languages:
// every non-white-space character; others: white-space separated words; false on invalid
// UTF-8), the longest non-decreasing subsequence, and the timestamp repair.
bool align_split_words(const std::string& text, const std::string& language, std::vector<std::string>& words);
std::vector<size_t> longest_increasing_subsequence(const std::vector<float>& v);
void fix_timestamps(std::vector<float>& ts);

// Host tables shared with the device (built with the reference's f32 formulas).
void build_mel_filters(std::vector<float>& filt);           // [128][201]  audio.rs:202-262
void build_hann(std::vector<float>& w);                     // [400]       audio.rs:305-311
void build_dft_tables(std::vector<float>& cos_t, std::vector<float>& sin_t);  // [201][400]
void build_rope_tables(int n_pos, int head_dim, float theta, std::vector<float>& cos_t,
                       std::vector<float>& sin_t);          // [n_pos][head_dim/2] decoder.rs:302-338
void build_sinusoidal_pe(int n_pos, int d, std::vector<float>& pe);  // kernels/mod.rs:1704-1716

}  // namespace qasr
