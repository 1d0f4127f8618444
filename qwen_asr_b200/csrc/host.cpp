// Host-side modules. Compiled with -ffp-contract=off so that every f32 expression rounds
// the way the reference's Rust code does (Rust never contracts a*b+c into an FMA).
#include "host.h"

#include <dirent.h>
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <cmath>
#include <cstring>
#include <fstream>
#include <sstream>

#include "common.h"

namespace qasr {

int g_verbose = 0;
static thread_local std::string t_last_error;
void set_error(const std::string& msg) {
  t_last_error = msg;
  if (g_verbose >= 1) fprintf(stderr, "qwen-asr: %s\n", msg.c_str());
}
std::string last_error() { return t_last_error; }

// =====================================================================================
// safetensors (safetensors.rs:72-281): 8-byte LE header length, JSON header, raw data.
// =====================================================================================
namespace {
struct JsonCursor {
  const char* p;
  const char* e;
  void ws() {
    while (p < e && (*p == ' ' || *p == '\n' || *p == '\r' || *p == '\t')) ++p;
  }
  bool eat(char c) {
    ws();
    if (p < e && *p == c) {
      ++p;
      return true;
    }
    return false;
  }
  bool str(std::string& out) {
    ws();
    if (p >= e || *p != '"') return false;
    ++p;
    out.clear();
    while (p < e && *p != '"') {
      if (*p == '\\') {
        ++p;
        if (p >= e) return false;
        char c = *p;
        if (c == 'n') out += '\n';
        else if (c == 't') out += '\t';
        else if (c == 'r') out += '\r';
        else if (c == 'b') out += '\b';
        else if (c == 'f') out += '\f';
        else if (c == 'u') {
          if (e - p < 5) return false;
          unsigned cp = 0;
          for (int i = 1; i <= 4; ++i) {
            char h = p[i];
            cp <<= 4;
            if (h >= '0' && h <= '9') cp |= h - '0';
            else if (h >= 'a' && h <= 'f') cp |= h - 'a' + 10;
            else if (h >= 'A' && h <= 'F') cp |= h - 'A' + 10;
            else return false;
          }
          p += 5;
          // char::from_u32 rejects surrogates: the reference drops them (tokenizer.rs).
          if (cp >= 0xD800 && cp <= 0xDFFF) continue;
          if (cp < 0x80) out += (char)cp;
          else if (cp < 0x800) {
            out += (char)(0xC0 | (cp >> 6));
            out += (char)(0x80 | (cp & 0x3F));
          } else {
            out += (char)(0xE0 | (cp >> 12));
            out += (char)(0x80 | ((cp >> 6) & 0x3F));
            out += (char)(0x80 | (cp & 0x3F));
          }
          continue;
        } else out += c;
        ++p;
      } else {
        out += *p++;
      }
    }
    if (p >= e) return false;
    ++p;
    return true;
  }
  bool integer(int64_t& v) {
    ws();
    bool neg = false;
    if (p < e && *p == '-') {
      neg = true;
      ++p;
    }
    bool found = false;
    v = 0;
    while (p < e && *p >= '0' && *p <= '9') {
      v = v * 10 + (*p - '0');
      ++p;
      found = true;
    }
    if (neg) v = -v;
    return found;
  }
  // Skips any JSON value (used for __metadata__).
  bool skip() {
    ws();
    if (p >= e) return false;
    if (*p == '"') {
      std::string s;
      return str(s);
    }
    if (*p == '{' || *p == '[') {
      int depth = 0;
      bool in_str = false;
      for (; p < e; ++p) {
        char c = *p;
        if (in_str) {
          if (c == '\\') ++p;
          else if (c == '"') in_str = false;
          continue;
        }
        if (c == '"') in_str = true;
        else if (c == '{' || c == '[') ++depth;
        else if (c == '}' || c == ']') {
          if (--depth == 0) {
            ++p;
            return true;
          }
        }
      }
      return false;
    }
    while (p < e && *p != ',' && *p != '}' && *p != ']') ++p;
    return true;
  }
};
}  // namespace

bool parse_safetensors_header(const char* json, size_t len, const uint8_t* data_base, size_t data_size,
                              std::unordered_map<std::string, TensorInfo>& out) {
  JsonCursor c{json, json + len};
  if (!c.eat('{')) return false;
  while (true) {
    c.ws();
    if (c.p >= c.e) return false;
    if (*c.p == '}') break;
    if (*c.p == ',') {
      ++c.p;
      continue;
    }
    std::string name;
    if (!c.str(name) || !c.eat(':')) return false;
    if (name == "__metadata__") {
      if (!c.skip()) return false;
      continue;
    }
    if (!c.eat('{')) return false;
    TensorInfo ti;
    int64_t off0 = -1, off1 = -1;
    while (true) {
      c.ws();
      if (c.p >= c.e) return false;
      if (*c.p == '}') {
        ++c.p;
        break;
      }
      if (*c.p == ',') {
        ++c.p;
        continue;
      }
      std::string key;
      if (!c.str(key) || !c.eat(':')) return false;
      if (key == "dtype") {
        if (!c.str(ti.dtype)) return false;
      } else if (key == "shape" || key == "data_offsets") {
        if (!c.eat('[')) return false;
        std::vector<int64_t> vals;
        while (true) {
          c.ws();
          if (c.p < c.e && *c.p == ']') {
            ++c.p;
            break;
          }
          if (c.p < c.e && *c.p == ',') {
            ++c.p;
            continue;
          }
          int64_t v;
          if (!c.integer(v)) return false;
          vals.push_back(v);
        }
        if (key == "shape") ti.shape = vals;
        else if (vals.size() == 2) {
          off0 = vals[0];
          off1 = vals[1];
        } else return false;
      } else if (!c.skip()) {
        return false;
      }
    }
    if (off0 < 0 || off1 < off0 || (size_t)off1 > data_size) return false;
    ti.data = data_base + off0;
    ti.nbytes = (size_t)(off1 - off0);
    size_t esz = ti.dtype == "F32" || ti.dtype == "I32" ? 4 : ti.dtype == "BF16" || ti.dtype == "F16" ? 2
               : ti.dtype == "I64" ? 8 : 1;
    if (ti.numel() * esz != ti.nbytes) return false;
    out.emplace(name, ti);
  }
  return true;
}

SafeTensors::~SafeTensors() {
  for (auto& m : maps_)
    if (m.base) munmap(m.base, m.size);
}

bool SafeTensors::open_file(const std::string& path) {
  int fd = ::open(path.c_str(), O_RDONLY);
  if (fd < 0) return false;
  struct stat sb;
  if (fstat(fd, &sb) != 0 || sb.st_size < 8) {
    ::close(fd);
    return false;
  }
  size_t size = (size_t)sb.st_size;
  void* base = mmap(nullptr, size, PROT_READ, MAP_PRIVATE, fd, 0);
  ::close(fd);
  if (base == MAP_FAILED) return false;
  maps_.push_back({base, size});
  const uint8_t* b = (const uint8_t*)base;
  uint64_t hlen = 0;
  memcpy(&hlen, b, 8);
  if (hlen > size - 8) {
    set_error("safetensors: header length exceeds file size in " + path);
    return false;
  }
  std::unordered_map<std::string, TensorInfo> m;
  if (!parse_safetensors_header((const char*)b + 8, (size_t)hlen, b + 8 + hlen, size - 8 - hlen, m)) {
    set_error("safetensors: malformed header in " + path);
    return false;
  }
  shards_.push_back(std::move(m));
  return true;
}

bool SafeTensors::open(const std::string& dir) {
  std::string single = dir + "/model.safetensors";
  struct stat sb;
  if (stat(single.c_str(), &sb) == 0) return open_file(single);
  std::vector<std::string> names;
  if (DIR* d = opendir(dir.c_str())) {
    while (dirent* de = readdir(d)) {
      std::string n = de->d_name;
      if (n.rfind("model-", 0) == 0 && n.size() > 12 && n.substr(n.size() - 12) == ".safetensors")
        names.push_back(n);
    }
    closedir(d);
  }
  if (names.empty()) {
    set_error("no safetensors files in " + dir);
    return false;
  }
  std::sort(names.begin(), names.end());
  for (auto& n : names)
    if (!open_file(dir + "/" + n)) {
      if (last_error().empty()) set_error("failed to open " + dir + "/" + n);
      return false;
    }
  return true;
}

const TensorInfo* SafeTensors::find(const std::string& name) const {
  for (auto& s : shards_) {
    auto it = s.find(name);
    if (it != s.end()) return &it->second;
  }
  return nullptr;
}

// =====================================================================================
// Config detection (config.rs:110-157) + shape inference extension.
// =====================================================================================
bool detect_config(const SafeTensors& st, Config& c) {
  c = Config();
  bool has18 = st.has("thinker.audio_tower.layers.18.self_attn.q_proj.weight");
  auto emb = st.find("thinker.model.embed_tokens.weight");
  auto gate = st.find("thinker.model.layers.0.mlp.gate_proj.weight");
  c.dec_hidden = (emb && emb->shape.size() == 2) ? (int)emb->shape[1] : (has18 ? 2048 : 1024);
  c.dec_intermediate = (gate && gate->shape.size() == 2) ? (int)gate->shape[0] : (c.dec_hidden >= 2048 ? 6144 : 3072);
  if (has18) {
    c.enc_d_model = 1024; c.enc_layers = 24; c.enc_heads = 16; c.enc_ffn_dim = 4096;
  } else {
    c.enc_d_model = 896; c.enc_layers = 18; c.enc_heads = 14; c.enc_ffn_dim = 3584;
  }
  // Shape inference: identical to the presets for the published checkpoints.
  if (auto co = st.find("thinker.audio_tower.conv_out.weight")) {
    c.enc_d_model = (int)co->shape[0];
    c.enc_heads = c.enc_d_model / 64;
  }
  int n = 0;
  while (st.has("thinker.audio_tower.layers." + std::to_string(n) + ".self_attn.q_proj.weight")) ++n;
  c.enc_layers = n;
  if (auto f1 = st.find("thinker.audio_tower.layers.0.fc1.weight")) c.enc_ffn_dim = (int)f1->shape[0];
  n = 0;
  while (st.has("thinker.model.layers." + std::to_string(n) + ".self_attn.q_proj.weight")) ++n;
  c.dec_layers = n;
  auto q = st.find("thinker.model.layers.0.self_attn.q_proj.weight");
  auto k = st.find("thinker.model.layers.0.self_attn.k_proj.weight");
  if (!q || !k || !emb || c.enc_layers == 0 || c.dec_layers == 0) {
    set_error("model: missing core tensors (embed_tokens / q_proj / k_proj / encoder layers)");
    return false;
  }
  c.dec_heads = (int)q->shape[0] / 128;
  c.dec_kv_heads = (int)k->shape[0] / 128;
  c.enc_output_dim = c.dec_hidden;
  c.enc_chunk_size = c.enc_n_window * 2;
  if (auto lm = st.find("thinker.lm_head.weight"))
    if (lm->shape.size() == 2 && lm->shape[0] != kVocab) c.classify_num = (int)lm->shape[0];
  return true;
}

static const char* kLanguages[] = {
    "Chinese", "English", "Cantonese", "Arabic", "German", "French", "Spanish", "Portuguese",
    "Indonesian", "Italian", "Korean", "Russian", "Thai", "Vietnamese", "Japanese", "Turkish",
    "Hindi", "Malay", "Dutch", "Swedish", "Danish", "Finnish", "Polish", "Czech", "Filipino",
    "Persian", "Greek", "Romanian", "Hungarian", "Macedonian"};

std::string normalize_language(const std::string& lang) {
  std::string t = rust_trim(lang);
  if (t.empty()) return "";
  // All supported names are ASCII; non-ASCII input can never match.
  for (unsigned char ch : t)
    if (ch >= 0x80) return "";
  std::string norm = t;
  norm[0] = (char)toupper((unsigned char)norm[0]);
  for (size_t i = 1; i < norm.size(); ++i) norm[i] = (char)tolower((unsigned char)norm[i]);
  for (auto l : kLanguages)
    if (norm == l) return norm;
  return "";
}

// =====================================================================================
// Tokenizer (tokenizer.rs)
// =====================================================================================
static void utf8_append(std::string& s, unsigned cp) {
  if (cp < 0x80) s += (char)cp;
  else if (cp < 0x800) {
    s += (char)(0xC0 | (cp >> 6));
    s += (char)(0x80 | (cp & 0x3F));
  } else if (cp < 0x10000) {
    s += (char)(0xE0 | (cp >> 12));
    s += (char)(0x80 | ((cp >> 6) & 0x3F));
    s += (char)(0x80 | (cp & 0x3F));
  } else {
    s += (char)(0xF0 | (cp >> 18));
    s += (char)(0x80 | ((cp >> 12) & 0x3F));
    s += (char)(0x80 | ((cp >> 6) & 0x3F));
    s += (char)(0x80 | (cp & 0x3F));
  }
}

// Decodes valid UTF-8 into code points (inputs here are valid by construction).
static std::vector<unsigned> utf8_cps(const std::string& s) {
  std::vector<unsigned> out;
  for (size_t i = 0; i < s.size();) {
    unsigned char b = (unsigned char)s[i];
    unsigned cp;
    int len;
    if (b < 0x80) { cp = b; len = 1; }
    else if ((b & 0xE0) == 0xC0) { cp = b & 0x1F; len = 2; }
    else if ((b & 0xF0) == 0xE0) { cp = b & 0x0F; len = 3; }
    else { cp = b & 0x07; len = 4; }
    for (int k = 1; k < len && i + k < s.size(); ++k) cp = (cp << 6) | ((unsigned char)s[i + k] & 0x3F);
    out.push_back(cp);
    i += len;
  }
  return out;
}

bool Tokenizer::load(const std::string& model_dir) {
  int n = 0;
  int u2b[512];
  for (int i = 0; i < 512; ++i) u2b[i] = -1;
  for (int b = 0; b < 256; ++b) {
    bool normal = (b >= 33 && b <= 126) || (b >= 161 && b <= 172) || (b >= 174 && b <= 255);
    byte_to_cp_[b] = normal ? b : 256 + n++;
  }
  for (int b = 0; b < 256; ++b) u2b[byte_to_cp_[b]] = b;

  std::ifstream f(model_dir + "/vocab.json", std::ios::binary);
  if (!f) {
    set_error("tokenizer: cannot read " + model_dir + "/vocab.json");
    return false;
  }
  std::stringstream ss;
  ss << f.rdbuf();
  std::string json = ss.str();
  JsonCursor c{json.data(), json.data() + json.size()};
  if (!c.eat('{')) {
    set_error("tokenizer: vocab.json is not an object");
    return false;
  }
  std::vector<std::pair<std::string, int>> entries;
  int max_id = 0;
  while (true) {
    c.ws();
    if (c.p >= c.e || *c.p == '}') break;
    if (*c.p == ',') {
      ++c.p;
      continue;
    }
    std::string key;
    int64_t id;
    if (!c.str(key) || !c.eat(':') || !c.integer(id)) {
      set_error("tokenizer: malformed vocab.json");
      return false;
    }
    if (id > max_id) max_id = (int)id;
    entries.emplace_back(key, (int)id);
  }
  id_bytes_.assign(max_id + 1, std::string());
  vocab_.clear();
  vocab_.reserve(entries.size() * 2);
  for (auto& kv : entries) {
    if (kv.second < 0) continue;
    std::string raw;
    for (unsigned cp : utf8_cps(kv.first)) raw += (cp < 512 && u2b[cp] >= 0) ? (char)u2b[cp] : '?';
    id_bytes_[kv.second] = raw;
    vocab_[kv.first] = kv.second;
  }
  merges_.clear();
  std::ifstream mf(model_dir + "/merges.txt", std::ios::binary);
  if (mf) {
    std::string line;
    int rank = 0;
    while (std::getline(mf, line)) {
      while (!line.empty() && (line.back() == '\r' || line.back() == ' ' || line.back() == '\t' ||
                               line.back() == '\n'))
        line.pop_back();
      if (line.empty() || line[0] == '#') continue;
      size_t sp = line.find(' ');
      if (sp == std::string::npos) continue;
      std::string a = line.substr(0, sp);
      size_t bpos = sp + 1;
      while (bpos < line.size() && (line[bpos] == ' ' || line[bpos] == '\t')) ++bpos;
      std::string b = line.substr(bpos);
      if (!a.empty() && !b.empty()) merges_[a + " " + b] = rank++;
    }
  }
  return true;
}

const std::string& Tokenizer::decode_bytes(int id) const {
  if (id < 0 || id >= (int)id_bytes_.size()) return empty_;
  return id_bytes_[id];
}

bool Tokenizer::encode(const std::string& text, std::vector<int>& ids) const {
  ids.clear();
  if (text.empty()) return false;
  std::vector<std::string> syms;
  for (unsigned char b : text) {
    std::string s;
    utf8_append(s, (unsigned)byte_to_cp_[b]);
    syms.push_back(s);
  }
  while (syms.size() > 1) {
    int best_rank = INT32_MAX, best_i = -1;
    for (size_t i = 0; i + 1 < syms.size(); ++i) {
      auto it = merges_.find(syms[i] + " " + syms[i + 1]);
      if (it != merges_.end() && it->second < best_rank) {
        best_rank = it->second;
        best_i = (int)i;
      }
    }
    if (best_i < 0) break;
    syms[best_i] += syms[best_i + 1];
    syms.erase(syms.begin() + best_i + 1);
  }
  for (auto& s : syms) {
    auto it = vocab_.find(s);
    if (it == vocab_.end()) return false;
    ids.push_back(it->second);
  }
  return true;
}

// =====================================================================================
// Audio (audio.rs)
// =====================================================================================
bool parse_wav_buffer(const uint8_t* d, size_t len, std::vector<float>& out) {
  int rate = 0;
  if (!parse_wav_native(d, len, out, rate)) return false;
  if (rate != kSampleRate) out = resample(out, rate, kSampleRate);
  return true;
}

bool parse_wav_native(const uint8_t* d, size_t len, std::vector<float>& out, int& rate_out) {
  if (len < 44 || memcmp(d, "RIFF", 4) != 0 || memcmp(d + 8, "WAVE", 4) != 0) {
    set_error("parse_wav_buffer: not a valid WAV file");
    return false;
  }
  auto u16 = [&](size_t o) { return (unsigned)d[o] | ((unsigned)d[o + 1] << 8); };
  auto u32 = [&](size_t o) { return (uint32_t)d[o] | ((uint32_t)d[o + 1] << 8) | ((uint32_t)d[o + 2] << 16) | ((uint32_t)d[o + 3] << 24); };
  int channels = 0, rate = 0, bits = 0, fmt = 0;
  const uint8_t* pcm = nullptr;
  size_t pcm_len = 0;
  size_t p = 12;
  while (p + 8 <= len) {
    size_t csz = u32(p + 4);
    if (p + 8 + csz > len) break;
    if (memcmp(d + p, "fmt ", 4) == 0 && csz >= 16) {
      fmt = (int)u16(p + 8);
      channels = (int)u16(p + 10);
      rate = (int)u32(p + 12);
      bits = (int)u16(p + 22);
    } else if (memcmp(d + p, "data", 4) == 0) {
      pcm = d + p + 8;
      pcm_len = std::min(csz, len - (p + 8));
    }
    p += 8 + csz;
    if (csz & 1) p += 1;
  }
  if (fmt != 1 || bits != 16 || channels < 1) {
    set_error("parse_wav_buffer: unsupported format (need 16-bit PCM)");
    return false;
  }
  if (!pcm) {
    set_error("parse_wav_buffer: no data chunk");
    return false;
  }
  size_t nf = pcm_len / ((size_t)channels * 2);
  out.assign(nf, 0.f);
  for (size_t i = 0; i < nf; ++i) {
    if (channels == 1) {
      int16_t v = (int16_t)u16(i * 2 + (pcm - d));
      out[i] = (float)v / 32768.0f;
    } else {
      float sum = 0.f;
      for (int ch = 0; ch < channels; ++ch) {
        int16_t v = (int16_t)u16((i * channels + ch) * 2 + (pcm - d));
        sum += (float)v;
      }
      out[i] = (sum / (float)channels) / 32768.0f;
    }
  }
  rate_out = rate;
  return true;
}

std::vector<float> resample(const std::vector<float>& in, int from_rate, int to_rate) {
  size_t n = in.size();
  size_t new_n = (size_t)((int64_t)n * to_rate / from_rate);
  std::vector<float> out(new_n, 0.f);
  const int sinc_half = 16;
  const double beta = 6.0;
  double ratio = (double)to_rate / (double)from_rate;
  double cutoff = ratio < 1.0 ? ratio : 1.0;
  auto i0 = [](double x) {
    double sum = 1.0, term = 1.0, xx = x * x;
    for (int k = 1; k <= 20; ++k) {
      term *= xx / (4.0 * (double)k * (double)k);
      sum += term;
    }
    return sum;
  };
  double inv_i0b = 1.0 / i0(beta);
  for (size_t i = 0; i < new_n; ++i) {
    double src_pos = (double)i / ratio;
    int center = (int)src_pos;
    double acc = 0.0, wsum = 0.0;
    for (int j = center - sinc_half + 1; j <= center + sinc_half; ++j) {
      double dd = (double)j - src_pos;
      double x = dd * cutoff;
      double s = std::fabs(x) < 1e-9 ? 1.0 : std::sin(M_PI * x) / (M_PI * x);
      double npos = dd / (double)sinc_half;
      double w = (npos <= -1.0 || npos >= 1.0) ? 0.0 : i0(beta * std::sqrt(1.0 - npos * npos)) * inv_i0b;
      double coeff = s * w * cutoff;
      if (j >= 0 && (size_t)j < n) acc += (double)in[j] * coeff;
      wsum += coeff;
    }
    out[i] = wsum > 1e-9 ? (float)(acc / wsum) : 0.f;
  }
  return out;
}

std::vector<float> compact_silence(const std::vector<float>& x) {
  size_t n = x.size();
  if (n == 0) return {};
  const size_t win = 160;
  const float base_thresh = 0.002f, max_thresh = 0.025f, alpha = 0.2f;
  size_t n_win = (n + win - 1) / win;
  std::vector<float> rms(n_win), smooth(n_win);
  for (size_t w = 0; w < n_win; ++w) {
    size_t a = w * win, b = std::min(a + win, n);
    float e = 0.f;
    for (size_t i = a; i < b; ++i) e += x[i] * x[i];
    rms[w] = std::sqrt(e / (float)std::max<size_t>(b - a, 1));
  }
  float s = rms[0];
  for (size_t w = 0; w < n_win; ++w) {
    s = (1.0f - alpha) * s + alpha * rms[w];
    smooth[w] = s;
  }
  std::vector<float> sorted = smooth;
  std::sort(sorted.begin(), sorted.end());
  size_t p25 = (size_t)((float)(n_win - 1) * 0.25f);
  float thresh = std::min(std::max(sorted[p25] * 1.8f, base_thresh), max_thresh);
  std::vector<char> voice(n_win), pv(n_win, 0);
  for (size_t w = 0; w < n_win; ++w) voice[w] = smooth[w] > thresh;
  for (size_t i = 0; i < n_win;) {
    if (!voice[i]) {
      ++i;
      continue;
    }
    size_t j = i + 1;
    while (j < n_win && voice[j]) ++j;
    if (j - i < 5)
      for (size_t k = i; k < j; ++k) voice[k] = 0;
    i = j;
  }
  for (size_t w = 0; w < n_win; ++w) {
    if (!voice[w]) continue;
    size_t a = w >= 3 ? w - 3 : 0, b = std::min(w + 3, n_win - 1);
    for (size_t k = a; k <= b; ++k) pv[k] = 1;
  }
  std::vector<float> out;
  out.reserve(n);
  int silence = 0;
  for (size_t w = 0; w < n_win; ++w) {
    size_t a = w * win, b = std::min(a + win, n);
    if (pv[w]) {
      out.insert(out.end(), x.begin() + a, x.begin() + b);
      silence = 0;
    } else if (++silence <= 60) {
      out.insert(out.end(), x.begin() + a, x.begin() + b);
    }
  }
  if (out.empty()) out.assign(x.begin(), x.begin() + std::min<size_t>(n, kSampleRate / 2));
  return out;
}

size_t find_split_point(const float* x, size_t n, size_t target, float search_sec) {
  size_t half = (size_t)(search_sec * (float)kSampleRate);
  size_t lo = target >= half ? target - half : 0;
  size_t hi = std::min(target + half, n);
  const size_t win = 1600;
  float best_e = 1e30f;
  size_t best_c = target;
  for (size_t pos = lo; pos + win <= hi; pos += win / 2) {
    size_t end = std::min(pos + win, n);
    float e = 0.f;
    for (size_t i = pos; i < end; ++i) e += x[i] * x[i];
    e /= (float)(end - pos);
    if (e < best_e) {
      best_e = e;
      best_c = pos + (end - pos) / 2;
    }
  }
  return best_c;
}

std::vector<size_t> split_points(const std::vector<float>& x, float segment_sec, float search_sec) {
  size_t target = segment_sec > 0 ? (size_t)(segment_sec * (float)kSampleRate) : 0;
  float search = std::min(search_sec, segment_sec / 2.0f);
  size_t margin = search > 0 ? (size_t)(search * (float)kSampleRate) : 0;
  if (segment_sec <= 0.0f || x.size() <= target + margin) return {0};
  std::vector<size_t> splits{0};
  size_t pos = 0;
  while (pos + target + margin < x.size()) {
    size_t sp = find_split_point(x.data(), x.size(), pos + target, search);
    splits.push_back(sp);
    pos = sp;
    if (splits.size() >= 127) break;
  }
  return splits;
}

static bool rust_ws_byte(uint8_t b) {
  return b == 0x09 || b == 0x0A || b == 0x0B || b == 0x0C || b == 0x0D || b == 0x20 || b == 0x85 || b == 0xA0;
}

bool should_insert_boundary_space(uint8_t prev, uint8_t next) {
  if (prev == 0 || next == 0) return false;
  if (rust_ws_byte(prev) || rust_ws_byte(next)) return false;
  if (next >= 33 && next <= 126 && !isalnum(next)) return false;
  return true;
}

std::string utf8_lossy(const std::string& s) {
  std::string out;
  out.reserve(s.size());
  const unsigned char* b = (const unsigned char*)s.data();
  size_t n = s.size(), i = 0;
  static const char kRepl[] = "\xEF\xBF\xBD";
  while (i < n) {
    unsigned c = b[i];
    if (c < 0x80) {
      out += (char)c;
      ++i;
      continue;
    }
    int len;
    unsigned lo = 0x80, hi = 0xBF;
    if (c >= 0xC2 && c <= 0xDF) len = 2;
    else if (c == 0xE0) { len = 3; lo = 0xA0; }
    else if (c >= 0xE1 && c <= 0xEC) len = 3;
    else if (c == 0xED) { len = 3; hi = 0x9F; }
    else if (c >= 0xEE && c <= 0xEF) len = 3;
    else if (c == 0xF0) { len = 4; lo = 0x90; }
    else if (c >= 0xF1 && c <= 0xF3) len = 4;
    else if (c == 0xF4) { len = 4; hi = 0x8F; }
    else {
      out += kRepl;
      ++i;
      continue;
    }
    int k = 1;
    bool ok = true;
    for (; k < len; ++k) {
      if (i + k >= n) {
        ok = false;
        break;
      }
      unsigned t = b[i + k];
      unsigned l = k == 1 ? lo : 0x80, h = k == 1 ? hi : 0xBF;
      if (t < l || t > h) {
        ok = false;
        break;
      }
    }
    if (ok) {
      out.append((const char*)b + i, len);
      i += len;
    } else {
      out += kRepl;
      i += k;
    }
  }
  return out;
}

static bool is_white_space_cp(unsigned cp) {
  return (cp >= 0x09 && cp <= 0x0D) || cp == 0x20 || cp == 0x85 || cp == 0xA0 || cp == 0x1680 ||
         (cp >= 0x2000 && cp <= 0x200A) || cp == 0x2028 || cp == 0x2029 || cp == 0x202F || cp == 0x205F ||
         cp == 0x3000;
}

std::string rust_trim(const std::string& s) {
  // Works on valid UTF-8; walks code points from both ends.
  size_t a = 0, b = s.size();
  while (a < b) {
    unsigned char c = (unsigned char)s[a];
    int len = c < 0x80 ? 1 : (c & 0xE0) == 0xC0 ? 2 : (c & 0xF0) == 0xE0 ? 3 : 4;
    if (a + len > b) break;
    auto cps = utf8_cps(s.substr(a, len));
    if (cps.empty() || !is_white_space_cp(cps[0])) break;
    a += len;
  }
  while (b > a) {
    size_t st = b - 1;
    while (st > a && ((unsigned char)s[st] & 0xC0) == 0x80) --st;
    auto cps = utf8_cps(s.substr(st, b - st));
    if (cps.empty() || !is_white_space_cp(cps[0])) break;
    b = st;
  }
  return s.substr(a, b - a);
}

// =====================================================================================
// Forced aligner host steps (align.rs).
// =====================================================================================
bool align_split_words(const std::string& text, const std::string& language, std::vector<std::string>& words) {
  words.clear();
  const bool cjk = language == "Chinese" || language == "Japanese" || language == "Korean" || language == "Cantonese";
  std::string cur;
  size_t i = 0;
  while (i < text.size()) {
    const unsigned char c = (unsigned char)text[i];
    const size_t len = c < 0x80 ? 1 : (c & 0xE0) == 0xC0 ? 2 : (c & 0xF0) == 0xE0 ? 3 : (c & 0xF8) == 0xF0 ? 4 : 0;
    if (len == 0 || i + len > text.size()) return false;
    const std::string ch = text.substr(i, len);
    const auto cps = utf8_cps(ch);
    if (cps.size() != 1) return false;
    const bool ws = is_white_space_cp(cps[0]);
    if (cjk) {
      if (!ws) words.push_back(ch);  // text.chars().filter(!whitespace) (align.rs:51-55)
    } else if (ws) {  // split_whitespace (align.rs:57-60)
      if (!cur.empty()) words.push_back(cur);
      cur.clear();
    } else {
      cur += ch;
    }
    i += len;
  }
  if (!cur.empty()) words.push_back(cur);
  return true;
}

// align.rs:97-137: O(n^2) DP over "vals[j] <= vals[i]", the first longest end, traced back.
std::vector<size_t> longest_increasing_subsequence(const std::vector<float>& v) {
  const size_t n = v.size();
  if (n == 0) return {};
  const size_t none = (size_t)-1;
  std::vector<size_t> dp(n, 1), prev(n, none);
  for (size_t i = 1; i < n; ++i)
    for (size_t j = 0; j < i; ++j)
      if (v[j] <= v[i] && dp[j] + 1 > dp[i]) {
        dp[i] = dp[j] + 1;
        prev[i] = j;
      }
  size_t best_len = 0, best_end = 0;
  for (size_t i = 0; i < n; ++i)
    if (dp[i] > best_len) {
      best_len = dp[i];
      best_end = i;
    }
  std::vector<size_t> out;
  for (size_t idx = best_end;; idx = prev[idx]) {
    out.push_back(idx);
    if (prev[idx] == none) break;
  }
  std::reverse(out.begin(), out.end());
  return out;
}

// align.rs:140-189: entries off the longest non-decreasing subsequence are repaired, blocks
// of <= 2 with the nearest normal value, longer blocks by linear interpolation.
void fix_timestamps(std::vector<float>& ts) {
  const size_t n = ts.size();
  if (n <= 1) return;
  const auto lis = longest_increasing_subsequence(ts);
  if (lis.size() == n) return;
  std::vector<char> normal(n, 0);
  for (size_t i : lis) normal[i] = 1;
  size_t i = 0;
  while (i < n) {
    if (normal[i]) {
      ++i;
      continue;
    }
    const size_t bs = i;
    while (i < n && !normal[i]) ++i;
    const size_t be = i, bl = be - bs;
    const float left = bs > 0 ? ts[bs - 1] : 0.0f;
    const float right = be < n ? ts[be] : left + (float)bl * 80.0f;
    if (bl <= 2) {
      const float fill = bs > 0 ? left : right;
      for (size_t k = bs; k < be; ++k) ts[k] = fill;
    } else {
      for (size_t j = 0; j < bl; ++j) {
        const float t = (float)(j + 1) / (float)(bl + 1);
        ts[bs + j] = left + t * (right - left);
      }
    }
  }
}

// =====================================================================================
// Tables shared with the device, computed with the reference's f32 formulas.
// =====================================================================================
static float hz_to_mel(float f) {
  const float min_log_hz = 1000.0f, min_log_mel = 15.0f;
  const float logstep = 27.0f / logf(6.4f);
  float mels = 3.0f * f / 200.0f;
  return f >= min_log_hz ? min_log_mel + logf(f / min_log_hz) * logstep : mels;
}
static float mel_to_hz(float m) {
  const float min_log_hz = 1000.0f, min_log_mel = 15.0f;
  const float logstep = logf(6.4f) / 27.0f;
  return m >= min_log_mel ? min_log_hz * expf(logstep * (m - min_log_mel)) : 200.0f * m / 3.0f;
}

void build_mel_filters(std::vector<float>& filt) {
  filt.assign(kMelBins * kNfreq, 0.f);
  std::vector<float> fft_freqs(kNfreq), ff(kMelBins + 2), diff(kMelBins + 1);
  for (int i = 0; i < kNfreq; ++i) fft_freqs[i] = (float)i * ((float)kSampleRate / 2.0f) / (float)(kNfreq - 1);
  float mel_min = hz_to_mel(0.0f), mel_max = hz_to_mel((float)kSampleRate / 2.0f);
  for (int i = 0; i < kMelBins + 2; ++i)
    ff[i] = mel_to_hz(mel_min + (mel_max - mel_min) * (float)i / (float)(kMelBins + 1));
  for (int i = 0; i < kMelBins + 1; ++i) {
    diff[i] = ff[i + 1] - ff[i];
    if (diff[i] == 0.0f) diff[i] = 1e-6f;
  }
  for (int m = 0; m < kMelBins; ++m) {
    float enorm = 2.0f / (ff[m + 2] - ff[m]);
    for (int f = 0; f < kNfreq; ++f) {
      float down = (fft_freqs[f] - ff[m]) / diff[m];
      float up = (ff[m + 2] - fft_freqs[f]) / diff[m + 1];
      float v = std::max(std::min(down, up), 0.0f);
      filt[m * kNfreq + f] = v * enorm;
    }
  }
}

void build_hann(std::vector<float>& w) {
  w.resize(kNfft);
  const float pi = 3.14159265358979323846f;
  for (int i = 0; i < kNfft; ++i) w[i] = 0.5f * (1.0f - cosf(2.0f * pi * (float)i / (float)kNfft));
}

void build_dft_tables(std::vector<float>& ct, std::vector<float>& st) {
  ct.resize(kNfreq * kNfft);
  st.resize(kNfreq * kNfft);
  const float pi = 3.14159265358979323846f;
  for (int k = 0; k < kNfreq; ++k)
    for (int n = 0; n < kNfft; ++n) {
      float ang = 2.0f * pi * (float)k * (float)n / (float)kNfft;
      ct[k * kNfft + n] = cosf(ang);
      st[k * kNfft + n] = sinf(ang);
    }
}

void build_rope_tables(int n_pos, int hd, float theta, std::vector<float>& ct, std::vector<float>& st) {
  int half = hd / 2;
  std::vector<float> inv(half);
  for (int d = 0; d < half; ++d) inv[d] = 1.0f / powf(theta, (float)(2 * d) / (float)hd);
  ct.resize((size_t)n_pos * half);
  st.resize((size_t)n_pos * half);
  for (int p = 0; p < n_pos; ++p)
    for (int d = 0; d < half; ++d) {
      float ang = (float)p * inv[d];
      ct[(size_t)p * half + d] = cosf(ang);
      st[(size_t)p * half + d] = sinf(ang);
    }
}

void build_sinusoidal_pe(int n_pos, int d, std::vector<float>& pe) {
  int half = d / 2;
  float log_ts = logf(10000.0f) / (float)(half - 1);
  pe.assign((size_t)n_pos * d, 0.f);
  for (int p = 0; p < n_pos; ++p)
    for (int i = 0; i < half; ++i) {
      float inv_ts = expf(-(float)i * log_ts);
      float ang = (float)p * inv_ts;
      pe[(size_t)p * d + i] = sinf(ang);
      pe[(size_t)p * d + half + i] = cosf(ang);
    }
}

}  // namespace qasr
