// Engine: weight upload, mel / encoder / prefill / decode stages on one GPU.
#include "engine.h"

#include <algorithm>
#include <cmath>
#include <cstring>

namespace qasr {

Engine::~Engine() {
  if (device_ >= 0) cudaSetDevice(device_);
  for (auto& g : graph_exec_)
    if (g) cudaGraphExecDestroy(g);
  for (auto& g : slot_graph_)
    if (g) cudaGraphExecDestroy(g);
  for (auto& kv : run_graphs_)
    if (kv.second.first) cudaGraphExecDestroy(kv.second.first);
  for (void* p : allocs_) cudaFree(p);
  if (hstate_) cudaFreeHost(hstate_);
  if (htokens_) cudaFreeHost(htokens_);
  if (ev0_) cudaEventDestroy(ev0_);
  if (ev1_) cudaEventDestroy(ev1_);
  if (stream_) cudaStreamDestroy(stream_);
}

void* Engine::dalloc(size_t bytes) {
  void* p = nullptr;
  if (cudaMalloc(&p, std::max<size_t>(bytes, 16)) != cudaSuccess) {
    set_error("cudaMalloc failed (" + std::to_string(bytes) + " bytes)");
    return nullptr;
  }
  allocs_.push_back(p);
  return p;
}

namespace {
// Host conversion of any float tensor (F32 or BF16) to f32.
bool tensor_f32(const SafeTensors& st, const std::string& name, std::vector<float>& out) {
  const TensorInfo* t = st.find(name);
  if (!t) {
    set_error("weight not found: " + name);
    return false;
  }
  size_t n = t->numel();
  out.resize(n);
  if (t->dtype == "F32") {
    memcpy(out.data(), t->data, n * 4);
  } else if (t->dtype == "BF16") {
    const uint16_t* s = (const uint16_t*)t->data;
    for (size_t i = 0; i < n; ++i) {
      uint32_t b = (uint32_t)s[i] << 16;
      memcpy(&out[i], &b, 4);
    }
  } else {
    set_error("unsupported dtype for " + name + ": " + t->dtype);
    return false;
  }
  return true;
}

const uint16_t* tensor_bf16(const SafeTensors& st, const std::string& name, size_t expect) {
  const TensorInfo* t = st.find(name);
  if (!t) {
    set_error("weight not found: " + name);
    return nullptr;
  }
  if (t->dtype != "BF16") {
    set_error(name + ": expected BF16, got " + t->dtype);
    return nullptr;
  }
  if (expect && t->numel() != expect) {
    set_error(name + ": unexpected shape");
    return nullptr;
  }
  return (const uint16_t*)t->data;
}
}  // namespace

bool Engine::load(const std::string& dir, int device, bool trunc_quant) {
  device_ = device;
  // Validate the model files before touching the GPU.
  SafeTensors st;
  if (!st.open(dir)) return false;
  if (!detect_config(st, cfg_)) return false;
  CUDA_OK(cudaSetDevice(device), false);
  decode_kernels_init();

  enc_kernels_init();
  CUDA_OK(cudaStreamCreateWithFlags(&stream_, cudaStreamNonBlocking), false);
  CUDA_OK(cudaEventCreate(&ev0_), false);
  CUDA_OK(cudaEventCreate(&ev1_), false);
  const Config& c = cfg_;
  if (c.dec_head_dim != 128 || c.enc_head_dim != 64 || c.dec_heads % c.dec_kv_heads != 0 ||
      c.dec_heads / c.dec_kv_heads > 4) {
    set_error("unsupported model geometry");
    return false;
  }
  QASR_LOG(1, "Detected: Qwen3-ASR (enc %dd %dL, dec %dd %dL, inter %d)\n", c.enc_d_model, c.enc_layers,
           c.dec_hidden, c.dec_layers, c.dec_intermediate);

  std::vector<float> f;
  auto up_f32 = [&](const std::string& name, float*& dst) -> bool {
    if (!tensor_f32(st, name, f)) return false;
    dst = dalloc_t<float>(f.size());
    return dst && cudaMemcpy(dst, f.data(), f.size() * 4, cudaMemcpyHostToDevice) == cudaSuccess;
  };
  auto up_bf16 = [&](const std::string& name, __nv_bfloat16*& dst, size_t n) -> bool {
    const uint16_t* p = tensor_bf16(st, name, n);
    if (!p) return false;
    dst = dalloc_t<__nv_bfloat16>(n);
    return dst && cudaMemcpy(dst, p, n * 2, cudaMemcpyHostToDevice) == cudaSuccess;
  };
  // Concatenates bf16 tensors row-wise into one device matrix.
  auto up_cat = [&](const std::vector<std::string>& names, size_t per_row, __nv_bfloat16*& dst) -> bool {
    size_t total = 0;
    std::vector<const TensorInfo*> ts;
    for (auto& n : names) {
      const TensorInfo* t = st.find(n);
      if (!t || t->dtype != "BF16") {
        set_error("missing/non-bf16 weight: " + n);
        return false;
      }
      if (t->numel() % per_row) {
        set_error("bad shape: " + n);
        return false;
      }
      ts.push_back(t);
      total += t->numel();
    }
    dst = dalloc_t<__nv_bfloat16>(total);
    if (!dst) return false;
    size_t off = 0;
    for (auto t : ts) {
      if (cudaMemcpy(dst + off, t->data, t->nbytes, cudaMemcpyHostToDevice) != cudaSuccess) return false;
      off += t->numel();
    }
    return true;
  };
  auto cat_f32 = [&](const std::vector<std::string>& names, float*& dst) -> bool {
    std::vector<float> all;
    for (auto& n : names) {
      if (!tensor_f32(st, n, f)) return false;
      all.insert(all.end(), f.begin(), f.end());
    }
    dst = dalloc_t<float>(all.size());
    return dst && cudaMemcpy(dst, all.data(), all.size() * 4, cudaMemcpyHostToDevice) == cudaSuccess;
  };

  const std::string p = "thinker.audio_tower.";
  const int d = c.enc_d_model, H = kConvHidden;
  // conv2d1 [480][1][3][3] -> f32 [480][9]
  if (!up_f32(p + "conv2d1.weight", conv1_w) || !up_f32(p + "conv2d1.bias", conv1_b)) return false;
  // conv2d2/3 [oc][ic][3][3] -> bf16 [oc][(ki*3+kj)*480 + ic] (im2col column order)
  for (int li = 2; li <= 3; ++li) {
    const uint16_t* w = tensor_bf16(st, p + "conv2d" + std::to_string(li) + ".weight", (size_t)H * H * 9);
    if (!w) return false;
    std::vector<uint16_t> perm((size_t)H * H * 9);
    for (int oc = 0; oc < H; ++oc)
      for (int ic = 0; ic < H; ++ic)
        for (int kk = 0; kk < 9; ++kk) perm[(size_t)oc * H * 9 + kk * H + ic] = w[((size_t)oc * H + ic) * 9 + kk];
    __nv_bfloat16*& dst = li == 2 ? conv2_w : conv3_w;
    dst = dalloc_t<__nv_bfloat16>(perm.size());
    if (!dst) return false;
    CUDA_OK(cudaMemcpy(dst, perm.data(), perm.size() * 2, cudaMemcpyHostToDevice), false);
    if (!up_f32(p + "conv2d" + std::to_string(li) + ".bias", li == 2 ? conv2_b : conv3_b)) return false;
  }
  {  // conv_out [d][ch*16 + f] -> [d][f*480 + ch] (matches the channels-last conv3 output)
    const uint16_t* w = tensor_bf16(st, p + "conv_out.weight", (size_t)d * H * 16);
    if (!w) return false;
    std::vector<uint16_t> perm((size_t)d * H * 16);
    for (int o = 0; o < d; ++o)
      for (int ch = 0; ch < H; ++ch)
        for (int fr = 0; fr < 16; ++fr) perm[(size_t)o * H * 16 + fr * H + ch] = w[(size_t)o * H * 16 + ch * 16 + fr];
    conv_out_w = dalloc_t<__nv_bfloat16>(perm.size());
    if (!conv_out_w) return false;
    CUDA_OK(cudaMemcpy(conv_out_w, perm.data(), perm.size() * 2, cudaMemcpyHostToDevice), false);
  }
  enc_layers_.resize(c.enc_layers);
  for (int i = 0; i < c.enc_layers; ++i) {
    std::string lp = p + "layers." + std::to_string(i) + ".";
    EncLayerW& L = enc_layers_[i];
    if (!up_cat({lp + "self_attn.q_proj.weight", lp + "self_attn.k_proj.weight", lp + "self_attn.v_proj.weight"}, d,
                L.wqkv) ||
        !cat_f32({lp + "self_attn.q_proj.bias", lp + "self_attn.k_proj.bias", lp + "self_attn.v_proj.bias"}, L.bqkv) ||
        !up_bf16(lp + "self_attn.out_proj.weight", L.wo, (size_t)d * d) ||
        !up_f32(lp + "self_attn.out_proj.bias", L.bo) || !up_f32(lp + "self_attn_layer_norm.weight", L.ln1w) ||
        !up_f32(lp + "self_attn_layer_norm.bias", L.ln1b) ||
        !up_bf16(lp + "fc1.weight", L.w1, (size_t)c.enc_ffn_dim * d) || !up_f32(lp + "fc1.bias", L.b1) ||
        !up_bf16(lp + "fc2.weight", L.w2, (size_t)c.enc_ffn_dim * d) || !up_f32(lp + "fc2.bias", L.b2) ||
        !up_f32(lp + "final_layer_norm.weight", L.ln2w) || !up_f32(lp + "final_layer_norm.bias", L.ln2b))
      return false;
  }
  if (!up_f32(p + "ln_post.weight", ln_post_w) || !up_f32(p + "ln_post.bias", ln_post_b) ||
      !up_bf16(p + "proj1.weight", proj1_w, (size_t)d * d) || !up_f32(p + "proj1.bias", proj1_b) ||
      !up_bf16(p + "proj2.weight", proj2_w, (size_t)c.enc_output_dim * d) || !up_f32(p + "proj2.bias", proj2_b))
    return false;

  // ---- decoder
  const std::string m = "thinker.model.";
  const int h = c.dec_hidden, qd = c.dec_heads * 128, kvd = c.dec_kv_heads * 128, inter = c.dec_intermediate;
  if (!up_bf16(m + "embed_tokens.weight", embed_, (size_t)c.vocab_size * h)) return false;
  dec_layers_.resize(c.dec_layers);
  std::vector<uint16_t> gu((size_t)2 * inter * h);
  for (int i = 0; i < c.dec_layers; ++i) {
    std::string lp = m + "layers." + std::to_string(i) + ".";
    DecLayerW& L = dec_layers_[i];
    if (!up_cat({lp + "self_attn.q_proj.weight", lp + "self_attn.k_proj.weight", lp + "self_attn.v_proj.weight"}, h,
                L.wqkv) ||
        !up_bf16(lp + "self_attn.o_proj.weight", L.wo, (size_t)h * qd) ||
        !up_bf16(lp + "mlp.down_proj.weight", L.wdown, (size_t)h * inter) ||
        !up_f32(lp + "self_attn.q_norm.weight", L.qn) || !up_f32(lp + "self_attn.k_norm.weight", L.kn) ||
        !up_f32(lp + "input_layernorm.weight", L.n1) || !up_f32(lp + "post_attention_layernorm.weight", L.n2))
      return false;
    const uint16_t* g = tensor_bf16(st, lp + "mlp.gate_proj.weight", (size_t)inter * h);
    const uint16_t* u = tensor_bf16(st, lp + "mlp.up_proj.weight", (size_t)inter * h);
    if (!g || !u) return false;
    for (int r = 0; r < inter; ++r) {
      memcpy(&gu[(size_t)(2 * r) * h], g + (size_t)r * h, h * 2);
      memcpy(&gu[(size_t)(2 * r + 1) * h], u + (size_t)r * h, h * 2);
    }
    L.wgu = dalloc_t<__nv_bfloat16>(gu.size());
    if (!L.wgu) return false;
    CUDA_OK(cudaMemcpy(L.wgu, gu.data(), gu.size() * 2, cudaMemcpyHostToDevice), false);
    // int8 decode weights, quantised on the device from the bf16 copies (decoder.rs:106-118)
    struct Q {
      const __nv_bfloat16* w;
      int rows, cols;
      int8_t** q;
      float** s;
    } qs[] = {{L.wqkv, qd + 2 * kvd, h, &L.qqkv, &L.sqkv},
              {L.wo, h, qd, &L.qo, &L.so},
              {L.wgu, 2 * inter, h, &L.qgu, &L.sgu},
              {L.wdown, h, inter, &L.qdown, &L.sdown}};
    for (auto& e : qs) {
      *e.q = dalloc_t<int8_t>((size_t)e.rows * e.cols);
      *e.s = dalloc_t<float>(e.rows);
      if (!*e.q || !*e.s) return false;
      quantize_rows_int8(e.w, e.rows, e.cols, trunc_quant, *e.q, *e.s, stream_);
    }
  }
  if (!up_f32(m + "norm.weight", final_norm_)) return false;
  // Tied lm_head unless thinker.lm_head.weight exists (decoder.rs:145-151).
  if (st.has("thinker.lm_head.weight")) {
    __nv_bfloat16* lm = nullptr;
    int rows = c.classify_num > 0 ? c.classify_num : c.vocab_size;
    if (!up_bf16("thinker.lm_head.weight", lm, (size_t)rows * h)) return false;
    lm_bf16_ = lm;
  } else {
    lm_bf16_ = embed_;
  }
  {
    int rows = c.classify_num > 0 ? c.classify_num : c.vocab_size;
    lm_q_ = dalloc_t<int8_t>((size_t)rows * h);
    lm_s_ = dalloc_t<float>(rows);
    if (!lm_q_ || !lm_s_) return false;
    quantize_rows_int8(lm_bf16_, rows, h, trunc_quant, lm_q_, lm_s_, stream_);
  }

  // ---- tables
  std::vector<float> t1, t2;
  build_hann(t1);
  hann_ = dalloc_t<float>(t1.size());
  CUDA_OK(cudaMemcpy(hann_, t1.data(), t1.size() * 4, cudaMemcpyHostToDevice), false);
  build_dft_tables(t1, t2);  // B matrix [408][400]: rows 0..200 cos, 201..401 sin, rest 0
  {
    std::vector<float> B((size_t)408 * kNfft, 0.f);
    memcpy(B.data(), t1.data(), t1.size() * 4);
    memcpy(B.data() + (size_t)kNfreq * kNfft, t2.data(), t2.size() * 4);
    dft_ = dalloc_t<float>(B.size());
    CUDA_OK(cudaMemcpy(dft_, B.data(), B.size() * 4, cudaMemcpyHostToDevice), false);
  }
  build_mel_filters(t1);  // [128][201] -> padded [128][208]
  {
    std::vector<float> B((size_t)kMelBins * 208, 0.f);
    for (int r = 0; r < kMelBins; ++r) memcpy(&B[(size_t)r * 208], &t1[(size_t)r * kNfreq], kNfreq * 4);
    mel_filt_ = dalloc_t<float>(B.size());
    CUDA_OK(cudaMemcpy(mel_filt_, B.data(), B.size() * 4, cudaMemcpyHostToDevice), false);
  }
  // Per-chunk sinusoidal PE (positions restart at 0 in every 100-frame chunk).
  build_sinusoidal_pe(64, d, t1);
  pe_ = dalloc_t<float>(t1.size());
  CUDA_OK(cudaMemcpy(pe_, t1.data(), t1.size() * 4, cudaMemcpyHostToDevice), false);

  // ---- decode state
  if (!ensure_kv(4096)) return false;
  CUDA_OK(cudaMallocHost(&hstate_, kMaxSlots * sizeof(StepState)), false);
  const int mb = kDecodeMaxBatch;
  if (!dx_.alloc((size_t)kMaxSlots * h) || !dqkv_.alloc((size_t)mb * (qd + 2 * kvd)) || !dattn_.alloc((size_t)mb * qd) ||
      !dffn_.alloc((size_t)mb * inter) || !dpart_.alloc((size_t)c.dec_heads * 16 * 130) ||
      !dticket_.alloc(c.dec_kv_heads) || !dam_ticket_.alloc(1) || !dam_part_.alloc((size_t)mb * 1024) ||
      !dstate_.alloc(kMaxSlots) || !dlogits_.alloc(c.vocab_size) || !derr_.alloc(1) ||
      !dstaged_.alloc(decode_staged_bytes(h, qd, inter)))
    return false;
  CUDA_OK(cudaMemset(dticket_.p, 0, c.dec_kv_heads * sizeof(int)), false);
  CUDA_OK(cudaMemset(dam_ticket_.p, 0, sizeof(int)), false);
  CUDA_OK(cudaMemset(derr_.p, 0, sizeof(int)), false);
  for (auto& L : dec_layers_) {
    pn1_.push_back(L.n1);
    pn2_.push_back(L.n2);
    pqn_.push_back(L.qn);
    pkn_.push_back(L.kn);
  }
  CUDA_OK(cudaStreamSynchronize(stream_), false);
  CUDA_OK(cudaGetLastError(), false);
  return true;
}

bool Engine::ensure_kv(int needed) {
  const Config& c = cfg_;
  if (needed <= max_seq_ && rope_cap_ >= max_seq_) return true;
  int nm = max_seq_ > 0 ? max_seq_ : 2048;
  while (nm < needed) nm *= 2;
  size_t per = (size_t)slots_ * c.dec_layers * c.dec_kv_heads * nm * 128;
  float *nk = nullptr, *nv = nullptr;
  CUDA_OK(cudaMalloc(&nk, per * 4), false);
  CUDA_OK(cudaMalloc(&nv, per * 4), false);
  if (kc_.p && max_seq_ > 0) {
    // copy every (slot, layer, head) row run into the wider layout (decoder.rs:199-231)
    size_t rows = (size_t)slots_ * c.dec_layers * c.dec_kv_heads;
    size_t used = (size_t)(slots_ > 1 ? max_seq_ : kv_len_) * 128 * 4;
    if (used > 0) {
      CUDA_OK(cudaMemcpy2DAsync(nk, (size_t)nm * 128 * 4, kc_.p, (size_t)max_seq_ * 128 * 4, used, rows,
                                cudaMemcpyDeviceToDevice, stream_),
              false);
      CUDA_OK(cudaMemcpy2DAsync(nv, (size_t)nm * 128 * 4, vc_.p, (size_t)max_seq_ * 128 * 4, used, rows,
                                cudaMemcpyDeviceToDevice, stream_),
              false);
      CUDA_OK(cudaStreamSynchronize(stream_), false);
    }
  }
  kc_.release();
  vc_.release();
  kc_.p = nk;
  kc_.n = per;
  vc_.p = nv;
  vc_.n = per;
  max_seq_ = nm;
  std::vector<float> rc, rs;
  build_rope_tables(nm, 128, c.dec_rope_theta, rc, rs);
  if (rope_cos_) {
    cudaFree(rope_cos_);
    cudaFree(rope_sin_);
    allocs_.erase(std::remove(allocs_.begin(), allocs_.end(), (void*)rope_cos_), allocs_.end());
    allocs_.erase(std::remove(allocs_.begin(), allocs_.end(), (void*)rope_sin_), allocs_.end());
  }
  rope_cos_ = dalloc_t<float>(rc.size());
  rope_sin_ = dalloc_t<float>(rs.size());
  if (!rope_cos_ || !rope_sin_) return false;
  CUDA_OK(cudaMemcpy(rope_cos_, rc.data(), rc.size() * 4, cudaMemcpyHostToDevice), false);
  CUDA_OK(cudaMemcpy(rope_sin_, rs.data(), rs.size() * 4, cudaMemcpyHostToDevice), false);
  rope_cap_ = nm;
  ++graph_gen_;
  return true;
}

bool Engine::ensure_slots(int n) {
  if (n <= slots_) return true;
  const size_t old = (size_t)slots_ * kv_slot_stride(), per = (size_t)n * kv_slot_stride();
  float *nk = nullptr, *nv = nullptr;
  CUDA_OK(cudaMalloc(&nk, per * 4), false);
  if (cudaMalloc(&nv, per * 4) != cudaSuccess) {
    cudaFree(nk);
    set_error("cudaMalloc failed for the KV cache slots");
    return false;
  }
  CUDA_OK(cudaMemcpyAsync(nk, kc_.p, old * 4, cudaMemcpyDeviceToDevice, stream_), false);
  CUDA_OK(cudaMemcpyAsync(nv, vc_.p, old * 4, cudaMemcpyDeviceToDevice, stream_), false);
  CUDA_OK(cudaStreamSynchronize(stream_), false);
  kc_.release();
  vc_.release();
  kc_.p = nk;
  kc_.n = per;
  vc_.p = nv;
  vc_.n = per;
  slots_ = n;
  ++graph_gen_;
  return true;
}

// ---------------------------------------------------------------------------- mel
int Engine::mel(const float* samples, int n, bool on_device) {
  cudaSetDevice(device_);
  int n_frames = n / kHop;  // (n + 400 - 400) / 160 + 1 - 1  (audio.rs:293-294)
  if (n <= 0 || n_frames <= 0) {
    set_error("mel_spectrogram: audio too short (" + std::to_string(n) + " samples)");
    return 0;
  }
  const float* dsamp = samples;
  if (!on_device) {
    if (!samples_.alloc(n)) return 0;
    CUDA_OK(cudaMemcpyAsync(samples_.p, samples, (size_t)n * 4, cudaMemcpyHostToDevice, stream_), 0);
    dsamp = samples_.p;
  }
  if (!frames_.alloc((size_t)n_frames * kNfft) || !spec_.alloc((size_t)n_frames * 408) ||
      !power_.alloc((size_t)n_frames * 208) || !mel_.alloc((size_t)n_frames * kMelBins) || !gmax_.alloc(1))
    return 0;
  cudaEventRecord(ev0_, stream_);
  launches += 6;
  mel_frames(dsamp, n, n_frames, hann_, frames_.p, stream_);
  GemmArgs g;
  g.M = n_frames; g.N = 408; g.K = kNfft;
  g.A = frames_.p; g.lda = kNfft; g.B = dft_; g.b_is_f32 = true; g.ldb = kNfft;
  g.C = spec_.p; g.ldc = 408;
  gemm_simt(g, stream_);
  mel_power(spec_.p, 408, n_frames, power_.p, 208, stream_);
  mel_reset_max(gmax_.p, stream_);
  GemmArgs g2;
  g2.M = n_frames; g2.N = kMelBins; g2.K = 208;
  g2.A = power_.p; g2.lda = 208; g2.B = mel_filt_; g2.b_is_f32 = true; g2.ldb = 208;
  g2.C = mel_.p; g2.ldc = kMelBins; g2.epi = EPI_LOG10_MAX; g2.gmax = gmax_.p;
  gemm_simt(g2, stream_);
  mel_normalize(mel_.p, n_frames, gmax_.p, stream_);
  cudaEventRecord(ev1_, stream_);
  CUDA_OK(cudaEventSynchronize(ev1_), 0);
  float ms = 0;
  cudaEventElapsedTime(&ms, ev0_, ev1_);
  perf.mel_ms += ms;
  CUDA_OK(cudaGetLastError(), 0);
  return n_frames;
}

// ---------------------------------------------------------------------------- encoder
float* Engine::mel_scratch(size_t floats) { return mel_keep_.alloc(floats) ? mel_keep_.p : nullptr; }

int Engine::encode(const float* d_mel, int F) {
  std::vector<int> seq;
  return encode_many({{d_mel, F}}, seq);
}

// Several inputs (mel matrices) through the encoder in one pass: each input's conv front
// end fills its rows of x_enc, the attention windows restart at every input's first row,
// and every transformer layer runs once over all rows. Rows depend only on their own
// input, so each equals the single-input encode bit for bit.
int Engine::encode_many(const std::vector<EncInput>& in, std::vector<int>& seq) {
  cudaSetDevice(device_);
  const Config& c = cfg_;
  const int d = c.enc_d_model, cs = c.enc_chunk_size, H = kConvHidden;
  auto cw = [](int w) { return (w + 2 - 3) / 2 + 1; };
  struct Grp { int input, c0, nc, w; };
  std::vector<Grp> groups;
  seq.assign(in.size(), 0);
  for (size_t i = 0; i < in.size(); ++i) {
    const int F = in[i].F;
    const int n_chunks = (F + cs - 1) / cs, full = F / cs;
    if (full > 0) groups.push_back({(int)i, 0, full, cs});
    if (full < n_chunks) groups.push_back({(int)i, full, 1, F - full * cs});
  }
  int T = 0;
  size_t max_cols = 0, max_a1 = 0, max_a2 = 0, max_a3 = 0;
  for (auto& g : groups) {
    int w1 = cw(g.w), w2 = cw(w1), w3 = cw(w2);
    T += g.nc * w3;
    seq[g.input] += g.nc * w3;
    max_a1 = std::max(max_a1, (size_t)g.nc * 64 * w1 * H);
    max_a2 = std::max(max_a2, (size_t)g.nc * 32 * w2 * H);
    max_a3 = std::max(max_a3, (size_t)g.nc * 16 * w3 * H);
    max_cols = std::max(max_cols, (size_t)g.nc * 32 * w2 * 9 * H);
  }
  if (T == 0) {
    set_error("encode: no input frames");
    return 0;
  }
  const bool conv_planes = !gemm_simt_forced();
  if (!act1_.alloc(max_a1) || !act2_.alloc(max_a2) || !act3_.alloc(max_a3) ||
      !cols_.alloc(conv_planes ? 1 : max_cols) || (conv_planes && !pl_conv_.alloc(3 * max_cols)) ||
      !x_enc_.alloc((size_t)T * d) || !xn_enc_.alloc((size_t)T * d) || !qkv_enc_.alloc((size_t)T * 3 * d) ||
      !att_enc_.alloc((size_t)T * d) || !mid_enc_.alloc((size_t)T * std::max(c.enc_ffn_dim, d)) ||
      !enc_.alloc((size_t)T * c.enc_output_dim) || !pl_a_.alloc(split_planes_elems(T, d)) ||
      !pl_b_.alloc(split_planes_elems(T, std::max(c.enc_ffn_dim, d))))
    return 0;
  const long fb0 = gemm_tc_fallbacks();
  cudaEventRecord(ev0_, stream_);
  launches += 7 * (long)groups.size() + 7 * (long)enc_layers_.size() + 3;
  int tok = 0;
  for (auto& g : groups) {
    int w1 = cw(g.w), w2 = cw(w1), w3 = cw(w2);
    conv1_gelu(in[g.input].mel, in[g.input].F, g.c0 * cs, cs, g.nc, g.w, conv1_w, conv1_b, act1_.p, stream_);
    // im2col straight into the tensor-core GEMM's bf16 planes (f32 columns under QASR_GEMM=simt)
    const bool planes = !gemm_simt_forced();
    GemmArgs a;
    a.M = g.nc * 32 * w2; a.N = H; a.K = 9 * H;
    long long pl = (long long)a.M * a.K;
    im2col_s2(act1_.p, g.nc, 64, w1, cols_.p, false, stream_, planes ? pl_conv_.p : nullptr, pl);
    a.A = cols_.p; a.lda = 9 * H; a.B = conv2_w; a.ldb = 9 * H;
    a.C = act2_.p; a.ldc = H; a.epi = EPI_BIAS_GELU; a.bias = conv2_b; a.split_k = -1;
    if (planes) {
      a.a_split = pl_conv_.p; a.a_split_ld = a.K; a.a_split_plane = pl;
    }
    gemm(a, stream_);
    a.M = g.nc * w3 * 16;
    pl = (long long)a.M * a.K;
    im2col_s2(act2_.p, g.nc, 32, w2, cols_.p, true, stream_, planes ? pl_conv_.p : nullptr, pl);
    a.A = cols_.p; a.B = conv3_w; a.C = act3_.p; a.bias = conv3_b;
    if (planes) a.a_split_plane = pl;
    gemm(a, stream_);
    GemmArgs o;
    o.M = g.nc * w3; o.N = d; o.K = 16 * H;
    o.A = act3_.p; o.lda = 16 * H; o.B = conv_out_w; o.ldb = 16 * H;
    o.C = x_enc_.p + (size_t)tok * d; o.ldc = d;
    gemm(o, stream_);
    add_pe_rows(x_enc_.p + (size_t)tok * d, g.nc * w3, d, w3, pe_, stream_);
    tok += g.nc * w3;
  }
  // attention windows (encoder.rs:292-298)
  int tpc = cw(cw(cw(cs)));
  int wts = tpc * (c.enc_n_window_infer / cs);
  std::vector<int> ws;
  for (size_t i = 0, t0 = 0; i < in.size(); t0 += seq[i], ++i)
    for (int s = 0; s < seq[i]; s += wts) ws.push_back((int)t0 + s);
  const int n_win = (int)ws.size();
  ws.push_back(T);
  int max_win = 0;
  for (int w = 0; w < n_win; ++w) max_win = std::max(max_win, ws[w + 1] - ws[w]);
  if (!win_starts_.alloc(n_win + 1)) return 0;
  CUDA_OK(cudaMemcpyAsync(win_starts_.p, ws.data(), ws.size() * 4, cudaMemcpyHostToDevice, stream_), 0);
  const float scale = 1.0f / sqrtf((float)c.enc_head_dim);
  const long long plT = (long long)T * d, plF = (long long)T * c.enc_ffn_dim;
  for (auto& L : enc_layers_) {
    layer_norm_rows(x_enc_.p, xn_enc_.p, T, d, L.ln1w, L.ln1b, 1e-5f, stream_, pl_a_.p, plT);
    GemmArgs a;
    a.M = T; a.N = 3 * d; a.K = d; a.A = xn_enc_.p; a.lda = d; a.B = L.wqkv; a.ldb = d;
    a.C = qkv_enc_.p; a.ldc = 3 * d; a.epi = EPI_BIAS; a.bias = L.bqkv;
    a.a_split = pl_a_.p; a.a_split_ld = d; a.a_split_plane = plT;
    gemm(a, stream_);
    // tensor-core windows (att planes feed the o projection); the SIMT kernel only for
    // windows above 128 rows or under QASR_ATTN=simt
    const bool tc_att = !simt_attention() && window_attention_tc(qkv_enc_.p, att_enc_.p, pl_a_.p, plT, d, c.enc_heads,
                                                                 c.enc_head_dim, win_starts_.p, n_win, max_win,
                                                                 scale, stream_);
    if (!tc_att)
      window_attention(qkv_enc_.p, att_enc_.p, T, d, c.enc_heads, win_starts_.p, n_win, max_win, scale, stream_);
    GemmArgs o;
    o.M = T; o.N = d; o.K = d; o.A = att_enc_.p; o.lda = d; o.B = L.wo; o.ldb = d;
    o.C = x_enc_.p; o.ldc = d; o.epi = EPI_RESID; o.resid = x_enc_.p; o.ldr = d; o.bias = L.bo;
    if (tc_att) {
      o.a_split = pl_a_.p; o.a_split_ld = d; o.a_split_plane = plT;
    }
    gemm(o, stream_);
    layer_norm_rows(x_enc_.p, xn_enc_.p, T, d, L.ln2w, L.ln2b, 1e-5f, stream_, pl_a_.p, plT);
    GemmArgs f1;
    f1.M = T; f1.N = c.enc_ffn_dim; f1.K = d; f1.A = xn_enc_.p; f1.lda = d; f1.B = L.w1; f1.ldb = d;
    f1.C = mid_enc_.p; f1.ldc = c.enc_ffn_dim; f1.epi = EPI_BIAS_GELU; f1.bias = L.b1;
    f1.a_split = pl_a_.p; f1.a_split_ld = d; f1.a_split_plane = plT;
    f1.c_split = pl_b_.p; f1.c_split_ld = c.enc_ffn_dim; f1.c_split_plane = plF;
    gemm(f1, stream_);
    GemmArgs f2;
    f2.M = T; f2.N = d; f2.K = c.enc_ffn_dim; f2.A = mid_enc_.p; f2.lda = c.enc_ffn_dim; f2.B = L.w2;
    f2.ldb = c.enc_ffn_dim; f2.C = x_enc_.p; f2.ldc = d; f2.epi = EPI_RESID; f2.resid = x_enc_.p; f2.ldr = d;
    f2.bias = L.b2;
    f2.a_split = pl_b_.p; f2.a_split_ld = c.enc_ffn_dim; f2.a_split_plane = plF;
    gemm(f2, stream_);
  }
  layer_norm_rows(x_enc_.p, xn_enc_.p, T, d, ln_post_w, ln_post_b, 1e-5f, stream_, pl_a_.p, plT);
  GemmArgs p1;
  p1.M = T; p1.N = d; p1.K = d; p1.A = xn_enc_.p; p1.lda = d; p1.B = proj1_w; p1.ldb = d;
  p1.C = mid_enc_.p; p1.ldc = d; p1.epi = EPI_BIAS_GELU; p1.bias = proj1_b;
  p1.a_split = pl_a_.p; p1.a_split_ld = d; p1.a_split_plane = plT;
  p1.c_split = pl_b_.p; p1.c_split_ld = d; p1.c_split_plane = plT;
  gemm(p1, stream_);
  GemmArgs p2;
  p2.M = T; p2.N = c.enc_output_dim; p2.K = d; p2.A = mid_enc_.p; p2.lda = d; p2.B = proj2_w; p2.ldb = d;
  p2.C = enc_.p; p2.ldc = c.enc_output_dim; p2.epi = EPI_BIAS; p2.bias = proj2_b;
  p2.a_split = pl_b_.p; p2.a_split_ld = d; p2.a_split_plane = plT;
  gemm(p2, stream_);
  cudaEventRecord(ev1_, stream_);
  CUDA_OK(cudaEventSynchronize(ev1_), 0);
  float ms = 0;
  cudaEventElapsedTime(&ms, ev0_, ev1_);
  perf.enc_ms += ms;
  if (!gemm_stage_ok(fb0)) return 0;
  CUDA_OK(cudaGetLastError(), 0);
  return T;
}

// ---------------------------------------------------------------------------- prefill
// Tensor-core GEMM health after a stage: a bounded device wait that gave up or a GEMM that
// left the tensor cores fails the stage with a recorded error.
bool Engine::simt_attention() {
  static int v = -1;
  if (v < 0) {
    const char* e = getenv("QASR_ATTN");
    v = (e && strcmp(e, "simt") == 0) ? 1 : 0;
  }
  return v == 1;
}

bool Engine::gemm_stage_ok(long fallbacks_before) {
  if (int e = attn_tc_error()) {
    set_error("tensor-core attention: a device-side wait timed out (code " + std::to_string(e) + ")");
    return false;
  }
  if (int e = gemm_tc_error()) {
    set_error("tensor-core GEMM: a device-side wait timed out (code " + std::to_string(e) + ")");
    return false;
  }
  if (gemm_tc_fallbacks() != fallbacks_before) {
    set_error("a bf16-weight GEMM left the tensor cores: " + last_error());
    return false;
  }
  return true;
}

// decoder_prefill's layer loop (decoder.rs:455-547) over R packed rows x: block b is
// rows [off, off + S) of one sequence at KV positions start.. in KV slot `slot`. The
// GEMMs run once over all rows; q/k norm + RoPE + KV append and attention per block.
bool Engine::prefill_layers(float* x, int R, const std::vector<RowBlock>& blocks) {
  const Config& c = cfg_;
  const int h = c.dec_hidden, qd = c.dec_heads * 128, kvd = c.dec_kv_heads * 128, inter = c.dec_intermediate;
  const int ldq = qd + 2 * kvd;
  const float scale = 1.0f / sqrtf(128.f);
  if (R <= 0) return true;
  if (!pl_a_.alloc(split_planes_elems(R, h)) || !pl_b_.alloc(split_planes_elems(R, inter)) ||
      !pl_c_.alloc(split_planes_elems(R, qd)))
    return false;
  const long long plH = (long long)R * h, plI = (long long)R * inter, plQ = (long long)R * qd;
  const bool simt_att = simt_attention();
  AttnPlan plan;
  if (!simt_att) {
    std::vector<AttnBlock> ab;
    for (const RowBlock& bk : blocks)
      if (bk.S > 0) ab.push_back({bk.off, bk.S, bk.start, bk.slot});
    if (!prefill_attention_plan(ab, c.dec_heads, kv_slot_stride(), stream_, plan)) {
      set_error("prefill: could not set up the attention work items");
      return false;
    }
    // per packed row: KV position and slot offset
    std::vector<int> rp(R, 0);
    std::vector<long long> rk(R, 0);
    for (const RowBlock& bk : blocks)
      for (int i = 0; i < bk.S; ++i) {
        rp[bk.off + i] = bk.start + i;
        rk[bk.off + i] = (long long)bk.slot * (long long)kv_slot_stride();
      }
    if (!prow_pos_.alloc(R) || !prow_kv_.alloc(R)) return false;
    CUDA_OK(cudaMemcpyAsync(prow_pos_.p, rp.data(), R * sizeof(int), cudaMemcpyHostToDevice, stream_), false);
    CUDA_OK(cudaMemcpyAsync(prow_kv_.p, rk.data(), R * sizeof(long long), cudaMemcpyHostToDevice, stream_), false);
  }
  for (int l = 0; l < c.dec_layers; ++l) {
    const DecLayerW& L = dec_layers_[l];
    rms_norm_rows(x, pxn_.p, R, h, L.n1, c.dec_rms_norm_eps, stream_, pl_a_.p, plH);
    GemmArgs a;
    a.M = R; a.N = ldq; a.K = h; a.A = pxn_.p; a.lda = h; a.B = L.wqkv; a.ldb = h;
    a.C = pqkv_.p; a.ldc = ldq;
    a.a_split = pl_a_.p; a.a_split_ld = h; a.a_split_plane = plH;
    gemm(a, stream_);
    if (simt_att) {
      for (const RowBlock& bk : blocks) {
        if (bk.S == 0) continue;
        const size_t so = (size_t)bk.slot * kv_slot_stride() + (size_t)l * c.dec_kv_heads * max_seq_ * 128;
        float* qk = pqkv_.p + (size_t)bk.off * ldq;
        prefill_qk_rope_kv(qk, bk.S, bk.start, c.dec_heads, c.dec_kv_heads, L.qn, L.kn, c.dec_rms_norm_eps,
                           rope_cos_, rope_sin_, kc_.p + so, vc_.p + so, max_seq_, stream_);
        prefill_attention(qk, bk.S, bk.start, c.dec_heads, c.dec_kv_heads, kc_.p + so, vc_.p + so, max_seq_, scale,
                          patt_.p + (size_t)bk.off * qd, stream_);
        launches += 2;
      }
    } else {
      // q/k norm + RoPE + KV append of every sequence's rows in one launch
      const size_t lo = (size_t)l * c.dec_kv_heads * max_seq_ * 128;
      prefill_qk_rope_kv_packed(pqkv_.p, R, prow_pos_.p, prow_kv_.p, c.dec_heads, c.dec_kv_heads, L.qn, L.kn,
                                c.dec_rms_norm_eps, rope_cos_, rope_sin_, kc_.p + lo, vc_.p + lo, max_seq_, stream_);
      launches += 1;
    }
    // every sequence's attention of this layer in one tensor-core launch
    if (!simt_att) {
      if (!prefill_attention_tc(plan, pqkv_.p, c.dec_heads, c.dec_kv_heads, kc_.p, vc_.p,
                                (long long)l * c.dec_kv_heads * max_seq_ * 128, max_seq_, scale, patt_.p, pl_c_.p,
                                plQ, stream_)) {
        set_error("prefill: the tensor-core attention kernel could not run");
        return false;
      }
      launches += 1;
    }
    GemmArgs o;
    o.M = R; o.N = h; o.K = qd; o.A = patt_.p; o.lda = qd; o.B = L.wo; o.ldb = qd;
    o.C = x; o.ldc = h; o.epi = EPI_RESID; o.resid = x; o.ldr = h;
    if (!simt_att) {
      o.a_split = pl_c_.p; o.a_split_ld = qd; o.a_split_plane = plQ;
    }
    gemm(o, stream_);
    rms_norm_rows(x, pxn_.p, R, h, L.n2, c.dec_rms_norm_eps, stream_, pl_a_.p, plH);
    GemmArgs g;
    g.M = R; g.N = 2 * inter; g.K = h; g.A = pxn_.p; g.lda = h; g.B = L.wgu; g.ldb = h;
    g.C = pmid_.p; g.ldc = inter; g.epi = EPI_SWIGLU;
    g.a_split = pl_a_.p; g.a_split_ld = h; g.a_split_plane = plH;
    g.c_split = pl_b_.p; g.c_split_ld = inter; g.c_split_plane = plI;
    gemm(g, stream_);
    GemmArgs dn;
    dn.M = R; dn.N = h; dn.K = inter; dn.A = pmid_.p; dn.lda = inter; dn.B = L.wdown; dn.ldb = inter;
    dn.C = x; dn.ldc = h; dn.epi = EPI_RESID; dn.resid = x; dn.ldr = h;
    dn.a_split = pl_b_.p; dn.a_split_ld = inter; dn.a_split_plane = plI;
    gemm(dn, stream_);
    launches += 6;
  }
  return true;
}

bool Engine::prefill_ids(const std::vector<int>& ids, const float* d_enc, int start_pos, int slot) {
  cudaSetDevice(device_);
  const int h = cfg_.dec_hidden, n = (int)ids.size();
  if (n < 1) return false;
  if (!ids_.alloc(n) || !px_.alloc((size_t)n * h)) return false;
  CUDA_OK(cudaMemcpyAsync(ids_.p, ids.data(), n * 4, cudaMemcpyHostToDevice, stream_), false);
  gather_embeds(ids_.p, n, embed_, d_enc, h, px_.p, stream_);
  launches += 1;
  return run_prefill(n, start_pos, slot);
}

bool Engine::prefill_many(const std::vector<PrefillJob>& jobs, const float* d_enc) {
  cudaSetDevice(device_);
  const Config& c = cfg_;
  const int h = c.dec_hidden, qd = c.dec_heads * 128, kvd = c.dec_kv_heads * 128, inter = c.dec_intermediate;
  const int J = (int)jobs.size();
  if (J == 0) return true;
  // packed rows: every job's rows [start_pos, n - 1), then every job's last row
  std::vector<int> packed, off(J + 1, 0);
  int max_n = 0, max_slot = 0;
  for (int j = 0; j < J; ++j) {
    const auto& ids = *jobs[j].ids;
    const int n = (int)ids.size(), s0 = jobs[j].start_pos;
    if (n < 1 || s0 < 0 || s0 > n - 1 || jobs[j].slot < 0 || jobs[j].slot >= kMaxSlots) {
      set_error("prefill_many: job " + std::to_string(j) + " has no rows to prefill or a bad slot");
      return false;
    }
    packed.insert(packed.end(), ids.begin() + s0, ids.end() - 1);
    off[j + 1] = (int)packed.size();
    max_n = std::max(max_n, n);
    max_slot = std::max(max_slot, jobs[j].slot);
  }
  const int R = (int)packed.size();
  for (int j = 0; j < J; ++j) packed.push_back(jobs[j].ids->back());
  if (!ensure_slots(max_slot + 1) || !ensure_kv(max_n + 1024)) return false;
  if (!ids_.alloc(packed.size()) || !px_.alloc(packed.size() * h) || !pxn_.alloc((size_t)std::max(R, 1) * h) ||
      !pqkv_.alloc((size_t)std::max(R, 1) * (qd + 2 * kvd)) || !patt_.alloc((size_t)std::max(R, 1) * qd) ||
      !pmid_.alloc((size_t)std::max(R, 1) * inter))
    return false;
  const long fb0 = gemm_tc_fallbacks();
  CUDA_OK(cudaMemcpyAsync(ids_.p, packed.data(), packed.size() * 4, cudaMemcpyHostToDevice, stream_), false);
  cudaEventRecord(ev0_, stream_);
  gather_embeds(ids_.p, (int)packed.size(), embed_, d_enc, h, px_.p, stream_);
  launches += 1;
  std::vector<RowBlock> blocks;
  for (int j = 0; j < J; ++j) blocks.push_back({off[j], off[j + 1] - off[j], jobs[j].start_pos, jobs[j].slot});
  if (!prefill_layers(px_.p, R, blocks)) return false;
  // each job's first decode input is its last prompt row (transcribe.rs:171-185)
  for (int j = 0; j < J; ++j) {
    const int slot = jobs[j].slot, n = (int)jobs[j].ids->size();
    CUDA_OK(cudaMemcpyAsync(dx_.p + (size_t)slot * h, px_.p + (size_t)(R + j) * h, (size_t)h * 4,
                            cudaMemcpyDeviceToDevice, stream_),
            false);
    StepState* hs = hstate_ + slot;
    hs->pos = n - 1;
    hs->step = 0;
    hs->cur_token = -1;
    hs->forced_mode = 0;
    CUDA_OK(cudaMemcpyAsync(dstate_.p + slot, hs, sizeof(StepState), cudaMemcpyHostToDevice, stream_), false);
    if (slot == 0) kv_len_ = n - 1;
  }
  cudaEventRecord(ev1_, stream_);
  CUDA_OK(cudaEventSynchronize(ev1_), false);
  float ms = 0;
  cudaEventElapsedTime(&ms, ev0_, ev1_);
  perf.prefill_ms += ms;
  if (!gemm_stage_ok(fb0)) return false;
  CUDA_OK(cudaGetLastError(), false);
  return true;
}

bool Engine::prefill_classify(const std::vector<int>& ids, const float* d_enc, const std::vector<int>& rows,
                              std::vector<int>& cls) {
  cudaSetDevice(device_);
  const Config& c = cfg_;
  const int h = c.dec_hidden, N = c.classify_num, m = (int)rows.size();
  if (N <= 0) {
    set_error("align: model is not a forced aligner (classify_num=0)");
    return false;
  }
  if (ids.empty()) {
    set_error("align: empty prompt");
    return false;
  }
  for (int r : rows)
    if (r < 0 || r >= (int)ids.size()) {
      set_error("align: classify row out of range");
      return false;
    }
  // prefill_many prefills rows [0, n - 1) of a job: one extra row makes every prompt row
  // part of the prefill (its own hidden state stays unused)
  std::vector<int> ext(ids);
  ext.push_back(ids.back());
  if (!prefill_many({{&ext, 0, 0}}, d_enc)) return false;
  cls.assign(m, 0);
  if (m == 0) return true;
  std::vector<int> g(m);
  for (int k = 0; k < m; ++k) g[k] = -(rows[k] + 1);  // rows of px_ through the encoder-row path
  if (!cls_ids_.alloc(m) || !cls_out_.alloc(m) || !cls_x_.alloc((size_t)m * h) || !cls_xn_.alloc((size_t)m * h) ||
      !cls_logits_.alloc((size_t)m * N))
    return false;
  const long fb0 = gemm_tc_fallbacks();
  CUDA_OK(cudaMemcpyAsync(cls_ids_.p, g.data(), m * 4, cudaMemcpyHostToDevice, stream_), false);
  gather_embeds(cls_ids_.p, m, embed_, px_.p, h, cls_x_.p, stream_);
  rms_norm_rows(cls_x_.p, cls_xn_.p, m, h, final_norm_, c.dec_rms_norm_eps, stream_);
  GemmArgs a;
  a.M = m; a.N = N; a.K = h; a.A = cls_xn_.p; a.lda = h; a.B = lm_bf16_; a.ldb = h;
  a.C = cls_logits_.p; a.ldc = N;
  gemm(a, stream_);
  rows_argmax(cls_logits_.p, m, N, cls_out_.p, stream_);
  launches += 4;
  CUDA_OK(cudaMemcpyAsync(cls.data(), cls_out_.p, m * 4, cudaMemcpyDeviceToHost, stream_), false);
  CUDA_OK(cudaStreamSynchronize(stream_), false);
  if (!gemm_stage_ok(fb0)) return false;
  CUDA_OK(cudaGetLastError(), false);
  return true;
}

bool Engine::prefill_rows(const float* rows, int n, int start_pos, int slot) {
  cudaSetDevice(device_);
  const int h = cfg_.dec_hidden;
  if (n < 1 || !px_.alloc((size_t)n * h)) return false;
  CUDA_OK(cudaMemcpyAsync(px_.p, rows, (size_t)n * h * 4, cudaMemcpyHostToDevice, stream_), false);
  return run_prefill(n, start_pos, slot);
}

// px_ holds all n prompt rows; rows [start_pos, n-1) are prefilled at positions
// start_pos.. and row n-1 becomes the first decode input (transcribe.rs:171-185).
bool Engine::run_prefill(int n, int start_pos, int slot) {
  const Config& c = cfg_;
  const int h = c.dec_hidden, qd = c.dec_heads * 128, kvd = c.dec_kv_heads * 128, inter = c.dec_intermediate;
  const int S = n - 1 - start_pos;
  if (S < 0 || slot < 0 || slot >= kMaxSlots) return false;
  if (!ensure_slots(slot + 1) || !ensure_kv(n + 1024)) return false;
  if (!pxn_.alloc((size_t)std::max(S, 1) * h) || !pqkv_.alloc((size_t)std::max(S, 1) * (qd + 2 * kvd)) ||
      !patt_.alloc((size_t)std::max(S, 1) * qd) || !pmid_.alloc((size_t)std::max(S, 1) * inter))
    return false;
  cudaEventRecord(ev0_, stream_);
  const long fb0 = gemm_tc_fallbacks();
  if (S > 0 && !prefill_layers(px_.p + (size_t)start_pos * h, S, {{0, S, start_pos, slot}})) return false;
  if (slot == 0) kv_len_ = n - 1;
  // first decode input: the last prompt row
  CUDA_OK(cudaMemcpyAsync(dx_.p + (size_t)slot * h, px_.p + (size_t)(n - 1) * h, (size_t)h * 4,
                          cudaMemcpyDeviceToDevice, stream_),
          false);
  StepState* hs = hstate_ + slot;
  hs->pos = n - 1;
  hs->step = 0;
  hs->cur_token = -1;
  hs->forced_mode = 0;
  CUDA_OK(cudaMemcpyAsync(dstate_.p + slot, hs, sizeof(StepState), cudaMemcpyHostToDevice, stream_), false);
  cudaEventRecord(ev1_, stream_);
  CUDA_OK(cudaEventSynchronize(ev1_), false);
  float ms = 0;
  cudaEventElapsedTime(&ms, ev0_, ev1_);
  perf.prefill_ms += ms;
  if (!gemm_stage_ok(fb0)) return false;
  CUDA_OK(cudaGetLastError(), false);
  return true;
}

const float* Engine::resample_to_device(const float* h_in, long n, int rate, long* n_out) {
  cudaSetDevice(device_);
  const long m = resampled_length(n, rate, kSampleRate);
  if (n <= 0 || rate <= 0 || m <= 0) {
    set_error("resample: empty input or bad rate");
    return nullptr;
  }
  if (!rs_in_.alloc(n) || !rs_out_.alloc(m)) return nullptr;
  CUDA_OK(cudaMemcpyAsync(rs_in_.p, h_in, (size_t)n * 4, cudaMemcpyHostToDevice, stream_), nullptr);
  resample_device(rs_in_.p, n, rate, kSampleRate, rs_out_.p, stream_);
  CUDA_OK(cudaGetLastError(), nullptr);
  *n_out = m;
  return rs_out_.p;
}

bool Engine::compact_silence(const float* h_in, long n, std::vector<float>& out) {
  cudaSetDevice(device_);
  out.clear();
  if (n <= 0) return true;
  if (!cs_in_.alloc(n) || !cs_out_.alloc(n) || !cs_scratch_.alloc(compact_silence_scratch(n)) || !cs_count_.alloc(2))
    return false;
  CUDA_OK(cudaMemcpyAsync(cs_in_.p, h_in, (size_t)n * 4, cudaMemcpyHostToDevice, stream_), false);
  compact_silence_device(cs_in_.p, n, cs_out_.p, cs_scratch_.p, cs_count_.p, stream_);
  CUDA_OK(cudaGetLastError(), false);
  long long cnt[2] = {0, 0};
  CUDA_OK(cudaMemcpyAsync(cnt, cs_count_.p, sizeof(cnt), cudaMemcpyDeviceToHost, stream_), false);
  CUDA_OK(cudaStreamSynchronize(stream_), false);
  if (cnt[0] < 0 || cnt[0] > n) {
    set_error("compact_silence: kept count out of range");
    return false;
  }
  out.resize((size_t)cnt[0]);
  if (cnt[0] > 0) {
    CUDA_OK(cudaMemcpyAsync(out.data(), cs_out_.p, (size_t)cnt[0] * 4, cudaMemcpyDeviceToHost, stream_), false);
    CUDA_OK(cudaStreamSynchronize(stream_), false);
  }
  return true;
}

bool Engine::copy_kv(int slot, int layer, int n_pos, float* k, float* v) {
  cudaSetDevice(device_);
  const Config& c = cfg_;
  if (slot < 0 || slot >= slots_ || layer < 0 || layer >= c.dec_layers || n_pos < 0 || n_pos > max_seq_) {
    set_error("copy_kv: slot, layer or position count out of range");
    return false;
  }
  CUDA_OK(cudaStreamSynchronize(stream_), false);
  for (int hh = 0; hh < c.dec_kv_heads; ++hh) {
    const size_t off = (size_t)slot * kv_slot_stride() + ((size_t)layer * c.dec_kv_heads + hh) * max_seq_ * 128;
    CUDA_OK(cudaMemcpy(k + (size_t)hh * n_pos * 128, kc_.p + off, (size_t)n_pos * 128 * 4, cudaMemcpyDeviceToHost),
            false);
    CUDA_OK(cudaMemcpy(v + (size_t)hh * n_pos * 128, vc_.p + off, (size_t)n_pos * 128 * 4, cudaMemcpyDeviceToHost),
            false);
  }
  return true;
}

long Engine::copy_quant(int layer, int which, int8_t* q, float* s, long cap_rows) {
  cudaSetDevice(device_);
  const Config& c = cfg_;
  const int h = c.dec_hidden, qd = c.dec_heads * 128, kvd = c.dec_kv_heads * 128, inter = c.dec_intermediate;
  const int8_t* dq = nullptr;
  const float* ds = nullptr;
  long rows = 0, cols = 0;
  if (which == 4) {
    dq = lm_q_; ds = lm_s_; rows = c.vocab_size; cols = h;
  } else {
    if (layer < 0 || layer >= c.dec_layers) return -1;
    const DecLayerW& L = dec_layers_[layer];
    switch (which) {
      case 0: dq = L.qqkv; ds = L.sqkv; rows = qd + 2 * kvd; cols = h; break;
      case 1: dq = L.qo; ds = L.so; rows = h; cols = qd; break;
      case 2: dq = L.qgu; ds = L.sgu; rows = 2 * inter; cols = h; break;
      case 3: dq = L.qdown; ds = L.sdown; rows = h; cols = inter; break;
      default: return -1;
    }
  }
  if (!dq || !ds) {
    set_error("copy_quant: the int8 weights are not resident");
    return -1;
  }
  if (rows > cap_rows) return rows;
  CUDA_OK(cudaStreamSynchronize(stream_), -1);
  CUDA_OK(cudaMemcpy(q, dq, (size_t)rows * cols, cudaMemcpyDeviceToHost), -1);
  CUDA_OK(cudaMemcpy(s, ds, (size_t)rows * 4, cudaMemcpyDeviceToHost), -1);
  return rows;
}

bool Engine::copy_prefill_hidden(std::vector<float>& out, int rows) {
  out.resize((size_t)rows * cfg_.dec_hidden);
  CUDA_OK(cudaMemcpy(out.data(), px_.p, out.size() * 4, cudaMemcpyDeviceToHost), false);
  return true;
}

// ---------------------------------------------------------------------------- decode
DecodeArgs Engine::dargs(const int* forced, float* logits, int slot) {
  const Config& c = cfg_;
  bool i8 = mode_ == DECODE_INT8;
  pw_qkv_.clear(); pw_o_.clear(); pw_gu_.clear(); pw_down_.clear();
  ps_qkv_.clear(); ps_o_.clear(); ps_gu_.clear(); ps_down_.clear();
  for (auto& L : dec_layers_) {
    pw_qkv_.push_back(i8 ? (const void*)L.qqkv : (const void*)L.wqkv);
    pw_o_.push_back(i8 ? (const void*)L.qo : (const void*)L.wo);
    pw_gu_.push_back(i8 ? (const void*)L.qgu : (const void*)L.wgu);
    pw_down_.push_back(i8 ? (const void*)L.qdown : (const void*)L.wdown);
    ps_qkv_.push_back(L.sqkv); ps_o_.push_back(L.so); ps_gu_.push_back(L.sgu); ps_down_.push_back(L.sdown);
  }
  DecodeArgs a{};
  a.hidden = c.dec_hidden; a.q_heads = c.dec_heads; a.kv_heads = c.dec_kv_heads; a.inter = c.dec_intermediate;
  a.vocab = c.classify_num > 0 ? c.classify_num : c.vocab_size; a.max_seq = max_seq_; a.eps = c.dec_rms_norm_eps;
  a.int8 = i8;
  a.w_qkv = pw_qkv_.data(); a.s_qkv = ps_qkv_.data(); a.w_o = pw_o_.data(); a.s_o = ps_o_.data();
  a.w_gu = pw_gu_.data(); a.s_gu = ps_gu_.data(); a.w_down = pw_down_.data(); a.s_down = ps_down_.data();
  a.n1 = pn1_.data(); a.n2 = pn2_.data(); a.qn = pqn_.data(); a.kn = pkn_.data();
  a.lm_w = i8 ? (const void*)lm_q_ : (const void*)lm_bf16_; a.lm_s = lm_s_; a.final_norm = final_norm_;
  a.embed = embed_; a.rope_cos = rope_cos_; a.rope_sin = rope_sin_;
  a.k_cache = kc_.p; a.v_cache = vc_.p; a.layers = c.dec_layers;
  a.x = dx_.p; a.qkv = dqkv_.p; a.attn = dattn_.p; a.ffn = dffn_.p; a.part = dpart_.p; a.ticket = dticket_.p;
  a.am_ticket = dam_ticket_.p; a.am_part = dam_part_.p; a.st = dstate_.p; a.tokens = dtokens_.p;
  a.staged = dstaged_.p;
  a.kv_slot_stride = kv_slot_stride(); a.tokens_ld = tokens_ld_; a.batch = 1;
  if (slot > 0) {  // one sequence in its own slot: offset the per-sequence buffers
    a.k_cache += (size_t)slot * kv_slot_stride();
    a.v_cache += (size_t)slot * kv_slot_stride();
    a.x += (size_t)slot * c.dec_hidden;
    a.st += slot;
    a.tokens += (size_t)slot * tokens_ld_;
  }
  a.forced = forced; a.logits = logits; a.err = derr_.p;
  if (timeline_) {
    a.tl = dtl_.p;
    a.tl_count = dtl_count_.p;
  }
  return a;
}

bool Engine::enqueue_step(const DecodeArgs& a) { return decode_step(a, stream_); }

// qkv+attention, o, gate/up, down per layer, then lm_head (batched steps add a q/k/v matvec)
int Engine::decode_step_launches_1() const {
  const bool split = decode_split_qkv(cfg_.dec_hidden, cfg_.dec_heads, cfg_.dec_kv_heads, mode_ == DECODE_INT8);
  return (split ? 5 : 4) * cfg_.dec_layers + 1;
}

bool Engine::decode(int max_steps, bool stop_on_eos, std::vector<int>& out, const std::vector<int>* forced,
                    std::vector<float>* logits, int slot) {
  cudaSetDevice(device_);
  out.clear();
  if (max_steps <= 0) return true;
  if (slot < 0 || slot >= kMaxSlots || slot >= slots_) {
    set_error("decode: slot " + std::to_string(slot) + " holds no prefilled sequence");
    return false;
  }
  StepState* hs = hstate_ + slot;
  const int start_pos = hs->pos;
  if (!ensure_kv(start_pos + max_steps + 1)) return false;
  if (!ensure_tokens(max_steps, slot + 1)) return false;
  if (timeline_) {
    size_t need = (size_t)max_steps * (cfg_.dec_layers * 9 + 2) * 8 * 4 + 64;  // 8 records a kernel
    if (dtl_.n < need) {
      if (!dtl_.alloc(need)) return false;
      ++graph_gen_;
    }
    if (!dtl_count_.alloc(1)) return false;
    CUDA_OK(cudaMemsetAsync(dtl_count_.p, 0, sizeof(int), stream_), false);
  }
  std::vector<float> rec;
  if (record_logits && !logits) logits = &rec;
  cudaEventRecord(ev0_, stream_);
  const bool direct = forced || logits || !use_graph || profile;
  if (direct) {
    // Teacher-forced / logits-recording path: plain launches, one step at a time.
    if (forced) {
      if (!dforced_.alloc(std::max<size_t>(forced->size(), 1))) return false;
      CUDA_OK(cudaMemcpyAsync(dforced_.p, forced->data(), forced->size() * 4, cudaMemcpyHostToDevice, stream_), false);
      hs->forced_mode = 1;
      CUDA_OK(cudaMemcpyAsync(&dstate_.p[slot].forced_mode, &hs->forced_mode, sizeof(int), cudaMemcpyHostToDevice,
                              stream_),
              false);
    }
    DecodeArgs a = dargs(forced ? dforced_.p : nullptr, logits ? dlogits_.p : nullptr, slot);
    if (profile) {
      a.on_launch = [](void* ctx, int kind) {
        Engine* e = (Engine*)ctx;
        cudaEvent_t ev;
        cudaEventCreate(&ev);
        cudaEventRecord(ev, e->stream_);
        e->prof_ev_.push_back({kind, ev});
      };
      a.hook_ctx = this;
    }
    const int V = a.vocab;
    if (logits) logits->resize((size_t)max_steps * V);
    for (int i = 0; i < max_steps; ++i) {
      if (profile) a.on_launch(this, -1);
      if (!decode_step(a, stream_)) {
        cudaStreamSynchronize(stream_);
        return false;
      }
      if (logits)
        CUDA_OK(cudaMemcpyAsync(logits->data() + (size_t)i * V, dlogits_.p, (size_t)V * 4, cudaMemcpyDeviceToHost,
                                stream_),
                false);
    }
    CUDA_OK(cudaMemcpyAsync(htokens_, dtokens_.p + (size_t)slot * tokens_ld_, max_steps * 4, cudaMemcpyDeviceToHost,
                            stream_),
            false);
    CUDA_OK(cudaStreamSynchronize(stream_), false);
    CUDA_OK(cudaGetLastError(), false);
    out.assign(htokens_, htokens_ + max_steps);
    if (record_logits) recorded_logits.insert(recorded_logits.end(), logits->end() - V, logits->end());
    launches += (long)max_steps * decode_step_launches_1();
    for (size_t i = 1; i < prof_ev_.size(); ++i) {
      int k = prof_ev_[i].first;
      if (k < 0) continue;
      float ms = 0;
      cudaEventElapsedTime(&ms, prof_ev_[i - 1].second, prof_ev_[i].second);
      prof_ms[k] += ms;
      prof_n[k] += 1;
    }
    for (auto& pe : prof_ev_) cudaEventDestroy(pe.second);
    prof_ev_.clear();
  } else {
    if (slot == 0 ? !graph_for(0) : !graph_for_slot(slot)) return false;
    cudaGraphExec_t step_graph = slot == 0 ? graph_exec_[0] : slot_graph_[slot];
    // Launch in chunks; after each chunk copy its ids back and look for EOS while the
    // next chunk runs (transcribe.rs:194-226 stop rule).
    const int chunk = 16;
    int launched = 0, checked = 0;
    bool stop = false;
    std::vector<cudaEvent_t> evs;
    auto launch_chunk = [&]() -> bool {
      int c = std::min(chunk, max_steps - launched);
      for (int i = 0; i < c; ++i) CUDA_OK(cudaGraphLaunch(step_graph, stream_), false);
      CUDA_OK(cudaMemcpyAsync(htokens_ + launched, dtokens_.p + (size_t)slot * tokens_ld_ + launched, c * 4,
                              cudaMemcpyDeviceToHost, stream_),
              false);
      cudaEvent_t e;
      cudaEventCreateWithFlags(&e, cudaEventDisableTiming);
      cudaEventRecord(e, stream_);
      evs.push_back(e);
      launched += c;
      return true;
    };
    if (!launch_chunk()) return false;
    size_t ev_i = 0;
    while (!stop) {
      if (launched < max_steps && !launch_chunk()) return false;
      CUDA_OK(cudaEventSynchronize(evs[ev_i]), false);
      int upto = std::min(max_steps, checked + chunk);
      for (int i = checked; i < upto; ++i) {
        out.push_back(htokens_[i]);
        if (stop_on_eos && (htokens_[i] == kTokEndOfText || htokens_[i] == kTokImEnd)) {
          stop = true;
          break;
        }
      }
      checked = upto;
      ++ev_i;
      if (checked >= max_steps) stop = true;
    }
    CUDA_OK(cudaStreamSynchronize(stream_), false);
    launches += (long)launched * decode_step_launches_1();
    for (auto e : evs) cudaEventDestroy(e);
    CUDA_OK(cudaGetLastError(), false);
  }
  {
    int herr = 0;
    CUDA_OK(cudaMemcpy(&herr, derr_.p, sizeof(int), cudaMemcpyDeviceToHost), false);
    if (herr) {
      cudaMemset(derr_.p, 0, sizeof(int));
      set_error("decode: a device-side wait timed out (code " + std::to_string(herr) + ")");
      return false;
    }
  }
  if (timeline_) {
    int cnt = 0;
    CUDA_OK(cudaMemcpy(&cnt, dtl_count_.p, sizeof(int), cudaMemcpyDeviceToHost), false);
    cnt = std::min<int>(cnt, (int)(dtl_.n / 4));
    last_timeline.resize((size_t)cnt * 4);
    CUDA_OK(cudaMemcpy(last_timeline.data(), dtl_.p, last_timeline.size() * 8, cudaMemcpyDeviceToHost), false);
  }
  // KV length after the steps the caller consumes (extra speculative steps are ignored).
  hs->pos = start_pos + (int)out.size();
  hs->forced_mode = 0;
  if (slot == 0) kv_len_ = hs->pos;
  cudaEventRecord(ev1_, stream_);
  cudaEventSynchronize(ev1_);
  float ms = 0;
  cudaEventElapsedTime(&ms, ev0_, ev1_);
  perf.decode_ms += ms;
  perf.decode_steps += (int)out.size();
  return true;
}

bool Engine::ensure_tokens(int max_steps, int B) {
  const int ld = std::max(tokens_ld_, std::max(max_steps, 2048));
  const int rows = std::max(B, tokens_rows_);
  if (ld == tokens_ld_ && rows == tokens_rows_) return true;
  if (!dtokens_.alloc((size_t)rows * ld)) return false;
  if (htokens_) cudaFreeHost(htokens_);
  htokens_ = nullptr;
  CUDA_OK(cudaMallocHost(&htokens_, (size_t)rows * ld * sizeof(int)), false);
  tokens_ld_ = ld;
  tokens_rows_ = rows;
  ++graph_gen_;
  return true;
}

// One captured decode step for batch size B (re-captured after any buffer moved).
// Slot 0 holds the single-sequence step of decode(); slot B >= 1 the batched step of
// decode_batch().
bool Engine::graph_for(int B) {
  if (built_gen_[B] == graph_gen_ && graph_exec_[B]) return true;
  if (graph_exec_[B]) cudaGraphExecDestroy(graph_exec_[B]);
  graph_exec_[B] = nullptr;
  DecodeArgs a = dargs(nullptr, nullptr);
  a.batch = std::max(B, 1);
  cudaGraph_t g = nullptr;
  CUDA_OK(cudaStreamBeginCapture(stream_, cudaStreamCaptureModeThreadLocal), false);
  const bool planned = decode_step(a, stream_);
  const cudaError_t e1 = cudaStreamEndCapture(stream_, &g);
  cudaError_t e2 = cudaErrorUnknown;
  if (planned && e1 == cudaSuccess) e2 = cudaGraphInstantiate(&graph_exec_[B], g, 0);
  if (g) cudaGraphDestroy(g);
  if (planned && e1 == cudaSuccess && e2 == cudaSuccess) {
    built_gen_[B] = graph_gen_;
    return true;
  }
  cudaGetLastError();
  graph_exec_[B] = nullptr;
  if (planned) set_error("decode: CUDA graph capture of the decode step failed");
  return false;
}

bool Engine::graph_for_slot(int slot) {
  if ((int)slot_graph_.size() <= slot) {
    slot_graph_.resize(slot + 1, nullptr);
    slot_graph_gen_.resize(slot + 1, 0);
  }
  if (slot_graph_gen_[slot] == graph_gen_ && slot_graph_[slot]) return true;
  if (slot_graph_[slot]) cudaGraphExecDestroy(slot_graph_[slot]);
  slot_graph_[slot] = nullptr;
  DecodeArgs a = dargs(nullptr, nullptr, slot);
  cudaGraph_t g = nullptr;
  CUDA_OK(cudaStreamBeginCapture(stream_, cudaStreamCaptureModeThreadLocal), false);
  const bool planned = enqueue_step(a);
  CUDA_OK(cudaStreamEndCapture(stream_, &g), false);
  if (!planned) {
    cudaGraphDestroy(g);
    return false;
  }
  const cudaError_t e = cudaGraphInstantiate(&slot_graph_[slot], g, 0);
  cudaGraphDestroy(g);
  CUDA_OK(e, false);
  slot_graph_gen_[slot] = graph_gen_;
  return true;
}

int Engine::max_decode_batch() {
  if (max_batch_ == 0) {
    cudaSetDevice(device_);
    const Config& c = cfg_;
    max_batch_ = decode_max_batch(c.dec_hidden, c.dec_intermediate, c.dec_heads, c.dec_kv_heads, mode_ == DECODE_INT8);
  }
  return max_batch_;
}

bool Engine::decode_batch(int B, int max_steps, bool stop_on_eos, std::vector<std::vector<int>>& out,
                          int first_slot) {
  cudaSetDevice(device_);
  out.assign(std::max(B, 0), {});
  if (B <= 0 || max_steps <= 0) return true;
  if (B > max_decode_batch() || first_slot < 0 || first_slot + B > slots_) {
    set_error("decode_batch: batch " + std::to_string(B) + " exceeds the prefilled slots or the kernel limit");
    return false;
  }
  int maxpos = 0;
  for (int b = 0; b < B; ++b) maxpos = std::max(maxpos, hstate_[first_slot + b].pos);
  if (!ensure_kv(maxpos + max_steps + 1) || !ensure_tokens(max_steps, first_slot + B)) return false;
  if (timeline_) {
    size_t need = (size_t)max_steps * (cfg_.dec_layers * 9 + 2) * 8 * 4 + 64;  // 8 records a kernel
    if (dtl_.n < need) {
      if (!dtl_.alloc(need)) return false;
      ++graph_gen_;
    }
    if (!dtl_count_.alloc(1)) return false;
    CUDA_OK(cudaMemsetAsync(dtl_count_.p, 0, sizeof(int), stream_), false);
  }
  cudaGraphExec_t run_graph = nullptr;
  if (record_logits) {
    // plain launches writing every sequence's logits at each step; the last step's are kept
    if (!drec_.alloc((size_t)B * cfg_.vocab_size)) return false;
  } else if (use_graph && first_slot == 0) {
    if (!graph_for(B)) return false;
    run_graph = graph_exec_[B];
  } else if (use_graph) {
    auto& entry = run_graphs_[first_slot * 64 + B];
    if (!entry.first || entry.second != graph_gen_) {
      if (entry.first) cudaGraphExecDestroy(entry.first);
      entry.first = nullptr;
      DecodeArgs ga = dargs(nullptr, nullptr, first_slot);
      ga.batch = B;
      cudaGraph_t g = nullptr;
      CUDA_OK(cudaStreamBeginCapture(stream_, cudaStreamCaptureModeThreadLocal), false);
      const bool planned = decode_step(ga, stream_);
      CUDA_OK(cudaStreamEndCapture(stream_, &g), false);
      if (!planned) {
        cudaGraphDestroy(g);
        return false;
      }
      const cudaError_t e = cudaGraphInstantiate(&entry.first, g, 0);
      cudaGraphDestroy(g);
      CUDA_OK(e, false);
      entry.second = graph_gen_;
    }
    run_graph = entry.first;
  }
  DecodeArgs direct_args = dargs(nullptr, record_logits ? drec_.p : nullptr, first_slot);
  direct_args.batch = B;
  cudaEventRecord(ev0_, stream_);
  // Chunks of steps; after each chunk the ids of every sequence come back (one 2-D copy)
  // and are scanned for EOS while the next chunk runs (transcribe.rs:194-226 per sequence).
  const int chunk = 16, ld = tokens_ld_;
  int launched = 0, checked = 0;
  std::vector<char> done(B, 0);
  int n_done = 0;
  std::vector<cudaEvent_t> evs;
  auto launch_chunk = [&]() -> bool {
    int c = std::min(chunk, max_steps - launched);
    for (int i = 0; i < c; ++i) {
      if (run_graph) CUDA_OK(cudaGraphLaunch(run_graph, stream_), false);
      else if (!decode_step(direct_args, stream_)) return false;
    }
    CUDA_OK(cudaMemcpy2DAsync(htokens_ + launched, (size_t)ld * 4, dtokens_.p + (size_t)first_slot * ld + launched,
                              (size_t)ld * 4, (size_t)c * 4, B, cudaMemcpyDeviceToHost, stream_),
            false);
    cudaEvent_t e;
    cudaEventCreateWithFlags(&e, cudaEventDisableTiming);
    cudaEventRecord(e, stream_);
    evs.push_back(e);
    launched += c;
    return true;
  };
  bool ok = launch_chunk();
  size_t ev_i = 0;
  bool stop = !ok;
  while (!stop) {
    if (launched < max_steps && !launch_chunk()) {
      ok = false;
      break;
    }
    if (cudaEventSynchronize(evs[ev_i]) != cudaSuccess) {
      ok = false;
      break;
    }
    const int upto = std::min(max_steps, checked + chunk);
    for (int b = 0; b < B; ++b) {
      for (int i = checked; i < upto && !done[b]; ++i) {
        const int t = htokens_[(size_t)b * ld + i];
        out[b].push_back(t);
        if (stop_on_eos && (t == kTokEndOfText || t == kTokImEnd)) {
          done[b] = 1;
          ++n_done;
        }
      }
    }
    checked = upto;
    ++ev_i;
    if (checked >= max_steps || n_done == B) stop = true;
  }
  cudaStreamSynchronize(stream_);
  for (auto e : evs) cudaEventDestroy(e);
  if (!ok) {
    set_error("decode_batch: launch or copy failed");
    return false;
  }
  CUDA_OK(cudaGetLastError(), false);
  launches += (long)launched * (B > 1 ? decode_batched_step_launches(cfg_.dec_layers, mode_ == DECODE_INT8) : decode_step_launches_1());
  int herr = 0;
  CUDA_OK(cudaMemcpy(&herr, derr_.p, sizeof(int), cudaMemcpyDeviceToHost), false);
  if (herr) {
    cudaMemset(derr_.p, 0, sizeof(int));
    set_error("decode: a device-side wait timed out (code " + std::to_string(herr) + ")");
    return false;
  }
  if (timeline_) {
    int cnt = 0;
    CUDA_OK(cudaMemcpy(&cnt, dtl_count_.p, sizeof(int), cudaMemcpyDeviceToHost), false);
    cnt = std::min<int>(cnt, (int)(dtl_.n / 4));
    last_timeline.resize((size_t)cnt * 4);
    CUDA_OK(cudaMemcpy(last_timeline.data(), dtl_.p, last_timeline.size() * 8, cudaMemcpyDeviceToHost), false);
  }
  size_t longest = 0;
  for (int b = 0; b < B; ++b) {
    hstate_[first_slot + b].pos += (int)out[b].size();
    longest = std::max(longest, out[b].size());
  }
  if (first_slot == 0) kv_len_ = hstate_[0].pos;
  if (record_logits) {
    const size_t n = (size_t)B * cfg_.vocab_size;
    recorded_logits.resize(recorded_logits.size() + n);
    CUDA_OK(cudaMemcpy(recorded_logits.data() + recorded_logits.size() - n, drec_.p, n * 4, cudaMemcpyDeviceToHost),
            false);
  }
  cudaEventRecord(ev1_, stream_);
  cudaEventSynchronize(ev1_);
  float ms = 0;
  cudaEventElapsedTime(&ms, ev0_, ev1_);
  perf.decode_ms += ms;
  perf.decode_steps += (int)longest;
  return true;
}

}  // namespace qasr
