// Device-resident Qwen3-ASR model and its forward stages on one GPU.
#pragma once
#include <map>
#include <memory>
#include <string>
#include <vector>

#include "common.h"
#include "host.h"
#include "kernels.h"

namespace qasr {

struct EncLayerW {
  __nv_bfloat16* wqkv;  // [3d][d] (q | k | v)
  float* bqkv;          // [3d]
  __nv_bfloat16* wo;
  float* bo;
  float *ln1w, *ln1b, *ln2w, *ln2b;
  __nv_bfloat16 *w1, *w2;
  float *b1, *b2;
};

struct DecLayerW {
  __nv_bfloat16* wqkv;  // [q + 2kv][h]
  __nv_bfloat16* wo;    // [h][q]
  __nv_bfloat16* wgu;   // [2*inter][h], rows interleaved gate0, up0, gate1, ... (decoder.rs:91-104)
  __nv_bfloat16* wdown; // [h][inter]
  int8_t *qqkv, *qo, *qgu, *qdown;
  float *sqkv, *so, *sgu, *sdown;
  float *qn, *kn, *n1, *n2;
};

enum DecodeMode { DECODE_INT8 = 0, DECODE_BF16 = 1 };

// Per-stage timings of the last call, in milliseconds (CUDA events).
struct StagePerf {
  double mel_ms = 0, enc_ms = 0, prefill_ms = 0, decode_ms = 0;
  int decode_steps = 0;
};

class Engine {
 public:
  ~Engine();
  bool load(const std::string& dir, int device, bool trunc_quant);
  const Config& cfg() const { return cfg_; }
  int device() const { return device_; }
  cudaStream_t stream() const { return stream_; }

  // Stage 1: samples (host or device) -> mel [F][128] in device memory. Returns F (0 = too short).
  int mel(const float* samples, int n, bool samples_on_device);
  // Stage 2: mel (device, [F][128]) -> encoder output rows [T][dec_hidden] in enc_out(). Returns T.
  int encode(const float* d_mel, int n_frames);
  // Several mel inputs through the encoder in one pass (rows of input i follow those of
  // inputs < i in enc_out; seq[i] = its row count); returns the total rows (0 on error).
  struct EncInput {
    const float* mel;
    int F;
  };
  int encode_many(const std::vector<EncInput>& in, std::vector<int>& seq);
  float* mel_scratch(size_t floats);  // grow-only device buffer for mels kept across calls
  float* mel_buf() { return mel_.p; }
  // Read-only device tables of the mel front end (Hann window, DFT matrix [408][400],
  // mel filterbank [128][208]).
  const float* hann_table() const { return hann_; }
  const float* dft_table() const { return dft_; }
  const float* mel_filter_table() const { return mel_filt_; }
  float* enc_out() { return enc_.p; }

  // Prompt rows: ids >= 0 are token embeddings, id = -(r+1) is encoder row r of `enc`.
  // Runs decoder_prefill over rows[0, n-1) starting at KV position `start_pos` (rows
  // before start_pos are not recomputed), then prepares the first decode step from the
  // last row. `enc` may be null when no id references it.
  // `slot` selects the KV cache / decode state of one sequence of a batched decode
  // (slot 0 is the one decode() continues).
  bool prefill_ids(const std::vector<int>& ids, const float* d_enc, int start_pos, int slot = 0);
  // Same with prompt embeddings already materialised on the host (streaming LCP path).
  bool prefill_rows(const float* h_rows, int n_rows, int start_pos, int slot = 0);
  // Several sequences' prefills in one pass: the rows every job recomputes are packed into
  // one matrix, so each GEMM reads the weights once for all of them; RoPE, the KV append and
  // attention run per job on its rows and slot. Each job is prefill_ids(ids, d_enc,
  // start_pos, slot) with its encoder rows inside the shared `d_enc`; per-row results equal
  // the single-job call's bit for bit (the GEMM tiles do not depend on the row count).
  struct PrefillJob {
    const std::vector<int>* ids;
    int start_pos;
    int slot;
  };
  bool prefill_many(const std::vector<PrefillJob>& jobs, const float* d_enc);
  // Forced aligner (decoder.rs:649-681, align.rs:275-301): prefill of every prompt row from
  // position 0 (the last row included) into slot 0, then the final RMSNorm and the classify
  // head (classify_num classes) at `rows`; cls[k] = the argmax class of row rows[k] (first
  // maximum).
  bool prefill_classify(const std::vector<int>& ids, const float* d_enc, const std::vector<int>& rows,
                        std::vector<int>& cls);
  // Greedy decode: runs up to max_steps decoder_forward steps from the prepared state and
  // returns the produced ids. With stop_on_eos the loop stops after the first
  // 151643/151645 (inclusive). forced (teacher forcing) gives the input id of step i+1.
  // `slot`: the KV cache / decode state of one sequence (0 = the offline path; batched
  // segments use 0..kDecodeMaxBatch-1; streams own slots from kDecodeMaxBatch up).
  bool decode(int max_steps, bool stop_on_eos, std::vector<int>& out, const std::vector<int>* forced = nullptr,
              std::vector<float>* logits = nullptr, int slot = 0);
  // Batched greedy decode of the sequences prefilled into slots 0..B-1: every step reads
  // the weights once for all B sequences. Runs until every sequence has produced EOS (with
  // stop_on_eos) or max_steps; out[b] holds sequence b's ids exactly as decode() would
  // return them for that sequence alone.
  bool decode_batch(int B, int max_steps, bool stop_on_eos, std::vector<std::vector<int>>& out, int first_slot = 0);
  // Largest B decode_batch accepts for this model (shared-memory bound, <= kDecodeMaxBatch).
  int max_decode_batch();
  void set_decode_mode(DecodeMode m) {
    mode_ = m;
    max_batch_ = 0;
    ++graph_gen_;
  }
  DecodeMode decode_mode() const { return mode_; }
  StagePerf perf;
  bool use_graph = true;
  long launches = 0;  // kernels enqueued by this engine (graph replays count their nodes)
  // Per-op decode profiler (CUDA events around every launch; disables the graph).
  bool profile = false;
  // Debug: every decode keeps each sequence's f32 logits of its last step here (plain
  // launches instead of graphs), so batched and single-sequence decodes can be compared.
  bool record_logits = false;
  std::vector<float> recorded_logits;
  double prof_ms[6] = {0, 0, 0, 0, 0, 0};
  long prof_n[6] = {0, 0, 0, 0, 0, 0};
  std::vector<std::pair<int, cudaEvent_t>> prof_ev_;
  // Kernel timeline (in-kernel %globaltimer stamps; graph-compatible).
  void set_timeline(bool on) { timeline_ = on; ++graph_gen_; }
  std::vector<unsigned long long> last_timeline;

  // Debug: final hidden of prefill rows (after the last layer, before final norm).
  bool copy_prefill_hidden(std::vector<float>& out, int rows);
  // Resamples host samples at `rate` to 16 kHz on the GPU (audio.rs:133-196); returns the
  // device buffer (valid until the next call) and its length in *n_out, or nullptr.
  const float* resample_to_device(const float* h_in, long n, int rate, long* n_out);
  // Silence compaction of host samples on the GPU (audio.rs:375-479, skip_silence): out gets
  // the kept samples, equal to the reference's compact_silence.
  bool compact_silence(const float* h_in, long n, std::vector<float>& out);
  // Debug: K and V rows [kv_heads][n_pos][128] of positions 0..n_pos-1 of one slot and layer.
  bool copy_kv(int slot, int layer, int n_pos, float* k, float* v);
  int kv_capacity() const { return max_seq_; }
  // Debug: grow the KV cache to hold `needed` positions (the doubling path of KvCache::grow).
  bool grow_kv(int needed) {
    cudaSetDevice(device_);
    return ensure_kv(needed);
  }
  // Debug: the int8 rows and f32 row scales of one quantised decoder matrix (which: 0 q/k/v,
  // 1 o, 2 gate/up interleaved, 3 down, 4 lm_head; layer ignored for 4). Returns the row count.
  long copy_quant(int layer, int which, int8_t* q, float* s, long cap_rows);

 private:
  Config cfg_;
  int device_ = 0;
  cudaStream_t stream_ = nullptr;
  DecodeMode mode_ = DECODE_INT8;
  std::vector<void*> allocs_;
  void* dalloc(size_t bytes);
  template <typename T>
  T* dalloc_t(size_t n) { return (T*)dalloc(n * sizeof(T)); }

  // encoder weights
  float *conv1_w = nullptr, *conv1_b = nullptr;
  __nv_bfloat16 *conv2_w = nullptr, *conv3_w = nullptr, *conv_out_w = nullptr;
  float *conv2_b = nullptr, *conv3_b = nullptr;
  std::vector<EncLayerW> enc_layers_;
  float *ln_post_w = nullptr, *ln_post_b = nullptr, *proj1_b = nullptr, *proj2_b = nullptr;
  __nv_bfloat16 *proj1_w = nullptr, *proj2_w = nullptr;
  // decoder weights
  __nv_bfloat16* embed_ = nullptr;  // [vocab][h]
  std::vector<DecLayerW> dec_layers_;
  float* final_norm_ = nullptr;
  const __nv_bfloat16* lm_bf16_ = nullptr;
  int8_t* lm_q_ = nullptr;
  float* lm_s_ = nullptr;
  // tables
  float *hann_ = nullptr, *dft_ = nullptr, *mel_filt_ = nullptr, *rope_cos_ = nullptr, *rope_sin_ = nullptr;
  float* pe_ = nullptr;
  int rope_cap_ = 0;

  // activations (grow-only)
  DevBuf<float> samples_, frames_, spec_, power_, mel_;
  DevBuf<int> gmax_;
  DevBuf<float> act1_, act2_, act3_, cols_, x_enc_, xn_enc_, qkv_enc_, att_enc_, mid_enc_, enc_;
  DevBuf<int> win_starts_;
  DevBuf<float> px_, pxn_, pqkv_, patt_, pmid_;
  DevBuf<int> ids_;
  DevBuf<float> mel_keep_, cls_x_, cls_xn_, cls_logits_;
  DevBuf<int> cls_ids_, cls_out_;
  // KV cache [slot][layers][kv][max_seq][128] f32
  DevBuf<float> kc_, vc_;
  int max_seq_ = 0;
  int kv_len_ = 0;
  int slots_ = 1;
  bool ensure_kv(int needed);
  bool ensure_slots(int n);
  size_t kv_slot_stride() const { return (size_t)cfg_.dec_layers * cfg_.dec_kv_heads * max_seq_ * 128; }
  // decode scratch
  DevBuf<float> dx_, dqkv_, dattn_, dffn_, dpart_, dlogits_, drec_;
  DevBuf<int> dticket_, dam_ticket_, dtokens_, dforced_, derr_;
  DevBuf<unsigned long long> dam_part_;
  DevBuf<unsigned char> dstaged_;  // batched steps: each matvec's inputs, staged once
  DevBuf<StepState> dstate_;
  bool timeline_ = false;
  DevBuf<unsigned long long> dtl_;
  DevBuf<int> dtl_count_;
  StepState* hstate_ = nullptr;  // pinned [kDecodeMaxBatch]
  int* htokens_ = nullptr;       // pinned [kDecodeMaxBatch][tokens_ld_]
  int tokens_ld_ = 0;            // per-sequence capacity of dtokens_ / htokens_
  int tokens_rows_ = 0;
  bool ensure_tokens(int max_steps, int B);
  int max_batch_ = 0;
  bool enqueue_step(const DecodeArgs& a);  // one single-sequence decode step (false: not planned)
  int decode_step_launches_1() const;
  // decode graphs, one per batch size; valid while built_gen_[B] == graph_gen_
  cudaGraphExec_t graph_exec_[kDecodeMaxBatch + 1] = {};
  unsigned graph_gen_ = 1, built_gen_[kDecodeMaxBatch + 1] = {};
  bool graph_for(int B);
  std::vector<const void*> pw_qkv_, pw_o_, pw_gu_, pw_down_;
  std::vector<const float*> ps_qkv_, ps_o_, ps_gu_, ps_down_, pn1_, pn2_, pqn_, pkn_;
  DecodeArgs dargs(const int* forced, float* logits, int slot = 0);
  std::vector<cudaGraphExec_t> slot_graph_;  // single-sequence step graphs of slots >= 1
  std::vector<unsigned> slot_graph_gen_;
  bool graph_for_slot(int slot);
  std::map<int, std::pair<cudaGraphExec_t, unsigned>> run_graphs_;  // batched steps of slot runs (first slot > 0)
  bool run_prefill(int n_rows, int start_pos, int slot = 0);  // rows already in px_
  struct RowBlock {
    int off, S, start, slot;
  };
  bool prefill_layers(float* x, int R, const std::vector<RowBlock>& blocks);
  bool gemm_stage_ok(long fallbacks_before);
  static bool simt_attention();  // QASR_ATTN=simt: the SIMT attention kernels (A/B checks)
  // bf16 planes (hi/mid/lo) of GEMM inputs written by their producers
  DevBuf<__nv_bfloat16> pl_a_, pl_b_, pl_c_, pl_conv_;
  DevBuf<float> rs_in_, rs_out_;  // resampler input / output
  DevBuf<float> cs_in_, cs_out_;  // silence compaction input / output
  DevBuf<unsigned char> cs_scratch_;
  DevBuf<long long> cs_count_;
  DevBuf<int> prow_pos_;        // packed prefill rows: KV position
  DevBuf<long long> prow_kv_;   // packed prefill rows: KV slot offset (floats)
  cudaEvent_t ev0_ = nullptr, ev1_ = nullptr;
};

}  // namespace qasr
