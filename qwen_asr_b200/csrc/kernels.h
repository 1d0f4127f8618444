// Launchers for the engine's CUDA kernels (sm_100a). All launches are asynchronous on
// the given stream; pointer arguments are device pointers unless stated otherwise.
#pragma once
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cstdint>
#include <vector>

namespace qasr {

// ---------------------------------------------------------------- GEMM
// C[m][n] (ldc) = epilogue( sum_k A[m][k] * B[n][k] ), A f32 [M][lda], B bf16 or f32
// [N][ldb]. K must be a multiple of 16 and rows of A/B must be 16-byte aligned.
enum GemmEpi : int {
  EPI_STORE = 0,       // v = acc
  EPI_BIAS = 1,        // v = acc + bias[n]
  EPI_BIAS_GELU = 2,   // v = gelu_tanh(acc + bias[n])
  EPI_RESID = 3,       // v = (resid[m][n] + bias[n]?) + acc   (resid may alias C)
  EPI_SWIGLU = 4,      // columns (2j, 2j+1) = (gate, up) -> C[m][j] = silu(gate) * up
  EPI_LOG10_MAX = 5,   // v = log10(max(acc, 1e-10)); atomic max into *gmax (ordered int)
};

struct GemmArgs {
  int M = 0, N = 0, K = 0;
  const float* A = nullptr;
  int lda = 0;
  const void* B = nullptr;
  bool b_is_f32 = false;
  int ldb = 0;
  float* C = nullptr;
  int ldc = 0;
  int epi = EPI_STORE;
  const float* bias = nullptr;   // [N] (EPI_BIAS, EPI_BIAS_GELU, optional for EPI_RESID)
  const float* resid = nullptr;  // [M][ldr] for EPI_RESID
  int ldr = 0;
  int* gmax = nullptr;           // EPI_LOG10_MAX
  // Tensor-core path only. a_split: A already as bf16 planes hi/mid/lo [3][a_split_plane]
  // of rows [M][a_split_ld] (written by the producing kernel; A is then only read by the
  // SIMT path). c_split: also write the result as planes (input of the next GEMM).
  const __nv_bfloat16* a_split = nullptr;
  int a_split_ld = 0;
  long long a_split_plane = 0;
  __nv_bfloat16* c_split = nullptr;
  int c_split_ld = 0;
  long long c_split_plane = 0;
  // K split policy: 0 = automatic from (N, K), -1 = never split, > 0 = that many splits.
  // Never depends on M, so per-row results do not depend on the row count.
  int split_k = 0;
};
// Bytes of a plane buffer for `rows` x `cols` (three bf16 planes).
inline size_t split_planes_elems(size_t rows, size_t cols) { return 3 * rows * cols; }
// Returns false (and records the error) when a bf16-weight GEMM could not run on the
// tensor cores; the result is then computed by the SIMT kernel from the f32 A, and
// gemm_tc_fallbacks() counts it.
bool gemm(const GemmArgs& a, cudaStream_t s);
// QASR_GEMM=simt: every GEMM runs on the SIMT f32 kernel (producers must then write f32 A).
bool gemm_simt_forced();
// Plain SIMT FP32 reference GEMM (kept for parity tests of the tensor-core path).
void gemm_simt(const GemmArgs& a, cudaStream_t s);
// tcgen05/TMEM tensor-core GEMM (bf16 B, f32 A as three bf16 planes). Returns false
// when the shape is unsupported.
bool gemm_tc(const GemmArgs& a, cudaStream_t s);
bool gemm_tc_available();
// Bf16-weight GEMMs that had to leave the tensor cores since the library loaded.
long gemm_tc_fallbacks();
// Debug: the next tensor-core GEMM launches write 8 %globaltimer stamps per CTA (148 x 8) here.
void gemm_tc_set_timeline(unsigned long long* dev_buf);
void gemm_tc_note_fallback();
// K splits the tensor-core GEMM uses for an (N, K) call under `policy` (GemmArgs::split_k).
int gemm_split_k(int N, int K, int policy);
// f32 rows [M][lda] -> bf16 planes hi/mid/lo at out, out + plane, out + 2 * plane (rows of K).
void split3_rows(const float* A, int lda, int M, int K, __nv_bfloat16* out, long long plane, cudaStream_t s);
// Nonzero when a bounded wait inside the tensor-core GEMM gave up (clears the flag).
int gemm_tc_error();
// 2-D TMA map over a row-major matrix of 16-bit elements [rows][cols], box = box_cols x
// box_rows; out-of-range boxes read zeros. swizzle128: 128-byte swizzle (box_cols = 64),
// the K-major operand layout of tcgen05.mma.
bool make_tma_2d_u16(void* map /* CUtensorMap* */, const void* base, int rows, int cols, int box_cols,
                     int box_rows, bool swizzle128 = false);

// ---------------------------------------------------------------- mel front end
// samples [n] -> windowed frames [F][400] (reflect padding, periodic Hann).
void mel_frames(const float* samples, int n, int n_frames, const float* hann, float* frames, cudaStream_t s);
// spec [F][ld_spec] (re 0..200, im 201..401) -> power [F][ld_pow] (cols >= 201 zeroed)
void mel_power(const float* spec, int ld_spec, int n_frames, float* power, int ld_pow, cudaStream_t s);
void mel_reset_max(int* gmax, cudaStream_t s);
// logmel [F][128] in place: (max(v, gmax - 8) + 4) / 4
void mel_normalize(float* logmel, int n_frames, const int* gmax, cudaStream_t s);

// Kaiser-sinc resampling (audio.rs:133-196) of n samples at from_rate into
// resampled_length(n, from_rate, to_rate) samples at to_rate; device buffers.
long resampled_length(long n, int from_rate, int to_rate);
void resample_device(const float* in, long n, int from_rate, int to_rate, float* out, cudaStream_t s);

// Silence compaction (audio.rs:375-479) of in[n] into out (capacity n) on the GPU; d_count[2]
// receives {kept samples, 1 if nothing was kept and the first 0.5 s was copied}. scratch holds
// compact_silence_scratch(n) bytes.
size_t compact_silence_scratch(long n);
void compact_silence_device(const float* in, long n, float* out, void* scratch, long long* d_count, cudaStream_t s);

// ---------------------------------------------------------------- encoder
// conv2d1 (1 -> 480, 3x3 s2 p1) + bias + GELU on `n_chunks` chunks of width w taken from
// mel [F][128] starting at frame f0 + c*cw; output channels-last [c][64][w1][480].
void conv1_gelu(const float* mel, int n_frames, int f0, int cw, int n_chunks, int w,
                const float* w1, const float* b1, float* out, cudaStream_t s);
// im2col for a 3x3 s2 p1 conv over channels-last input [c][H][W][480]; rows ordered
// (c, oh, ow) or, with col_major_rows, (c, ow, oh); columns k = (ki*3+kj)*480 + ic.
// planes (optional): write the columns as the tensor-core GEMM's bf16 planes [3][plane]
// instead of f32 `cols`.
void im2col_s2(const float* in, int n_chunks, int H, int W, float* cols, bool col_major_rows,
               cudaStream_t s, __nv_bfloat16* planes = nullptr, long long plane = 0);
void add_pe_rows(float* x, int rows, int d, int period, const float* pe, cudaStream_t s);
// planes (optional): the normalised rows also as bf16 planes [3][plane] of rows [rows][d].
void layer_norm_rows(const float* x, float* y, int rows, int d, const float* w, const float* b, float eps,
                     cudaStream_t s, __nv_bfloat16* planes = nullptr, long long plane = 0);
// Windowed bidirectional attention; qkv [T][3d] (q | k | v), out [T][d].
void window_attention(const float* qkv, float* out, int T, int d, int n_heads, const int* win_starts,
                      int n_windows, int max_win, float scale, cudaStream_t s);

// Tensor-core (tcgen05) attention, f32-level accuracy (attn_tc.cu). Optional `planes`: the
// output also as bf16 planes [3][plane] (the o-projection GEMM's A). Return false when the
// shape is outside the kernel (head_dim != 64 or a window above 128 rows for the encoder).
bool window_attention_tc(const float* qkv, float* out, __nv_bfloat16* planes, long long plane, int d, int n_heads,
                         int head_dim, const int* win_starts, int n_windows, int max_win, float scale,
                         cudaStream_t s);
// Prefill attention of several sequences in one launch: block b is packed rows
// [off, off + S) at KV positions start.. in KV slot `slot`. A query tile whose keys exceed
// the key chunk is split over several CTAs and merged in split order (deterministic: the
// split depends only on the sequence's own positions). Measured on C2, C3 and C5 the split
// never paid for its partial round trip (e.g. C3 prefill 14.9 ms unsplit, 16.1 ms at 256-key
// chunks), so by default tiles are not split; QASR_ATTN_KEY_CHUNK=<keys> enables it.
constexpr int kAttnKeyChunk = 1 << 30;
struct AttnBlock {
  int off, S, start, slot;
};
struct AttnPlan {
  const void* items = nullptr;  // device work items
  int n_items = 0;
  float* ws = nullptr;
  int* tickets = nullptr;
};
// Builds and uploads the work items of `blocks` (the same for every layer of one prefill).
bool prefill_attention_plan(const std::vector<AttnBlock>& blocks, int n_heads, size_t kv_slot_stride,
                            cudaStream_t s, AttnPlan& plan);
// kc / vc: slot 0's cache base; kv_layer_off: floats to the layer within a slot.
bool prefill_attention_tc(const AttnPlan& plan, const float* qkv, int n_heads, int n_kv, const float* kc,
                          const float* vc, long long kv_layer_off, int max_seq, float scale, float* out,
                          __nv_bfloat16* planes, long long plane, cudaStream_t s);
// Nonzero when a bounded wait inside the attention kernels gave up (clears the flag).
int attn_tc_error();
// Debug: attention launches stamp phase times (64 u64) of one CTA here while set.
void attn_tc_set_timeline(unsigned long long* dev_buf);

// ---------------------------------------------------------------- decoder
void rms_norm_rows(const float* x, float* y, int rows, int d, const float* w, float eps, cudaStream_t s,
                   __nv_bfloat16* planes = nullptr, long long plane = 0);
// Prefill: per-head RMSNorm + NeoX RoPE of q/k rows in qkv [S][q_dim + 2*kv_dim] at
// positions start..start+S-1, then writes k/v into the f32 cache
// [kv_heads][max_seq][128] of this layer.
void prefill_qk_rope_kv(float* qkv, int S, int start, int n_heads, int n_kv, const float* qn, const float* kn,
                        float eps, const float* rope_cos, const float* rope_sin, float* kc, float* vc,
                        int max_seq, cudaStream_t s);
// Same over R packed rows of several sequences: row r at KV position row_pos[r], its K/V
// written at kc / vc + row_kv[r] (the row's slot offset; kc / vc: slot 0 of the layer).
void prefill_qk_rope_kv_packed(float* qkv, int R, const int* row_pos, const long long* row_kv, int n_heads, int n_kv,
                               const float* qn, const float* kn, float eps, const float* rope_cos,
                               const float* rope_sin, float* kc, float* vc, int max_seq, cudaStream_t s);
// Causal GQA attention of S queries at positions start.. over the cache; out [S][n_heads*128].
void prefill_attention(const float* qkv, int S, int start, int n_heads, int n_kv, const float* kc,
                       const float* vc, int max_seq, float scale, float* out, cudaStream_t s);
// Gathers prompt rows: row r = ids[r] >= 0 ? embed[ids[r]] : enc[-ids[r]-1].
void gather_embeds(const int* ids, int rows, const __nv_bfloat16* embed, const float* enc, int d, float* out,
                   cudaStream_t s);
// Per-row argmax of f32 [rows][n] (the first index of the maximum, as align.rs:290-301's
// strictly-greater scan picks it).
void rows_argmax(const float* x, int rows, int n, int* out, cudaStream_t s);
// Per-row symmetric int8 quantisation of a bf16 [rows][cols] matrix (load time).
void quantize_rows_int8(const __nv_bfloat16* w, int rows, int cols, bool truncate, int8_t* q, float* scale,
                        cudaStream_t s);

// Decode-step state living in device memory so that one CUDA graph serves every step.
struct StepState {
  int pos;         // KV position of the token being computed
  int step;        // index into tokens[]
  int cur_token;   // input token id of this step; < 0: x already holds the input row
  int forced_mode; // teacher forcing: input token of step i+1 comes from forced[i]
};

struct DecodeArgs {
  // model shape
  int hidden, q_heads, kv_heads, inter, vocab, max_seq;
  float eps;
  bool int8;
  // per-layer weights (arrays of device pointers, host-side)
  const void* const* w_qkv;    // [layers] int8 or bf16 [q+2kv][hidden]
  const float* const* s_qkv;   // [layers] int8 scales
  const void* const* w_o;
  const float* const* s_o;
  const void* const* w_gu;     // interleaved gate/up rows
  const float* const* s_gu;
  const void* const* w_down;
  const float* const* s_down;
  const float* const* n1;
  const float* const* n2;
  const float* const* qn;
  const float* const* kn;
  const void* lm_w;            // int8 or bf16 [vocab][hidden]
  const float* lm_s;
  const float* final_norm;
  const __nv_bfloat16* embed;
  const float* rope_cos;
  const float* rope_sin;
  float* k_cache;              // [layers][kv][max_seq][128]
  float* v_cache;
  int layers;
  // scratch
  float* x;        // [hidden] residual stream
  float* qkv;      // [batch][q_dim + 2 kv_dim] projected q/k/v (split q/k/v path)
  float* attn;     // [q_dim]
  float* ffn;      // [inter]
  float* part;     // attention split partials
  int* ticket;     // [kv_heads] arrival counters (zero at rest)
  float* amax_part;
  int* am_ticket;  // [1]
  unsigned long long* am_part;  // argmax partials
  StepState* st;
  int* tokens;     // [max tokens] output ids
  const int* forced;  // teacher-forced ids or nullptr
  float* logits;   // optional [vocab] f32 logits of the last step (debug)
  int* err;        // device error flag (bounded waits that gave up)
  // Optional host hook called after each launch (kind: 0 qkv, 1 attention, 2 o-proj,
  // 3 gate/up, 4 down, 5 lm_head) - used by the per-op profiler.
  void (*on_launch)(void* ctx, int kind) = nullptr;
  void* hook_ctx = nullptr;
  // Optional timeline: CTA 0 of every kernel appends {kind, t_entry, t_after_wait, t_exit}
  // (%globaltimer ns) at tl[4 * atomicAdd(tl_count, 1)].
  unsigned long long* tl = nullptr;
  int* tl_count = nullptr;
  // Batched step: `batch` sequences (<= kDecodeMaxBatch) share every weight read. x, attn,
  // ffn, logits, st and am_part hold one row per sequence; sequence b's KV cache starts
  // kv_slot_stride floats after sequence b-1's, and its tokens at tokens + b * tokens_ld.
  int batch = 1;
  size_t kv_slot_stride = 0;
  int tokens_ld = 0;
  // Batched steps: device buffer of decode_staged_bytes() where each matvec's inputs are
  // staged once (stage_kernel) instead of by every CTA; null stages in every CTA.
  void* staged = nullptr;
};
constexpr int kDecodeMaxBatch = 8;
constexpr int kMaxSlots = 64;  // KV slots / decode states an engine can hold
// Largest batch the decode kernels' shared memory admits for this model shape.
int decode_max_batch(int hidden, int inter, int q_heads, int kv_heads, bool int8);
// Bytes of DecodeArgs::staged for these widths, and whether batched steps use it
// (QASR_STAGE_ONCE=0 turns it off); kernels a batched step launches.
size_t decode_staged_bytes(int hidden, int q_dim, int inter);
bool decode_stage_once();
int decode_batched_step_launches(int layers, bool int8);
// Whether a single-sequence step projects q/k/v with a separate matvec (5 kernels per layer).
bool decode_split_qkv(int hidden, int q_heads, int kv_heads, bool int8);
// Per-device kernel attributes (dynamic shared memory limits); call once per device.
void decode_kernels_init();
void enc_kernels_init();
// Enqueues one full decode step (embedding -> layers -> lm_head argmax).
// false (with the reason in last_error) when a launch of the step could not be planned or
// was refused; the caller must not use the step's results.
bool decode_step(const DecodeArgs& a, cudaStream_t s);

}  // namespace qasr
