/*
 * qwen_asr_ext.h — extensions of libqwen_asr beyond the reference's C-FFI.
 *
 * Each entry names the reference item it exposes. None changes the behaviour of the
 * functions in qwen_asr.h.
 */
#ifndef QWEN_ASR_EXT_H
#define QWEN_ASR_EXT_H

#include "qwen_asr.h"

#ifdef __cplusplus
extern "C" {
#endif

/* Load onto an explicit CUDA device (-1 = $QASR_DEVICE or the current device). */
QwenAsrEngine* qwen_asr_load_model_on_device(const char* model_dir, int32_t device, int32_t verbosity);
/* Message of the last failure on this thread ("" if none). */
const char* qwen_asr_last_error(void);
/* QwenCtx::set_prompt (context.rs:167-175); 0 ok. */
int32_t qwen_asr_set_prompt(QwenAsrEngine* engine, const char* prompt);
/* QwenCtx.past_text_conditioning (context.rs:56; CLI --past-text). */
void qwen_asr_set_past_text(QwenAsrEngine* engine, int32_t on);
/* QwenCtx.skip_silence (context.rs:57; compact_silence, audio.rs:375-479). */
void qwen_asr_set_skip_silence(QwenAsrEngine* engine, int32_t on);
/* Decode weights: 0 = int8 per-row (the reference's decode, decoder.rs:106-118, default),
 * 1 = bf16 (the reference's bf16 matvec family, kernels/mod.rs:630-835). */
int32_t qwen_asr_set_decode_mode(QwenAsrEngine* engine, int32_t mode);
/* Benchmark mode: run exactly n decode steps per segment, ignoring EOS (0 = off). */
void qwen_asr_set_force_n_tokens(QwenAsrEngine* engine, int32_t n);
/* Pushes audio to `count` distinct streams at once: each stream runs exactly the chunks
 * qwen_asr_stream_push would run for it, and the chunks of streams with adjacent KV slots
 * decode as one batch (one weight read per step for all of them). deltas_out[i] receives
 * stream i's delta (NULL when empty; free with qwen_asr_free_string). Returns 0, or -1
 * on error (qwen_asr_last_error). */
int32_t qwen_asr_stream_push_many(QwenAsrEngine* engine, QwenAsrStreamState* const* states,
                                  const float* const* samples, const int32_t* n_samples, int32_t count,
                                  int32_t finalize, char** deltas_out);
/* Transcribes `count` independent segments [starts[i], ends[i]) of one buffer (each padded
 * to 0.5 s like the -S loop, transcribe.rs:374-384), decoding them in batches. texts_out[i]
 * receives segment i's text (free with qwen_asr_free_string). Returns 0, or -1 on error
 * (qwen_asr_last_error). Used to shard one clip's segments over several GPUs. */
int32_t qwen_asr_transcribe_segments(QwenAsrEngine* engine, const float* samples, int64_t n_samples,
                                     const int64_t* starts, const int64_t* ends, int32_t count, char** texts_out);
/* Segmented transcription (segment_sec > 0, past-text conditioning off) decodes up to n
 * segments together, reading the decoder weights once per step for all of them; the text
 * is identical to one-at-a-time decoding. 0 (default) = the largest batch the decode
 * kernels admit for the loaded model, 1 = sequential. Returns the batch that will be used. */
int32_t qwen_asr_set_decode_batch(QwenAsrEngine* engine, int32_t n);
/* 1 (default): decode steps replay a CUDA graph; 0: plain launches. */
void qwen_asr_set_use_graph(QwenAsrEngine* engine, int32_t on);
/* Forced alignment (the reference's align::forced_align, align.rs:207-351; an aligner
 * model directory, classify_num > 0): word (CJK languages: character) timestamps of `text`
 * in `samples` (16 kHz mono). `language` is normalised as the CLI does (main.rs:355). Returns a
 * JSON array [{"text": "...", "start_ms": s, "end_ms": e}, ...] to release with
 * qwen_asr_free_string(), or NULL (qwen_asr_last_error()). */
char* qwen_asr_forced_align(QwenAsrEngine* engine, const float* samples, int64_t n_samples, const char* text,
                            const char* language);
/* Debug: the aligner's units of `text` joined by '\n' (align.rs:44-61); returns the count,
 * -1 on invalid UTF-8 or a short buffer. */
int32_t qwen_asr_debug_align_words(const char* text, const char* language, char* out, int32_t cap);
/* Debug: the aligner's timestamp repair in place (align.rs:140-189). */
void qwen_asr_debug_fix_timestamps(float* ts, int32_t n);
/* Debug: when on, every decode keeps each sequence's f32 logits of its final step (decode
 * runs as plain launches); switching it on or off clears what was kept. */
void qwen_asr_set_record_logits(QwenAsrEngine* engine, int32_t on);
/* Copies up to cap floats of the kept logits (rows of vocab_size, in decode order); returns
 * the number kept. */
int64_t qwen_asr_recorded_logits(QwenAsrEngine* engine, float* out, int64_t cap);
/* Per-op decode profiler (the reference's --profile counters, kernels/mod.rs:78-168): when
 * on, decode steps run as plain launches with CUDA events around each kernel. */
void qwen_asr_set_profile(QwenAsrEngine* engine, int32_t on);
/* Accumulated GPU ms and launch counts per op: qkv, attention, o_proj, gate_up, down,
 * lm_head_argmax. Returns 6. */
int32_t qwen_asr_profile_report(QwenAsrEngine* engine, double* ms, int64_t* counts, int32_t cap);
/* Offline transcription of f32 16 kHz samples already in this engine's device memory
 * (same result as qwen_asr_transcribe_pcm on the same samples). */
char* qwen_asr_transcribe_device(QwenAsrEngine* engine, const float* d_samples, int32_t n_samples);
/* The engine's CUDA stream (cudaStream_t): every kernel of the engine runs on it. */
void* qwen_asr_cuda_stream(QwenAsrEngine* engine);
/* Number of kernels this engine has enqueued so far (graph replays count their nodes). */
int64_t qwen_asr_launch_count(QwenAsrEngine* engine);
/* Kernel timeline of the next decode calls: CTA 0 of every decode kernel records
 * {kind, t_entry, t_after_dependency_wait, t_exit} (GPU %globaltimer, ns); kinds as in
 * qwen_asr_profile_report. Works with the CUDA-graph path. */
void qwen_asr_set_timeline(QwenAsrEngine* engine, int32_t on);
/* Copies the last decode call's timeline (4 values per kernel); returns the value count. */
int64_t qwen_asr_get_timeline(QwenAsrEngine* engine, uint64_t* out, int64_t cap);
/* Generated ids of segment/chunk `segment` of the last call (including the stop token);
 * returns the count (copies at most cap), -1 if out of range. */
int32_t qwen_asr_last_tokens(QwenAsrEngine* engine, int32_t segment, int32_t* out, int32_t cap);
int32_t qwen_asr_last_segments(QwenAsrEngine* engine);
/* Perf counters of the last call (context.rs:67-73 + per-stage GPU times):
 * total_ms, audio_ms, encode_ms, decode_ms, text_tokens, mel_ms, enc_ms, prefill_ms,
 * decode_ms(gpu), decode_steps. Returns the number of values. */
int32_t qwen_asr_get_perf(QwenAsrEngine* engine, double* out, int32_t cap);
/* enc_d, enc_layers, enc_heads, enc_ffn, dec_hidden, dec_layers, dec_heads, dec_kv_heads,
 * dec_inter, vocab, device. */
int32_t qwen_asr_model_info(QwenAsrEngine* engine, int32_t* out, int32_t cap);

/* ---- parity hooks (tests) ---- */
/* mel_spectrogram (audio.rs:273-372): out [n_frames][128] (frame-major). Returns n_frames. */
int32_t qwen_asr_debug_mel(QwenAsrEngine* engine, const float* samples, int32_t n, float* out, int64_t cap);
/* Encoder::forward (encoder.rs:186-358) of mel [n_frames][128]: out [T][dec_hidden]; returns T. */
int32_t qwen_asr_debug_encode(QwenAsrEngine* engine, const float* mel, int32_t n_frames, float* out, int64_t cap);
/* decoder_prefill over rows[0..n_rows-1) then n_steps decoder_forward steps starting from
 * row n_rows-1 (transcribe.rs:171-226). With `forced`, step i+1's input is forced[i]
 * (teacher forcing). out_ids [n_steps]; out_logits [n_steps][vocab] (optional);
 * out_hidden [n_rows][hidden] final prefill hidden states (optional). Returns n_steps. */
int32_t qwen_asr_debug_decode(QwenAsrEngine* engine, const float* rows, int32_t n_rows, const int32_t* forced,
                              int32_t n_steps, int32_t* out_ids, float* out_logits, float* out_hidden);

/* One GEMM of the engine on the current device: C = epi(A[M][K] f32 * B[N][K]^T bf16 bits),
 * epi as the engine's GemmEpi (0 store, 1 +bias, 2 gelu(+bias), 3 resid(+bias)+acc,
 * 4 swiglu -> C[M][N/2]); impl 0 = SIMT FP32 kernel, 1 = tcgen05 tensor-core kernel.
 * Host buffers. Returns 0, or < 0 on error. (Parity hook for the contraction kernels.) */
int32_t qwen_asr_debug_gemm(int32_t M, int32_t N, int32_t K, const float* A, const uint16_t* B, const float* bias,
                            const float* resid, int32_t epi, int32_t impl, float* C);
/* Mean CUDA-event time in ms of `reps` back-to-back tensor-core GEMMs of the given shape and
 * epilogue on the current device (zero operands); timeline (optional, 148 x 8 u64) receives
 * per-CTA %globaltimer stamps of the last launch. Returns 0 or < 0. */
int32_t qwen_asr_debug_gemm_timed(int32_t M, int32_t N, int32_t K, int32_t epi, int32_t reps, float* ms,
                                  uint64_t* timeline);
/* Debug: while dev_buf (device memory, 64 u64) is set, the tensor-core attention kernels write
 * %globaltimer stamps of their phases (one CTA) into it; NULL turns it off. Returns 0. */
int32_t qwen_asr_debug_attn_timeline(uint64_t* dev_buf);
/* Bf16-weight GEMMs that could not run on the tensor cores since the library loaded (each
 * one also failed its stage with an error); 0 in a healthy process. */
int64_t qwen_asr_gemm_fallbacks(void);
/* KV cache (decoder.rs:185-253) of one slot and layer: k, v [kv_heads][n_pos][128] f32 for
 * positions 0..n_pos-1 (slot 0 = the offline path). Returns 0 or -1. */
int32_t qwen_asr_debug_kv(QwenAsrEngine* engine, int32_t slot, int32_t layer, int32_t n_pos, float* k, float* v);
/* Current KV capacity in positions (KvCache::max_seq). */
int32_t qwen_asr_debug_kv_capacity(QwenAsrEngine* engine);
/* Grows the KV cache to hold `needed` positions by doubling, keeping the rows already
 * written (KvCache::grow, decoder.rs:199-231). Returns the new capacity or -1. */
int32_t qwen_asr_debug_grow_kv(QwenAsrEngine* engine, int32_t needed);
/* Device int8 weights of one decoder matrix (which: 0 q/k/v rows [q | k | v], 1 o, 2 gate/up
 * rows interleaved gate0, up0, ..., 3 down, 4 lm_head) as quantised at load
 * (kernels/mod.rs:1805-1829 / kernels/neon.rs:636-694): q [rows][cols], s [rows]. Returns
 * the row count (nothing copied when it exceeds cap_rows) or -1. */
int64_t qwen_asr_debug_quant(QwenAsrEngine* engine, int32_t layer, int32_t which, int8_t* q, float* s,
                             int64_t cap_rows);

/* ---- allocation-free mel front end (no counterpart in the reference) ----
 * For callers that must not allocate device memory during a call: processes holding a
 * fixed device-memory budget, real-time audio threads that may not block in the
 * allocator, or hosts that forbid device allocations after start-up. Computes the same
 * features as qwen_asr_debug_mel (mel_spectrogram, audio.rs:273-372), but from samples
 * already in device memory into a caller-owned device buffer d_mel [F][128] (frame-major,
 * capacity mel_cap floats), F = n_samples / 160, and keeps its intermediate buffers in one
 * library-owned device array (about 4 MB, held on every GPU that loads the library until
 * the process exits). It calls no cudaMalloc/cudaFree. Limit: F <= QWEN_ASR_MEL_NOALLOC_MAX_FRAMES
 * (10 s of 16 kHz audio); longer input returns -1 with a message in qwen_asr_last_error().
 * The first call on a device looks up the array's device address (cudaGetSymbolAddress),
 * so make that first call before any stream capture. All calls share the one array: calls
 * whose GPU work overlaps (other engines or threads on the same device) race and must be
 * serialised by the caller. Runs on the engine's stream and returns after it completes;
 * returns F or -1. */
#define QWEN_ASR_MEL_NOALLOC_MAX_FRAMES 1000
int32_t qwen_asr_mel_noalloc(QwenAsrEngine* engine, const float* d_samples, int32_t n_samples, float* d_mel,
                             int64_t mel_cap);

/* ---- host-only hooks (no GPU needed) ---- */
/* QwenTokenizer::encode (tokenizer.rs:227-279): returns the id count, -2 if unencodable. */
int32_t qwen_asr_debug_tokenize(const char* model_dir, const char* text, int32_t* out, int32_t cap);
/* Concatenated decode_bytes (tokenizer.rs:217-225) of ids; returns the byte count. */
int32_t qwen_asr_debug_detokenize(const char* model_dir, const int32_t* ids, int32_t n, char* out, int32_t cap);
/* parse_wav_buffer (audio.rs:22-91) incl. resample (audio.rs:133-196); returns sample count. */
int64_t qwen_asr_debug_parse_wav(const uint8_t* data, int64_t len, float* out, int64_t cap);
/* Segment start offsets of transcribe_audio (transcribe.rs:253-346); returns the count. */
int32_t qwen_asr_debug_split_points(const float* samples, int64_t n, float segment_sec, float search_sec,
                                    int64_t* out, int32_t cap);
/* compact_silence (audio.rs:375-479) as the host restatement (the oracle's check of the
 * algorithm); returns the kept sample count. */
int64_t qwen_asr_debug_compact_silence(const float* samples, int64_t n, float* out, int64_t cap);
/* The same on the engine's GPU (the path skip_silence takes); NULL out queries the count. */
int64_t qwen_asr_debug_compact_silence_gpu(QwenAsrEngine* e, const float* samples, int64_t n, float* out,
                                           int64_t cap);
/* String::from_utf8_lossy + str::trim as used on transcripts (transcribe.rs:237-238). */
int32_t qwen_asr_debug_lossy_trim(const char* bytes, int32_t n, char* out, int32_t cap);
/* normalize_language (config.rs:167-182); "" when unsupported. */
/* GPU Kaiser-sinc resampling (audio.rs:133-196) of n host samples at from_rate to 16 kHz, the
 * step qwen_asr_transcribe_file / _wav_buffer run on the engine's GPU for non-16 kHz files.
 * out (host, optional) receives the samples when cap is large enough. Returns the output
 * length or -1. */
int64_t qwen_asr_debug_resample(QwenAsrEngine* engine, const float* in, int64_t n, int32_t from_rate, float* out,
                                int64_t cap);
/* 1 when the NUL-terminated bytes are strict UTF-8 as CStr::to_str accepts them (the check
 * qwen_asr_load_model, qwen_asr_transcribe_file and qwen_asr_set_language apply), else 0. */
int32_t qwen_asr_debug_valid_utf8(const char* s);
int32_t qwen_asr_debug_normalize_language(const char* lang, char* out, int32_t cap);

/* ---- multi-GPU pool (no counterpart in c_api.rs; the reference runs one context) ----
 * One engine per GPU, each on its own worker thread. Segmented transcription shards the
 * `-S` segments (transcribe.rs:328-423) over the GPUs longest-first and joins the texts in
 * segment order (transcribe.rs:401-422); with past-text conditioning on, or one segment, the
 * first GPU transcribes alone. n_devices = 0 uses every visible GPU; a device may be listed
 * more than once (several engines on one GPU). */
typedef struct QwenAsrPool QwenAsrPool;
QwenAsrPool* qwen_asr_pool_new(const char* model_dir, const int32_t* devices, int32_t n_devices, int32_t verbosity);
void qwen_asr_pool_free(QwenAsrPool* pool);
int32_t qwen_asr_pool_size(const QwenAsrPool* pool);
/* The engine of worker i (for per-engine settings and statistics); owned by the pool. */
QwenAsrEngine* qwen_asr_pool_engine(QwenAsrPool* pool, int32_t i);
void qwen_asr_pool_set_segment_sec(QwenAsrPool* pool, float sec);
int32_t qwen_asr_pool_set_language(QwenAsrPool* pool, const char* language);
void qwen_asr_pool_set_decode_mode(QwenAsrPool* pool, int32_t mode); /* 0 int8, 1 bf16 */
void qwen_asr_pool_set_force_n_tokens(QwenAsrPool* pool, int32_t n);
void qwen_asr_pool_stream_set_max_new_tokens(QwenAsrPool* pool, int32_t n);
/* Like qwen_asr_transcribe_pcm, the segments spread over the pool's GPUs. */
char* qwen_asr_pool_transcribe_pcm(QwenAsrPool* pool, const float* samples, int32_t n_samples);
/* Like qwen_asr_stream_push_many; stream i runs on worker i % size, so a stream must keep
 * its position in the list from call to call. */
int32_t qwen_asr_pool_stream_push_many(QwenAsrPool* pool, QwenAsrStreamState* const* states,
                                       const float* const* samples, const int32_t* n_samples, int32_t count,
                                       int32_t finalize, char** deltas_out);
/* The pool's segment assignment (host only): worker_of[i] for segment lengths[i] over
 * `workers` workers, longest first to the least-loaded worker. Returns 0 or -1. */
int32_t qwen_asr_debug_assign_longest_first(const int64_t* lengths, int32_t n, int32_t workers, int32_t* worker_of);

#ifdef __cplusplus
}
#endif
#endif /* QWEN_ASR_EXT_H */
