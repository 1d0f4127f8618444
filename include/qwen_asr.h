/*
 * qwen_asr.h — C ABI of libqwen_asr (B200 / sm_100a engine for Qwen3-ASR).
 *
 * Drop-in for the C-FFI of huanglizhuo/QwenASR: every declaration below replaces the
 * `#[no_mangle] extern "C"` function of the same name in crates/qwen-asr/src/c_api.rs
 * (line ranges cited per entry), with the same argument meaning, ownership and error
 * convention: failures return NULL or -1, never abort. Returned strings are NUL-terminated
 * UTF-8 allocated by the library; release them with qwen_asr_free_string().
 *
 * Differences a caller can observe:
 *  - n_threads of qwen_asr_load_model() is accepted and ignored (the math runs on the GPU).
 *    The GPU is $QASR_DEVICE if set, else the calling thread's current CUDA device.
 *  - Each stream keeps its prompt rows in its own device KV slot (up to 32 streams per
 *    engine; beyond that the least recently used stream's slot is reassigned and that
 *    stream re-prefills on its next push). The reference shares one KV cache between all
 *    streams and offline calls (context.rs:34), so interleaving streams there reuses another
 *    stream's rows; here interleaved streams give the same deltas as streams run alone.
 * An engine is not thread-safe: serialise calls on one engine (as the reference's &mut does).
 */
#ifndef QWEN_ASR_H
#define QWEN_ASR_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct QwenAsrEngine QwenAsrEngine;
typedef struct QwenAsrStreamState QwenAsrStreamState;

/* c_api.rs:20-46 — load a model directory (model*.safetensors + vocab.json). */
QwenAsrEngine* qwen_asr_load_model(const char* model_dir, int32_t n_threads, int32_t verbosity);
/* c_api.rs:50-70 — transcribe a 16-bit PCM WAV file. */
char* qwen_asr_transcribe_file(QwenAsrEngine* engine, const char* wav_path);
/* c_api.rs:75-93 — transcribe f32 16 kHz mono samples; NULL if n_samples <= 0. */
char* qwen_asr_transcribe_pcm(QwenAsrEngine* engine, const float* samples, int32_t n_samples);
/* c_api.rs:98-121 — transcribe a whole WAV file held in memory. */
char* qwen_asr_transcribe_wav_buffer(QwenAsrEngine* engine, const uint8_t* wav_data, int32_t wav_len);
/* c_api.rs:125-129 — segment length for long audio (0 = no segmentation). */
void qwen_asr_set_segment_sec(QwenAsrEngine* engine, float sec);
/* c_api.rs:133-148 — force a language ("" = auto); 0 ok, -1 unknown language. */
int32_t qwen_asr_set_language(QwenAsrEngine* engine, const char* language);
/* c_api.rs:152-156 */
void qwen_asr_free_string(char* s);
/* c_api.rs:160-164 */
void qwen_asr_free(QwenAsrEngine* engine);
/* c_api.rs:179-185 */
QwenAsrStreamState* qwen_asr_stream_new(void);
/* c_api.rs:188-193 */
void qwen_asr_stream_free(QwenAsrStreamState* stream);
/* c_api.rs:196-203 */
void qwen_asr_stream_reset(QwenAsrStreamState* stream);
/* c_api.rs:212-245 — append samples, run incremental streaming, return the text delta
 * (NULL when nothing new was emitted). */
char* qwen_asr_stream_push(QwenAsrEngine* engine, QwenAsrStreamState* stream, const float* samples,
                           int32_t n_samples, int32_t finalize);
/* c_api.rs:250-265 — full stable transcript so far (NULL if empty). */
char* qwen_asr_stream_get_result(QwenAsrStreamState* stream);
/* c_api.rs:269-297 — streaming knobs (ignored unless > 0 / >= 0 / >= 0 / > 0). */
void qwen_asr_stream_set_chunk_sec(QwenAsrEngine* engine, float sec);
void qwen_asr_stream_set_rollback(QwenAsrEngine* engine, int32_t tokens);
void qwen_asr_stream_set_unfixed_chunks(QwenAsrEngine* engine, int32_t chunks);
void qwen_asr_stream_set_max_new_tokens(QwenAsrEngine* engine, int32_t tokens);

#ifdef __cplusplus
}
#endif
#endif /* QWEN_ASR_H */
