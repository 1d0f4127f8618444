"""Python binding of libqwen_asr (the B200 Qwen3-ASR engine) over its C ABI.

Mirrors the reference's public surface (crates/qwen-asr/src/c_api.rs and the Rust API
QwenCtx::load / transcribe / transcribe_audio / StreamState / stream_push_audio): an
`Engine` owns one loaded model on one GPU; `Stream` is an incremental streaming state.
Every call goes through ctypes into the CUDA library; there is no CPU fallback — if the
library is missing, importing `lib()` raises.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libqwen_asr.so")
_lib = None

_F32P = C.POINTER(C.c_float)
_I32P = C.POINTER(C.c_int32)
_I64P = C.POINTER(C.c_int64)
_U8P = C.POINTER(C.c_uint8)
_VP = C.c_void_p

# name: (restype, argtypes)
SIGNATURES = {
    "qwen_asr_load_model": (_VP, [C.c_char_p, C.c_int32, C.c_int32]),
    "qwen_asr_transcribe_file": (_VP, [_VP, C.c_char_p]),
    "qwen_asr_transcribe_pcm": (_VP, [_VP, _F32P, C.c_int32]),
    "qwen_asr_transcribe_wav_buffer": (_VP, [_VP, _U8P, C.c_int32]),
    "qwen_asr_set_segment_sec": (None, [_VP, C.c_float]),
    "qwen_asr_set_language": (C.c_int32, [_VP, C.c_char_p]),
    "qwen_asr_free_string": (None, [_VP]),
    "qwen_asr_free": (None, [_VP]),
    "qwen_asr_stream_new": (_VP, []),
    "qwen_asr_stream_free": (None, [_VP]),
    "qwen_asr_stream_reset": (None, [_VP]),
    "qwen_asr_stream_push": (_VP, [_VP, _VP, _F32P, C.c_int32, C.c_int32]),
    "qwen_asr_stream_get_result": (_VP, [_VP]),
    "qwen_asr_stream_set_chunk_sec": (None, [_VP, C.c_float]),
    "qwen_asr_stream_set_rollback": (None, [_VP, C.c_int32]),
    "qwen_asr_stream_set_unfixed_chunks": (None, [_VP, C.c_int32]),
    "qwen_asr_stream_set_max_new_tokens": (None, [_VP, C.c_int32]),
    # extensions
    "qwen_asr_load_model_on_device": (_VP, [C.c_char_p, C.c_int32, C.c_int32]),
    "qwen_asr_last_error": (C.c_char_p, []),
    "qwen_asr_set_prompt": (C.c_int32, [_VP, C.c_char_p]),
    "qwen_asr_set_past_text": (None, [_VP, C.c_int32]),
    "qwen_asr_set_skip_silence": (None, [_VP, C.c_int32]),
    "qwen_asr_set_decode_mode": (C.c_int32, [_VP, C.c_int32]),
    "qwen_asr_set_force_n_tokens": (None, [_VP, C.c_int32]),
    "qwen_asr_set_use_graph": (None, [_VP, C.c_int32]),
    "qwen_asr_set_decode_batch": (C.c_int32, [_VP, C.c_int32]),
    "qwen_asr_stream_push_many": (C.c_int32, [_VP, C.POINTER(C.c_void_p), C.POINTER(C.c_void_p), _I32P, C.c_int32,
                                              C.c_int32, C.POINTER(C.c_void_p)]),
    "qwen_asr_transcribe_segments": (C.c_int32, [_VP, _F32P, C.c_int64, C.POINTER(C.c_int64), C.POINTER(C.c_int64),
                                                 C.c_int32, C.POINTER(C.c_void_p)]),
    "qwen_asr_last_tokens": (C.c_int32, [_VP, C.c_int32, _I32P, C.c_int32]),
    "qwen_asr_set_profile": (None, [_VP, C.c_int32]),
    "qwen_asr_set_record_logits": (None, [_VP, C.c_int32]),
    "qwen_asr_recorded_logits": (C.c_int64, [_VP, C.POINTER(C.c_float), C.c_int64]),
    "qwen_asr_set_timeline": (None, [_VP, C.c_int32]),
    "qwen_asr_transcribe_device": (_VP, [_VP, C.c_void_p, C.c_int32]),
    "qwen_asr_cuda_stream": (C.c_void_p, [_VP]),
    "qwen_asr_launch_count": (C.c_int64, [_VP]),
    "qwen_asr_debug_gemm": (C.c_int32, [C.c_int32, C.c_int32, C.c_int32, _F32P, C.POINTER(C.c_uint16), _F32P,
                                         _F32P, C.c_int32, C.c_int32, _F32P]),
    "qwen_asr_gemm_fallbacks": (C.c_int64, []),
    "qwen_asr_debug_resample": (C.c_int64, [_VP, _F32P, C.c_int64, C.c_int32, _F32P, C.c_int64]),
    "qwen_asr_pool_new": (_VP, [C.c_char_p, _I32P, C.c_int32, C.c_int32]),
    "qwen_asr_pool_free": (None, [_VP]),
    "qwen_asr_pool_size": (C.c_int32, [_VP]),
    "qwen_asr_pool_engine": (_VP, [_VP, C.c_int32]),
    "qwen_asr_pool_set_segment_sec": (None, [_VP, C.c_float]),
    "qwen_asr_pool_set_language": (C.c_int32, [_VP, C.c_char_p]),
    "qwen_asr_pool_set_decode_mode": (None, [_VP, C.c_int32]),
    "qwen_asr_pool_set_force_n_tokens": (None, [_VP, C.c_int32]),
    "qwen_asr_pool_stream_set_max_new_tokens": (None, [_VP, C.c_int32]),
    "qwen_asr_pool_transcribe_pcm": (_VP, [_VP, _F32P, C.c_int32]),
    "qwen_asr_pool_stream_push_many": (C.c_int32, [_VP, C.POINTER(C.c_void_p), C.POINTER(_F32P), _I32P, C.c_int32,
                                                   C.c_int32, C.POINTER(C.c_void_p)]),
    "qwen_asr_debug_assign_longest_first": (C.c_int32, [_I64P, C.c_int32, C.c_int32, _I32P]),
    "qwen_asr_debug_attn_timeline": (C.c_int32, [C.c_void_p]),
    "qwen_asr_debug_gemm_timed": (C.c_int32, [C.c_int32, C.c_int32, C.c_int32, C.c_int32, C.c_int32,
                                              C.POINTER(C.c_float), C.POINTER(C.c_uint64)]),
    "qwen_asr_debug_valid_utf8": (C.c_int32, [C.c_char_p]),
    "qwen_asr_debug_kv": (C.c_int32, [_VP, C.c_int32, C.c_int32, C.c_int32, _F32P, _F32P]),
    "qwen_asr_debug_kv_capacity": (C.c_int32, [_VP]),
    "qwen_asr_debug_grow_kv": (C.c_int32, [_VP, C.c_int32]),
    "qwen_asr_debug_quant": (C.c_int64, [_VP, C.c_int32, C.c_int32, C.POINTER(C.c_int8), _F32P, C.c_int64]),
    "qwen_asr_mel_noalloc": (C.c_int32, [_VP, C.c_void_p, C.c_int32, C.c_void_p, C.c_int64]),
    "qwen_asr_get_timeline": (C.c_int64, [_VP, C.POINTER(C.c_uint64), C.c_int64]),
    "qwen_asr_profile_report": (C.c_int32, [_VP, C.POINTER(C.c_double), _I64P, C.c_int32]),
    "qwen_asr_last_segments": (C.c_int32, [_VP]),
    "qwen_asr_get_perf": (C.c_int32, [_VP, C.POINTER(C.c_double), C.c_int32]),
    "qwen_asr_model_info": (C.c_int32, [_VP, _I32P, C.c_int32]),
    "qwen_asr_debug_mel": (C.c_int32, [_VP, _F32P, C.c_int32, _F32P, C.c_int64]),
    "qwen_asr_debug_encode": (C.c_int32, [_VP, _F32P, C.c_int32, _F32P, C.c_int64]),
    "qwen_asr_debug_decode": (C.c_int32, [_VP, _F32P, C.c_int32, _I32P, C.c_int32, _I32P, _F32P, _F32P]),
    "qwen_asr_debug_tokenize": (C.c_int32, [C.c_char_p, C.c_char_p, _I32P, C.c_int32]),
    "qwen_asr_debug_detokenize": (C.c_int32, [C.c_char_p, _I32P, C.c_int32, C.c_char_p, C.c_int32]),
    "qwen_asr_debug_parse_wav": (C.c_int64, [_U8P, C.c_int64, _F32P, C.c_int64]),
    "qwen_asr_debug_split_points": (C.c_int32, [_F32P, C.c_int64, C.c_float, C.c_float, _I64P, C.c_int32]),
    "qwen_asr_debug_compact_silence": (C.c_int64, [_F32P, C.c_int64, _F32P, C.c_int64]),
    "qwen_asr_debug_compact_silence_gpu": (C.c_int64, [_VP, _F32P, C.c_int64, _F32P, C.c_int64]),
    "qwen_asr_debug_lossy_trim": (C.c_int32, [C.c_char_p, C.c_int32, C.c_char_p, C.c_int32]),
    "qwen_asr_debug_normalize_language": (C.c_int32, [C.c_char_p, C.c_char_p, C.c_int32]),
    "qwen_asr_forced_align": (_VP, [_VP, _F32P, C.c_int64, C.c_char_p, C.c_char_p]),
    "qwen_asr_debug_align_words": (C.c_int32, [C.c_char_p, C.c_char_p, C.c_char_p, C.c_int32]),
    "qwen_asr_debug_fix_timestamps": (None, [C.POINTER(C.c_float), C.c_int32]),
}


def lib():
    """Loads libqwen_asr.so (raises if it has not been built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"{LIB_PATH} is missing: build it with `python -m qwen_asr_b200.build`")
        L = C.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def _f32(a):
    a = np.ascontiguousarray(a, dtype=np.float32)
    return a, a.ctypes.data_as(_F32P)


def _take_string(ptr):
    if not ptr:
        return None
    s = C.string_at(ptr).decode("utf-8")
    lib().qwen_asr_free_string(ptr)
    return s


def last_error() -> str:
    return (lib().qwen_asr_last_error() or b"").decode("utf-8", "replace")


class Engine:
    """QwenCtx equivalent on one GPU (context.rs:86-163 via c_api.rs:20-46)."""

    def __init__(self, model_dir: str, device: int = -1, verbosity: int = 0):
        self._h = lib().qwen_asr_load_model_on_device(model_dir.encode(), device, verbosity)
        if not self._h:
            raise RuntimeError(f"qwen_asr_load_model failed: {last_error()}")

    def close(self):
        if getattr(self, "_h", None):
            lib().qwen_asr_free(self._h)
            self._h = None

    def __del__(self):
        self.close()

    # --- reference C-FFI surface ---
    def transcribe_pcm(self, samples) -> str | None:
        a, p = _f32(samples)
        return _take_string(lib().qwen_asr_transcribe_pcm(self._h, p, len(a)))

    def forced_align(self, samples, text: str, language: str = "English") -> list | None:
        """Word (CJK: character) timestamps of `text` in `samples` with an aligner model:
        [{"text", "start_ms", "end_ms"}, ...], or None (see last_error())."""
        import json
        a, p = _f32(samples)
        s = _take_string(lib().qwen_asr_forced_align(self._h, p, len(a), text.encode(), language.encode()))
        return None if s is None else json.loads(s)

    def transcribe_file(self, path: str) -> str | None:
        return _take_string(lib().qwen_asr_transcribe_file(self._h, path.encode()))

    def transcribe_wav_buffer(self, data: bytes) -> str | None:
        buf = (C.c_uint8 * len(data)).from_buffer_copy(data)
        return _take_string(lib().qwen_asr_transcribe_wav_buffer(self._h, buf, len(data)))

    def set_segment_sec(self, sec: float):
        lib().qwen_asr_set_segment_sec(self._h, sec)

    def set_language(self, lang: str) -> int:
        return lib().qwen_asr_set_language(self._h, lang.encode())

    def stream_set_chunk_sec(self, sec):
        lib().qwen_asr_stream_set_chunk_sec(self._h, sec)

    def stream_set_rollback(self, n):
        lib().qwen_asr_stream_set_rollback(self._h, n)

    def stream_set_unfixed_chunks(self, n):
        lib().qwen_asr_stream_set_unfixed_chunks(self._h, n)

    def stream_set_max_new_tokens(self, n):
        lib().qwen_asr_stream_set_max_new_tokens(self._h, n)

    # --- extensions ---
    def set_prompt(self, prompt: str) -> int:
        return lib().qwen_asr_set_prompt(self._h, prompt.encode())

    def set_past_text(self, on: bool):
        lib().qwen_asr_set_past_text(self._h, int(on))

    def set_skip_silence(self, on: bool):
        lib().qwen_asr_set_skip_silence(self._h, int(on))

    def set_decode_mode(self, mode: str):
        if lib().qwen_asr_set_decode_mode(self._h, {"int8": 0, "bf16": 1}[mode]) != 0:
            raise ValueError(mode)

    def set_force_n_tokens(self, n: int):
        lib().qwen_asr_set_force_n_tokens(self._h, n)

    def transcribe_segments(self, samples, bounds) -> list[str | None]:
        """Texts of the independent segments [a, b) of `samples`, decoded in batches."""
        a, p = _f32(samples)
        k = len(bounds)
        st = (C.c_int64 * max(k, 1))(*[int(s) for s, _ in bounds])
        en = (C.c_int64 * max(k, 1))(*[int(e) for _, e in bounds])
        out = (C.c_void_p * max(k, 1))()
        if lib().qwen_asr_transcribe_segments(self._h, p, len(a), st, en, k, out) != 0:
            raise RuntimeError(last_error())
        return [_take_string(out[i]) for i in range(k)]

    def set_decode_batch(self, n: int) -> int:
        return lib().qwen_asr_set_decode_batch(self._h, n)

    def set_use_graph(self, on: bool):
        lib().qwen_asr_set_use_graph(self._h, int(on))

    def set_record_logits(self, on: bool):
        """Debug: keep each decoded sequence's logits of its final step (clears the store)."""
        lib().qwen_asr_set_record_logits(self._h, int(on))

    def recorded_logits(self) -> np.ndarray:
        """The kept logits, one row of vocab_size per decoded sequence, in decode order."""
        n = lib().qwen_asr_recorded_logits(self._h, None, 0)
        out = np.zeros(max(n, 0), np.float32)
        if n > 0:
            lib().qwen_asr_recorded_logits(self._h, out.ctypes.data_as(C.POINTER(C.c_float)), n)
        return out

    def set_profile(self, on: bool):
        lib().qwen_asr_set_profile(self._h, int(on))

    def profile_report(self) -> dict:
        ms = (C.c_double * 6)()
        n = (C.c_int64 * 6)()
        lib().qwen_asr_profile_report(self._h, ms, n, 6)
        names = ["qkv", "attention", "o_proj", "gate_up", "down", "lm_head_argmax"]
        return {k: (ms[i], n[i]) for i, k in enumerate(names)}

    def transcribe_device(self, d_ptr: int, n: int) -> str | None:
        """Samples already in this engine's device memory (e.g. a torch CUDA tensor's data_ptr())."""
        return _take_string(lib().qwen_asr_transcribe_device(self._h, C.c_void_p(d_ptr), n))

    def cuda_stream(self) -> int:
        return lib().qwen_asr_cuda_stream(self._h) or 0

    def launch_count(self) -> int:
        return lib().qwen_asr_launch_count(self._h)

    def set_timeline(self, on: bool):
        lib().qwen_asr_set_timeline(self._h, int(on))

    def timeline(self) -> np.ndarray:
        """[n_kernels, 4] = kind, t_entry, t_after_wait, t_exit (ns) of the last decode."""
        n = lib().qwen_asr_get_timeline(self._h, None, 0)
        buf = np.zeros(max(n, 4), dtype=np.uint64)
        lib().qwen_asr_get_timeline(self._h, buf.ctypes.data_as(C.POINTER(C.c_uint64)), n)
        return buf[:n].reshape(-1, 4)

    def last_tokens(self):
        L = lib()
        out = []
        for s in range(L.qwen_asr_last_segments(self._h)):
            n = L.qwen_asr_last_tokens(self._h, s, None, 0)
            buf = (C.c_int32 * max(n, 1))()
            L.qwen_asr_last_tokens(self._h, s, buf, n)
            out.append(list(buf[:n]))
        return out

    def perf(self) -> dict:
        v = (C.c_double * 16)()
        n = lib().qwen_asr_get_perf(self._h, v, 16)
        keys = ["total_ms", "audio_ms", "encode_ms", "decode_ms", "text_tokens", "gpu_mel_ms", "gpu_enc_ms",
                "gpu_prefill_ms", "gpu_decode_ms", "decode_steps"]
        return {k: v[i] for i, k in enumerate(keys[:n])}

    def model_info(self) -> dict:
        v = (C.c_int32 * 16)()
        n = lib().qwen_asr_model_info(self._h, v, 16)
        keys = ["enc_d_model", "enc_layers", "enc_heads", "enc_ffn_dim", "dec_hidden", "dec_layers", "dec_heads",
                "dec_kv_heads", "dec_intermediate", "vocab_size", "device"]
        return {k: v[i] for i, k in enumerate(keys[:n])}

    # --- parity hooks ---
    def debug_mel(self, samples) -> np.ndarray:
        a, p = _f32(samples)
        F = lib().qwen_asr_debug_mel(self._h, p, len(a), None, 0)
        if F <= 0:
            raise RuntimeError(last_error())
        out = np.empty((F, 128), dtype=np.float32)
        lib().qwen_asr_debug_mel(self._h, p, len(a), out.ctypes.data_as(_F32P), out.size)
        return out

    def debug_encode(self, mel_fm: np.ndarray) -> np.ndarray:
        m, p = _f32(mel_fm)
        hid = self.model_info()["dec_hidden"]
        F = m.shape[0]
        cap = (F // 8 + 16) * hid
        out = np.empty(cap, dtype=np.float32)
        T = lib().qwen_asr_debug_encode(self._h, p, F, out.ctypes.data_as(_F32P), cap)
        if T <= 0:
            raise RuntimeError(last_error())
        return out[:T * hid].reshape(T, hid).copy()

    def debug_resample(self, samples, from_rate: int) -> np.ndarray:
        """GPU resampling to 16 kHz (the transcribe_file path for non-16 kHz WAV files)."""
        x, p = _f32(samples)
        n = lib().qwen_asr_debug_resample(self._h, p, len(x), from_rate, None, 0)
        if n < 0:
            raise RuntimeError(last_error())
        out = np.zeros(n, dtype=np.float32)
        if lib().qwen_asr_debug_resample(self._h, p, len(x), from_rate, out.ctypes.data_as(_F32P), n) != n:
            raise RuntimeError(last_error())
        return out

    def debug_compact_silence(self, samples) -> np.ndarray:
        """GPU silence compaction (the skip_silence path); at most len(samples) samples."""
        x, p = _f32(samples)
        out = np.zeros(max(len(x), 1), dtype=np.float32)
        n = lib().qwen_asr_debug_compact_silence_gpu(self._h, p, len(x), out.ctypes.data_as(_F32P), len(x))
        if n < 0:
            raise RuntimeError(last_error())
        return out[:n]

    def debug_kv(self, layer: int, n_pos: int, slot: int = 0):
        """(k, v) f32 [kv_heads][n_pos][128] of one layer of a KV slot."""
        kvh = self.model_info()["dec_kv_heads"]
        k = np.zeros((kvh, n_pos, 128), dtype=np.float32)
        v = np.zeros_like(k)
        if lib().qwen_asr_debug_kv(self._h, slot, layer, n_pos, k.ctypes.data_as(_F32P), v.ctypes.data_as(_F32P)) != 0:
            raise RuntimeError(last_error())
        return k, v

    def kv_capacity(self) -> int:
        return lib().qwen_asr_debug_kv_capacity(self._h)

    def grow_kv(self, needed: int) -> int:
        n = lib().qwen_asr_debug_grow_kv(self._h, needed)
        if n < 0:
            raise RuntimeError(last_error())
        return n

    def debug_quant(self, layer: int, which: int):
        """Device int8 rows and f32 scales of a decoder matrix (0 qkv, 1 o, 2 gate/up, 3 down, 4 lm_head)."""
        n = lib().qwen_asr_debug_quant(self._h, layer, which, C.cast(None, C.POINTER(C.c_int8)),
                                       C.cast(None, _F32P), 0)
        if n < 0:
            raise RuntimeError(last_error())
        info = self.model_info()
        h, inter, qd = info["dec_hidden"], info["dec_intermediate"], info["dec_heads"] * 128
        cols = {0: h, 1: qd, 2: h, 3: inter, 4: h}[which]
        q = np.zeros((n, cols), dtype=np.int8)
        s = np.zeros(n, dtype=np.float32)
        if lib().qwen_asr_debug_quant(self._h, layer, which, q.ctypes.data_as(C.POINTER(C.c_int8)),
                                      s.ctypes.data_as(_F32P), n) != n:
            raise RuntimeError(last_error())
        return q, s

    def debug_decode(self, rows: np.ndarray, n_steps: int, forced=None, want_logits=False, want_hidden=False):
        r, p = _f32(rows)
        info = self.model_info()
        ids = np.zeros(max(n_steps, 1), dtype=np.int32)
        fz = None
        if forced is not None:
            fz = np.ascontiguousarray(forced, dtype=np.int32)
        lg = np.zeros((n_steps, info["vocab_size"]), dtype=np.float32) if want_logits else None
        hd = np.zeros((r.shape[0], info["dec_hidden"]), dtype=np.float32) if want_hidden else None
        n = lib().qwen_asr_debug_decode(
            self._h, p, r.shape[0], fz.ctypes.data_as(_I32P) if fz is not None else None, n_steps,
            ids.ctypes.data_as(_I32P), lg.ctypes.data_as(_F32P) if lg is not None else None,
            hd.ctypes.data_as(_F32P) if hd is not None else None)
        if n < 0:
            raise RuntimeError(last_error())
        return ids[:n_steps], lg, hd


class Pool:
    """One engine per GPU behind the C ABI (qwen_asr_pool_*): segmented transcription and
    concurrent streams sharded over the GPUs by the library's own worker threads."""

    def __init__(self, model_dir: str, devices=(), verbosity: int = 0):
        d = np.ascontiguousarray(list(devices), dtype=np.int32)
        self._h = lib().qwen_asr_pool_new(model_dir.encode(), d.ctypes.data_as(_I32P) if len(d) else None, len(d),
                                          verbosity)
        if not self._h:
            raise RuntimeError(f"pool load failed: {last_error()}")

    def close(self):
        if getattr(self, "_h", None):
            lib().qwen_asr_pool_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def size(self) -> int:
        return lib().qwen_asr_pool_size(self._h)

    def set_segment_sec(self, sec: float):
        lib().qwen_asr_pool_set_segment_sec(self._h, sec)

    def set_language(self, lang: str) -> int:
        return lib().qwen_asr_pool_set_language(self._h, lang.encode())

    def set_decode_mode(self, mode: str):
        lib().qwen_asr_pool_set_decode_mode(self._h, 1 if mode == "bf16" else 0)

    def set_force_n_tokens(self, n: int):
        lib().qwen_asr_pool_set_force_n_tokens(self._h, n)

    def stream_set_max_new_tokens(self, n: int):
        lib().qwen_asr_pool_stream_set_max_new_tokens(self._h, n)

    def transcribe_pcm(self, samples) -> str | None:
        x, p = _f32(samples)
        return _take_string(lib().qwen_asr_pool_transcribe_pcm(self._h, p, len(x)))

    def stream_push_many(self, streams, chunks, finalize: bool = False) -> list:
        n = len(streams)
        arrs = [np.ascontiguousarray(c, dtype=np.float32) for c in chunks]
        st = (C.c_void_p * n)(*[s._h for s in streams])
        ptrs = (_F32P * n)(*[a.ctypes.data_as(_F32P) for a in arrs])
        lens = np.array([len(a) for a in arrs], dtype=np.int32)
        out = (C.c_void_p * n)()
        if lib().qwen_asr_pool_stream_push_many(self._h, st, ptrs, lens.ctypes.data_as(_I32P), n, int(finalize),
                                                out) != 0:
            raise RuntimeError(last_error())
        return [_take_string(out[i]) for i in range(n)]


def assign_longest_first(lengths, workers: int) -> list[int]:
    """The pool's segment-to-GPU assignment (host only)."""
    l = np.ascontiguousarray(lengths, dtype=np.int64)
    out = np.zeros(len(l), dtype=np.int32)
    if lib().qwen_asr_debug_assign_longest_first(l.ctypes.data_as(_I64P), len(l), workers,
                                                 out.ctypes.data_as(_I32P)) != 0:
        raise RuntimeError("assign failed")
    return out.tolist()


def gemm_fallbacks() -> int:
    """Bf16-weight GEMMs that could not run on the tensor cores in this process."""
    return int(lib().qwen_asr_gemm_fallbacks())


def stream_push_many(engine, streams, chunks, finalize: bool = False) -> list:
    """Pushes chunks[i] to streams[i] for every i in one call (batched decode across the
    streams); returns the deltas (None when empty)."""
    k = len(streams)
    arrs = [np.ascontiguousarray(c, dtype=np.float32) for c in chunks]
    st = (C.c_void_p * max(k, 1))(*[s._h for s in streams])
    sp = (C.c_void_p * max(k, 1))(*[a.ctypes.data for a in arrs])
    ns = (C.c_int32 * max(k, 1))(*[len(a) for a in arrs])
    out = (C.c_void_p * max(k, 1))()
    if lib().qwen_asr_stream_push_many(engine._h, st, sp, ns, k, int(finalize), out) != 0:
        raise RuntimeError(last_error())
    return [_take_string(out[i]) for i in range(k)]


class Stream:
    """Incremental streaming state (transcribe.rs:801-893 via c_api.rs:179-265)."""

    def __init__(self):
        self._h = lib().qwen_asr_stream_new()

    def push(self, engine: Engine, samples, finalize: bool = False) -> str | None:
        a, p = _f32(samples)
        return _take_string(lib().qwen_asr_stream_push(engine._h, self._h, p, len(a), int(finalize)))

    def result(self) -> str | None:
        return _take_string(lib().qwen_asr_stream_get_result(self._h))

    def reset(self):
        lib().qwen_asr_stream_reset(self._h)

    def close(self):
        if getattr(self, "_h", None):
            lib().qwen_asr_stream_free(self._h)
            self._h = None

    def __del__(self):
        self.close()


def debug_align_words(text: str, language: str) -> list | None:
    """The forced aligner's units of `text` (align.rs:44-61)."""
    buf = C.create_string_buffer(4 * len(text.encode()) + 16)
    n = lib().qwen_asr_debug_align_words(text.encode(), language.encode(), buf, len(buf))
    if n < 0:
        return None
    return buf.value.decode().split("\n") if n > 0 else []


def debug_fix_timestamps(ts) -> np.ndarray:
    """The forced aligner's timestamp repair (align.rs:140-189)."""
    a = np.ascontiguousarray(ts, dtype=np.float32).copy()
    lib().qwen_asr_debug_fix_timestamps(a.ctypes.data_as(C.POINTER(C.c_float)), len(a))
    return a
