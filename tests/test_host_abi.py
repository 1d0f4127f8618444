"""CPU tests of libqwen_asr's host side through its C ABI (no GPU needed): every symbol
declared in include/*.h is exported, and the host logic (tokenizer, WAV parsing +
resampling, segmentation, silence compaction, text handling, config/lang) matches the
oracle restatement of the reference bit for bit."""
import ctypes as C
import os
import re
import struct

import numpy as np
import pytest

import qwen_asr_b200 as Q
from oracle import qwen_oracle as O
from qwen_asr_b200 import synth

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
F32P = C.POINTER(C.c_float)


def declared_symbols():
    names = set()
    for h in ("qwen_asr.h", "qwen_asr_ext.h"):
        src = open(os.path.join(ROOT, "include", h)).read()
        src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
        names |= set(re.findall(r"\b(qwen_asr_[a-z0-9_]+)\s*\(", src))
    return names


def test_library_exports_every_declared_symbol():
    L = Q.lib()
    names = declared_symbols()
    assert len(names) >= 17 + 20
    for n in sorted(names):
        assert hasattr(L, n), n
        assert n in Q.SIGNATURES, n


def test_reference_c_ffi_surface_is_complete():
    # the 17 exports of crates/qwen-asr/src/c_api.rs
    ref = {"qwen_asr_load_model", "qwen_asr_transcribe_file", "qwen_asr_transcribe_pcm",
           "qwen_asr_transcribe_wav_buffer", "qwen_asr_set_segment_sec", "qwen_asr_set_language",
           "qwen_asr_free_string", "qwen_asr_free", "qwen_asr_stream_new", "qwen_asr_stream_free",
           "qwen_asr_stream_reset", "qwen_asr_stream_push", "qwen_asr_stream_get_result",
           "qwen_asr_stream_set_chunk_sec", "qwen_asr_stream_set_rollback",
           "qwen_asr_stream_set_unfixed_chunks", "qwen_asr_stream_set_max_new_tokens"}
    assert ref <= declared_symbols()


def test_null_arguments_return_null_or_minus_one():
    L = Q.lib()
    assert not L.qwen_asr_load_model(None, 0, 0)
    assert not L.qwen_asr_transcribe_pcm(None, None, 0)
    assert not L.qwen_asr_transcribe_file(None, b"x.wav")
    assert L.qwen_asr_set_language(None, b"English") == -1
    assert not L.qwen_asr_stream_push(None, None, None, 0, 1)
    assert not L.qwen_asr_stream_get_result(None)
    L.qwen_asr_free(None)
    L.qwen_asr_free_string(None)
    L.qwen_asr_set_segment_sec(None, 1.0)
    s = L.qwen_asr_stream_new()
    assert s
    assert not L.qwen_asr_stream_get_result(s)  # empty -> NULL (c_api.rs:250-265)
    L.qwen_asr_stream_reset(s)
    L.qwen_asr_stream_free(s)


def test_non_utf8_arguments_are_rejected(tmp_path):
    """c_api.rs:28-31, 59-62, 141-144: CStr::to_str failures give NULL / -1."""
    L = Q.lib()
    assert not L.qwen_asr_load_model(b"/tmp/\xff\xfe-model", 0, 0)
    assert "UTF-8" in Q.last_error()
    assert not L.qwen_asr_load_model(b"/tmp/\xed\xa0\x80", 0, 0)  # encoded surrogate
    assert "UTF-8" in Q.last_error()
    rng = np.random.default_rng(5)
    cases = [b"plain", "真棒🦀".encode(), b"\xc0\xaf", b"\xe0\x80\xaf", b"\xf4\x90\x80\x80", b"\xf0\x9f\xa6",
             b"\xc3", b"\x80", "\U0010ffff".encode(), b"\xef\xbf\xbf"]
    cases += [bytes(rng.integers(1, 256, int(rng.integers(1, 8))).astype(np.uint8)) for _ in range(2000)]
    for b in cases:
        try:
            b.decode("utf-8")
            want = 1
        except UnicodeDecodeError:
            want = 0
        assert L.qwen_asr_debug_valid_utf8(b) == want, b


def test_missing_and_corrupt_model_fail_cleanly(tmp_path):
    L = Q.lib()
    assert not L.qwen_asr_load_model(str(tmp_path).encode(), 0, 0)
    assert "safetensors" in Q.last_error()
    p = tmp_path / "model.safetensors"
    p.write_bytes(struct.pack("<Q", 1 << 40) + b"{}")  # header length beyond file size
    assert not L.qwen_asr_load_model(str(tmp_path).encode(), 0, 0)
    assert "header" in Q.last_error()
    p.write_bytes(struct.pack("<Q", 10) + b'{"a": 12}xx')  # malformed tensor entry
    assert not L.qwen_asr_load_model(str(tmp_path).encode(), 0, 0)
    assert "malformed" in Q.last_error()
    hdr = b'{"thinker.model.embed_tokens.weight":{"dtype":"BF16","shape":[2,2],"data_offsets":[0,8]}}'
    p.write_bytes(struct.pack("<Q", len(hdr)) + hdr + b"\0" * 8)  # parses, but core tensors missing
    assert not L.qwen_asr_load_model(str(tmp_path).encode(), 0, 0)
    assert "missing" in Q.last_error()


# ----------------------------------------------------------------- tokenizer
TEXTS = ["language English", "hello world", "Rust🦀真棒", "a", "  spaced  out ", "地址", "The quick brown fox",
         "language Chinese", "ünïcödé"]


def test_tokenizer_encode_matches_oracle(tiny_dir):
    L = Q.lib()
    tok = O.Tokenizer(tiny_dir)
    for t in TEXTS:
        buf = (C.c_int32 * 512)()
        n = L.qwen_asr_debug_tokenize(tiny_dir.encode(), t.encode(), buf, 512)
        ref = tok.encode(t)
        assert ref is not None
        assert list(buf[:n]) == ref, t


def test_tokenizer_decode_bytes_matches_oracle(tiny_dir):
    L = Q.lib()
    tok = O.Tokenizer(tiny_dir)
    rng = np.random.default_rng(0)
    ids = np.concatenate([rng.integers(0, 151936, 300), [151643, 151645, 151704, -1, 10 ** 7]]).astype(np.int32)
    out = C.create_string_buffer(8192)
    n = L.qwen_asr_debug_detokenize(tiny_dir.encode(), ids.ctypes.data_as(C.POINTER(C.c_int32)), len(ids), out, 8192)
    ref = b"".join(tok.decode_bytes(int(i)) for i in ids)
    assert out.raw[:n] == ref


def test_gpt2_byte_mapping_bijective_roundtrip(tiny_dir):
    # tokenizer.rs tests: every byte survives byte->unicode->byte; split UTF-8 sequences
    # decode only when their bytes are accumulated (tokenizer.rs:569-621)
    tok = O.Tokenizer(tiny_dir)
    b2u = synth.gpt2_byte_to_unicode()
    assert len(set(b2u)) == 256 and all(0 <= c < 512 for c in b2u)
    single = {bytes([b]): tok.vocab[chr(b2u[b])] for b in range(256)}
    for raw in ("地".encode(), "é".encode(), "🦀".encode(), "Rust🦀真棒".encode()):
        acc = b"".join(tok.decode_bytes(single[bytes([b])]) for b in raw)
        assert acc == raw
    parts = [b"\xE5\x9C", b"\xB0\xE5", b"\x9D\x80"]
    assert "�" in "".join(O.lossy(p) for p in parts)
    assert O.lossy(b"".join(parts)) == "地址"


# ----------------------------------------------------------------- audio / wav
def _wav_bytes(samples, sr, channels=1):
    x = np.asarray(samples, dtype=np.float32)
    s16 = np.clip(np.round(x * 32767), -32768, 32767).astype("<i2")
    if channels > 1:
        s16 = np.stack([s16] + [(s16 // (c + 1)).astype("<i2") for c in range(1, channels)], axis=1).reshape(-1)
    data = s16.tobytes()
    hdr = b"RIFF" + struct.pack("<I", 36 + len(data)) + b"WAVE"
    hdr += b"fmt " + struct.pack("<IHHIIHH", 16, 1, channels, sr, sr * channels * 2, channels * 2, 16)
    hdr += b"LIST" + struct.pack("<I", 3) + b"abc\0"  # odd-sized chunk before data (padding byte)
    return hdr + b"data" + struct.pack("<I", len(data)) + data


@pytest.mark.parametrize("sr,ch", [(16000, 1), (16000, 2), (44100, 1), (8000, 3)])
def test_parse_wav_matches_oracle(sr, ch):
    L = Q.lib()
    x = synth.synth_audio(sr // 2 + 37, seed=sr + ch)
    wav = _wav_bytes(x, sr, ch)
    buf = (C.c_uint8 * len(wav)).from_buffer_copy(wav)
    n = L.qwen_asr_debug_parse_wav(buf, len(wav), None, 0)
    out = np.empty(n, dtype=np.float32)
    L.qwen_asr_debug_parse_wav(buf, len(wav), out.ctypes.data_as(F32P), n)
    ref = O.parse_wav_buffer(wav)
    assert n == len(ref)
    # identical f64 algorithm; libm vs numpy transcendental ulps only
    assert np.max(np.abs(out - ref)) < 1e-6


def test_parse_wav_rejects_non_pcm16():
    L = Q.lib()
    wav = bytearray(_wav_bytes(np.zeros(100), 16000))
    wav[34] = 32  # bits per sample
    buf = (C.c_uint8 * len(wav)).from_buffer_copy(bytes(wav))
    assert L.qwen_asr_debug_parse_wav(buf, len(wav), None, 0) == -1
    assert L.qwen_asr_debug_parse_wav(buf, 20, None, 0) == -1  # truncated


@pytest.mark.parametrize("seconds,seg", [(95.0, 30.0), (61.0, 30.0), (33.0, 30.0), (200.0, 10.0), (20.0, 0.0),
                                         (45.3, 7.5), (1300.0, 30.0)])
def test_split_points_bit_exact(seconds, seg):
    L = Q.lib()
    x = synth.synth_audio(int(16000 * seconds), seed=int(seconds * 10))
    out = (C.c_int64 * 256)()
    n = L.qwen_asr_debug_split_points(x.ctypes.data_as(F32P), len(x), seg, 3.0, out, 256)
    assert list(out[:n]) == O.split_points(x, seg, 3.0)


def test_compact_silence_matches_oracle():
    # audio.rs tests: tone - 2 s silence - tone gets shorter but keeps the tones
    L = Q.lib()
    sr = 16000
    t = np.arange(sr // 2) / sr
    tone = (np.sin(2 * np.pi * 440 * t) * 0.3).astype(np.float32)
    x = np.concatenate([tone, np.zeros(2 * sr, np.float32), tone]).astype(np.float32)
    out = np.empty(len(x), dtype=np.float32)
    n = L.qwen_asr_debug_compact_silence(x.ctypes.data_as(F32P), len(x), out.ctypes.data_as(F32P), len(x))
    ref = O.compact_silence(x)
    assert n == len(ref) and np.array_equal(out[:n], ref)
    assert len(tone) < n < len(x)


@pytest.mark.parametrize("raw", [b"  hello  ", b"\xe5\x9c\xb0\xe5", b"\x00abc\x85", b"\xc2\xa0x\xe3\x80\x80",
                                 b"\xf0\x9f\xa6", b"\xed\xa0\x80z", b"\t\n", b"", b"\xff\xfe a"])
def test_lossy_trim_matches_oracle(raw):
    L = Q.lib()
    out = C.create_string_buffer(256)
    n = L.qwen_asr_debug_lossy_trim(raw, len(raw), out, 256)
    assert out.raw[:n].decode("utf-8") == O.rust_trim(O.lossy(raw))


@pytest.mark.parametrize("lang", ["english", " ENGLISH ", "Chinese", "klingon", "", "macedonian", "Ünglish"])
def test_normalize_language(lang):
    L = Q.lib()
    out = C.create_string_buffer(64)
    L.qwen_asr_debug_normalize_language(lang.encode(), out, 64)
    assert out.value.decode() == (O.normalize_language(lang) or "")


def test_boundary_space_rule():
    assert O.should_insert_boundary_space(ord("a"), ord("b"))
    assert not O.should_insert_boundary_space(ord("a"), ord(","))
    assert not O.should_insert_boundary_space(ord(" "), ord("b"))
    assert not O.should_insert_boundary_space(0xA0, ord("b"))


# ----------------------------------------------------------------- multi-GPU pool (host logic)
def test_pool_assignment_matches_shard_assign():
    """The C++ pool's longest-first assignment equals the Python sharding helper's, so the
    torch.distributed driver (qwen_asr_b200.shard) and the library pool split work alike."""
    from qwen_asr_b200 import shard
    rng = np.random.default_rng(3)
    for n, w in [(41, 8), (41, 1), (5, 8), (0, 3), (17, 4), (100, 7)]:
        lens = rng.integers(8000, 480000, n)
        lens[: n // 4] = 480000  # ties
        segs = []
        a = 0
        for L in lens:
            segs.append((a, a + int(L)))
            a += int(L)
        want = shard.assign(segs, w)
        got = Q.assign_longest_first(lens, w)
        assert [[i for i in range(n) if got[i] == r] for r in range(w)] == want


def test_pool_rejects_bad_arguments():
    L = Q.lib()
    assert not L.qwen_asr_pool_new(None, None, 0, 0)
    assert not L.qwen_asr_pool_new(b"/nonexistent", None, -1, 0)
    assert L.qwen_asr_pool_size(None) == 0
    assert not L.qwen_asr_pool_transcribe_pcm(None, None, 0)
    L.qwen_asr_pool_free(None)
