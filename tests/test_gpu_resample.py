"""GPU Kaiser-sinc resampler (audio.rs:133-196): the step qwen_asr_transcribe_file and
qwen_asr_transcribe_wav_buffer run on the GPU for files that are not 16 kHz. Every f64
operation matches the host restatement (which matches the oracle) except sin(), where the
device's and the host C library's results may differ in the last f64 bit; so the samples
must be bit-equal except for rare one-ulp f32 differences, and a transcription of a 44.1 kHz
WAV must equal the transcription of the host-resampled samples."""
import ctypes as C
import os

import numpy as np
import pytest

from qwen_asr_b200 import synth

pytestmark = pytest.mark.gpu
F32P = C.POINTER(C.c_float)


def host_resampled(Q, wav: bytes) -> np.ndarray:
    L = Q.lib()
    buf = (C.c_uint8 * len(wav)).from_buffer_copy(wav)
    n = L.qwen_asr_debug_parse_wav(buf, len(wav), None, 0)
    out = np.empty(n, dtype=np.float32)
    L.qwen_asr_debug_parse_wav(buf, len(wav), out.ctypes.data_as(F32P), n)
    return out


def wav_bytes(x, sr, path):
    synth.write_wav(path, x, sr)
    with open(path, "rb") as f:
        return f.read()


@pytest.mark.parametrize("sr", [44100, 48000, 22050, 8000, 11025])
def test_gpu_resample_equals_host(tiny_dir, tmp_path, sr):
    import qwen_asr_b200 as Q
    eng = Q.Engine(tiny_dir)
    x = synth.synth_audio(int(sr * 3.3) + 17, seed=sr)
    wav = wav_bytes(x, sr, str(tmp_path / "a.wav"))
    ref = host_resampled(Q, wav)
    s16 = np.frombuffer(wav[44:], dtype="<i2").astype(np.float32) / 32768.0
    got = eng.debug_resample(s16, sr)
    assert got.shape == ref.shape
    ulps = np.abs(got.view(np.int32).astype(np.int64) - ref.view(np.int32).astype(np.int64))
    diff = ulps[got != ref]
    assert diff.size == 0 or int(diff.max()) <= 1, int(diff.max())
    assert float(np.mean(got == ref)) >= 0.999, float(np.mean(got == ref))


def test_transcribe_44k_file_equals_host_resampled(tiny_dir, tmp_path):
    import qwen_asr_b200 as Q
    eng = Q.Engine(tiny_dir)
    eng.set_language("English")
    eng.set_force_n_tokens(10)
    x = synth.synth_audio(44100 * 5, seed=5)
    path = str(tmp_path / "c.wav")
    wav = wav_bytes(x, 44100, path)
    ref_text = eng.transcribe_pcm(host_resampled(Q, wav))
    ref_ids = eng.last_tokens()
    assert eng.transcribe_file(path) == ref_text
    assert eng.last_tokens() == ref_ids
    assert eng.transcribe_wav_buffer(wav) == ref_text
    # segmented: the resampled samples come back to the host for the split search
    eng.set_segment_sec(2.0)
    a = eng.transcribe_pcm(host_resampled(Q, wav))
    assert eng.transcribe_file(path) == a
