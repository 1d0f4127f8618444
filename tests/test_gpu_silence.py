"""GPU silence compaction (skip_silence; audio.rs:375-479 compact_silence): the window RMS,
smoothing, 25th-percentile threshold, run filter, widening and pause rule on the device give
the oracle's output sample for sample, on the reference's own test shape (tone, 2 s of
silence, tone), on speech-like audio with pauses, on edge lengths and all-silent input (the
first 0.5 s is kept), and on a 20-minute clip against the host restatement. A transcription
with skip_silence equals the transcription of the oracle-compacted samples."""
import ctypes as C

import numpy as np
import pytest

from qwen_asr_b200 import synth

pytestmark = pytest.mark.gpu
F32P = C.POINTER(C.c_float)
SR = 16000


@pytest.fixture(scope="module")
def eng(tiny_dir):
    import qwen_asr_b200 as Q
    return Q.Engine(tiny_dir)


def _with_pauses(seed, seconds=12.0):
    rng = np.random.default_rng(seed)
    x = synth.synth_audio(int(SR * seconds), seed=seed).copy()
    for _ in range(4):  # pauses of 0.3-2.5 s with a faint noise floor
        a = int(rng.integers(0, len(x) - SR))
        b = min(len(x), a + int(rng.uniform(0.3, 2.5) * SR))
        x[a:b] = (rng.standard_normal(b - a) * 1e-4).astype(np.float32)
    return x


def _cases():
    t = np.arange(SR // 2) / SR
    tone = (np.sin(2 * np.pi * 440 * t) * 0.3).astype(np.float32)
    rng = np.random.default_rng(3)
    return {
        "tone_gap_tone": np.concatenate([tone, np.zeros(2 * SR, np.float32), tone]),
        "pauses_a": _with_pauses(11),
        "pauses_b": _with_pauses(12, 31.7),
        "silent_long": np.zeros(3 * SR + 77, np.float32),      # nothing kept: first 0.5 s
        "silent_short": np.zeros(5000, np.float32),            # nothing kept, shorter than 0.5 s
        "one_window": (rng.standard_normal(100) * 0.1).astype(np.float32),
        "one_sample": np.array([0.25], np.float32),
        "ragged_tail": _with_pauses(13, 4.0)[:SR * 4 - 37],
    }


@pytest.mark.parametrize("name", list(_cases()))
def test_gpu_compact_silence_matches_oracle(eng, name):
    from oracle import qwen_oracle as O
    x = _cases()[name]
    got = eng.debug_compact_silence(x)
    ref = O.compact_silence(x)
    assert len(got) == len(ref), (name, len(got), len(ref))
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32)), name


def test_gpu_compact_silence_20_minutes_matches_host(eng):
    """C4's 20-minute clip with pauses cut in (120,000 windows: every CTA-chunk boundary of
    the scans is crossed) against the host restatement, bit for bit."""
    import qwen_asr_b200 as Q
    x = synth.synth_audio(SR * 1200, seed=3).copy()
    rng = np.random.default_rng(5)
    for _ in range(200):
        a = int(rng.integers(0, len(x) - 3 * SR))
        x[a:a + int(rng.uniform(0.2, 3.0) * SR)] = 0.0
    got = eng.debug_compact_silence(x)
    out = np.empty(len(x), dtype=np.float32)
    n = Q.lib().qwen_asr_debug_compact_silence(x.ctypes.data_as(F32P), len(x), out.ctypes.data_as(F32P), len(x))
    assert n == len(got) and np.array_equal(got.view(np.uint32), out[:n].view(np.uint32))
    assert len(got) < len(x)


def test_transcribe_skip_silence_uses_compacted_audio(tiny_dir):
    import qwen_asr_b200 as Q
    from oracle import qwen_oracle as O
    x = _with_pauses(21, 9.0)
    a = Q.Engine(tiny_dir)
    a.set_skip_silence(True)
    ta = a.transcribe_pcm(x)
    b = Q.Engine(tiny_dir)
    tb = b.transcribe_pcm(O.compact_silence(x))
    assert ta == tb and a.last_tokens() == b.last_tokens()
