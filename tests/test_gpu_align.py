"""Forced alignment through the C ABI (qwen_asr_forced_align) against the oracle's
restatement of align.rs on seeded aligner checkpoints: same words, per-word times equal
for the <timestamp> rows whose classify argmax agrees (random weights leave near-ties,
so a small share may pick a neighbouring class), and the non-decreasing property."""
import numpy as np
import pytest

from oracle import qwen_oracle as O
from qwen_asr_b200 import synth

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("preset,seconds,text,lang", [
    ("tiny-aligner", 4.0, "the quick brown fox jumps over the lazy dog", "English"),
    ("tiny-aligner", 3.0, "你好世界今天", "Chinese"),
    ("aligner", 8.0, "forced alignment gives every word a start and an end time in milliseconds", "English"),
])
def test_forced_align_matches_oracle(preset, seconds, text, lang):
    import qwen_asr_b200 as Q
    from conftest import model_dir
    d = model_dir(preset, 0)
    x = synth.synth_audio(int(16000 * seconds), seed=31)
    eng = Q.Engine(d)
    got = eng.forced_align(x, text, lang)
    assert got is not None, Q.last_error()
    ctx = O.Ctx(d, decode_mode="bf16")
    want, cls = O.forced_align(ctx, x, text, lang)
    assert [g["text"] for g in got] == [w for w, _, _ in want]
    flat = [t for g in got for t in (g["start_ms"], g["end_ms"])]
    assert all(a <= b for a, b in zip(flat, flat[1:]))
    same = np.mean([g["start_ms"] == s and g["end_ms"] == e for g, (_, s, e) in zip(got, want)])
    assert same >= 0.8, (got, want)


def test_forced_align_rejects_asr_model(tiny_dir):
    import qwen_asr_b200 as Q
    eng = Q.Engine(tiny_dir)
    assert eng.forced_align(synth.synth_audio(16000, seed=1), "hello", "English") is None
    assert "aligner" in Q.last_error()
