"""Forced-aligner host steps (align.rs) without a GPU: the C++ word split and timestamp
repair against the oracle's restatement, bit for bit, plus the oracle's own invariants and
an end-to-end oracle alignment on the tiny aligner checkpoint."""
import numpy as np
import pytest

from oracle import qwen_oracle as O

WORD_CASES = [
    ("Hello world", "English"),
    ("  leading and   trailing  ", "English"),
    ("tabs\tand\nnewlines\r\nmixed", "German"),
    ("ideographic　space em", "English"),
    ("no\x1cbreak\x1fhere", "English"),  # U+001C..U+001F are not Rust white space
    ("nbsp splits", "French"),
    ("", "English"),
    ("   ", "English"),
    ("你好 世界", "Chinese"),
    ("こんにちは　世界", "Japanese"),
    ("안녕 하세요", "Korean"),
    ("mixed 中文 text", "Cantonese"),
    ("Grüße, café! ☕", "English"),
]


@pytest.mark.parametrize("text,lang", WORD_CASES)
def test_split_words_matches_oracle(text, lang):
    import qwen_asr_b200 as Q
    assert Q.debug_align_words(text, lang) == O.align_split_words(text, lang)


def _fix_cases():
    rng = np.random.default_rng(11)
    cases = [[], [5.0], [0, 80, 160], [160, 80, 0], [0, 80, 40, 160, 240, 100, 320, 400, 80, 480],
             [400, 0, 0, 0, 80], [0, 0, 0, 0], [80, 40, 30, 20, 10, 0, 500], [0, 960, 80, 160, 240, 320]]
    for n in (2, 3, 7, 16, 33, 64):
        for _ in range(6):
            base = np.sort(rng.integers(0, 300, n)) * 80.0
            noise = rng.random(n) < 0.3
            v = np.where(noise, rng.integers(0, 300, n) * 80.0, base)
            cases.append(v.tolist())
    return cases


@pytest.mark.parametrize("ts", _fix_cases())
def test_fix_timestamps_matches_oracle(ts):
    import qwen_asr_b200 as Q
    got = Q.debug_fix_timestamps(np.asarray(ts, np.float32))
    want = np.asarray(O.fix_timestamps(ts), np.float32)
    assert got.view(np.uint32).tolist() == want.view(np.uint32).tolist()
    if len(ts):
        assert np.all(np.diff(want) >= 0)  # the repair leaves a non-decreasing sequence


def test_lis_is_longest_and_non_decreasing():
    rng = np.random.default_rng(3)
    for n in range(1, 12):
        v = rng.integers(0, 5, n).astype(np.float32).tolist()
        idx = O.longest_increasing_subsequence(v)
        assert all(v[a] <= v[b] for a, b in zip(idx, idx[1:]))
        # brute force: no longer non-decreasing subsequence exists
        best = 0
        for mask in range(1, 1 << n):
            s = [v[i] for i in range(n) if mask >> i & 1]
            if all(a <= b for a, b in zip(s, s[1:])):
                best = max(best, len(s))
        assert len(idx) == best


def test_oracle_forced_align_tiny():
    from conftest import model_dir
    from qwen_asr_b200 import synth
    d = model_dir("tiny-aligner", 0)
    ctx = O.Ctx(d, decode_mode="bf16")
    assert ctx.model.cfg.classify_num == synth.ALIGNER_CLASSES["tiny-aligner"]
    x = synth.synth_audio(16000 * 3, seed=21)
    words = "hello there general kenobi"
    out, cls = O.forced_align(ctx, x, words, "English")
    assert [w for w, _, _ in out] == words.split()
    assert len(cls) == 2 * len(out)
    flat = [t for _, s, e in out for t in (s, e)]
    assert all(a <= b for a, b in zip(flat, flat[1:]))
