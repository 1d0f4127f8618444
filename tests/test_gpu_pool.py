"""GPU tests of the library's multi-GPU pool (qwen_asr_pool_*, pool.cpp) and of more
concurrent streams than KV slots. The pool runs two workers on GPU 0 here (a device may be
listed twice), which exercises the sharded path - split, assignment, per-worker batched
transcription, ordered join - on a one-GPU box."""
import numpy as np
import pytest

from qwen_asr_b200 import synth

pytestmark = pytest.mark.gpu


def test_pool_segmented_equals_single_engine(tiny_dir):
    import qwen_asr_b200 as Q
    x = synth.synth_audio(16000 * 95, seed=81)
    eng = Q.Engine(tiny_dir)
    pool = Q.Pool(tiny_dir, devices=[0, 0])
    assert pool.size() == 2
    for e in (eng, pool):
        e.set_segment_sec(30.0)
        assert e.set_language("English") == 0
        e.set_force_n_tokens(8)
    want = eng.transcribe_pcm(x)
    got = pool.transcribe_pcm(x)
    assert got == want and want
    # one segment: the first worker alone
    pool.set_segment_sec(0.0)
    eng.set_segment_sec(0.0)
    y = synth.synth_audio(16000 * 4, seed=82)
    assert pool.transcribe_pcm(y) == eng.transcribe_pcm(y)


def test_pool_streams_equal_single_engine(tiny_dir):
    import qwen_asr_b200 as Q
    eng = Q.Engine(tiny_dir)
    pool = Q.Pool(tiny_dir, devices=[0, 0])
    for e in (eng, pool):
        e.set_decode_mode("bf16")
        e.set_language("English")
        e.stream_set_max_new_tokens(6)
    xs = [synth.synth_audio(16000 * 6, seed=90 + i) for i in range(3)]
    solo = []
    for x in xs:
        s = Q.Stream()
        solo.append([s.push(eng, x[i:i + 16000], finalize=i + 16000 >= len(x)) for i in range(0, len(x), 16000)])
    ss = [Q.Stream() for _ in xs]
    got = [[] for _ in xs]
    for i in range(0, len(xs[0]), 16000):
        d = pool.stream_push_many(ss, [x[i:i + 16000] for x in xs], finalize=i + 16000 >= len(xs[0]))
        for k in range(len(xs)):
            got[k].append(d[k])
    assert got == solo


def test_more_streams_than_kv_slots(tiny_dir):
    """33 streams in one stream_push_many call (32 KV slots): the library pushes them in
    groups that never share a slot, so every stream's deltas equal that stream alone."""
    import qwen_asr_b200 as Q
    eng = Q.Engine(tiny_dir)
    eng.set_decode_mode("bf16")
    eng.set_language("English")
    eng.stream_set_max_new_tokens(4)
    n = 33
    xs = [synth.synth_audio(16000 * 3, seed=200 + i) for i in range(n)]
    ss = [Q.Stream() for _ in range(n)]
    got = [[] for _ in range(n)]
    for i in range(0, 16000 * 3, 16000):
        d = Q.stream_push_many(eng, ss, [x[i:i + 16000] for x in xs], finalize=i + 16000 >= 16000 * 3)
        for k in range(n):
            got[k].append(d[k])
    for k in (0, 1, 16, 31, 32):
        s = Q.Stream()
        alone = [s.push(eng, xs[k][i:i + 16000], finalize=i + 16000 >= 16000 * 3) for i in range(0, 16000 * 3, 16000)]
        assert got[k] == alone, k
