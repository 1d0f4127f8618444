"""GPU parity of incremental streaming (qwen_asr_stream_push, c_api.rs:212-245 ->
stream_push_audio, transcribe.rs:902-1304) against the oracle's restatement: the text
deltas of every push, the final result, and the generated ids of every chunk.

Decode runs with bf16 weights here: its logits match the oracle to ~3e-5, so greedy ids
are stable across implementations; the int8 path's quantisation noise would make long
free-running token sequences diverge at near-ties (see test_gpu_parity)."""
import numpy as np
import pytest

from qwen_asr_b200 import synth

pytestmark = pytest.mark.gpu


def _run(tiny_dir, past_text, push_sec, total_sec, seed, chunk_sec=2.0, max_new=12):
    import qwen_asr_b200 as Q
    from oracle import qwen_oracle as O
    eng = Q.Engine(tiny_dir)
    eng.set_decode_mode("bf16")
    eng.set_language("English")
    eng.set_past_text(past_text)
    eng.stream_set_chunk_sec(chunk_sec)
    eng.stream_set_max_new_tokens(max_new)
    ctx = O.Ctx(tiny_dir, decode_mode="bf16")
    ctx.set_force_language("English")
    ctx.past_text_conditioning = past_text
    ctx.stream_chunk_sec = chunk_sec
    ctx.stream_max_new_tokens = max_new
    x = synth.synth_audio(int(16000 * total_sec), seed=seed)
    s = Q.Stream()
    st = O.StreamState()
    step = int(16000 * push_sec)
    got, want = [], []
    for i in range(0, len(x), step):
        fin = i + step >= len(x)
        got.append(s.push(eng, x[i:i + step], finalize=fin))
        d = O.stream_push_audio(ctx, x[:i + step], st, fin)
        want.append(O.lossy(d) or None)
    return got, want, s.result(), (O.lossy(st.result_bytes) or None)


def _c(t):
    return None if t is None or "\x00" in t else t


@pytest.mark.parametrize("past_text", [False, True])
def test_stream_matches_oracle(tiny_dir, past_text):
    got, want, res, ref = _run(tiny_dir, past_text, push_sec=0.7, total_sec=19.0, seed=61)
    assert [_c(w) for w in want] == got
    assert _c(ref) == res


def test_stream_interleaved_streams_stay_independent(tiny_dir):
    """Two streams pushed alternately on one engine give the same text as each alone."""
    import qwen_asr_b200 as Q
    eng = Q.Engine(tiny_dir)
    eng.set_decode_mode("bf16")
    eng.set_language("English")
    eng.set_past_text(True)
    eng.stream_set_max_new_tokens(8)
    xa = synth.synth_audio(16000 * 9, seed=71)
    xb = synth.synth_audio(16000 * 9, seed=72)

    def alone(x):
        s = Q.Stream()
        for i in range(0, len(x), 16000):
            s.push(eng, x[i:i + 16000], finalize=i + 16000 >= len(x))
        return s.result()

    ra, rb = alone(xa), alone(xb)
    sa, sb = Q.Stream(), Q.Stream()
    for i in range(0, len(xa), 16000):
        fin = i + 16000 >= len(xa)
        sa.push(eng, xa[i:i + 16000], finalize=fin)
        sb.push(eng, xb[i:i + 16000], finalize=fin)
    assert sa.result() == ra and sb.result() == rb


def test_stream_reset_and_empty(tiny_dir):
    import qwen_asr_b200 as Q
    eng = Q.Engine(tiny_dir)
    s = Q.Stream()
    assert s.push(eng, np.zeros(100, np.float32)) is None  # less than a chunk: nothing yet
    assert s.result() is None
    s.reset()
    assert s.push(eng, np.zeros(0, np.float32), finalize=True) is None


@pytest.mark.parametrize("mode", ["int8", "bf16"])
def test_stream_push_many_matches_single_streams(tiny_dir, mode):
    """Streams advanced together (one prefill pass and a batched decode across their KV
    slots) produce exactly the deltas, ids and final-step logits (bit for bit) that each
    produces when pushed alone."""
    import qwen_asr_b200 as Q
    n_streams, n_chunks, chunk = 3, 4, 32000
    audio = [synth.synth_audio(chunk * n_chunks, seed=300 + i) for i in range(n_streams)]

    def make():
        eng = Q.Engine(tiny_dir)
        eng.set_decode_mode(mode)
        eng.set_language("English")
        eng.set_record_logits(True)
        return eng

    eng_a = make()
    many = [Q.Stream() for _ in range(n_streams)]
    got = []
    for c in range(n_chunks):
        fin = c == n_chunks - 1
        got.append(Q.stream_push_many(eng_a, many, [a[c * chunk:(c + 1) * chunk] for a in audio], finalize=fin))
    eng_b = make()
    want = []
    singles = [Q.Stream() for _ in range(n_streams)]
    for c in range(n_chunks):
        fin = c == n_chunks - 1
        want.append([s.push(eng_b, a[c * chunk:(c + 1) * chunk], finalize=fin) for s, a in zip(singles, audio)])
    assert got == want
    assert [s.result() for s in many] == [s.result() for s in singles]
    # generated ids of every chunk of every stream, accumulated round by round in both engines
    ids_a, ids_b = eng_a.last_tokens(), eng_b.last_tokens()
    assert ids_a == ids_b and len(ids_a) == n_chunks * n_streams and sum(len(g) for g in ids_a) > 0
    la, lb = eng_a.recorded_logits(), eng_b.recorded_logits()
    assert la.size > 0 and la.shape == lb.shape
    assert np.array_equal(la.view(np.uint32), lb.view(np.uint32))
