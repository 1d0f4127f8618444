"""GPU parity: the CUDA engine (through its C ABI) against the CPU oracle on the same
seeded weights and audio. Tolerances are stated per test."""
import numpy as np
import pytest

from qwen_asr_b200 import synth

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def Q():
    import qwen_asr_b200 as Q
    return Q


@pytest.fixture(scope="module")
def O():
    from oracle import qwen_oracle as O
    return O


@pytest.fixture(scope="module")
def tiny(Q, tiny_dir):
    return Q.Engine(tiny_dir)


@pytest.fixture(scope="module")
def tiny_oracle(O, tiny_dir):
    return O.Model(tiny_dir)


@pytest.fixture(scope="module")
def m06(Q, m06_dir):
    return Q.Engine(m06_dir)


@pytest.fixture(scope="module")
def m06_oracle(O, m06_dir):
    return O.Model(m06_dir)


def c_abi_text(text):
    """What c_api.rs returns for a transcript: NULL when CString::new fails on an
    interior NUL (c_api.rs:85-90)."""
    return None if text is None or "\x00" in text else text


def rel_err(a, b):
    return float(np.max(np.abs(a - b)) / max(1e-12, float(np.max(np.abs(b)))))


# --------------------------------------------------------------------------- mel
@pytest.mark.parametrize("n", [161, 401, 8000, 16000 * 3 + 77, 451200])
def test_mel_matches_oracle(tiny, O, n):
    x = synth.synth_audio(n, seed=n)
    ref = O.mel_spectrogram(x)  # [128, F]
    got = tiny.debug_mel(x)     # [F, 128]
    assert got.shape == (ref.shape[1], 128)
    # f32 math in both; summation order differs -> absolute tolerance on values in [-1, 2]
    assert np.max(np.abs(got.T - ref)) < 2e-4


def test_mel_too_short(tiny):
    with pytest.raises(RuntimeError):
        tiny.debug_mel(np.zeros(100, dtype=np.float32))  # < one hop: reference returns None


# --------------------------------------------------------------------------- encoder
@pytest.mark.parametrize("seconds", [0.5, 3.0, 9.3])
def test_encoder_tiny_matches_oracle(tiny, tiny_oracle, O, seconds):
    x = synth.synth_audio(int(16000 * seconds), seed=7)
    mel = O.mel_spectrogram(x)
    ref = tiny_oracle.encode(mel)
    got = tiny.debug_encode(np.ascontiguousarray(mel.T))
    assert got.shape == ref.shape
    assert rel_err(got, ref) < 1e-3


@pytest.mark.parametrize("seconds", [1.3, 8.7])
def test_encoder_06b_matches_oracle(m06, m06_oracle, O, seconds):
    x = synth.synth_audio(int(16000 * seconds), seed=11)
    mel = O.mel_spectrogram(x)
    ref = m06_oracle.encode(mel)
    got = m06.debug_encode(np.ascontiguousarray(mel.T))
    assert got.shape == ref.shape
    assert rel_err(got, ref) < 2e-3


# --------------------------------------------------------------------------- decoder
def _rows_for(model, O, seconds, seed):
    x = synth.synth_audio(int(16000 * seconds), seed=seed)
    enc = model.encode(O.mel_spectrogram(x))
    ctx_like = O.Ctx.__new__(O.Ctx)
    ctx_like.model = model
    ctx_like.tok = None
    ctx_like.prompt = None
    ctx_like.force_language = None
    return O.prompt_rows(ctx_like, enc)


def _teacher_forced_case(eng, model, O, seconds, n_steps, mode, seed):
    """GPU and oracle teacher-forced decodes of one prompt, plus (int8) the oracle re-run with
    f64-accumulated RMSNorm and prefill products: an equally valid f32 ordering whose
    deviation from the default oracle is the noise floor int8 parity is judged against."""
    eng.set_decode_mode(mode)
    rows = _rows_for(model, O, seconds, seed)
    rng = np.random.default_rng(seed)
    forced = rng.integers(0, 151643, n_steps).astype(np.int32)
    ref_ids, ref_lg = O.teacher_forced(model, rows, forced, n_steps)
    ids, lg, _ = eng.debug_decode(rows, n_steps, forced=forced, want_logits=True)
    alt = None
    if mode == "int8":
        O.RMS_SUM_F64 = True
        try:
            alt = O.teacher_forced(model, rows, forced, n_steps)
        finally:
            O.RMS_SUM_F64 = False
    return ids, lg, ref_ids, ref_lg, alt


def _check_agreement(ids, lg, ref_ids, ref_lg, mode, alt=None):
    """bf16: >= 99.5% of teacher-forced ids agree and logits within 2e-2 max-rel (spec).

    int8: the per-vector activation quantiser (kernels/mod.rs:1795-1802) turns any last-bit
    f32 difference into whole-LSB flips that compound over 28 layers. The oracle itself,
    re-run with f64-accumulated RMSNorm and prefill products (`alt`), moves its logits by the
    same ~2-5% of max|logit| as the GPU does and flips ids where the top-2 gap is below that.
    So int8 must meet 99.5% overall, or be no further from the oracle than the oracle is
    from itself (mismatches <= the reordered oracle's + 2); every mismatch must pick a token
    the oracle scores within the measured noise of its best; logits within 5e-2 max-rel or
    twice the reordered oracle's deviation."""
    errs = np.array([rel_err(lg[s], ref_lg[s]) for s in range(len(ids))])
    agree = float(np.mean(ids == ref_ids))
    if mode == "bf16":
        assert agree >= 0.995, (ids, ref_ids)
        assert errs.max() < 2e-2
        return agree
    alt_ids, alt_lg = alt
    # logits: within 5e-2 max-rel, or within twice the reordered oracle's own deviation (the
    # LSB-flip cascade grows with the width: 1.7B's hidden 2048 moves logits further)
    self_rel = np.array([rel_err(alt_lg[s], ref_lg[s]) for s in range(len(ids))])
    assert errs.max() < max(5e-2, 2 * self_rel.max()), (errs.max(), self_rel.max())
    self_noise = np.max(np.abs(alt_lg - ref_lg), axis=1)  # per step, absolute
    gpu_noise = np.max(np.abs(lg - ref_lg), axis=1)
    bound = 2 * np.maximum(self_noise, gpu_noise)
    n_mis, n_self = int(np.sum(ids != ref_ids)), int(np.sum(alt_ids != ref_ids))
    assert agree >= 0.995 or n_mis <= n_self + 2, (n_mis, n_self, len(ids))
    for s in np.nonzero(ids != ref_ids)[0]:
        assert ref_lg[s, ref_ids[s]] - ref_lg[s, ids[s]] <= bound[s], s
    return agree


@pytest.mark.parametrize("mode", ["int8", "bf16"])
def test_decode_teacher_forced_tiny(tiny, O, tiny_dir, mode):
    model = O.Model(tiny_dir, decode_mode=mode)
    ids, lg, ref_ids, ref_lg, alt = _teacher_forced_case(tiny, model, O, 2.0, 64, mode, 5)
    _check_agreement(ids, lg, ref_ids, ref_lg, mode, alt)


@pytest.mark.parametrize("mode", ["int8", "bf16"])
def test_decode_teacher_forced_06b(m06, O, m06_dir, mode):
    model = O.Model(m06_dir, decode_mode=mode)
    ids, lg, ref_ids, ref_lg, alt = _teacher_forced_case(m06, model, O, 3.0, 96, mode, 9)
    _check_agreement(ids, lg, ref_ids, ref_lg, mode, alt)


@pytest.mark.parametrize("mode", ["int8", "bf16"])
def test_decode_teacher_forced_c2_clip(m06, O, m06_dir, mode):
    """The benchmarked C1/C2 shape: the 28.2 s clip (367 encoder rows, 381 prefill rows,
    positions up to 445)."""
    model = O.Model(m06_dir, decode_mode=mode)
    ids, lg, ref_ids, ref_lg, alt = _teacher_forced_case(m06, model, O, 28.2, 64, mode, 1)
    _check_agreement(ids, lg, ref_ids, ref_lg, mode, alt)


# --------------------------------------------------------------------------- end to end
def test_transcribe_offline_tiny(Q, O, tiny_dir):
    eng = Q.Engine(tiny_dir)
    ctx = O.Ctx(tiny_dir)
    x = synth.synth_audio(16000 * 4, seed=21)
    for e in (eng,):
        assert e.set_language("english") == 0
    ctx.set_force_language("english")
    eng.set_force_n_tokens(20)
    ctx.force_n_tokens = 20
    text = eng.transcribe_pcm(x)
    ref = c_abi_text(ctx.transcribe_audio(x))
    got_tokens = eng.last_tokens()[0]
    assert got_tokens[:20] == ctx.last_tokens[:20]
    assert text == ref


def test_transcribe_segmented_tiny(Q, O, tiny_dir):
    eng = Q.Engine(tiny_dir)
    ctx = O.Ctx(tiny_dir)
    x = synth.synth_audio(16000 * 70, seed=33)
    eng.set_segment_sec(30.0)
    ctx.segment_sec = 30.0
    eng.set_language("English")
    ctx.set_force_language("English")
    eng.set_force_n_tokens(8)
    ctx.force_n_tokens = 8
    text = eng.transcribe_pcm(x)
    ref = c_abi_text(ctx.transcribe_audio(x))
    segs = eng.last_tokens()
    assert len(segs) == len(ctx.segments_tokens) == len(O.split_points(x, 30.0, 3.0))
    for a, b in zip(segs, ctx.segments_tokens):
        assert a[:8] == b[:8]
    assert text == ref


def test_transcribe_without_language_is_empty_text(Q, tiny_dir):
    # random weights never emit <asr_text>, so nothing is text (transcribe.rs:196-219)
    eng = Q.Engine(tiny_dir)
    eng.set_force_n_tokens(6)
    assert eng.transcribe_pcm(synth.synth_audio(16000, seed=3)) == ""


def test_graph_and_direct_decode_agree(Q, tiny_dir):
    eng = Q.Engine(tiny_dir)
    eng.set_language("English")
    eng.set_force_n_tokens(40)
    x = synth.synth_audio(16000 * 2, seed=44)
    eng.set_use_graph(True)
    a = eng.transcribe_pcm(x)
    ta = eng.last_tokens()
    eng.set_use_graph(False)
    b = eng.transcribe_pcm(x)
    tb = eng.last_tokens()
    assert a == b and ta == tb


def test_prefill_attention_key_split_matches_oracle(m06_dir):
    """The prefill attention's optional key split (QASR_ATTN_KEY_CHUNK, 64-key chunks here:
    every query tile of the 28.2 s clip splits, partials merged in split order) keeps the
    bf16 teacher-forced tolerances. Runs in a child process (the setting is read once)."""
    import os
    import subprocess
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    code = (
        "import sys; sys.path.insert(0, %r); sys.path.insert(0, %r)\n"
        "import qwen_asr_b200 as Q\n"
        "from oracle import qwen_oracle as O\n"
        "from test_gpu_parity import _teacher_forced_case, _check_agreement\n"
        "eng = Q.Engine(%r)\n"
        "model = O.Model(%r, decode_mode='bf16')\n"
        "r = _teacher_forced_case(eng, model, O, 28.2, 16, 'bf16', 1)\n"
        "print('agree', _check_agreement(*r[:4], 'bf16'))\n" % (root, os.path.join(root, "tests"), m06_dir, m06_dir))
    env = dict(os.environ, QASR_ATTN_KEY_CHUNK="64")
    p = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True, cwd=root)
    assert p.returncode == 0 and "agree" in p.stdout, p.stdout + p.stderr
