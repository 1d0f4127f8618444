"""GPU parity at the Qwen3-ASR-1.7B widths (config.rs:110-157: encoder d=1024, 24 layers,
16 heads, FFN 4096; decoder hidden 2048, SwiGLU 6144) that the C3 and C5 workloads run:
encoder rows, teacher-forced decode in both weight modes (bf16 takes the split q/k/v path by
default at this width), and a long incremental stream through the re-anchor at chunk 45
(transcribe.rs:689-737) on a 4-layer model of the same widths."""
import numpy as np
import pytest

from qwen_asr_b200 import synth
from test_gpu_parity import _check_agreement, _teacher_forced_case, rel_err

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def m17(m17_dir):
    import qwen_asr_b200 as Q
    return Q.Engine(m17_dir)


def test_17b_shapes(m17):
    info = m17.model_info()
    assert (info["enc_d_model"], info["enc_layers"], info["enc_ffn_dim"]) == (1024, 24, 4096)
    assert (info["dec_hidden"], info["dec_layers"], info["dec_intermediate"]) == (2048, 28, 6144)


def test_encoder_17b_matches_oracle(m17, m17_dir):
    from oracle import qwen_oracle as O
    model = O.Model(m17_dir, decode_mode="bf16")
    x = synth.synth_audio(int(16000 * 9.3), seed=13)
    mel = O.mel_spectrogram(x)
    ref = model.encode(mel)
    got = m17.debug_encode(np.ascontiguousarray(mel.T))
    assert got.shape == ref.shape
    assert rel_err(got, ref) < 2e-3


@pytest.mark.parametrize("mode", ["bf16", "int8"])
def test_decode_teacher_forced_17b(m17, m17_dir, mode):
    from oracle import qwen_oracle as O
    model = O.Model(m17_dir, decode_mode=mode)
    ids, lg, ref_ids, ref_lg, alt = _teacher_forced_case(m17, model, O, 4.0, 48, mode, 17)
    _check_agreement(ids, lg, ref_ids, ref_lg, mode, alt)


def test_stream_17b_widths_46_chunks(m17l4_dir):
    """92 s pushed in 2 s steps = 46 chunks, so the prefix re-anchor at chunk 45 runs; every
    delta and the final text equal the oracle's stream_push_audio (bf16 decode: free-running
    int8 ids diverge at near-ties, see test_gpu_parity)."""
    import qwen_asr_b200 as Q
    from oracle import qwen_oracle as O
    eng = Q.Engine(m17l4_dir)
    eng.set_decode_mode("bf16")
    eng.set_language("English")
    eng.stream_set_max_new_tokens(6)
    ctx = O.Ctx(m17l4_dir, decode_mode="bf16")
    ctx.set_force_language("English")
    ctx.stream_max_new_tokens = 6
    x = synth.synth_audio(16000 * 92, seed=1000)
    s, st = Q.Stream(), O.StreamState()
    step = 32000
    for i in range(0, len(x), step):
        fin = i + step >= len(x)
        got = s.push(eng, x[i:i + step], finalize=fin)
        want = O.lossy(O.stream_push_audio(ctx, x[:i + step], st, fin)) or None
        assert got == (None if want is None or "\x00" in want else want), i // step
    ref = O.lossy(st.result_bytes) or None
    assert s.result() == (None if ref is None or "\x00" in ref else ref)


def _child(env_extra, code, model_dir):
    import os
    import subprocess
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    prog = ("import sys, hashlib; sys.path.insert(0, %r)\n"
            "import numpy as np\n"
            "import qwen_asr_b200 as Q\n"
            "eng = Q.Engine(%r)\n"
            "h = eng.model_info()['dec_hidden']\n"
            "rows = (np.random.default_rng(1).standard_normal((300, h)) * 0.02).astype(np.float32)\n"
            "forced = np.random.default_rng(2).integers(0, 151643, 6).astype(np.int32)\n" % (root, model_dir)) + code
    return subprocess.run([sys.executable, "-c", prog], env=dict(os.environ, **env_extra), capture_output=True,
                          text=True, cwd=root)


def test_streaming_matvec_stage_size_keeps_bits(m17l4_dir):
    """The streaming decode matvec (1.7B gate/up at one sequence) may put several 512-byte
    column chunks in one ring stage; every lane still adds its chunks in column order, so the
    logits are bit-identical for 8 KB and 64 KB stages, in both weight modes."""
    code = ("for mode in ('bf16', 'int8'):\n"
            "    eng.set_decode_mode(mode)\n"
            "    _, lg, _ = eng.debug_decode(rows, 6, forced=forced, want_logits=True)\n"
            "    print(mode, hashlib.sha1(lg.tobytes()).hexdigest())\n")
    outs = []
    for kb in ("8", "64"):
        p = _child({"QASR_MV_STAGE_KB": kb}, code, m17l4_dir)
        assert p.returncode == 0, p.stdout + p.stderr
        outs.append([ln for ln in p.stdout.splitlines() if ln.startswith(("bf16", "int8"))])
    assert len(outs[0]) == 2 and outs[0] == outs[1], outs


def test_unplannable_matvec_fails_loudly(m17l4_dir):
    """A decode matvec whose ring of two stages does not fit its shared-memory budget is not
    launched, and the decode reports that instead of returning tokens from a partial step."""
    code = ("eng.set_decode_mode('bf16')\n"
            "try:\n"
            "    eng.debug_decode(rows, 4, forced=forced)\n"
            "    print('decoded')\n"
            "except RuntimeError as e:\n"
            "    print('raised:', e)\n")
    p = _child({"QASR_MV_BUDGET_KB": "16"}, code, m17l4_dir)
    assert p.returncode == 0, p.stdout + p.stderr
    assert "raised:" in p.stdout and "two stages" in p.stdout, p.stdout + p.stderr
