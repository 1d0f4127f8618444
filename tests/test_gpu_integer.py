"""Bit-exact integer work on the GPU: the int8 weight rows and scales quantised on the device
at load against the oracle's quantiser (kernels/mod.rs:1805-1829 round, kernels/neon.rs:636-694
truncation), and the KV cache (decoder.rs:185-253): rows at exactly the positions the oracle
writes, and the doubling grow (KvCache::grow, decoder.rs:199-231) keeping every row bit for bit.
All through the C ABI."""
import os
import subprocess
import sys

import numpy as np
import pytest

from qwen_asr_b200 import synth

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _layer_mats(O, d, layer):
    """Decoder matrices of one layer in the engine's row order, as bf16 bits."""
    st = O.SafeTensors(d)
    lp = f"thinker.model.layers.{layer}."
    wq, wk, wv, wo = (st.bf16(lp + f"self_attn.{n}.weight") for n in ("q_proj", "k_proj", "v_proj", "o_proj"))
    gate, up, down = (st.bf16(lp + f"mlp.{n}.weight") for n in ("gate_proj", "up_proj", "down_proj"))
    gu = np.empty((2 * gate.shape[0], gate.shape[1]), dtype=np.uint16)
    gu[0::2], gu[1::2] = gate, up
    return {0: np.concatenate([wq, wk, wv]), 1: wo, 2: gu, 3: down}, st


def _check_quant(eng, O, d, mode, layers):
    for layer in layers:
        mats, st = _layer_mats(O, d, layer)
        for which, bits in mats.items():
            q, s = eng.debug_quant(layer, which)
            rq, rs = O.quantize_weights(bits, mode)
            assert np.array_equal(q, rq), (mode, layer, which, int(np.sum(q != rq)))
            assert np.array_equal(s.view(np.uint32), rs.view(np.uint32)), (mode, layer, which)
    q, s = eng.debug_quant(0, 4)
    rq, rs = O.quantize_weights(st.bf16("thinker.model.embed_tokens.weight"), mode)  # tied lm_head
    assert np.array_equal(q, rq) and np.array_equal(s.view(np.uint32), rs.view(np.uint32))


@pytest.mark.parametrize("preset", ["tiny", "0.6b"])
def test_int8_weights_trunc_bit_exact(preset, tiny_dir, m06_dir):
    import qwen_asr_b200 as Q
    from oracle import qwen_oracle as O
    d = tiny_dir if preset == "tiny" else m06_dir
    eng = Q.Engine(d)
    _check_quant(eng, O, d, "trunc", [0, eng.model_info()["dec_layers"] - 1])


def test_int8_weights_round_bit_exact(tiny_dir):
    """QASR_WEIGHT_QUANT=round selects the generic round-half-away quantiser at load (read
    once per process, so it runs in a child process)."""
    code = (
        "import sys; sys.path.insert(0, %r)\n"
        "import qwen_asr_b200 as Q\n"
        "from oracle import qwen_oracle as O\n"
        "from tests.test_gpu_integer import _check_quant\n"
        "e = Q.Engine(%r)\n"
        "_check_quant(e, O, %r, 'round', [0, 1])\n"
        "print('round ok')\n" % (ROOT, tiny_dir, tiny_dir))
    env = dict(os.environ, QASR_WEIGHT_QUANT="round")
    r = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True, cwd=ROOT)
    assert r.returncode == 0 and "round ok" in r.stdout, r.stdout + r.stderr


def _oracle_run(O, model, rows, forced, n_steps):
    dec = O.Decoder(model)
    dec.record_logits = True
    dec.prefill(rows[:-1])
    x = rows[-1]
    lg = []
    for i in range(n_steps):
        dec.forward(x)
        lg.append(dec.last_logits)
        if i + 1 < n_steps:
            x = model.embed(int(forced[i]))
    return dec, np.stack(lg)


@pytest.mark.parametrize("preset,mode", [("tiny", "bf16"), ("tiny", "int8"), ("0.6b", "bf16")])
def test_kv_cache_rows_match_oracle(preset, mode, tiny_dir, m06_dir):
    """After prefill + N decode steps every written KV row sits at the oracle's position:
    values within f32 tolerance, and each engine row is nearest to the oracle row of the same
    position (an off-by-one or a head/layer mix-up fails)."""
    import qwen_asr_b200 as Q
    from oracle import qwen_oracle as O
    d = tiny_dir if preset == "tiny" else m06_dir
    eng = Q.Engine(d)
    eng.set_decode_mode(mode)
    model = O.Model(d, decode_mode=mode)
    x = synth.synth_audio(16000 * 2, seed=71)
    c = O.Ctx.__new__(O.Ctx)
    c.model, c.tok, c.prompt, c.force_language = model, None, None, None
    rows = O.prompt_rows(c, model.encode(O.mel_spectrogram(x)))
    n_steps = 12
    forced = np.random.default_rng(71).integers(0, 151643, n_steps).astype(np.int32)
    dec, _ = _oracle_run(O, model, rows, forced, n_steps)
    eng.debug_decode(rows, n_steps, forced=forced)
    P = rows.shape[0] - 1 + n_steps  # prefill rows + one row per decode step
    assert dec.kv.len == P
    for layer in range(model.cfg.dec_layers):
        k, v = eng.debug_kv(layer, P)
        rk, rv = dec.kv.k[layer, :, :P], dec.kv.v[layer, :, :P]
        for got, ref in ((k, rk), (v, rv)):
            scale = float(np.max(np.abs(ref)))
            tol = 5e-2 if mode == "int8" else 1e-4
            assert float(np.max(np.abs(got - ref))) <= tol * scale, (layer, mode)
            for hh in range(got.shape[0]):
                # every engine row is nearest to the oracle row of its own position; repeated
                # prompt tokens give (nearly) identical V rows at several positions, so rows
                # closer than the value tolerance count as ties
                dist = ((got[hh][:, None, :].astype(np.float64) - ref[hh][None, :, :]) ** 2).sum(-1)  # [P][P]
                tie = 128 * (tol * scale) ** 2
                assert np.all(np.diag(dist) <= dist.min(axis=1) + tie), (layer, hh)


def test_kv_grow_keeps_rows_bit_exact(tiny_dir):
    """Forcing the cache past its 4096 positions doubles it; every written row survives bit
    for bit, and a decode after the grow (new row pitch, rebuilt step graph) gives the same
    logits as before it."""
    import qwen_asr_b200 as Q
    from oracle import qwen_oracle as O
    eng = Q.Engine(tiny_dir)
    eng.set_decode_mode("bf16")
    model = O.Model(tiny_dir, decode_mode="bf16")
    x = synth.synth_audio(16000 * 2, seed=72)
    c = O.Ctx.__new__(O.Ctx)
    c.model, c.tok, c.prompt, c.force_language = model, None, None, None
    rows = O.prompt_rows(c, model.encode(O.mel_spectrogram(x)))
    forced = np.random.default_rng(72).integers(0, 151643, 10).astype(np.int32)
    _, lg0, _ = eng.debug_decode(rows, 10, forced=forced, want_logits=True)
    P = rows.shape[0] - 1 + 10
    before = [eng.debug_kv(layer, P) for layer in range(model.cfg.dec_layers)]
    cap0 = eng.kv_capacity()
    assert cap0 >= 4096
    cap1 = eng.grow_kv(cap0 + 1)
    assert cap1 == 2 * cap0  # doubling (decoder.rs:205-208)
    for layer in range(model.cfg.dec_layers):
        k, v = eng.debug_kv(layer, P)
        assert np.array_equal(k.view(np.uint32), before[layer][0].view(np.uint32))
        assert np.array_equal(v.view(np.uint32), before[layer][1].view(np.uint32))
    _, lg1, _ = eng.debug_decode(rows, 10, forced=forced, want_logits=True)
    assert np.array_equal(lg0.view(np.uint32), lg1.view(np.uint32))
