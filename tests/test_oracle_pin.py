"""Pins the CPU oracle against independent implementations of the same network and
tokeniser: transformers' Qwen3-Omni audio encoder (Qwen3OmniMoeAudioEncoder) for the audio
tower and Qwen3ForCausalLM for the text decoder, loaded with the synthetic checkpoint's
weights in f32, and the `tokenizers` library's byte-level BPE for the tokeniser.

The reference's encoder (crates/qwen-asr/src/encoder.rs:186-358) and decoder
(crates/qwen-asr/src/decoder.rs:455-645) are the same network as those classes, with three
differences that these tests bridge:
  * the reference uses the tanh GELU everywhere (kernels/mod.rs:1283-1288); transformers'
    audio encoder calls the erf GELU after each conv, so it is swapped for the tanh form;
  * the reference attends inside windows of 104 tokens (encoder.rs:292-298); transformers'
    eager attention only windows when given the block mask, which its forward does not pass,
    so each layer is handed `_prepare_attention_mask`;
  * transformers zero-pads a ragged last 100-frame chunk to a full chunk before the convs,
    whereas the reference convolves it at its own width (encoder.rs:213-247), which changes the
    last token; the encoder case therefore uses whole chunks.
Everything else (conv front end, the col = channel*16 + freq flattening, the per-chunk
sinusoid, LayerNorm eps, biases, scaling, windows, GQA, q/k RMSNorm, NeoX RoPE at theta 1e6,
tied lm_head) is compared as is, to f32 rounding."""
import types

import numpy as np
import pytest

from qwen_asr_b200 import synth

torch = pytest.importorskip("torch")
pytest.importorskip("transformers")


def _encoder(model, monkeypatch):
    import torch.nn.functional as TF
    import transformers.models.qwen3_omni_moe.modeling_qwen3_omni_moe as MM
    from transformers.models.qwen3_omni_moe.configuration_qwen3_omni_moe import Qwen3OmniMoeAudioEncoderConfig
    from oracle import qwen_oracle as O

    c = model.cfg
    cfg = Qwen3OmniMoeAudioEncoderConfig(
        num_mel_bins=O.MEL_BINS, d_model=c.enc_d_model, encoder_layers=c.enc_layers,
        encoder_attention_heads=c.enc_heads, encoder_ffn_dim=c.enc_ffn_dim,
        downsample_hidden_size=O.CONV_HIDDEN, output_dim=c.dec_hidden, n_window=c.enc_n_window,
        n_window_infer=c.enc_n_window_infer, conv_chunksize=500,
        activation_function="gelu_pytorch_tanh", max_source_positions=1500, scale_embedding=False)
    cfg._attn_implementation = "eager"
    tanh_f = types.SimpleNamespace(**{k: getattr(TF, k) for k in dir(TF) if not k.startswith("__")})
    tanh_f.gelu = lambda t: TF.gelu(t, approximate="tanh")
    monkeypatch.setattr(MM, "F", tanh_f)
    enc = MM.Qwen3OmniMoeAudioEncoder(cfg).eval()
    st = O.SafeTensors(model.model_dir)
    sd = {k: torch.from_numpy(st.f32("thinker.audio_tower." + k).reshape(v.shape).copy())
          for k, v in enc.state_dict().items()}
    enc.load_state_dict(sd)
    for layer in enc.layers:
        fwd = layer.forward
        layer.forward = (lambda fwd: lambda hs, cu, **kw: fwd(
            hs, cu, attention_mask=enc._prepare_attention_mask(hs, cu)))(fwd)
    return enc


def _decoder(model):
    from transformers import Qwen3Config, Qwen3ForCausalLM
    from oracle import qwen_oracle as O

    c = model.cfg
    cfg = Qwen3Config(
        vocab_size=c.vocab_size, hidden_size=c.dec_hidden, intermediate_size=c.dec_intermediate,
        num_hidden_layers=c.dec_layers, num_attention_heads=c.dec_heads,
        num_key_value_heads=c.dec_kv_heads, head_dim=c.dec_head_dim, rms_norm_eps=float(c.eps),
        rope_theta=float(c.theta), tie_word_embeddings=True, hidden_act="silu",
        attention_bias=False, max_position_embeddings=65536)
    cfg._attn_implementation = "eager"
    lm = Qwen3ForCausalLM(cfg).eval()
    st = O.SafeTensors(model.model_dir)
    sd = {}
    for k, v in lm.state_dict().items():
        name = ("thinker.model." + k[len("model."):]) if k.startswith("model.") else "thinker.model.embed_tokens.weight"
        sd[k] = torch.from_numpy(st.f32(name).reshape(v.shape).copy())
    lm.load_state_dict(sd)
    return lm


@pytest.fixture(params=["tiny", "1.7b-l4"])
def pin_model(request, tiny_dir):
    from oracle import qwen_oracle as O
    from tests.conftest import model_dir
    d = tiny_dir if request.param == "tiny" else model_dir("1.7b-l4", 1)
    return O.Model(d, decode_mode="bf16")


def test_encoder_matches_transformers(pin_model, monkeypatch):
    """Model.encode over two windows (11 chunks = 143 tokens) equals the transformers audio
    encoder to f32 rounding."""
    from oracle import qwen_oracle as O
    mel = O.mel_spectrogram(synth.synth_audio(16000 * 11 + 800, seed=5))[:, :1100].copy()
    ref = pin_model.encode(mel)
    enc = _encoder(pin_model, monkeypatch)
    with torch.no_grad():
        got = enc(torch.from_numpy(mel), feature_lens=torch.tensor([mel.shape[1]])).last_hidden_state.numpy()
    assert got.shape == ref.shape == (143, pin_model.cfg.dec_hidden)
    assert float(np.max(np.abs(got - ref))) <= 1e-5 * float(np.max(np.abs(ref)))


def test_decoder_logits_match_transformers(pin_model):
    """Oracle prefill + bf16-mode decode steps (weights widened to f32, as the reference's
    bf16 matvecs compute) give the logits of Qwen3ForCausalLM over the same embedding rows
    (audio rows from Model.encode, the prompt and three forced tokens), to f32 rounding, with
    the same argmax at every step."""
    from oracle import qwen_oracle as O
    m = pin_model
    ctx = O.Ctx.__new__(O.Ctx)
    ctx.model, ctx.tok, ctx.prompt, ctx.force_language = m, None, None, None
    rows = O.prompt_rows(ctx, m.encode(O.mel_spectrogram(synth.synth_audio(16000 * 3, seed=9))))
    forced = [17, 9000, O.TOKEN_ENDOFTEXT]
    dec = O.Decoder(m)
    dec.record_logits = True
    dec.prefill(rows[:-1])
    x, lg = rows[-1], []
    for t in forced + [None]:
        dec.forward(x)
        lg.append(dec.last_logits)
        if t is not None:
            x = m.embed(t)
    emb = np.concatenate([rows] + [m.embed(t)[None] for t in forced]).astype(np.float32)
    lm = _decoder(m)
    with torch.no_grad():
        out = lm(inputs_embeds=torch.from_numpy(emb[None])).logits[0, -len(lg):].numpy()
    for step, (a, b) in enumerate(zip(lg, out)):
        assert float(np.max(np.abs(a - b))) <= 1e-5 * float(np.max(np.abs(a))), step
        assert int(np.argmax(a)) == int(np.argmax(b)), step


def test_tokenizer_matches_hf_tokenizers(tiny_dir):
    """The oracle's whole-string byte-level BPE (tokenizer.rs:227-279: no pre-tokenizer split,
    lowest-rank merge first) and its id -> bytes table equal the `tokenizers` library's BPE
    model on the same vocab.json / merges.txt with a byte-level pre-tokenizer that does not
    split (the host C++ tokenizer is checked against the oracle in test_host_abi.py)."""
    import json
    import os
    import random
    tokenizers = pytest.importorskip("tokenizers")
    from oracle import qwen_oracle as O
    T = O.Tokenizer(tiny_dir)
    with open(os.path.join(tiny_dir, "vocab.json"), encoding="utf-8") as f:
        vocab = json.load(f)
    merges = []
    with open(os.path.join(tiny_dir, "merges.txt"), encoding="utf-8") as f:
        for line in f.read().splitlines():
            if line and not line.startswith("#"):
                a, b = line.split(" ", 1)
                merges.append((a, b))
    tk = tokenizers.Tokenizer(tokenizers.models.BPE(vocab=vocab, merges=merges))
    tk.pre_tokenizer = tokenizers.pre_tokenizers.ByteLevel(add_prefix_space=False, use_regex=False)
    rng = random.Random(1)
    words = ["the", " and", " speech", " model", "ing", " 你好", "é", "\n", " 123", "!?", " 😀", "  "]
    texts = ["hello world", " The quick brown fox.", "Zürich — 東京 😀", "a" * 50, "language English<asr_text>"]
    texts += ["".join(rng.choice(words) for _ in range(rng.randint(1, 12))) for _ in range(200)]
    for t in texts:
        assert T.encode(t) == tk.encode(t).ids, t
    for tid in range(0, len(vocab), 7):
        tok = tk.id_to_token(tid)
        assert bytes(T.b2u.index(ord(c)) for c in tok) == T.decode_bytes(tid), tid
