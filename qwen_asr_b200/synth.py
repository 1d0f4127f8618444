"""Seeded synthetic Qwen3-ASR checkpoints and audio.

Real Qwen3-ASR weights and speech are not available offline, so every test and
benchmark runs on random-init weights written in the exact safetensors layout the
reference loader reads (tensor names from crates/qwen-asr/src/encoder.rs:126-164 and
crates/qwen-asr/src/decoder.rs:71-151; shapes as detected by
crates/qwen-asr/src/config.rs:110-157), plus a synthetic byte-level BPE
vocab.json/merges.txt (format read by crates/qwen-asr/src/tokenizer.rs:128-201,281-312)
and seeded speech-like audio.

Weights: matrices and biases ~ N(0, 0.02) rounded to bf16, norm weights 1, LayerNorm
biases 0, tied lm_head (no thinker.lm_head.weight). Every tensor has its own generator
seeded by (seed, crc32(name)), so the content does not depend on write order.
"""
from __future__ import annotations

import json
import os
import struct
import zlib

import numpy as np

VOCAB_SIZE = 151936
N_REGULAR_TOKENS = 151643  # ids 0..151642 live in vocab.json; specials do not
CONV_HIDDEN = 480

PRESETS = {
    # name: (enc_d, enc_layers, enc_ffn, dec_hidden, dec_layers, dec_inter, q_heads, kv_heads)
    "0.6b": (896, 18, 3584, 1024, 28, 3072, 16, 8),
    "1.7b": (1024, 24, 4096, 2048, 28, 6144, 16, 8),
    # 1.7B widths with 4 encoder and 4 decoder layers: long streaming parity runs at C5's
    # shapes while the CPU oracle keeps up.
    "1.7b-l4": (1024, 4, 4096, 2048, 4, 6144, 16, 8),
    # Small shapes for CPU tests (loaded through the shape-inferring config path).
    "tiny": (128, 2, 256, 256, 2, 512, 4, 2),
    # Forced aligner: the large (1.7B) encoder with the 0.6B decoder (config.rs:109-110) and
    # an untied lm_head of classify classes (config.rs:145-151).
    "aligner": (1024, 24, 4096, 1024, 28, 3072, 16, 8),
    "tiny-aligner": (128, 2, 256, 256, 2, 512, 4, 2),
}
ALIGNER_CLASSES = {"aligner": 5000, "tiny-aligner": 300}


def tensor_specs(preset: str):
    """Yield (name, shape, init) for every tensor of a preset; init in {normal, one, zero}."""
    enc_d, enc_l, enc_ffn, hid, dec_l, inter, qh, kvh = PRESETS[preset]
    p = "thinker.audio_tower."
    specs = []
    specs += [(p + "conv2d1.weight", (CONV_HIDDEN, 1, 3, 3), "normal"),
              (p + "conv2d1.bias", (CONV_HIDDEN,), "normal")]
    for i in (2, 3):
        specs += [(p + f"conv2d{i}.weight", (CONV_HIDDEN, CONV_HIDDEN, 3, 3), "normal"),
                  (p + f"conv2d{i}.bias", (CONV_HIDDEN,), "normal")]
    specs.append((p + "conv_out.weight", (enc_d, CONV_HIDDEN * 16), "normal"))
    for i in range(enc_l):
        lp = f"{p}layers.{i}."
        for nm in ("q_proj", "k_proj", "v_proj", "out_proj"):
            specs += [(lp + f"self_attn.{nm}.weight", (enc_d, enc_d), "normal"),
                      (lp + f"self_attn.{nm}.bias", (enc_d,), "normal")]
        specs += [(lp + "self_attn_layer_norm.weight", (enc_d,), "one"),
                  (lp + "self_attn_layer_norm.bias", (enc_d,), "zero"),
                  (lp + "fc1.weight", (enc_ffn, enc_d), "normal"),
                  (lp + "fc1.bias", (enc_ffn,), "normal"),
                  (lp + "fc2.weight", (enc_d, enc_ffn), "normal"),
                  (lp + "fc2.bias", (enc_d,), "normal"),
                  (lp + "final_layer_norm.weight", (enc_d,), "one"),
                  (lp + "final_layer_norm.bias", (enc_d,), "zero")]
    specs += [(p + "ln_post.weight", (enc_d,), "one"),
              (p + "ln_post.bias", (enc_d,), "zero"),
              (p + "proj1.weight", (enc_d, enc_d), "normal"),
              (p + "proj1.bias", (enc_d,), "normal"),
              (p + "proj2.weight", (hid, enc_d), "normal"),
              (p + "proj2.bias", (hid,), "normal")]
    m = "thinker.model."
    specs.append((m + "embed_tokens.weight", (VOCAB_SIZE, hid), "normal"))
    for i in range(dec_l):
        lp = f"{m}layers.{i}."
        specs += [(lp + "self_attn.q_proj.weight", (qh * 128, hid), "normal"),
                  (lp + "self_attn.k_proj.weight", (kvh * 128, hid), "normal"),
                  (lp + "self_attn.v_proj.weight", (kvh * 128, hid), "normal"),
                  (lp + "self_attn.o_proj.weight", (hid, qh * 128), "normal"),
                  (lp + "self_attn.q_norm.weight", (128,), "one"),
                  (lp + "self_attn.k_norm.weight", (128,), "one"),
                  (lp + "input_layernorm.weight", (hid,), "one"),
                  (lp + "post_attention_layernorm.weight", (hid,), "one"),
                  (lp + "mlp.gate_proj.weight", (inter, hid), "normal"),
                  (lp + "mlp.up_proj.weight", (inter, hid), "normal"),
                  (lp + "mlp.down_proj.weight", (hid, inter), "normal")]
    specs.append((m + "norm.weight", (hid,), "one"))
    if preset in ALIGNER_CLASSES:
        specs.append(("thinker.lm_head.weight", (ALIGNER_CLASSES[preset], hid), "normal"))
    return specs


def _bf16_bits(n: int, seed: int, name: str, init: str, device: str) -> np.ndarray:
    if init == "one":
        return np.full(n, 0x3F80, dtype=np.uint16)
    if init == "zero":
        return np.zeros(n, dtype=np.uint16)
    import torch  # fixture generation only: fast seeded normals + RNE rounding to bf16
    g = torch.Generator(device=device)
    g.manual_seed((seed * 1000003 + zlib.crc32(name.encode())) & 0x7FFFFFFFFFFF)
    t = torch.randn(n, generator=g, dtype=torch.float32, device=device).mul_(0.02)
    return t.to(torch.bfloat16).view(torch.int16).cpu().numpy().view(np.uint16)


def write_model(out_dir: str, preset: str = "0.6b", seed: int = 0, device: str = "cpu") -> str:
    """Write model.safetensors + vocab.json + merges.txt into out_dir; returns out_dir.

    Skips the work if a completed model with the same preset/seed is already there.
    """
    os.makedirs(out_dir, exist_ok=True)
    stamp = os.path.join(out_dir, "SYNTH_DONE")
    tag = f"{preset} seed={seed} device={device}\n"
    if os.path.exists(stamp) and open(stamp).read() == tag:
        return out_dir
    specs = tensor_specs(preset)
    header = {}
    off = 0
    for name, shape, _ in specs:
        nbytes = int(np.prod(shape)) * 2
        header[name] = {"dtype": "BF16", "shape": list(shape), "data_offsets": [off, off + nbytes]}
        off += nbytes
    hjson = json.dumps(header, separators=(",", ":")).encode()
    hjson += b" " * ((8 - len(hjson) % 8) % 8)
    path = os.path.join(out_dir, "model.safetensors")
    with open(path + ".tmp", "wb") as f:
        f.write(struct.pack("<Q", len(hjson)))
        f.write(hjson)
        for name, shape, init in specs:
            f.write(_bf16_bits(int(np.prod(shape)), seed, name, init, device).tobytes())
    os.replace(path + ".tmp", path)
    write_vocab(out_dir, seed)
    with open(stamp, "w") as f:
        f.write(tag)
    return out_dir


def gpt2_byte_to_unicode():
    """GPT-2 byte->codepoint table (same construction as tokenizer.rs:6-31)."""
    table = [0] * 256
    n = 0
    for b in range(256):
        if 33 <= b <= 126 or 161 <= b <= 172 or 174 <= b <= 255:
            table[b] = b
        else:
            table[b] = 256 + n
            n += 1
    return table


def write_vocab(out_dir: str, seed: int = 0, n_merges: int = 4000) -> None:
    """Synthetic byte-level BPE vocabulary with N_REGULAR_TOKENS entries.

    ids 0..255 are the single-byte symbols; the next n_merges ids are produced by a
    ranked merge list (so encode() has real merges to apply); the rest are distinct
    random 2..6-byte strings that only decode.
    """
    rng = np.random.default_rng(10_000 + seed)
    b2u = gpt2_byte_to_unicode()
    sym = [chr(b2u[b]) for b in range(256)]
    vocab = {s: i for i, s in enumerate(sym)}
    tokens = list(sym)
    merges = []
    # Favour printable ASCII letters/space so "language English" style prompts merge.
    base = [chr(b2u[b]) for b in list(range(97, 123)) + list(range(65, 91)) + [32]]
    pool = list(base)
    while len(merges) < n_merges:
        a = pool[int(rng.integers(len(pool)))]
        b = pool[int(rng.integers(len(pool)))]
        t = a + b
        if t in vocab or len(t) > 8:
            continue
        vocab[t] = len(tokens)
        tokens.append(t)
        merges.append(f"{a} {b}")
        pool.append(t)
    while len(tokens) < N_REGULAR_TOKENS:
        ln = int(rng.integers(2, 7))
        t = "".join(sym[int(x)] for x in rng.integers(0, 256, ln))
        if t in vocab:
            continue
        vocab[t] = len(tokens)
        tokens.append(t)
    with open(os.path.join(out_dir, "vocab.json"), "w", encoding="utf-8") as f:
        json.dump(vocab, f, ensure_ascii=False)
    with open(os.path.join(out_dir, "merges.txt"), "w", encoding="utf-8") as f:
        f.write("#version: synthetic\n")
        f.write("\n".join(merges) + "\n")


def synth_audio(n_samples: int, seed: int) -> np.ndarray:
    """Seeded speech-like audio, returned as f32 in [-1, 1] quantised to s16 steps.

    Sum of 3-5 harmonics of an f0 track wandering in 80-400 Hz, times a ~4 Hz
    raised-cosine syllable envelope, plus pink noise at -30 dBFS, peak-normalised to
    -3 dBFS and quantised to 16-bit PCM at 16 kHz.
    """
    sr = 16000
    rng = np.random.default_rng(seed)
    t = np.arange(n_samples, dtype=np.float64) / sr
    # f0: smoothed random walk in log-frequency
    n_ctl = max(2, n_samples // 800 + 2)
    ctl = np.cumsum(rng.normal(0, 0.08, n_ctl))
    ctl = np.log(80.0) + (np.log(400.0) - np.log(80.0)) * (0.5 + 0.5 * np.tanh(ctl))
    f0 = np.exp(np.interp(np.arange(n_samples) / 800.0, np.arange(n_ctl), ctl))
    phase = 2 * np.pi * np.cumsum(f0) / sr
    n_h = int(rng.integers(3, 6))
    sig = np.zeros(n_samples)
    for h in range(1, n_h + 1):
        sig += (0.6 ** (h - 1)) * np.sin(h * phase + rng.uniform(0, 2 * np.pi))
    syl_rate = rng.uniform(3.5, 4.5)
    env = 0.5 - 0.5 * np.cos(2 * np.pi * syl_rate * t + rng.uniform(0, 2 * np.pi))
    sig *= env ** 1.5
    # pink noise via 1/sqrt(f) spectral shaping
    white = rng.normal(0, 1, n_samples)
    spec = np.fft.rfft(white)
    f = np.arange(spec.size)
    f[0] = 1
    pink = np.fft.irfft(spec / np.sqrt(f), n_samples)
    pink /= max(1e-12, np.max(np.abs(pink)))
    peak = max(1e-12, np.max(np.abs(sig)))
    sig = sig / peak * 10 ** (-3 / 20) * 0.97 + pink * 10 ** (-30 / 20)
    sig = sig / max(1e-12, np.max(np.abs(sig))) * 10 ** (-3 / 20)
    s16 = np.clip(np.round(sig * 32767.0), -32768, 32767).astype(np.int16)
    return (s16.astype(np.float32) / np.float32(32768.0)).astype(np.float32)


def write_wav(path: str, samples: np.ndarray, sr: int = 16000, channels: int = 1) -> None:
    """16-bit PCM WAV writer (the only format parse_wav_buffer accepts, audio.rs:22-91)."""
    x = np.asarray(samples, dtype=np.float32)
    s16 = np.clip(np.round(x * 32768.0), -32768, 32767).astype("<i2")
    data = s16.tobytes()
    hdr = b"RIFF" + struct.pack("<I", 36 + len(data)) + b"WAVE"
    hdr += b"fmt " + struct.pack("<IHHIIHH", 16, 1, channels, sr, sr * channels * 2, channels * 2, 16)
    hdr += b"data" + struct.pack("<I", len(data))
    with open(path, "wb") as f:
        f.write(hdr + data)
