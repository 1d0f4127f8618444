"""CPU ORACLE (test infrastructure only) — numpy restatement of the reference's
Qwen3-ASR transcription path (huanglizhuo/QwenASR, crates/qwen-asr).

This module is the checker for the CUDA engine. Only tests/, __graft_entry__.smoke()
and bench.py's cpu_baseline / --impl reference legs may import it. The product
(qwen_asr_b200 + libqwen_asr.so) never calls it.

Parity status: the reference is Rust and cannot be built here (no cargo/rustc), and
its int8 decode is `unimplemented!()` on x86_64 (kernels/mod.rs:876-880), so no
reference output can be produced on this machine. The reference ships no golden
vectors; its unit tests only pin envelopes (tests/kernels.rs, tests/audio.rs), which
tests/test_oracle.py re-checks against this module. End-to-end parity of this
restatement is therefore UNPINNED against the reference binary; its mel front end
is additionally cross-checked against transformers' WhisperFeatureExtractor where
that package is importable.

Arithmetic follows the reference's order where it changes f32 rounding:
* float32 GEMMs go through numpy matmul (OpenBLAS sgemm — the same third-party
  routine crates/qwen-asr/build.rs links on Linux; it is not vendored in the
  reference, no version is pinned there; numpy 2.3 bundles OpenBLAS 0.3.30);
* int8 dot products are exact int32 (K-chunks of <=1024 in float32 are exact);
* quantisers reproduce kernels/mod.rs:1795-1829 and kernels/neon.rs:637-694;
* activations use the exact generic formulas (tanh GELU, exp SiLU), not the
  AVX/NEON polynomial exp approximations (kernels/avx.rs:487).
"""
from __future__ import annotations

import json
import math
import os
import struct

import numpy as np

F32 = np.float32

# config.rs:3-20
SAMPLE_RATE = 16000
MEL_BINS = 128
HOP_LENGTH = 160
WINDOW_SIZE = 400
N_FFT = 400
N_FREQ = 201
VOCAB_SIZE = 151936
TOKEN_IM_START = 151644
TOKEN_IM_END = 151645
TOKEN_ENDOFTEXT = 151643
TOKEN_AUDIO_START = 151669
TOKEN_AUDIO_END = 151670
TOKEN_ASR_TEXT = 151704
CONV_HIDDEN = 480

# transcribe.rs:13-23
PREFIX_HEAD = [151644, 8948, 198]
PREFIX_TAIL = [151645, 198, 151644, 872, 198, 151669]
SUFFIX_BASE = [151670, 151645, 198, 151644, 77091, 198]
STREAM_DEGEN_MAX_PERIOD = 6
STREAM_DEGEN_MIN_REPEATS = 4
STREAM_STALE_CHUNKS = 4
STREAM_RESET_INTERVAL_CHUNKS = 45
STREAM_RESET_CARRY_TOKENS = 24
STREAM_MAX_ENC_WINDOWS = 4

SUPPORTED_LANGUAGES = [  # config.rs:159-165
    "Chinese", "English", "Cantonese", "Arabic", "German", "French",
    "Spanish", "Portuguese", "Indonesian", "Italian", "Korean", "Russian",
    "Thai", "Vietnamese", "Japanese", "Turkish", "Hindi", "Malay", "Dutch",
    "Swedish", "Danish", "Finnish", "Polish", "Czech", "Filipino",
    "Persian", "Greek", "Romanian", "Hungarian", "Macedonian",
]

# Rust char::is_whitespace (Unicode White_Space), used by str::trim.
_RUST_WS = set([0x09, 0x0A, 0x0B, 0x0C, 0x0D, 0x20, 0x85, 0xA0, 0x1680, 0x2028, 0x2029,
                0x202F, 0x205F, 0x3000] + list(range(0x2000, 0x200B)))


def rust_trim(s: str) -> str:
    a, b = 0, len(s)
    while a < b and ord(s[a]) in _RUST_WS:
        a += 1
    while b > a and ord(s[b - 1]) in _RUST_WS:
        b -= 1
    return s[a:b]


def lossy(b: bytes) -> str:
    """String::from_utf8_lossy (maximal-subpart U+FFFD substitution)."""
    return b.decode("utf-8", errors="replace")


def normalize_language(lang: str):
    """config.rs:167-182."""
    t = rust_trim(lang)
    if not t:
        return None
    norm = t[0].upper() + t[1:].lower()
    return norm if norm in SUPPORTED_LANGUAGES else None


def bf16_to_f32(bits: np.ndarray) -> np.ndarray:
    return (bits.astype(np.uint32) << 16).view(np.float32)


def round_half_away(v: np.ndarray) -> np.ndarray:
    """Rust f32::round on float32 input (evaluated in float64, which is exact)."""
    d = v.astype(np.float64)
    return np.sign(d) * np.floor(np.abs(d) + 0.5)


# ---------------------------------------------------------------------------
# safetensors (safetensors.rs:72-281) + config detection (config.rs:110-157)
# ---------------------------------------------------------------------------

class SafeTensors:
    def __init__(self, model_dir: str):
        single = os.path.join(model_dir, "model.safetensors")
        if os.path.exists(single):
            paths = [single]
        else:
            names = sorted(n for n in os.listdir(model_dir)
                           if n.startswith("model-") and n.endswith(".safetensors"))
            if not names:
                raise FileNotFoundError(f"no safetensors files in {model_dir}")
            paths = [os.path.join(model_dir, n) for n in names]
        self.meta = {}
        for p in paths:
            mm = np.memmap(p, dtype=np.uint8, mode="r")
            hlen = struct.unpack("<Q", bytes(mm[:8]))[0]
            if hlen > len(mm) - 8:
                raise ValueError("bad safetensors header length")
            hdr = json.loads(bytes(mm[8:8 + hlen]).decode("utf-8"))
            for name, info in hdr.items():
                if name == "__metadata__":
                    continue
                a, b = info["data_offsets"]
                if name not in self.meta:
                    self.meta[name] = (mm, 8 + hlen + a, 8 + hlen + b, info["dtype"], tuple(info["shape"]))

    def has(self, name):
        return name in self.meta

    def shape(self, name):
        return self.meta[name][4] if name in self.meta else None

    def bf16(self, name) -> np.ndarray:
        mm, a, b, dt, shape = self.meta[name]
        if dt != "BF16":
            raise ValueError(f"{name}: expected BF16, got {dt}")
        return np.frombuffer(mm[a:b], dtype=np.uint16).reshape(shape)

    def f32(self, name) -> np.ndarray:
        mm, a, b, dt, shape = self.meta[name]
        if dt == "F32":
            return np.frombuffer(mm[a:b], dtype=np.float32).reshape(shape).copy()
        if dt == "BF16":
            return bf16_to_f32(self.bf16(name))
        raise ValueError(f"{name}: unsupported dtype {dt}")


class Config:
    pass


def detect_config(st: SafeTensors) -> Config:
    """QwenConfig::detect (config.rs:110-157), extended to infer encoder/decoder depth and
    widths from tensor shapes so small test checkpoints load; for the two published
    variants the inferred values equal the reference's fixed presets."""
    c = Config()
    has18 = st.has("thinker.audio_tower.layers.18.self_attn.q_proj.weight")
    emb = st.shape("thinker.model.embed_tokens.weight")
    gate = st.shape("thinker.model.layers.0.mlp.gate_proj.weight")
    c.dec_hidden = emb[1] if emb and len(emb) == 2 else (2048 if has18 else 1024)
    c.dec_intermediate = gate[0] if gate and len(gate) == 2 else (6144 if c.dec_hidden >= 2048 else 3072)
    if has18:
        c.enc_d_model, c.enc_layers, c.enc_heads, c.enc_head_dim, c.enc_ffn_dim = 1024, 24, 16, 64, 4096
    else:
        c.enc_d_model, c.enc_layers, c.enc_heads, c.enc_head_dim, c.enc_ffn_dim = 896, 18, 14, 64, 3584
    # shape inference (extension; identical for published checkpoints)
    co = st.shape("thinker.audio_tower.conv_out.weight")
    if co:
        c.enc_d_model = co[0]
        c.enc_heads = c.enc_d_model // 64
    n = 0
    while st.has(f"thinker.audio_tower.layers.{n}.self_attn.q_proj.weight"):
        n += 1
    c.enc_layers = n
    f1 = st.shape("thinker.audio_tower.layers.0.fc1.weight")
    if f1:
        c.enc_ffn_dim = f1[0]
    n = 0
    while st.has(f"thinker.model.layers.{n}.self_attn.q_proj.weight"):
        n += 1
    c.dec_layers = n
    c.dec_head_dim = 128
    c.dec_heads = st.shape("thinker.model.layers.0.self_attn.q_proj.weight")[0] // 128
    c.dec_kv_heads = st.shape("thinker.model.layers.0.self_attn.k_proj.weight")[0] // 128
    c.enc_output_dim = c.dec_hidden
    c.enc_n_window = 50
    c.enc_n_window_infer = 800
    c.enc_chunk_size = 100
    c.vocab_size = VOCAB_SIZE
    c.eps = F32(1e-6)
    c.theta = F32(1e6)
    lm = st.shape("thinker.lm_head.weight")
    c.classify_num = lm[0] if lm and lm[0] != VOCAB_SIZE else 0
    return c


# ---------------------------------------------------------------------------
# Audio (audio.rs)
# ---------------------------------------------------------------------------

def parse_wav_buffer(data: bytes):
    """audio.rs:22-91: 16-bit PCM only, downmix, resample to 16 kHz."""
    if len(data) < 44 or data[0:4] != b"RIFF" or data[8:12] != b"WAVE":
        return None
    channels = sample_rate = bits = fmt = 0
    pcm = None
    p = 12
    while p + 8 <= len(data):
        cid = data[p:p + 4]
        size = struct.unpack("<I", data[p + 4:p + 8])[0]
        if p + 8 + size > len(data):
            break
        if cid == b"fmt " and size >= 16:
            fmt, channels, sample_rate = struct.unpack("<HHI", data[p + 8:p + 16])
            bits = struct.unpack("<H", data[p + 22:p + 24])[0]
        elif cid == b"data":
            pcm = data[p + 8:min(p + 8 + size, len(data))]
        p += 8 + size + (size & 1)
    if fmt != 1 or bits != 16 or channels < 1 or pcm is None:
        return None
    n = len(pcm) // (channels * 2)
    s = np.frombuffer(pcm[:n * channels * 2], dtype="<i2").reshape(n, channels)
    if channels == 1:
        out = s[:, 0].astype(F32) / F32(32768.0)
    else:
        acc = np.zeros(n, dtype=F32)
        for ch in range(channels):  # sequential f32 sum, audio.rs:72-77
            acc = (acc + s[:, ch].astype(F32)).astype(F32)
        out = (acc / F32(channels)).astype(F32) / F32(32768.0)
    out = out.astype(F32)
    if sample_rate != SAMPLE_RATE:
        out = resample(out, sample_rate, SAMPLE_RATE)
    return out


def resample(samples: np.ndarray, from_rate: int, to_rate: int) -> np.ndarray:
    """Kaiser-windowed sinc resampler, audio.rs:133-196 (f64 arithmetic)."""
    n = len(samples)
    new_n = n * to_rate // from_rate
    sinc_half = 16
    beta = 6.0
    ratio = to_rate / from_rate
    cutoff = ratio if ratio < 1.0 else 1.0

    def i0(x):
        s = np.ones_like(x)
        term = np.ones_like(x)
        xx = x * x
        for k in range(1, 21):
            term = term * xx / (4.0 * k * k)
            s = s + term
        return s

    inv_i0b = 1.0 / i0(np.array(beta))
    out = np.zeros(new_n, dtype=F32)
    src64 = samples.astype(np.float64)
    blk = 65536
    offs = np.arange(-sinc_half + 1, sinc_half + 1)
    for b0 in range(0, new_n, blk):
        i = np.arange(b0, min(new_n, b0 + blk))
        src_pos = i / ratio
        center = src_pos.astype(np.int64)  # `as i32` truncation; src_pos >= 0
        j = center[:, None] + offs[None, :]
        d = j - src_pos[:, None]
        x = d * cutoff
        with np.errstate(divide="ignore", invalid="ignore"):
            s = np.where(np.abs(x) < 1e-9, 1.0, np.sin(np.pi * x) / (np.pi * x))
        npos = d / sinc_half
        inside = (npos > -1.0) & (npos < 1.0)
        w = np.where(inside, i0(beta * np.sqrt(np.maximum(0.0, 1.0 - npos * npos))) * inv_i0b, 0.0)
        coeff = s * w * cutoff
        valid = (j >= 0) & (j < n)
        vals = np.where(valid, src64[np.clip(j, 0, n - 1)], 0.0)
        # sequential accumulation order j_lo..j_hi as in the reference loop
        acc = np.zeros(len(i))
        wsum = np.zeros(len(i))
        for t in range(offs.size):
            acc = acc + vals[:, t] * coeff[:, t]
            wsum = wsum + coeff[:, t]
        out[i - 0] = np.where(wsum > 1e-9, acc / np.where(wsum > 1e-9, wsum, 1.0), 0.0).astype(F32)
    return out


def _hz_to_mel(f):
    f = F32(f)
    logstep = F32(27.0) / F32(np.log(F32(6.4)))
    if f >= F32(1000.0):
        return F32(F32(15.0) + F32(np.log(F32(f / F32(1000.0)))) * logstep)
    return F32(F32(3.0) * f / F32(200.0))


def _mel_to_hz(m):
    m = F32(m)
    logstep = F32(np.log(F32(6.4))) / F32(27.0)
    if m >= F32(15.0):
        return F32(F32(1000.0) * F32(np.exp(F32(logstep * F32(m - F32(15.0))))))
    return F32(F32(200.0) * m / F32(3.0))


_MEL_CACHE = {}


def mel_filters() -> np.ndarray:
    """Slaney mel filterbank [128, 201], audio.rs:202-262 (f32)."""
    if "f" in _MEL_CACHE:
        return _MEL_CACHE["f"]
    fft_freqs = np.array([F32(i) * (F32(SAMPLE_RATE) / F32(2.0)) / F32(N_FREQ - 1) for i in range(N_FREQ)], dtype=F32)
    mel_min = _hz_to_mel(0.0)
    mel_max = _hz_to_mel(SAMPLE_RATE / 2.0)
    ff = np.array([_mel_to_hz(mel_min + (mel_max - mel_min) * F32(i) / F32(MEL_BINS + 1))
                   for i in range(MEL_BINS + 2)], dtype=F32)
    diff = (ff[1:] - ff[:-1]).astype(F32)
    diff[diff == 0] = F32(1e-6)
    filt = np.zeros((MEL_BINS, N_FREQ), dtype=F32)
    for m in range(MEL_BINS):
        enorm = F32(2.0) / F32(ff[m + 2] - ff[m])
        down = ((fft_freqs - ff[m]) / diff[m]).astype(F32)
        up = ((ff[m + 2] - fft_freqs) / diff[m + 1]).astype(F32)
        filt[m] = (np.maximum(np.minimum(down, up), F32(0.0)) * enorm).astype(F32)
    _MEL_CACHE["f"] = filt
    return filt


def hann_window() -> np.ndarray:
    """Periodic Hann, audio.rs:305-311 (f32)."""
    two_pi = F32(2.0) * F32(np.pi)
    i = np.arange(WINDOW_SIZE, dtype=F32)
    return (F32(0.5) * (F32(1.0) - np.cos((two_pi * i / F32(WINDOW_SIZE)).astype(F32)))).astype(F32)


def dft_tables():
    """cos/sin tables [201, 400], audio.rs:315-326: angle = 2*pi*k*n/400 in f32."""
    if "d" in _MEL_CACHE:
        return _MEL_CACHE["d"]
    two_pi = F32(2.0) * F32(np.pi)
    k = np.arange(N_FREQ, dtype=F32)[:, None]
    n = np.arange(N_FFT, dtype=F32)[None, :]
    ang = ((two_pi * k) * n / F32(N_FFT)).astype(F32)
    _MEL_CACHE["d"] = (np.cos(ang).astype(F32), np.sin(ang).astype(F32))
    return _MEL_CACHE["d"]


def mel_spectrogram(samples: np.ndarray):
    """audio.rs:273-372. Returns mel [128, n_frames] (mel-major) or None."""
    x = np.asarray(samples, dtype=F32)
    n = len(x)
    pad = N_FFT // 2
    padded = np.zeros(n + 2 * pad, dtype=F32)
    for i in range(pad):  # reflect pad with zero fallback, audio.rs:280-291
        src = pad - i
        padded[i] = x[src] if src < n else F32(0.0)
    padded[pad:pad + n] = x
    for i in range(pad):
        src = n - 2 - i
        padded[pad + n + i] = x[src] if src >= 0 else F32(0.0)
    n_frames = (len(padded) - N_FFT) // HOP_LENGTH + 1 - 1
    if n_frames <= 0:
        return None
    win = hann_window()
    idx = np.arange(n_frames)[None, :] * HOP_LENGTH + np.arange(N_FFT)[:, None]
    windowed = (padded[idx] * win[:, None]).astype(F32)  # [400, F]
    cos_t, sin_t = dft_tables()
    re = cos_t @ windowed
    im = sin_t @ windowed
    power = (re * re + im * im).astype(F32)
    mel = (mel_filters() @ power).astype(F32)
    mel = np.log10(np.maximum(mel, F32(1e-10))).astype(F32)
    gmax = mel.max()
    mel = ((np.maximum(mel, F32(gmax - F32(8.0))) + F32(4.0)) / F32(4.0)).astype(F32)
    return mel


def compact_silence(samples: np.ndarray) -> np.ndarray:
    """audio.rs:375-479."""
    x = np.asarray(samples, dtype=F32)
    n = len(x)
    if n == 0:
        return x.copy()
    win = 160
    n_win = (n + win - 1) // win
    rms = np.zeros(n_win, dtype=F32)
    for w in range(n_win):
        seg = x[w * win:min(n, w * win + win)]
        e = np.cumsum((seg * seg).astype(F32), dtype=F32)[-1]
        rms[w] = np.sqrt(F32(e / F32(max(1, len(seg)))))
    smooth = np.zeros(n_win, dtype=F32)
    s = rms[0]
    for w in range(n_win):
        s = F32(F32(F32(1.0) - F32(0.2)) * s + F32(0.2) * rms[w])
        smooth[w] = s
    srt = np.sort(smooth)
    p25 = int(F32(n_win - 1) * F32(0.25))
    thresh = min(max(F32(srt[p25] * F32(1.8)), F32(0.002)), F32(0.025))
    voice = smooth > thresh
    i = 0
    while i < n_win:
        if not voice[i]:
            i += 1
            continue
        j = i + 1
        while j < n_win and voice[j]:
            j += 1
        if j - i < 5:
            voice[i:j] = False
        i = j
    pv = np.zeros(n_win, dtype=bool)
    for w in range(n_win):
        if voice[w]:
            pv[max(0, w - 3):min(n_win - 1, w + 3) + 1] = True
    out = []
    silence = 0
    for w in range(n_win):
        seg = x[w * win:min(n, w * win + win)]
        if pv[w]:
            out.append(seg)
            silence = 0
        else:
            silence += 1
            if silence <= 60:
                out.append(seg)
    if not out:
        return x[:min(n, SAMPLE_RATE // 2)].copy()
    return np.concatenate(out).astype(F32)


# ---------------------------------------------------------------------------
# Kernels (kernels/mod.rs)
# ---------------------------------------------------------------------------

def gelu(x):
    """Tanh GELU, kernels/mod.rs:1283-1288."""
    x = x.astype(F32)
    inner = (F32(0.7978845608028654) * (x + F32(0.044715) * (x * x * x))).astype(F32)
    return (F32(0.5) * x * (F32(1.0) + np.tanh(inner))).astype(F32)


def silu_mul(g, u):
    """g / (1 + exp(-g)) * u, kernels/mod.rs:1335-1337."""
    return (g / (F32(1.0) + np.exp(-g)) * u).astype(F32)


def layer_norm(x, w, b, eps=F32(1e-5)):
    """kernels/mod.rs:1160-1189 (population variance)."""
    h = x.shape[-1]
    mean = (x.sum(axis=-1, keepdims=True, dtype=F32) / F32(h)).astype(F32)
    d = (x - mean).astype(F32)
    var = ((d * d).sum(axis=-1, keepdims=True, dtype=F32) / F32(h)).astype(F32)
    inv = (F32(1.0) / np.sqrt(var + eps)).astype(F32)
    return (d * inv * w + b).astype(F32)


# Noise-floor switch for parity statistics: True accumulates the RMSNorm sums of squares and
# the decoder-prefill products in f64 and rounds the results to f32 - equally valid f32
# implementations of kernels/mod.rs:1191-1212 and of the prefill sgemm calls that differ from
# the default only in the last bits. Comparing the oracle with itself under this switch
# measures how often int8 decode ids flip from rounding order alone.
RMS_SUM_F64 = False


def _mm(a, w):
    """a @ w^T rounded to f32 (f64 accumulation under RMS_SUM_F64)."""
    if RMS_SUM_F64:
        return (a.astype(np.float64) @ w.T.astype(np.float64)).astype(F32)
    return (a @ w.T).astype(F32)


def rms_norm(x, w, eps):
    """kernels/mod.rs:1191-1212."""
    h = x.shape[-1]
    if RMS_SUM_F64:
        ss = (x.astype(np.float64) ** 2).sum(axis=-1, keepdims=True).astype(F32)
    else:
        ss = (x * x).sum(axis=-1, keepdims=True, dtype=F32)
    inv = (F32(1.0) / np.sqrt(ss / F32(h) + eps)).astype(F32)
    return (x * inv * w).astype(F32)


def linear(x, w, b=None):
    """y = x @ W^T (+ b), kernels/mod.rs:550-584 (sgemm then bias add)."""
    y = x @ w.T
    if b is not None:
        y = (y + b).astype(F32)
    return y.astype(F32)


def sinusoidal_pe(n_pos, d):
    """kernels/mod.rs:1704-1716."""
    half = d // 2
    log_ts = F32(np.log(F32(10000.0))) / F32(half - 1)
    inv_ts = np.exp((-(np.arange(half, dtype=F32)) * log_ts).astype(F32)).astype(F32)
    ang = (np.arange(n_pos, dtype=F32)[:, None] * inv_ts[None, :]).astype(F32)
    return np.concatenate([np.sin(ang), np.cos(ang)], axis=1).astype(F32)


def quantize_act(x):
    """quantize_f32_to_int8, kernels/mod.rs:1795-1802: (int8 values, scale)."""
    x = np.asarray(x, dtype=F32)
    max_abs = F32(np.max(np.abs(x))) if x.size else F32(0.0)
    scale = F32(max_abs / F32(127.0)) if max_abs > 0 else F32(1.0)
    inv = F32(F32(127.0) / max(max_abs, F32(1e-10)))
    q = np.clip(round_half_away((x * inv).astype(F32)), -127, 127).astype(np.int8)
    return q, scale


def quantize_weights(w_bits: np.ndarray, mode: str = "trunc"):
    """Per-row symmetric int8 of a bf16 matrix.

    mode="trunc": kernels/neon.rs:637-694 — the quantiser of the only platform on
    which the reference's int8 decode runs (vcvtq truncation toward zero; in_dim is a
    multiple of 8 so the rounding scalar tail never runs).
    mode="round": the generic path kernels/mod.rs:1805-1829 (round half away, clamp).
    """
    w = bf16_to_f32(w_bits)
    max_abs = np.abs(w).max(axis=1).astype(F32)
    scale = np.where(max_abs > 0, (max_abs / F32(127.0)).astype(F32), F32(1.0)).astype(F32)
    inv = (F32(127.0) / np.maximum(max_abs, F32(1e-10))).astype(F32)
    v = (w * inv[:, None]).astype(F32)
    if mode == "trunc":
        q = np.clip(np.trunc(v), -127, 127)
    else:
        q = np.clip(round_half_away(v), -127, 127)
    return q.astype(np.int8), scale


def int8_dot(wq_f32chunks, xq: np.ndarray) -> np.ndarray:
    """Exact int32 sum_k w[o,k]*x[k]: float32 GEMV on K-chunks of <= 1024 (every partial
    sum is an integer < 2^24, hence exact), chunk results summed in int64."""
    xs = xq.astype(F32)
    acc = None
    for (k0, k1, wc) in wq_f32chunks:
        part = (wc @ xs[k0:k1]).astype(np.int64)
        acc = part if acc is None else acc + part
    return acc


def int8_chunks(q: np.ndarray):
    k = q.shape[1]
    return [(k0, min(k, k0 + 1024), np.ascontiguousarray(q[:, k0:min(k, k0 + 1024)], dtype=F32))
            for k0 in range(0, k, 1024)]


def int8_matvec(wc, w_scale, x, bias=None):
    """neon.rs:716-800: y[o] = (sum as f32) * x_scale * w_scale[o] (+ bias[o])."""
    xq, xs = quantize_act(x)
    s = int8_dot(wc, xq).astype(F32)
    y = ((s * xs).astype(F32) * w_scale).astype(F32)
    if bias is not None:
        y = (y + bias).astype(F32)
    return y


def conv2d_s2(inp, w, b):
    """3x3 stride-2 pad-1 conv as im2col + sgemm (kernels/mod.rs:1077-1156).
    inp [B, C, H, W] -> [B, 480, Ho, Wo]."""
    bsz, c, h, wd = inp.shape
    ho = (h + 2 - 3) // 2 + 1
    wo = (wd + 2 - 3) // 2 + 1
    p = np.zeros((bsz, c, h + 2, wd + 2), dtype=F32)
    p[:, :, 1:h + 1, 1:wd + 1] = inp
    cols = np.empty((bsz, c, 3, 3, ho, wo), dtype=F32)
    for ki in range(3):
        for kj in range(3):
            cols[:, :, ki, kj] = p[:, :, ki:ki + 2 * ho:2, kj:kj + 2 * wo:2]
    cols = cols.reshape(bsz, c * 9, ho * wo)
    wm = w.reshape(w.shape[0], -1)
    out = np.matmul(wm[None], cols).astype(F32)
    out = (out + b[None, :, None]).astype(F32)
    return out.reshape(bsz, w.shape[0], ho, wo)


# ---------------------------------------------------------------------------
# Model
# ---------------------------------------------------------------------------

class Model:
    """Weights in the forms the reference keeps them (encoder.rs:123-182,
    decoder.rs:70-167): encoder f32, decoder bf16 (-> f32 for prefill), int8 decode."""

    def __init__(self, model_dir: str, weight_quant: str = "trunc", decode_mode: str = "int8"):
        st = SafeTensors(model_dir)
        self.cfg = c = detect_config(st)
        self.model_dir = model_dir
        self.decode_mode = decode_mode
        p = "thinker.audio_tower."
        self.conv = [(st.f32(f"{p}conv2d{i}.weight"), st.f32(f"{p}conv2d{i}.bias")) for i in (1, 2, 3)]
        self.conv_out = st.f32(p + "conv_out.weight")
        self.enc_layers = []
        for i in range(c.enc_layers):
            lp = f"{p}layers.{i}."
            g = lambda n: st.f32(lp + n)
            self.enc_layers.append(dict(
                wq=g("self_attn.q_proj.weight"), bq=g("self_attn.q_proj.bias"),
                wk=g("self_attn.k_proj.weight"), bk=g("self_attn.k_proj.bias"),
                wv=g("self_attn.v_proj.weight"), bv=g("self_attn.v_proj.bias"),
                wo=g("self_attn.out_proj.weight"), bo=g("self_attn.out_proj.bias"),
                ln1w=g("self_attn_layer_norm.weight"), ln1b=g("self_attn_layer_norm.bias"),
                w1=g("fc1.weight"), b1=g("fc1.bias"), w2=g("fc2.weight"), b2=g("fc2.bias"),
                ln2w=g("final_layer_norm.weight"), ln2b=g("final_layer_norm.bias")))
        self.ln_post = (st.f32(p + "ln_post.weight"), st.f32(p + "ln_post.bias"))
        self.proj1 = (st.f32(p + "proj1.weight"), st.f32(p + "proj1.bias"))
        self.proj2 = (st.f32(p + "proj2.weight"), st.f32(p + "proj2.bias"))
        m = "thinker.model."
        self.embed_bits = st.bf16(m + "embed_tokens.weight")
        self.dec_layers = []
        for i in range(c.dec_layers):
            lp = f"{m}layers.{i}."
            wq, wk, wv, wo = (st.bf16(lp + f"self_attn.{n}.weight") for n in ("q_proj", "k_proj", "v_proj", "o_proj"))
            gate, up, down = (st.bf16(lp + f"mlp.{n}.weight") for n in ("gate_proj", "up_proj", "down_proj"))
            gu = np.empty((2 * gate.shape[0], gate.shape[1]), dtype=np.uint16)  # decoder.rs:91-104
            gu[0::2] = gate
            gu[1::2] = up
            L = dict(wq=bf16_to_f32(wq), wk=bf16_to_f32(wk), wv=bf16_to_f32(wv), wo=bf16_to_f32(wo),
                     gu=bf16_to_f32(gu), down=bf16_to_f32(down),
                     qn=st.f32(lp + "self_attn.q_norm.weight"), kn=st.f32(lp + "self_attn.k_norm.weight"),
                     n1=st.f32(lp + "input_layernorm.weight"), n2=st.f32(lp + "post_attention_layernorm.weight"))
            if decode_mode == "int8":
                for key, bits in (("wq", wq), ("wk", wk), ("wv", wv), ("wo", wo), ("gu", gu), ("down", down)):
                    q, s = quantize_weights(bits, weight_quant)
                    L[key + "_q"] = int8_chunks(q)
                    L[key + "_s"] = s
                    L[key + "_i8"] = q
            self.dec_layers.append(L)
        self.norm = st.f32(m + "norm.weight")
        lm_name = "thinker.lm_head.weight"
        self.lm_bits = st.bf16(lm_name) if st.has(lm_name) else self.embed_bits
        if decode_mode == "int8":
            q, s = quantize_weights(self.lm_bits, weight_quant)
            self.lm_q = int8_chunks(q)
            self.lm_s = s
            self.lm_i8 = q
        else:
            self.lm_f32 = bf16_to_f32(self.lm_bits)
        # RoPE inverse frequencies, decoder.rs:302-309 (f32 powf)
        hd = c.dec_head_dim
        self.inv_freq = np.array([F32(1.0) / np.power(c.theta, F32(F32(2 * d) / F32(hd)), dtype=F32)
                                  for d in range(hd // 2)], dtype=F32)

    def embed(self, tok: int) -> np.ndarray:
        return bf16_to_f32(self.embed_bits[tok])

    # ---------------- encoder (encoder.rs:186-358) ----------------
    def encode(self, mel: np.ndarray) -> np.ndarray:
        c = self.cfg
        frames = mel.shape[1]
        cs = c.enc_chunk_size
        n_chunks = (frames + cs - 1) // cs
        outs = []
        full = frames // cs
        groups = []
        if full:
            groups.append((0, full, cs))
        if full < n_chunks:
            groups.append((full, full + 1, frames - full * cs))
        for c0, c1, w in groups:
            xin = np.stack([mel[:, k * cs:k * cs + w] for k in range(c0, c1)])[:, None].astype(F32)
            h = xin
            for (cw, cb) in self.conv:
                h = gelu(conv2d_s2(h, cw, cb))
            bsz, ch, f, w3 = h.shape
            r = h.transpose(0, 3, 1, 2).reshape(bsz, w3, ch * f)  # col = ch*16 + f
            proj = (r @ self.conv_out.T).astype(F32)
            proj = (proj + sinusoidal_pe(w3, c.enc_d_model)[None]).astype(F32)
            outs.extend(list(proj))
        x = np.concatenate(outs, axis=0).astype(F32)
        total = x.shape[0]
        # window boundaries, encoder.rs:292-298
        w = cs
        w1 = (w + 2 - 3) // 2 + 1
        w2 = (w1 + 2 - 3) // 2 + 1
        tpc = (w2 + 2 - 3) // 2 + 1
        wts = tpc * (c.enc_n_window_infer // cs)
        starts = list(range(0, total, wts)) + [total]
        nh, hd = c.enc_heads, c.enc_head_dim
        scale = F32(1.0) / F32(math.sqrt(hd))
        for L in self.enc_layers:
            xn = layer_norm(x, L["ln1w"], L["ln1b"])
            q = linear(xn, L["wq"], L["bq"])
            k = linear(xn, L["wk"], L["bk"])
            v = linear(xn, L["wv"], L["bv"])
            att = np.zeros_like(q)
            for a, b in zip(starts[:-1], starts[1:]):
                qh = q[a:b].reshape(b - a, nh, hd).transpose(1, 0, 2)
                kh = k[a:b].reshape(b - a, nh, hd).transpose(1, 0, 2)
                vh = v[a:b].reshape(b - a, nh, hd).transpose(1, 0, 2)
                s = (np.matmul(qh, kh.transpose(0, 2, 1)) * scale).astype(F32)
                s = np.exp((s - s.max(axis=-1, keepdims=True)).astype(F32)).astype(F32)
                s = (s / s.sum(axis=-1, keepdims=True, dtype=F32)).astype(F32)
                att[a:b] = np.matmul(s, vh).transpose(1, 0, 2).reshape(b - a, nh * hd)
            # linear_accumulate: x += bias, then x += att @ Wo^T (mod.rs:591-627)
            x = ((x + L["bo"]).astype(F32) + (att @ L["wo"].T)).astype(F32)
            xn = layer_norm(x, L["ln2w"], L["ln2b"])
            mid = gelu(linear(xn, L["w1"], L["b1"]))
            x = ((x + L["b2"]).astype(F32) + (mid @ L["w2"].T)).astype(F32)
        x = layer_norm(x, *self.ln_post)
        x = gelu(linear(x, *self.proj1))
        return linear(x, *self.proj2)


class KvCache:
    """f32 [layer][kv_head][pos][head_dim], decoder.rs:174-271."""

    def __init__(self, cfg, max_seq=2048):
        self.cfg = cfg
        self.max_seq = max_seq
        self.k = np.zeros((cfg.dec_layers, cfg.dec_kv_heads, max_seq, cfg.dec_head_dim), dtype=F32)
        self.v = np.zeros_like(self.k)
        self.len = 0

    def grow(self, required):
        if required <= self.max_seq:
            return
        nm = self.max_seq
        while nm < required:
            nm *= 2
        k = np.zeros(self.k.shape[:2] + (nm, self.k.shape[3]), dtype=F32)
        v = np.zeros_like(k)
        k[:, :, :self.len] = self.k[:, :, :self.len]
        v[:, :, :self.len] = self.v[:, :, :self.len]
        self.k, self.v, self.max_seq = k, v, nm


class Decoder:
    """decoder_prefill / decoder_forward (decoder.rs:455-645) over a Model."""

    def __init__(self, model: Model):
        self.m = model
        self.kv = KvCache(model.cfg)
        self.record_logits = False
        self.last_logits = None

    def _rope(self, pos0, n):
        p = np.arange(pos0, pos0 + n, dtype=F32)[:, None]
        ang = (p * self.m.inv_freq[None, :]).astype(F32)
        return np.cos(ang).astype(F32), np.sin(ang).astype(F32)

    @staticmethod
    def _apply_rope(x, c, s):
        # x [S, H, 128]; c,s [S, 64]; generic path kernels/mod.rs:1780-1788
        half = x.shape[-1] // 2
        x1 = x[..., :half]
        x2 = x[..., half:]
        cc = c[:, None, :]
        ss = s[:, None, :]
        o1 = ((x1 * cc).astype(F32) + ((-x2) * ss).astype(F32)).astype(F32)
        o2 = ((x2 * cc).astype(F32) + (x1 * ss).astype(F32)).astype(F32)
        return np.concatenate([o1, o2], axis=-1)

    def _attend(self, q, L, start, seq):
        """Causal GQA attention of q [S, H, D] at positions start.. over the cache."""
        c = self.m.cfg
        hpk = c.dec_heads // c.dec_kv_heads
        scale = F32(1.0) / F32(math.sqrt(c.dec_head_dim))
        total = start + seq
        out = np.zeros_like(q)
        for h in range(c.dec_heads):
            kh = self.kv.k[L, h // hpk, :total]
            vh = self.kv.v[L, h // hpk, :total]
            s = ((q[:, h] @ kh.T) * scale).astype(F32)  # [S, total]
            mask = np.arange(total)[None, :] > (start + np.arange(seq))[:, None]
            s[mask] = -np.inf
            s = np.exp((s - s.max(axis=1, keepdims=True)).astype(F32)).astype(F32)
            s = (s / s.sum(axis=1, keepdims=True, dtype=F32)).astype(F32)
            out[:, h] = s @ vh
        return out

    def prefill(self, embeds: np.ndarray):
        """decoder_prefill over embeds [S, hidden] starting at kv.len."""
        m, c = self.m, self.m.cfg
        seq = embeds.shape[0]
        start = self.kv.len
        if start + seq > self.kv.max_seq:
            self.kv.grow(start + seq + 1024)
        x = embeds.astype(F32).copy()
        cos, sin = self._rope(start, seq)
        for li, L in enumerate(m.dec_layers):
            xn = rms_norm(x, L["n1"], c.eps)
            q = _mm(xn, L["wq"]).reshape(seq, c.dec_heads, 128)
            k = _mm(xn, L["wk"]).reshape(seq, c.dec_kv_heads, 128)
            v = _mm(xn, L["wv"]).reshape(seq, c.dec_kv_heads, 128)
            q = self._apply_rope(rms_norm(q, L["qn"], c.eps), cos, sin)
            k = self._apply_rope(rms_norm(k, L["kn"], c.eps), cos, sin)
            self.kv.k[li, :, start:start + seq] = k.transpose(1, 0, 2)
            self.kv.v[li, :, start:start + seq] = v.transpose(1, 0, 2)
            att = self._attend(q, li, start, seq).reshape(seq, -1)
            x = (x + _mm(att, L["wo"])).astype(F32)
            xn = rms_norm(x, L["n2"], c.eps)
            gu = _mm(xn, L["gu"])
            mid = silu_mul(gu[:, 0::2], gu[:, 1::2])
            x = (x + _mm(mid, L["down"])).astype(F32)
        self.kv.len = start + seq
        return x

    def forward(self, embed: np.ndarray) -> int:
        """decoder_forward: one token at kv.len; returns the greedy token id."""
        m, c = self.m, self.m.cfg
        pos = self.kv.len
        if pos >= self.kv.max_seq:
            self.kv.grow(pos + 1024)
        x = embed.astype(F32).copy()
        cos, sin = self._rope(pos, 1)
        int8 = m.decode_mode == "int8"
        for li, L in enumerate(m.dec_layers):
            xn = rms_norm(x, L["n1"], c.eps)
            if int8:
                xq, xs = quantize_act(xn)  # one quantisation shared by q/k/v (mod.rs:884-967)
                def mv(key):
                    s = int8_dot(L[key + "_q"], xq).astype(F32)
                    return ((s * xs).astype(F32) * L[key + "_s"]).astype(F32)
                q, k, v = mv("wq"), mv("wk"), mv("wv")
            else:
                q, k, v = (L["wq"] @ xn).astype(F32), (L["wk"] @ xn).astype(F32), (L["wv"] @ xn).astype(F32)
            q = self._apply_rope(rms_norm(q.reshape(1, c.dec_heads, 128), L["qn"], c.eps), cos, sin)
            k = self._apply_rope(rms_norm(k.reshape(1, c.dec_kv_heads, 128), L["kn"], c.eps), cos, sin)
            self.kv.k[li, :, pos] = k[0]
            self.kv.v[li, :, pos] = v.reshape(c.dec_kv_heads, 128)
            att = self._attend(q, li, pos, 1).reshape(-1)
            if int8:
                x = int8_matvec(L["wo_q"], L["wo_s"], att, bias=x)
            else:
                x = ((L["wo"] @ att).astype(F32) + x).astype(F32)
            xn = rms_norm(x, L["n2"], c.eps)
            if int8:
                gu = int8_matvec(L["gu_q"], L["gu_s"], xn)
            else:
                gu = (L["gu"] @ xn).astype(F32)
            mid = silu_mul(gu[0::2], gu[1::2])
            if int8:
                x = int8_matvec(L["down_q"], L["down_s"], mid, bias=x)
            else:
                x = ((L["down"] @ mid).astype(F32) + x).astype(F32)
        self.kv.len = pos + 1
        xn = rms_norm(x, m.norm, c.eps)
        if int8:
            xq, xs = quantize_act(xn)  # argmax_matvec_int8, mod.rs:1832-1893
            logits = ((int8_dot(m.lm_q, xq).astype(F32) * xs).astype(F32) * m.lm_s).astype(F32)
        else:
            logits = (m.lm_f32 @ xn).astype(F32)
        if self.record_logits:
            self.last_logits = logits
        return int(np.argmax(logits))  # first maximum wins, as the strict `>` scans do


# ---------------------------------------------------------------------------
# Tokenizer (tokenizer.rs)
# ---------------------------------------------------------------------------

class Tokenizer:
    def __init__(self, model_dir: str):
        b2u = [0] * 256
        n = 0
        for b in range(256):
            if 33 <= b <= 126 or 161 <= b <= 172 or 174 <= b <= 255:
                b2u[b] = b
            else:
                b2u[b] = 256 + n
                n += 1
        self.b2u = b2u
        u2b = {cp: b for b, cp in enumerate(b2u)}
        with open(os.path.join(model_dir, "vocab.json"), encoding="utf-8") as f:
            vocab = json.load(f)
        self.vocab = vocab
        self.vocab_size = max(vocab.values()) + 1
        self.id_bytes = [b""] * self.vocab_size
        for key, i in vocab.items():
            self.id_bytes[i] = bytes(u2b.get(ord(ch), ord("?")) if ord(ch) < 512 and ord(ch) in u2b else ord("?")
                                     for ch in key)
        self.merges = {}
        mp = os.path.join(model_dir, "merges.txt")
        if os.path.exists(mp):
            rank = 0
            with open(mp, encoding="utf-8") as f:
                for line in f.read().splitlines():
                    line = line.rstrip()
                    if not line or line.startswith("#"):
                        continue
                    sp = line.find(" ")
                    if sp >= 0:
                        a, b = line[:sp], line[sp + 1:].lstrip()
                        if a and b:
                            self.merges[a + " " + b] = rank
                            rank += 1

    def decode_bytes(self, tok: int) -> bytes:
        if tok < 0 or tok >= self.vocab_size:
            return b""
        return self.id_bytes[tok]

    def encode(self, text: str):
        """Whole-string byte-level BPE without a pre-tokenizer (tokenizer.rs:227-279)."""
        if not text:
            return None
        syms = [chr(self.b2u[b]) for b in text.encode("utf-8")]
        while len(syms) > 1:
            best, bi = None, -1
            for i in range(len(syms) - 1):
                r = self.merges.get(syms[i] + " " + syms[i + 1])
                if r is not None and (best is None or r < best):
                    best, bi = r, i
            if bi < 0:
                break
            syms[bi:bi + 2] = [syms[bi] + syms[bi + 1]]
        ids = []
        for s in syms:
            if s not in self.vocab:
                return None
            ids.append(self.vocab[s])
        return ids


# ---------------------------------------------------------------------------
# Orchestration (context.rs, transcribe.rs)
# ---------------------------------------------------------------------------

def find_split_point(samples, target, search_sec):
    """transcribe.rs:253-278 (sequential f32 energy sums)."""
    half = int(F32(search_sec) * F32(SAMPLE_RATE))
    lo = max(0, target - half)
    hi = min(target + half, len(samples))
    win = 1600
    best_e = F32(1e30)
    best_c = target
    pos = lo
    while pos + win <= hi:
        end = min(pos + win, len(samples))
        seg = samples[pos:end]
        e = np.cumsum((seg * seg).astype(F32), dtype=F32)[-1]
        e = F32(e / F32(end - pos))
        if e < best_e:
            best_e = e
            best_c = pos + (end - pos) // 2
        pos += win // 2
    return best_c


def split_points(samples, segment_sec, search_sec=3.0):
    """Segment start offsets used by transcribe_audio (transcribe.rs:328-346); a single
    [0] when no splitting applies."""
    seg = F32(segment_sec)
    target = int(seg * F32(SAMPLE_RATE)) if seg > 0 else 0
    search = min(F32(search_sec), F32(seg / F32(2.0)))
    margin = int(F32(search) * F32(SAMPLE_RATE)) if search > 0 else 0
    if seg <= 0 or len(samples) <= target + margin:
        return [0]
    splits = [0]
    pos = 0
    while pos + target + margin < len(samples):
        sp = find_split_point(samples, pos + target, search)
        splits.append(sp)
        pos = sp
        if len(splits) >= 127:
            break
    return splits


def _is_rust_ws_byte(b):
    return b in (0x09, 0x0A, 0x0B, 0x0C, 0x0D, 0x20, 0x85, 0xA0)


def should_insert_boundary_space(prev, nxt):
    """transcribe.rs:280-286 (bytes viewed as chars)."""
    if prev == 0 or nxt == 0:
        return False
    if _is_rust_ws_byte(prev) or _is_rust_ws_byte(nxt):
        return False
    if 33 <= nxt <= 126 and not chr(nxt).isalnum():
        return False
    return True


class Ctx:
    """QwenCtx + transcribe.rs over the oracle model (context.rs:26-162)."""

    def __init__(self, model_dir, weight_quant="trunc", decode_mode="int8"):
        self.model = Model(model_dir, weight_quant, decode_mode)
        self.dec = Decoder(self.model)
        self.segment_sec = 0.0
        self.search_sec = 3.0
        self.stream_chunk_sec = 2.0
        self.stream_rollback = 5
        self.stream_unfixed_chunks = 2
        self.stream_max_new_tokens = 32
        self.past_text_conditioning = False
        self.skip_silence = False
        self.prompt = None
        self.force_language = None
        self.force_n_tokens = 0  # benchmark extension: decode exactly N tokens, EOS ignored
        self.tok = Tokenizer(model_dir)
        self.last_tokens = []  # generated ids of the last segment (for parity tests)
        self.segments_tokens = []

    def set_force_language(self, lang):
        if not lang:
            self.force_language = None
            return 0
        n = normalize_language(lang)
        if n is None:
            return -1
        self.force_language = n
        return 0

    def prompt_tokens(self):
        pt = self.tok.encode(self.prompt) if self.prompt else None
        ft = None
        if self.force_language:
            ft = self.tok.encode("language " + self.force_language)
            if ft is not None:
                ft = ft + [TOKEN_ASR_TEXT]
        return pt, ft

    def build_embeds(self, enc, prompt_toks, force_toks, tail_toks, tail_asr_text):
        m = self.model
        rows = [m.embed(t) for t in PREFIX_HEAD]
        rows += [m.embed(t) for t in (prompt_toks or [])]
        rows += [m.embed(t) for t in PREFIX_TAIL]
        parts = [np.stack(rows), enc.astype(F32)]
        rows = [m.embed(t) for t in SUFFIX_BASE] + [m.embed(t) for t in (force_toks or [])]
        rows += [m.embed(t) for t in (tail_toks or [])]
        if tail_asr_text:
            rows.append(m.embed(TOKEN_ASR_TEXT))
        parts.append(np.stack(rows))
        return np.concatenate(parts).astype(F32)

    def transcribe_segment(self, samples, past_tokens=None):
        """transcribe.rs:63-247; returns (text, n_text_tokens)."""
        mel = mel_spectrogram(samples)
        if mel is None:
            return None
        enc = self.model.encode(mel)
        pt, ft = self.prompt_tokens()
        emb = self.build_embeds(enc, pt, ft, past_tokens, bool(past_tokens))
        self.dec.kv.len = 0
        n = emb.shape[0] - 1
        self.dec.prefill(emb[:n])
        token = self.dec.forward(emb[n])
        past_asr = bool(ft) or bool(past_tokens)
        text = bytearray()
        n_text = 0
        n_gen = 0
        gen = [token]
        limit = self.force_n_tokens if self.force_n_tokens > 0 else 2048
        while n_gen < limit:
            n_gen += 1
            if self.force_n_tokens <= 0 and token in (TOKEN_ENDOFTEXT, TOKEN_IM_END):
                break
            if token == TOKEN_ASR_TEXT:
                past_asr = True
            elif past_asr:
                text += self.tok.decode_bytes(token)
                n_text += 1
            if self.force_n_tokens > 0 and n_gen >= limit:
                break
            token = self.dec.forward(self.model.embed(token))
            gen.append(token)
        self.last_tokens = gen
        return rust_trim(lossy(bytes(text))), n_text

    def transcribe_audio(self, samples):
        """transcribe.rs:297-426 (offline / segmented)."""
        x = np.asarray(samples, dtype=F32)
        if self.skip_silence:
            x = compact_silence(x)
        splits = split_points(x, self.segment_sec, self.search_sec)
        self.segments_tokens = []
        if len(splits) == 1:
            r = self.transcribe_segment(x)
            self.segments_tokens.append(self.last_tokens)
            return None if r is None else r[0]
        result = ""
        min_samples = SAMPLE_RATE // 2
        for s in range(len(splits)):
            a = splits[s]
            b = splits[s + 1] if s + 1 < len(splits) else len(x)
            seg = x[a:b]
            if len(seg) < min_samples:
                seg = np.concatenate([seg, np.zeros(min_samples - len(seg), dtype=F32)])
            past = self.tok.encode(result) if (self.past_text_conditioning and result) else None
            r = self.transcribe_segment(seg, past)
            self.segments_tokens.append(self.last_tokens)
            if r is None or not r[0]:
                continue
            t = r[0]
            if result:
                if should_insert_boundary_space(result.encode()[-1], t.encode()[0]):
                    result += " "
            result += t
        return result


def teacher_forced(model: Model, rows: np.ndarray, forced, n_steps: int):
    """decoder_prefill(rows[:-1]) then n_steps decoder_forward steps: step 0 consumes
    rows[-1], step i>0 consumes embed(forced[i-1]). Returns (argmax ids, logits [n, V])."""
    dec = Decoder(model)
    dec.record_logits = True
    dec.prefill(rows[:-1])
    ids, lg = [], []
    x = rows[-1]
    for i in range(n_steps):
        ids.append(dec.forward(x))
        lg.append(dec.last_logits)
        if i + 1 < n_steps:
            x = model.embed(int(forced[i]))
    return np.array(ids, dtype=np.int32), np.stack(lg)


def prompt_rows(ctx: "Ctx", enc: np.ndarray) -> np.ndarray:
    """Prompt embeddings of transcribe_segment (transcribe.rs:96-169) for the ctx settings."""
    pt, ft = ctx.prompt_tokens()
    return ctx.build_embeds(enc, pt, ft, None, False)


# ---------------------------------------------------------------------------
# Incremental streaming (transcribe.rs:801-1304)
# ---------------------------------------------------------------------------

def stream_tail_repeat_blocks(tokens, max_period):
    """transcribe.rs:36-55."""
    n = len(tokens)
    if n < 2:
        return 1, 0
    cap = min(n // 2, max_period if max_period > 0 else n // 2)
    best_reps, best_p = 1, 0
    for p in range(1, cap + 1):
        reps = 1
        while (reps + 1) * p <= n:
            if tokens[n - (reps + 1) * p:n - reps * p] != tokens[n - reps * p:n - (reps - 1) * p]:
                break
            reps += 1
        if reps > best_reps:
            best_reps, best_p = reps, p
    return best_reps, best_p


class StreamState:
    """transcribe.rs:801-893 (the oracle keeps one decoder per stream)."""

    def __init__(self):
        self.enc_cache = []          # list of encoder outputs per completed window
        self.enc_cache_base_windows = 0
        self.raw_tokens = []
        self.stable_text_tokens = []
        self.result_bytes = b""
        self.prev_prefill = None     # f32 rows of the previous prefill
        self.prev_tail_snapshot = []
        self.stale_count = 0
        self.last_partial_cursor = 0
        self.last_partial_enc = None
        self.audio_cursor = 0
        self.chunk_idx = 0
        self.dec = None


def stream_push_audio(ctx: "Ctx", samples, st: StreamState, finalize: bool) -> bytes:
    """transcribe.rs:902-1304: processes every full chunk of `samples` (the whole buffer so
    far) from st.audio_cursor, plus the tail when finalising; returns the emitted bytes."""
    m = ctx.model
    if st.dec is None:
        st.dec = Decoder(m)
    dec = st.dec
    chunk_samples = int(F32(ctx.stream_chunk_sec) * F32(SAMPLE_RATE))
    rollback, unfixed = ctx.stream_rollback, ctx.stream_unfixed_chunks
    max_new = ctx.stream_max_new_tokens if ctx.stream_max_new_tokens > 0 else 32
    pt, ft = ctx.prompt_tokens()
    n_force = len(ft) if ft else 0
    x = np.asarray(samples, dtype=F32)
    available = max(0, len(x) - st.audio_cursor)
    if (available < chunk_samples and not finalize) or available == 0:
        return b""
    win = min(max(m.cfg.enc_n_window_infer, 100), 800) * HOP_LENGTH
    delta = b""

    def text_start(rt):
        if n_force:
            return 0
        return rt.index(TOKEN_ASR_TEXT) + 1 if TOKEN_ASR_TEXT in rt else 0

    def emit(cand, a, b):
        nonlocal delta
        for i in range(a, b):
            if i < len(cand):
                if i >= len(st.stable_text_tokens):
                    st.stable_text_tokens.append(cand[i])
                pb = ctx.tok.decode_bytes(cand[i])
                st.result_bytes += pb
                delta += pb

    def reset_context():
        carry = min(len(st.stable_text_tokens), STREAM_RESET_CARRY_TOKENS)
        st.raw_tokens = ([TOKEN_ASR_TEXT] + st.stable_text_tokens[len(st.stable_text_tokens) - carry:]) if carry else []
        st.prev_prefill = None
        st.stale_count = 0
        st.prev_tail_snapshot = []
        if len(st.enc_cache) >= STREAM_MAX_ENC_WINDOWS:
            st.enc_cache_base_windows += len(st.enc_cache)
            st.enc_cache = []

    while st.audio_cursor < len(x):
        if len(x) - st.audio_cursor < chunk_samples and not finalize:
            break
        st.audio_cursor = min(st.audio_cursor + chunk_samples, len(x))
        is_final = finalize and st.audio_cursor >= len(x)
        full_end = (st.audio_cursor // win) * win
        while (st.enc_cache_base_windows + len(st.enc_cache)) * win < full_end:
            ws = (st.enc_cache_base_windows + len(st.enc_cache)) * win
            st.enc_cache.append(m.encode(mel_spectrogram(x[ws:ws + win])))
        need = st.last_partial_cursor == 0 or (st.audio_cursor - st.last_partial_cursor) >= 2 * chunk_samples or is_final
        partial = None
        if full_end < st.audio_cursor:
            if need:
                mel = mel_spectrogram(x[full_end:st.audio_cursor])
                if mel is not None:
                    st.last_partial_enc = m.encode(mel)
                    st.last_partial_cursor = st.audio_cursor
            partial = st.last_partial_enc
        parts = list(st.enc_cache) + ([partial] if partial is not None and len(partial) else [])
        if not parts:
            st.chunk_idx += 1
            return b""  # the reference returns an empty delta here (transcribe.rs:1004-1007)
        enc = np.concatenate(parts).astype(F32)
        n_prefix = max(len(st.raw_tokens) - rollback, 0) if (ctx.past_text_conditioning and st.chunk_idx >= unfixed
                                                              and st.raw_tokens) else 0
        emb = ctx.build_embeds(enc, pt, ft, st.raw_tokens[:n_prefix], False)
        prefill_len = emb.shape[0] - 1
        reused = 0
        if st.prev_prefill is not None and len(st.prev_prefill):
            cmp = min(prefill_len, len(st.prev_prefill))
            while reused < cmp and np.array_equal(st.prev_prefill[reused], emb[reused]):
                reused += 1
        dec.kv.len = reused
        if prefill_len - reused > 0:
            dec.prefill(emb[reused:prefill_len])
        token = dec.forward(emb[prefill_len])
        st.prev_prefill = emb[:prefill_len].copy()
        chunk_tokens = []
        n_gen = 0
        while n_gen < max_new:
            n_gen += 1
            if token in (TOKEN_ENDOFTEXT, TOKEN_IM_END):
                break
            chunk_tokens.append(token)
            token = dec.forward(m.embed(token))
        speech_ended = not chunk_tokens and bool(st.raw_tokens) and st.chunk_idx >= unfixed
        if speech_ended:
            cand = st.raw_tokens[text_start(st.raw_tokens):]
            emit(cand, len(st.stable_text_tokens), len(cand))
        st.raw_tokens = st.raw_tokens[:n_prefix] + chunk_tokens
        if not speech_ended:
            if st.raw_tokens == st.prev_tail_snapshot:
                st.stale_count += 1
            else:
                st.stale_count = 0
                st.prev_tail_snapshot = list(st.raw_tokens)
            reps, _ = stream_tail_repeat_blocks(st.raw_tokens, STREAM_DEGEN_MAX_PERIOD)
            if st.stale_count >= STREAM_STALE_CHUNKS or reps >= STREAM_DEGEN_MIN_REPEATS:
                reset_context()
            if st.chunk_idx > 0 and st.chunk_idx % STREAM_RESET_INTERVAL_CHUNKS == 0:
                reset_context()
            ts = text_start(st.raw_tokens)
            n_text = max(len(st.raw_tokens) - ts, 0)
            if is_final:
                cand_len = n_text
            elif st.chunk_idx >= unfixed:
                cand_len = max(n_text - rollback, 0)
            else:
                cand_len = 0
            cand = st.raw_tokens[ts:]
            a = len(st.stable_text_tokens)
            emit(cand, a, max(cand_len, a))
        st.chunk_idx += 1
        if speech_ended:
            break
    return delta


# ---------------------------------------------------------------------------- forced aligner
TOKEN_TIMESTAMP = 151705  # config.rs:20
_CJK = ("Chinese", "Japanese", "Korean", "Cantonese")


def align_split_words(text: str, language: str):
    """align.rs:44-61: CJK languages -> every non-white-space character, otherwise
    white-space separated words (Rust char::is_whitespace)."""
    if language in _CJK:
        return [ch for ch in text if ord(ch) not in _RUST_WS]
    words, cur = [], ""
    for ch in text:
        if ord(ch) in _RUST_WS:
            if cur:
                words.append(cur)
            cur = ""
        else:
            cur += ch
    if cur:
        words.append(cur)
    return words


def longest_increasing_subsequence(vals):
    """align.rs:97-137 (non-decreasing; the first longest end; traced back)."""
    n = len(vals)
    if n == 0:
        return []
    dp, prev = [1] * n, [None] * n
    for i in range(1, n):
        for j in range(i):
            if vals[j] <= vals[i] and dp[j] + 1 > dp[i]:
                dp[i] = dp[j] + 1
                prev[i] = j
    best_len, best_end = 0, 0
    for i in range(n):
        if dp[i] > best_len:
            best_len, best_end = dp[i], i
    out, idx = [], best_end
    while True:
        out.append(idx)
        if prev[idx] is None:
            break
        idx = prev[idx]
    return out[::-1]


def fix_timestamps(ts):
    """align.rs:140-189 in f32: blocks off the LIS of <= 2 take the nearest normal value,
    longer blocks are interpolated linearly."""
    ts = [F32(t) for t in ts]
    n = len(ts)
    if n <= 1:
        return ts
    lis = longest_increasing_subsequence(ts)
    if len(lis) == n:
        return ts
    normal = [False] * n
    for i in lis:
        normal[i] = True
    i = 0
    while i < n:
        if normal[i]:
            i += 1
            continue
        bs = i
        while i < n and not normal[i]:
            i += 1
        be, bl = i, i - bs
        left = ts[bs - 1] if bs > 0 else F32(0.0)
        right = ts[be] if be < n else F32(left + F32(F32(bl) * F32(80.0)))
        if bl <= 2:
            fill = left if bs > 0 else right
            for k in range(bs, be):
                ts[k] = fill
        else:
            for j in range(bl):
                t = F32(F32(j + 1) / F32(bl + 1))
                ts[bs + j] = F32(left + F32(t * F32(right - left)))
    return ts


def forced_align(ctx, samples: np.ndarray, text: str, language: str):
    """align.rs:207-351: [(word, start_ms, end_ms)], or None. Also returns the raw argmax
    classes of the <timestamp> rows (for parity tests)."""
    m, c = ctx.model, ctx.model.cfg
    words = align_split_words(text, language)
    if not words:
        return None
    text_tokens = []
    for i, w in enumerate(words):  # encode_timestamp, align.rs:66-93
        wt = ctx.tok.encode(w)
        if wt is None:
            return None
        text_tokens += list(wt) + [TOKEN_TIMESTAMP, TOKEN_TIMESTAMP]
        if i == 0 and not wt:
            return None
    mel = mel_spectrogram(samples)
    if mel is None:
        return None
    enc = m.encode(mel)
    ids = PREFIX_HEAD + PREFIX_TAIL
    rows = [m.embed(t) for t in ids] + [enc[i] for i in range(enc.shape[0])]
    rows += [m.embed(t) for t in SUFFIX_BASE]
    text_off = len(rows)
    rows += [m.embed(t) for t in text_tokens]
    ctx.dec.kv.len = 0
    x = ctx.dec.prefill(np.stack(rows).astype(F32))
    ts_rows = [text_off + i for i, t in enumerate(text_tokens) if t == TOKEN_TIMESTAMP]
    xn = rms_norm(x[ts_rows], m.norm, c.eps)
    logits = (xn @ bf16_to_f32(m.lm_bits).T).astype(F32)
    cls = [int(np.argmax(r)) for r in logits]  # first maximum, as the strictly-greater scan
    ts = fix_timestamps([F32(k) * F32(80.0) for k in cls])
    out = []
    for i, w in enumerate(words):
        s = ts[2 * i] if 2 * i < len(ts) else F32(0.0)
        e = ts[2 * i + 1] if 2 * i + 1 < len(ts) else s
        out.append((w, float(s), float(e)))
    return out, cls

