"""ctypes front of oracle/decode_ref.c, the C restatement of the reference's decode step
(decoder.rs:550-645). Test infrastructure only: the timed CPU baseline of bench.py and a
checker in tests/, never imported by the product path.

`decode(model, dec, x0, n_steps, forced)` continues an oracle `Decoder` whose KV cache holds
the prefill (qwen_oracle.Decoder.prefill) with n_steps decoder_forward steps in C, using
every host core through OpenMP (the reference's thread pool, kernels/mod.rs:839-881)."""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
SRC = os.path.join(HERE, "decode_ref.c")
LIB = os.path.join(HERE, "_build", "libqasr_ref_decode.so")
# x86-64-v3 (AVX2/FMA) so the library built here also runs on the GPU boxes' host CPUs
CFLAGS = ["-O3", "-march=x86-64-v3", "-fopenmp", "-ffp-contract=off", "-shared", "-fPIC", "-std=c11"]

_lib = None


def build(force: bool = False) -> str:
    os.makedirs(os.path.dirname(LIB), exist_ok=True)
    if force or not os.path.exists(LIB) or os.path.getmtime(LIB) < os.path.getmtime(SRC):
        r = subprocess.run(["gcc"] + CFLAGS + [SRC, "-o", LIB, "-lm"], capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError("decode_ref.c build failed:\n" + r.stderr)
    return LIB


PP = C.POINTER(C.c_void_p)


class RefModel(C.Structure):
    _fields_ = [("hidden", C.c_int), ("q_heads", C.c_int), ("kv_heads", C.c_int), ("inter", C.c_int),
                ("layers", C.c_int), ("vocab", C.c_int), ("max_seq", C.c_int), ("int8", C.c_int),
                ("eps", C.c_float)] + \
               [(n, PP) for n in ("q_qkv", "s_qkv", "q_o", "s_o", "q_gu", "s_gu", "q_down", "s_down",
                                  "b_qkv", "b_o", "b_gu", "b_down", "n1", "n2", "qn", "kn")] + \
               [(n, C.c_void_p) for n in ("final_norm", "lm_q", "lm_s", "lm_b", "embed", "inv_freq",
                                          "k_cache", "v_cache")]


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB):
            build()
        L = C.CDLL(LIB)
        L.qasr_ref_decode.restype = C.c_int
        L.qasr_ref_decode.argtypes = [C.POINTER(RefModel), C.c_void_p, C.c_int, C.c_int, C.c_void_p, C.c_void_p,
                                      C.c_void_p]
        L.qasr_ref_set_threads.restype = None
        L.qasr_ref_set_threads.argtypes = [C.c_int]
        _lib = L
    return _lib


def _bits(f32: np.ndarray) -> np.ndarray:
    """bf16 bits of an f32 array holding bf16 values (exact)."""
    return np.ascontiguousarray((np.ascontiguousarray(f32, dtype=np.float32).view(np.uint32) >> 16)
                                .astype(np.uint16))


class Prepared:
    """A Model's decoder weights laid out for the C step (kept alive with the struct)."""

    def __init__(self, model):
        c = model.cfg
        self.keep = []
        self.int8 = model.decode_mode == "int8"

        def arr(a, dt):
            a = np.ascontiguousarray(a, dtype=dt)
            self.keep.append(a)
            return a.ctypes.data

        def ptrs(vals):
            p = (C.c_void_p * len(vals))(*vals)
            self.keep.append(p)
            return C.cast(p, PP)

        Ls = model.dec_layers
        m = RefModel()
        m.hidden, m.q_heads, m.kv_heads = c.dec_hidden, c.dec_heads, c.dec_kv_heads
        m.inter, m.layers, m.vocab, m.int8 = c.dec_intermediate, c.dec_layers, c.vocab_size, int(self.int8)
        m.eps = float(c.eps)
        if self.int8:
            m.q_qkv = ptrs([arr(np.concatenate([L["wq_i8"], L["wk_i8"], L["wv_i8"]]), np.int8) for L in Ls])
            m.s_qkv = ptrs([arr(np.concatenate([L["wq_s"], L["wk_s"], L["wv_s"]]), np.float32) for L in Ls])
            for key, qn, sn in (("wo", "q_o", "s_o"), ("gu", "q_gu", "s_gu"), ("down", "q_down", "s_down")):
                setattr(m, qn, ptrs([arr(L[key + "_i8"], np.int8) for L in Ls]))
                setattr(m, sn, ptrs([arr(L[key + "_s"], np.float32) for L in Ls]))
            m.lm_q = arr(model.lm_i8, np.int8)
            m.lm_s = arr(model.lm_s, np.float32)
        else:
            m.b_qkv = ptrs([arr(_bits(np.concatenate([L["wq"], L["wk"], L["wv"]])), np.uint16) for L in Ls])
            m.b_o = ptrs([arr(_bits(L["wo"]), np.uint16) for L in Ls])
            m.b_gu = ptrs([arr(_bits(L["gu"]), np.uint16) for L in Ls])
            m.b_down = ptrs([arr(_bits(L["down"]), np.uint16) for L in Ls])
            m.lm_b = arr(model.lm_bits, np.uint16)
        for name, key in (("n1", "n1"), ("n2", "n2"), ("qn", "qn"), ("kn", "kn")):
            setattr(m, name, ptrs([arr(L[key], np.float32) for L in Ls]))
        m.final_norm = arr(model.norm, np.float32)
        m.embed = arr(model.embed_bits, np.uint16)
        m.inv_freq = arr(model.inv_freq, np.float32)
        self.m = m


def decode(prep: Prepared, dec, x0: np.ndarray, n_steps: int, forced=None, want_logits: bool = False):
    """n_steps decode steps after `dec`'s prefill; returns (ids, last-step logits or None)."""
    kv = dec.kv
    need = kv.len + n_steps
    if need > kv.max_seq:
        kv.grow(need + 1024)
    k = kv.k if kv.k.flags.c_contiguous else np.ascontiguousarray(kv.k)
    v = kv.v if kv.v.flags.c_contiguous else np.ascontiguousarray(kv.v)
    kv.k, kv.v = k, v
    m = prep.m
    m.max_seq = kv.max_seq
    m.k_cache, m.v_cache = k.ctypes.data, v.ctypes.data
    x = np.ascontiguousarray(x0, dtype=np.float32)
    ids = np.zeros(max(n_steps, 1), dtype=np.int32)
    f = None if forced is None else np.ascontiguousarray(forced, dtype=np.int32)
    lg = np.zeros(m.vocab, dtype=np.float32) if want_logits else None
    rc = lib().qasr_ref_decode(C.byref(m), x.ctypes.data, kv.len, n_steps,
                               None if f is None else f.ctypes.data, ids.ctypes.data,
                               None if lg is None else lg.ctypes.data)
    if rc != 0:
        raise RuntimeError("qasr_ref_decode failed")
    kv.len += n_steps
    return ids[:n_steps], lg


def set_threads(n: int) -> None:
    lib().qasr_ref_set_threads(int(n))
