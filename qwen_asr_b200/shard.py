"""Segmented long-audio transcription sharded over GPUs (one process per GPU).

The reference transcribes the segments of `-S` mode one after another on one context
(crates/qwen-asr/src/transcribe.rs:328-423). With past-text conditioning off (the default,
context.rs:150) the segments are independent, so here every rank transcribes its share of
them with its own engine and rank 0 joins the texts in segment order with the reference's
boundary-space rule (transcribe.rs:280-286, 401-422). Split points come from the library
(the same find_split_point search as the reference, bit-exact). Nothing crosses GPUs but
the finished strings, gathered through torch.distributed (NCCL or gloo).
"""
from __future__ import annotations

import ctypes as C

import numpy as np

SAMPLE_RATE = 16000
MIN_SAMPLES = SAMPLE_RATE // 2  # segments shorter than 0.5 s are zero-padded (transcribe.rs:374-384)


def split_points(samples: np.ndarray, segment_sec: float, search_sec: float = 3.0) -> list[int]:
    """Segment start offsets exactly as transcribe_audio computes them (via the library)."""
    from . import lib
    x = np.ascontiguousarray(samples, dtype=np.float32)
    out = (C.c_int64 * 256)()
    n = lib().qwen_asr_debug_split_points(x.ctypes.data_as(C.POINTER(C.c_float)), len(x), segment_sec, search_sec,
                                          out, 256)
    return list(out[:n])


def segments(samples: np.ndarray, segment_sec: float, search_sec: float = 3.0) -> list[tuple[int, int]]:
    sp = split_points(samples, segment_sec, search_sec)
    return [(a, sp[i + 1] if i + 1 < len(sp) else len(samples)) for i, a in enumerate(sp)]


def assign(segs: list[tuple[int, int]], world: int) -> list[list[int]]:
    """Longest-processing-time-first assignment of segment indices to ranks."""
    load = [0] * world
    out: list[list[int]] = [[] for _ in range(world)]
    for i in sorted(range(len(segs)), key=lambda i: (-(segs[i][1] - segs[i][0]), i)):
        r = min(range(world), key=lambda r: (load[r], r))
        out[r].append(i)
        load[r] += segs[i][1] - segs[i][0]
    for lst in out:
        lst.sort()
    return out


_RUST_WS = {0x09, 0x0A, 0x0B, 0x0C, 0x0D, 0x20, 0x85, 0xA0}


def _boundary_space(prev: int, nxt: int) -> bool:
    if prev == 0 or nxt == 0 or prev in _RUST_WS or nxt in _RUST_WS:
        return False
    if 33 <= nxt <= 126 and not chr(nxt).isalnum():
        return False
    return True


def join_texts(texts: list[str | None]) -> str:
    """Joins per-segment texts in order, skipping empty ones (transcribe.rs:401-422)."""
    result = ""
    for t in texts:
        if not t:
            continue
        if result and _boundary_space(result.encode()[-1], t.encode()[0]):
            result += " "
        result += t
    return result


def padded(samples: np.ndarray, a: int, b: int) -> np.ndarray:
    seg = np.asarray(samples[a:b], dtype=np.float32)
    if len(seg) < MIN_SAMPLES:
        seg = np.concatenate([seg, np.zeros(MIN_SAMPLES - len(seg), np.float32)])
    return seg


def transcribe_sharded(transcribe_one, samples: np.ndarray, segment_sec: float, rank: int, world: int,
                       search_sec: float = 3.0, segs=None, transcribe_many=None):
    """Every rank transcribes its segments with `transcribe_one(segment_samples) -> str`, or
    all of them at once with `transcribe_many(samples, [(a, b), ...]) -> [str]` (the engine's
    batched-decode entry point); returns the joined text on rank 0 (None elsewhere).
    Collective: all ranks must call."""
    if segs is None:
        segs = segments(samples, segment_sec, search_sec)
    mine = assign(segs, world)[rank]
    if transcribe_many is not None:
        local = list(zip(mine, transcribe_many(samples, [segs[i] for i in mine]) if mine else []))
    else:
        local = [(i, transcribe_one(padded(samples, *segs[i]))) for i in mine]
    if world == 1:
        gathered = [local]
    else:
        import torch.distributed as dist
        gathered = [None] * world if rank == 0 else None
        dist.gather_object(local, gathered, dst=0)
    if rank != 0:
        return None
    texts: list[str | None] = [None] * len(segs)
    for part in gathered:
        for i, t in part:
            texts[i] = t
    return join_texts(texts)
