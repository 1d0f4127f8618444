#!/usr/bin/env python
"""Benchmark of the Qwen3-ASR transcription path on B200 (one process per GPU).

A step is one offline transcription of one clip (mel -> encoder -> prefill -> greedy
decode) on each GPU. Default workload ("C2"): Qwen3-ASR-0.6B,
28.2 s seeded synthetic clip, int8 decode of 256 tokens (EOS ignored), weights
random-init in the reference's safetensors layout. Every rank transcribes its own clip
(replicas, weak scaling, no collective on the data path; NCCL only carries the
barrier and the max-over-ranks timing).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--config c1|c2|c3]

Prints one JSON line on rank 0.
"""
from __future__ import annotations

import argparse
import ctypes
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

CONFIGS = {
    # name: (preset, samples, audio seed, decode tokens, decode mode, weight seed)
    "c1": ("0.6b", 451200, 1, 128, "bf16", 0),
    "c2": ("0.6b", 451200, 1, 256, "int8", 0),
    "c3": ("1.7b", 960000, 2, 512, "bf16", 1),
    # C4: 20-minute clip split with -S 30, segments sharded over the ranks (strong scaling)
    "c4": ("0.6b", 19200000, 3, 200, "bf16", 0),
    # C5: independent 120 s streams fed in 2 s chunks (<= 32 new tokens per chunk), streams
    # sharded over the ranks; a step is one round in which every stream pushes one chunk
    "c5": ("1.7b", 1920000, 5, 32, "int8", 1),
}
C5_STREAMS = 256
PRESET_DIMS = {"0.6b": (1024, 3072), "1.7b": (2048, 6144)}  # dec hidden, intermediate
N_LAYERS, KV_HEADS, HEAD_DIM, VOCAB, Q_DIM = 28, 8, 128, 151936, 2048


def decode_step_bytes(preset: str, mode: str, pos: float) -> float:
    """Algorithmic HBM bytes of one decode step: every decoder weight once (int8 or bf16),
    the int8 row scales, and the f32 KV cache rows 0..pos of every layer."""
    h, inter = PRESET_DIMS[preset]
    per_layer = (Q_DIM + 2 * KV_HEADS * HEAD_DIM) * h + h * Q_DIM + 2 * inter * h + h * inter
    n_w = N_LAYERS * per_layer + VOCAB * h
    esz = 1 if mode == "int8" else 2
    scales = (N_LAYERS * (Q_DIM + 2 * KV_HEADS * HEAD_DIM + h + 2 * inter + h) + VOCAB) * 4 if mode == "int8" else 0
    kv = N_LAYERS * KV_HEADS * HEAD_DIM * 4 * 2 * (pos + 1)
    return n_w * esz + scales + kv


def measured_hbm_peak():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def profile_traffic(avg_pos: float):
    """DRAM bytes of one decode step, from the committed ncu capture of a step at a known KV
    position scaled to avg_pos: the weight bytes are fixed, the KV part grows with position."""
    p = os.path.join(ROOT, "profiles", "decode_step_int8_c2.md")
    vals = {}
    try:
        for line in open(p):
            k, _, v = line.partition(":")
            if k in ("captured_bytes_per_step", "captured_pos", "kv_bytes_per_position"):
                vals[k] = float(v.strip())
    except OSError:
        return None
    if len(vals) != 3:
        return None
    return int(vals["captured_bytes_per_step"] + vals["kv_bytes_per_position"] * (avg_pos - vals["captured_pos"]))


class ClockSampler:
    """nvidia-smi clock / throttle-reason sampling during the timed region."""

    def __init__(self, gpu_index: int):
        self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        try:
            self.p = subprocess.Popen(["nvidia-smi", "-i", str(gpu_index), f"--query-gpu={q}",
                                       "--format=csv,noheader,nounits", "-lms", "200"],
                                      stdout=self.f, stderr=subprocess.DEVNULL)
        except Exception:
            self.p = None

    def stop(self):
        if self.p is None:
            return None
        self.p.terminate()
        try:
            self.p.wait(timeout=5)
        except Exception:
            self.p.kill()
        self.f.seek(0)
        rows = [r.split(", ") for r in self.f.read().strip().splitlines() if r.strip()]
        os.unlink(self.f.name)
        if not rows:
            return None
        sm = [float(r[1]) for r in rows if len(r) > 2 and r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if len(r) > 2 and r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows if len(r) >= 9 for i in range(4) if r[5 + i].strip() == "Active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows)}


def dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    import torch
    if world > 1:
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    return world, rank, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def max_over_ranks(world, v: float, local: int) -> float:
    if world == 1:
        return v
    import torch
    import torch.distributed as dist
    t = torch.tensor([v], dtype=torch.float64, device=f"cuda:{local}")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def model_dir(preset, seed, world, rank, local):
    from qwen_asr_b200 import synth
    d = os.path.join(os.environ.get("QASR_BENCH_DIR", "/tmp/qasr_bench"), f"{preset}-s{seed}")
    if rank == 0:
        synth.write_model(d, preset, seed, device="cpu")  # identical weights for both arms
    barrier(world)
    return d


# ------------------------------------------------------------------------ CPU baseline
def cpu_sample(preset, n_samples, seed, tokens, mode, wseed, model_path, model=None, prep=None):
    """One full transcription of the workload on the host, measured end to end (nothing
    extrapolated): mel + encoder + prefill of the whole clip with the numpy restatement of the
    reference's CPU path (oracle/qwen_oracle.py, float32 sgemm on every core), then all
    `tokens` greedy decode steps with the C restatement of decoder_forward
    (oracle/decode_ref.c, OpenMP over every core). Returns (audio-sec/sec, seconds, model, prep)."""
    import numpy as np
    from oracle import qwen_oracle as O
    from oracle import ref_decode as R
    from qwen_asr_b200 import synth
    if model is None:
        model = O.Model(model_path, decode_mode=mode)
        prep = R.Prepared(model)
    x = synth.synth_audio(n_samples, seed)
    t0 = time.perf_counter()
    mel = O.mel_spectrogram(x)
    enc = model.encode(mel)
    ctx = O.Ctx.__new__(O.Ctx)
    ctx.model, ctx.tok, ctx.prompt, ctx.force_language = model, None, None, None
    rows = O.prompt_rows(ctx, enc)
    dec = O.Decoder(model)
    dec.prefill(rows[:-1])
    ids, _ = R.decode(prep, dec, rows[-1], tokens)
    t1 = time.perf_counter()
    assert len(ids) == tokens and np.all(ids >= 0)
    return (n_samples / 16000.0) / (t1 - t0), t1 - t0, model, prep


def host_cpu():
    """CPU model, logical and physical core counts of this host."""
    model, phys = None, set()
    try:
        cur = {}
        for line in open("/proc/cpuinfo"):
            k, _, v = line.partition(":")
            k, v = k.strip(), v.strip()
            if k == "model name" and model is None:
                model = v
            if k in ("physical id", "core id"):
                cur[k] = v
            if not line.strip():
                if cur:
                    phys.add((cur.get("physical id"), cur.get("core id")))
                cur = {}
    except OSError:
        pass
    return {"model": model, "logical": os.cpu_count(), "physical": len(phys) or None}


def set_host_threads(n):
    """BLAS pool (numpy sgemm) and OpenMP pool (C decode) sized to n threads (torchrun sets
    OMP_NUM_THREADS=1, so both are set explicitly)."""
    from threadpoolctl import threadpool_limits
    from oracle import ref_decode as R
    R.set_threads(n)
    return threadpool_limits(limits=n)


# ------------------------------------------------------------------------ main arms
def run_reference(args, world, rank, local):
    if rank != 0:
        return
    preset, n, seed, tokens, mode, wseed = CONFIGS[args.config]
    if args.tokens:
        tokens = args.tokens
    from qwen_asr_b200 import synth
    d = os.path.join(os.environ.get("QASR_BENCH_DIR", "/tmp/qasr_bench"), f"{preset}-s{wseed}")
    synth.write_model(d, preset, wseed, device="cpu")  # same file as the GPU arm writes
    cpu = host_cpu()
    threads = cpu["logical"]
    set_host_threads(threads)
    model = prep = None
    for _ in range(args.warmup):
        _, _, model, prep = cpu_sample(preset, n, seed, tokens, mode, wseed, d, model, prep)
    secs = []
    for _ in range(args.steps):
        _, s, model, prep = cpu_sample(preset, n, seed, tokens, mode, wseed, d, model, prep)
        secs.append(s)
    total = sum(secs)
    value = args.steps * (n / 16000.0) / total
    t16 = min(16, threads)
    set_host_threads(t16)
    v16, s16, _, _ = cpu_sample(preset, n, seed, tokens, mode, wseed, d, model, prep)
    sample = (f"every step one full transcription of the {n / 16000:.1f} s clip: numpy mel+encoder+prefill and "
              f"all {tokens} decode steps in C, measured")
    line = {
        "impl": "reference", "metric": "audio-sec/sec", "value": round(value, 4), "unit": "audio-s/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(1000 * total / args.steps, 2), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "int8+f32" if mode == "int8" else "bf16+f32", "data": "synthetic",
        "config": config_dict(args.config, world),
        "cpu_baseline": {"value": round(value, 4), "unit": "audio-s/s", "cores": threads, "kind": "port",
                         "sample": sample, "cpu": cpu,
                         f"at_{t16}_threads": {"value": round(v16, 4), "seconds": round(s16, 2)}},
        "e2e": {"value": round(value, 4), "unit": "audio-s/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "reference = restatement of the reference CPU path (oracle/qwen_oracle.py numpy + oracle/decode_ref.c "
                "OpenMP decode); the Rust reference cannot be built here (no cargo) and its int8 decode is "
                "unimplemented on x86_64",
    }
    print(json.dumps(line), flush=True)


def config_dict(name, world):
    preset, n, seed, tokens, mode, wseed = CONFIGS[name]
    return {"workload": f"{name.upper()}: Qwen3-ASR-{preset.upper()} offline transcription of a {n / 16000:.1f} s "
                        f"clip, {mode} decode of {tokens} tokens (EOS ignored), one clip per GPU",
            "clip_sec": n / 16000.0, "decode_tokens": tokens, "decode_weights": mode,
            "l2": "no flush: each step streams >1 GB of weights, far larger than the 126 MB L2",
            "parallelism": f"replicas x{world}"}


def run_streams(args, world, rank, local):
    """C5: every rank serves its share of the concurrent streams through the C ABI's
    streaming calls (qwen_asr_stream_push, per-stream KV slots). The timed region is K rounds
    of one 2 s chunk per stream (after W warm-up rounds) on a bounded sample of the streams."""
    import numpy as np
    import torch
    import qwen_asr_b200 as Q
    from qwen_asr_b200 import synth

    preset, n, seed, tokens, mode, wseed = CONFIGS[args.config]
    d = model_dir(preset, wseed, world, rank, local)
    torch.cuda.set_device(local)
    eng = Q.Engine(d, device=local)
    eng.set_decode_mode(mode)
    mine = list(range(rank, C5_STREAMS, world))
    sample = mine[:max(1, args.streams)]
    chunk = 32000
    # every stream runs its whole 120 s (60 chunks of 2 s), so the re-anchor at chunk 45,
    # degeneracy resets and speech ends happen inside the timed region; the first `warmup`
    # chunks are untimed
    rounds = n // chunk
    args.steps = rounds - args.warmup
    audio = {i: synth.synth_audio(chunk * rounds, seed * 1000 + i) for i in sample}
    streams = {i: Q.Stream() for i in sample}
    stream = torch.cuda.ExternalStream(eng.cuda_stream(), device=f"cuda:{local}")
    order = [streams[i] for i in sample]

    def push_round(r):
        return Q.stream_push_many(eng, order, [audio[i][r * chunk:(r + 1) * chunk] for i in sample])

    for r in range(args.warmup):
        push_round(r)
    barrier(world)
    torch.cuda.synchronize()
    clocks = ClockSampler(local)
    l0 = eng.launch_count()
    p0 = eng.perf()
    lat = []
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for r in range(args.warmup, rounds):
        t0 = time.perf_counter()
        push_round(r)  # every stream's chunk is done when the batched round returns
        lat += [1000.0 * (time.perf_counter() - t0)] * len(sample)
    e1.record(stream)
    torch.cuda.synchronize()
    clk = clocks.stop()
    launches = eng.launch_count() - l0
    p1 = eng.perf()
    stage = {k: round((p1[k] - p0[k]) / args.steps, 2) for k in ("gpu_mel_ms", "gpu_enc_ms", "gpu_prefill_ms",
                                                                  "gpu_decode_ms")}
    ms = max_over_ranks(world, e0.elapsed_time(e1), local)
    value = world * len(sample) * args.steps * 2.0 / (ms / 1000.0)
    lat_all = lat
    if world > 1:
        import torch.distributed as dist
        got = [None] * world
        dist.all_gather_object(got, lat)
        lat_all = [x for part in got for x in part]
    if rank == 0:
        p50, p99 = float(np.percentile(lat_all, 50)), float(np.percentile(lat_all, 99))
        line = {
            "metric": "audio-sec/sec", "value": round(value, 3), "unit": "audio-s/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 2),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int8+f32",
            "data": "synthetic",
            "config": {"workload": f"C5: Qwen3-ASR-1.7B int8, {C5_STREAMS} independent 120 s streams in 2 s chunks "
                                   f"(<= {tokens} new tokens per chunk), streams sharded over {world} GPU(s), each round's chunks decoded as "
                                   f"one batch; timed "
                                   f"sample: {len(sample)} streams per GPU, chunks {args.warmup + 1}..{rounds} of every stream "
                                   f"(whole 120 s streams; the first {args.warmup} chunks untimed)",
                       "streams_per_gpu_sample": len(sample),
                       "parallelism": f"stream shards x{world}", "l2": "no flush: every chunk streams >1.7 GB of weights"},
            "latency_ms_per_chunk": {"p50": round(p50, 2), "p99": round(p99, 2),
                                     "note": "a stream's chunk latency is the wall time of the push call that "
                                             "returns its delta; every stream of a GPU is pushed in one batched call"},
            "stage_ms_per_round": stage,
            "e2e": {"value": round(value, 3), "unit": "audio-s/s", "h2d_bytes_per_step": 4 * chunk * len(sample),
                    "d2h_bytes_per_step": 0, "note": "streams run from host buffers through the C ABI"},
            "gpu_launches": int(launches), "clocks": clk,
        }
        print(json.dumps(line), flush=True)
    barrier(world)


def measure_segmented(eng, world, rank, local, steps, warmup):
    """C4 on an already loaded 0.6B engine: every rank transcribes its share of the -S 30
    segments of one 20-minute clip (qwen_asr_b200.shard, longest-first); rank 0 joins the
    texts. Total work is fixed (strong scaling). Device time, max over ranks."""
    import torch
    from qwen_asr_b200 import shard, synth
    preset, n, seed, tokens, mode, wseed = CONFIGS["c4"]
    eng.set_decode_mode(mode)
    eng.set_force_n_tokens(tokens)
    x = synth.synth_audio(n, seed)
    segs = shard.segments(x, 30.0)
    stream = torch.cuda.ExternalStream(eng.cuda_stream(), device=f"cuda:{local}")
    batch = eng.set_decode_batch(0)
    mine = shard.assign(segs, world)[rank]
    for _ in range(max(1, warmup)):
        eng.transcribe_segments(x, [segs[i] for i in mine[:batch]])
    barrier(world)
    torch.cuda.synchronize()
    l0 = eng.launch_count()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        shard.transcribe_sharded(eng.transcribe_pcm, x, 30.0, rank, world, segs=segs,
                                 transcribe_many=eng.transcribe_segments)
    e1.record(stream)
    torch.cuda.synchronize()
    launches = eng.launch_count() - l0
    ms = max_over_ranks(world, e0.elapsed_time(e1), local)
    per_rank = [len(m) for m in shard.assign(segs, world)]
    return {"value": round(steps * (n / 16000.0) / (ms / 1000.0), 3), "unit": "audio-s/s",
            "ms_per_step": round(ms / steps, 2), "steps": steps, "scaling": "strong",
            "workload": f"C4: Qwen3-ASR-0.6B, {n / 16000 / 60:.0f}-minute clip split with -S 30 into {len(segs)} "
                        f"segments sharded over {world} GPU(s) (longest first), {mode} decode of {tokens} tokens per "
                        f"segment, up to {batch} segments per batched decode",
            "segments": len(segs), "segments_per_gpu_max": max(per_rank), "decode_batch": batch,
            "gpu_launches": int(launches)}


def run_segmented(args, world, rank, local):
    """C4 as the line's own workload (--config c4)."""
    import torch
    import qwen_asr_b200 as Q

    preset, n, seed, tokens, mode, wseed = CONFIGS[args.config]
    d = model_dir(preset, wseed, world, rank, local)
    torch.cuda.set_device(local)
    eng = Q.Engine(d, device=local)
    clocks = ClockSampler(local)
    seg = measure_segmented(eng, world, rank, local, args.steps, args.warmup)
    clk = clocks.stop()
    if rank == 0:
        line = {
            "metric": "audio-sec/sec", "value": seg["value"], "unit": "audio-s/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": seg["ms_per_step"],
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "bf16+f32" if mode == "bf16" else "int8+f32", "data": "synthetic",
            "config": {"workload": seg["workload"], "segments": seg["segments"], "decode_batch": seg["decode_batch"],
                       "parallelism": f"segment shards x{world}",
                       "l2": "no flush: each segment streams >1 GB of weights"},
            "e2e": {"value": seg["value"], "unit": "audio-s/s", "h2d_bytes_per_step": 4 * n,
                    "d2h_bytes_per_step": 4 * tokens * seg["segments"],
                    "note": "the segmented path always runs from host buffers through the C ABI"},
            "gpu_launches": seg["gpu_launches"], "clocks": clk,
        }
        print(json.dumps(line), flush=True)
    barrier(world)


def run_ours(args, world, rank, local):
    import numpy as np
    import torch
    import qwen_asr_b200 as Q
    from qwen_asr_b200 import synth

    preset, n, seed, tokens, mode, wseed = CONFIGS[args.config]
    if args.tokens:
        tokens = args.tokens
    d = model_dir(preset, wseed, world, rank, local)
    torch.cuda.set_device(local)
    eng = Q.Engine(d, device=local)
    eng.set_decode_mode(mode)
    eng.set_force_n_tokens(tokens)
    x = synth.synth_audio(n, seed + rank)
    x_dev = torch.from_numpy(x).to(f"cuda:{local}")
    x_pin = torch.from_numpy(x).pin_memory()
    stream = torch.cuda.ExternalStream(eng.cuda_stream(), device=f"cuda:{local}")
    torch.cuda.synchronize()

    for _ in range(args.warmup):
        if eng.transcribe_device(x_dev.data_ptr(), n) is None:
            raise RuntimeError(f"transcription failed: {Q.last_error()}")

    # ---- device-resident timed region
    barrier(world)
    torch.cuda.synchronize()
    clocks = ClockSampler(local)
    l0 = eng.launch_count()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    dec_ms, steps_done = 0.0, 0
    for _ in range(args.steps):
        eng.transcribe_device(x_dev.data_ptr(), n)
        p = eng.perf()
        dec_ms += p["gpu_decode_ms"]
        steps_done += int(p["decode_steps"])
    e1.record(stream)
    torch.cuda.synchronize()
    launches = eng.launch_count() - l0
    clk = clocks.stop()
    barrier(world)
    ms = max_over_ranks(world, e0.elapsed_time(e1), local)
    ms_step = ms / args.steps
    value = world * args.steps * (n / 16000.0) / (ms / 1000.0)

    # ---- end to end through the C ABI with host buffers (H2D inside the timed region); the
    # host-buffer path gets its own untimed warm-up (its first call allocates the staging
    # buffer the device path never needs)
    lib = Q.lib()
    host_ptr = ctypes.cast(x_pin.data_ptr(), Q._F32P)  # pinned host samples
    Q._take_string(lib.qwen_asr_transcribe_pcm(eng._h, host_ptr, n))
    barrier(world)
    torch.cuda.synchronize()
    h0, h1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    h0.record(stream)
    for _ in range(args.steps):
        Q._take_string(lib.qwen_asr_transcribe_pcm(eng._h, host_ptr, n))
    h1.record(stream)
    torch.cuda.synchronize()
    barrier(world)
    e2e_ms = max_over_ranks(world, h0.elapsed_time(h1), local)
    e2e_value = world * args.steps * (n / 16000.0) / (e2e_ms / 1000.0)

    # ---- the same clip as a 44.1 kHz WAV file in host memory through qwen_asr_transcribe_wav_buffer
    # (the reference's own benchmark input is a 44.1 kHz WAV): parsing, H2D and GPU resampling
    # inside the timed region
    wav44 = None
    if not args.no_segmented:
        import io
        import struct
        x44 = synth.synth_audio(int(n * 44100 / 16000), seed + rank)
        s16 = np.clip(np.round(x44 * 32768.0), -32768, 32767).astype("<i2").tobytes()
        hdr = b"RIFF" + struct.pack("<I", 36 + len(s16)) + b"WAVE" + b"fmt " + \
            struct.pack("<IHHIIHH", 16, 1, 1, 44100, 88200, 2, 16) + b"data" + struct.pack("<I", len(s16))
        blob = hdr + s16
        cbuf = (ctypes.c_uint8 * len(blob)).from_buffer_copy(blob)
        Q._take_string(lib.qwen_asr_transcribe_wav_buffer(eng._h, cbuf, len(blob)))  # untimed warm-up
        barrier(world)
        torch.cuda.synchronize()
        w0, w1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        w0.record(stream)
        for _ in range(args.steps):
            Q._take_string(lib.qwen_asr_transcribe_wav_buffer(eng._h, cbuf, len(blob)))
        w1.record(stream)
        torch.cuda.synchronize()
        wms = max_over_ranks(world, w0.elapsed_time(w1), local)
        wav44 = {"value": round(world * args.steps * (n / 16000.0) / (wms / 1000.0), 3), "unit": "audio-s/s",
                 "h2d_bytes_per_step": len(blob), "d2h_bytes_per_step": 4 * tokens,
                 "note": "the clip as a 44.1 kHz 16-bit WAV buffer through qwen_asr_transcribe_wav_buffer "
                         "(parse, copy, GPU Kaiser-sinc resampling to 16 kHz, transcription)"}

    # ---- roofline of the int8 decode step (HBM-bound), timed by the engine's CUDA events
    perf = eng.perf()
    step_ms = dec_ms / max(steps_done, 1)
    # prompt rows = 9 prefix + T_enc + 6 suffix (transcribe.rs:96-169)
    frames = n // 160
    def cw(w):
        return (w + 2 - 3) // 2 + 1
    t_enc = (frames // 100) * 13 + (cw(cw(cw(frames % 100))) if frames % 100 else 0)
    prompt = 9 + t_enc + 6
    avg_pos = prompt - 1 + tokens / 2.0
    bytes_step = decode_step_bytes(preset, mode, avg_pos)
    achieved = bytes_step / (step_ms / 1000.0) / 1e9
    peak, peak_kind = measured_hbm_peak()
    traffic = profile_traffic(avg_pos) if (preset, mode) == ("0.6b", "int8") else None
    roofline = {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                "frac": round(achieved / peak, 4), "traffic": traffic,
                "kernel": f"decode step ({mode} weight matvec chain + attention + lm_head argmax)",
                "algorithmic_bytes_per_step": int(bytes_step), "avg_step_ms": round(step_ms, 4),
                "peak_source": peak_kind}

    # ---- the C4 segmented strong-scaling measurement at this N (same weights, bf16 decode)
    segmented = None
    if not args.no_segmented:
        segmented = measure_segmented(eng, world, rank, local, steps=min(args.steps, 3), warmup=1)

    line = None
    if rank == 0:
        cb = None
        if not args.no_cpu_baseline:
            cpu = host_cpu()
            try:
                set_host_threads(cpu["logical"])
                v1, s1, _, _ = cpu_sample(preset, n, seed, tokens, mode, wseed, d)
                cb = {"value": round(v1, 4), "unit": "audio-s/s", "cores": cpu["logical"], "kind": "port",
                      "sample": f"one full transcription of the {n / 16000:.1f} s clip on the host ({s1:.1f} s): numpy "
                                f"mel+encoder+prefill and all {tokens} decode steps in C, measured", "cpu": cpu}
            except Exception as ex:  # the baseline must not break the GPU line
                cb = {"value": None, "unit": "audio-s/s", "cores": cpu["logical"], "kind": "port",
                      "sample": f"failed: {ex}"}
        line = {
            "metric": "audio-sec/sec", "value": round(value, 3), "unit": "audio-s/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_step, 3),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "int8+f32" if mode == "int8" else "bf16+f32",
            "data": "synthetic: seeded random-init weights in the reference safetensors layout + seeded speech-like audio",
            "config": config_dict(args.config, world),
            "decode_tok_s_per_gpu": round(1000.0 / step_ms, 1),
            "stage_ms": {k: round(perf[k], 3) for k in ("gpu_mel_ms", "gpu_enc_ms", "gpu_prefill_ms", "gpu_decode_ms")},
            "e2e": {"value": round(e2e_value, 3), "unit": "audio-s/s", "h2d_bytes_per_step": 4 * n,
                    "d2h_bytes_per_step": 4 * tokens},
            "e2e_wav44k": wav44,
            "gpu_launches": int(launches),
            "roofline": roofline,
            "cpu_baseline": cb,
            "clocks": clk,
            "segmented": segmented,
        }
        print(json.dumps(line), flush=True)
    barrier(world)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--config", choices=sorted(CONFIGS), default="c2")
    ap.add_argument("--tokens", type=int, default=0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-segmented", action="store_true", help="skip the C4 sub-measurement of the default line")
    ap.add_argument("--streams", type=int, default=8, help="C5: streams per GPU in the timed sample")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3) if args.impl == "ours" else args.warmup
    world, rank, local = dist_setup()
    if args.impl == "reference":
        run_reference(args, world, rank, local)
    elif args.config == "c4":
        run_segmented(args, world, rank, local)
    elif args.config == "c5":
        run_streams(args, world, rank, local)
    else:
        run_ours(args, world, rank, local)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
