"""CPU tests of the multi-GPU segment sharding host logic (qwen_asr_b200/shard.py):
world_size-2 `gloo` ranks with a deterministic stand-in transcriber must produce the
same joined text as the single-process reference order, segment boundaries come from the
library bit-exactly, and the join rule matches the oracle's restatement."""
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

from oracle import qwen_oracle as O
from qwen_asr_b200 import shard, synth


def fake_text(seg: np.ndarray) -> str:
    # deterministic per-segment text incl. empty results and punctuation-led pieces
    h = int(abs(float(seg[:4000].astype(np.float64).sum())) * 1e4) % 7
    return ["", "alpha", ",beta", " gamma", "delta.", "x", "été"][h]


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def fake_many(x, bounds):
    return [fake_text(shard.padded(x, a, b)) for a, b in bounds]


def _worker(rank, world, port, x, q, many=False):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    segs = shard.segments(x, 30.0)
    out = shard.transcribe_sharded(fake_text, x, 30.0, rank, world, segs=segs,
                                   transcribe_many=fake_many if many else None)
    if rank == 0:
        q.put(out)
    dist.destroy_process_group()


def test_segments_match_oracle_split_points():
    x = synth.synth_audio(16000 * 200, seed=5)
    segs = shard.segments(x, 30.0)
    sp = O.split_points(x, 30.0, 3.0)
    assert [a for a, _ in segs] == sp
    assert segs[-1][1] == len(x) and all(a < b for a, b in segs)


def test_assign_covers_all_and_balances():
    segs = [(0, 100), (100, 400), (400, 450), (450, 900), (900, 1000)]
    parts = shard.assign(segs, 2)
    assert sorted(i for p in parts for i in p) == list(range(5))
    loads = [sum(segs[i][1] - segs[i][0] for i in p) for p in parts]
    assert max(loads) - min(loads) <= 300


def test_join_matches_oracle_rule():
    texts = ["alpha", ",beta", "", "gamma", "été", "x"]
    want = ""
    for t in texts:
        if not t:
            continue
        if want and O.should_insert_boundary_space(want.encode()[-1], t.encode()[0]):
            want += " "
        want += t
    assert shard.join_texts(texts) == want


@pytest.mark.parametrize("many", [False, True])
def test_two_gloo_ranks_match_single_process(many):
    x = synth.synth_audio(16000 * 130, seed=9)
    segs = shard.segments(x, 30.0)
    single = shard.join_texts([fake_text(shard.padded(x, a, b)) for a, b in segs])
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, x, q, many)) for r in range(2)]
    for p in procs:
        p.start()
    out = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert out == single
