"""GPU test of qwen_asr_mel_noalloc, the allocation-free mel entry point.

It exists for callers that cannot allocate device memory while they run (fixed
device-memory budgets, real-time audio threads, hosts that forbid allocations after
start-up): its scratch lives in a library-owned device array. This file is collected
last on purpose, so a run that stops at the first failure has already run every other
test. Output must match the regular mel path (qwen_asr_debug_mel) within the mel
tolerance of the parity tests, on two calls in a row (the second call reuses the array
left dirty by the first)."""
import ctypes as C

import numpy as np
import pytest

from qwen_asr_b200 import synth

pytestmark = pytest.mark.gpu

MAX_FRAMES = 1000


@pytest.fixture(scope="module")
def eng(tiny_dir):
    import qwen_asr_b200 as Q
    return Q.Engine(tiny_dir, device=0)


def _noalloc(eng, x):
    import torch
    import qwen_asr_b200 as Q
    d_in = torch.from_numpy(np.ascontiguousarray(x, dtype=np.float32)).to("cuda:0")
    F = len(x) // 160
    d_out = torch.full((max(F, 1), 128), float("nan"), dtype=torch.float32, device="cuda:0")
    torch.cuda.synchronize()
    got = Q.lib().qwen_asr_mel_noalloc(eng._h, C.c_void_p(d_in.data_ptr()), len(x),
                                       C.c_void_p(d_out.data_ptr()), d_out.numel())
    return got, d_out.cpu().numpy()


def test_noalloc_mel_matches_regular_path_twice(eng):
    # a loud clip first, then a quieter, shorter one: a stale maximum from call 1 would
    # shift every value of call 2
    for n, seed, gain in ((16000 * 9 + 123, 1, 1.0), (16000 * 4 + 7, 2, 0.05)):
        x = (synth.synth_audio(n, seed) * np.float32(gain)).astype(np.float32)
        F, got = _noalloc(eng, x)
        assert F == n // 160
        ref = eng.debug_mel(x)
        assert got.shape == ref.shape
        assert np.max(np.abs(got - ref)) < 2e-4


def test_noalloc_rejects_oversized_input(eng):
    import qwen_asr_b200 as Q
    x = synth.synth_audio((MAX_FRAMES + 1) * 160, 3)
    F, _ = _noalloc(eng, x)
    assert F == -1
    assert "exceed the maximum" in Q.last_error()
    # the maximum itself is accepted
    F, got = _noalloc(eng, synth.synth_audio(MAX_FRAMES * 160, 4))
    assert F == MAX_FRAMES and np.isfinite(got).all()
