"""GPU parity of the contraction kernels: the tcgen05 tensor-core GEMM and the SIMT FP32
GEMM against a float64 numpy product, for the shapes and fused epilogues the encoder and
prefill use (bias, GELU, residual, SwiGLU), ragged edges included."""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

F32P = C.POINTER(C.c_float)


def bf16_bits(x):
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)


def ref(A, Bf, epi, bias, resid):
    acc = A.astype(np.float64) @ Bf.astype(np.float64).T
    if epi == 1:
        return acc + bias
    if epi == 2:
        v = acc + bias
        return 0.5 * v * (1 + np.tanh(0.7978845608028654 * (v + 0.044715 * v ** 3)))
    if epi == 3:
        return resid + (bias if bias is not None else 0) + acc
    if epi == 4:
        g, u = acc[:, 0::2], acc[:, 1::2]
        return g / (1 + np.exp(-g)) * u
    return acc


def run(impl, A, Bbits, epi, bias, resid, M, N, K):
    import qwen_asr_b200 as Q
    out = np.zeros((M, N // 2 if epi == 4 else N), np.float32)
    rc = Q.lib().qwen_asr_debug_gemm(M, N, K, A.ctypes.data_as(F32P), Bbits.ctypes.data_as(C.POINTER(C.c_uint16)),
                                     bias.ctypes.data_as(F32P) if bias is not None else None,
                                     resid.ctypes.data_as(F32P) if resid is not None else None, epi, impl,
                                     out.ctypes.data_as(F32P))
    assert rc == 0, rc
    return out


@pytest.mark.parametrize("M,N,K,epi", [
    (367, 896, 896, 1),      # encoder q/k/v-sized, ragged M
    (367, 3584, 896, 2),     # fc1 + GELU
    (367, 896, 3584, 3),     # fc2 + bias + residual
    (381, 6144, 1024, 4),    # prefill gate/up + SwiGLU
    (1, 4096, 1024, 0),      # single row (streaming delta prefill)
    (130, 480, 4320, 2),     # conv via im2col, K not a multiple of 64
    (26, 896, 7680, 0),      # conv_out
    (5, 200, 48, 0),         # tiny, N and K ragged
])
def test_gemm_matches_f64(M, N, K, epi):
    rng = np.random.default_rng(M * 7 + N + K)
    A = rng.standard_normal((M, K)).astype(np.float32)
    Bbits = bf16_bits(rng.standard_normal((N, K)).astype(np.float32) * 0.02)
    Bf = (Bbits.astype(np.uint32) << 16).view(np.float32)
    bias = (rng.standard_normal(N) * 0.02).astype(np.float32) if epi in (1, 2, 3) else None
    resid = rng.standard_normal((M, N)).astype(np.float32) if epi == 3 else None
    want = ref(A, Bf, epi, bias, resid)
    scale = max(1e-12, float(np.max(np.abs(want))))
    # both kernels at f32-level accuracy: the tensor-core GEMM takes A as three bf16 planes
    for impl, tol in ((0, 1e-5), (1, 1e-5)):
        got = run(impl, A, Bbits, epi, bias, resid, M, N, K)
        err = float(np.max(np.abs(got - want))) / scale
        assert err < tol, (impl, err)


@pytest.mark.parametrize("N,K", [(896, 3584), (1024, 2048), (2688, 896), (200, 48)])
def test_gemm_rows_independent_of_row_count(N, K):
    """A row's result must not depend on how many rows share the call (split-K is chosen
    from N and K only): batched segments and streams rely on it to equal single ones."""
    rng = np.random.default_rng(N + K)
    A = rng.standard_normal((381, K)).astype(np.float32)
    Bbits = bf16_bits(rng.standard_normal((N, K)).astype(np.float32) * 0.02)
    full = run(1, A, Bbits, 0, None, None, 381, N, K)
    for m in (1, 5, 130):
        part = run(1, np.ascontiguousarray(A[:m]), Bbits, 0, None, None, m, N, K)
        assert np.array_equal(part.view(np.uint32), full[:m].view(np.uint32)), m
