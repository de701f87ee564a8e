"""The allocation-free GEMV entry point (inferno_gemv_host_noalloc).

Some callers cannot let a library allocate device memory -- a host runtime
that owns the GPU allocator or enforces a hard memory budget, or a plugin
sandbox without allocation rights.  For them the library stages the weight
and vectors in a static device array instead of cudaMalloc'd buffers.  These
tests call that entry through the C ABI several times in a row (the array
keeps the previous call's contents) and check each result against the CPU
oracle and against the allocating compatibility entry (q*_gemv), in both of
their numerics: the replaced library's Q8_K path (the default, bit for bit)
and fp32 activations (INFERNO_COMPAT_FP32=1, within the GEMV tolerance).  The
file sits on its own and is collected last.
"""
import ctypes as C

import numpy as np
import pytest

import oracle as O
from inferno_b200 import synth as S
from inferno_b200._lib import lib

pytestmark = pytest.mark.gpu

GEMV_RTOL = 1e-5      # same bound as the other GEMV parity tests
P = C.c_void_p


def _case(t, rows, inner, seed):
    rng = np.random.default_rng(seed)
    q = np.ascontiguousarray(S.quantize((rng.standard_normal((rows, inner)) * 0.02).astype(np.float32), t))
    x = rng.standard_normal(inner).astype(np.float32)
    return q, x


def _compat(t, q, x, rows, inner):
    y = np.zeros(rows, np.float32)
    if t == S.Q8_0:
        lib().q8_0_gemv(P(q.ctypes.data), P(x.ctypes.data), P(y.ctypes.data), inner, rows)
    else:
        fn = {S.Q4_K: lib().q4_k_gemv, S.Q5_K: lib().q5_k_gemv, S.Q6_K: lib().q6_k_gemv}[t]
        fn(P(q.ctypes.data), P(x.ctypes.data), P(y.ctypes.data), None, inner, rows)
    return y


def _noalloc(t, q, x, rows, inner):
    y = np.full(rows, np.nan, np.float32)
    rc = lib().inferno_gemv_host_noalloc(t, P(q.ctypes.data), P(x.ctypes.data), P(y.ctypes.data), inner, rows)
    assert rc == 0, lib().inferno_last_error()
    return y


def _rel(a, b):
    return float(np.abs(a - b).max() / np.abs(b).max())


CASES = [(S.Q4_K, 3584, 1024, 1), (S.Q6_K, 1024, 3584, 2), (S.Q5_K, 1000, 2048, 3), (S.Q8_0, 777, 1024, 4)]


def test_noalloc_default_numerics_match_compat_entry(monkeypatch):
    """Default: the replaced library's Q8_K numerics, bit-identical to q*_gemv
    and to the oracle's restatement of quant_kernels.c; calls in a row."""
    monkeypatch.delenv("INFERNO_COMPAT_FP32", raising=False)
    for t, rows, inner, seed in CASES:
        q, x = _case(t, rows, inner, seed)
        got = _noalloc(t, q, x, rows, inner)
        assert np.array_equal(got.view(np.uint32), _compat(t, q, x, rows, inner).view(np.uint32)), S.TYPE_NAME[t]
        assert np.array_equal(got.view(np.uint32), O.ref_numerics_gemv(t, q, x, inner, rows).view(np.uint32))


def test_noalloc_fp32_numerics_match_oracle(monkeypatch):
    """INFERNO_COMPAT_FP32=1: fp32 activations, against the oracle's Dequant.jl
    dequantization + fp32 matmul and against q*_gemv in the same mode."""
    monkeypatch.setenv("INFERNO_COMPAT_FP32", "1")
    for t, rows, inner, seed in CASES:
        q, x = _case(t, rows, inner, seed)
        got = _noalloc(t, q, x, rows, inner)
        ref = O.gemv(t, q, x[None], inner, rows)[0]
        assert _rel(got, ref) < GEMV_RTOL, (S.TYPE_NAME[t], _rel(got, ref))
        assert _rel(got, _compat(t, q, x, rows, inner)) < GEMV_RTOL


def test_noalloc_iq2xxs_and_f32_match_oracle():
    """IQ2_XXS and F32 (no q*_gemv counterpart): fp32 activations vs the oracle."""
    for t, rows, inner, seed in [(S.IQ2_XXS, 300, 1024, 5), (S.F32, 100, 512, 6)]:
        q, x = _case(t, rows, inner, seed)
        for _ in range(2):
            got = _noalloc(t, q, x, rows, inner)
            ref = O.gemv(t, q, x[None], inner, rows)[0]
            assert _rel(got, ref) < GEMV_RTOL, (S.TYPE_NAME[t], _rel(got, ref))


def test_noalloc_rejects_bad_sizes():
    y = np.zeros(1, np.float32)
    rows, inner = 248320, 1024            # 208 MB Q6_K: beyond the static scratch
    rc = lib().inferno_gemv_host_noalloc(S.Q6_K, P(y.ctypes.data), P(y.ctypes.data), P(y.ctypes.data), inner, rows)
    assert rc == -1
    assert b"static scratch" in lib().inferno_last_error()
    # F32 rows must be a whole number of 32-element chunks
    rc = lib().inferno_gemv_host_noalloc(S.F32, P(y.ctypes.data), P(y.ctypes.data), P(y.ctypes.data), 100, 4)
    assert rc == -1
