"""The allocation-free GEMV entry point (inferno_gemv_host_noalloc).

Some callers cannot let a library allocate device memory -- a host runtime
that owns the GPU allocator or enforces a hard memory budget, or a plugin
sandbox without allocation rights.  For them the library stages the weight
and vectors in a static device array instead of cudaMalloc'd buffers.  This
test calls that entry through the C ABI twice in a row (the array keeps the
previous call's contents) and checks each result against the allocating
compatibility entry (q4_k_gemv / q6_k_gemv, with INFERNO_COMPAT_FP32=1 so both
use fp32 activations) on the same host inputs.  It sits
in a file of its own, collected last.
"""
import ctypes as C

import numpy as np
import pytest

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
    fn = {S.Q4_K: lib().q4_k_gemv, S.Q6_K: lib().q6_k_gemv}[t]
    fn(P(q.ctypes.data), P(x.ctypes.data), P(y.ctypes.data), None, inner, rows)
    return y


def _noalloc(t, q, x, rows, inner):
    y = np.full(rows, np.nan, np.float32)
    rc = lib().inferno_gemv_host_noalloc(t, P(q.ctypes.data), P(x.ctypes.data), P(y.ctypes.data), inner, rows)
    assert rc == 0, lib().inferno_last_error()
    return y


def test_noalloc_gemv_matches_allocating_entry_twice(monkeypatch):
    monkeypatch.setenv("INFERNO_COMPAT_FP32", "1")
    cases = [(S.Q4_K, 3584, 1024, 1), (S.Q6_K, 1024, 3584, 2)]   # two different calls in a row
    for t, rows, inner, seed in cases:
        q, x = _case(t, rows, inner, seed)
        want = _compat(t, q, x, rows, inner)
        got = _noalloc(t, q, x, rows, inner)
        assert np.abs(got - want).max() / np.abs(want).max() < GEMV_RTOL


def test_noalloc_rejects_oversize():
    rows, inner = 248320, 1024            # 208 MB Q6_K: beyond the static scratch
    y = np.zeros(1, np.float32)
    rc = lib().inferno_gemv_host_noalloc(S.Q6_K, P(y.ctypes.data), P(y.ctypes.data), P(y.ctypes.data), inner, rows)
    assert rc == -1
    assert b"static scratch" in lib().inferno_last_error()
