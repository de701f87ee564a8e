"""Failure detection on one GPU without a GPU fault: a bounded device-side
wait is made to run out (the tensor-parallel exchange reader polling partials
that nothing writes) and must come back as INFERNO_EDEVICE with the device
error word set, after which the context keeps working."""
import ctypes as C

import numpy as np
import pytest

import oracle as O
from inferno_b200 import synth as S
from inferno_b200._lib import EDEVICE, call, lib

pytestmark = pytest.mark.gpu


def test_exchange_reader_times_out_and_returns():
    err = C.c_int(0)
    rc = lib().inferno_debug_xch_timeout(2000, C.byref(err))
    assert rc == EDEVICE, lib().inferno_last_error()
    assert err.value == 1                      # DERR_MBAR_TIMEOUT
    assert b"timed out" in lib().inferno_last_error()
    # the context is intact: an ordinary GEMV still runs and is correct
    import torch
    rows, inner, t = 256, 1024, S.Q4_K
    rng = np.random.default_rng(1)
    q = S.quantize((rng.standard_normal((rows, inner)) * 0.02).astype(np.float32), t)
    x = rng.standard_normal(inner).astype(np.float32)
    dW, dx = torch.from_numpy(q).cuda(), torch.from_numpy(x).cuda()
    dy = torch.zeros(rows, dtype=torch.float32, device="cuda")
    call("inferno_gemv", t, C.c_void_p(dW.data_ptr()), C.c_void_p(dx.data_ptr()), C.c_void_p(dy.data_ptr()),
         inner, rows, 1, None)
    torch.cuda.synchronize()
    ref = O.gemv(t, q, x[None], inner, rows)[0]
    assert np.abs(dy.cpu().numpy() - ref).max() / np.abs(ref).max() < 1e-5


def test_exchange_timeout_argument_checks():
    assert lib().inferno_debug_xch_timeout(0, None) < 0
