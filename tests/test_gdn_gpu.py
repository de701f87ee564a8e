"""Config 3: the gated delta-rule recurrence in isolation (H 2048 = 16 heads x
128, dk = dv = 128) on the GPU against the oracle's sequential CPU recurrence
(oracle/oracle.cpp orc_gdn_recurrence, src/ModelCPU.jl:640-674).  Inputs as
N(0,1) activations, beta = sigmoid(N(0,1)),
g = -softplus(N(0,1)), L2-normalised q and k."""
import ctypes as C

import numpy as np
import pytest
import torch

import oracle as O
from inferno_b200._lib import call

pytestmark = pytest.mark.gpu


def inputs(T, H=16, d=128, seed=3):
    rng = np.random.default_rng(seed)
    q = rng.standard_normal((T, H, d)).astype(np.float32)
    k = rng.standard_normal((T, H, d)).astype(np.float32)
    q /= np.linalg.norm(q, axis=-1, keepdims=True)
    k /= np.linalg.norm(k, axis=-1, keepdims=True)
    v = rng.standard_normal((T, H, d)).astype(np.float32)
    beta = (1 / (1 + np.exp(-rng.standard_normal((T, H))))).astype(np.float32)
    g = (-np.log1p(np.exp(rng.standard_normal((T, H))))).astype(np.float32)
    return q, k, v, beta, g


def run_gpu(q, k, v, beta, g, S0):
    T, H, dk = q.shape
    dv = v.shape[2]
    dev = [torch.from_numpy(a).cuda() for a in (q, k, v, beta, g)]
    S = torch.from_numpy(S0.copy()).cuda()
    y = torch.empty((T, H, dv), device="cuda")
    P = lambda t: C.c_void_p(t.data_ptr())  # noqa: E731
    call("inferno_gdn_recurrence", T, H, dk, dv, *[P(t) for t in dev], P(S), P(y), None)
    torch.cuda.synchronize()
    return S.cpu().numpy(), y.cpu().numpy()


def rel(a, b):
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-30))


@pytest.mark.parametrize("T", [1, 31, 33, 1024])
def test_gdn_recurrence_matches_oracle(T):
    q, k, v, beta, g = inputs(T)
    S0 = np.zeros((16, 128, 128), np.float32)
    S_ref = S0.copy()
    y_ref = O.gdn_recurrence(q, k, v, beta, g, S_ref)
    S, y = run_gpu(q, k, v, beta, g, S0)
    assert rel(y, y_ref) < 1e-5, rel(y, y_ref)
    assert rel(S, S_ref) < 1e-5, rel(S, S_ref)


def test_gdn_recurrence_continues_from_state():
    """Two launches of T/2 steps equal one launch of T (state carried in S)."""
    q, k, v, beta, g = inputs(96, seed=4)
    S0 = np.zeros((16, 128, 128), np.float32)
    S_a, y_a = run_gpu(q, k, v, beta, g, S0)
    S_1, y_1 = run_gpu(q[:40], k[:40], v[:40], beta[:40], g[:40], S0)
    S_2, y_2 = run_gpu(q[40:], k[40:], v[40:], beta[40:], g[40:], S_1)
    assert rel(np.concatenate([y_1, y_2]), y_a) < 1e-6
    assert rel(S_2, S_a) < 1e-6


def run_gpu_chunked(q, k, v, beta, g, S0):
    T, H, dk = q.shape
    dv = v.shape[2]
    dev = [torch.from_numpy(np.ascontiguousarray(a)).cuda() for a in (q, k, v, beta, g)]
    S = torch.from_numpy(S0.copy()).cuda()
    y = torch.empty((T, H, dv), device="cuda")
    P = lambda t: C.c_void_p(t.data_ptr())  # noqa: E731
    call("inferno_gdn_chunked", T, H, dk, dv, *[P(t) for t in dev], P(S), P(y), 64, None)
    torch.cuda.synchronize()
    return S.cpu().numpy(), y.cpu().numpy()


@pytest.mark.parametrize("T", [1, 64, 200, 4096])
def test_gdn_chunked_matches_oracle(T):
    """Config-3 prefill mode: the chunked (WY) form in chunks of 64 against
    the oracle's sequential recurrence, at north_star's 2e-3 (the chunked
    form reorders the fp32 sums); 200 = 3 chunks + a ragged 8-token one."""
    q, k, v, beta, g = inputs(T, seed=5)
    S0 = np.zeros((16, 128, 128), np.float32)
    S_ref = S0.copy()
    y_ref = O.gdn_recurrence(q, k, v, beta, g, S_ref)
    S, y = run_gpu_chunked(q, k, v, beta, g, S0)
    assert rel(y, y_ref) < 2e-3, rel(y, y_ref)
    assert rel(S, S_ref) < 2e-3, rel(S, S_ref)


def test_gdn_chunked_from_state_and_strong_decay():
    """Nonzero initial state, dv = 64, and decays down to e^-30 per token
    (cumulative decay far below fp32 range inside a chunk)."""
    T, H = 150, 4
    q, k, v, beta, g = inputs(T, H=H, seed=6)
    v = v[:, :, :64].copy()
    g = g * np.random.default_rng(7).uniform(0, 15, g.shape).astype(np.float32)
    S0 = (np.random.default_rng(8).standard_normal((H, 64, 128)) * 0.1).astype(np.float32)
    S_ref = S0.copy()
    y_ref = O.gdn_recurrence(q, k, v, beta, g, S_ref)
    S, y = run_gpu_chunked(q, k, v, beta, g, S0)
    assert np.isfinite(y).all() and np.isfinite(S).all()
    assert rel(y, y_ref) < 2e-3, rel(y, y_ref)
    assert rel(S, S_ref) < 2e-3, rel(S, S_ref)
