"""GPU parity: bit-exact dequant and fused dequant-GEMV vs the CPU oracle
(config-2 shapes and formats, plus ragged row counts).  Calls go through the
C ABI of libinferno_b200.so with device pointers."""
import ctypes as C

import numpy as np
import pytest

import oracle as O
from inferno_b200 import synth as S
from inferno_b200._lib import call, lib

pytestmark = pytest.mark.gpu

TYPES = [S.Q4_K, S.Q5_K, S.Q6_K, S.Q8_0, S.IQ2_XXS, S.F32]
GEMV_RTOL = 1e-5          # max|y - y_ref| / max|y_ref|, fp32 CUDA-core path
TC_RTOL = 1e-4            # tensor-core GEMM (batch >= 16): see tests/test_gemm_tc_gpu.py


def _dev(a):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def _stream():
    import torch
    return C.c_void_p(torch.cuda.current_stream().cuda_stream)


def _sync():
    import torch
    torch.cuda.synchronize()
    assert lib().inferno_device_error(0, 1) == 0


def _matrix(t, rows, inner, seed):
    rng = np.random.default_rng(seed)
    w = (rng.standard_normal((rows, inner)) * 0.02).astype(np.float32)
    return S.quantize(w, t)


def _rel(a, b):
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-30))


@pytest.mark.parametrize("t", TYPES, ids=[S.TYPE_NAME[t] for t in TYPES])
def test_dequant_bitexact(t):
    q = _matrix(t, 67, 1024, 1)
    n = 67 * 1024
    ref = O.dequant(t, q.reshape(-1), n)
    dq = _dev(q.reshape(-1))
    out = _dev(np.zeros(n, np.float32))
    call("inferno_dequantize", t, C.c_void_p(dq.data_ptr()), n, C.c_void_p(out.data_ptr()), _stream())
    _sync()
    got = out.cpu().numpy()
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))


SHAPES = [(3584, 1024), (1024, 3584), (1000, 1024), (37, 512), (6144, 1024), (512, 2048)]


@pytest.mark.parametrize("t", TYPES, ids=[S.TYPE_NAME[t] for t in TYPES])
@pytest.mark.parametrize("shape", SHAPES, ids=[f"{o}x{i}" for o, i in SHAPES])
@pytest.mark.parametrize("batch", [1, 4])
def test_gemv_parity(t, shape, batch):
    rows, inner = shape
    q = _matrix(t, rows, inner, 2)
    x = np.random.default_rng(3).standard_normal((batch, inner)).astype(np.float32)
    ref = O.gemv(t, q, x, inner, rows)
    dW, dx = _dev(q), _dev(x)
    dy = _dev(np.zeros((batch, rows), np.float32))
    call("inferno_gemv", t, C.c_void_p(dW.data_ptr()), C.c_void_p(dx.data_ptr()), C.c_void_p(dy.data_ptr()),
         inner, rows, batch, _stream())
    _sync()
    got = dy.cpu().numpy()
    assert _rel(got, ref) < GEMV_RTOL, _rel(got, ref)


# BASELINE config-2 shapes (out x in): the large ones, every type, batch 1 /
# 4 / 16 (and 128 on 12288x4096).  Weights are seeded random GGUF blocks
# (arbitrary quant bytes, finite fp16 scales): quantizing a 254M-element
# matrix to IQ2_XXS in numpy takes minutes, and the GEMV's parity does not
# depend on where the block bytes came from.  Reference: the oracle's
# Dequant.jl dequantization followed by an fp32 matmul.
CONFIG2_BIG = [(12288, 4096), (4096, 12288), (248320, 1024)]
_BIG_CACHE = {}


def _big_matrix(t, rows, inner):
    key = (t, rows, inner)
    if key not in _BIG_CACHE:
        from q8k_cases import random_blocks
        _BIG_CACHE.clear()
        qk, bb = S.BLOCK[t]
        nb = rows * inner // qk
        rng = np.random.default_rng(1000 + 7 * t + rows)
        _BIG_CACHE[key] = random_blocks(rng, t, nb).reshape(rows, inner // qk * bb)
    return _BIG_CACHE[key]


@pytest.mark.parametrize("batch", [1, 4, 16, 128])
@pytest.mark.parametrize("shape", CONFIG2_BIG, ids=[f"{o}x{i}" for o, i in CONFIG2_BIG])
@pytest.mark.parametrize("t", TYPES[:5], ids=[S.TYPE_NAME[t] for t in TYPES[:5]])
def test_gemv_parity_config2(t, shape, batch):
    rows, inner = shape
    if batch == 128 and shape != (12288, 4096):
        pytest.skip("batch 128 runs on the 12288x4096 shape only")
    q = _big_matrix(t, rows, inner)
    x = np.random.default_rng(50 + batch).standard_normal((batch, inner)).astype(np.float32)
    ref = O.gemv(t, q, x, inner, rows)
    dW, dx = _dev(q), _dev(x)
    dy = _dev(np.full((batch, rows), np.nan, np.float32))
    call("inferno_gemv", t, C.c_void_p(dW.data_ptr()), C.c_void_p(dx.data_ptr()), C.c_void_p(dy.data_ptr()),
         inner, rows, batch, _stream())
    _sync()
    got = dy.cpu().numpy()
    # batch >= 16 of Q4_K / Q5_K / Q6_K / Q8_0 runs on the tcgen05 GEMM (fp16
    # hi/lo operands, fp32 tensor-core accumulation): TC_RTOL
    tol = TC_RTOL if (batch >= 16 and t != S.IQ2_XXS) else GEMV_RTOL
    for v in range(batch):
        assert _rel(got[v], ref[v]) < tol, (v, _rel(got[v], ref[v]))


@pytest.mark.parametrize("force_r", [1, 2, 4])
def test_gemv_rows_per_warp(force_r):
    rows, inner, t = 777, 2048, S.Q4_K
    q = _matrix(t, rows, inner, 4)
    x = np.random.default_rng(5).standard_normal((1, inner)).astype(np.float32)
    ref = O.gemv(t, q, x, inner, rows)
    dW, dx = _dev(q), _dev(x)
    dy = _dev(np.zeros(rows, np.float32))
    call("inferno_gemv_ex", t, C.c_void_p(dW.data_ptr()), C.c_void_p(dx.data_ptr()), C.c_void_p(dy.data_ptr()),
         inner, rows, 1, 0, None, C.c_float(0), 0, None, force_r, _stream())
    _sync()
    assert _rel(dy.cpu().numpy(), ref[0]) < GEMV_RTOL


def test_gemv_rmsnorm_residual_argmax():
    rows, inner, t = 5000, 1024, S.Q6_K
    q = _matrix(t, rows, inner, 6)
    rng = np.random.default_rng(7)
    x = rng.standard_normal(inner).astype(np.float32)
    w = (1 + 0.02 * rng.standard_normal(inner)).astype(np.float32)
    ss = np.float32((x.astype(np.float32) ** 2).sum())
    xn = x * (np.float32(1) / np.sqrt(ss / np.float32(inner) + np.float32(1e-6))) * w
    ref = O.gemv(t, q, xn[None], inner, rows)[0]
    dW, dx, dw = _dev(q), _dev(x), _dev(w)
    # residual epilogue: y starts at 1.0
    dy = _dev(np.ones(rows, np.float32))
    call("inferno_gemv_ex", t, C.c_void_p(dW.data_ptr()), C.c_void_p(dx.data_ptr()), C.c_void_p(dy.data_ptr()),
         inner, rows, 1, 1, C.c_void_p(dw.data_ptr()), C.c_float(1e-6), 1, None, 0, _stream())
    _sync()
    assert _rel(dy.cpu().numpy() - 1.0, ref) < 1e-4
    # argmax epilogue (first max), logits stored as well
    dl = _dev(np.zeros(rows, np.float32))
    am = _dev(np.zeros(1, np.uint64))
    call("inferno_gemv_ex", t, C.c_void_p(dW.data_ptr()), C.c_void_p(dx.data_ptr()), C.c_void_p(dl.data_ptr()),
         inner, rows, 1, 1, C.c_void_p(dw.data_ptr()), C.c_float(1e-6), 3, C.c_void_p(am.data_ptr()), 0, _stream())
    _sync()
    logits = dl.cpu().numpy()
    key = int(am.cpu().numpy().view(np.uint64)[0])
    idx = 0xFFFFFFFF - (key & 0xFFFFFFFF)
    assert idx == int(np.argmax(logits))
    assert idx == int(np.argmax(ref)) or abs(ref[idx] - ref.max()) < 1e-5 * np.abs(ref).max()


def test_gemv_argmax_first_max_tie():
    # identical rows -> identical logits: the first index must win
    # (tests/unit/test_engine.jl:45-79)
    inner, t = 1024, S.Q8_0
    row = _matrix(t, 1, inner, 8)
    q = np.repeat(row, 300, axis=0)
    x = np.random.default_rng(9).standard_normal(inner).astype(np.float32)
    dW, dx = _dev(q), _dev(x)
    am = _dev(np.zeros(1, np.uint64))
    call("inferno_gemv_ex", t, C.c_void_p(dW.data_ptr()), C.c_void_p(dx.data_ptr()), None,
         inner, 300, 1, 0, None, C.c_float(0), 3, C.c_void_p(am.data_ptr()), 0, _stream())
    _sync()
    key = int(am.cpu().numpy().view(np.uint64)[0])
    assert 0xFFFFFFFF - (key & 0xFFFFFFFF) == 0


def test_gemv_swiglu():
    rows, inner, t = 3584, 1024, S.Q4_K
    g, u = _matrix(t, rows, inner, 10), _matrix(t, rows, inner, 11)
    x = np.random.default_rng(12).standard_normal(inner).astype(np.float32)
    rg, ru = O.gemv(t, g, x[None], inner, rows)[0], O.gemv(t, u, x[None], inner, rows)[0]
    ref = rg / (1 + np.exp(-rg)) * ru
    dg, du, dx = _dev(g), _dev(u), _dev(x)
    dh = _dev(np.zeros(rows, np.float32))
    call("inferno_gemv_swiglu", t, C.c_void_p(dg.data_ptr()), C.c_void_p(du.data_ptr()), C.c_void_p(dx.data_ptr()),
         C.c_void_p(dh.data_ptr()), inner, rows, 1, None, C.c_float(0), _stream())
    _sync()
    assert _rel(dh.cpu().numpy(), ref) < 1e-4


@pytest.mark.parametrize("t", [S.Q4_K, S.Q5_K, S.Q6_K, S.Q8_0])
@pytest.mark.parametrize("numerics", ["reference", "fp32"])
def test_compat_tier_host_pointers(t, numerics, monkeypatch):
    """q*_gemv with host pointers (the QuantizedKernels.jl ccall signature).
    Default: the replaced library's numerics (Q8_K activations, AVX2 lane
    order), bit-identical to its restatement; INFERNO_COMPAT_FP32=1: fp32
    activations through the engine's GEMV."""
    rows, inner = 1024, 2048
    q = _matrix(t, rows, inner, 13)
    x = np.random.default_rng(14).standard_normal(inner).astype(np.float32)
    y = np.zeros(rows, np.float32)
    if numerics == "fp32":
        monkeypatch.setenv("INFERNO_COMPAT_FP32", "1")
        ref = O.gemv(t, q, x[None], inner, rows)[0]
    else:
        monkeypatch.delenv("INFERNO_COMPAT_FP32", raising=False)
        ref = O.ref_numerics_gemv(t, q, x, inner, rows)
    P = C.c_void_p
    for _ in range(2):   # second call hits the weight cache
        if t == S.Q8_0:
            lib().q8_0_gemv(P(q.ctypes.data), P(x.ctypes.data), P(y.ctypes.data), inner, rows)
        else:
            fn = {S.Q4_K: lib().q4_k_gemv, S.Q5_K: lib().q5_k_gemv, S.Q6_K: lib().q6_k_gemv}[t]
            fn(P(q.ctypes.data), P(x.ctypes.data), P(y.ctypes.data), None, inner, rows)
        if numerics == "fp32":
            assert _rel(y, ref) < GEMV_RTOL
        else:
            assert np.array_equal(y.view(np.uint32), ref.view(np.uint32))


# ---- batched tensor-core path (prefill chunks): several columns per launch ----
def _rms_ref(x, w, eps=np.float32(1e-6)):
    ss = (x.astype(np.float32) ** 2).sum(axis=-1, keepdims=True).astype(np.float32)
    return (x * (np.float32(1) / np.sqrt(ss / np.float32(x.shape[-1]) + eps)) * w).astype(np.float32)


@pytest.mark.parametrize("t", [S.Q4_K, S.Q6_K], ids=["Q4_K", "Q6_K"])
@pytest.mark.parametrize("batch", [2, 8, 11])
@pytest.mark.parametrize("shape", [(1024, 1024), (6144, 1024), (1024, 3584), (100, 2048)],
                         ids=["1024x1024", "6144x1024", "1024x3584", "100x2048"])
def test_gemv_batch_rmsnorm_residual(t, batch, shape):
    """RMSNorm prologue + residual epilogue over `batch` columns (the prefill
    GEMVs): every column against the fp32 oracle of its own normalised input."""
    rows, inner = shape
    q = _matrix(t, rows, inner, 31)
    rng = np.random.default_rng(32)
    x = (rng.standard_normal((batch, inner)) * rng.uniform(0.1, 10, (batch, 1))).astype(np.float32)
    w = (1 + 0.02 * rng.standard_normal(inner)).astype(np.float32)
    ref = O.gemv(t, q, _rms_ref(x, w), inner, rows)
    y0 = rng.standard_normal((batch, rows)).astype(np.float32)
    dW, dx, dw, dy = _dev(q), _dev(x), _dev(w), _dev(y0)
    call("inferno_gemv_ex", t, C.c_void_p(dW.data_ptr()), C.c_void_p(dx.data_ptr()), C.c_void_p(dy.data_ptr()),
         inner, rows, batch, 1, C.c_void_p(dw.data_ptr()), C.c_float(1e-6), 1, None, 0, _stream())
    _sync()
    got = dy.cpu().numpy() - y0
    for v in range(batch):
        assert _rel(got[v], ref[v]) < 1e-4, (v, _rel(got[v], ref[v]))


@pytest.mark.parametrize("batch", [3, 8])
def test_gemv_batch_swiglu(batch):
    rows, inner, t = 3584, 1024, S.Q4_K
    g, u = _matrix(t, rows, inner, 33), _matrix(t, rows, inner, 34)
    x = np.random.default_rng(35).standard_normal((batch, inner)).astype(np.float32)
    rg, ru = O.gemv(t, g, x, inner, rows), O.gemv(t, u, x, inner, rows)
    ref = rg / (1 + np.exp(-rg)) * ru
    dg, du, dx = _dev(g), _dev(u), _dev(x)
    dh = _dev(np.zeros((batch, rows), np.float32))
    call("inferno_gemv_swiglu", t, C.c_void_p(dg.data_ptr()), C.c_void_p(du.data_ptr()), C.c_void_p(dx.data_ptr()),
         C.c_void_p(dh.data_ptr()), inner, rows, batch, None, C.c_float(0), _stream())
    _sync()
    got = dh.cpu().numpy()
    for v in range(batch):
        assert _rel(got[v], ref[v]) < 1e-4


def test_gemv_batch_nonfinite_column_is_isolated():
    """A NaN in one column makes that column's outputs NaN and leaves the others exact."""
    rows, inner, t, batch = 512, 1024, S.Q4_K, 8
    q = _matrix(t, rows, inner, 36)
    x = np.random.default_rng(37).standard_normal((batch, inner)).astype(np.float32)
    x[3, 17] = np.nan
    dW, dx = _dev(q), _dev(x)
    dy = _dev(np.zeros((batch, rows), np.float32))
    call("inferno_gemv", t, C.c_void_p(dW.data_ptr()), C.c_void_p(dx.data_ptr()), C.c_void_p(dy.data_ptr()),
         inner, rows, batch, _stream())
    _sync()
    got = dy.cpu().numpy()
    assert np.isnan(got[3]).all()
    ok = [v for v in range(batch) if v != 3]
    ref = O.gemv(t, q, x[ok], inner, rows)
    assert _rel(got[ok], ref) < GEMV_RTOL


# ---- Q8_K helpers of the compatibility tier vs the oracle (bit-exact) -------
def test_compat_quantize_row_q8k_bitwise():
    rng = np.random.default_rng(21)
    for n, scale in ((256, 1.0), (4096, 1e-3), (65536, 30.0)):
        x = (rng.standard_normal(n) * scale).astype(np.float32)
        x[256:512] = 0.0 if n > 256 else x[256:512]
        y = np.zeros(n // 256 * O.Q8K_BYTES, np.uint8)
        lib().quantize_row_q8_K(x.ctypes.data, y.ctypes.data, n)
        assert np.array_equal(y, O.quantize_q8k(x))


@pytest.mark.parametrize("t", [S.Q4_K, S.Q5_K, S.Q6_K, S.Q8_0])
def test_compat_vec_dot_bitwise(t):
    from q8k_cases import random_blocks, random_q8k
    rng = np.random.default_rng(100 + t)
    fn = {S.Q4_K: lib().vec_dot_q4_K_q8_K, S.Q5_K: lib().vec_dot_q5_K_q8_K, S.Q6_K: lib().vec_dot_q6_K_q8_K,
          S.Q8_0: lib().vec_dot_q8_0_q8_0}[t]
    for nb in [1, 2, 31, 32, 33, 64, 200] + [int(v) for v in rng.integers(1, 100, 40)]:
        x = random_blocks(rng, t, nb)
        y = random_blocks(rng, S.Q8_0, nb) if t == S.Q8_0 else random_q8k(rng, nb)
        a = np.float32(fn(x.ctypes.data, y.ctypes.data, nb))
        b = np.float32(O.vec_dot_q8k(t, x, y, nb))
        assert a.view(np.uint32) == b.view(np.uint32), (nb, a, b)
