"""CPU tests of the oracle (test infrastructure): pinned against the
reference's known-answer tests, against gguf-py golden vectors, and against an
independent numpy restatement of the forward pass."""
import math
import os
from pathlib import Path

import numpy as np
import pytest

import oracle as O
from inferno_b200 import synth as S

GOLDEN = Path(__file__).resolve().parent / "golden" / "dequant_golden.npz"
# the reference source tree (INFERNO_REFERENCE_ROOT, else a checkout beside
# this repository); tests that read it skip when it is absent
REF_ROOT = Path(os.environ.get("INFERNO_REFERENCE_ROOT", Path(__file__).resolve().parents[2] / "reference"))
REF_QUANTSDATA = REF_ROOT / "src" / "QuantsData.jl"


# ---- tests/unit/core_components.jl:114-122 (IQ2_XXS known answers) --------
def test_iq2xxs_known_answers():
    data = np.zeros(66, np.uint8)
    data[1] = 0x3C                     # d = 1.0
    y = O.dequant(S.IQ2_XXS, data, 256)
    assert np.all(y == 0)
    data[2] = 0x01                     # grid[1] = 0x08...082b
    y = O.dequant(S.IQ2_XXS, data, 256)
    assert y[0] == np.float32(4.375)   # (43 - 8) * 0.125
    assert np.all(y[1:8] == 0)


def test_iq2xxs_grid_matches_reference_source():
    if not REF_QUANTSDATA.exists():
        pytest.skip("reference tree not present")
    import importlib.util
    spec = importlib.util.spec_from_file_location(
        "gen", Path(__file__).resolve().parent.parent / "inferno.jl_b200" / "csrc" / "gen_iq2xxs_grid.py")
    gen = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(gen)
    ref = np.array(gen.extract(REF_QUANTSDATA.read_text()), dtype=np.uint64)
    assert np.array_equal(ref, S.IQ2XXS_GRID)


def test_ksigns_table():
    # src/QuantsData.jl:7-16 first row
    assert list(S.KSIGNS[:16]) == [0, 129, 130, 3, 132, 5, 6, 135, 136, 9, 10, 139, 12, 141, 142, 15]


# ---- golden vectors (gguf-py 0.19.0, ggml semantics) ------------------------
@pytest.mark.parametrize("name,t", [("Q8_0", S.Q8_0), ("Q4_K", S.Q4_K), ("Q5_K", S.Q5_K), ("Q6_K", S.Q6_K)])
def test_dequant_bitexact_vs_golden(name, t):
    g = np.load(GOLDEN)
    q, want = g[f"{name}_bytes"], g[f"{name}_ggml"]
    got = O.dequant(t, q, want.size)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


def test_iq2xxs_inferno_semantics_vs_golden():
    g = np.load(GOLDEN)
    q, inf, ggml = g["IQ2_XXS_bytes"], g["IQ2_XXS_inferno"], g["IQ2_XXS_ggml"]
    got = O.dequant(S.IQ2_XXS, q, inf.size)
    assert np.array_equal(got.view(np.uint32), inf.view(np.uint32))
    # Inferno = ggml - 8*db*sign (src/Dequant.jl:46 vs ggml)
    nb = q.size // 66
    d = q.reshape(nb, 66)[:, :2].copy().view(np.float16).astype(np.float32).reshape(nb)
    a2 = q.reshape(nb, 66)[:, 2:].copy().view("<u4").reshape(nb, 8, 2)[..., 1]
    db = (d[:, None] * (0.5 + (a2 >> 28).astype(np.float32))) * 0.25
    sign = np.sign(ggml.reshape(nb, 8, 32))
    off = 8 * db[..., None] * sign
    np.testing.assert_allclose(inf.reshape(nb, 8, 32), ggml.reshape(nb, 8, 32) - off, atol=1e-6)


def test_packers_round_trip():
    rng = np.random.default_rng(1)
    w = (rng.standard_normal((8, 1024)) * 0.02).astype(np.float32)
    for t, tol in ((S.Q8_0, 0.01), (S.Q6_K, 0.03), (S.Q5_K, 0.05), (S.Q4_K, 0.1)):
        d = O.dequant(t, S.quantize(w, t).reshape(-1), w.size).reshape(w.shape)
        assert np.abs(d - w).max() / np.abs(w).max() < tol, S.TYPE_NAME[t]


# ---- tests/flash_attention_verification.jl:55-101 ---------------------------
@pytest.mark.parametrize("seq", [32, 64, 128, 256, 512, 1024, 2048])
def test_flash_vs_standard_attention(seq):
    rng = np.random.default_rng(42)
    hd, nkv = 256, 2
    q = rng.random(hd, dtype=np.float32)
    ck = rng.random((seq, nkv, hd), dtype=np.float32)
    cv = rng.random((seq, nkv, hd), dtype=np.float32)
    scale = np.float32(1.0 / math.sqrt(hd))
    a = O.flash_attention(q, ck, cv, 0, seq, scale, hd, nkv)
    b = O.flash_attention(q, ck, cv, 0, seq, scale, hd, nkv, standard=True)
    assert np.abs(a - b).max() < 1e-4


def test_gemv_matches_dequant_matmul():
    rng = np.random.default_rng(3)
    w = (rng.standard_normal((37, 512)) * 0.02).astype(np.float32)
    for t in (S.Q4_K, S.Q6_K, S.Q8_0, S.IQ2_XXS):
        q = S.quantize(w, t)
        x = rng.standard_normal((2, 512)).astype(np.float32)
        y = O.gemv(t, q, x, 512, 37)
        ref = x.astype(np.float64) @ O.dequant(t, q.reshape(-1), w.size).reshape(w.shape).T.astype(np.float64)
        assert np.abs(y - ref).max() / np.abs(ref).max() < 1e-5


def test_gdn_recurrence_vs_numpy():
    rng = np.random.default_rng(4)
    T, H, dk, dv = 5, 2, 16, 8
    q = rng.standard_normal((T, H, dk)).astype(np.float32)
    k = rng.standard_normal((T, H, dk)).astype(np.float32)
    q /= np.linalg.norm(q, axis=-1, keepdims=True)
    k /= np.linalg.norm(k, axis=-1, keepdims=True)
    v = rng.standard_normal((T, H, dv)).astype(np.float32)
    beta = (1 / (1 + np.exp(-rng.standard_normal((T, H))))).astype(np.float32)
    g = (-np.log1p(np.exp(rng.standard_normal((T, H))))).astype(np.float32)
    S0 = np.zeros((H, dv, dk), np.float32)
    y = O.gdn_recurrence(q, k, v, beta, g, S0)
    Sr = np.zeros((H, dv, dk))
    for t in range(T):
        for h in range(H):
            Sr[h] *= np.exp(g[t, h])
            d = beta[t, h] * (v[t, h] - Sr[h] @ k[t, h])
            Sr[h] += np.outer(d, k[t, h])
            np.testing.assert_allclose(y[t, h], Sr[h] @ q[t, h], rtol=1e-4, atol=1e-5)
    np.testing.assert_allclose(S0, Sr, rtol=1e-4, atol=1e-5)


# ---- the full forward against the numpy restatement -------------------------
@pytest.fixture(scope="module")
def tiny_pair():
    from numpy_ref import NumpyModel
    spec = S.CONFIGS["tiny"]
    T = S.make_model(spec, seed=5)
    return spec, T, O.OracleModel(spec, T), NumpyModel(spec, T)


def test_oracle_forward_vs_numpy(tiny_pair):
    spec, T, orc, ref = tiny_pair
    prompt = S.tokens(5, 6, spec.vocab)
    orc.reset()
    ref.reset()
    a, la = orc.forward(prompt, 0)
    b, lb = ref.forward(prompt, 0)
    assert np.abs(la - lb).max() / np.abs(lb).max() < 1e-4
    assert a == b
    for step in range(3):
        a, la = orc.forward([a], len(prompt) + step)
        b, lb = ref.forward([b], len(prompt) + step)
        assert a == b
        assert np.abs(la - lb).max() / np.abs(lb).max() < 1e-4


def test_oracle_greedy_first_max():
    """Julia argmax returns the first maximum (tests/unit/test_engine.jl:45-79);
    the oracle's argmax scan uses a strict '>' so ties keep the lower index."""
    spec = S.CONFIGS["tiny"]
    T = S.make_model(spec, seed=6)
    e = T["token_embd.weight"]
    row = e.data.reshape(spec.vocab, -1)[0]
    T["token_embd.weight"] = S.Tensor(e.ggml_type, e.ne, np.tile(row, spec.vocab))
    m = O.OracleModel(spec, T)
    tok, lg = m.forward([7], 0)
    assert np.all(lg == lg[0]) and tok == 0


# ---- sampler restatement (src/ModelCPU.jl:1123-1225) -------------------------
def _np_softmax_sample(logits, temperature, top_p=1.0, top_k=0, min_p=0.0, presence=0.0, repetition=1.0,
                       seen=(), r=0.5):
    """Independent numpy statement of generate_cpu's penalties + softmax_sample."""
    l = np.asarray(logits, np.float64).copy()
    for t in set(int(s) for s in seen):
        l[t] -= presence
        if repetition != 1.0:
            l[t] = l[t] / repetition if l[t] > 0 else l[t] * repetition
    if temperature == 0:
        return int(np.argmax(l))
    l = l / temperature
    if top_k > 0:
        keep = np.argsort(-l, kind="stable")[:top_k]
        m = np.full_like(l, -np.inf)
        m[keep] = l[keep]
        l = m
    p = np.exp(l - l.max())
    p /= p.sum()
    if top_p < 1.0:
        order = np.argsort(-p, kind="stable")
        c = np.cumsum(p[order])
        cut = int(np.searchsorted(c, top_p)) + 1
        q = np.zeros_like(p)
        q[order[:cut]] = p[order[:cut]]
        p = q / q.sum()
    if min_p > 0:
        p[p < p.max() * min_p] = 0
        p /= p.sum()
    c = np.cumsum(p)
    i = int(np.searchsorted(c, r))
    return min(i, len(p) - 1)


@pytest.mark.parametrize("kw", [dict(temperature=0.0), dict(temperature=1.0, top_k=1),
                                dict(temperature=0.8, top_k=10), dict(temperature=1.2, top_p=0.7),
                                dict(temperature=0.9, top_k=50, top_p=0.9, min_p=0.1),
                                dict(temperature=1.0, presence=1.5, repetition=1.2, top_k=20)])
def test_oracle_sampler_vs_numpy(kw):
    rng = np.random.default_rng(9)
    agree = 0
    for _ in range(40):
        logits = (rng.standard_normal(2000) * 3).astype(np.float32)
        seen = rng.integers(0, 2000, 30)
        r = float(rng.random())
        a = O.softmax_sample(logits, kw.get("temperature", 1.0), kw.get("top_p", 1.0), kw.get("top_k", 0),
                             kw.get("min_p", 0.0), kw.get("presence", 0.0), kw.get("repetition", 1.0), seen, r)
        b = _np_softmax_sample(logits, seen=seen, r=r, **kw)
        agree += a == b
    assert agree >= 39     # fp32 vs fp64 can move a draw that lands on a boundary


def test_oracle_sampler_first_max_and_ties():
    l = np.array([1, 5, 5, 2], np.float32)
    assert O.softmax_sample(l, 0.0) == 1                       # argmax: first maximum
    assert O.softmax_sample(l, 1.0, top_k=1, r=0.99) == 1      # stable top-k keeps the lower index


# ---- Q8_K activation path of quant_kernels.c, pinned to the reference's own build
from q8k_cases import random_blocks as _random_blocks, random_q8k as _random_q8k


@pytest.fixture(scope="module")
def ref():
    L = O.ref_lib()
    if L is None:
        pytest.skip("oracle/_ref not built (reference sources absent)")
    return L


def test_quantize_q8k_matches_reference_bitwise(ref):
    rng = np.random.default_rng(3)
    for n, scale in ((256, 1.0), (1024, 1e-3), (4096, 50.0)):
        x = (rng.standard_normal(n) * scale).astype(np.float32)
        x[:256] = 0.0 if n == 1024 else x[:256]      # an all-zero block: d = 0, id = 0
        a = O.quantize_q8k(x)
        b = np.zeros_like(a)
        ref.quantize_row_q8_K(O._ptr(x), O._ptr(b), n)
        assert np.array_equal(a, b)


@pytest.mark.parametrize("ggml_type", [12, 13, 14, 8])
def test_vec_dot_matches_reference_bitwise(ref, ggml_type):
    rng = np.random.default_rng(ggml_type)
    fn = {12: ref.vec_dot_q4_K_q8_K, 13: ref.vec_dot_q5_K_q8_K, 14: ref.vec_dot_q6_K_q8_K,
          8: ref.vec_dot_q8_0_q8_0}[ggml_type]
    # 400 draws: enough to separate fused from unfused multiply-adds
    for nb in [1, 3, 4, 16, 57] + list(rng.integers(1, 40, 400)):
        nb = int(nb)
        x = _random_blocks(rng, ggml_type, nb)
        y = _random_blocks(rng, 8, nb) if ggml_type == 8 else _random_q8k(rng, nb)
        a = np.float32(O.vec_dot_q8k(ggml_type, x, y, nb))
        b = np.float32(fn(O._ptr(x), O._ptr(y), nb))
        assert a.view(np.uint32) == b.view(np.uint32), (nb, a, b)


@pytest.mark.parametrize("ggml_type", [12, 13, 14, 8])
def test_ref_numerics_gemv_matches_reference_bitwise(ref, ggml_type):
    """The compatibility tier's default numerics, restated, equal the reference
    library's q*_gemv output bit for bit (quant_kernels.c:602-697)."""
    rng = np.random.default_rng(40 + ggml_type)
    for rows, inner in ((64, 256), (100, 2048), (300, 1024)):
        W = S.random_quant_matrix(rng, rows, inner, ggml_type)
        x = (rng.standard_normal(inner) * 2).astype(np.float32)
        a = O.ref_numerics_gemv(ggml_type, W, x, inner, rows)
        b = O.ref_gemv(ggml_type, W, x, inner, rows, ref)
        assert np.array_equal(a.view(np.uint32), b.view(np.uint32))


# ---- the reference's sampler unit expectations (tests/unit/test_engine.jl:45-227)
# stated for softmax_sample (0-based ids) over a sweep of uniform draws r in
# (0, 1).  (r == 0 exactly -- probability 2^-24 for rand(Float32) -- returns
# index 0 in the reference's `r <= cumsum` walk even when its probability is 0;
# the restatement keeps that, and the sweep leaves it out.)
_RS = [(i + 0.5) / 64 for i in range(64)] + [0.999999]


def _support(logits, **kw):
    return {O.softmax_sample(np.asarray(logits, np.float32), r=r, **kw) for r in _RS}


def test_sampler_reference_argmax_cases():
    """:45-80 temperature 0 = argmax, first occurrence on ties."""
    assert O.softmax_sample(np.float32([1, 5, 2, 4]), 0.0) == 1
    assert O.softmax_sample(np.float32([-10, -5, -1]), 0.0) == 2
    assert O.softmax_sample(np.float32([1, 5, 2, 5]), 0.0) == 1
    assert O.softmax_sample(np.float32([42]), 0.0) == 0
    assert O.softmax_sample(np.float32([3, 3, 3]), 0.0) == 0
    assert O.softmax_sample(np.float32([100, 500, 1000]), 0.0) == 2
    assert O.softmax_sample(np.float32([-1e4, -1e5, -1e3]), 0.0) == 2


def test_sampler_reference_topk_topp_cases():
    """:82-126 and :219-227: top-k / top-p supports."""
    assert _support([1, 10, 2, 9], temperature=0.7, top_k=2) <= {1, 3}
    assert _support([1, 5, 3], temperature=0.7, top_k=1) == {1}
    assert _support([1, 2, 3], temperature=0.5, top_k=100) <= {0, 1, 2}       # k beyond the vocabulary
    assert _support([10, 1, 1, 1], temperature=0.5, top_k=0) <= {0, 1, 2, 3}
    assert _support([1, 100, 2], temperature=0.5, top_p=0.01) == {1}
    s = [O.softmax_sample(np.float32([1, 2, 3, 10]), 0.5, top_p=0.5, r=r) for r in _RS]
    assert s.count(3) > len(s) // 2
    assert _support([1, 10, 2, 9, 3, 8], temperature=0.5, top_p=0.8, top_k=3) <= {1, 3, 5}


def test_sampler_reference_temperature_cases():
    """:128-146: high temperature spreads, low temperature concentrates."""
    assert len(_support([1, 10, 2], temperature=2.0)) >= 2
    low = [O.softmax_sample(np.float32([1, 10, 2]), 0.1, r=r) for r in _RS]
    assert low.count(1) > 0.75 * len(low)
