"""GPU parity of the gated decode-attention step (inferno_attention_step,
the part of FullAttentionCPU after the q/k/v projections,
src/ModelCPU.jl:766-851 with flash_attention_cpu!, src/FlashAttention.jl:16-74)
against the oracle's restatement, through the C ABI.

Sizes: the reference's own verification sweep
(tests/flash_attention_verification.jl:55-101: head_dim 256, 2 KV heads,
sequence lengths 32..2048, seed 42, uniform [0, 1) queries and caches) and
the config-4 geometry (16 query / 4 KV heads, max_ctx 32896 -> 288 positions
per split, 115 splits) at positions 300, 4096 and 32000."""
import ctypes as C

import numpy as np
import pytest

import oracle as O
from inferno_b200._lib import call, lib

pytestmark = pytest.mark.gpu

HD = 256
ATT_RTOL = 1e-4        # max|out - ref| / max|ref| (the reference sweep's 1e-4 bound)


def _dev(a):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def _stream():
    import torch
    return C.c_void_p(torch.cuda.current_stream().cuda_stream)


def _case(seed, nh, nkv, ctx, pos):
    rng = np.random.default_rng(seed)
    qg = rng.random((nh, 2 * HD), dtype=np.float32)
    qg[:, HD:] = rng.standard_normal((nh, HD)).astype(np.float32)      # gate logits
    k = rng.random((nkv, HD), dtype=np.float32)
    v = rng.random((nkv, HD), dtype=np.float32)
    qn = (1 + 0.02 * rng.standard_normal(HD)).astype(np.float32)
    kn = (1 + 0.02 * rng.standard_normal(HD)).astype(np.float32)
    kc = np.zeros((ctx, nkv, HD), np.float32)
    vc = np.zeros((ctx, nkv, HD), np.float32)
    kc[:pos] = rng.random((pos, nkv, HD), dtype=np.float32)
    vc[:pos] = rng.random((pos, nkv, HD), dtype=np.float32)
    return qg, k, v, qn, kn, kc, vc


def _run(nh, nkv, ctx, pos, split_len=0, seed=42, rd=64, theta=1e7, eps=1e-6):
    qg, k, v, qn, kn, kc, vc = _case(seed, nh, nkv, ctx, pos)
    d = [_dev(a) for a in (qg, k, v, qn, kn)]
    dkc, dvc = _dev(kc), _dev(vc)
    dout = _dev(np.full(nh * HD, np.nan, np.float32))
    P = lambda t: C.c_void_p(t.data_ptr())
    call("inferno_attention_step", *[P(t) for t in d], C.c_float(eps), nh, nkv, HD, rd, C.c_float(theta),
         P(dkc), P(dvc), ctx, pos, split_len, P(dout), _stream())
    assert lib().inferno_device_error(0, 1) == 0
    ref = O.attention_step(qg, k, v, qn, kn, eps, nh, nkv, HD, rd, theta, kc, vc, pos)
    got = dout.cpu().numpy()
    return got, ref, dkc.cpu().numpy(), dvc.cpu().numpy(), kc, vc


def _rel(a, b):
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-30))


@pytest.mark.parametrize("seq", [32, 64, 128, 256, 512, 1024, 2048])
def test_attention_reference_sweep(seq):
    """flash_attention_verification.jl sizes: 2 KV heads (4 query heads, GQA 2),
    the new row at position seq-1, a 2048-position cache."""
    got, ref, gk, gv, kc, vc = _run(nh=4, nkv=2, ctx=2048, pos=seq - 1)
    assert _rel(got, ref) < ATT_RTOL, _rel(got, ref)
    # the appended K row is the normalised, rotated key; V is stored as is
    assert _rel(gk[seq - 1], kc[seq - 1]) < 1e-5
    assert np.array_equal(gv[seq - 1], vc[seq - 1])
    assert np.array_equal(gk[: seq - 1], kc[: seq - 1])


@pytest.mark.parametrize("pos", [300, 4096, 32000])
def test_attention_config4_geometry(pos):
    """16 Q / 4 KV heads, max_ctx 32896: 288 positions per split (115 splits)."""
    got, ref, *_ = _run(nh=16, nkv=4, ctx=32896, pos=pos, seed=7 + pos)
    assert _rel(got, ref) < ATT_RTOL, _rel(got, ref)


@pytest.mark.parametrize("split_len", [32, 96, 288])
def test_attention_split_lengths_agree(split_len):
    """The split-K merge gives the oracle's result for any split length."""
    got, ref, *_ = _run(nh=8, nkv=2, ctx=4096, pos=1500, split_len=split_len, seed=11)
    assert _rel(got, ref) < ATT_RTOL, _rel(got, ref)


@pytest.mark.parametrize("nh,nkv,ctx,pos", [(4, 2, 2048, 1023), (16, 4, 32896, 300), (16, 4, 32896, 32000),
                                            (16, 2, 4096, 1500)])
def test_attention_gqa_grouped_variant(monkeypatch, nh, nkv, ctx, pos):
    """The GQA-grouped kernel (one CTA per KV head for its 2 / 4 / 8 query
    heads, INFERNO_ATT_GROUPED=1) gives the oracle's result and the same bits
    as the one-CTA-per-query-head kernel."""
    monkeypatch.setenv("INFERNO_ATT_GROUPED", "1")
    got, ref, gk, *_ = _run(nh=nh, nkv=nkv, ctx=ctx, pos=pos, seed=5)
    monkeypatch.setenv("INFERNO_ATT_GROUPED", "0")
    got0, _, gk0, *_ = _run(nh=nh, nkv=nkv, ctx=ctx, pos=pos, seed=5)
    assert _rel(got, ref) < ATT_RTOL, _rel(got, ref)
    assert np.array_equal(got, got0)
    assert np.array_equal(gk, gk0)


def test_attention_position_zero_and_bad_args():
    got, ref, *_ = _run(nh=8, nkv=2, ctx=64, pos=0, seed=3)
    assert _rel(got, ref) < ATT_RTOL
    z = _dev(np.zeros(16 * 2 * HD, np.float32))
    P = C.c_void_p(z.data_ptr())
    args = [P] * 5 + [C.c_float(1e-6), 8, 2, HD, 64, C.c_float(1e7), P, P, 64]
    assert lib().inferno_attention_step(*args, 64, 0, P, _stream()) < 0        # pos == max_ctx
    assert lib().inferno_attention_step(*args, 3, 40, P, _stream()) < 0        # split not a multiple of 32
    args[8] = 128                                                               # head_dim != 256
    assert lib().inferno_attention_step(*args, 3, 0, P, _stream()) < 0
