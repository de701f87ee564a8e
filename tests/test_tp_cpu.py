"""Tensor-parallel sharding on the CPU: N ranks simulated in one process with
the numpy restatement of the reference layer (tests/numpy_ref.py).  For every
layer the sum over ranks of the sharded GDN / attention / FFN partials must
equal the unsharded sublayer (the engine sums them with one all-reduce of the
residual stream per sublayer)."""
import numpy as np
import pytest

from inferno_b200 import synth as S
from inferno_b200 import tp
from numpy_ref import NumpyModel


def _layers_match(spec, T, n, steps=3):
    full = NumpyModel(spec, T)
    parts = [NumpyModel(*tp.shard(spec, T, r, n)) for r in range(n)]
    rng = np.random.default_rng(5)
    for pos in range(steps):
        x = rng.standard_normal(spec.hidden)
        for i in range(spec.layers):
            p = f"blk.{i}."
            W = full.W
            xn = full.rms(x, W[p + "attn_norm.weight"])
            if spec.is_attn(i):
                want = full.attn(i, xn, pos)
                got = sum(m.attn(i, xn, pos) for m in parts)
            else:
                want = full.gdn(i, xn)
                got = sum(m.gdn(i, xn) for m in parts)
            assert np.abs(got - want).max() <= 1e-9 * max(1.0, np.abs(want).max()), (i, pos)
            x1 = x + want
            xn2 = full.rms(x1, W[p + "post_attention_norm.weight"])

            def ffn(m):
                g = m.W[p + "ffn_gate.weight"] @ xn2
                u = m.W[p + "ffn_up.weight"] @ xn2
                return m.W[p + "ffn_down.weight"] @ (g / (1 + np.exp(-g)) * u)
            want_f, got_f = ffn(full), sum(ffn(m) for m in parts)
            assert np.abs(got_f - want_f).max() <= 1e-9 * max(1.0, np.abs(want_f).max()), (i, pos)
            x = x1 + want_f


def test_tp2_tiny_layers_sum_to_unsharded():
    spec = S.CONFIGS["tiny-tp"]
    _layers_match(spec, S.make_model(spec, seed=31), 2)


@pytest.mark.parametrize("n", [2, 4, 8])
def test_tp_small_layers_sum_to_unsharded(n):
    spec = S.CONFIGS["small-tp"]
    _layers_match(spec, S.make_model(spec, seed=32, layers=4), n, steps=2)


def test_local_head_order_keeps_modulo_map():
    spec = S.CONFIGS["qwen35-9b"]
    for n in (2, 4, 8):
        ls = tp.local_spec(spec, n)
        seen = []
        for r in range(n):
            heads = tp.gdn_local_heads(spec, r, n)
            for hl, h in enumerate(heads):
                # local group of local head == local index of the global group
                assert hl % ls.ssm_nk == (h % spec.ssm_nk) - r * ls.ssm_nk
            seen += heads
        assert sorted(seen) == list(range(spec.ssm_nv))


def test_unsplittable_shapes_are_rejected():
    with pytest.raises(ValueError):
        tp.check(S.CONFIGS["tiny"], 2)            # 2 QK groups -> 128-column runs
    with pytest.raises(ValueError):
        tp.check(S.CONFIGS["qwen35-9b"], 16)
    with pytest.raises(ValueError):
        tp.check(S.CONFIGS["tiny-moe"], 2)


def test_expert_shards_cover_every_expert_once():
    spec = S.CONFIGS["tiny-moe"]
    T = S.make_model(spec, seed=33)
    for n in (2, 4):
        parts = [tp.shard(spec, T, r, n)[1] for r in range(n)]
        for name, t in T.items():
            if name.endswith("_exps.weight"):
                joined = np.concatenate([p[name].data for p in parts])
                assert np.array_equal(joined, t.data), name
                assert all(p[name].ne[2] == spec.n_experts // n for p in parts)
            else:
                assert all(p[name] is t for p in parts), name


@pytest.mark.parametrize("n", [2, 4, 8])
def test_config4_splits_as_planned(n):
    """The 9B shape over 2 / 4 / 8 ranks: QK groups, V heads (modulo map),
    query heads, KV heads (replicated once N exceeds them), FFN columns in
    whole super-blocks, vocab rows of the lm_head."""
    spec = S.CONFIGS["qwen35-9b"]
    tp.check(spec, n)
    ls = tp.local_spec(spec, n)
    assert ls.ssm_nk == 16 // n and ls.ssm_nv == 32 // n
    assert ls.n_heads == 16 // n
    assert ls.n_kv == (4 // n if n <= 4 else 1)
    assert ls.ffn == 12288 // n and ls.ffn % 256 == 0
    assert spec.vocab % n == 0
    heads = sorted(h for r in range(n) for h in tp.gdn_local_heads(spec, r, n))
    assert heads == list(range(spec.ssm_nv))
    # every rank's ssm_out column runs are super-block aligned
    nk_l = spec.ssm_nk // n
    assert (nk_l * spec.ssm_dv) % 256 == 0


@pytest.mark.parametrize("n", [2, 4, 8])
def test_config5_expert_split(n):
    spec = S.CONFIGS["qwen35-35b-a3b"]
    assert spec.n_experts % n == 0
    with pytest.raises(ValueError):
        tp.check(spec, n)                       # MoE layers are expert-parallel, not tensor-parallel
