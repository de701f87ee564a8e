"""Batched decode (inferno_decode_batch): B sequences with their own prompts,
KV caches and recurrent states decoded in lockstep must each reproduce the
oracle's greedy tokens for that sequence alone (and the engine's own
single-sequence decode).  B = 3 and 5 run the batched GEMV path, B = 17 the
tensor-core GEMM; prompts have different lengths, so the sequences sit at
different positions."""
import numpy as np
import pytest

import oracle as O
from inferno_b200 import synth as S
from inferno_b200.model import Model

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def tiny():
    spec = S.CONFIGS["tiny"]
    T = S.make_model(spec, seed=41)
    return spec, T, O.OracleModel(spec, T)


@pytest.mark.parametrize("B", [3, 5, 17])
def test_decode_batch_matches_oracle_per_sequence(tiny, B):
    spec, T, orc = tiny
    n = 12
    m = Model(spec, T, max_batch=B)
    m.reset()
    toks, pos, want = [], [], []
    for b in range(B):
        prompt = S.tokens(100 + b, 3 + 2 * b % 11, spec.vocab)
        m.select_sequence(b)
        first, _ = m.forward(prompt, 0, want_logits=False)
        toks.append(first)
        pos.append(len(prompt))
        ref = orc.generate(prompt, n + 1)          # [first, then n greedy tokens]
        assert ref[0] == first
        want.append(ref[1:])
    out = m.decode_batch(toks, pos, n)
    m.close()
    for b in range(B):
        assert out[:, b].tolist() == want[b], b


def test_decode_batch_moe_matches_oracle_per_sequence():
    """tiny-moe at B = 4: every sequence's token routes to its own experts."""
    spec = S.CONFIGS["tiny-moe"]
    T = S.make_model(spec, seed=43)
    orc = O.OracleModel(spec, T)
    B, n = 4, 10
    m = Model(spec, T, max_batch=B)
    m.reset()
    toks, pos, want = [], [], []
    for b in range(B):
        prompt = S.tokens(200 + b, 4 + 3 * b, spec.vocab)
        m.select_sequence(b)
        first, _ = m.forward(prompt, 0, want_logits=False)
        toks.append(first)
        pos.append(len(prompt))
        ref = orc.generate(prompt, n + 1)
        assert ref[0] == first
        want.append(ref[1:])
    out = m.decode_batch(toks, pos, n)
    m.close()
    for b in range(B):
        assert out[:, b].tolist() == want[b], b
