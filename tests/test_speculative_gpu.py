"""Speculative / multi-token verification on the engine against the oracle:
every-position logits (inferno_forward_tokens_all, the full_logits forward of
mtp_verify_step!, src/ModelCPU.jl:1914-1930), the verify step's accepted
count, and speculate_and_verify (src/SpeculativeDecoding.jl:37-112) with a
draft model."""
import numpy as np
import pytest

import oracle as O
from inferno_b200 import synth as S
from inferno_b200.model import Model
from inferno_b200.speculative import speculate_and_verify

pytestmark = pytest.mark.gpu


def rel(a, b):
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-30))


@pytest.fixture(scope="module")
def tiny():
    spec = S.CONFIGS["tiny"]
    T = S.make_model(spec, seed=31)
    return spec, T, O.OracleModel(spec, T)


def test_forward_all_matches_oracle_token_loop(tiny):
    spec, T, orc = tiny
    prompt = S.tokens(31, 10, spec.vocab)
    toks = S.tokens(32, 6, spec.vocab)
    m = Model(spec, T)
    m.reset()
    m.forward(prompt, 0, want_logits=False)
    am, lg = m.forward_all(toks, len(prompt))
    m.close()
    orc.reset()
    orc.forward(prompt, 0, want_logits=False)
    for i, t in enumerate(toks):
        a_o, l_o = orc.forward([int(t)], len(prompt) + i)
        assert int(am[i]) == a_o
        assert rel(lg[i], l_o) < 2e-3


def test_mtp_verify_step_accepted_count(tiny):
    """Drafts = the oracle's greedy continuation with the 4th token replaced:
    the first three drafts after the fed token are accepted, then it stops."""
    spec, T, orc = tiny
    prompt = S.tokens(33, 9, spec.vocab)
    want = orc.generate(prompt, 7)                 # greedy continuation (first = argmax after the prompt)
    draft = [want[0]] + want[1:6]
    draft[4] = (draft[4] + 1) % spec.vocab          # wrong token at index 4
    m = Model(spec, T)
    m.reset()
    m.forward(prompt, 0, want_logits=False)
    acc, logits = m.mtp_verify_step(draft, len(prompt))
    m.close()
    assert logits.shape == (len(draft), spec.vocab)
    assert acc == 3


def test_speculate_and_verify_same_model_accepts_every_draft(tiny):
    """Draft model == target model: every acceptance ratio is 1, so all gamma
    drafts are kept and one more token is sampled (gamma + 1)."""
    spec, T, _ = tiny
    prompt = [int(t) for t in S.tokens(34, 8, spec.vocab)]
    draft, target = Model(spec, T), Model(spec, T)
    for m in (draft, target):
        m.reset()
        m.forward(prompt[:-1], 0, want_logits=False)
    rng = np.random.default_rng(5)
    acc, n, tl = speculate_and_verify(draft, target, prompt, len(prompt), gamma=4, rng=rng, temperature=1.0)
    draft.close()
    target.close()
    assert n == 5 and len(acc) == 5
    assert tl.shape == (5, spec.vocab)
    assert all(0 <= t < spec.vocab for t in acc)
