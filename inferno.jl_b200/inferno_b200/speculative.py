"""Speculative decoding with a draft model over two engines: the host loop of
Inferno.jl's SpeculativeDecoding.jl (speculate_and_verify,
src/SpeculativeDecoding.jl:37-112) with the engines doing every forward pass.

Token ids are 0-based here (the reference's are 1-based); the draft model's
gamma tokens are sampled one at a time (draft.forward at successive
positions), the target runs [last prompt token, drafts...] at position - 1
with every position's logits (Model.forward_all), and each draft is accepted
with probability min(1, p_target / p_draft); on the first rejection a token is
drawn from the residual max(p_target - p_draft, 0) (the reference subtracts
the draft token's probability from every entry) and the step ends; if all
gamma drafts are accepted one more token is sampled from the last position.
"""
from __future__ import annotations

import numpy as np


def softmax_sample(logits, rng, temperature=1.0, top_p=1.0, top_k=0):
    """softmax_sample (src/ModelCPU.jl:1123-1170) on the host: temperature 0
    is argmax; top-k by logit, softmax, top-p by cumulative probability."""
    logits = np.asarray(logits, dtype=np.float32)
    if temperature == 0.0:
        return int(np.argmax(logits))
    if temperature != 1.0:
        logits = logits / np.float32(temperature)
    if top_k > 0:
        keep = np.argsort(-logits, kind="stable")[:min(top_k, logits.size)]
        masked = np.full_like(logits, -np.inf)
        masked[keep] = logits[keep]
        logits = masked
    e = np.exp(logits - logits.max())
    probs = e / e.sum()
    if top_p < 1.0:
        order = np.argsort(-probs, kind="stable")
        c = np.cumsum(probs[order])
        n = int(np.searchsorted(c, np.float32(top_p))) + 1
        mask = np.zeros_like(probs)
        mask[order[:n]] = 1
        probs = probs * mask
        probs = probs / probs.sum()
    return sample_from_probs(probs, rng)


def sample_from_probs(probs, rng):
    """sample_from_probs (src/SpeculativeDecoding.jl:21-30): first index whose
    running sum reaches the uniform draw."""
    r = np.float32(rng.random())
    c = np.cumsum(np.asarray(probs, dtype=np.float32))
    i = int(np.searchsorted(c, r))
    return min(i, len(probs) - 1)


def _log_softmax(v):
    v = v - v.max()
    return v - np.log(np.exp(v).sum())


def speculate_and_verify(draft, target, prompt_tokens, position, gamma, rng, temperature=1.0, top_p=1.0,
                         top_k=0):
    """One speculative step (src/SpeculativeDecoding.jl:37-112).  `draft` and
    `target` are Models whose states hold the sequence up to position - 1
    (the last prompt token is fed again by both, as in the reference).
    Returns (accepted tokens, count, target logits [gamma + 1][vocab])."""
    prompt_tokens = [int(t) for t in prompt_tokens]
    draft_tokens, draft_logprobs = [], []
    pos = position
    for _ in range(gamma):
        inp = prompt_tokens[-1] if not draft_tokens else draft_tokens[-1]
        _, logits = draft.forward_all([inp], pos, want_logits=True)
        lv = logits[0]
        nxt = softmax_sample(lv, rng, temperature, top_p, top_k)
        draft_tokens.append(nxt)
        draft_logprobs.append(float(_log_softmax(lv.astype(np.float64))[nxt]))
        pos += 1
    full = [prompt_tokens[-1]] + draft_tokens
    _, tl = target.forward_all(full, position - 1, want_logits=True)
    accepted = []
    for i, tok in enumerate(draft_tokens):
        z = tl[i].astype(np.float32) - tl[i].max()
        tp = np.exp(z) / np.exp(z).sum()
        dp = np.float32(np.exp(draft_logprobs[i]))
        ratio = min(1.0, float(tp[tok] / dp))
        if rng.random() < ratio:
            accepted.append(tok)
        else:
            resid = np.maximum(tp - dp, 0)
            resid = resid / resid.sum()
            accepted.append(sample_from_probs(resid, rng))
            break
    if len(accepted) == gamma:
        accepted.append(softmax_sample(tl[-1], rng, temperature, top_p, top_k))
    return accepted, len(accepted), tl
