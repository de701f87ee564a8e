"""GPU parity of the decode engine against the CPU oracle on seeded models:
per-layer hidden states (rel 2e-3), logits, greedy token identity, state
export/import and reset.  All calls go through the C ABI."""
import os

import numpy as np
import pytest

import oracle as O
from inferno_b200 import synth as S
from inferno_b200.model import Model

pytestmark = pytest.mark.gpu

LAYER_RTOL = 2e-3      # per-layer hidden state, max|d| / max|ref| (north_star)
LOGIT_RTOL = 2e-3


def rel(a, b):
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-30))


@pytest.fixture(scope="module")
def tiny():
    spec = S.CONFIGS["tiny"]
    T = S.make_model(spec, seed=11)
    return spec, T, O.OracleModel(spec, T)


@pytest.mark.parametrize("graphs", [True, False])
def test_tiny_generate_matches_oracle(tiny, graphs):
    spec, T, orc = tiny
    prompt = S.tokens(11, 12, spec.vocab)
    m = Model(spec, T, use_graphs=graphs)
    got = m.generate(prompt, 24)
    want = orc.generate(prompt, 24)
    m.close()
    assert got == want


def test_tiny_logits_and_layers(tiny):
    spec, T, orc = tiny
    prompt = S.tokens(12, 9, spec.vocab)
    m = Model(spec, T)
    orc.reset()
    m.reset()
    am_o, lg_o = orc.forward(prompt, 0)
    am_g, lg_g = m.forward(prompt, 0)
    assert rel(lg_g, lg_o) < LOGIT_RTOL
    assert am_g == am_o
    # layer-by-layer on the same input, continuing at the next position
    x = orc.embed(int(am_o))
    for i in range(spec.layers):
        xo = orc.layer(i, x, len(prompt))
        xg = m.layer(i, x, len(prompt))
        assert rel(xg, xo) < LAYER_RTOL, (i, rel(xg, xo))
        x = xo
    m.close()


def test_tiny_dump_hidden(tiny, monkeypatch):
    spec, T, orc = tiny
    monkeypatch.setenv("INFERNO_B200_DUMP", "1")
    m = Model(spec, T)
    prompt = S.tokens(13, 7, spec.vocab)
    orc.reset()
    orc.forward(prompt, 0, want_logits=False)
    m.forward(prompt, 0, want_logits=False)
    for i in range(spec.layers):
        assert rel(m.hidden(i), orc.hidden(i)) < LAYER_RTOL, i
    m.close()


def test_state_export_import_and_reset(tiny):
    spec, T, _ = tiny
    m = Model(spec, T)
    prompt = S.tokens(14, 10, spec.vocab)
    m.reset()
    tok, _ = m.forward(prompt, 0, want_logits=False)
    snap = m.state_export()
    a = m.decode_greedy(tok, len(prompt), 6)
    m.state_import(snap)
    b = m.decode_greedy(tok, len(prompt), 6)
    assert np.array_equal(a, b)
    m.reset()
    t2, _ = m.forward(prompt, 0, want_logits=False)
    assert t2 == tok
    m.close()


def test_errors_are_reported(tiny):
    from inferno_b200._lib import InfernoError
    spec, T, _ = tiny
    m = Model(spec, T)
    with pytest.raises(InfernoError):
        m.forward([spec.vocab + 5], 0)            # token out of range
    with pytest.raises(InfernoError):
        m.decode_greedy(1, spec.ctx - 2, 8)       # beyond max_ctx
    with pytest.raises(InfernoError):
        m.layer(spec.layers, np.zeros(spec.hidden, np.float32), 0)
    m.close()
    bad = dict(T)
    del bad["blk.0.ssm_a"]
    with pytest.raises(InfernoError):
        Model(spec, bad)                            # layer 0 becomes attention without its tensors


@pytest.fixture(scope="module")
def config1():
    if os.environ.get("INFERNO_SKIP_08B") == "1":
        pytest.skip("config-1 tests disabled")
    spec = S.CONFIGS["qwen35-0.8b"]
    T = S.make_model(spec, seed=0)
    return spec, T, O.OracleModel(spec, T)


def test_config1_greedy_identity(config1):
    """Config 1 (0.8B-shaped hybrid): 32-token prompt, 64 greedy tokens
    identical to the oracle's (north_star asks >= 64)."""
    spec, T, orc = config1
    prompt = S.tokens(0, 32, spec.vocab)
    m = Model(spec, T, max_ctx=512)
    got = m.generate(prompt, 64)
    m.close()
    want = orc.generate(prompt, 64)
    assert got == want


def test_config1_decode_batch_matches_single(config1):
    """Config 1, batched decode (B = 8 sequences, own prompts): each sequence's
    greedy tokens equal the engine's own single-sequence decode (which the
    identity test pins to the oracle), and two replays from the same saved
    state agree (the whole-head GDN kernel of the batched step once read its
    shared-memory weight rows without a barrier)."""
    spec, T, orc = config1
    B, P, n = 8, 16, 24
    m = Model(spec, T, max_ctx=256, max_batch=B)
    toks = []
    for b in range(B):
        m.select_sequence(b)
        first, _ = m.forward(S.tokens(50 + b, P, spec.vocab), 0, want_logits=False)
        toks.append(first)
    m.select_sequence(0)
    m.save_device()
    out1 = m.decode_batch(toks, [P] * B, n)
    m.restore_device()
    out2 = m.decode_batch(toks, [P] * B, n)
    m.restore_device()
    single = []
    for b in range(B):
        m.select_sequence(b)
        single.append(list(m.decode_greedy(toks[b], P, n)))
    m.close()
    assert np.array_equal(out1, out2)
    for b in range(B):
        assert out1[:, b].tolist() == single[b], b


def test_config1_per_layer_hidden(config1, monkeypatch):
    """Config 1: hidden state after every one of the 24 layers for the last
    of the 32 prompt tokens, and its logits, within rel 2e-3 of the oracle
    (north_star's per-layer bound; fp32 activations, exact-integer tensor-core
    dots)."""
    spec, T, orc = config1
    monkeypatch.setenv("INFERNO_B200_DUMP", "1")
    prompt = S.tokens(0, 32, spec.vocab)
    m = Model(spec, T, max_ctx=512)
    m.reset()
    am_g, lg_g = m.forward(prompt, 0)
    orc.reset()
    am_o, lg_o = orc.forward(prompt, 0)
    worst = max(rel(m.hidden(i), orc.hidden(i)) for i in range(spec.layers))
    m.close()
    assert worst < LAYER_RTOL, worst
    assert rel(lg_g, lg_o) < LOGIT_RTOL
    assert am_g == am_o


def test_q6k_regrouping_is_bitwise_neutral(tiny, monkeypatch):
    """The engine regroups Q6_K ffn_down / lm_head bytes per 16 rows for the
    tensor-core GEMV (T_Q6_KR): the same arithmetic in the same order, so
    logits are bit-identical to the GGUF-layout path."""
    spec, T, _ = tiny
    prompt = S.tokens(13, 6, spec.vocab)
    monkeypatch.setenv("INFERNO_NO_REPACK", "1")
    m = Model(spec, T)
    am0, lg0 = m.forward(prompt, 0)
    m.close()
    monkeypatch.delenv("INFERNO_NO_REPACK")
    m = Model(spec, T)
    am1, lg1 = m.forward(prompt, 0)
    m.close()
    assert am0 == am1
    assert np.array_equal(lg0, lg1)


@pytest.mark.parametrize("n", [2, 8, 21, 64, 150])
def test_chunked_prefill_matches_token_loop(tiny, monkeypatch, n):
    """forward_tokens runs prompts in chunks of up to 128 tokens: chunks of
    >= 16 tokens on the tcgen05 GEMM with the token-parallel GDN prep + the
    sequential recurrence, shorter ones on the batched GEMV and the chunk GDN
    kernel (150 = 128 + 22, 2 and 8 the short path); logits, argmax and the
    state it leaves (checked through the greedy continuation) match the
    token-by-token path and the oracle."""
    spec, T, orc = tiny
    prompt = S.tokens(17, n, spec.vocab)
    monkeypatch.setenv("INFERNO_B200_NO_PREFILL", "1")
    m0 = Model(spec, T)
    am0, lg0 = m0.forward(prompt, 0)
    cont0 = m0.decode_greedy(am0, n, 12).tolist()
    m0.close()
    monkeypatch.delenv("INFERNO_B200_NO_PREFILL")
    m1 = Model(spec, T)
    am1, lg1 = m1.forward(prompt, 0)
    cont1 = m1.decode_greedy(am1, n, 12).tolist()
    m1.close()
    assert rel(lg1, lg0) < 1e-4, rel(lg1, lg0)
    assert am1 == am0
    assert cont1 == cont0
    orc.reset()
    am_o, lg_o = orc.forward(prompt, 0)
    assert am1 == am_o and rel(lg1, lg_o) < LOGIT_RTOL


def test_prefill_graph_replays_match_eager(tiny):
    """The second forward_tokens call with the same (tokens, position) key is
    captured into a CUDA graph and later calls replay it: same results as the
    eager first call, for a new prompt of the same length too."""
    spec, T, _ = tiny
    m = Model(spec, T)
    p1 = S.tokens(19, 12, spec.vocab)
    p2 = S.tokens(20, 12, spec.vocab)
    outs = []
    for p in (p1, p1, p1, p2):
        m.reset()
        outs.append(m.forward(p, 0))
    m.reset()
    m2 = Model(spec, T)
    ref2 = m2.forward(p2, 0)
    m2.close()
    m.close()
    assert outs[0][0] == outs[1][0] == outs[2][0]
    assert np.array_equal(outs[0][1], outs[1][1]) and np.array_equal(outs[1][1], outs[2][1])
    assert outs[3][0] == ref2[0] and np.array_equal(outs[3][1], ref2[1])


def test_fused_inproj_gdn_opt_in(monkeypatch):
    """INFERNO_B200_FUSED_GDN=1 (configs with one value head per q/k group):
    the 8-CTA cluster kernel replaces the in_proj GEMV + GDN step; logits and
    greedy tokens match the two-kernel path and the oracle."""
    import dataclasses
    spec = dataclasses.replace(S.CONFIGS["tiny"], ssm_nk=4)      # nv == nk == 4
    T = S.make_model(spec, seed=23)
    prompt = S.tokens(23, 9, spec.vocab)
    m0 = Model(spec, T)
    want = m0.generate(prompt, 12)
    am0, lg0 = m0.forward(prompt, 0)
    m0.close()
    monkeypatch.setenv("INFERNO_B200_FUSED_GDN", "1")
    m1 = Model(spec, T)
    got = m1.generate(prompt, 12)
    am1, lg1 = m1.forward(prompt, 0)
    m1.close()
    assert got == want and am1 == am0
    assert rel(lg1, lg0) < 1e-4
    orc = O.OracleModel(spec, T)
    assert got == orc.generate(prompt, 12)


def test_native_gguf_upload_matches_python_upload(tiny, tmp_path):
    """Model.from_gguf through the library's reader and pinned staging
    (inferno_engine_load_gguf) generates the same tokens and logits as the
    same weights uploaded tensor by tensor from Python, and as the oracle."""
    spec, T, orc = tiny
    path = tmp_path / "tiny.gguf"
    S.write_gguf(path, spec, T)
    prompt = S.tokens(12, 10, spec.vocab)
    a = Model.from_gguf(path, native=True)
    b = Model(spec, T)
    assert a.spec.vocab == spec.vocab and a.spec.layers == spec.layers
    _, la = a.forward(prompt, 0)
    _, lb = b.forward(prompt, 0)
    assert np.array_equal(la, lb)
    a.reset()
    b.reset()
    got = a.generate(prompt, 16)
    assert got == b.generate(prompt, 16) == orc.generate(prompt, 16)
    a.close()
    b.close()
