"""GPU parity of the MoE FFN (config-5 semantics, src/Model.jl:478-561) on a
seeded tiny MoE hybrid: router softmax + stable top-k on the device, routed
IQ2_XXS gate/up experts gathered through device expert ids, Q4_K down over all
selected experts plus the shared expert, deterministic combine.  Checked
against the CPU oracle through the C ABI."""
import dataclasses

import numpy as np
import pytest

import oracle as O
from inferno_b200 import synth as S
from inferno_b200.model import Model

pytestmark = pytest.mark.gpu

RTOL = 2e-3


def rel(a, b):
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-30))


@pytest.fixture(scope="module", params=["shared", "no-shared"])
def moe(request):
    spec = S.CONFIGS["tiny-moe"]
    if request.param == "no-shared":
        spec = dataclasses.replace(spec, shexp_ffn=0)
    T = S.make_model(spec, seed=21)
    return spec, T, O.OracleModel(spec, T)


def test_moe_generate_matches_oracle(moe):
    spec, T, orc = moe
    prompt = S.tokens(21, 10, spec.vocab)
    m = Model(spec, T)
    got = m.generate(prompt, 20)
    m.close()
    assert got == orc.generate(prompt, 20)


def test_moe_logits_and_layers(moe):
    spec, T, orc = moe
    prompt = S.tokens(22, 7, spec.vocab)
    m = Model(spec, T)
    orc.reset()
    am_o, lg_o = orc.forward(prompt, 0)
    am_g, lg_g = m.forward(prompt, 0)
    assert rel(lg_g, lg_o) < RTOL
    assert am_g == am_o
    x = orc.embed(int(am_o))
    for i in range(spec.layers):
        xo = orc.layer(i, x, len(prompt))
        xg = m.layer(i, x, len(prompt))
        assert rel(xg, xo) < RTOL, (i, rel(xg, xo))
        x = xo
    m.close()
