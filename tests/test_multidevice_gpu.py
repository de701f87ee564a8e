"""Two engines on two devices of one process: every kernel attribute the
engine sets once (dynamic shared memory, carve-out) is set per device, so the
engine on the second device launches the same kernels correctly.  Both
engines' greedy tokens equal the oracle's.  Skipped on boxes with one GPU."""
import pytest

import oracle as O
from inferno_b200 import synth as S
from inferno_b200.model import Model

pytestmark = pytest.mark.gpu


def _ngpus():
    try:
        import torch
        return torch.cuda.device_count()
    except Exception:
        return 0


@pytest.mark.skipif(_ngpus() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("spec_name", ["tiny", "tiny-moe"])
def test_engines_on_two_devices_in_one_process(spec_name):
    spec = S.CONFIGS[spec_name]
    T = S.make_model(spec, seed=23)
    prompt = S.tokens(5, 24, spec.vocab)          # 24 tokens: the chunked prefill runs too
    want = O.OracleModel(spec, T).generate(prompt, 12)
    m0 = Model(spec, T, device=0)
    m1 = Model(spec, T, device=1)                 # second device: its own attribute set-up
    try:
        got1 = m1.generate(prompt, 12)
        got0 = m0.generate(prompt, 12)
    finally:
        m0.close()
        m1.close()
    assert got0 == want
    assert got1 == want
