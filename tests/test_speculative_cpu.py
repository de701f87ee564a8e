"""Host-side sampling of the speculative loop (softmax_sample /
sample_from_probs restated from src/ModelCPU.jl:1123-1170 and
src/SpeculativeDecoding.jl:21-30), on CPU."""
import numpy as np

from inferno_b200.speculative import sample_from_probs, softmax_sample


def test_temperature_zero_and_top_k_one_are_argmax():
    rng = np.random.default_rng(0)
    v = rng.standard_normal(1000).astype(np.float32)
    assert softmax_sample(v, rng, temperature=0.0) == int(np.argmax(v))
    for _ in range(20):
        assert softmax_sample(v, rng, temperature=1.0, top_k=1) == int(np.argmax(v))


def test_top_p_restricts_to_nucleus():
    rng = np.random.default_rng(1)
    v = np.array([10.0, 9.5, 0.0, -1.0, -5.0], np.float32)
    got = {softmax_sample(v, rng, temperature=1.0, top_p=0.5) for _ in range(200)}
    assert got <= {0, 1}


def test_sample_from_probs_first_index_reaching_draw():
    class R:
        def __init__(self, r):
            self.r = r

        def random(self):
            return self.r
    p = np.array([0.1, 0.2, 0.3, 0.4], np.float32)
    assert sample_from_probs(p, R(0.05)) == 0
    assert sample_from_probs(p, R(0.25)) == 1
    assert sample_from_probs(p, R(0.61)) == 3
    assert sample_from_probs(p, R(0.9999)) == 3
