"""Seeded inputs of the Q8_K helpers (quantize_row_q8_K / vec_dot_*_q8_K)
shared by the oracle pin tests and the GPU parity tests."""
import numpy as np

import oracle as O

_BB = {12: 144, 13: 176, 14: 210, 8: 34, 16: 66}


def random_blocks(rng, ggml_type, nb):
    """Raw weight blocks with arbitrary quant bytes and finite fp16 scales
    (IQ2_XXS: any grid / sign index byte is valid, d is the leading fp16)."""
    bb = _BB[ggml_type]
    a = rng.integers(0, 256, (nb, bb), dtype=np.uint8)
    halves = (rng.standard_normal((nb, 2)) * 0.01).astype(np.float16).view(np.uint8).reshape(nb, 4)
    if ggml_type in (12, 13):
        a[:, 0:4] = halves
    elif ggml_type == 14:
        a[:, 208:210] = halves[:, :2]
    else:
        a[:, 0:2] = halves[:, :2]
    return a.reshape(-1)


def random_q8k(rng, nb):
    """block_q8_K bytes: quantized from a random vector, then with raw extremes mixed in."""
    x = (rng.standard_normal(nb * 256) * rng.uniform(0.1, 10)).astype(np.float32)
    y = O.quantize_q8k(x).reshape(nb, O.Q8K_BYTES)
    y[0, 4:8] = [0x80, 0x7F, 0x80, 0x81]              # -128 / 127 quants
    return y.reshape(-1)
