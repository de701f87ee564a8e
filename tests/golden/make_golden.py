"""Generate the dequantization golden vectors in this directory.

Third-party cross-check (the reference's own method, examples/checks/
gen_dequant_ref.py + compare_dequant.jl:57-95): seeded N(0,0.02) matrices are
packed with inferno_b200.synth's packers and dequantized by gguf-py 0.19.0
(ggml semantics).  For Q4_K/Q5_K/Q6_K/Q8_0 ggml and Inferno.jl decode
identically; for IQ2_XXS Inferno.jl subtracts 8 from every grid byte
(src/Dequant.jl:46), so the file also stores the IQ2_XXS expectation
restated here in numpy from src/Dequant.jl:12-54.
Run: python tests/golden/make_golden.py   (writes dequant_golden.npz)
"""
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent.parent / "inferno.jl_b200"))
from inferno_b200 import synth as S  # noqa: E402


def iq2xxs_inferno(q: np.ndarray) -> np.ndarray:
    """src/Dequant.jl:12-54 in numpy: db*(grid_byte-8)*sign per element."""
    nb = q.size // 66
    b = q.reshape(nb, 66)
    d = b[:, 0:2].copy().view(np.float16).astype(np.float32).reshape(nb)
    aux = b[:, 2:].copy().view("<u4").reshape(nb, 8, 2)
    a1, a2 = aux[..., 0], aux[..., 1]
    db = (d[:, None] * (np.float32(0.5) + (a2 >> 28).astype(np.float32))) * np.float32(0.25)
    out = np.empty((nb, 8, 4, 8), np.float32)
    for l in range(4):
        gidx = (a1 >> (8 * l)) & 0xFF
        grid = S.IQ2XXS_GRID_BYTES[gidx].astype(np.int32) - 8          # (nb,8,8)
        signs = S.KSIGNS[(a2 >> (7 * l)) & 127]                       # (nb,8)
        neg = ((signs[..., None] >> np.arange(8)) & 1).astype(bool)
        v = (db[..., None] * grid.astype(np.float32)) * np.where(neg, np.float32(-1), np.float32(1))
        out[:, :, l, :] = v
    return out.reshape(-1)


def main():
    import gguf
    from gguf import quants
    rng = np.random.default_rng(2024)
    w = (rng.standard_normal((4, 512)) * 0.02).astype(np.float32)
    res = {}
    for t in (S.Q8_0, S.Q4_K, S.Q5_K, S.Q6_K, S.IQ2_XXS):
        q = S.quantize(w, t).reshape(-1)
        g = quants.dequantize(q, gguf.GGMLQuantizationType(t)).reshape(-1).astype(np.float32)
        res[f"{S.TYPE_NAME[t]}_bytes"] = q
        res[f"{S.TYPE_NAME[t]}_ggml"] = g
    res["IQ2_XXS_inferno"] = iq2xxs_inferno(res["IQ2_XXS_bytes"])
    np.savez_compressed(HERE / "dequant_golden.npz", **res)


if __name__ == "__main__":
    main()
