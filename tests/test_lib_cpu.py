"""CPU tests of the C-ABI library and host logic (no compute calls on a GPU):
the library loads, exports every function the header declares, rejects bad
arguments with a status + message, and the host-side GGUF / config / byte
accounting matches the reference's loader conventions."""
import ctypes as C
import math
import re
from pathlib import Path

import numpy as np
import pytest

from inferno_b200 import synth as S
from inferno_b200._lib import EXPORTS, InfernoConfig, lib
import oracle as O

ROOT = Path(__file__).resolve().parent.parent
HEADER = ROOT / "include" / "inferno_b200.h"


def header_functions():
    txt = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    return sorted(set(re.findall(r"\b([a-z_][A-Za-z0-9_]*)\s*\([^;{]*\)\s*;", txt)) - {"sizeof"})


def test_library_exports_every_header_symbol():
    L = lib()
    fns = header_functions()
    assert len(fns) >= 25
    missing = [f for f in fns if not hasattr(L, f)]
    assert not missing, missing
    assert set(EXPORTS) <= set(fns)


COMPAT = ("q4_k_gemv", "q5_k_gemv", "q6_k_gemv", "q8_0_gemv", "quantize_row_q8_K",
          "vec_dot_q4_K_q8_K", "vec_dot_q5_K_q8_K", "vec_dot_q6_K_q8_K", "vec_dot_q8_0_q8_0")


def test_compat_symbols_match_reference_names():
    # src/kernels/quant_kernels.c:166-697 / src/QuantizedKernels.jl:88-176
    for f in COMPAT:
        assert hasattr(lib(), f)
    ref = O.ref_lib()
    if ref is not None:      # every symbol the reference's library exports is here too
        import subprocess
        out = subprocess.run(["nm", "-D", "--defined-only", str(O.REF_LIB_PATH)], capture_output=True, text=True)
        names = {ln.split()[-1] for ln in out.stdout.splitlines() if " T " in ln}
        assert names == set(COMPAT), names


def test_q8k_helpers_argument_errors_without_gpu():
    L = lib()
    assert math.isnan(L.vec_dot_q4_K_q8_K(None, None, -1))
    assert b"nb = -1" in L.inferno_last_error()
    x, y = np.zeros(100, np.float32), np.zeros(292, np.uint8)
    L.quantize_row_q8_K(x.ctypes.data, y.ctypes.data, 100)
    assert b"multiple of 256" in L.inferno_last_error()
    assert L.vec_dot_q6_K_q8_K(None, None, 0) == 0.0       # empty row: no device work


def test_argument_errors_without_gpu():
    L = lib()
    assert L.inferno_gemv(S.Q4_K, None, None, None, 1024, 8, 1, None) == -1
    assert b"null" in L.inferno_last_error()
    assert L.inferno_dequantize(S.Q4_K, None, 256, None, None) == -1
    assert L.inferno_engine_create(None, None) == -1
    c = InfernoConfig()
    c.struct_size = 4     # wrong ABI size
    h = C.c_void_p()
    assert L.inferno_engine_create(C.byref(c), C.byref(h)) == -1
    assert b"struct_size" in L.inferno_last_error()


def test_config_struct_size_matches_header():
    # InfernoConfig: 20 int32 + 3 float + 4 int32 + pointer (8-byte aligned)
    assert C.sizeof(InfernoConfig) == 120


def test_gguf_round_trip_and_config(tmp_path):
    from inferno_b200.model import config_from_metadata, read_gguf, spec_from_config
    spec = S.CONFIGS["tiny"]
    T = S.make_model(spec, seed=9)
    path = tmp_path / "tiny.gguf"
    S.write_gguf(path, spec, T)
    md, T2 = read_gguf(path)
    assert set(T2) == set(T)
    for k, t in T.items():
        assert T2[k].ggml_type == t.ggml_type and tuple(T2[k].ne) == tuple(t.ne), k
        assert np.array_equal(T2[k].data, t.data), k
    s2 = spec_from_config(config_from_metadata(md, T2))
    for f in ("hidden", "layers", "n_heads", "n_kv", "head_dim", "ffn", "vocab", "ssm_nv", "ssm_nk",
              "ssm_dk", "ssm_dv", "conv_k", "ctx"):
        assert getattr(s2, f) == getattr(spec, f), f


def test_metadata_key_precedence():
    """src/LoaderCPU.jl:398-414 reads qwen3.* then bare keys; real files carry
    qwen35.*, which must win when present."""
    from inferno_b200.model import config_from_metadata
    T = {"token_embd.weight": S.Tensor(S.Q6_K, (512, 4096), np.zeros(1, np.uint8))}
    md = {"general.architecture": "qwen35", "qwen35.embedding_length": 512, "qwen3.embedding_length": 999,
          "embedding_length": 7}
    assert config_from_metadata(md, T)["hidden"] == 512
    md = {"general.architecture": "qwen35", "qwen3.embedding_length": 640, "embedding_length": 7}
    assert config_from_metadata(md, T)["hidden"] == 640


def _config1_shapes(spec):
    H = spec.hidden
    d = {"token_embd.weight": (S.Q6_K, spec.vocab, H)}
    for i in range(spec.layers):
        p = f"blk.{i}."
        if spec.is_attn(i):
            d[p + "attn_q.weight"] = (S.Q4_K, 2 * spec.n_heads * spec.head_dim, H)
            d[p + "attn_k.weight"] = (S.Q4_K, spec.n_kv * spec.head_dim, H)
            d[p + "attn_v.weight"] = (S.Q4_K, spec.n_kv * spec.head_dim, H)
            d[p + "attn_output.weight"] = (S.Q4_K, H, spec.n_heads * spec.head_dim)
        else:
            d[p + "attn_qkv.weight"] = (S.Q4_K, spec.conv_channels, H)
            d[p + "attn_gate.weight"] = (S.Q4_K, spec.d_inner, H)
            d[p + "ssm_out.weight"] = (S.Q4_K, H, spec.d_inner)
        d[p + "ffn_gate.weight"] = (S.Q4_K, spec.ffn, H)
        d[p + "ffn_up.weight"] = (S.Q4_K, spec.ffn, H)
        d[p + "ffn_down.weight"] = (S.Q6_K, H, spec.ffn)
    return d


def test_config1_algorithmic_bytes():
    """Bytes per decode token of config 1 (~559 MB at mean position ~96)."""
    from inferno_b200.model import algorithmic_bytes_per_token
    spec = S.CONFIGS["qwen35-0.8b"]
    T = {}
    for name, (t, rows, inner) in _config1_shapes(spec).items():
        T[name] = S.Tensor(t, (inner, rows), np.empty(rows * S.row_bytes(t, inner), np.uint8))
    for i in range(spec.layers):
        if not spec.is_attn(i):
            T[f"blk.{i}.ssm_a"] = S.Tensor(S.F32, (spec.ssm_nv,), np.empty(spec.ssm_nv * 4, np.uint8))
    b = algorithmic_bytes_per_token(spec, T, 96)
    assert 540e6 < b < 575e6, b


@pytest.mark.parametrize("t", [S.Q4_K, S.Q5_K, S.Q6_K, S.Q8_0, S.IQ2_XXS])
def test_block_sizes(t):
    # src/QuantsCPU.jl:22-25 and the IQ2_XXS 66-byte block
    assert S.row_bytes(t, 256 if t != S.Q8_0 else 32) == {S.Q4_K: 144, S.Q5_K: 176, S.Q6_K: 210,
                                                           S.Q8_0: 34, S.IQ2_XXS: 66}[t]


def test_struct_layouts_match_the_c_header(tmp_path):
    """InfernoConfig / InfernoSampling field offsets of the Python binding equal
    what a C compiler makes of include/inferno_b200.h."""
    import shutil
    import subprocess
    from inferno_b200._lib import InfernoSampling
    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        pytest.skip("no C compiler")
    structs = {"InfernoConfig": InfernoConfig, "InfernoSampling": InfernoSampling}
    lines = ['#include <stdio.h>', '#include <stddef.h>', '#include "inferno_b200.h"', 'int main(void) {']
    for sname, cls in structs.items():
        lines.append(f'  printf("{sname} sizeof %zu\\n", sizeof({sname}));')
        for f, _ in cls._fields_:
            lines.append(f'  printf("{sname} {f} %zu\\n", offsetof({sname}, {f}));')
    lines += ["  return 0;", "}"]
    src = tmp_path / "layout.c"
    src.write_text("\n".join(lines))
    exe = tmp_path / "layout"
    subprocess.run([cc, "-I", str(HEADER.parent), str(src), "-o", str(exe)], check=True)
    out = subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout.split("\n")
    got = {(a, b): int(c) for a, b, c in (ln.split() for ln in out if ln.strip())}
    for sname, cls in structs.items():
        assert got[(sname, "sizeof")] == C.sizeof(cls), sname
        for f, _ in cls._fields_:
            assert got[(sname, f)] == getattr(cls, f).offset, (sname, f)


def test_missing_library_fails_loudly(tmp_path):
    """No CPU fallback: without the built library every entry point raises."""
    import subprocess
    import sys
    code = ("import sys; sys.path.insert(0, 'inferno.jl_b200')\n"
            "from inferno_b200 import _lib\n"
            "try:\n    _lib.lib()\nexcept RuntimeError as e:\n    print('raised', 'not built' in str(e))\n"
            "else:\n    print('loaded')\n")
    env = dict(__import__("os").environ, INFERNO_B200_LIB=str(tmp_path / "absent.so"))
    out = subprocess.run([sys.executable, "-c", code], cwd=str(ROOT), env=env, capture_output=True, text=True,
                         check=True).stdout.strip()
    assert out == "raised True"
