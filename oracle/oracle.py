"""ctypes binding of the CPU oracle (oracle.cpp) -- test infrastructure.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg use this
module, and only as the checker (or the timed CPU baseline).  The engine in
inferno.jl_b200/ never imports it.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "_build" / "liboracle.so"
REF_LIB_PATH = HERE / "_ref" / "libquant_kernels_ref.so"

_lib = None


def build(quiet: bool = True) -> None:
    subprocess.run(["make", "-C", str(HERE)], check=True,
                   stdout=subprocess.DEVNULL if quiet else None)


def lib():
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            build()
        L = C.CDLL(str(LIB_PATH))
        p, i, i64 = C.c_void_p, C.c_int, C.c_int64
        L.orc_dequant.argtypes = [i, p, i64, p]
        L.orc_gemv.argtypes = [i, p, p, p, i, i, i]
        L.orc_flash_attention.argtypes = [p, p, p, p, i, i, C.c_float, i, i]
        L.orc_standard_attention.argtypes = [p, p, p, p, i, i, C.c_float, i, i]
        L.orc_attention_step.argtypes = [p, p, p, p, p, C.c_float, i, i, i, i, C.c_float, p, p, i, p]
        L.orc_quantize_row_q8_K.argtypes = [p, p, i64]
        L.orc_vec_dot_q8k.argtypes = [i, p, p, i]
        L.orc_vec_dot_q8k.restype = C.c_float
        L.orc_ref_gemv.argtypes = [i, p, p, p, i, i]
        L.orc_gdn_recurrence.argtypes = [i, i, i, i, p, p, p, p, p, p, p]
        L.orc_model_create.restype = p
        L.orc_model_create.argtypes = [p, p]
        L.orc_model_destroy.argtypes = [p]
        L.orc_model_set_tensor.argtypes = [p, C.c_char_p, i, p, i, p, i64]
        L.orc_model_finalize.argtypes = [p]
        L.orc_model_reset.argtypes = [p]
        L.orc_layer_forward.argtypes = [p, i, p, i]
        L.orc_forward.argtypes = [p, p, i, i, p, p]
        L.orc_get_hidden.argtypes = [p, i, p]
        L.orc_embed.argtypes = [p, i, p]
        _lib = L
    return _lib


def _ptr(a: np.ndarray):
    return a.ctypes.data_as(C.c_void_p)


def dequant(ggml_type: int, data: np.ndarray, n: int) -> np.ndarray:
    data = np.ascontiguousarray(data, dtype=np.uint8)
    out = np.empty(n, np.float32)
    rc = lib().orc_dequant(ggml_type, _ptr(data), n, _ptr(out))
    if rc:
        raise ValueError(f"orc_dequant rc={rc}")
    return out


def gemv(ggml_type: int, W: np.ndarray, x: np.ndarray, inner: int, outer: int) -> np.ndarray:
    """x: (batch, inner) fp32 -> (batch, outer)."""
    W = np.ascontiguousarray(W, dtype=np.uint8)
    x = np.ascontiguousarray(np.atleast_2d(x), dtype=np.float32)
    y = np.empty((x.shape[0], outer), np.float32)
    rc = lib().orc_gemv(ggml_type, _ptr(W), _ptr(x), _ptr(y), inner, outer, x.shape[0])
    if rc:
        raise ValueError(f"orc_gemv rc={rc}")
    return y


Q8K_BYTES = 292     # block_q8_K: float d, int8 qs[256], int16 bsums[16]


def quantize_q8k(x) -> np.ndarray:
    """quantize_row_q8_K (src/kernels/quant_kernels.c:166-196) -> raw block bytes."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.zeros(x.size // 256 * Q8K_BYTES, np.uint8)
    lib().orc_quantize_row_q8_K(_ptr(x), _ptr(y), x.size)
    return y


def vec_dot_q8k(ggml_type: int, xblocks, yblocks, nb: int) -> float:
    """vec_dot_q{4,5,6}_K_q8_K / vec_dot_q8_0_q8_0 (quant_kernels.c:204-559),
    restated with the lane and accumulation order of the AVX2 + FMA build."""
    xb = np.ascontiguousarray(xblocks, dtype=np.uint8)
    yb = np.ascontiguousarray(yblocks, dtype=np.uint8)
    return float(lib().orc_vec_dot_q8k(ggml_type, _ptr(xb), _ptr(yb), nb))


def ref_numerics_gemv(ggml_type: int, W, x, inner: int, outer: int) -> np.ndarray:
    """q*_k_gemv / q8_0_gemv of the reference library (quant_kernels.c:602-697)
    restated: Q8_K activations for the K-quants, the AVX2 lane order."""
    W = np.ascontiguousarray(W, dtype=np.uint8)
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.empty(outer, np.float32)
    lib().orc_ref_gemv(ggml_type, _ptr(W), _ptr(x), _ptr(y), inner, outer)
    return y


def flash_attention(q, ck, cv, kvh, seq_len, scale, hd, nkv, standard=False):
    out = np.empty(hd, np.float32)
    f = lib().orc_standard_attention if standard else lib().orc_flash_attention
    f(_ptr(out), _ptr(q), _ptr(ck), _ptr(cv), kvh, seq_len, scale, hd, nkv)
    return out


def attention_step(qg, k, v, q_norm, k_norm, eps, nh, nkv, hd, rd, theta, kc, vc, pos):
    """One gated attention step after the projections (src/ModelCPU.jl:766-851):
    qg [nh][2*hd], k/v [nkv][hd]; kc/vc [ctx][nkv][hd] are updated at pos.
    Returns the gated output [nh*hd]."""
    out = np.empty(nh * hd, np.float32)
    args = [np.ascontiguousarray(a, dtype=np.float32) for a in (qg, k, v, q_norm, k_norm)]
    assert kc.dtype == np.float32 and kc.flags.c_contiguous and vc.dtype == np.float32 and vc.flags.c_contiguous
    lib().orc_attention_step(*[_ptr(a) for a in args], eps, nh, nkv, hd, rd, theta, _ptr(kc), _ptr(vc), pos,
                             _ptr(out))
    return out


def gdn_recurrence(q, k, v, beta, g, S):
    """q,k (T,H,dk); v (T,H,dv); beta,g (T,H); S (H,dv,dk) updated in place."""
    T, H, dk = q.shape
    dv = v.shape[2]
    y = np.empty((T, H, dv), np.float32)
    args = [np.ascontiguousarray(a, dtype=np.float32) for a in (q, k, v, beta, g)]
    assert S.dtype == np.float32 and S.flags.c_contiguous
    lib().orc_gdn_recurrence(T, H, dk, dv, *[_ptr(a) for a in args], _ptr(S), _ptr(y))
    return y


def softmax_sample(logits, temperature, top_p=1.0, top_k=0, min_p=0.0, presence=0.0, repetition=1.0,
                   seen=(), r=0.5):
    """src/ModelCPU.jl:1123-1225 with the uniform draw r given; 0-based token."""
    lg = np.ascontiguousarray(logits, dtype=np.float32)
    sn = np.ascontiguousarray(seen, dtype=np.int32) if len(seen) else np.zeros(1, np.int32)
    L = lib()
    L.orc_softmax_sample.restype = C.c_int
    return int(L.orc_softmax_sample(_ptr(lg), lg.size, C.c_float(temperature), C.c_float(top_p), int(top_k),
                                    C.c_float(min_p), C.c_float(presence), C.c_float(repetition), _ptr(sn),
                                    len(seen), C.c_float(r)))


class OracleModel:
    """The reference CPU model (load_model_cpu + forward_cpu!) restated."""

    def __init__(self, spec, tensors: dict, dequant_at_load: bool = True):
        self.spec = spec
        ip = np.array([spec.hidden, spec.layers, spec.n_heads, spec.n_kv, spec.head_dim, spec.ffn,
                       spec.vocab, spec.ssm_nv, spec.ssm_nk, spec.ssm_dk, spec.ssm_dv, spec.conv_k,
                       spec.ctx, spec.n_experts, spec.n_experts_used, spec.expert_ffn,
                       spec.shexp_ffn, int(dequant_at_load)], dtype=np.int64)
        fp = np.array([spec.eps, spec.rope_theta, spec.partial_rotary], dtype=np.float64)
        self.h = lib().orc_model_create(_ptr(ip), _ptr(fp))
        for name, t in tensors.items():
            ne = np.array(t.ne, dtype=np.int64)
            lib().orc_model_set_tensor(self.h, name.encode(), t.ggml_type, _ptr(ne), len(t.ne),
                                       _ptr(t.data), t.nbytes)
        rc = lib().orc_model_finalize(self.h)
        if rc:
            raise ValueError(f"orc_model_finalize rc={rc}")

    def __del__(self):
        if getattr(self, "h", None):
            lib().orc_model_destroy(self.h)
            self.h = None

    def reset(self):
        lib().orc_model_reset(self.h)

    def forward(self, toks, pos, want_logits=True):
        toks = np.ascontiguousarray(toks, dtype=np.int32)
        logits = np.empty(self.spec.vocab, np.float32) if want_logits else None
        am = np.zeros(1, np.int32)
        rc = lib().orc_forward(self.h, _ptr(toks), len(toks), pos,
                               _ptr(logits) if want_logits else None, _ptr(am))
        if rc:
            raise ValueError(f"orc_forward rc={rc}")
        return int(am[0]), logits

    def layer(self, i, x, pos):
        x = np.ascontiguousarray(x, dtype=np.float32).copy()
        rc = lib().orc_layer_forward(self.h, i, _ptr(x), pos)
        if rc:
            raise ValueError(f"orc_layer_forward rc={rc}")
        return x

    def hidden(self, i):
        out = np.empty(self.spec.hidden, np.float32)
        lib().orc_get_hidden(self.h, i, _ptr(out))
        return out

    def embed(self, tok):
        out = np.empty(self.spec.hidden, np.float32)
        lib().orc_embed(self.h, tok, _ptr(out))
        return out

    def generate(self, prompt, n_steps):
        """Greedy decode with the corrected position schedule
        (test/benchmark_e2e.jl:43-59): prompt at 0..P-1, token i at P+i."""
        self.reset()
        tok, _ = self.forward(prompt, 0, want_logits=False)
        out = [tok]
        pos = len(prompt)
        for _ in range(n_steps - 1):
            tok, _ = self.forward([tok], pos, want_logits=False)
            out.append(tok)
            pos += 1
        return out


# ---- the reference's own C kernels (oracle/_ref), timed baseline only -------
def ref_lib():
    if not REF_LIB_PATH.exists():
        return None
    L = C.CDLL(str(REF_LIB_PATH))
    p, i = C.c_void_p, C.c_int
    for nm in ("q4_k_gemv", "q5_k_gemv", "q6_k_gemv"):
        getattr(L, nm).argtypes = [p, p, p, p, i, i]
    L.q8_0_gemv.argtypes = [p, p, p, i, i]
    L.quantize_row_q8_K.argtypes = [p, p, C.c_int64]
    for nm in ("vec_dot_q4_K_q8_K", "vec_dot_q5_K_q8_K", "vec_dot_q6_K_q8_K", "vec_dot_q8_0_q8_0"):
        getattr(L, nm).argtypes = [p, p, i]
        getattr(L, nm).restype = C.c_float
    return L


def ref_gemv(ggml_type, W, x, inner, outer, L=None):
    """Inferno.jl's keep_quantized GEMV (src/QuantizedKernels.jl:82-146):
    quantizes x to Q8_K, integer dots.  Loose numerics by design."""
    L = L or ref_lib()
    y = np.empty(outer, np.float32)
    x = np.ascontiguousarray(x, dtype=np.float32)
    if ggml_type == 8:
        L.q8_0_gemv(_ptr(W), _ptr(x), _ptr(y), inner, outer)
    else:
        q8 = np.zeros((inner // 256) * 292 + 64, np.uint8)
        fn = {12: L.q4_k_gemv, 13: L.q5_k_gemv, 14: L.q6_k_gemv}[ggml_type]
        fn(_ptr(W), _ptr(x), _ptr(y), _ptr(q8), inner, outer)
    return y


def cpu_count() -> int:
    return len(os.sched_getaffinity(0))
