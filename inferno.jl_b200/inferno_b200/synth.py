"""Seeded synthetic Qwen3.5-hybrid models in GGUF block formats.

The reference's headline numbers are quoted on real Qwen3.5 GGUF files that are
not available here; these generators stand in for them with the same tensor
names, shapes and quantization types and seeded values:

* matrices N(0, 0.02), quantized by this module's own round-to-nearest packers
  into Q4_K / Q5_K / Q6_K / Q8_0 / IQ2_XXS super-blocks in the native GGUF byte
  layout (decoded by Inferno.jl src/Dequant.jl:12-54, 304-441, 558-601);
* RMSNorm weights 1 + N(0, 0.02) (GGUF norms already carry the +1);
* ssm_conv1d N(0, 0.5), ssm_a = -exp(U[log 0.01, 0]), ssm_dt.bias = 0.

Tensor naming follows the reference loader (src/LoaderCPU.jl:420-643):
``blk.{i}.attn_qkv / attn_gate / ssm_out / ssm_conv1d / ssm_alpha / ssm_beta /
ssm_a / ssm_dt.bias / ssm_norm`` for Gated-DeltaNet layers and
``blk.{i}.attn_q / attn_k / attn_v / attn_output / attn_q_norm / attn_k_norm``
for full-attention layers.  A layer is a GDN layer iff ``blk.{i}.ssm_a`` exists
(src/LoaderCPU.jl:431).  MoE layers use the llama.cpp names
``ffn_gate_inp / ffn_{gate,up,down}_exps / ffn_{gate,up,down}_shexp``.

Every tensor is a ``Tensor(ggml_type, ne, data)`` with ``ne`` in GGUF order
(ne[0] = inner / fastest dimension) and ``data`` the raw little-endian bytes.
"""
from __future__ import annotations

import dataclasses
import math
from pathlib import Path

import numpy as np

# ggml type ids (GGUF spec; Inferno.jl src/GGUF.jl:25-60)
F32, F16, Q8_0, Q4_K, Q5_K, Q6_K, IQ2_XXS = 0, 1, 8, 12, 13, 14, 16

# (elements per block, bytes per block)  -- src/QuantsCPU.jl:22-25
BLOCK = {F32: (1, 4), F16: (1, 2), Q8_0: (32, 34), Q4_K: (256, 144),
         Q5_K: (256, 176), Q6_K: (256, 210), IQ2_XXS: (256, 66)}
TYPE_NAME = {F32: "F32", F16: "F16", Q8_0: "Q8_0", Q4_K: "Q4_K", Q5_K: "Q5_K",
             Q6_K: "Q6_K", IQ2_XXS: "IQ2_XXS"}


def row_bytes(ggml_type: int, inner: int) -> int:
    qk, bb = BLOCK[ggml_type]
    if inner % qk:
        raise ValueError(f"inner dim {inner} not a multiple of {qk} for {TYPE_NAME[ggml_type]}")
    return inner // qk * bb


@dataclasses.dataclass
class Tensor:
    ggml_type: int
    ne: tuple            # GGUF order, ne[0] fastest
    data: np.ndarray     # uint8 raw bytes

    @property
    def nbytes(self) -> int:
        return int(self.data.nbytes)


# ----------------------------------------------------------------------------
# IQ2_XXS codebook (format data, shared with the CUDA sources)
# ----------------------------------------------------------------------------
def _load_grid() -> np.ndarray:
    inc = Path(__file__).resolve().parent.parent / "csrc" / "iq2xxs_grid.inc"
    vals = []
    for line in inc.read_text().splitlines():
        if line.lstrip().startswith("//"):
            continue
        for tok in line.replace("ULL", "").split(","):
            tok = tok.strip()
            if tok:
                vals.append(int(tok, 16))
    assert len(vals) == 256
    return np.array(vals, dtype=np.uint64)


IQ2XXS_GRID = _load_grid()
# 256 x 8 grid bytes
IQ2XXS_GRID_BYTES = IQ2XXS_GRID.view(np.uint8).reshape(256, 8)
# KSIGNS_IQ2XS[i] = i with bit 7 set to the parity of i (src/QuantsData.jl:7-16)
KSIGNS = np.array([i | ((bin(i).count("1") & 1) << 7) for i in range(128)], dtype=np.uint8)


# ----------------------------------------------------------------------------
# round-to-nearest packers (own design; produce bytes the reference decodes)
# ----------------------------------------------------------------------------
def _f16(a):
    return np.asarray(a, dtype=np.float32).astype(np.float16)


def pack_q8_0(w: np.ndarray) -> np.ndarray:
    """w: (rows, inner) fp32 -> (rows, inner/32*34) bytes."""
    rows, inner = w.shape
    b = w.reshape(rows, inner // 32, 32).astype(np.float32)
    amax = np.abs(b).max(-1)
    d16 = _f16(amax / 127.0)
    d = d16.astype(np.float32)
    inv = np.where(d > 0, 1.0 / np.where(d > 0, d, 1), 0.0)
    q = np.clip(np.rint(b * inv[..., None]), -127, 127).astype(np.int8)
    out = np.empty((rows, inner // 32, 34), np.uint8)
    out[..., 0:2] = d16.view(np.uint8).reshape(rows, inner // 32, 2)
    out[..., 2:] = q.view(np.uint8)
    return out.reshape(rows, -1)


def _pack_kscales(sc: np.ndarray, m: np.ndarray) -> np.ndarray:
    """8 six-bit scales + 8 six-bit mins -> 12 bytes (inverse of
    src/Dequant.jl:345-362 unpack)."""
    sc = sc.astype(np.uint8)
    m = m.astype(np.uint8)
    out = np.zeros(sc.shape[:-1] + (12,), np.uint8)
    for j in range(4):
        out[..., j] = (sc[..., j] & 63) | ((sc[..., j + 4] >> 4) << 6)
        out[..., j + 4] = (m[..., j] & 63) | ((m[..., j + 4] >> 4) << 6)
        out[..., j + 8] = (sc[..., j + 4] & 15) | ((m[..., j + 4] & 15) << 4)
    return out


def _kquant_affine(w, nlev):
    """Shared scale/min search for Q4_K (nlev=15) and Q5_K (nlev=31).
    Returns d16, dmin16 (nb,), sc, m (nb,8) and q (nb,256) in [0, nlev]."""
    nb = w.shape[0]
    sub = w.reshape(nb, 8, 32)
    mn = np.minimum(sub.min(-1), 0.0)
    mx = sub.max(-1)
    scale = (mx - mn) / nlev
    mins = -mn
    dmax = scale.max(-1)
    mmax = mins.max(-1)
    d16 = _f16(dmax / 63.0)
    dmin16 = _f16(mmax / 63.0)
    d = d16.astype(np.float32)
    dmin = dmin16.astype(np.float32)
    sc = np.clip(np.rint(np.where(d[:, None] > 0, scale / np.where(d[:, None] > 0, d[:, None], 1), 0)), 0, 63)
    m = np.clip(np.rint(np.where(dmin[:, None] > 0, mins / np.where(dmin[:, None] > 0, dmin[:, None], 1), 0)), 0, 63)
    d1 = (d[:, None] * sc).astype(np.float32)
    m1 = (dmin[:, None] * m).astype(np.float32)
    q = np.rint((sub + m1[..., None]) / np.where(d1 > 0, d1, 1)[..., None])
    q = np.where(d1[..., None] > 0, q, 0)
    q = np.clip(q, 0, nlev).astype(np.uint8).reshape(nb, 256)
    return d16, dmin16, sc.astype(np.uint8), m.astype(np.uint8), q


def pack_q4_k(w: np.ndarray) -> np.ndarray:
    rows, inner = w.shape
    nb = rows * inner // 256
    d16, dmin16, sc, m, q = _kquant_affine(w.reshape(nb, 256).astype(np.float32), 15)
    out = np.empty((nb, 144), np.uint8)
    out[:, 0:2] = d16.view(np.uint8).reshape(nb, 2)
    out[:, 2:4] = dmin16.view(np.uint8).reshape(nb, 2)
    out[:, 4:16] = _pack_kscales(sc, m)
    qq = q.reshape(nb, 4, 2, 32)           # [j][lo/hi][l]
    out[:, 16:] = (qq[:, :, 0, :] | (qq[:, :, 1, :] << 4)).reshape(nb, 128)
    return out.reshape(rows, -1)


def pack_q5_k(w: np.ndarray) -> np.ndarray:
    rows, inner = w.shape
    nb = rows * inner // 256
    d16, dmin16, sc, m, q = _kquant_affine(w.reshape(nb, 256).astype(np.float32), 31)
    out = np.empty((nb, 176), np.uint8)
    out[:, 0:2] = d16.view(np.uint8).reshape(nb, 2)
    out[:, 2:4] = dmin16.view(np.uint8).reshape(nb, 2)
    out[:, 4:16] = _pack_kscales(sc, m)
    qq = q.reshape(nb, 4, 2, 32)
    lo = qq & 15
    hi = (qq >> 4) & 1
    out[:, 48:] = (lo[:, :, 0, :] | (lo[:, :, 1, :] << 4)).reshape(nb, 128)
    qh = np.zeros((nb, 32), np.uint8)
    for j in range(4):
        qh |= hi[:, j, 0, :] << (2 * j)
        qh |= hi[:, j, 1, :] << (2 * j + 1)
    out[:, 16:48] = qh
    return out.reshape(rows, -1)


def pack_q6_k(w: np.ndarray) -> np.ndarray:
    rows, inner = w.shape
    nb = rows * inner // 256
    b = w.reshape(nb, 16, 16).astype(np.float32)
    amax = np.abs(b).max(-1)                    # (nb,16)
    scale = amax / 31.0
    d16 = _f16(scale.max(-1) / 127.0)
    d = d16.astype(np.float32)
    isc = np.clip(np.rint(np.where(d[:, None] > 0, scale / np.where(d[:, None] > 0, d[:, None], 1), 0)), 0, 127).astype(np.int8)
    eff = (d[:, None] * isc.astype(np.float32))
    q = np.rint(b / np.where(eff > 0, eff, 1)[..., None])
    q = np.where(eff[..., None] > 0, q, 0)
    raw = (np.clip(q, -32, 31) + 32).astype(np.uint8).reshape(nb, 2, 4, 32)   # [n][k][l]
    out = np.empty((nb, 210), np.uint8)
    ql = np.empty((nb, 2, 2, 32), np.uint8)
    ql[:, :, 0, :] = (raw[:, :, 0, :] & 15) | ((raw[:, :, 2, :] & 15) << 4)
    ql[:, :, 1, :] = (raw[:, :, 1, :] & 15) | ((raw[:, :, 3, :] & 15) << 4)
    qh = ((raw[:, :, 0, :] >> 4) | ((raw[:, :, 1, :] >> 4) << 2) |
          ((raw[:, :, 2, :] >> 4) << 4) | ((raw[:, :, 3, :] >> 4) << 6))
    out[:, 0:128] = ql.reshape(nb, 128)
    out[:, 128:192] = qh.reshape(nb, 64)
    out[:, 192:208] = isc.view(np.uint8)
    out[:, 208:210] = d16.view(np.uint8).reshape(nb, 2)
    return out.reshape(rows, -1)


def pack_iq2_xxs(w: np.ndarray) -> np.ndarray:
    """IQ2_XXS with Inferno's decode (grid byte - 8, src/Dequant.jl:46):
    magnitudes {0, 17, 35} * db with db = d*(0.5+s)*0.25, s 4-bit per 32."""
    rows, inner = w.shape
    nb = rows * inner // 256
    b = w.reshape(nb, 8, 4, 8).astype(np.float32)          # [blk][ib32][l][j]
    amax = np.abs(b).reshape(nb, 8, 32).max(-1)            # (nb,8)
    want_db = amax / 35.0
    d16 = _f16(want_db.max(-1) / (15.5 * 0.25))
    d = d16.astype(np.float32)
    s = np.clip(np.rint(np.where(d[:, None] > 0, want_db / np.where(d[:, None] > 0, d[:, None], 1) / 0.25 - 0.5, 0)), 0, 15).astype(np.uint32)
    db = (d[:, None] * (0.5 + s.astype(np.float32))) * 0.25
    mag = np.abs(b) / np.where(db > 0, db, 1)[:, :, None, None]
    neg = b < 0
    # even sign parity: flip the smallest-magnitude element if needed
    par = neg.sum(-1) & 1
    flip_idx = np.argmin(mag, axis=-1)
    fl = np.zeros_like(neg)
    np.put_along_axis(fl, flip_idx[..., None], (par == 1)[..., None], axis=-1)
    neg = neg ^ fl
    gvals = IQ2XXS_GRID_BYTES.astype(np.float32) - 8.0       # (256,8)
    flat = mag.reshape(-1, 8)
    dist = (gvals ** 2).sum(-1)[None, :] - 2.0 * flat @ gvals.T
    gidx = np.argmin(dist, axis=-1).astype(np.uint32).reshape(nb, 8, 4)
    sbits = np.zeros((nb, 8, 4), np.uint32)
    for j in range(7):
        sbits |= neg[..., j].astype(np.uint32) << j
    aux1 = gidx[..., 0] | (gidx[..., 1] << 8) | (gidx[..., 2] << 16) | (gidx[..., 3] << 24)
    aux2 = sbits[..., 0] | (sbits[..., 1] << 7) | (sbits[..., 2] << 14) | (sbits[..., 3] << 21) | (s << 28)
    out = np.empty((nb, 66), np.uint8)
    out[:, 0:2] = d16.view(np.uint8).reshape(nb, 2)
    q = np.stack([aux1, aux2], -1).astype("<u4")             # (nb,8,2)
    out[:, 2:] = q.view(np.uint8).reshape(nb, 64)
    return out.reshape(rows, -1)


PACKERS = {Q8_0: pack_q8_0, Q4_K: pack_q4_k, Q5_K: pack_q5_k, Q6_K: pack_q6_k,
           IQ2_XXS: pack_iq2_xxs}


def quantize(w: np.ndarray, ggml_type: int, chunk_rows: int = 1 << 14) -> np.ndarray:
    """(rows, inner) fp32 -> (rows, row_bytes) uint8 in GGUF layout."""
    w = np.asarray(w, dtype=np.float32)
    if ggml_type == F32:
        return w.view(np.uint8).reshape(w.shape[0], -1).copy()
    if ggml_type == F16:
        return w.astype(np.float16).view(np.uint8).reshape(w.shape[0], -1).copy()
    rb = row_bytes(ggml_type, w.shape[1])
    out = np.empty((w.shape[0], rb), np.uint8)
    for r0 in range(0, w.shape[0], chunk_rows):
        out[r0:r0 + chunk_rows] = PACKERS[ggml_type](w[r0:r0 + chunk_rows])
    return out


def random_quant_matrix(rng: np.random.Generator, rows: int, inner: int, ggml_type: int,
                        std: float = 0.02, chunk_rows: int = 1 << 13, pool: int = 0) -> np.ndarray:
    """N(0, std) matrix quantized chunk by chunk (bounded host memory).

    pool > 0 (throughput runs of the multi-GB configs): quantize `pool` rows
    and fill the matrix with rows drawn from them at random -- the same value
    distribution and byte count, without quantizing billions of weights."""
    rb = row_bytes(ggml_type, inner)
    if pool and rows > pool:
        base = random_quant_matrix(rng, pool, inner, ggml_type, std, chunk_rows)
        return base[rng.integers(0, pool, rows)]
    out = np.empty((rows, rb), np.uint8)
    for r0 in range(0, rows, chunk_rows):
        n = min(chunk_rows, rows - r0)
        w = rng.standard_normal((n, inner), dtype=np.float32) * np.float32(std)
        out[r0:r0 + n] = quantize(w, ggml_type)
    return out


# ----------------------------------------------------------------------------
# model specs (4, 5 and a small test model)
# ----------------------------------------------------------------------------
@dataclasses.dataclass
class ModelSpec:
    name: str
    hidden: int
    layers: int
    n_heads: int
    n_kv: int
    head_dim: int
    ffn: int
    vocab: int
    ssm_nv: int          # GDN value heads
    ssm_nk: int          # GDN q/k heads (ssm.group_count)
    ssm_dk: int = 128
    ssm_dv: int = 128
    conv_k: int = 4
    interval: int = 4    # full attention at (i+1) % interval == 0
    ctx: int = 640
    eps: float = 1e-6
    rope_theta: float = 1e7
    partial_rotary: float = 0.25
    n_experts: int = 0
    n_experts_used: int = 0
    expert_ffn: int = 0
    shexp_ffn: int = 0
    # quantization mix
    t_attn: int = Q4_K      # attn_q/k/output, attn_qkv, attn_gate, ssm_out
    t_attn_v: int = Q4_K
    t_ffn_gu: int = Q4_K
    t_ffn_down: int = Q6_K
    t_embd: int = Q6_K
    t_exp_gu: int = IQ2_XXS
    t_exp_down: int = Q4_K

    @property
    def d_inner(self):
        return self.ssm_nv * self.ssm_dv

    @property
    def conv_channels(self):
        return 2 * self.ssm_nk * self.ssm_dk + self.d_inner

    def is_attn(self, i):
        return (i + 1) % self.interval == 0


CONFIGS = {
    # config 1: Qwen3.5-0.8B-shaped hybrid
    "qwen35-0.8b": ModelSpec("qwen35-0.8b", hidden=1024, layers=24, n_heads=8, n_kv=2,
                             head_dim=256, ffn=3584, vocab=248320, ssm_nv=16, ssm_nk=16),
    # config 4: Qwen3.5-9B-shaped hybrid, Q4_K_M mix (Q6_K ffn_down/attn_v/embd)
    "qwen35-9b": ModelSpec("qwen35-9b", hidden=4096, layers=32, n_heads=16, n_kv=4,
                           head_dim=256, ffn=12288, vocab=248320, ssm_nv=32, ssm_nk=16,
                           ctx=32768 + 128, t_attn_v=Q6_K),
    # config 5: Qwen3.5-35B-A3B-shaped MoE hybrid
    "qwen35-35b-a3b": ModelSpec("qwen35-35b-a3b", hidden=2048, layers=40, n_heads=16, n_kv=2,
                                head_dim=256, ffn=0, vocab=248320, ssm_nv=32, ssm_nk=16,
                                ctx=4096 + 128, n_experts=256, n_experts_used=8,
                                expert_ffn=512, shexp_ffn=512),
    # small model with the same kernel shapes (dk=dv=128, head_dim 256, nk != nv)
    "tiny": ModelSpec("tiny", hidden=512, layers=4, n_heads=4, n_kv=2, head_dim=256,
                      ffn=1024, vocab=4096, ssm_nv=4, ssm_nk=2, ctx=256),
    # tensor-parallel test models: GDN QK groups / heads / FFN split on super-block boundaries
    "tiny-tp": ModelSpec("tiny-tp", hidden=512, layers=4, n_heads=4, n_kv=2, head_dim=256,
                         ffn=1024, vocab=4096, ssm_nv=8, ssm_nk=4, ctx=256),
    "small-tp": ModelSpec("small-tp", hidden=1024, layers=4, n_heads=16, n_kv=4, head_dim=256,
                          ffn=2048, vocab=8192, ssm_nv=32, ssm_nk=16, ctx=256),
    "tiny-moe": ModelSpec("tiny-moe", hidden=512, layers=4, n_heads=4, n_kv=2, head_dim=256,
                          ffn=0, vocab=4096, ssm_nv=4, ssm_nk=2, ctx=256, n_experts=16,
                          n_experts_used=4, expert_ffn=256, shexp_ffn=256),
}


def _f32_tensor(a: np.ndarray, ne) -> Tensor:
    a = np.ascontiguousarray(a, dtype=np.float32)
    return Tensor(F32, tuple(ne), a.view(np.uint8).reshape(-1))


def _q_tensor(rng, ggml_type, rows, inner, std=0.02, pool=0) -> Tensor:
    data = random_quant_matrix(rng, rows, inner, ggml_type, std, pool=pool)
    return Tensor(ggml_type, (inner, rows), data.reshape(-1))


def make_model(spec: ModelSpec, seed: int = 0, layers: int | None = None, pool: int = 0) -> dict:
    """Return {name: Tensor} for a seeded model of ``spec`` (optionally only the
    first ``layers`` layers -- used by tests to bound memory).  pool > 0 draws
    the rows of every quantized matrix from `pool` quantized rows (see
    random_quant_matrix): for throughput runs of the 9B / MoE configs."""
    rng = np.random.Generator(np.random.PCG64(seed))

    def qt(rng, t, rows, inner, std=0.02):
        return _q_tensor(rng, t, rows, inner, std, pool=pool)
    H = spec.hidden
    T = {}

    def norm(n):
        return (1.0 + 0.02 * rng.standard_normal(n)).astype(np.float32)

    T["token_embd.weight"] = qt(rng, spec.t_embd, spec.vocab, H)
    T["output_norm.weight"] = _f32_tensor(norm(H), (H,))
    nl = spec.layers if layers is None else layers
    for i in range(nl):
        p = f"blk.{i}."
        T[p + "attn_norm.weight"] = _f32_tensor(norm(H), (H,))
        T[p + "post_attention_norm.weight"] = _f32_tensor(norm(H), (H,))
        if spec.is_attn(i):
            hd = spec.head_dim
            T[p + "attn_q.weight"] = qt(rng, spec.t_attn, 2 * spec.n_heads * hd, H)
            T[p + "attn_k.weight"] = qt(rng, spec.t_attn, spec.n_kv * hd, H)
            T[p + "attn_v.weight"] = qt(rng, spec.t_attn_v, spec.n_kv * hd, H)
            T[p + "attn_output.weight"] = qt(rng, spec.t_attn, H, spec.n_heads * hd)
            T[p + "attn_q_norm.weight"] = _f32_tensor(norm(hd), (hd,))
            T[p + "attn_k_norm.weight"] = _f32_tensor(norm(hd), (hd,))
        else:
            cc, di = spec.conv_channels, spec.d_inner
            T[p + "attn_qkv.weight"] = qt(rng, spec.t_attn, cc, H)
            T[p + "attn_gate.weight"] = qt(rng, spec.t_attn, di, H)
            T[p + "ssm_out.weight"] = qt(rng, spec.t_attn, H, di)
            conv = (0.5 * rng.standard_normal((cc, spec.conv_k))).astype(np.float32)
            T[p + "ssm_conv1d.weight"] = _f32_tensor(conv, (spec.conv_k, cc))
            T[p + "ssm_alpha.weight"] = _f32_tensor(
                0.02 * rng.standard_normal((spec.ssm_nv, H)), (H, spec.ssm_nv))
            T[p + "ssm_beta.weight"] = _f32_tensor(
                0.02 * rng.standard_normal((spec.ssm_nv, H)), (H, spec.ssm_nv))
            a = -np.exp(rng.uniform(math.log(0.01), 0.0, spec.ssm_nv))
            T[p + "ssm_a"] = _f32_tensor(a, (spec.ssm_nv,))
            T[p + "ssm_dt.bias"] = _f32_tensor(np.zeros(spec.ssm_nv), (spec.ssm_nv,))
            T[p + "ssm_norm.weight"] = _f32_tensor(norm(spec.ssm_dv), (spec.ssm_dv,))
        if spec.n_experts:
            E, Ie = spec.n_experts, spec.expert_ffn
            T[p + "ffn_gate_inp.weight"] = _f32_tensor(
                0.02 * rng.standard_normal((E, H)), (H, E))
            for nm, t, rows, inner in (("ffn_gate_exps", spec.t_exp_gu, Ie, H),
                                       ("ffn_up_exps", spec.t_exp_gu, Ie, H),
                                       ("ffn_down_exps", spec.t_exp_down, H, Ie)):
                data = random_quant_matrix(rng, rows * E, inner, t, pool=pool)
                T[p + nm + ".weight"] = Tensor(t, (inner, rows, E), data.reshape(-1))
            if spec.shexp_ffn:
                S = spec.shexp_ffn
                T[p + "ffn_gate_shexp.weight"] = qt(rng, Q4_K, S, H)
                T[p + "ffn_up_shexp.weight"] = qt(rng, Q4_K, S, H)
                T[p + "ffn_down_shexp.weight"] = qt(rng, Q4_K, H, S)
        else:
            T[p + "ffn_gate.weight"] = qt(rng, spec.t_ffn_gu, spec.ffn, H)
            T[p + "ffn_up.weight"] = qt(rng, spec.t_ffn_gu, spec.ffn, H)
            T[p + "ffn_down.weight"] = qt(rng, spec.t_ffn_down, H, spec.ffn)
    return T


def metadata(spec: ModelSpec) -> dict:
    """GGUF metadata under both the ``qwen35.*`` keys real files carry and the
    ``qwen3.*`` keys src/LoaderCPU.jl:393-418 reads."""
    md = {"general.architecture": "qwen35"}
    vals = {
        "vocab_size": spec.vocab, "embedding_length": spec.hidden,
        "feed_forward_length": spec.ffn, "block_count": spec.layers,
        "attention.head_count": spec.n_heads, "attention.head_count_kv": spec.n_kv,
        "attention.key_length": spec.head_dim,
        "attention.layer_norm_rms_epsilon": float(spec.eps),
        "rope.freq_base": float(spec.rope_theta), "context_length": spec.ctx,
        "rope.partial_rotary_factor": float(spec.partial_rotary),
        "full_attention_interval": spec.interval,
        "ssm.inner_size": spec.d_inner, "ssm.state_size": spec.ssm_dk,
        "ssm.group_count": spec.ssm_nk, "ssm.time_step_rank": spec.ssm_nv,
        "ssm.conv_kernel": spec.conv_k,
    }
    if spec.n_experts:
        vals.update({"expert_count": spec.n_experts, "expert_used_count": spec.n_experts_used,
                     "expert_feed_forward_length": spec.expert_ffn,
                     "expert_shared_feed_forward_length": spec.shexp_ffn})
    for k, v in vals.items():
        md["qwen35." + k] = v
        md["qwen3." + k] = v
    return md


def write_gguf(path, spec: ModelSpec, tensors: dict) -> None:
    import gguf
    w = gguf.GGUFWriter(str(path), "qwen35")
    for k, v in metadata(spec).items():
        if k == "general.architecture":
            continue
        if isinstance(v, float):
            w.add_float32(k, v)
        elif isinstance(v, int):
            w.add_uint32(k, v)
        else:
            w.add_string(k, v)
    for name, t in tensors.items():
        shape = tuple(reversed(t.ne))                     # numpy order
        if t.ggml_type == F32:
            w.add_tensor(name, t.data.view(np.float32).reshape(shape))
        else:
            qk, bb = BLOCK[t.ggml_type]
            byte_shape = shape[:-1] + (shape[-1] // qk * bb,)
            w.add_tensor(name, t.data.reshape(byte_shape),
                         raw_dtype=gguf.GGMLQuantizationType(t.ggml_type))
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()


def tokens(seed: int, n: int, vocab: int) -> np.ndarray:
    """Prompt token ids (0-based) drawn from PCG64(seed + 1)."""
    rng = np.random.Generator(np.random.PCG64(seed + 1))
    return rng.integers(0, vocab, n).astype(np.int32)
