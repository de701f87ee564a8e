"""Tensor-parallel sharding of a Qwen3.5-hybrid model's GGUF tensors.

One process per GPU; rank r of N holds (layout of the engine's local model):

* Gated DeltaNet (src/ModelCPU.jl:531-700): the QK groups G_r = [r*nk/N,
  (r+1)*nk/N) and, because of the modulo head map g = h % nk (:587), the V
  heads {g + j*nk : g in G_r}.  Local V head h_l = g_l + j*nk_l stands for
  global head g0 + g_l + j*nk, so the local model again satisfies
  h_l % nk_l == g_l.  in_proj / attn_gate rows, conv channels, alpha / beta /
  ssm_a / dt_bias entries follow; ssm_out keeps all rows and takes the columns
  of the local heads (runs of nk_l * dv columns, super-block aligned when
  nk_l * dv % 256 == 0), so its output is a partial sum.
* Gated attention (:756-856): query heads [r*nh/N, (r+1)*nh/N) (rows
  [q | gate] per head), their KV heads (blocked GQA, kv = h / (nh/nkv)),
  replicated when nkv < N; attn_output takes the matching columns.
* FFN (:447-473): gate/up rows [r*I/N, (r+1)*I/N), down the matching columns.
* Norms and token_embd are replicated; the engine itself takes rows
  [r*V/N, (r+1)*V/N) of the tied lm_head and all-reduces the packed argmax.

The partial outputs of ssm_out / attn_output / ffn_down are summed by an
all-reduce of the residual stream in the engine (rank 0 adds the residual,
the others contribute their partial only).
"""
from __future__ import annotations

import dataclasses

import numpy as np

from . import synth as S


def _layout(t: S.Tensor):
    """(rows, inner, block elements, block bytes) of a 2-D-like tensor."""
    inner = int(t.ne[0])
    rows = int(np.prod(t.ne[1:])) if len(t.ne) > 1 else 1
    if t.ggml_type == S.F32:
        return rows, inner, 1, 4
    qk = 32 if t.ggml_type == S.Q8_0 else 256
    return rows, inner, qk, S.row_bytes(t.ggml_type, qk)


def take_rows(t: S.Tensor, rows_idx) -> S.Tensor:
    rows, inner, qk, bb = _layout(t)
    rb = inner // qk * bb
    a = t.data.reshape(rows, rb)[np.asarray(rows_idx, np.int64)]
    ne = (inner, len(rows_idx)) + tuple(t.ne[2:]) if len(t.ne) > 2 else (inner, len(rows_idx))
    return S.Tensor(t.ggml_type, ne, np.ascontiguousarray(a).reshape(-1))


def take_entries(t: S.Tensor, idx) -> S.Tensor:
    """1-D F32 tensor entries."""
    a = t.data.view(np.float32)[np.asarray(idx, np.int64)]
    return S.Tensor(t.ggml_type, (len(idx),), np.ascontiguousarray(a).view(np.uint8).reshape(-1))


def take_cols(t: S.Tensor, runs) -> S.Tensor:
    """Columns (input elements) given as [(c0, c1), ...] runs, each aligned to
    the block size of the type."""
    rows, inner, qk, bb = _layout(t)
    a = t.data.reshape(rows, inner // qk, bb)
    parts = []
    for c0, c1 in runs:
        if c0 % qk or c1 % qk:
            raise ValueError(f"column run [{c0}, {c1}) not aligned to {qk}-element blocks")
        parts.append(a[:, c0 // qk:c1 // qk])
    b = np.concatenate(parts, axis=1)
    new_inner = sum(c1 - c0 for c0, c1 in runs)
    return S.Tensor(t.ggml_type, (new_inner,) + tuple(t.ne[1:]), np.ascontiguousarray(b).reshape(-1))


def check(spec: S.ModelSpec, n: int) -> None:
    """Raise ValueError when `spec` cannot be split over n ranks."""
    if n < 1:
        raise ValueError("tp size must be >= 1")
    if spec.n_experts:
        raise ValueError("tensor parallelism of MoE layers is not supported")
    nk_l = spec.ssm_nk // n if spec.ssm_nk % n == 0 else 0
    errs = []
    if not nk_l or (nk_l * spec.ssm_dv) % 256:
        errs.append(f"GDN: {spec.ssm_nk} QK groups over {n} ranks must leave a 256-column multiple per run")
    if spec.n_heads % n:
        errs.append(f"attention: {spec.n_heads} heads over {n} ranks")
    elif not (spec.n_kv % n == 0 or (n % spec.n_kv == 0 and (spec.n_heads // spec.n_kv) % (spec.n_heads // n) == 0)):
        errs.append(f"attention: {spec.n_kv} KV heads cannot be split or replicated over {n} ranks")
    if spec.ffn % n or (spec.ffn // n) % 256:
        errs.append(f"FFN: {spec.ffn} over {n} ranks is not a 256 multiple")
    if spec.vocab % n:
        errs.append(f"lm_head: vocab {spec.vocab} over {n} ranks")
    if errs:
        raise ValueError("; ".join(errs))


def local_spec(spec: S.ModelSpec, n: int) -> S.ModelSpec:
    check(spec, n)
    nkv_l = spec.n_kv // n if spec.n_kv % n == 0 else 1
    return dataclasses.replace(spec, n_heads=spec.n_heads // n, n_kv=nkv_l, ffn=spec.ffn // n,
                               ssm_nv=spec.ssm_nv // n, ssm_nk=spec.ssm_nk // n)


def gdn_local_heads(spec: S.ModelSpec, rank: int, n: int) -> list:
    """Global V heads of rank `rank` in local order h_l = g_l + j * nk_l."""
    nk, nv = spec.ssm_nk, spec.ssm_nv
    nk_l = nk // n
    g0 = rank * nk_l
    return [g0 + gl + j * nk for j in range(nv // nk) for gl in range(nk_l)]


def shard_experts(spec: S.ModelSpec, tensors: dict, rank: int, n: int) -> dict:
    """Expert parallelism for MoE models: rank r keeps
    routed experts [r*E/n, (r+1)*E/n) of every ffn_{gate,up,down}_exps tensor
    (GGUF ne = [in, out, E], experts contiguous); every other tensor -- router,
    shared expert, attention, GDN, embedding -- is replicated.  The engine
    computes the router and top-k on every rank, evaluates only its own
    selected experts and sums the ranks' partial FFN outputs."""
    E = spec.n_experts
    if E % n:
        raise ValueError(f"{E} experts over {n} ranks")
    el = E // n
    out = {}
    for name, t in tensors.items():
        if name.endswith("_exps.weight"):
            per = t.nbytes // E
            a = t.data.reshape(E, per)[rank * el:(rank + 1) * el]
            t = S.Tensor(t.ggml_type, tuple(t.ne[:2]) + (el,), np.ascontiguousarray(a).reshape(-1))
        out[name] = t
    return out


def shard(spec: S.ModelSpec, tensors: dict, rank: int, n: int):
    """(local spec, local tensors) of `rank` in an n-way split: tensor
    parallel for dense models, expert parallel for MoE models (the local spec
    then keeps the global dimensions)."""
    if n == 1:
        return spec, dict(tensors)
    if spec.n_experts:
        return spec, shard_experts(spec, tensors, rank, n)
    ls = local_spec(spec, n)
    H, dk, dv, hd = spec.hidden, spec.ssm_dk, spec.ssm_dv, spec.head_dim
    nk, nk_l = spec.ssm_nk, ls.ssm_nk
    g0 = rank * nk_l
    heads = gdn_local_heads(spec, rank, n)
    q_ch = list(range(g0 * dk, (g0 + nk_l) * dk))
    k_ch = [nk * dk + c for c in q_ch]
    v_ch = [2 * nk * dk + h * dv + i for h in heads for i in range(dv)]
    z_rows = [h * dv + i for h in heads for i in range(dv)]
    # ssm_out column runs: consecutive local heads of one j-slice are contiguous globally
    ssm_runs = [((g0 + j * nk) * dv, (g0 + j * nk + nk_l) * dv) for j in range(spec.ssm_nv // nk)]
    nh_l = ls.n_heads
    h0 = rank * nh_l
    if spec.n_kv % n == 0:
        kv_heads = list(range(rank * ls.n_kv, (rank + 1) * ls.n_kv))
    else:
        kv_heads = [h0 // (spec.n_heads // spec.n_kv)]
    I_l = ls.ffn
    ffn_rows = list(range(rank * I_l, (rank + 1) * I_l))

    out = {}
    for name, t in tensors.items():
        if not name.startswith("blk."):
            out[name] = t
            continue
        i = int(name.split(".")[1])
        key = name.split(".", 2)[2]
        if spec.is_attn(i):
            if key == "attn_q.weight":
                t = take_rows(t, range(h0 * 2 * hd, (h0 + nh_l) * 2 * hd))
            elif key in ("attn_k.weight", "attn_v.weight"):
                t = take_rows(t, [kv * hd + d for kv in kv_heads for d in range(hd)])
            elif key == "attn_output.weight":
                t = take_cols(t, [(h0 * hd, (h0 + nh_l) * hd)])
        else:
            if key == "attn_qkv.weight":
                t = take_rows(t, q_ch + k_ch + v_ch)
            elif key == "ssm_conv1d.weight":
                t = take_rows(t, q_ch + k_ch + v_ch)     # ne (K, C): channel c is a row of K taps
            elif key == "attn_gate.weight":
                t = take_rows(t, z_rows)
            elif key in ("ssm_alpha.weight", "ssm_beta.weight"):
                t = take_rows(t, heads)
            elif key in ("ssm_a", "ssm_dt.bias"):
                t = take_entries(t, heads)
            elif key == "ssm_out.weight":
                t = take_cols(t, ssm_runs)
        if key in ("ffn_gate.weight", "ffn_up.weight"):
            t = take_rows(t, ffn_rows)
        elif key == "ffn_down.weight":
            t = take_cols(t, [(rank * I_l, (rank + 1) * I_l)])
        out[name] = t
    return ls, out
