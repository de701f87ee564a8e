#!/usr/bin/env python
"""Decode throughput of the B200 engine on BASELINE config 1.

Workload: Qwen3.5-0.8B-shaped hybrid (hidden 1024,
24 layers [3 GDN + 1 gated attention] x 6, Q4_K/Q6_K, vocab 248320 tied),
seeded N(0,0.02) weights in GGUF block formats, 32 seeded prompt tokens,
greedy decode of 128 tokens at batch 1, KV capacity 512.

One "step" = restore the post-prompt state (device snapshot) and decode the
128 tokens (positions 32..159) with the captured CUDA graphs.  `value` is
decode tokens/s over the K timed steps (whole job: summed over ranks; config 1
does not shard, so N GPUs run N independent replicas -> weak scaling).
`e2e` is the same metric through the public API with host buffers: reset,
prompt upload, prefill, 128 decode tokens and the token read-back, per step.

--impl reference times the reference's CPU path (the C++ restatement in
oracle/, F32 dequantized weights, all host threads -- what load_model_cpu +
forward_cpu! do by default) on a bounded sample of the same workload.
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "inferno.jl_b200"))

METRIC = "decode tokens/s @batch1 (Qwen3.5-0.8B-shaped hybrid, Q4_K/Q6_K)"
UNIT = "tokens/s"
PROMPT, NDEC, CTX, SEED = 32, 128, 512, 0
CONFIG = {"workload": "config1 qwen35-0.8b-shaped hybrid, 32-token prompt, greedy decode 128 @batch1, ctx 512",
          "model": "qwen35-0.8b-shaped (random-init, seeded)", "global_batch": 1, "seq_len": PROMPT + NDEC,
          "parallelism": "replicas", "l2": "weights 515 MB per token > 126 MB L2 (no flush needed)"}


def dist_env():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return ws, rank, local


class ClockSampler:
    """nvidia-smi clock / throttle samples during the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu: int):
        self.gpu = gpu
        self.lines = []
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            threading.Thread(target=self._read, daemon=True).start()
        except Exception:
            self.proc = None

    def _read(self):
        for ln in self.proc.stdout:
            self.lines.append(ln.strip())

    def stop(self) -> dict:
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for nm, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(nm)
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


def max_over_ranks(v: float, device: str = "cuda") -> float:
    """Max of a per-rank scalar over all ranks (device times: slowest rank)."""
    import torch
    import torch.distributed as dist
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return float(v)
    t = torch.tensor([float(v)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def build_model(spec_name="qwen35-0.8b"):
    from inferno_b200 import synth as S
    spec = S.CONFIGS[spec_name]
    T = S.make_model(spec, seed=SEED)
    return spec, T


def cpu_baseline(spec, T, tokens_to_decode=6, prefill=2) -> dict:
    """The oracle (reference CPU path restated) on a bounded sample: `prefill`
    prompt tokens then `tokens_to_decode` greedy tokens, all host threads."""
    sys.path.insert(0, str(ROOT / "oracle"))
    import oracle as O
    from inferno_b200 import synth as S
    m = O.OracleModel(spec, T)
    prompt = S.tokens(SEED, prefill, spec.vocab)
    m.reset()
    tok, _ = m.forward(prompt, 0, want_logits=False)
    pos = len(prompt)
    # warm-up token (excluded), then timed tokens
    tok, _ = m.forward([tok], pos, want_logits=False)
    pos += 1
    t0 = time.perf_counter()
    for _ in range(tokens_to_decode):
        tok, _ = m.forward([tok], pos, want_logits=False)
        pos += 1
    dt = time.perf_counter() - t0
    return {"value": tokens_to_decode / dt, "unit": UNIT, "cores": O.cpu_count(), "kind": "port",
            "sample": f"config1 model, {prefill}-token prompt, {tokens_to_decode} timed greedy decode tokens "
                      f"(positions {prefill + 1}..{prefill + tokens_to_decode}), F32 dequantized weights, "
                      f"OpenMP over {O.cpu_count()} threads"}


def reference_kernel_gbs(T, reps=5) -> dict | None:
    """The reference's own quantized GEMV (src/kernels/quant_kernels.c
    q6_k_gemv, compiled from source into oracle/_ref) on the dominant kernel's
    shape -- the tied lm_head, Q6_K 248320 x 1024 -- on the host cores, for
    comparison with the GPU kernel's `roofline.achieved`.  None when the
    reference library is not built."""
    try:
        sys.path.insert(0, str(ROOT / "oracle"))
        import oracle as O
        L = O.ref_lib()
        if L is None:
            return None
        t = T["token_embd.weight"]
        inner, rows = int(t.ne[0]), int(t.ne[1])
        x = np.random.default_rng(SEED).standard_normal(inner).astype(np.float32)
        O.ref_gemv(14, t.data, x, inner, rows, L)                  # warm-up
        t0 = time.perf_counter()
        for _ in range(reps):
            O.ref_gemv(14, t.data, x, inner, rows, L)
        dt = (time.perf_counter() - t0) / reps
        return {"kernel": "reference q6_k_gemv (Q8_K activations, AVX2 + FMA, OpenMP)", "shape": [rows, inner],
                "ms": 1e3 * dt, "gbs": t.data.nbytes / dt / 1e9, "threads": O.cpu_count(),
                "note": "the reference's own C kernel on the lm_head bytes, host cores"}
    except Exception:
        return None


def run_reference(args):
    ws, rank, _ = dist_env()
    if rank != 0:
        return 0
    spec, T = build_model()
    sys.path.insert(0, str(ROOT / "oracle"))
    import oracle as O
    from inferno_b200 import synth as S
    m = O.OracleModel(spec, T)
    prompt = S.tokens(SEED, PROMPT, spec.vocab)
    per_step = 4   # decode tokens per reference step (bounded sample)

    def step(tok, pos):
        for _ in range(per_step):
            tok, _ = m.forward([tok], pos, want_logits=False)
            pos += 1
        return tok, pos

    # the workload's schedule: the 32-token prompt (untimed), then greedy
    # decode from position 32; a step decodes `per_step` tokens, continuing
    # the same sequence (positions stay inside the 32..159 window for the
    # default --steps / --warmup; later steps wrap back to the prompt state)
    m.reset()
    tok, _ = m.forward(prompt, 0, want_logits=False)
    pos = PROMPT
    snap = (tok, pos)
    for _ in range(args.warmup):
        tok, pos = step(tok, pos)
    dt = 0.0
    for _ in range(args.steps):
        if pos + per_step > PROMPT + NDEC:
            # window exhausted: replay the post-prompt state (untimed)
            m.reset()
            tok, _ = m.forward(prompt, 0, want_logits=False)
            pos = PROMPT
        t0 = time.perf_counter()
        tok, pos = step(tok, pos)
        dt += time.perf_counter() - t0
    v = per_step * args.steps / dt
    line = {"metric": METRIC, "value": v, "unit": UNIT, "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": dt * 1000 / args.steps, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded)",
            "config": dict(CONFIG, parallelism="host CPU"), "impl": "reference",
            "cpu_baseline": {"value": v, "unit": UNIT, "cores": O.cpu_count(), "kind": "port",
                             "sample": f"{per_step} greedy decode tokens per step after the {PROMPT}-token "
                                       f"prompt (positions {PROMPT}..{PROMPT + NDEC - 1}), F32 dequantized "
                                       "weights, all host threads (the reference's default load_model_cpu "
                                       "path, restated)"},
            "e2e": {"value": v, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


# Kernel classes of the per-token graph, with the INFERNO_B200_ABLATE bits
# that leave them out: the marginal device time of a class inside the
# PDL-chained graph is (token time) - (token time without the class).
# Ablated runs compute garbage; only their timing is used.
GRAPH_CLASSES = {"q4k_gemv": 1 | 8 | 16, "q6k_ffn_down": 32, "gdn": 2, "attention": 4, "lm_head": 64}


def q4k_launch_bytes(spec, T):
    """Algorithmic bytes of the config-1 Q4_K per-layer GEMVs of one token:
    weights once plus fp32 input and output vectors, and their launch count."""
    tot, n = 0, 0
    for i in range(spec.layers):
        p = f"blk.{i}."
        groups = ([["attn_qkv.weight", "attn_gate.weight"], ["ssm_out.weight"]] if p + "ssm_a" in T else
                  [["attn_q.weight", "attn_k.weight", "attn_v.weight"], ["attn_output.weight"]])
        groups.append(["ffn_gate.weight", "ffn_up.weight"])
        for g in groups:
            ts = [T[p + nm] for nm in g]
            assert all(t.ggml_type == 12 for t in ts), g
            inner, rows = int(ts[0].ne[0]), sum(int(t.ne[1]) for t in ts)
            if g[0] == "ffn_gate.weight":
                rows //= 2            # SwiGLU writes one vector of the two products
            tot += sum(t.nbytes for t in ts) + 4 * (inner + rows)
            n += 1
    return tot, n


def graph_class_times(spec, T, prompt, tok0, device, base_ms, reps=3):
    """Per-token marginal device time (ms) of each kernel class in the graph."""
    from inferno_b200.model import Model
    out = {}
    for name, bits in GRAPH_CLASSES.items():
        os.environ["INFERNO_B200_ABLATE"] = str(bits)
        try:
            m = Model(spec, T, device=device, max_ctx=CTX)
        finally:
            del os.environ["INFERNO_B200_ABLATE"]
        m.reset()
        best = 1e30
        for _ in range(reps + 1):
            m.reset()
            m.decode_greedy(tok0, PROMPT, NDEC)
            best = min(best, m.last_decode_ms())
        m.close()
        out[name] = (base_ms - best) / NDEC
    return out


def run_ours(args):
    import torch
    ws, rank, local = dist_env()
    if ws > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    torch.cuda.set_device(local)
    from inferno_b200 import synth as S
    from inferno_b200.model import Model, algorithmic_bytes_per_token
    spec, T = build_model()
    m = Model(spec, T, device=local, max_ctx=CTX)
    prompt = S.tokens(SEED, PROMPT, spec.vocab)
    m.reset()
    tok0, _ = m.forward(prompt, 0, want_logits=False)
    m.save_device()

    def step():
        m.restore_device()
        return m.decode_greedy(tok0, PROMPT, NDEC)

    for _ in range(args.warmup):
        out = step()
    ref_tokens = out.copy()

    def barrier():
        torch.cuda.synchronize()
        if ws > 1:
            torch.distributed.barrier()
        torch.cuda.synchronize()

    clocks = ClockSampler(local)
    clocks.start()
    barrier()
    # device time: each step's graphs are bracketed by CUDA events on the
    # engine stream (inferno_last_decode_ms); the restore copy is included via
    # a torch-side event pair around the whole region as well.
    t_dev = 0.0
    wall0 = time.perf_counter()
    for _ in range(args.steps):
        out = step()
        t_dev += m.last_decode_ms()
    barrier()
    wall = time.perf_counter() - wall0
    clk = clocks.stop()
    assert np.array_equal(out, ref_tokens), "decode is not deterministic across steps"
    ms_step = max_over_ranks(t_dev / args.steps)
    value = ws * NDEC / (ms_step / 1000.0)

    # ---- e2e through the public API (host prompt in, host tokens out) ----
    e2e_steps = max(2, min(args.steps, 5))
    for _ in range(max(2, min(args.warmup, 3))):    # untimed: the prefill graphs are captured here
        m.generate(prompt, NDEC + 1)
    torch.cuda.synchronize()
    barrier()
    w0 = time.perf_counter()
    for _ in range(e2e_steps):
        toks = m.generate(prompt, NDEC + 1)      # prefill + 128 decode tokens
    torch.cuda.synchronize()
    e2e_s = max_over_ranks((time.perf_counter() - w0) / e2e_steps)
    e2e = {"value": ws * NDEC / e2e_s, "unit": UNIT, "h2d_bytes_per_step": PROMPT * 4 + 32,
           "d2h_bytes_per_step": (NDEC + 1) * 4 + 32,
           "note": "wall time of Model.generate (reset, prompt H2D, 32-token prefill, 128 greedy tokens, "
                   "token read-back) per step; tokens/s counts the 128 decode tokens"}
    assert toks[1:] == [int(t) for t in ref_tokens], "generate() disagrees with the timed decode"
    # where the e2e step goes (one extra, separately synchronised call)
    t0 = time.perf_counter()
    m.reset()
    torch.cuda.synchronize()
    t1 = time.perf_counter()
    tok_e, _ = m.forward(prompt, 0, want_logits=False)
    torch.cuda.synchronize()
    t2 = time.perf_counter()
    m.decode_greedy(tok_e, PROMPT, NDEC)
    torch.cuda.synchronize()
    t3 = time.perf_counter()
    e2e["breakdown_ms"] = {"reset": 1e3 * (t1 - t0), "prefill": 1e3 * (t2 - t1), "decode": 1e3 * (t3 - t2)}

    peaks = {}
    try:
        peaks = json.loads((ROOT / "MEASURED_PEAKS.json").read_text())
    except Exception:
        pass
    peak = float(peaks.get("hbm_gbs", 6650.0))
    peak_src = "measured" if "hbm_gbs" in peaks else "fallback"

    # ---- where the token goes inside the graph: marginal device time of each
    # kernel class (ablation, CUDA events around the same graph replays) ----
    tok_ms = ms_step / NDEC
    graph_ms = graph_class_times(spec, T, prompt, tok0, local, ms_step)
    # dominant class: the 72 Q4_K per-layer tensor-core GEMVs of a token
    q4_bytes, q4_n = q4k_launch_bytes(spec, T)
    q4_ms = graph_ms["q4k_gemv"] / q4_n
    q4_achieved = q4_bytes / q4_n / (q4_ms / 1000.0) / 1e9
    traffic = None
    try:
        for ln in (ROOT / "profiles" / "gemv_q4k_6144x1024.md").read_text().splitlines():
            if ln.startswith("dram_bytes_per_launch:"):
                traffic = int(ln.split(":")[1].strip())
    except Exception:
        pass

    # ---- lm_head (Q6_K 248320x1024 GEMV + argmax) alone, live on the engine
    # stream with CUDA events (eager pass, same inputs) ----
    m.restore_device()
    prof = m.profile(tok0, PROMPT, 16)
    lm_ms, lm_n = prof["lm_head"]
    lm_bytes = T["token_embd.weight"].nbytes + spec.hidden * 4 * 2
    achieved = lm_bytes / (lm_ms / lm_n / 1000.0) / 1e9
    pos_mid = PROMPT + NDEC // 2
    tok_bytes = algorithmic_bytes_per_token(spec, T, pos_mid)
    tok_gbs = tok_bytes / (ms_step / NDEC / 1000.0) / 1e9
    lm_traffic = None
    try:
        # DRAM bytes of one lm_head launch from the committed ncu summary
        for ln in (ROOT / "profiles" / "lm_head_q6k_248320x1024.md").read_text().splitlines():
            if ln.startswith("dram_bytes_per_launch:"):
                lm_traffic = int(ln.split(":")[1].strip())
    except Exception:
        pass
    line = {"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": ws, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32 (fp32 activations, Q4_K/Q6_K weights)",
            "data": "synthetic (seeded N(0,0.02) weights quantized to GGUF blocks; seeded token ids)",
            "config": CONFIG, "clocks": clk, "e2e": e2e,
            "gpu_launches": m.kernels_per_token() * NDEC,
            "roofline": {"bound": "hbm", "kernel": "Q4_K per-layer tensor-core GEMV (gemv_mma_kernel<12>), "
                                                  f"{q4_n} launches per token",
                         "achieved": q4_achieved, "peak": peak, "unit": "GB/s", "frac": q4_achieved / peak,
                         "peak_source": peak_src, "traffic": traffic,
                         "algorithmic_bytes_per_launch": q4_bytes / q4_n, "launch_ms": q4_ms,
                         "timing": "marginal in-graph device time per launch: token time with and without "
                                   "the class (CUDA events around the same graph replays), / launches"},
            "lm_head_roofline": {"bound": "hbm", "kernel": "lm_head Q6_K 248320x1024 GEMV + argmax",
                                 "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                                 "traffic": lm_traffic, "algorithmic_bytes_per_launch": lm_bytes,
                                 "launch_ms": lm_ms / lm_n, "timing": "CUDA events around the launch (eager)"},
            "token_roofline": {"algorithmic_bytes_per_token": tok_bytes, "achieved_gbs": tok_gbs,
                               "frac": tok_gbs / peak, "peak": peak},
            "kernel_time_share": {k: round(v / tok_ms, 4) for k, v in graph_ms.items()},
            "kernel_time_share_note": "marginal in-graph time of each class / token time (ablation); the rest "
                                      "is embedding, finalize and the dependency chain between kernels",
            "wall_s": wall}
    # the sharded configs over the same launched ranks (config 4 tensor
    # parallel, config 5 expert parallel): the 1 -> N curve north_star asks
    # for, next to the config-1 replicas headline
    if not args.no_sharded:
        m.close()
        for wl, key in (("config4", "tp_config4"), ("config5", "ep_config5")):
            try:
                sub_line = measure_big(wl, 2, 1, ws, rank, local)
                line[key] = {k: sub_line[k] for k in ("value", "unit", "ms_per_token", "prefill_s",
                                                      "prefill_tokens_per_s", "comm", "token_roofline")}
                line[key]["n_gpus"] = ws
                line[key]["parallelism"] = sub_line["config"]["parallelism"]
            except Exception as ex:          # reported, never fatal to the headline line
                line[key] = {"error": str(ex)[:200]}
    if rank == 0 and ws == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(spec, T)
        ref_k = reference_kernel_gbs(T)
        if ref_k:
            line["cpu_reference_kernel"] = ref_k
    if rank == 0:
        print(json.dumps(line), flush=True)
    if args.no_sharded:
        m.close()
    if ws > 1:
        torch.distributed.destroy_process_group()
    return 0


BIG = {
    # 9B-shaped hybrid, 2048-token prompt, 256 greedy steps,
    # tensor parallel over the launched ranks (strong scaling: one sequence)
    "config4": dict(spec="qwen35-9b", prompt=2048, ndec=256, ctx=32768 + 128, tp=True,
                    metric="decode tokens/s @batch1 (Qwen3.5-9B-shaped hybrid, Q4_K_M mix, tensor parallel)"),
    # 35B-A3B-shaped MoE hybrid at batch 1, ctx 4096;
    # expert parallel over the launched ranks (strong scaling: one sequence)
    # the config-1 model at batch 8 (eight sequences, own 32-token prompts)
    "config1-b8": dict(spec="qwen35-0.8b", prompt=32, ndec=128, ctx=512, tp=False, batch=8,
                       metric="decode tokens/s @batch8 (Qwen3.5-0.8B-shaped hybrid, 8 sequences)"),
    # BASELINE configs[3] at batch 8: eight sequences (own 2048-token prompts)
    # decoded in lockstep, one weight read per step for all eight
    "config4-b8": dict(spec="qwen35-9b", prompt=2048, ndec=256, ctx=2048 + 256 + 64, tp=False, batch=8,
                       metric="decode tokens/s @batch8 (Qwen3.5-9B-shaped hybrid, Q4_K_M mix, 8 sequences)"),
    # BASELINE configs[4] at batch 16: sixteen sequences in lockstep (attention /
    # GDN / router batched over the sequences, each token's experts its own)
    "config5-b16": dict(spec="qwen35-35b-a3b", prompt=32, ndec=128, ctx=4096 + 128, tp=False, batch=16,
                        metric="decode tokens/s @batch16 (Qwen3.5-35B-A3B-shaped MoE hybrid, 16 sequences)"),
    "config5": dict(spec="qwen35-35b-a3b", prompt=32, ndec=128, ctx=4096 + 128, tp=True,
                    metric="decode tokens/s @batch1 (Qwen3.5-35B-A3B-shaped MoE hybrid, IQ2_XXS/Q4_K experts, "
                           "expert parallel)"),
}


def run_big(args):
    """Configs 4 and 5: decode throughput on the multi-GB models (weights drawn
    from a pool of 256 quantized N(0,0.02) rows per matrix: same bytes and value
    distribution, generated in seconds)."""
    import torch
    import torch.distributed as dist
    ws, rank, local = dist_env()
    torch.cuda.set_device(local)
    if ws > 1:
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    line = measure_big(args.workload, args.steps, args.warmup, ws, rank, local)
    if rank == 0:
        print(json.dumps(line), flush=True)
    if ws > 1:
        dist.destroy_process_group()
    return 0


def measure_big(workload, steps, warmup, ws, rank, local):
    """One config-4 / config-5 measurement over the launched ranks (tensor /
    expert parallel when ws > 1); returns the JSON-line dict (rank 0's)."""
    import torch
    import torch.distributed as dist
    W = BIG[workload]
    from inferno_b200 import synth as S
    from inferno_b200.model import Model, algorithmic_bytes_per_token
    spec = S.CONFIGS[W["spec"]]
    T = S.make_model(spec, seed=SEED, pool=256)
    tp = W["tp"] and ws > 1
    kw = {}
    if tp:
        uid = [Model.tp_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(uid, src=0)
        kw = dict(tp_rank=rank, tp_size=ws, tp_uid=uid[0])
    B = W.get("batch", 1)
    m = Model(spec, T, device=local, max_ctx=W["ctx"], max_batch=B, **kw)
    P, ND = W["prompt"], W["ndec"]
    tok_bytes = algorithmic_bytes_per_token(spec, T, P + ND // 2)
    del T
    if B == 1:
        prompt = S.tokens(SEED, P, spec.vocab)
        t0 = time.perf_counter()
        tok0, _ = m.forward(prompt, 0, want_logits=False)
        prefill_s = time.perf_counter() - t0
    else:
        # each sequence its own seeded prompt, prefilled into its own slice
        toks0 = []
        t0 = time.perf_counter()
        for b in range(B):
            m.select_sequence(b)
            tb, _ = m.forward(S.tokens(SEED + b, P, spec.vocab), 0, want_logits=False)
            toks0.append(tb)
        prefill_s = (time.perf_counter() - t0) / B
        m.select_sequence(0)
    m.save_device()

    def step():
        m.restore_device()
        if B == 1:
            return m.decode_greedy(tok0, P, ND)
        return m.decode_batch(toks0, [P] * B, ND)

    for _ in range(max(1, warmup)):
        ref = step()

    def barrier():
        torch.cuda.synchronize()
        if ws > 1:
            dist.barrier()
        torch.cuda.synchronize()

    clocks = ClockSampler(local)
    clocks.start()
    barrier()
    t_dev = 0.0
    for _ in range(steps):
        out = step()
        t_dev += m.last_decode_ms()
    barrier()
    clk = clocks.stop()
    assert np.array_equal(out, ref), "decode is not deterministic across steps"
    ms_step = max_over_ranks(t_dev / steps)
    prefill_s = max_over_ranks(prefill_s)
    seqs = (1 if tp else ws) * B
    value = seqs * ND / (ms_step / 1000.0)
    peaks = {}
    try:
        peaks = json.loads((ROOT / "MEASURED_PEAKS.json").read_text())
    except Exception:
        pass
    peak = float(peaks.get("hbm_gbs", 6650.0))
    # weights are read once per batched step: bytes per step, not per token
    per_gpu_gbs = tok_bytes / (ws if tp else 1) / (ms_step / ND / 1000.0) / 1e9
    comm = m.comm_mode()
    line = {"metric": W["metric"], "value": value, "unit": UNIT, "n_gpus": ws, "steps": steps,
            "warmup": warmup, "ms_per_step": ms_step, "higher_is_better": True,
            "scaling": "strong" if tp else "weak", "vs_baseline": None,
            "dtype": "f32 (fp32 activations, GGUF block weights)",
            "data": "synthetic (seeded; rows of each matrix drawn from 256 quantized N(0,0.02) rows)",
            "config": {"workload": f"{W['spec']}: {P}-token prompt (untimed), {ND} greedy decode tokens @batch{B}",
                       "model": W["spec"], "global_batch": B, "seq_len": P + ND,
                       "parallelism": (("ep" if spec.n_experts else "tp") + str(ws)) if tp else
                                      ("replicas" if ws > 1 else "single"),
                       "l2": "weights per token >> 126 MB L2 (no flush needed)"},
            "clocks": clk, "gpu_launches": m.kernels_per_token() * ND,
            "token_roofline": {"algorithmic_bytes_per_token": tok_bytes, "achieved_gbs_per_gpu": per_gpu_gbs,
                               "frac": per_gpu_gbs / peak, "peak": peak},
            "ms_per_token": ms_step / ND, "prefill_s": prefill_s,
            "prefill_tokens_per_s": P / prefill_s,
            "comm": {"peer-exchange": "fused peer-memory residual exchange in the GEMV epilogue / prologue"
                              + (" (expert FFN partials)" if spec.n_experts else ""),
                     "nccl": "NCCL all-reduce of the residual",
                     "none": None}[comm] if tp else None}
    m.close()
    return line


def run_gdn(args):
    """the gated delta-rule recurrence in isolation (16
    heads x 128, dk = dv = 128), decode mode (1024 steps from a zero state)
    timed on the device; the oracle's sequential CPU recurrence on a bounded
    sample as the CPU baseline.  Whole job = all ranks (independent replicas)."""
    import ctypes as C
    import torch
    ws, rank, local = dist_env()
    torch.cuda.set_device(local)
    if ws > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    from inferno_b200._lib import call
    T, H, d = 1024, 16, 128
    rng = np.random.default_rng(SEED)
    q = rng.standard_normal((T, H, d)).astype(np.float32)
    k = rng.standard_normal((T, H, d)).astype(np.float32)
    q /= np.linalg.norm(q, axis=-1, keepdims=True)
    k /= np.linalg.norm(k, axis=-1, keepdims=True)
    v = rng.standard_normal((T, H, d)).astype(np.float32)
    beta = (1 / (1 + np.exp(-rng.standard_normal((T, H))))).astype(np.float32)
    g = (-np.log1p(np.exp(rng.standard_normal((T, H))))).astype(np.float32)
    dev = [torch.from_numpy(a).cuda() for a in (q, k, v, beta, g)]
    S = torch.zeros((H, d, d), device="cuda")
    y = torch.empty((T, H, d), device="cuda")
    P = lambda t: C.c_void_p(t.data_ptr())  # noqa: E731
    st = torch.cuda.current_stream()

    def step():
        S.zero_()
        call("inferno_gdn_recurrence", T, H, d, d, *[P(t) for t in dev], P(S), P(y), C.c_void_p(st.cuda_stream))

    for _ in range(args.warmup):
        step()
    clocks = ClockSampler(local)
    clocks.start()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        step()
    e1.record()
    torch.cuda.synchronize()
    clk = clocks.stop()
    ms = max_over_ranks(e0.elapsed_time(e1) / args.steps)
    line = {"metric": "GDN recurrence decode steps/s (16 heads x 128x128 fp32 state, 1024 steps)",
            "value": ws * T / (ms / 1000.0), "unit": "steps/s", "n_gpus": ws, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded, BASELINE configs[2] distributions)",
            "config": {"workload": "config3 gated delta-rule recurrence, decode mode, 1024 steps from zero state",
                       "model": "gdn-isolated H2048", "global_batch": 1, "seq_len": T, "parallelism": "replicas",
                       "l2": "state resident in registers; per-step inputs 25 KB"},
            "us_per_recurrence_step": ms * 1000.0 / T, "clocks": clk, "gpu_launches": 1}
    # prefill mode: 4096 tokens in chunks of 64, the
    # chunked (WY) form, next to the sequential kernel on the same tokens
    Tp = 4096
    rngp = np.random.default_rng(SEED + 1)
    qp = rngp.standard_normal((Tp, H, d)).astype(np.float32)
    kp = rngp.standard_normal((Tp, H, d)).astype(np.float32)
    qp /= np.linalg.norm(qp, axis=-1, keepdims=True)
    kp /= np.linalg.norm(kp, axis=-1, keepdims=True)
    vp = rngp.standard_normal((Tp, H, d)).astype(np.float32)
    bp = (1 / (1 + np.exp(-rngp.standard_normal((Tp, H))))).astype(np.float32)
    gp = (-np.log1p(np.exp(rngp.standard_normal((Tp, H))))).astype(np.float32)
    devp = [torch.from_numpy(a).cuda() for a in (qp, kp, vp, bp, gp)]
    yp = torch.empty((Tp, H, d), device="cuda")

    def timed(fn, reps):
        for _ in range(2):
            fn()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(reps):
            fn()
        b.record()
        torch.cuda.synchronize()
        return a.elapsed_time(b) / reps

    def chunked():
        S.zero_()
        call("inferno_gdn_chunked", Tp, H, d, d, *[P(t) for t in devp], P(S), P(yp), 64, C.c_void_p(st.cuda_stream))

    def sequential():
        S.zero_()
        call("inferno_gdn_recurrence", Tp, H, d, d, *[P(t) for t in devp], P(S), P(yp), C.c_void_p(st.cuda_stream))

    ms_chunk = max_over_ranks(timed(chunked, max(3, args.steps)))
    ms_seq = max_over_ranks(timed(sequential, 3))
    Cc = 64
    flops = (Tp // Cc) * H * (3 * 2 * Cc * Cc * d + 2 * Cc * Cc * d + 3 * 2 * Cc * d * d + 2 * Cc * Cc * d)
    fp32_peak = 148 * 128 * 2 * 1.965e9 / 1e12
    line["prefill_mode"] = {
        "workload": "4096 tokens, chunks of 64 (chunked WY form), 16 heads x 128x128 fp32 state from zero",
        "tokens_per_s": ws * Tp / (ms_chunk / 1000.0), "ms": ms_chunk,
        "tflops": flops / (ms_chunk / 1000.0) / 1e12,
        "tflops_peak": fp32_peak,
        "frac": flops / (ms_chunk / 1000.0) / 1e12 / fp32_peak,
        "peak_note": "fp32 CUDA-core nominal (148 SMs x 128 FMA/clk x 1.965 GHz): the chunked products run as "
                     "fp32 FMA, not on the tensor cores",
        "flops_note": "dense-equivalent FLOPs of the chunk products (K K^T, Q K^T, W, U, W S^T, Q S^T, P D, D^T K)",
        "sequential_ms": ms_seq, "speedup_vs_sequential": ms_seq / ms_chunk}
    if rank == 0 and not args.no_cpu_baseline:
        sys.path.insert(0, str(ROOT / "oracle"))
        import oracle as O
        n = 64
        S0 = np.zeros((H, d, d), np.float32)
        t0 = time.perf_counter()
        O.gdn_recurrence(q[:n], k[:n], v[:n], beta[:n], g[:n], S0)
        dt = time.perf_counter() - t0
        line["cpu_baseline"] = {"value": n / dt, "unit": "steps/s", "cores": O.cpu_count(), "kind": "port",
                                "sample": f"{n} recurrence steps of the same inputs, OpenMP over heads"}
    if rank == 0:
        print(json.dumps(line), flush=True)
    if ws > 1:
        torch.distributed.destroy_process_group()
    return 0


GEMM_TYPES = {"Q4_K": 12, "Q5_K": 13, "Q6_K": 14, "Q8_0": 8, "IQ2_XXS": 16}


def run_gemm(args):
    """the quantized GEMV / GEMM microbench.  One shape
    (--shape OUTxIN), type and batch; seeded random GGUF blocks; y = W x for
    `batch` columns through inferno_gemv (batch >= 16 of Q4_K / Q5_K / Q6_K /
    Q8_0 runs the tcgen05 GEMM).  Reports weight GB/s against the HBM peak
    and, for batch >= 16, TFLOP/s against the bf16 tensor peak."""
    import ctypes as C
    import torch
    ws, rank, local = dist_env()
    torch.cuda.set_device(local)
    sys.path.insert(0, str(ROOT / "tests"))
    from q8k_cases import random_blocks
    from inferno_b200._lib import call
    rows, inner = (int(v) for v in args.shape.split("x"))
    t = GEMM_TYPES[args.type]
    qk, bb = (32, 34) if t == 8 else (256, {12: 144, 13: 176, 14: 210, 16: 66}[t])
    rng = np.random.default_rng(SEED)
    W = random_blocks(rng, t, rows * inner // qk)
    x = rng.standard_normal((args.batch, inner)).astype(np.float32)
    dW, dx = torch.from_numpy(W).cuda(), torch.from_numpy(x).cuda()
    dy = torch.empty((args.batch, rows), dtype=torch.float32, device="cuda")
    st = torch.cuda.current_stream()
    P = lambda a: C.c_void_p(a.data_ptr())  # noqa: E731
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")     # > L2 (126 MB)

    def step():
        call("inferno_gemv", t, P(dW), P(dx), P(dy), inner, rows, args.batch, C.c_void_p(st.cuda_stream))

    for _ in range(args.warmup):
        step()
    clocks = ClockSampler(local)
    clocks.start()
    times = []
    for _ in range(args.steps):
        flush.zero_()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        step()
        b.record()
        torch.cuda.synchronize()
        times.append(a.elapsed_time(b))
    clk = clocks.stop()
    ms = max_over_ranks(float(np.median(times)))
    peaks = {}
    try:
        peaks = json.loads((ROOT / "MEASURED_PEAKS.json").read_text())
    except Exception:
        pass
    wbytes = W.nbytes + 4 * args.batch * (inner + rows)
    gbs = wbytes / (ms / 1000.0) / 1e9
    tflops = 2.0 * rows * inner * args.batch / (ms / 1000.0) / 1e12
    tc = args.batch >= 16 and t != 16
    line = {"metric": f"quantized GEMV/GEMM {args.type} {rows}x{inner} batch {args.batch}",
            "value": ws * gbs if not tc else ws * tflops, "unit": "GB/s" if not tc else "TFLOP/s",
            "n_gpus": ws, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "fp16 hi/lo split (tensor cores)" if tc else "f32",
            "data": "synthetic (seeded random GGUF blocks, N(0,1) activations)",
            "config": {"workload": f"config2 {args.type} {rows}x{inner} @batch{args.batch}", "model": "gemm",
                       "global_batch": args.batch, "seq_len": 1, "parallelism": "replicas",
                       "l2": "256 MB written between timed launches (L2 flush)"},
            "clocks": clk, "weight_gbs": gbs, "tflops": tflops,
            "hbm_frac": gbs / float(peaks.get("hbm_gbs", 6650.0)),
            "tensor_frac": (tflops / float(peaks.get("bf16_tflops", 1590.0)) / 3.0) if tc else None,
            "tensor_note": "three fp16 MMAs per product (hi*hi + hi*lo + lo*hi): tensor_frac counts the "
                           "issued MMA work against the bf16 peak" if tc else None}
    if rank == 0:
        print(json.dumps(line), flush=True)
    return 0


def run_prefill(args):
    """Prompt processing of the config-1 model: Model.forward over the 32-token
    seeded prompt (chunked prefill, 8 tokens per chunk).  The first call runs
    eagerly, the second captures the prefill graph; `warmup` >= 2 keeps both
    out of the timed region.  Each step is reset + forward (host prompt in,
    first generated token out), timed by wall clock around a synchronize."""
    import torch
    ws, rank, local = dist_env()
    torch.cuda.set_device(local)
    from inferno_b200 import synth as S
    from inferno_b200.model import Model
    spec, T = build_model()
    m = Model(spec, T, device=local, max_ctx=CTX)
    prompt = S.tokens(SEED, PROMPT, spec.vocab)
    for _ in range(max(2, args.warmup)):
        m.reset()
        m.forward(prompt, 0, want_logits=False)
    clocks = ClockSampler(local)
    clocks.start()
    times = []
    for _ in range(args.steps):
        m.reset()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        m.forward(prompt, 0, want_logits=False)
        torch.cuda.synchronize()
        times.append(time.perf_counter() - t0)
    clk = clocks.stop()
    s_step = max_over_ranks(float(np.median(times)))
    line = {"metric": "prefill prompt tokens/s @batch1 (Qwen3.5-0.8B-shaped hybrid, Q4_K/Q6_K)",
            "value": ws * PROMPT / s_step, "unit": "tokens/s", "n_gpus": ws, "steps": args.steps,
            "warmup": max(2, args.warmup), "ms_per_step": 1e3 * s_step, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32 (fp32 activations, Q4_K/Q6_K weights)",
            "data": "synthetic (seeded N(0,0.02) weights quantized to GGUF blocks; seeded token ids)",
            "config": {"workload": f"config1 qwen35-0.8b-shaped hybrid, {PROMPT}-token prompt, chunked prefill",
                       "model": "qwen35-0.8b-shaped (random-init, seeded)", "global_batch": 1,
                       "seq_len": PROMPT, "parallelism": "replicas",
                       "l2": "weights 515 MB per chunk > 126 MB L2 (no flush needed)"},
            "clocks": clk, "timing": "median wall time of reset + Model.forward (synchronised)"}
    if rank == 0:
        print(json.dumps(line), flush=True)
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--workload", default="config1", choices=["config1", "config3", "prefill1", "gemm"] + sorted(BIG),
                    help="config1 (the headline metric, default), config3 / config4 / config5, or prefill1 "
                         "(config-1 prompt processing)")
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--shape", default="12288x4096", help="gemm workload: OUTxIN")
    ap.add_argument("--type", default="Q4_K", choices=sorted(GEMM_TYPES), help="gemm workload: weight type")
    ap.add_argument("--batch", type=int, default=128, help="gemm workload: columns")
    ap.add_argument("--no-sharded", action="store_true",
                    help="skip the config-4 (tensor parallel) / config-5 (expert parallel) keys of the config-1 line")
    args = ap.parse_args()
    if args.impl == "reference":
        return run_reference(args)
    if args.workload == "config3":
        return run_gdn(args)
    if args.workload == "prefill1":
        return run_prefill(args)
    if args.workload == "gemm":
        return run_gemm(args)
    if args.workload != "config1":
        return run_big(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
