"""Host-side mirror of the reference's model API over the B200 engine.

The reference host (Inferno.jl) loads a GGUF file, builds a model and drives
it per token: ``layer(x, pos, rope, cache)`` per decoder layer
(src/ModelCPU.jl:870-891), ``forward_cpu!(model, tokens, pos, caches)``
(:945-989), greedy ``argmax`` (:1123-1127) and the decode loop of
test/benchmark_e2e.jl:43-59.  ``Model`` offers the same calls on top of
libinferno_b200.so; all compute runs on the GPU.
"""
from __future__ import annotations

import ctypes as C
import math
from pathlib import Path

import numpy as np

from . import synth as S
from ._lib import InfernoConfig, InfernoSampling, call, check, lib


def _p(a: np.ndarray):
    return a.ctypes.data_as(C.c_void_p)


def config_from_metadata(md: dict, tensors: dict) -> dict:
    """LoaderCPU.get_config (src/LoaderCPU.jl:393-418): each key is looked up
    under the architecture prefix (``qwen35.``), then ``qwen3.``, then bare.
    GDN dims follow src/LoaderCPU.jl:498-516 but take the q/k head count from
    ``ssm.group_count`` (the reference assumes nk == nv, which is wrong for the
    9B shape)."""
    arch = md.get("general.architecture", "qwen35")

    def g(key, default):
        for k in (f"{arch}.{key}", f"qwen3.{key}", key):
            if k in md:
                return md[k]
        return default

    emb = tensors["token_embd.weight"]
    cfg = dict(
        hidden=int(g("embedding_length", 1024)),
        ffn=int(g("feed_forward_length", 3584)),
        layers=int(g("block_count", 24)),
        n_heads=int(g("attention.head_count", 8)),
        n_kv=int(g("attention.head_count_kv", 2)),
        head_dim=int(g("attention.key_length", 256)),
        eps=float(g("attention.layer_norm_rms_epsilon", 1e-6)),
        rope_theta=float(g("rope.freq_base", 1e7)),
        ctx=int(g("context_length", 4096)),
        partial_rotary=float(g("rope.partial_rotary_factor", 0.25)),
        interval=int(g("full_attention_interval", 4)),
        ssm_dk=int(g("ssm.state_size", 128)),
        ssm_nk=int(g("ssm.group_count", 16)),
        conv_k=int(g("ssm.conv_kernel", 4)),
        n_experts=int(g("expert_count", 0)),
        n_experts_used=int(g("expert_used_count", 0)),
        expert_ffn=int(g("expert_feed_forward_length", 0)),
        shexp_ffn=int(g("expert_shared_feed_forward_length", 0)),
        vocab=int(emb.ne[1]),          # actual vocab from the embedding (src/LoaderCPU.jl:301-306)
    )
    # nv from ssm_a, dv from the gate projection (src/LoaderCPU.jl:498-507)
    for i in range(cfg["layers"]):
        a = tensors.get(f"blk.{i}.ssm_a")
        if a is not None:
            cfg["ssm_nv"] = int(a.ne[0])
            cfg["ssm_dv"] = int(tensors[f"blk.{i}.attn_gate.weight"].ne[1]) // cfg["ssm_nv"]
            break
    else:
        cfg["ssm_nv"], cfg["ssm_dv"] = cfg["ssm_nk"], cfg["ssm_dk"]
    return cfg


def spec_from_config(cfg: dict, name: str = "gguf") -> S.ModelSpec:
    return S.ModelSpec(name, hidden=cfg["hidden"], layers=cfg["layers"], n_heads=cfg["n_heads"],
                       n_kv=cfg["n_kv"], head_dim=cfg["head_dim"], ffn=cfg["ffn"], vocab=cfg["vocab"],
                       ssm_nv=cfg["ssm_nv"], ssm_nk=cfg["ssm_nk"], ssm_dk=cfg["ssm_dk"],
                       ssm_dv=cfg["ssm_dv"], conv_k=cfg["conv_k"], interval=cfg["interval"],
                       ctx=cfg["ctx"], eps=cfg["eps"], rope_theta=cfg["rope_theta"],
                       partial_rotary=cfg["partial_rotary"], n_experts=cfg["n_experts"],
                       n_experts_used=cfg["n_experts_used"], expert_ffn=cfg["expert_ffn"],
                       shexp_ffn=cfg["shexp_ffn"])


def read_gguf(path) -> tuple:
    """GGUF file -> (metadata dict, {name: Tensor}) with raw block bytes
    (memory-mapped; the keep_quantized view of src/LoaderCPU.jl:131-155)."""
    import gguf
    r = gguf.GGUFReader(str(path))
    md = {}
    for f in r.fields.values():
        if not f.types:
            continue
        try:
            v = f.contents()
        except Exception:
            continue
        md[f.name] = v
    tensors = {}
    for t in r.tensors:
        ne = tuple(int(x) for x in t.shape)
        tensors[t.name] = S.Tensor(int(t.tensor_type), ne, np.asarray(t.data).view(np.uint8).reshape(-1))
    return md, tensors


class Model:
    """A Qwen3.5-hybrid model resident on one B200."""

    def __init__(self, spec: S.ModelSpec, tensors: dict, device: int = 0, max_ctx: int | None = None,
                 use_graphs: bool = True, use_pdl: bool = True, tp_rank: int = 0, tp_size: int = 1,
                 tp_uid: bytes | None = None, gguf=None, max_batch: int = 1):
        """tp_size > 1: this process is rank `tp_rank` of a tensor-parallel group;
        `tensors` is the full model (sharded here, inferno_b200.tp) and
        `tp_uid` the group's NCCL unique id (Model.tp_unique_id() on rank 0,
        shared by the caller).  All ranks must construct concurrently.
        `gguf` (a gguf_file.GgufFile, one GPU): the weights are uploaded from
        the file mapping by the library itself and `tensors` is not used.
        `max_batch` > 1 keeps that many sequences' states for decode_batch."""
        self.spec = spec
        lspec = spec
        if gguf is not None and tp_size > 1:
            raise ValueError("the native GGUF upload loads whole tensors; shard through `tensors` for tp_size > 1")
        if tp_size > 1:
            from . import tp as _tp
            if tp_uid is None or len(tp_uid) != 128:
                raise ValueError("tensor parallel needs the group's 128-byte NCCL unique id")
            lspec, tensors = _tp.shard(spec, tensors, tp_rank, tp_size)
        c = InfernoConfig()
        c.struct_size = C.sizeof(InfernoConfig)
        c.device = device
        c.hidden_size = spec.hidden
        c.intermediate_size = lspec.ffn
        c.num_layers = spec.layers
        c.vocab_size = spec.vocab
        c.n_heads, c.n_kv_heads, c.head_dim = lspec.n_heads, lspec.n_kv, spec.head_dim
        c.ssm_nv, c.ssm_nk, c.ssm_dk, c.ssm_dv = lspec.ssm_nv, lspec.ssm_nk, spec.ssm_dk, spec.ssm_dv
        c.ssm_conv_kernel = spec.conv_k
        c.max_ctx = max_ctx or spec.ctx
        c.n_experts, c.n_experts_used = spec.n_experts, spec.n_experts_used
        c.expert_ffn, c.shared_expert_ffn = spec.expert_ffn, spec.shexp_ffn
        c.max_batch = int(max_batch)
        c.rms_eps, c.rope_theta, c.partial_rotary_factor = spec.eps, spec.rope_theta, spec.partial_rotary
        c.use_graphs, c.use_pdl = int(use_graphs), int(use_pdl)
        c.tp_rank, c.tp_size = tp_rank, tp_size
        if tp_size > 1:
            self._uid = C.create_string_buffer(bytes(tp_uid), 128)
            c.nccl_unique_id = C.cast(self._uid, C.c_void_p)
        self.cfg = c
        h = C.c_void_p()
        call("inferno_engine_create", C.byref(c), C.byref(h))
        self.h = h
        try:
            if gguf is not None:
                call("inferno_engine_load_gguf", self.h, gguf.h)
                tensors = {}
            for name, t in tensors.items():
                ne = np.ones(4, np.int64)
                ne[:len(t.ne)] = t.ne
                data = np.ascontiguousarray(t.data)
                call("inferno_engine_upload_tensor", self.h, name.encode(), t.ggml_type, _p(ne), _p(data),
                     data.nbytes)
            call("inferno_engine_finalize", self.h)
        except Exception:
            self.close()
            raise

    @staticmethod
    def tp_unique_id() -> bytes:
        """A fresh NCCL unique id for a tensor-parallel group (call on rank 0)."""
        buf = C.create_string_buffer(128)
        call("inferno_tp_unique_id", buf, 128)
        return buf.raw

    @classmethod
    def from_gguf(cls, path, native: bool = True, **kw) -> "Model":
        """load_model_cpu (src/LoaderCPU.jl:450-643) from a GGUF file.  native:
        the library parses the file and uploads the tensors from its mapping
        (inferno_gguf_open + inferno_engine_load_gguf); otherwise gguf-py reads
        it and each tensor goes through inferno_engine_upload_tensor (needed
        for tp_size > 1, where the host shards the tensors)."""
        if native and kw.get("tp_size", 1) == 1:
            from .gguf_file import GgufFile
            g = GgufFile(path)
            try:
                infos = {t.name: t for t in g.tensors()}
                spec = spec_from_config(config_from_metadata(g.metadata(), infos), Path(path).stem)
                return cls(spec, None, gguf=g, **kw)
            finally:
                g.close()
        md, tensors = read_gguf(path)
        return cls(spec_from_config(config_from_metadata(md, tensors), Path(path).stem), tensors, **kw)

    def close(self):
        if getattr(self, "h", None):
            lib().inferno_engine_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # ---- the reference's per-call API -------------------------------------
    def layer(self, i: int, x: np.ndarray, pos: int) -> np.ndarray:
        """DecoderLayerCPU(x, pos, rope, cache): returns the updated x."""
        x = np.ascontiguousarray(x, dtype=np.float32).copy()
        call("inferno_layer_forward", self.h, i, _p(x), pos)
        return x

    def forward(self, tokens, pos: int, want_logits: bool = True):
        """forward_cpu! on 0-based token ids -> (argmax, logits or None)."""
        toks = np.ascontiguousarray(tokens, dtype=np.int32)
        logits = np.empty(self.spec.vocab, np.float32) if want_logits else None
        am = np.zeros(1, np.int32)
        call("inferno_forward_tokens", self.h, _p(toks), len(toks), pos,
             _p(logits) if want_logits else None, _p(am))
        return int(am[0]), logits

    def forward_all(self, tokens, pos: int, want_logits: bool = True):
        """forward_cpu! with full_logits: (argmax of every position, logits
        [n][vocab] or None); the state advances over all tokens."""
        toks = np.ascontiguousarray(tokens, dtype=np.int32).reshape(-1)
        am = np.zeros(toks.size, np.int32)
        logits = np.empty((toks.size, self.spec.vocab), np.float32) if want_logits else None
        call("inferno_forward_tokens_all", self.h, _p(toks), int(toks.size), int(pos),
             _p(logits) if want_logits else None, _p(am))
        return am, logits

    def mtp_verify_step(self, draft_tokens, pos: int):
        """mtp_verify_step! (src/ModelCPU.jl:1914-1930): run the draft tokens
        at pos.. with every position's logits and count the leading drafts
        that equal the argmax of the previous position.  Returns (accepted,
        logits [n][vocab])."""
        draft = np.asarray(draft_tokens, dtype=np.int32).reshape(-1)
        am, logits = self.forward_all(draft, pos, want_logits=True)
        accepted = 0
        for i in range(draft.size - 1):
            if int(am[i]) == int(draft[i + 1]):
                accepted += 1
            else:
                break
        return accepted, logits

    def select_sequence(self, seq: int):
        """Point the single-sequence calls (forward, decode_greedy, layer,
        reset excepted -- it clears every sequence) at state slice `seq`."""
        call("inferno_select_sequence", self.h, int(seq))

    def decode_batch(self, toks, positions, n: int) -> np.ndarray:
        """Greedy decode of sequences 0..B-1 in lockstep: sequence b feeds
        toks[b] at positions[b]; returns [n][B] tokens."""
        t = np.ascontiguousarray(toks, dtype=np.int32).reshape(-1)
        p = np.ascontiguousarray(positions, dtype=np.int32).reshape(-1)
        if t.size != p.size:
            raise ValueError("one token and one position per sequence")
        out = np.zeros((n, t.size), np.int32)
        call("inferno_decode_batch", self.h, _p(t), _p(p), int(t.size), int(n), _p(out))
        return out

    def decode_greedy(self, tok: int, pos: int, n: int) -> np.ndarray:
        out = np.zeros(n, np.int32)
        call("inferno_decode_greedy", self.h, int(tok), int(pos), int(n), _p(out))
        return out

    def generate(self, prompt, n_steps: int) -> list:
        """Greedy generation with the corrected position schedule
        (test/benchmark_e2e.jl:43-59): prompt at 0..P-1, output i at P+i."""
        self.reset()
        tok, _ = self.forward(prompt, 0, want_logits=False)
        if n_steps == 1:
            return [tok]
        rest = self.decode_greedy(tok, len(prompt), n_steps - 1)
        return [tok] + [int(t) for t in rest]

    def decode_sample(self, tok: int, pos: int, n: int, *, temperature: float = 1.0, top_p: float = 1.0,
                      top_k: int = 0, min_p: float = 0.0, repetition_penalty: float = 1.0,
                      presence_penalty: float = 0.0, seed: int = 0, seen=()) -> np.ndarray:
        """n sampled tokens on the device: tok is fed at pos, every later token
        is drawn by softmax_sample (src/ModelCPU.jl:1123-1225) from the
        previous token's logits after the presence / repetition penalties on
        `seen` (0-based ids) and on the tokens drawn so far; draws come from
        Philox(seed, step), so a seed reproduces a sequence."""
        s = InfernoSampling(temperature, top_p, top_k, min_p, repetition_penalty, presence_penalty, seed)
        ids = np.ascontiguousarray(np.asarray(seen, dtype=np.int32).reshape(-1))
        out = np.zeros(n, np.int32)
        call("inferno_decode_sample", self.h, int(tok), int(pos), int(n), C.byref(s),
             _p(ids) if ids.size else None, int(ids.size), _p(out))
        return out

    def generate_sampled(self, prompt, n_steps: int, **sampling) -> list:
        """generate_stream_cpu's sampled loop (src/ModelCPU.jl:1277-1370) with
        the corrected positions: the prompt but its last token is prefilled,
        the last prompt token is fed at position P-1 and its logits give the
        first sampled token; the penalties count the prompt tokens and every
        sampled token.  Keyword arguments as decode_sample."""
        prompt = np.asarray(prompt, dtype=np.int32).reshape(-1)
        if prompt.size == 0 or n_steps <= 0:
            raise ValueError("generate_sampled needs a prompt and n_steps > 0")
        self.reset()
        if prompt.size > 1:
            self.forward(prompt[:-1], 0, want_logits=False)
        out = self.decode_sample(int(prompt[-1]), int(prompt.size) - 1, n_steps, seen=prompt, **sampling)
        return [int(t) for t in out]

    def reset(self):
        call("inferno_reset_states", self.h)

    def hidden(self, i: int) -> np.ndarray:
        out = np.empty(self.spec.hidden, np.float32)
        call("inferno_dump_hidden", self.h, i, _p(out))
        return out

    def last_decode_ms(self) -> float:
        return float(lib().inferno_last_decode_ms(self.h))

    def save_device(self):
        call("inferno_state_save_device", self.h)

    def restore_device(self):
        call("inferno_state_restore_device", self.h)

    def comm_mode(self) -> str:
        """How the ranks of a sharded engine sum residuals."""
        m = check(lib().inferno_comm_mode(self.h), "inferno_comm_mode")
        return {0: "none", 1: "peer-exchange", 2: "nccl"}[m]

    def kernels_per_token(self) -> int:
        return check(lib().inferno_kernels_per_token(self.h), "inferno_kernels_per_token")

    KERNEL_CLASSES = ("embed", "gemv", "gdn", "attention", "lm_head", "finalize")

    def profile(self, tok: int, pos: int, n: int) -> dict:
        """Per-kernel-class device time (eager pass with CUDA events)."""
        ms = np.zeros(6, np.float32)
        cnt = np.zeros(6, np.int32)
        call("inferno_profile_tokens", self.h, int(tok), int(pos), int(n), _p(ms), _p(cnt))
        return {k: (float(ms[i]), int(cnt[i])) for i, k in enumerate(self.KERNEL_CLASSES)}

    def state_export(self) -> np.ndarray:
        n = check(lib().inferno_state_size(self.h), "inferno_state_size")
        buf = np.empty(n, np.uint8)
        call("inferno_state_export", self.h, _p(buf), n)
        return buf

    def state_import(self, buf: np.ndarray):
        buf = np.ascontiguousarray(buf, dtype=np.uint8)
        call("inferno_state_import", self.h, _p(buf), buf.nbytes)


def algorithmic_bytes_per_token(spec: S.ModelSpec, tensors: dict, pos: int) -> int:
    """Bytes a decode token must move (the roofline accounting): every weight
    read once, KV read of pos+1 rows + write of 1 row per attention layer, GDN
    recurrent state and conv state read + write."""
    skip = {"token_embd.weight"} if "output.weight" in tensors else set()
    w = sum(t.nbytes for n, t in tensors.items() if n not in skip and not n.endswith("_exps.weight"))
    if spec.n_experts:   # routed experts: the top-k of E are read per token
        w += sum(t.nbytes for n, t in tensors.items() if n.endswith("_exps.weight")) * spec.n_experts_used // spec.n_experts
    if "output.weight" in tensors:
        w += spec.hidden * S.BLOCK[tensors["token_embd.weight"].ggml_type][1] // S.BLOCK[tensors["token_embd.weight"].ggml_type][0]
    n_attn = sum(1 for i in range(spec.layers) if f"blk.{i}.ssm_a" not in tensors)
    n_gdn = spec.layers - n_attn
    kv = n_attn * (2 * spec.n_kv * spec.head_dim * 4 * (pos + 1) + 2 * spec.n_kv * spec.head_dim * 4)
    state = n_gdn * 2 * (spec.ssm_nv * spec.ssm_dv * spec.ssm_dk * 4 + spec.conv_k * spec.conv_channels * 4)
    return int(w + kv + state)
