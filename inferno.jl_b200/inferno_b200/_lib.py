"""ctypes binding of libinferno_b200.so (the C ABI in include/inferno_b200.h).

The library is built in-tree (``make -C inferno.jl_b200``); loading fails
loudly if it is missing -- there is no CPU fallback.
"""
from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

PKG_ROOT = Path(__file__).resolve().parent.parent
LIB_PATH = PKG_ROOT / "lib" / "libinferno_b200.so"

OK, EINVAL, ECUDA, ENOMEM, ESTATE, EDEVICE, ENCCL = 0, -1, -2, -3, -4, -5, -6


class InfernoError(RuntimeError):
    def __init__(self, fn: str, rc: int, msg: str):
        super().__init__(f"{fn} failed (status {rc}): {msg}")
        self.rc = rc


class InfernoConfig(C.Structure):
    _fields_ = [(n, C.c_int32) for n in (
        "struct_size", "device", "hidden_size", "intermediate_size", "num_layers", "vocab_size",
        "n_heads", "n_kv_heads", "head_dim", "ssm_nv", "ssm_nk", "ssm_dk", "ssm_dv",
        "ssm_conv_kernel", "max_ctx", "n_experts", "n_experts_used", "expert_ffn",
        "shared_expert_ffn", "max_batch")] + [
        ("rms_eps", C.c_float), ("rope_theta", C.c_float), ("partial_rotary_factor", C.c_float),
        ("use_graphs", C.c_int32), ("use_pdl", C.c_int32), ("tp_rank", C.c_int32),
        ("tp_size", C.c_int32), ("nccl_unique_id", C.c_void_p)]


class InfernoSampling(C.Structure):
    """include/inferno_b200.h InfernoSampling (softmax_sample's parameters)."""
    _fields_ = [("temperature", C.c_float), ("top_p", C.c_float), ("top_k", C.c_int32), ("min_p", C.c_float),
                ("repetition_penalty", C.c_float), ("presence_penalty", C.c_float), ("seed", C.c_uint64)]


# every symbol the header declares (checked by the CPU tests)
EXPORTS = [
    "inferno_last_error", "inferno_version", "inferno_device_error",
    "q4_k_gemv", "q5_k_gemv", "q6_k_gemv", "q8_0_gemv", "inferno_compat_release",
    "quantize_row_q8_K", "vec_dot_q4_K_q8_K", "vec_dot_q5_K_q8_K", "vec_dot_q6_K_q8_K", "vec_dot_q8_0_q8_0",
    "inferno_dequantize", "inferno_gemv", "inferno_gemv_ex", "inferno_gemv_swiglu",
    "inferno_engine_create", "inferno_engine_upload_tensor", "inferno_engine_finalize",
    "inferno_layer_forward", "inferno_forward_tokens", "inferno_decode_greedy",
    "inferno_reset_states", "inferno_dump_hidden", "inferno_state_size", "inferno_state_export",
    "inferno_state_import", "inferno_last_decode_ms", "inferno_engine_destroy",
    "inferno_state_save_device", "inferno_state_restore_device", "inferno_kernels_per_token", "inferno_comm_mode",
    "inferno_profile_tokens", "inferno_gemv_host_noalloc", "inferno_debug_trace", "inferno_tp_unique_id",
    "inferno_gdn_recurrence", "inferno_gdn_chunked", "inferno_attention_step", "inferno_select_sequence", "inferno_decode_batch", "inferno_forward_tokens_all", "inferno_debug_xch_timeout", "inferno_sample_logits", "inferno_decode_sample",
    "inferno_gguf_open", "inferno_gguf_close", "inferno_gguf_version", "inferno_gguf_n_tensors", "inferno_gguf_n_kv",
    "inferno_gguf_data_offset", "inferno_gguf_key", "inferno_gguf_tensor_info", "inferno_gguf_get_int",
    "inferno_gguf_get_float", "inferno_gguf_get_string", "inferno_gguf_get_array", "inferno_engine_load_gguf",
]

_lib = None


class _Opt:
    """Attribute sink for symbols a partial build does not export."""

    def __setattr__(self, k, v):
        pass


def _sig(L0):
    class _L:
        def __getattr__(self, nm):
            return getattr(L0, nm) if hasattr(L0, nm) else _Opt()
    L = _L()
    p, i, i64, f = C.c_void_p, C.c_int, C.c_int64, C.c_float
    L.inferno_last_error.restype = C.c_char_p
    L.inferno_device_error.argtypes = [i, i]
    for nm in ("q4_k_gemv", "q5_k_gemv", "q6_k_gemv"):
        getattr(L, nm).argtypes = [p, p, p, p, i, i]
        getattr(L, nm).restype = None
    L.q8_0_gemv.argtypes = [p, p, p, i, i]
    L.q8_0_gemv.restype = None
    L.quantize_row_q8_K.argtypes = [p, p, i64]
    L.quantize_row_q8_K.restype = None
    for nm in ("vec_dot_q4_K_q8_K", "vec_dot_q5_K_q8_K", "vec_dot_q6_K_q8_K", "vec_dot_q8_0_q8_0"):
        getattr(L, nm).argtypes = [p, p, i]
        getattr(L, nm).restype = f
    L.inferno_dequantize.argtypes = [i, p, i64, p, p]
    L.inferno_gemv.argtypes = [i, p, p, p, i, i, i, p]
    L.inferno_gemv_ex.argtypes = [i, p, p, p, i, i, i, i, p, f, i, p, i, p]
    L.inferno_gemv_swiglu.argtypes = [i, p, p, p, p, i, i, i, p, f, p]
    L.inferno_engine_create.argtypes = [p, p]
    L.inferno_engine_upload_tensor.argtypes = [p, C.c_char_p, i, p, p, C.c_size_t]
    L.inferno_engine_finalize.argtypes = [p]
    L.inferno_layer_forward.argtypes = [p, i, p, i]
    L.inferno_forward_tokens.argtypes = [p, p, i, i, p, p]
    L.inferno_forward_tokens_all.argtypes = [p, p, i, i, p, p]
    L.inferno_select_sequence.argtypes = [p, i]
    L.inferno_decode_batch.argtypes = [p, p, p, i, i, p]
    L.inferno_decode_greedy.argtypes = [p, C.c_int32, i, i, p]
    L.inferno_reset_states.argtypes = [p]
    L.inferno_dump_hidden.argtypes = [p, i, p]
    L.inferno_state_size.argtypes = [p]
    L.inferno_state_size.restype = i64
    L.inferno_state_export.argtypes = [p, p, i64]
    L.inferno_state_import.argtypes = [p, p, i64]
    L.inferno_last_decode_ms.argtypes = [p]
    L.inferno_last_decode_ms.restype = f
    L.inferno_engine_destroy.argtypes = [p]
    L.inferno_gemv_host_noalloc.argtypes = [i, p, p, p, i, i]
    L.inferno_debug_trace.argtypes = [p, p, i]
    L.inferno_state_save_device.argtypes = [p]
    L.inferno_state_restore_device.argtypes = [p]
    L.inferno_kernels_per_token.argtypes = [p]
    L.inferno_comm_mode.argtypes = [p]
    L.inferno_profile_tokens.argtypes = [p, C.c_int32, i, i, p, p]
    L.inferno_decode_sample.argtypes = [p, C.c_int32, i, i, p, p, i, p]
    L.inferno_gguf_open.argtypes = [C.c_char_p, p]
    L.inferno_gguf_close.argtypes = [p]
    L.inferno_gguf_version.argtypes = [p]
    for nm in ("inferno_gguf_n_tensors", "inferno_gguf_n_kv", "inferno_gguf_data_offset"):
        getattr(L, nm).argtypes = [p]
        getattr(L, nm).restype = i64
    L.inferno_gguf_key.argtypes = [p, i64]
    L.inferno_gguf_key.restype = C.c_char_p
    L.inferno_gguf_tensor_info.argtypes = [p, i64, p, p, p, p, p]
    L.inferno_gguf_get_int.argtypes = [p, C.c_char_p, p]
    L.inferno_gguf_get_float.argtypes = [p, C.c_char_p, p]
    L.inferno_gguf_get_string.argtypes = [p, C.c_char_p, p]
    L.inferno_gguf_get_array.argtypes = [p, C.c_char_p, p, p, p]
    L.inferno_engine_load_gguf.argtypes = [p, p]
    L.inferno_debug_xch_timeout.argtypes = [i, p]
    L.inferno_attention_step.argtypes = [p, p, p, p, p, f, i, i, i, i, f, p, p, i, i, i, p, p]


def lib():
    """Load the in-tree library (raises if it has not been built)."""
    global _lib
    if _lib is None:
        path = Path(os.environ.get("INFERNO_B200_LIB", LIB_PATH))
        if not path.exists():
            raise RuntimeError(f"libinferno_b200.so not built at {path}: run `make -C {PKG_ROOT}`")
        L = C.CDLL(str(path))
        _sig(L)
        _lib = L
    return _lib


def check(rc: int, fn: str) -> int:
    if rc < 0:
        raise InfernoError(fn, rc, lib().inferno_last_error().decode(errors="replace"))
    return rc


def call(fn: str, *args) -> int:
    return check(getattr(lib(), fn)(*args), fn)
