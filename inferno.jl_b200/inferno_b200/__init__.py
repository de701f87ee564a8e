"""inferno_b200: host side of the B200 decode engine for Inferno.jl models.

The compute path is libinferno_b200.so (hand-written sm_100a CUDA behind a C
ABI, include/inferno_b200.h).  This package binds it with ctypes and mirrors
the reference's host API (load a GGUF model, call layers / forward / greedy
generate).
"""
from . import synth  # noqa: F401
from ._lib import lib, InfernoError  # noqa: F401
