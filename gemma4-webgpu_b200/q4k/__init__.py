"""q4k -- host side of the B200 Q4_K matmul path (libq4k.so).

Operators mirror the reference's matmul-path pipelines (src/engine.ts,
shaders/matmul_quant*.wgsl, logit_softcap, argmax, topk256, gelu_mul); the
compute runs in libq4k.so's sm_100a kernels, loaded through ctypes.
"""
from ._lib import Q4KError, lib  # noqa: F401
from .ops import Context, Plan, Selection, context  # noqa: F401
from . import gguf, synth  # noqa: F401

__all__ = ["Context", "Plan", "Selection", "context", "synth", "gguf", "Q4KError", "lib"]
