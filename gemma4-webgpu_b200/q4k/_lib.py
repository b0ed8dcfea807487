"""Loader of libq4k.so (the C ABI of include/q4k.h) via ctypes.

The library is the product path: there is no CPU or PyTorch fallback.  If the
shared object is missing or a GPU call fails, the caller gets an exception.
"""
from __future__ import annotations

import ctypes
import os
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parents[1]
LIB_PATH = PKG_DIR / "lib" / "libq4k.so"

Q4K_OK = 0
Q4K_ERR_INVALID_ARG = -1
Q4K_ERR_CUDA = -2
Q4K_ERR_UNSUPPORTED = -3
Q4K_ERR_TIMEOUT = -4
Q4K_ERR_SCRATCH_LIMIT = -5

# Every function include/q4k.h declares, with its ctypes signature.
_P, _U32, _U64, _F, _I = ctypes.c_void_p, ctypes.c_uint32, ctypes.c_uint64, ctypes.c_float, ctypes.c_int
SIGNATURES: dict[str, tuple[list, object]] = {
    "q4k_version": ([], _I),
    "q4k_create": ([_I, ctypes.POINTER(_P)], _I),
    "q4k_destroy": ([_P], None),
    "q4k_last_error": ([_P], ctypes.c_char_p),
    "q4k_check": ([_P], _I),
    "q4k_set_wait_limit": ([_P, _U32], _I),
    "q4k_matmul_quant": ([_P, _P, _P, _P, _U32, _U32, _P], _I),
    "q4k_gemv": ([_P, _P, _P, _P, _U32, _U32, _U32, _P], _I),
    "q4k_gemm": ([_P, _P, _P, _P, _U32, _U32, _U32, _P], _I),
    "q4k_gemm_f16x": ([_P, _P, _P, _P, _U32, _U32, _U32, _P], _I),
    "q4k_dequant_f16": ([_P, _P, _P, _U64, _P], _I),
    "q4k_logit_softcap": ([_P, _P, _U32, _F, _P], _I),
    "q4k_argmax": ([_P, _P, _U32, _P, _P], _I),
    "q4k_topk256": ([_P, _P, _U32, _P, _P], _I),
    "q4k_select_rows": ([_P, _P, _U32, _U32, _F, _P, _P, _P, _P], _I),
    "q4k_gelu_mul": ([_P, _P, _P, _P, _U32, _P], _I),
    "q4k_lmhead_select": ([_P, _P, _P, _U32, _U32, _F, _U32, _P, _P, _P, _P, _P], _I),
    "q4k_merge_candidates": ([_P, _P, _P, _U32, _P, _P, _P, _P], _I),
    "q4k_lmhead_select_static": ([_P, _P, _U32, _U32, _F, _U32, _P, _P, _P, _P, _P], _I),
    "q4k_check_static": ([], _I),
    "q4k_exchange_create": ([_P, _U32, _U32, ctypes.POINTER(_P), _P], _I),
    "q4k_exchange_open": ([_P, _U32, _P], _I),
    "q4k_exchange_open_local": ([_P, _U32, _P], _I),
    "q4k_exchange_destroy": ([_P], None),
    "q4k_lmhead_select_sharded": ([_P, _P, _P, _P, _U32, _U32, _F, _U32, _P, _P, _P, _P], _I),
    "q4k_q6k_device_bytes": ([_U32, _U32], _U64),
    "q4k_q6k_repack": ([_P, _P, _P, _U32, _U32, _P], _I),
    "q4k_q6k_dequant_f16": ([_P, _P, _U32, _U32, _P, _P], _I),
    "q4k_q6k_gemv": ([_P, _P, _P, _P, _U32, _U32, _U32, _P], _I),
    "q4k_q6k_lmhead_select": ([_P, _P, _P, _U32, _U32, _F, _U32, _P, _P, _P, _P, _P], _I),
    "q4k_q5k_dequant_f16": ([_P, _P, _P, _U64, _P], _I),
    "q4k_ple_stage1": ([_P, _P, _P, _U32, _U32, _U32, _P, _P, _F, _P, _P], _I),
    "q4k_chain_create": ([_P, _U32, _U32, _U32, _U32, _U32, _F, _P, _P, _P, ctypes.POINTER(_P)], _I),
    "q4k_chain_lmhead": ([_P, _P, _U32, _F, _P, _P, _P], _I),
    "q4k_chain_run": ([_P, _P], _I),
    "q4k_chain_launches": ([_P], _I),
    "q4k_chain_destroy": ([_P], None),
    "q4k_plan_create": ([_P, _U32, ctypes.POINTER(_P)], _I),
    "q4k_plan_gemm_exact": ([_P, _I], _I),
    "q4k_plan_destroy": ([_P], None),
    "q4k_plan_gemv": ([_P, _U32, _P, _P, _P, _U32, _U32], _I),
    "q4k_plan_gelu_mul": ([_P, _U32, _P, _P, _P, _U32], _I),
    "q4k_plan_lmhead": ([_P, _U32, _P, _P, _U32, _U32, _F, _U32, _P, _P, _P, _P], _I),
    "q4k_plan_gemv_q6k": ([_P, _U32, _P, _P, _P, _U32, _U32], _I),
    "q4k_plan_lmhead_q6k": ([_P, _U32, _P, _P, _U32, _U32, _F, _U32, _P, _P, _P, _P], _I),
    "q4k_plan_commit": ([_P], _I),
    "q4k_plan_run": ([_P, _P], _I),
    "q4k_plan_launches": ([_P], _I),
}


class Q4KError(RuntimeError):
    """A libq4k call returned an error status."""

    def __init__(self, code: int, message: str):
        super().__init__(f"libq4k error {code}: {message}")
        self.code = code


_lib: ctypes.CDLL | None = None


def lib() -> ctypes.CDLL:
    """Load libq4k.so (built by gemma4-webgpu_b200/build.py).  Raises if absent."""
    global _lib
    if _lib is not None:
        return _lib
    path = Path(os.environ.get("Q4K_LIB", LIB_PATH))
    if not path.exists():
        raise FileNotFoundError(
            f"{path} is missing: build it with `python gemma4-webgpu_b200/build.py` "
            "(there is no fallback implementation)"
        )
    L = ctypes.CDLL(str(path))
    for name, (args, res) in SIGNATURES.items():
        fn = getattr(L, name)
        fn.argtypes = args
        fn.restype = res
    _lib = L
    return L


def check(rc: int, ctx: int | None) -> None:
    if rc != Q4K_OK:
        msg = lib().q4k_last_error(ctx).decode() if ctx else "no context"
        raise Q4KError(rc, msg)
