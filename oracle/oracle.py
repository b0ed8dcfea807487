"""ctypes binding of the CPU oracle (oracle/q4k_oracle.c).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and the
CPU-baseline legs of bench.py.  The product (libq4k.so and the q4k package)
never imports this module.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
BUILD = HERE / "_build"

_lib = None


def build() -> None:
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)


def _cpu_has_v3() -> bool:
    try:
        flags = Path("/proc/cpuinfo").read_text().split("flags", 1)[1].split("\n", 1)[0].split()
    except (OSError, IndexError):
        return False
    return all(f in flags for f in ("avx2", "fma", "bmi2", "f16c"))


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is not None:
        return _lib
    name = "liboracle_q4k_v3.so" if _cpu_has_v3() else "liboracle_q4k.so"
    path = BUILD / name
    if not path.exists():
        build()
    L = ctypes.CDLL(str(path))
    P, I64, I = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int
    L.orc_f16_to_f32.argtypes = [ctypes.c_uint16]
    L.orc_f16_to_f32.restype = ctypes.c_float
    L.orc_f32_to_f16_rne.argtypes = [ctypes.c_float]
    L.orc_f32_to_f16_rne.restype = ctypes.c_uint16
    L.orc_f32_to_f16_trunc.argtypes = [ctypes.c_float]
    L.orc_f32_to_f16_trunc.restype = ctypes.c_uint16
    L.orc_q4k_scale_min.argtypes = [P, I, ctypes.POINTER(I), ctypes.POINTER(I)]
    L.orc_q4k_dequant_f32.argtypes = [P, I64, P]
    L.orc_q4k_dequant_f16.argtypes = [P, I64, P, I]
    L.orc_matmul_quant_f16.argtypes = [P, P, P, I64, I64, I64, I]
    L.orc_q4k_gemv.argtypes = [P, P, P, I64, I64, I64, I]
    L.orc_q4k_gemv_f64.argtypes = [P, P, P, P, I64, I64, I64, I]
    L.orc_q6k_dequant_f32.argtypes = [P, I64, P]
    L.orc_q6k_dequant_f16.argtypes = [P, I64, P]
    L.orc_q6k_gemv.argtypes = [P, P, P, I64, I64, I64, I]
    L.orc_q6k_gemv_f64.argtypes = [P, P, P, P, I64, I64, I64, I]
    L.orc_q5k_dequant_f32.argtypes = [P, I64, P]
    L.orc_q5k_dequant_f16.argtypes = [P, I64, P]
    L.orc_ple_stage1.argtypes = [P, P, I64, I64, P, P, ctypes.c_float, P]
    L.orc_logit_softcap.argtypes = [P, I64, ctypes.c_float]
    L.orc_argmax.argtypes = [P, I64]
    L.orc_argmax.restype = ctypes.c_uint32
    L.orc_topk256.argtypes = [P, I64, P, P]
    L.orc_gelu_mul.argtypes = [P, P, P, I64]
    L.orc_max_threads.restype = I
    _lib = L
    return L


def _p(a: np.ndarray) -> int:
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data


def max_threads() -> int:
    return lib().orc_max_threads()


def f32_to_f16_rne(v: float) -> int:
    return lib().orc_f32_to_f16_rne(v)


def f32_to_f16_trunc(v: float) -> int:
    return lib().orc_f32_to_f16_trunc(v)


def scale_min(block: np.ndarray, j: int) -> tuple[int, int]:
    sc, m = ctypes.c_int(), ctypes.c_int()
    b = np.ascontiguousarray(block, dtype=np.uint8)
    lib().orc_q4k_scale_min(_p(b), j, ctypes.byref(sc), ctypes.byref(m))
    return sc.value, m.value


def dequant_f32(blocks: np.ndarray) -> np.ndarray:
    b = np.ascontiguousarray(blocks, dtype=np.uint8).reshape(-1)
    nb = b.size // 144
    out = np.empty(nb * 256, dtype=np.float32)
    lib().orc_q4k_dequant_f32(_p(b), nb, _p(out))
    return out


def dequant_f16(blocks: np.ndarray, truncate: bool = False) -> np.ndarray:
    """f16 bit patterns (uint16) of the decoded weights."""
    b = np.ascontiguousarray(blocks, dtype=np.uint8).reshape(-1)
    nb = b.size // 144
    out = np.empty(nb * 256, dtype=np.uint16)
    lib().orc_q4k_dequant_f16(_p(b), nb, _p(out), 1 if truncate else 0)
    return out


def matmul_quant_f16(w16: np.ndarray, x: np.ndarray, M: int, N: int, threads: int = 0) -> np.ndarray:
    w = np.ascontiguousarray(w16, dtype=np.uint16)
    xx = np.ascontiguousarray(x, dtype=np.float32).reshape(-1, N)
    batch = xx.shape[0]
    y = np.empty((batch, M), dtype=np.float32)
    lib().orc_matmul_quant_f16(_p(w), _p(xx), _p(y), M, N, batch, threads)
    return y


def q4k_gemv(w: np.ndarray, x: np.ndarray, M: int, N: int, threads: int = 0) -> np.ndarray:
    """y[b, m] with the reference semantics (RNE f16 weights, WGSL order)."""
    wb = np.ascontiguousarray(w, dtype=np.uint8)
    xx = np.ascontiguousarray(x, dtype=np.float32).reshape(-1, N)
    batch = xx.shape[0]
    y = np.empty((batch, M), dtype=np.float32)
    lib().orc_q4k_gemv(_p(wb), _p(xx), _p(y), M, N, batch, threads)
    return y


def q4k_gemv_f64(w: np.ndarray, x: np.ndarray, M: int, N: int, threads: int = 0):
    """(y_f64 [batch, M], ||w_row||_2 [M]) on the same f16-rounded weights."""
    wb = np.ascontiguousarray(w, dtype=np.uint8)
    xx = np.ascontiguousarray(x, dtype=np.float32).reshape(-1, N)
    batch = xx.shape[0]
    y = np.empty((batch, M), dtype=np.float64)
    wn = np.empty(M, dtype=np.float64)
    lib().orc_q4k_gemv_f64(_p(wb), _p(xx), _p(y), _p(wn), M, N, batch, threads)
    return y, wn


def q6k_dequant_f32(blocks: np.ndarray) -> np.ndarray:
    """Q6_K super-blocks (GGUF layout, 210 bytes each) -> f32 (src/gguf.ts:316-368)."""
    b = np.ascontiguousarray(blocks, dtype=np.uint8).reshape(-1)
    nb = b.size // 210
    out = np.empty(nb * 256, dtype=np.float32)
    lib().orc_q6k_dequant_f32(_p(b), nb, _p(out))
    return out


def q6k_dequant_f16(blocks: np.ndarray) -> np.ndarray:
    """f16 bit patterns (uint16) of the decoded Q6_K weights (RNE)."""
    b = np.ascontiguousarray(blocks, dtype=np.uint8).reshape(-1)
    nb = b.size // 210
    out = np.empty(nb * 256, dtype=np.uint16)
    lib().orc_q6k_dequant_f16(_p(b), nb, _p(out))
    return out


def q6k_gemv(w: np.ndarray, x: np.ndarray, M: int, N: int, threads: int = 0) -> np.ndarray:
    """y[b, m] for a Q6_K matrix (GGUF bytes [M, N/256*210]), reference semantics."""
    wb = np.ascontiguousarray(w, dtype=np.uint8)
    xx = np.ascontiguousarray(x, dtype=np.float32).reshape(-1, N)
    y = np.empty((xx.shape[0], M), dtype=np.float32)
    lib().orc_q6k_gemv(_p(wb), _p(xx), _p(y), M, N, xx.shape[0], threads)
    return y


def q6k_gemv_f64(w: np.ndarray, x: np.ndarray, M: int, N: int, threads: int = 0):
    """(y_f64 [batch, M], ||w_row||_2 [M]) on the f16-rounded Q6_K weights."""
    wb = np.ascontiguousarray(w, dtype=np.uint8)
    xx = np.ascontiguousarray(x, dtype=np.float32).reshape(-1, N)
    y = np.empty((xx.shape[0], M), dtype=np.float64)
    wn = np.empty(M, dtype=np.float64)
    lib().orc_q6k_gemv_f64(_p(wb), _p(xx), _p(y), _p(wn), M, N, xx.shape[0], threads)
    return y, wn


def q5k_dequant_f32(blocks: np.ndarray) -> np.ndarray:
    """Q5_K super-blocks (GGUF layout, 176 bytes each) -> f32 (src/gguf.ts:212-256)."""
    b = np.ascontiguousarray(blocks, dtype=np.uint8).reshape(-1)
    nb = b.size // 176
    out = np.empty(nb * 256, dtype=np.float32)
    lib().orc_q5k_dequant_f32(_p(b), nb, _p(out))
    return out


def q5k_dequant_f16(blocks: np.ndarray) -> np.ndarray:
    """f16 bit patterns (uint16) of the decoded Q5_K values (RNE), the
    per-layer embedding the reference uploads."""
    b = np.ascontiguousarray(blocks, dtype=np.uint8).reshape(-1)
    nb = b.size // 176
    out = np.empty(nb * 256, dtype=np.uint16)
    lib().orc_q5k_dequant_f16(_p(b), nb, _p(out))
    return out


def ple_stage1(table: np.ndarray, tokens: np.ndarray, layers: int, projected: np.ndarray,
               norm_w16: np.ndarray, eps: float) -> np.ndarray:
    """shaders/ple_stage1_fuse.wgsl for every layer of T tokens: out [T, layers*256]."""
    tb = np.ascontiguousarray(table, dtype=np.uint8).reshape(-1)
    tk = np.ascontiguousarray(tokens, dtype=np.uint32).reshape(-1)
    pr = np.ascontiguousarray(projected, dtype=np.float32).reshape(tk.size, layers * 256)
    nw = np.ascontiguousarray(norm_w16, dtype=np.uint16).reshape(256)
    out = np.empty_like(pr)
    lib().orc_ple_stage1(_p(tb), _p(tk), tk.size, layers, _p(pr), _p(nw), eps, _p(out))
    return out


def logit_softcap(logits: np.ndarray, cap: float) -> np.ndarray:
    out = np.array(logits, dtype=np.float32, copy=True)
    lib().orc_logit_softcap(_p(out), out.size, cap)
    return out


def argmax(logits: np.ndarray) -> int:
    a = np.ascontiguousarray(logits, dtype=np.float32)
    return int(lib().orc_argmax(_p(a), a.size))


def topk256(logits: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    a = np.ascontiguousarray(logits, dtype=np.float32)
    vals = np.empty(256, dtype=np.float32)
    idx = np.empty(256, dtype=np.uint32)
    lib().orc_topk256(_p(a), a.size, _p(vals), _p(idx))
    return vals, idx


def gelu_mul(gate: np.ndarray, up: np.ndarray) -> np.ndarray:
    g = np.ascontiguousarray(gate, dtype=np.float32)
    u = np.ascontiguousarray(up, dtype=np.float32)
    out = np.empty_like(g)
    lib().orc_gelu_mul(_p(g), _p(u), _p(out), g.size)
    return out


def tolerance_ok(y: np.ndarray, y_ref: np.ndarray, wnorm: np.ndarray, x: np.ndarray,
                 rel: float = 1e-3, abs_scale: float = 1e-6):
    """Per-output bound |y - y_ref| <= rel*|y_ref| + abs_scale*||w_row||*||x||.

    Returns (ok, worst_ratio, l2_rel).  y, y_ref: [batch, M]; x: [batch, N].
    """
    y = np.asarray(y, dtype=np.float64)
    y_ref = np.asarray(y_ref, dtype=np.float64)
    xn = np.linalg.norm(np.asarray(x, dtype=np.float64).reshape(y.shape[0], -1), axis=1)
    bound = rel * np.abs(y_ref) + abs_scale * wnorm[None, :] * xn[:, None]
    err = np.abs(y - y_ref)
    ratio = float(np.max(err / bound)) if err.size else 0.0
    l2 = float(np.linalg.norm(y - y_ref) / max(np.linalg.norm(y_ref), 1e-300))
    return ratio <= 1.0, ratio, l2
