"""Host-side mirror of the reference's matmul-path operators on torch tensors.

Each method wraps one libq4k.so entry point and keeps the name, argument
meaning and error behaviour of the WebGPU pipeline it replaces in
src/engine.ts (matmulQuant, matmulQuantMR4, logitSoftcap, argmax, topk256,
geluMul and the lmHead sequence of sampleNextTokenSubmit).  PyTorch is only
the plumbing here: device memory, streams and tensors.  Every call launches
CUDA kernels of libq4k.so; there is no CPU or PyTorch fallback, and a failed
call raises Q4KError.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import torch

from . import _lib
from ._lib import Q4KError

QK_K = 256
BLOCK_BYTES = 144
Q5K_BLOCK_BYTES = 176  # Q5_K super-block (per-layer embedding table)
PLE_DIM = 256  # per_layer_input_dim: one Q5_K super-block per layer and token
Q6K_BLOCK_BYTES = 210


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _stream(stream: torch.cuda.Stream | None) -> int:
    s = stream if stream is not None else torch.cuda.current_stream()
    return s.cuda_stream


def _need(t: torch.Tensor, dtype: torch.dtype, name: str, device: torch.device) -> None:
    if not isinstance(t, torch.Tensor):
        raise TypeError(f"{name} must be a torch.Tensor")
    if t.device != device:
        raise ValueError(f"{name} is on {t.device}, expected {device}")
    if t.dtype != dtype:
        raise TypeError(f"{name} has dtype {t.dtype}, expected {dtype}")
    if not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")


@dataclass
class Selection:
    """Outputs of the fused LM head (one shard or the whole vocabulary)."""

    cand_val: torch.Tensor  # f32 [256]: per-residue max (topk256 values)
    cand_idx: torch.Tensor  # u32-as-int32 [256]: their global indices
    argmax: torch.Tensor  # int32 [1]
    logits: torch.Tensor | None  # f32 [V] softcapped logits, when requested

    def topk256_buffer(self) -> torch.Tensor:
        """The reference's topk256Result layout: f32[512] of (val, bitcast idx)
        pairs (shaders/topk256.wgsl:19-20)."""
        out = torch.empty(512, dtype=torch.float32, device=self.cand_val.device)
        out[0::2] = self.cand_val
        out[1::2] = self.cand_idx.view(torch.float32)
        return out


class Context:
    """A libq4k context on one CUDA device (q4k_create / q4k_destroy)."""

    def __init__(self, device: int | torch.device = 0):
        dev = torch.device("cuda", device) if isinstance(device, int) else torch.device(device)
        if dev.type != "cuda":
            raise ValueError("libq4k runs on CUDA devices only")
        self.device = torch.device("cuda", dev.index if dev.index is not None else torch.cuda.current_device())
        self._L = _lib.lib()
        handle = ctypes.c_void_p()
        with torch.cuda.device(self.device):
            rc = self._L.q4k_create(self.device.index, ctypes.byref(handle))
        if rc != _lib.Q4K_OK:
            raise Q4KError(rc, f"q4k_create(device={self.device.index}) failed")
        self._h = handle.value

    def close(self) -> None:
        if getattr(self, "_h", None):
            self._L.q4k_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def _check(self, rc: int) -> None:
        _lib.check(rc, self._h)

    def check(self) -> None:
        """Synchronize and raise Q4KError if a kernel gave up a bounded wait
        since the last check (q4k_check)."""
        self._check(self._L.q4k_check(self._h))

    def set_wait_limit(self, polls: int) -> None:
        """Polls each bounded wait of this context's kernels makes before it
        gives up (0: the built-in default; q4k_set_wait_limit)."""
        self._check(self._L.q4k_set_wait_limit(self._h, polls))

    # ---- matmulQuant / matmulQuantMR4 -----------------------------------

    def matmul_quant(self, input: torch.Tensor, weight: torch.Tensor, output: torch.Tensor, M: int, N: int,
                     stream: torch.cuda.Stream | None = None) -> torch.Tensor:
        """output[m] = sum_k f32(w16[m, k]) * input[k] -- the matmulQuant
        pipeline with bind group {input, weight, output, {M, N}}
        (shaders/matmul_quant.wgsl:12-16, src/engine.ts:332-341).  `weight`
        holds Q4_K bytes (uint8, M*N/256*144)."""
        _need(input, torch.float32, "input", self.device)
        _need(weight, torch.uint8, "weight", self.device)
        _need(output, torch.float32, "output", self.device)
        if input.numel() < N or output.numel() < M or weight.numel() < M * (N // QK_K) * BLOCK_BYTES:
            raise ValueError("buffer smaller than {M, N} requires")
        self._check(self._L.q4k_matmul_quant(self._h, _ptr(input), _ptr(weight), _ptr(output), M, N,
                                             _stream(stream)))
        return output

    def gemv(self, weight: torch.Tensor, x: torch.Tensor, M: int, N: int, out: torch.Tensor | None = None,
             stream: torch.cuda.Stream | None = None) -> torch.Tensor:
        """y[b, m] for x [batch, N] (or [N]); one weight stream per call."""
        _need(weight, torch.uint8, "weight", self.device)
        _need(x, torch.float32, "x", self.device)
        if x.numel() % N:
            raise ValueError(f"x has {x.numel()} elements, not a multiple of N={N}")
        batch = x.numel() // N
        if weight.numel() < M * (N // QK_K) * BLOCK_BYTES:
            raise ValueError("weight buffer smaller than M*N/256*144 bytes")
        if out is None:
            out = torch.empty((batch, M), dtype=torch.float32, device=self.device)
        _need(out, torch.float32, "out", self.device)
        if out.numel() < batch * M:
            raise ValueError("out smaller than batch*M")
        self._check(self._L.q4k_gemv(self._h, _ptr(weight), _ptr(x), _ptr(out), M, N, batch, _stream(stream)))
        return out

    def gemm(self, weight: torch.Tensor, x: torch.Tensor, M: int, N: int, out: torch.Tensor | None = None,
             stream: torch.cuda.Stream | None = None, f16x: bool = False) -> torch.Tensor:
        """y[t, m] for x [T, N] on the tensor cores (q4k_gemm): the batched
        prefill form of matmul_quant for many activation rows.  f16x: each
        activation row rounded once to f16 (q4k_gemm_f16x, half the
        tensor-core work, 2e-3 relative tolerance) instead of exact hi + lo."""
        _need(weight, torch.uint8, "weight", self.device)
        _need(x, torch.float32, "x", self.device)
        if x.numel() % N:
            raise ValueError(f"x has {x.numel()} elements, not a multiple of N={N}")
        T = x.numel() // N
        if weight.numel() < M * (N // QK_K) * BLOCK_BYTES:
            raise ValueError("weight buffer smaller than M*N/256*144 bytes")
        if out is None:
            out = torch.empty((T, M), dtype=torch.float32, device=self.device)
        _need(out, torch.float32, "out", self.device)
        if out.numel() < T * M:
            raise ValueError("out smaller than T*M")
        fn = self._L.q4k_gemm_f16x if f16x else self._L.q4k_gemm
        self._check(fn(self._h, _ptr(weight), _ptr(x), _ptr(out), M, N, T, _stream(stream)))
        return out

    def dequant_f16(self, weight: torch.Tensor, stream: torch.cuda.Stream | None = None) -> torch.Tensor:
        """The f16 weights the reference uploads (as int16 bit patterns)."""
        _need(weight, torch.uint8, "weight", self.device)
        if weight.numel() % BLOCK_BYTES:
            raise ValueError("weight size is not a whole number of 144-byte super-blocks")
        nb = weight.numel() // BLOCK_BYTES
        out = torch.empty(nb * QK_K, dtype=torch.int16, device=self.device)
        self._check(self._L.q4k_dequant_f16(self._h, _ptr(weight), _ptr(out), nb, _stream(stream)))
        return out

    # ---- per-layer embeddings (Q5_K table; see include/q4k.h) ---------------

    def q5k_dequant_f16(self, table: torch.Tensor, stream: torch.cuda.Stream | None = None) -> torch.Tensor:
        """The f16 values (int16 bit patterns) the reference uploads for a Q5_K
        table (decodeQ5_KBlock + f32ToF16Array), 256 per 176-byte super-block."""
        _need(table, torch.uint8, "table", self.device)
        if table.numel() % Q5K_BLOCK_BYTES:
            raise ValueError("table size is not a whole number of 176-byte super-blocks")
        nb = table.numel() // Q5K_BLOCK_BYTES
        out = torch.empty(nb * QK_K, dtype=torch.int16, device=self.device)
        self._check(self._L.q4k_q5k_dequant_f16(self._h, _ptr(table), _ptr(out), nb, _stream(stream)))
        return out

    def ple_stage1(self, table: torch.Tensor, token_ids: torch.Tensor, vocab: int, layers: int,
                   projected: torch.Tensor, norm_w: torch.Tensor, eps: float = 1e-6,
                   out: torch.Tensor | None = None, stream: torch.cuda.Stream | None = None) -> torch.Tensor:
        """shaders/ple_stage1_fuse.wgsl for every layer of T tokens (one
        launch): per-layer embedding rows gathered from the Q5_K table
        [vocab, layers*176 bytes], fused with the RMS-normalised projection.
        token_ids: int32 [T] on the device; projected: f32 [T, layers*256];
        norm_w: f16 bit patterns (int16) [256].  Returns f32 [T, layers*256]."""
        _need(table, torch.uint8, "table", self.device)
        _need(token_ids, torch.int32, "token_ids", self.device)
        _need(projected, torch.float32, "projected", self.device)
        _need(norm_w, torch.int16, "norm_w", self.device)
        T = token_ids.numel()
        if table.numel() < vocab * layers * Q5K_BLOCK_BYTES:
            raise ValueError("table smaller than vocab*layers*176 bytes")
        if projected.numel() != T * layers * PLE_DIM or norm_w.numel() != PLE_DIM:
            raise ValueError("projected must be [T, layers*256] and norm_w [256]")
        if out is None:
            out = torch.empty((T, layers * PLE_DIM), dtype=torch.float32, device=self.device)
        _need(out, torch.float32, "out", self.device)
        if out.numel() != T * layers * PLE_DIM:
            raise ValueError("out must be [T, layers*256]")
        self._check(self._L.q4k_ple_stage1(self._h, _ptr(table), _ptr(token_ids), T, vocab, layers, _ptr(projected),
                                           _ptr(norm_w), eps, _ptr(out), _stream(stream)))
        return out

    # ---- Q6_K matrices (device layout; see include/q4k.h) ---------------------

    def q6k_device_bytes(self, M: int, N: int) -> int:
        """Bytes of the device layout of an M x N Q6_K matrix."""
        if N % QK_K:
            raise ValueError(f"N={N} is not a multiple of {QK_K}")
        return int(self._L.q4k_q6k_device_bytes(M, N))

    def q6k_repack(self, w_gguf: torch.Tensor, M: int, N: int, out: torch.Tensor | None = None,
                   stream: torch.cuda.Stream | None = None) -> torch.Tensor:
        """GGUF Q6_K bytes (uint8, M*N/256*210, on the device) -> the device
        layout the Q6_K calls read: the load-time step that replaces the
        reference's dequantizeQ6_K + f32ToF16Array upload."""
        _need(w_gguf, torch.uint8, "w_gguf", self.device)
        if w_gguf.numel() < M * (N // QK_K) * Q6K_BLOCK_BYTES:
            raise ValueError("w_gguf smaller than M*N/256*210 bytes")
        nbytes = self.q6k_device_bytes(M, N)
        if out is None:
            out = torch.empty(nbytes, dtype=torch.uint8, device=self.device)
        _need(out, torch.uint8, "out", self.device)
        if out.numel() < nbytes:
            raise ValueError(f"out smaller than {nbytes} bytes")
        self._check(self._L.q4k_q6k_repack(self._h, _ptr(w_gguf), _ptr(out), M, N, _stream(stream)))
        return out

    def _need_q6(self, w_dev: torch.Tensor, M: int, N: int) -> None:
        _need(w_dev, torch.uint8, "w_dev", self.device)
        if w_dev.numel() < self.q6k_device_bytes(M, N):
            raise ValueError("w_dev smaller than q6k_device_bytes(M, N)")

    def q6k_dequant_f16(self, w_dev: torch.Tensor, M: int, N: int,
                        stream: torch.cuda.Stream | None = None) -> torch.Tensor:
        """The f16 weights (int16 bit patterns, [M, N]) the Q6_K GEMV multiplies."""
        self._need_q6(w_dev, M, N)
        out = torch.empty((M, N), dtype=torch.int16, device=self.device)
        self._check(self._L.q4k_q6k_dequant_f16(self._h, _ptr(w_dev), M, N, _ptr(out), _stream(stream)))
        return out

    def q6k_gemv(self, w_dev: torch.Tensor, x: torch.Tensor, M: int, N: int, out: torch.Tensor | None = None,
                 stream: torch.cuda.Stream | None = None) -> torch.Tensor:
        """y[b, m] for a Q6_K matrix in the device layout, x [batch, N] (or [N])."""
        self._need_q6(w_dev, M, N)
        _need(x, torch.float32, "x", self.device)
        if x.numel() % N:
            raise ValueError(f"x has {x.numel()} elements, not a multiple of N={N}")
        batch = x.numel() // N
        if out is None:
            out = torch.empty((batch, M), dtype=torch.float32, device=self.device)
        _need(out, torch.float32, "out", self.device)
        if out.numel() < batch * M:
            raise ValueError("out smaller than batch*M")
        self._check(self._L.q4k_q6k_gemv(self._h, _ptr(w_dev), _ptr(x), _ptr(out), M, N, batch, _stream(stream)))
        return out

    def q6k_lmhead_select(self, w_dev: torch.Tensor, x: torch.Tensor, V: int, N: int, cap: float = 30.0,
                          row_offset: int = 0, return_logits: bool = False, out: Selection | None = None,
                          stream: torch.cuda.Stream | None = None) -> Selection:
        """The fused LM head (lmHead matmul + logitSoftcap + argmax/topk256) of
        a Q6_K head in the device layout."""
        self._need_q6(w_dev, V, N)
        _need(x, torch.float32, "x", self.device)
        if x.numel() != N:
            raise ValueError(f"x has {x.numel()} elements, expected N={N}")
        if out is None:
            out = Selection(
                cand_val=torch.empty(256, dtype=torch.float32, device=self.device),
                cand_idx=torch.empty(256, dtype=torch.int32, device=self.device),
                argmax=torch.empty(1, dtype=torch.int32, device=self.device),
                logits=torch.empty(V, dtype=torch.float32, device=self.device) if return_logits else None,
            )
        self._check(self._L.q4k_q6k_lmhead_select(
            self._h, _ptr(w_dev), _ptr(x), V, N, cap, row_offset, _ptr(out.logits), _ptr(out.cand_val),
            _ptr(out.cand_idx), _ptr(out.argmax), _stream(stream)))
        return out

    # ---- LM-head consumers ------------------------------------------------

    def logit_softcap(self, logits: torch.Tensor, cap: float = 30.0,
                      stream: torch.cuda.Stream | None = None) -> torch.Tensor:
        """In place, shaders/logit_softcap.wgsl:9-16."""
        _need(logits, torch.float32, "logits", self.device)
        self._check(self._L.q4k_logit_softcap(self._h, _ptr(logits), logits.numel(), cap, _stream(stream)))
        return logits

    def argmax(self, logits: torch.Tensor, out: torch.Tensor | None = None,
               stream: torch.cuda.Stream | None = None) -> torch.Tensor:
        """int32 [1], shaders/argmax.wgsl:7-34 tie rule."""
        _need(logits, torch.float32, "logits", self.device)
        out = torch.empty(1, dtype=torch.int32, device=self.device) if out is None else out
        self._check(self._L.q4k_argmax(self._h, _ptr(logits), logits.numel(), _ptr(out), _stream(stream)))
        return out

    def topk256(self, logits: torch.Tensor, out: torch.Tensor | None = None,
                stream: torch.cuda.Stream | None = None) -> torch.Tensor:
        """f32 [512] (val, bitcast idx) pairs, shaders/topk256.wgsl:5-21."""
        _need(logits, torch.float32, "logits", self.device)
        out = torch.empty(512, dtype=torch.float32, device=self.device) if out is None else out
        self._check(self._L.q4k_topk256(self._h, _ptr(logits), logits.numel(), _ptr(out), _stream(stream)))
        return out

    def select_rows(self, logits: torch.Tensor, cap: float = 30.0, cand_val: torch.Tensor | None = None,
                    cand_idx: torch.Tensor | None = None, argmax: torch.Tensor | None = None,
                    stream: torch.cuda.Stream | None = None) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
        """Softcap (cap > 0, in place) + topk256 + argmax of every row of
        logits [B, n] in one launch (q4k_select_rows).  Returns (cand_val
        [B, 256] f32, cand_idx [B, 256] int32, argmax [B] int32)."""
        _need(logits, torch.float32, "logits", self.device)
        if logits.dim() != 2:
            raise ValueError("logits must be [B, n]")
        B, n = logits.shape
        f32 = dict(dtype=torch.float32, device=self.device)
        i32 = dict(dtype=torch.int32, device=self.device)
        cand_val = torch.empty((B, 256), **f32) if cand_val is None else cand_val
        cand_idx = torch.empty((B, 256), **i32) if cand_idx is None else cand_idx
        argmax = torch.empty(B, **i32) if argmax is None else argmax
        _need(cand_val, torch.float32, "cand_val", self.device)
        _need(cand_idx, torch.int32, "cand_idx", self.device)
        _need(argmax, torch.int32, "argmax", self.device)
        if cand_val.numel() < B * 256 or cand_idx.numel() < B * 256 or argmax.numel() < B:
            raise ValueError("output buffers smaller than [B, 256] / [B]")
        self._check(self._L.q4k_select_rows(self._h, _ptr(logits), B, n, cap, _ptr(cand_val), _ptr(cand_idx),
                                            _ptr(argmax), _stream(stream)))
        return cand_val, cand_idx, argmax

    def gelu_mul(self, gate: torch.Tensor, up: torch.Tensor, out: torch.Tensor | None = None,
                 stream: torch.cuda.Stream | None = None) -> torch.Tensor:
        """GELU_tanh(gate) * up, shaders/gelu_mul.wgsl."""
        _need(gate, torch.float32, "gate", self.device)
        _need(up, torch.float32, "up", self.device)
        if gate.numel() != up.numel():
            raise ValueError("gate and up differ in size")
        out = torch.empty_like(gate) if out is None else out
        self._check(self._L.q4k_gelu_mul(self._h, _ptr(gate), _ptr(up), _ptr(out), gate.numel(), _stream(stream)))
        return out

    def lmhead_select(self, weight: torch.Tensor, x: torch.Tensor, V: int, N: int, cap: float = 30.0,
                      row_offset: int = 0, return_logits: bool = False,
                      out: Selection | None = None, stream: torch.cuda.Stream | None = None) -> Selection:
        """lmHead matmul + logitSoftcap + argmax/topk256 in one launch
        (src/engine.ts:1686-1741) over vocabulary rows [row_offset, row_offset+V)."""
        _need(weight, torch.uint8, "weight", self.device)
        _need(x, torch.float32, "x", self.device)
        if x.numel() != N:
            raise ValueError(f"x has {x.numel()} elements, expected N={N}")
        if weight.numel() < V * (N // QK_K) * BLOCK_BYTES:
            raise ValueError("weight buffer smaller than V*N/256*144 bytes")
        if out is None:
            out = Selection(
                cand_val=torch.empty(256, dtype=torch.float32, device=self.device),
                cand_idx=torch.empty(256, dtype=torch.int32, device=self.device),
                argmax=torch.empty(1, dtype=torch.int32, device=self.device),
                logits=torch.empty(V, dtype=torch.float32, device=self.device) if return_logits else None,
            )
        self._check(self._L.q4k_lmhead_select(
            self._h, _ptr(weight), _ptr(x), V, N, cap, row_offset, _ptr(out.logits), _ptr(out.cand_val),
            _ptr(out.cand_idx), _ptr(out.argmax), _stream(stream)))
        return out

    def exchange(self, rank: int, world: int) -> "Exchange":
        """A mailbox for the fused sharded LM head (see Exchange)."""
        return Exchange(self, rank, world)

    def lmhead_select_sharded(self, ex: "Exchange", weight: torch.Tensor, x: torch.Tensor, V: int, N: int,
                              cap: float = 30.0, row_offset: int = 0, out: Selection | None = None,
                              stream: torch.cuda.Stream | None = None) -> Selection:
        """This rank's rows [row_offset, row_offset+V) of a vocabulary-sharded
        LM head, the candidate exchange with every rank over NVLink and the
        merge, in one launch: the whole head's candidates and argmax."""
        _need(weight, torch.uint8, "weight", self.device)
        _need(x, torch.float32, "x", self.device)
        if x.numel() != N:
            raise ValueError(f"x has {x.numel()} elements, expected N={N}")
        if weight.numel() < V * (N // QK_K) * BLOCK_BYTES:
            raise ValueError("weight buffer smaller than V*N/256*144 bytes")
        if out is None:
            out = Selection(
                cand_val=torch.empty(256, dtype=torch.float32, device=self.device),
                cand_idx=torch.empty(256, dtype=torch.int32, device=self.device),
                argmax=torch.empty(1, dtype=torch.int32, device=self.device),
                logits=None,
            )
        self._check(self._L.q4k_lmhead_select_sharded(
            self._h, ex._h, _ptr(weight), _ptr(x), V, N, cap, row_offset, _ptr(out.cand_val), _ptr(out.cand_idx),
            _ptr(out.argmax), _stream(stream)))
        return out

    def merge_candidates(self, vals: torch.Tensor, idx: torch.Tensor, out: Selection | None = None,
                         stream: torch.cuda.Stream | None = None) -> Selection:
        """[G, 256] gathered shard candidates -> one Selection (no logits)."""
        _need(vals, torch.float32, "vals", self.device)
        _need(idx, torch.int32, "idx", self.device)
        G = vals.numel() // 256
        if vals.numel() != G * 256 or idx.numel() != G * 256:
            raise ValueError("vals/idx must hold G*256 entries")
        if out is None:
            out = Selection(
                cand_val=torch.empty(256, dtype=torch.float32, device=self.device),
                cand_idx=torch.empty(256, dtype=torch.int32, device=self.device),
                argmax=torch.empty(1, dtype=torch.int32, device=self.device),
                logits=None,
            )
        self._check(self._L.q4k_merge_candidates(self._h, _ptr(vals), _ptr(idx), G, _ptr(out.cand_val),
                                                 _ptr(out.cand_idx), _ptr(out.argmax), _stream(stream)))
        return out


class Exchange:
    """This rank's mailbox for the fused sharded LM head (q4k_exchange_*):
    create on every rank, share `handle` with the other ranks out of band,
    then `open(peer, handle)` every peer."""

    HANDLE_BYTES = 64

    def __init__(self, ctx: "Context", rank: int, world: int):
        self._ctx = ctx
        self._L = ctx._L
        self.rank, self.world = rank, world
        h = ctypes.c_void_p()
        buf = ctypes.create_string_buffer(self.HANDLE_BYTES)
        ctx._check(self._L.q4k_exchange_create(ctx._h, rank, world, ctypes.byref(h), buf))
        self._h = h
        self.handle = bytes(buf.raw)

    def open(self, peer: int, handle: bytes) -> None:
        if len(handle) != self.HANDLE_BYTES:
            raise ValueError("bad exchange handle")
        buf = ctypes.create_string_buffer(handle, self.HANDLE_BYTES)
        self._ctx._check(self._L.q4k_exchange_open(self._h, peer, buf))

    def open_local(self, peer: int, other: "Exchange") -> None:
        """Map `other`, rank `peer`'s mailbox created in this process
        (q4k_exchange_open_local)."""
        self._ctx._check(self._L.q4k_exchange_open_local(self._h, peer, other._h))

    def close(self) -> None:
        if self._h:
            self._L.q4k_exchange_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class Plan:
    """A recorded matmul-path step replayed with two launches per stage
    (q4k_plan_*): the engine's "encode once, submit per token" model
    (encodeTransformerPass + queue.submit, src/engine.ts:1466-1626, 1748).
    Tensors are bound at record time, like bind groups, and kept alive by the
    plan.  Operations in one stage must not depend on each other, except that
    a GEMV may read the `act` of a gelu_mul recorded in the same stage.

    batch 1..16 runs on the GEMV engine; batch >= 64 (prefill, or many
    sequences sharing the weights) runs each stage as one tcgen05 GEMM launch
    over all its matrices, with activations rounded once to f16 (the 2e-3
    prefill tolerance) unless `exact` asks for the exact f16 hi + lo split
    (the GEMV tolerance, twice the tensor-core work)."""

    def __init__(self, ctx: Context, batch: int = 1, exact: bool = False):
        self.ctx = ctx
        self.batch = batch
        self._L = ctx._L
        h = ctypes.c_void_p()
        ctx._check(self._L.q4k_plan_create(ctx._h, batch, ctypes.byref(h)))
        self._h = h.value
        self._keep: list[torch.Tensor] = []
        self.committed = False
        self.exact = exact
        if batch > 16 and exact:
            ctx._check(self._L.q4k_plan_gemm_exact(self._h, 1))

    def _bind(self, *ts):
        for t in ts:
            if t is not None:
                self._keep.append(t)

    def gemv(self, stage: int, weight: torch.Tensor, x: torch.Tensor, y: torch.Tensor, M: int, N: int) -> None:
        dev = self.ctx.device
        _need(weight, torch.uint8, "weight", dev)
        _need(x, torch.float32, "x", dev)
        _need(y, torch.float32, "y", dev)
        if x.numel() < self.batch * N or y.numel() < self.batch * M:
            raise ValueError("x / y smaller than batch x N / batch x M")
        if weight.numel() < M * (N // QK_K) * BLOCK_BYTES:
            raise ValueError("weight buffer smaller than M*N/256*144 bytes")
        self.ctx._check(self._L.q4k_plan_gemv(self._h, stage, _ptr(weight), _ptr(x), _ptr(y), M, N))
        self._bind(weight, x, y)

    def gemv_q6k(self, stage: int, w_dev: torch.Tensor, x: torch.Tensor, y: torch.Tensor, M: int, N: int) -> None:
        """A Q6_K GEMV (weights in the device layout, Context.q6k_repack)."""
        dev = self.ctx.device
        self.ctx._need_q6(w_dev, M, N)
        _need(x, torch.float32, "x", dev)
        _need(y, torch.float32, "y", dev)
        if x.numel() < self.batch * N or y.numel() < self.batch * M:
            raise ValueError("x / y smaller than batch x N / batch x M")
        self.ctx._check(self._L.q4k_plan_gemv_q6k(self._h, stage, _ptr(w_dev), _ptr(x), _ptr(y), M, N))
        self._bind(w_dev, x, y)

    def gelu_mul(self, stage: int, gate: torch.Tensor, up: torch.Tensor, act: torch.Tensor) -> None:
        dev = self.ctx.device
        for t, n in ((gate, "gate"), (up, "up"), (act, "act")):
            _need(t, torch.float32, n, dev)
        n = gate.numel() // self.batch
        self.ctx._check(self._L.q4k_plan_gelu_mul(self._h, stage, _ptr(gate), _ptr(up), _ptr(act), n))
        self._bind(gate, up, act)

    def lmhead(self, stage: int, weight: torch.Tensor, x: torch.Tensor, V: int, N: int, cap: float,
               out: Selection, row_offset: int = 0) -> None:
        dev = self.ctx.device
        _need(weight, torch.uint8, "weight", dev)
        _need(x, torch.float32, "x", dev)
        self.ctx._check(self._L.q4k_plan_lmhead(
            self._h, stage, _ptr(weight), _ptr(x), V, N, cap, row_offset, _ptr(out.logits), _ptr(out.cand_val),
            _ptr(out.cand_idx), _ptr(out.argmax)))
        self._bind(weight, x, out.logits, out.cand_val, out.cand_idx, out.argmax)

    def lmhead_q6k(self, stage: int, w_dev: torch.Tensor, x: torch.Tensor, V: int, N: int, cap: float,
                   out: Selection, row_offset: int = 0) -> None:
        """The fused LM head of a Q6_K head in the device layout."""
        dev = self.ctx.device
        self.ctx._need_q6(w_dev, V, N)
        _need(x, torch.float32, "x", dev)
        self.ctx._check(self._L.q4k_plan_lmhead_q6k(
            self._h, stage, _ptr(w_dev), _ptr(x), V, N, cap, row_offset, _ptr(out.logits), _ptr(out.cand_val),
            _ptr(out.cand_idx), _ptr(out.argmax)))
        self._bind(w_dev, x, out.logits, out.cand_val, out.cand_idx, out.argmax)

    def commit(self) -> "Plan":
        self.ctx._check(self._L.q4k_plan_commit(self._h))
        self.committed = True
        return self

    def run(self, stream: torch.cuda.Stream | None = None) -> None:
        self.ctx._check(self._L.q4k_plan_run(self._h, _stream(stream)))

    def launches(self) -> int:
        return self._L.q4k_plan_launches(self._h)

    def close(self) -> None:
        if getattr(self, "_h", None):
            self._L.q4k_plan_destroy(self._h)
            self._h = None
            self._keep.clear()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


_contexts: dict[int, Context] = {}


def context(device: int | None = None) -> Context:
    """The cached per-device Context (created on first use)."""
    if device is None:
        device = torch.cuda.current_device()
    if device not in _contexts:
        _contexts[device] = Context(device)
    return _contexts[device]

