"""The matmul call sites of one synthetic Gemma-4-E2B-shaped decode step.

Mirrors the per-token matmul dispatch list of encodeTransformerPass
(src/engine.ts:1539-1619) and the LM head of sampleNextTokenSubmit
(src/engine.ts:1686-1741), at the shapes of the benchmark's config 3:
35 layers x {q 2048x1536, k 256x1536, v 256x1536, o 1536x2048,
gate 6144x1536, up 6144x1536, down 1536x6144} + the 262144x1536 LM head,
all Q4_K from the seeded synthetic generator.

Only the matmul path is in scope, so the non-matmul passes between the
GEMVs (norms, RoPE, attention, residual adds) are not run.  Each layer
therefore reads fixed seeded activations: q/k/v/gate/up and the LM head
read x_h [batch, 1536], o reads x_attn [batch, 2048]; down reads
gelu_mul(gate, up) of the same layer, as in the reference
(src/engine.ts:1589-1605).  Layers do not feed one another, so the step's
only data dependency is gate/up -> gelu_mul -> down.

Two ways to run it:
  * run()        -- a Plan with two stages (every GEMV that reads x_h/x_attn
                    plus the fused LM head; then gelu_mul + down for all
                    layers): 4 kernel launches per step;
  * run_serial() -- one libq4k call per reference dispatch, in the
                    reference's order (246 calls per step at batch 1).
"""
from __future__ import annotations

from dataclasses import dataclass, field

import ctypes

import numpy as np
import torch

from . import synth
from .ops import Context, Plan, Selection

CONFIG = 3  # seeds: synth.seed_for(3, matrix_id)


@dataclass
class E2BShape:
    layers: int = 35
    hidden: int = 1536
    q: int = 2048  # 8 heads x 256
    kv: int = 256  # 1 KV head x 256
    ffn: int = 6144
    vocab: int = 262144
    softcap: float = 30.0


LAYER_MATS = ("q", "k", "v", "o", "gate", "up", "down")


def layer_shapes(s: E2BShape) -> dict[str, tuple[int, int]]:
    """(rows M, cols N) of each per-layer matrix."""
    return {
        "q": (s.q, s.hidden),
        "k": (s.kv, s.hidden),
        "v": (s.kv, s.hidden),
        "o": (s.hidden, s.q),
        "gate": (s.ffn, s.hidden),
        "up": (s.ffn, s.hidden),
        "down": (s.hidden, s.ffn),
    }


def matrix_seed(layer: int, name: str) -> int:
    return synth.seed_for(CONFIG, 8 * layer + LAYER_MATS.index(name))


LMHEAD_SEED = synth.seed_for(CONFIG, 999)


@dataclass
class DecodeStep:
    """Device-resident weights, activations and outputs of the synthetic step."""

    ctx: Context
    shape: E2BShape = field(default_factory=E2BShape)
    batch: int = 1
    weights: dict = field(default_factory=dict)  # (layer, name) -> uint8 tensor
    lm_head: torch.Tensor | None = None
    share_weights_with: "DecodeStep | None" = None  # reuse another step's (same-shape) device weights

    def __post_init__(self):
        dev = self.ctx.device
        s, B = self.shape, self.batch
        shapes = layer_shapes(s)
        if self.share_weights_with is not None:
            other = self.share_weights_with
            if other.shape != s:
                raise ValueError("shared weights need the same shape")
            self.weights = other.weights
            self.lm_head = other.lm_head
        else:
            for layer in range(s.layers):
                for name in LAYER_MATS:
                    M, N = shapes[name]
                    w = synth.q4k_matrix(M, N, matrix_seed(layer, name))
                    self.weights[(layer, name)] = torch.from_numpy(w).to(dev)
            self.lm_head = torch.from_numpy(synth.q4k_matrix(s.vocab, s.hidden, LMHEAD_SEED)).to(dev)
        # the step's inputs share one buffer (one host->device copy per token)
        self.inputs = torch.empty(B * (s.hidden + s.q), dtype=torch.float32, device=dev)
        self.x_h = self.inputs[: B * s.hidden].view(B, s.hidden)
        self.x_attn = self.inputs[B * s.hidden:].view(B, s.q)
        self.x_h.copy_(torch.from_numpy(synth.activations(B, s.hidden, synth.seed_for(CONFIG, 100))))
        self.x_attn.copy_(torch.from_numpy(synth.activations(B, s.q, synth.seed_for(CONFIG, 101))))
        f32 = dict(dtype=torch.float32, device=dev)
        # distinct outputs per layer: a plan runs the layers concurrently
        self.out = {(layer, name): torch.empty((B, shapes[name][0]), **f32)
                    for layer in range(s.layers) for name in LAYER_MATS}
        self.act = [torch.empty((B, s.ffn), **f32) for _ in range(s.layers)]
        if B == 1:
            # candidates and argmax share one buffer (one device->host copy per token)
            self.results = torch.empty(513, dtype=torch.int32, device=dev)
            self.sel = Selection(
                cand_val=self.results[:256].view(torch.float32),
                cand_idx=self.results[256:512],
                argmax=self.results[512:],
                logits=None,
            )
        else:
            self.logits = torch.empty((B, s.vocab), **f32)
            # per row: candidates and argmax, all rows in one buffer (one copy back)
            self.results = torch.empty(B * 513, dtype=torch.int32, device=dev)
            self.cand_val = self.results[: 256 * B].view(torch.float32).view(B, 256)
            self.cand_idx = self.results[256 * B: 512 * B].view(B, 256)
            self.argmax = self.results[512 * B:]
        self._plan: Plan | None = None

    # ---- accounting ---------------------------------------------------------

    def weight_bytes(self) -> int:
        s = self.shape
        per_layer = sum(synth.q4k_bytes(M, N) for M, N in layer_shapes(s).values())
        return s.layers * per_layer + synth.q4k_bytes(s.vocab, s.hidden)

    def algorithmic_bytes(self) -> int:
        """Bytes one step must move at minimum: Q4_K weights, each GEMV's f32
        input and output, the gelu_mul operands, and the LM head's input plus
        its 2 KB of candidates (per activation row)."""
        s, B = self.shape, self.batch
        total = self.weight_bytes()
        for M, N in layer_shapes(s).values():
            total += s.layers * 4 * B * (M + N)
        total += s.layers * 3 * 4 * B * s.ffn           # gelu_mul: gate, up in; act out
        total += 4 * B * s.hidden + B * (256 * 8 + 4)   # LM head: x in, candidates + argmax out
        return total

    def stage0_bytes(self) -> int:
        """Algorithmic bytes of the plan's first engine launch: every GEMV but
        down, and the LM head."""
        s, B = self.shape, self.batch
        total = 0
        for name, (M, N) in layer_shapes(s).items():
            if name != "down":
                total += s.layers * (synth.q4k_bytes(M, N) + 4 * B * (M + N))
        return total + synth.q4k_bytes(s.vocab, s.hidden) + 4 * B * s.hidden + B * (256 * 8 + 4)

    def stage1_bytes(self) -> int:
        """Algorithmic bytes of the plan's second engine launch: gelu_mul
        (gate, up in; act out) and the down projections."""
        s, B = self.shape, self.batch
        M, N = layer_shapes(s)["down"]
        return s.layers * (synth.q4k_bytes(M, N) + 4 * B * (M + N) + 3 * 4 * B * s.ffn)

    def launches_per_step(self) -> int:
        return self.plan().launches() + (0 if self.batch == 1 else 1)

    def serial_calls_per_step(self) -> int:
        per_layer = len(LAYER_MATS) + 1  # 7 GEMVs + gelu_mul
        lm = 1 if self.batch == 1 else 2
        return self.shape.layers * per_layer + lm

    # ---- the plan ---------------------------------------------------------------

    def plan(self, stages: tuple[int, ...] = (0, 1)) -> Plan:
        """Record the step (or some of its stages) as a Plan.  Stage 0: every
        GEMV reading x_h / x_attn and the LM head; stage 1: gelu_mul and down."""
        if stages == (0, 1) and self._plan is not None:
            return self._plan
        c, s, B = self.ctx, self.shape, self.batch
        shapes = layer_shapes(s)
        p = Plan(c, batch=B)
        if 0 in stages:
            for layer in range(s.layers):
                for name in ("q", "k", "v", "o", "gate", "up"):
                    M, N = shapes[name]
                    x = self.x_attn if name == "o" else self.x_h
                    p.gemv(0, self.weights[(layer, name)], x, self.out[(layer, name)], M, N)
            if B == 1:
                p.lmhead(0, self.lm_head, self.x_h, s.vocab, s.hidden, s.softcap, self.sel)
            else:
                p.gemv(0, self.lm_head, self.x_h, self.logits, s.vocab, s.hidden)
        if 1 in stages:
            st = 1 if 0 in stages else 0
            for layer in range(s.layers):
                p.gelu_mul(st, self.out[(layer, "gate")], self.out[(layer, "up")], self.act[layer])
                M, N = shapes["down"]
                p.gemv(st, self.weights[(layer, "down")], self.act[layer], self.out[(layer, "down")], M, N)
        p.commit()
        if stages == (0, 1):
            self._plan = p
        return p

    def _select_rows(self, stream) -> None:
        """Softcap + topk256 + argmax of every row's logits, one launch."""
        self.ctx.select_rows(self.logits, self.shape.softcap, self.cand_val, self.cand_idx, self.argmax,
                             stream=stream)

    def run(self, stream: torch.cuda.Stream | None = None) -> None:
        """One decode step through the plan (4 launches at batch 1)."""
        self.plan().run(stream)
        if self.batch > 1:
            self._select_rows(stream)

    def run_serial(self, stream: torch.cuda.Stream | None = None) -> None:
        """One decode step as one libq4k call per reference dispatch, in the
        order of encodeTransformerPass + sampleNextTokenSubmit."""
        c, s, B = self.ctx, self.shape, self.batch
        shapes = layer_shapes(s)
        W, O = self.weights, self.out
        for layer in range(s.layers):
            for name in ("q", "k", "v"):
                M, N = shapes[name]
                c.gemv(W[(layer, name)], self.x_h, M, N, out=O[(layer, name)], stream=stream)
            M, N = shapes["o"]
            c.gemv(W[(layer, "o")], self.x_attn, M, N, out=O[(layer, "o")], stream=stream)
            for name in ("gate", "up"):
                M, N = shapes[name]
                c.gemv(W[(layer, name)], self.x_h, M, N, out=O[(layer, name)], stream=stream)
            c.gelu_mul(O[(layer, "gate")], O[(layer, "up")], out=self.act[layer], stream=stream)
            M, N = shapes["down"]
            c.gemv(W[(layer, "down")], self.act[layer], M, N, out=O[(layer, "down")], stream=stream)
        if B == 1:
            c.lmhead_select(self.lm_head, self.x_h, s.vocab, s.hidden, s.softcap, out=self.sel, stream=stream)
        else:
            c.gemv(self.lm_head, self.x_h, s.vocab, s.hidden, out=self.logits, stream=stream)
            self._select_rows(stream)

    def result_tensors(self) -> list[torch.Tensor]:
        """What a decode step hands back to the host: the sampled token and the
        2 KB topk256 candidates (src/engine.ts:1731-1741)."""
        # batch 1: cand_val [256] f32 | cand_idx [256] | argmax [1]; batch B:
        # cand_val [B][256] | cand_idx [B][256] | argmax [B]
        return [self.results]

    def sample_matrices(self, layers: int = 1) -> list[tuple[np.ndarray, int, int]]:
        """Host copies (regenerated from the same seeds) of the first `layers`
        layers' matrices, for CPU timing samples."""
        out = []
        for layer in range(layers):
            for name, (M, N) in layer_shapes(self.shape).items():
                out.append((synth.q4k_matrix(M, N, matrix_seed(layer, name)), M, N))
        return out


class StepGraph:
    """A decode step captured once as a CUDA graph and replayed per token (the
    way the engine pre-builds its bind groups and only re-dispatches).

    host_io = (inputs_host, results_host), pinned host tensors shaped like
    step.inputs and step.results: the graph then also copies the token's
    inputs in and its results out, so one replay is the whole host-visible
    step (read results_host after synchronizing the stream)."""

    def __init__(self, step: DecodeStep, stream: torch.cuda.Stream | None = None, body=None,
                 host_io: tuple[torch.Tensor, torch.Tensor] | None = None):
        self.step = step
        self.stream = stream or torch.cuda.Stream(device=step.ctx.device)
        body = body or step.run
        if host_io is not None:
            x_host, r_host = host_io
            inner = body

            def body(st):  # noqa: F811 -- the step with its host copies around it
                step.inputs.copy_(x_host, non_blocking=True)
                inner(st)
                r_host.copy_(step.results, non_blocking=True)
        with torch.cuda.stream(self.stream):
            body(self.stream)  # warm-up outside capture
        self.stream.synchronize()
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph, stream=self.stream):
            body(self.stream)

    def replay(self) -> None:
        with torch.cuda.stream(self.stream):
            self.graph.replay()


class BatchedSweep:
    """Config 4: the 35 layers' seven matrices at T activation rows per step
    (prefill, or T independent sequences sharing the weights), without the
    LM head, as a two-stage Plan: stage 0 = every q/k/v/o/gate/up, stage 1 =
    gelu_mul + every down (src/engine.ts:1589-1605).  T <= 16 runs on the
    GEMV engine (one weight stream per matrix for all T rows); T >= 64 runs
    each stage as ONE tcgen05 GEMM launch over all of its matrices (after one
    activation-preparation launch), activations rounded once to f16 (the
    2e-3 prefill tolerance) unless exact=True asks for the exact f16 hi + lo
    split.  mode="streams" (T >= 64) instead calls q4k_gemm per matrix,
    spreading the independent layers over `streams` CUDA streams with a
    library context each -- the earlier form, kept for comparison."""

    def __init__(self, step: DecodeStep, T: int, streams: int = 18, f16x: bool | None = None,
                 exact: bool | None = None, mode: str = "plan"):
        if exact is None:
            exact = not f16x if f16x is not None else False
        self.step, self.T, self.exact, self.mode = step, T, exact, mode
        self.f16x = not exact
        ctx, s = step.ctx, step.shape
        dev = ctx.device
        shapes = layer_shapes(s)
        self.x_h = torch.from_numpy(synth.activations(T, s.hidden, synth.seed_for(4, 100))).to(dev)
        self.x_attn = torch.from_numpy(synth.activations(T, s.q, synth.seed_for(4, 101))).to(dev)
        f32 = dict(dtype=torch.float32, device=dev)
        self.out = {(layer, name): torch.empty((T, shapes[name][0]), **f32)
                    for layer in range(s.layers) for name in LAYER_MATS}
        self.act = [torch.empty((T, s.ffn), **f32) for _ in range(s.layers)]
        self.plan = None
        if T <= 16 or mode == "plan":
            p = Plan(ctx, batch=T, exact=exact)
            for layer in range(s.layers):
                for name in ("q", "k", "v", "o", "gate", "up"):
                    M, N = shapes[name]
                    x = self.x_attn if name == "o" else self.x_h
                    p.gemv(0, step.weights[(layer, name)], x, self.out[(layer, name)], M, N)
                p.gelu_mul(1, self.out[(layer, "gate")], self.out[(layer, "up")], self.act[layer])
                M, N = shapes["down"]
                p.gemv(1, step.weights[(layer, "down")], self.act[layer], self.out[(layer, "down")], M, N)
            p.commit()
            self.plan = p
        else:
            self.ctxs = [Context(dev) for _ in range(streams)]
            self.streams = [torch.cuda.Stream(device=dev) for _ in range(streams)]

    def launches(self) -> int:
        """Kernel launches per step."""
        if self.plan is not None:
            return self.plan.launches()
        shapes = layer_shapes(self.step.shape)
        return self.step.shape.layers * (2 * len(shapes) + 1)  # (prep + GEMM) per matrix + gelu_mul

    def _layer(self, c: Context, layer: int, stream) -> None:
        s, W, O = self.step.shape, self.step.weights, self.out
        shapes = layer_shapes(s)
        for name in ("q", "k", "v", "o", "gate", "up"):
            M, N = shapes[name]
            x = self.x_attn if name == "o" else self.x_h
            c.gemm(W[(layer, name)], x, M, N, out=O[(layer, name)], stream=stream, f16x=self.f16x)
        c.gelu_mul(O[(layer, "gate")], O[(layer, "up")], out=self.act[layer], stream=stream)
        M, N = shapes["down"]
        c.gemm(W[(layer, "down")], self.act[layer], M, N, out=O[(layer, "down")], stream=stream, f16x=self.f16x)

    def run(self, stream: torch.cuda.Stream | None = None) -> None:
        if self.plan is not None:
            self.plan.run(stream)
            return
        main = stream or torch.cuda.current_stream(self.step.ctx.device)
        fork = torch.cuda.Event()
        fork.record(main)
        joins = []
        for k, (c, st) in enumerate(zip(self.ctxs, self.streams)):
            st.wait_event(fork)
            for layer in range(k, self.step.shape.layers, len(self.streams)):
                self._layer(c, layer, st)
            e = torch.cuda.Event()
            e.record(st)
            joins.append(e)
        for e in joins:
            main.wait_event(e)

    def close(self) -> None:
        if self.plan is not None:
            self.plan.close()
            self.plan = None
        for c in getattr(self, "ctxs", []):
            c.close()
        self.ctxs = []

    def weights(self) -> int:
        """Weights one step multiplies (each by all T rows)."""
        return self.step.shape.layers * sum(M * N for M, N in layer_shapes(self.step.shape).values())

    def flops(self) -> int:
        return 2 * self.T * self.weights()


CHAIN_BUFFERS = ("q", "k", "v", "o", "g", "u", "act", "d", "h_attn", "h_out")


class ChainLayer(ctypes.Structure):
    """q4k_chain_layer of include/q4k.h: one layer's weights and outputs."""

    _fields_ = [(name, ctypes.c_void_p) for name in ("wq", "wk", "wv", "wo", "wg", "wu", "wd") + CHAIN_BUFFERS]


class ChainedStep:
    """Config 3 as a true dependency chain: layer l+1 reads layer l's output,
    the way encodeTransformerPass runs (src/engine.ts:1538-1619), with the
    reference's norms, residual adds, v norm and position-0 attention between
    the GEMVs (all norm weights 1; see q4k_chain_create in include/q4k.h),
    then final.rmsNorm and the fused LM head.  One persistent launch for all
    layers plus the LM head launch.  Uses the seeded weights of `step`
    (the same matrices as the sweep); h_in = the step's x_h row 0."""

    def __init__(self, step: DecodeStep, layers: int | None = None, with_head: bool = True, eps: float = 1e-6):
        if step.batch != 1:
            raise ValueError("the chained step is one token (batch 1)")
        self.step = step
        ctx, s = step.ctx, step.shape
        self.ctx = ctx
        self.layers = layers or s.layers
        self.eps = eps
        dev = ctx.device
        f32 = dict(dtype=torch.float32, device=dev)
        sizes = {"q": s.q, "k": s.kv, "v": s.kv, "o": s.hidden, "g": s.ffn, "u": s.ffn, "act": s.ffn,
                 "d": s.hidden, "h_attn": s.hidden, "h_out": s.hidden}
        self.out = [{name: torch.empty(sizes[name], **f32) for name in CHAIN_BUFFERS} for _ in range(self.layers)]
        # inputs and results each in one buffer: one copy each way per token
        self.inputs = torch.empty(s.hidden, **f32)
        self.inputs.copy_(step.x_h[0])
        self.h_in = self.inputs
        self.normed = torch.empty(s.hidden, **f32)
        self.results = torch.empty(513, dtype=torch.int32, device=dev)
        self.sel = Selection(cand_val=self.results[:256].view(torch.float32), cand_idx=self.results[256:512],
                             argmax=self.results[512:], logits=None)
        arr = (ChainLayer * self.layers)()
        for layer in range(self.layers):
            W = {n: step.weights[(layer, n)] for n in LAYER_MATS}
            o = self.out[layer]
            arr[layer] = ChainLayer(W["q"].data_ptr(), W["k"].data_ptr(), W["v"].data_ptr(), W["o"].data_ptr(),
                                    W["gate"].data_ptr(), W["up"].data_ptr(), W["down"].data_ptr(),
                                    *[o[n].data_ptr() for n in CHAIN_BUFFERS])
        self._L = ctx._L
        h = ctypes.c_void_p()
        ctx._check(self._L.q4k_chain_create(ctx._h, self.layers, s.hidden, s.q, s.kv, s.ffn, eps,
                                            ctypes.cast(arr, ctypes.c_void_p), self.h_in.data_ptr(),
                                            self.normed.data_ptr(), ctypes.byref(h)))
        self._h = h.value
        self._arr = arr
        self.with_head = with_head
        if with_head:
            ctx._check(self._L.q4k_chain_lmhead(self._h, step.lm_head.data_ptr(), s.vocab, s.softcap,
                                                self.sel.cand_val.data_ptr(), self.sel.cand_idx.data_ptr(),
                                                self.sel.argmax.data_ptr()))

    def run(self, stream: torch.cuda.Stream | None = None) -> None:
        st = stream if stream is not None else torch.cuda.current_stream(self.ctx.device)
        self.ctx._check(self._L.q4k_chain_run(self._h, st.cuda_stream))

    def launches(self) -> int:
        return self._L.q4k_chain_launches(self._h)

    def result_tensors(self) -> list[torch.Tensor]:
        return [self.results]

    def weight_bytes(self) -> int:
        s = self.step.shape
        per_layer = sum(synth.q4k_bytes(M, N) for M, N in layer_shapes(s).values())
        return self.layers * per_layer + (synth.q4k_bytes(s.vocab, s.hidden) if self.with_head else 0)

    def close(self) -> None:
        if getattr(self, "_h", None):
            self._L.q4k_chain_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
