"""The matmul call sites of one decode step of the real Gemma-4-E2B shapes,
with a Q4_K_M-style mix of Q4_K and Q6_K matrices.

The benchmark's config 3 (q4k/decode.py) simplifies the model to 35 equal
layers.  The real model (src/config/gemma4-e2b.ts:16-63, the dispatch list of
src/engine.ts:1520-1614 and the LM head of :1686-1741) differs:

  * full-attention layers 4, 9, 14, 19, 24, 29, 34 use head_dim 512 (q is
    4096 x 1536, k/v 512 x 1536, o 1536 x 4096); sliding layers head_dim 256;
  * only the 15 KV-producer layers (0-14) run k and v (consumers reuse the
    cache, src/engine.ts:1545-1553);
  * the FFN width is 6144 in layers 0-14 and 12288 in layers 15-34;
  * every layer runs the two per-layer-embedding GEMVs, inp_gate 256 x 1536
    and post_proj 1536 x 256 (src/engine.ts:1612-1614), and the step starts
    with the global per-layer projection 8960 x 1536 (:1520-1525);
  * the LM head is the tied 262144 x 1536 token embedding;
  * per token, the per-layer embeddings of the current token (a Q5_K table
    [262144, 35*256]) are gathered and fused with the normalised projection
    (ple_stage1_fuse, src/engine.ts:1528-1535).

A Q4_K_M file stores most matrices as Q4_K and some as Q6_K
(docs/findings/why-q4km.md:33).  The mix used here follows the usual
Q4_K_M recipe: the LM head, and v and down in "more bits" layers (layer i
of n with i < n/8, i >= 7n/8 or (i - n/8) % 3 == 2; n = 15 layers with a v
matrix, 35 with a down matrix), are Q6_K; everything else Q4_K.  Weights
are seeded synthetic super-blocks (q4k/synth.py); activations are fixed
seeded vectors, and as in config 3 only the matmul path runs: the layers do
not feed one another, and the step is two plan stages (every GEMV reading
the hidden state / attention output / PLE input plus the fused LM head; then
gelu_mul + down), each split into one launch per weight format.
"""
from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np
import torch

from . import synth
from .ops import Context, Plan, Selection

CONFIG = 5  # seeds: synth.seed_for(5, matrix_id)
FULL_ATTENTION = (4, 9, 14, 19, 24, 29, 34)
FMT_Q4K, FMT_Q6K = "q4k", "q6k"


@dataclass(frozen=True)
class RealE2B:
    layers: int = 35
    hidden: int = 1536
    heads: int = 8
    kv_heads: int = 1
    head_dim_local: int = 256
    head_dim_global: int = 512
    producers: int = 15
    ffn_producer: int = 6144
    ffn_consumer: int = 12288
    ple_dim: int = 256
    vocab: int = 262144
    softcap: float = 30.0


def more_bits(i: int, n: int) -> bool:
    return i < n // 8 or i >= 7 * n // 8 or (i - n // 8) % 3 == 2


def layer_matrices(s: RealE2B, layer: int) -> dict[str, tuple[int, int, str, str]]:
    """name -> (M rows, N cols, format, input) of every GEMV of `layer`.
    Inputs: "h" hidden state, "attn" attention output, "p" PLE activation,
    "act" gelu_mul(gate, up)."""
    hd = s.head_dim_global if layer in FULL_ATTENTION else s.head_dim_local
    q, kv = s.heads * hd, s.kv_heads * hd
    ffn = s.ffn_producer if layer < s.producers else s.ffn_consumer
    mats = {"q": (q, s.hidden, FMT_Q4K, "h")}
    if layer < s.producers:
        mats["k"] = (kv, s.hidden, FMT_Q4K, "h")
        mats["v"] = (kv, s.hidden, FMT_Q6K if more_bits(layer, s.producers) else FMT_Q4K, "h")
    mats["o"] = (s.hidden, q, FMT_Q4K, "attn")
    mats["gate"] = (ffn, s.hidden, FMT_Q4K, "h")
    mats["up"] = (ffn, s.hidden, FMT_Q4K, "h")
    mats["down"] = (s.hidden, ffn, FMT_Q6K if more_bits(layer, s.layers) else FMT_Q4K, "act")
    mats["ple_gate"] = (s.ple_dim, s.hidden, FMT_Q4K, "h")
    mats["ple_proj"] = (s.hidden, s.ple_dim, FMT_Q4K, "p")
    return mats


MAT_IDS = ("q", "k", "v", "o", "gate", "up", "down", "ple_gate", "ple_proj")


def matrix_bytes(M: int, N: int, fmt: str) -> int:
    return synth.q6k_bytes(M, N) if fmt == FMT_Q6K else synth.q4k_bytes(M, N)


def matrix_host(M: int, N: int, fmt: str, seed: int) -> np.ndarray:
    return synth.q6k_matrix(M, N, seed) if fmt == FMT_Q6K else synth.q4k_matrix(M, N, seed)


@dataclass
class RealE2BStep:
    """Device-resident weights (Q6_K ones in the device layout), activations
    and outputs of the real-shape step; `layers` selects a subset (tests)."""

    ctx: Context
    shape: RealE2B = field(default_factory=RealE2B)
    layers: tuple[int, ...] | None = None
    with_lm_head: bool = True
    with_ple_table: bool = True

    def __post_init__(self):
        s, dev = self.shape, self.ctx.device
        self.layer_ids = tuple(range(s.layers)) if self.layers is None else tuple(self.layers)
        self.mats = {(i, n): spec for i in self.layer_ids for n, spec in layer_matrices(s, i).items()}
        self.weights: dict = {}
        for (i, name), (M, N, fmt, _) in self.mats.items():
            self.weights[(i, name)] = self._upload(M, N, fmt, synth.seed_for(CONFIG, 16 * i + MAT_IDS.index(name)))
        ple_out = s.layers * s.ple_dim
        self.ple_global = self._upload(ple_out, s.hidden, FMT_Q4K, synth.seed_for(CONFIG, 900))
        self.lm_head = (self._upload(s.vocab, s.hidden, FMT_Q6K, synth.seed_for(CONFIG, 999))
                        if self.with_lm_head else None)
        f32 = dict(dtype=torch.float32, device=dev)
        q_max = s.heads * s.head_dim_global
        self.x = {
            "h": torch.from_numpy(synth.activations(1, s.hidden, synth.seed_for(CONFIG, 100))[0]).to(dev),
            "p": torch.from_numpy(synth.activations(1, s.ple_dim, synth.seed_for(CONFIG, 102))[0]).to(dev),
        }
        attn = torch.from_numpy(synth.activations(1, q_max, synth.seed_for(CONFIG, 101))[0]).to(dev)
        self.x_attn = {hd: attn[: s.heads * hd] for hd in (s.head_dim_local, s.head_dim_global)}
        self.out = {k: torch.empty(M, **f32) for k, (M, _, _, _) in self.mats.items()}
        self.act = {i: torch.empty(self.mats[(i, "gate")][0], **f32) for i in self.layer_ids}
        self.ple_out = torch.empty(ple_out, **f32)
        self.ple_table = self._ple_table() if self.with_ple_table else None
        gen = torch.Generator(device="cpu").manual_seed(synth.seed_for(CONFIG, 903))
        self.ple_norm = torch.empty(s.ple_dim, dtype=torch.float16).uniform_(0.5, 1.5, generator=gen).view(
            torch.int16).to(dev)
        self.ple_inputs = torch.empty(ple_out, **f32)
        self.sel = Selection(cand_val=torch.empty(256, **f32),
                             cand_idx=torch.empty(256, dtype=torch.int32, device=dev),
                             argmax=torch.empty(1, dtype=torch.int32, device=dev), logits=None)
        self._plan: Plan | None = None

    def _ple_table(self) -> torch.Tensor:
        """The Q5_K per-layer embedding table [vocab, layers*176 bytes], made
        on the device (1.6 GB): uniform bytes for the scales, qh and qs, and
        d, dmin ~ |U(0, 4e-3)| as f16 in every super-block."""
        s, dev = self.shape, self.ctx.device
        nb = s.vocab * s.layers
        gen = torch.Generator(device=dev).manual_seed(synth.seed_for(CONFIG, 902))
        t = torch.randint(0, 256, (nb, synth.Q5K_BLOCK_BYTES), dtype=torch.uint8, device=dev, generator=gen)
        dd = torch.empty((nb, 2), dtype=torch.float16, device=dev).uniform_(0.0, 4e-3, generator=gen)
        t[:, 0:4] = dd.view(torch.uint8)
        return t.reshape(s.vocab, s.layers * synth.Q5K_BLOCK_BYTES)

    def ple_stage1(self, stream: torch.cuda.Stream | None = None) -> None:
        """Per-layer embedding stage 1 of the current token: the token id is
        the LM head's last argmax, read on the device."""
        s = self.shape
        self.ctx.ple_stage1(self.ple_table, self.sel.argmax, s.vocab, s.layers, self.ple_out, self.ple_norm,
                            1e-6, out=self.ple_inputs, stream=stream)

    def _upload(self, M: int, N: int, fmt: str, seed: int) -> torch.Tensor:
        w = torch.from_numpy(matrix_host(M, N, fmt, seed)).to(self.ctx.device)
        return self.ctx.q6k_repack(w.reshape(-1), M, N) if fmt == FMT_Q6K else w

    def _input(self, layer: int, name: str) -> torch.Tensor:
        src = self.mats[(layer, name)][3]
        if src == "attn":
            return self.x_attn[self.mats[(layer, name)][1] // self.shape.heads]
        if src == "act":
            return self.act[layer]
        return self.x[src]

    def weight_bytes(self) -> dict[str, int]:
        """GGUF bytes of the step's weights by format."""
        s = self.shape
        out = {FMT_Q4K: synth.q4k_bytes(s.layers * s.ple_dim, s.hidden), FMT_Q6K: 0}
        for (M, N, fmt, _) in self.mats.values():
            out[fmt] += matrix_bytes(M, N, fmt)
        if self.with_lm_head:
            out[FMT_Q6K] += synth.q6k_bytes(s.vocab, s.hidden)
        return out

    def algorithmic_bytes(self) -> int:
        """Weights (GGUF size), every GEMV's f32 input and output, gelu_mul
        operands, the LM head's input and candidates."""
        s = self.shape
        total = sum(self.weight_bytes().values())
        for (M, N, _, _) in self.mats.values():
            total += 4 * (M + N)
        total += 4 * (s.layers * s.ple_dim + s.hidden)
        for i in self.layer_ids:
            total += 3 * 4 * self.mats[(i, "gate")][0]
        if self.with_lm_head:
            total += 4 * s.hidden + 256 * 8 + 4
        if self.ple_table is not None:
            # one token's 35 Q5_K super-blocks, the projection in, the PLE inputs out, the norm weight
            total += s.layers * synth.Q5K_BLOCK_BYTES + 2 * 4 * s.layers * s.ple_dim + 2 * s.ple_dim
        return total

    def plan(self) -> Plan:
        if self._plan is not None:
            return self._plan
        s = self.shape
        p = Plan(self.ctx, batch=1)
        p.gemv(0, self.ple_global, self.x["h"], self.ple_out, s.layers * s.ple_dim, s.hidden)
        for (i, name), (M, N, fmt, _) in self.mats.items():
            if name == "down":
                continue
            (p.gemv_q6k if fmt == FMT_Q6K else p.gemv)(0, self.weights[(i, name)], self._input(i, name),
                                                       self.out[(i, name)], M, N)
        if self.with_lm_head:
            p.lmhead_q6k(0, self.lm_head, self.x["h"], s.vocab, s.hidden, s.softcap, self.sel)
        for i in self.layer_ids:
            p.gelu_mul(1, self.out[(i, "gate")], self.out[(i, "up")], self.act[i])
            M, N, fmt, _ = self.mats[(i, "down")]
            (p.gemv_q6k if fmt == FMT_Q6K else p.gemv)(1, self.weights[(i, "down")], self.act[i],
                                                       self.out[(i, "down")], M, N)
        p.commit()
        self._plan = p
        return p

    def run(self, stream: torch.cuda.Stream | None = None) -> None:
        """The step's plan, then the per-layer embedding stage 1 of the token
        the LM head just chose (the reference runs it at the start of the next
        forward, right after the projection GEMV; the work is the same)."""
        self.plan().run(stream)
        if self.ple_table is not None and self.with_lm_head:
            self.ple_stage1(stream)

    def run_serial(self, stream: torch.cuda.Stream | None = None) -> None:
        """One libq4k call per reference dispatch, in encodeTransformerPass order."""
        c, s = self.ctx, self.shape
        c.gemv(self.ple_global, self.x["h"], s.layers * s.ple_dim, s.hidden, out=self.ple_out, stream=stream)
        order = ("q", "k", "v", "o", "gate", "up", "down", "ple_gate", "ple_proj")
        for i in self.layer_ids:
            for name in order:
                if (i, name) not in self.mats:
                    continue
                if name == "down":
                    c.gelu_mul(self.out[(i, "gate")], self.out[(i, "up")], out=self.act[i], stream=stream)
                M, N, fmt, _ = self.mats[(i, name)]
                fn = c.q6k_gemv if fmt == FMT_Q6K else c.gemv
                fn(self.weights[(i, name)], self._input(i, name), M, N, out=self.out[(i, name)], stream=stream)
        if self.with_lm_head:
            c.q6k_lmhead_select(self.lm_head, self.x["h"], s.vocab, s.hidden, s.softcap, out=self.sel,
                                stream=stream)
            if self.ple_table is not None:
                self.ple_stage1(stream)

    def result_tensors(self) -> list[torch.Tensor]:
        return [self.sel.argmax, self.sel.cand_val, self.sel.cand_idx]
