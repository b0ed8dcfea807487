"""Small, self-contained launches of one libq4k kernel, for profiler captures.

    python gemma4-webgpu_b200/q4k/profile_case.py gemv [--batch B] [--reps R]
    python gemma4-webgpu_b200/q4k/profile_case.py lmhead [--reps R]
    python gemma4-webgpu_b200/q4k/profile_case.py sweep [--layers L] [--reps R]
    python gemma4-webgpu_b200/q4k/profile_case.py gemm [--batch T] [--reps R] [--f16x]
    python gemma4-webgpu_b200/q4k/profile_case.py q6head [--reps R]
    python gemma4-webgpu_b200/q4k/profile_case.py ple [--batch T] [--reps R]
    python gemma4-webgpu_b200/q4k/profile_case.py downs [--reps R]

`gemv` rotates over 35 distinct 6144x1536 Q4_K matrices (186 MB, more than
the 126 MB L2, so each launch reads its weights from HBM); `lmhead` runs the
fused 262144-row LM head (226 MB); `sweep` runs the decode-step plan of
q4k.decode with L layers (default 8: 159 MB of layer weights plus a
16384-row LM head); `gemm` runs q4k_gemm on one 6144x1536 matrix with T
activation rows (default 512); `q6head` runs the fused LM head on a
131072 x 1536 Q6_K matrix in the device layout (165 MB); `ple` runs the
per-layer-embedding stage 1 for T tokens (default 1) on a 262144 x 35
super-block Q5_K table (1.6 GB, made on the device), each rep a new
random token; `downs` runs the decode step's second plan stage alone
(gelu_mul + the 35 down projections 1536 x 6144, 186 MB, 4 warps per tile).  A few hundred MB of device memory at most;
the process exits after `reps` runs.
"""
from __future__ import annotations

import argparse
import sys
from pathlib import Path

sys.path.insert(0, str(Path(__file__).resolve().parents[1]))

import torch  # noqa: E402

from q4k import Context, synth  # noqa: E402


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("kernel", choices=["gemv", "lmhead", "sweep", "gemm", "q6head", "ple", "downs"])
    ap.add_argument("--layers", type=int, default=8)
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--reps", type=int, default=40)
    ap.add_argument("--f16x", action="store_true", help="gemm: activations rounded to f16 (q4k_gemm_f16x)")
    a = ap.parse_args()
    dev = torch.device("cuda", 0)
    ctx = Context(0)
    if a.kernel == "gemv":
        M, N = 6144, 1536
        ws = [torch.from_numpy(synth.q4k_matrix(M, N, synth.seed_for(3, 8 * i + 4))).to(dev) for i in range(35)]
        x = torch.from_numpy(synth.activations(a.batch, N, 1)).to(dev)
        y = torch.empty((a.batch, M), dtype=torch.float32, device=dev)
        for r in range(a.reps):
            ctx.gemv(ws[r % len(ws)], x, M, N, out=y)
    elif a.kernel == "gemm":
        M, N = 6144, 1536
        w = torch.from_numpy(synth.q4k_matrix(M, N, synth.seed_for(4, 1))).to(dev)
        T = a.batch if a.batch > 1 else 512
        x = torch.from_numpy(synth.activations(T, N, 2)).to(dev)
        y = torch.empty((T, M), dtype=torch.float32, device=dev)
        for _ in range(a.reps):
            ctx.gemm(w, x, M, N, out=y, f16x=a.f16x)
    elif a.kernel == "sweep":
        from q4k.decode import DecodeStep, E2BShape

        step = DecodeStep(ctx, E2BShape(layers=a.layers, vocab=16384), batch=a.batch)
        for _ in range(a.reps):
            step.run()
    elif a.kernel == "downs":
        from q4k.decode import DecodeStep, E2BShape

        step = DecodeStep(ctx, E2BShape(vocab=256), batch=1)
        step.run()  # gate/up outputs for the stage below
        p = step.plan(stages=(1,))
        for _ in range(a.reps):
            p.run()
    elif a.kernel == "ple":
        vocab, layers, T = 262144, 35, a.batch
        gen = torch.Generator(device=dev).manual_seed(7)
        table = torch.randint(0, 256, (vocab * layers, 176), dtype=torch.uint8, device=dev, generator=gen)
        table[:, 0:4] = torch.empty((vocab * layers, 2), dtype=torch.float16, device=dev).uniform_(
            0.0, 4e-3, generator=gen).view(torch.uint8)
        proj = torch.randn((T, layers * 256), device=dev, generator=gen)
        norm = torch.ones(256, dtype=torch.float16, device=dev).view(torch.int16)
        for _ in range(a.reps):
            tok = torch.randint(0, vocab, (T,), dtype=torch.int32, device=dev, generator=gen)
            ctx.ple_stage1(table, tok, vocab, layers, proj, norm)
    elif a.kernel == "q6head":
        V, N = 131072, 1536
        w = ctx.q6k_repack(torch.from_numpy(synth.q6k_matrix(V, N, synth.seed_for(5, 999)).reshape(-1)).to(dev),
                           V, N)
        x = torch.from_numpy(synth.activations(1, N, 1)).to(dev)
        for _ in range(a.reps):
            ctx.q6k_lmhead_select(w, x[0], V, N, 30.0)
    else:
        V, N = 262144, 1536
        w = torch.from_numpy(synth.q4k_matrix(V, N, synth.seed_for(3, 999))).to(dev)
        x = torch.from_numpy(synth.activations(1, N, 1)).to(dev)
        for _ in range(a.reps):
            ctx.lmhead_select(w, x[0], V, N, 30.0)
    torch.cuda.synchronize()
    ctx.close()
    print("done")


if __name__ == "__main__":
    main()
