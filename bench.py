#!/usr/bin/env python
"""Benchmark of the Q4_K matmul path on B200 (one JSON line on rank 0).

Workload (M=1): one synthetic Gemma-4-E2B-shaped decode
step's matmul path -- 35 layers x {q, k, v, o, gate, up, down} Q4_K GEMVs +
gelu_mul + the fused 262144-row LM head (softcap, argmax, topk256) -- captured
as a CUDA graph and replayed once per step.  923 MB of Q4_K weights per step,
more than the 126 MB L2, so every step streams the weights from HBM.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--batch B] [--impl ours|reference]
    python bench.py --case {gemv,lmhead,sweep,gemm,q6head,ple,downs} [--reps R] ...   (profiler cases)

N > 1 (torchrun, one rank per GPU): every rank runs its own replica of the
step (independent sequences, no collective on the data path: the M=1 sweep
does not shard); value = bytes all ranks moved / max-over-ranks time.  At
N > 1 the line also carries kernels.lmhead_sharded: config 2's LM head split
by vocabulary rows over the N ranks (q4k.sharded), timed as the max over
ranks, and whether its merged candidates equal the unsharded head's.

--impl reference times the CPU restatement of the reference's algorithm
(oracle/, the reference itself is TypeScript + WGSL and cannot run here) on
the host cores, on a bounded sample of the same workload per step.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import time
from datetime import timedelta
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "gemma4-webgpu_b200"))

METRIC = "Q4_K GEMV achieved HBM GB/s vs ~8 TB/s; synthetic E2B decode tokens/s"
UNIT = "GB/s"
PROFILE_TRAFFIC = ROOT / "profiles" / "traffic.txt"


def peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"],
                "bf16_tflops_sustained": d.get("bf16_tflops_sustained", d["bf16_tflops"]), "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}


# ---- clocks ---------------------------------------------------------------------

class ClockSampler:
    """SM clocks and throttle reasons sampled during the timed region: NVML
    polled from a thread every 5 ms (nvidia-smi as a fallback)."""

    REASONS = {  # nvmlClocksEventReason bits
        0x8: "hw_slowdown",
        0x40: "hw_thermal_slowdown",
        0x20: "sw_thermal_slowdown",
        0x4: "sw_power_cap",
    }

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.samples: list[tuple[float, int]] = []
        self.max_mhz = None
        self._stop = None
        self._thread = None
        self._error = None

    def start(self):
        import threading

        try:
            import pynvml

            pynvml.nvmlInit()
            h = pynvml.nvmlDeviceGetHandleByIndex(self.gpu)
            self.max_mhz = float(pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM))
        except Exception as e:  # no NVML: report it
            self._error = f"nvml unavailable: {e}"
            return
        self._stop = threading.Event()

        def loop():
            while not self._stop.is_set():
                try:
                    mhz = float(pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM))
                    reasons = int(pynvml.nvmlDeviceGetCurrentClocksEventReasons(h))
                    self.samples.append((mhz, reasons))
                except Exception as e:
                    self._error = str(e)
                    return
                self._stop.wait(0.005)

        self._thread = threading.Thread(target=loop, daemon=True)
        self._thread.start()

    def stop(self) -> dict:
        if self._thread is not None:
            self._stop.set()
            self._thread.join(timeout=2)
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": [self._error or "no samples"],
                    "samples": 0}
        seen = set()
        for _, r in self.samples:
            for bit, name in self.REASONS.items():
                if r & bit:
                    seen.add(name)
        return {"sm_mhz": statistics.median(m for m, _ in self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(seen), "samples": len(self.samples)}


# ---- distributed plumbing ----------------------------------------------------------

def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def init_dist(world: int, local: int, backend: str = "nccl"):
    import torch
    import torch.distributed as dist

    if world > 1 and not dist.is_initialized():
        if backend == "nccl":
            torch.cuda.set_device(local)
        dist.init_process_group(backend, timeout=timedelta(seconds=300))


def max_over_ranks(v: float, world: int, device) -> float:
    if world == 1:
        return v
    import torch
    import torch.distributed as dist

    t = torch.tensor([v], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(world: int):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


# ---- CPU baseline (oracle port) -----------------------------------------------------

def cpu_sample_rate(mats, target_s: float, threads: int, variant: str = "fused"):
    """Time the oracle on the sample matrices, repeating until target_s.
    variant "fused": the Q4_K GEMV with the decode in every call (Q4_K decode
    + RNE f16 + WGSL-order f32 dot); "f16": the reference's per-token work,
    the matmul_quant GEMV over weights dequantized to f16 beforehand (the
    reference decodes once at load, src/gguf.ts:157-210, 425-473, and its
    shaders/matmul_quant.wgsl:21-54 reads the f16 buffer; the decode is not
    timed).  Returns (GB/s of the sample's algorithmic bytes -- Q4_K weight
    bytes + f32 I/O, the unit of the GPU figure --, seconds, bytes, passes)."""
    sys.path.insert(0, str(ROOT / "oracle"))
    import numpy as np
    import oracle as O

    xs = {}
    total_bytes = 0
    for w, M, N in mats:
        if N not in xs:
            xs[N] = np.random.default_rng(N).standard_normal((1, N), dtype=np.float32)
        total_bytes += w.nbytes + 4 * (M + N)
    if variant == "f16":
        w16 = [O.dequant_f16(w) for w, _, _ in mats]

        def one_pass():
            for (_, M, N), w in zip(mats, w16):
                O.matmul_quant_f16(w, xs[N], M, N, threads=threads)
    else:
        def one_pass():
            for w, M, N in mats:
                O.q4k_gemv(w, xs[N], M, N, threads=threads)
    passes, t0 = 0, time.perf_counter()
    while True:
        one_pass()
        passes += 1
        el = time.perf_counter() - t0
        if el >= target_s:
            break
    return passes * total_bytes / el / 1e9, el, total_bytes, passes


def cpu_baseline_variants(mats, seconds: float, bytes_step: int) -> dict:
    """The CPU restatement on the host cores in both forms (fused decode +
    GEMV, and the GEMV over pre-dequantized f16 weights) on 1 core and on all
    cores, seconds/4 each; GB/s of algorithmic bytes and the decode
    tokens/s each rate would give on the full step."""
    cores = os.cpu_count() or 1
    out = {}
    for variant in ("fused", "f16"):
        for threads in (1, cores):
            gbs, el, nbytes, passes = cpu_sample_rate(mats, seconds / 4, threads, variant)
            out[f"{variant}_{threads}core" + ("s" if threads > 1 else "")] = {
                "GB/s": round(gbs, 3), "cores": threads, "seconds": round(el, 2), "passes": passes,
                "tokens_per_s_equiv": round(gbs * 1e9 / bytes_step, 3)}
    return out


# ---- our arm ------------------------------------------------------------------------------

def run_ours(args) -> None:
    import torch

    world, rank, local = dist_env()
    init_dist(world, local)
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)

    from q4k import Context
    from q4k.decode import DecodeStep, E2BShape, StepGraph

    ctx = Context(local)
    step = DecodeStep(ctx, E2BShape(), batch=args.batch)
    graph = StepGraph(step)
    s = graph.stream
    bytes_step = step.algorithmic_bytes()
    launches = step.launches_per_step()

    # warm-up, then K timed replays bracketed by barrier + synchronize
    for _ in range(args.warmup):
        graph.replay()
    torch.cuda.synchronize()
    barrier(world)
    clocks = ClockSampler(local)
    clocks.start()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    barrier(world)
    torch.cuda.nvtx.range_push("timed")
    start.record(s)
    for _ in range(args.steps):
        graph.replay()
    end.record(s)
    torch.cuda.nvtx.range_pop()
    torch.cuda.synchronize()
    barrier(world)
    ms_local = start.elapsed_time(end)
    clk = clocks.stop()
    ms = max_over_ranks(ms_local, world, dev)
    ms_per_step = ms / args.steps
    value = world * bytes_step * args.steps / (ms / 1e3) / 1e9
    tokens_per_s = world * args.batch * args.steps / (ms / 1e3)

    def time_body(body, reps):
        g = StepGraph(step, body=body)
        for _ in range(3):
            g.replay()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(g.stream)
        for _ in range(reps):
            g.replay()
        b.record(g.stream)
        torch.cuda.synchronize()
        return a.elapsed_time(b) / reps, g

    reps = min(max(5, args.steps), 200)
    # dominant kernel: the engine launch of stage 0 (every GEMV but down, and
    # the LM head), timed alone with its activation-prep launch in front
    stage0 = step.plan(stages=(0,))
    s0_ms, s0_graph = time_body(lambda st: stage0.run(st), reps)
    s0_bytes = step.stage0_bytes()
    s0_gbs = s0_bytes / (s0_ms / 1e3) / 1e9
    # the second launch: gelu_mul + the 35 down projections (4 warps per tile)
    stage1 = step.plan(stages=(1,))
    s1_ms, s1_graph = time_body(lambda st: stage1.run(st), reps)
    s1_gbs = step.stage1_bytes() / (s1_ms / 1e3) / 1e9
    del s1_graph
    # the same step as one libq4k call per reference dispatch (246 launches)
    serial_ms, serial_graph = time_body(step.run_serial, reps)
    # the LM head alone
    lm_ms = None
    if args.batch == 1:
        lm_ms, lm_graph = time_body(
            lambda st: ctx.lmhead_select(step.lm_head, step.x_h, 262144, 1536, 30.0, out=step.sel, stream=st), reps)
        del lm_graph
    lm_bytes = 226_492_416 + 4 * 1536 + 2052

    # config 3 at M = 4 (the MR4 kernel's shape): the same sweep for 4
    # activation rows per step, on the same resident weights
    sweep4 = None
    if args.batch == 1:
        step4 = DecodeStep(ctx, E2BShape(), batch=4, share_weights_with=step)
        s4_ms, s4_graph = time_body(step4.run, reps)
        s4_ms = max_over_ranks(s4_ms, world, dev)
        sweep4 = {"ms": round(s4_ms, 4), "tokens_per_s": round(world * 4 / (s4_ms / 1e3), 1),
                  "GB/s": round(step4.algorithmic_bytes() / (s4_ms / 1e3) / 1e9, 1),
                  "launches": step4.launches_per_step()}
        del s4_graph, step4

    # config 4: the layer weights at T activation rows per step (no LM head):
    # the GEMV engine for T <= 16, the tcgen05 GEMM for T >= 64
    batched = None
    if args.batch == 1 and not args.no_c4:
        from q4k.decode import BatchedSweep

        batched = {}
        bf16_peak = peaks()["bf16_tflops"]
        bf16_sus = peaks()["bf16_tflops_sustained"]
        # (T, exact, mode): T <= 16 runs on the GEMV engine; T >= 64 on the
        # tcgen05 GEMM, one launch per plan stage over all 210 / 35 matrices,
        # activations rounded once to f16 (the 2e-3 prefill tolerance) or, with
        # exact, split into f16 hi + lo (the GEMV tolerance); "streams" is the
        # earlier per-matrix form (18 streams of q4k_gemm calls), for comparison
        cases = ((4, True, "plan"), (16, True, "plan"), (64, False, "plan"), (512, False, "plan"),
                 (64, True, "plan"), (512, True, "plan"), (512, False, "streams"))
        for T, exact, mode in cases:
            bs = BatchedSweep(step, T, exact=exact, mode=mode)
            t_ms, t_graph = time_body(bs.run, max(5, min(reps, 2000 // T)))
            t_ms = max_over_ranks(t_ms, world, dev)  # each rank runs its own T rows (data parallel)
            tf = world * bs.flops() / (t_ms / 1e3) / 1e12
            if T <= 16:
                path, key = "GEMV engine plan, 2 launches", f"T={T}"
            else:
                form = "exact f16 hi+lo activations" if exact else "activations rounded to f16 (tolerance 2e-3)"
                if mode == "plan":
                    path = f"tcgen05 GEMM plan, one launch per stage ({bs.launches()} launches), {form}"
                    key = f"T={T}" + (" exact" if exact else " f16x")
                else:
                    path = f"tcgen05 GEMM per matrix over 18 streams ({bs.launches()} launches), {form}"
                    key = f"T={T}" + (" exact" if exact else " f16x") + " per-matrix"
            batched[key] = {
                "ms": round(t_ms, 4), "tokens_per_s": round(world * T / (t_ms / 1e3), 1), "TFLOP/s": round(tf, 2),
                "frac_of_bf16_peak": round(tf / (world * bf16_peak), 4),
                "frac_of_bf16_sustained": round(tf / (world * bf16_sus), 4), "path": path}
            del t_graph
            bs.close()

    # the real E2B shapes with a Q4_K_M-style Q4_K/Q6_K mix (q4k/e2b.py):
    # the same two-stage plan, one engine launch per format per stage
    real = None
    if args.batch == 1 and not args.no_real:
        from q4k.e2b import RealE2BStep

        rstep = RealE2BStep(ctx)
        r_ms, r_graph = time_body(rstep.run, reps)
        rs_ms, rs_graph = time_body(rstep.run_serial, reps)
        pl_ms, pl_graph = time_body(rstep.ple_stage1, reps)
        rl_ms, rl_graph = time_body(
            lambda st: ctx.q6k_lmhead_select(rstep.lm_head, rstep.x["h"], 262144, 1536, 30.0, out=rstep.sel,
                                             stream=st), reps)
        rb = rstep.algorithmic_bytes()
        wb = rstep.weight_bytes()
        q6_lm = 262144 * 6 * 210 + 4 * 1536 + 2052
        real = {"ms": round(r_ms, 4), "tokens_per_s": round(world / (r_ms / 1e3), 1),
                "GB/s": round(rb / (r_ms / 1e3) / 1e9, 1), "launches": rstep.plan().launches(),
                "weight_bytes": {"q4k": wb["q4k"], "q6k": wb["q6k"]}, "algorithmic_bytes": rb,
                "serial_ms": round(rs_ms, 4),
                "lmhead_q6k": {"ms": round(rl_ms, 4), "GB/s": round(q6_lm / (rl_ms / 1e3) / 1e9, 1)},
                "ple_stage1": {"us": round(pl_ms * 1e3, 2), "launches": 1,
                               "what": "35 Q5_K super-blocks of the argmax token gathered from the 1.6 GB "
                                       "table, decoded and fused with the normalised projection"}}
        del r_graph, rs_graph, rl_graph, pl_graph, rstep

    # config 2 at N > 1: the LM head split by vocabulary rows over the ranks,
    # one all-gather of 2 KB of candidates per rank, merged on every rank
    sharded = None
    if world > 1 and args.batch == 1:
        from q4k.sharded import ShardedLMHead

        head = ShardedLMHead(262144, 1536, 30.0, ctx=ctx)
        w_shard = step.lm_head[head.row0:head.row0 + head.rows]
        x0 = step.x_h[0]
        for _ in range(args.warmup):
            merged = head(w_shard, x0)
        torch.cuda.synchronize()
        step.plan().run()  # the unsharded head on the same input, for the check below
        torch.cuda.synchronize()
        same = bool(torch.equal(merged.cand_idx, step.sel.cand_idx) and torch.equal(merged.argmax, step.sel.argmax))
        barrier(world)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(reps):
            head(w_shard, x0)
        b.record()
        torch.cuda.synchronize()
        sh_ms = max_over_ranks(a.elapsed_time(b) / reps, world, dev)
        same = max_over_ranks(0.0 if same else 1.0, world, dev) == 0.0
        sh_gbs = lm_bytes / (sh_ms / 1e3) / 1e9
        sharded = {"ms": round(sh_ms, 4), "GB/s": round(sh_gbs, 1), "shards": world,
                   "rows_per_rank": head.rows, "frac_of_peak": None,
                   "collective": "all_gather 2 KB/rank (NCCL) + on-device merge",
                   "matches_unsharded": same}
        # the same head with the exchange fused into the launch (peer stores
        # over NVLink into every rank's mailbox, bounded wait, merge)
        fhead = ShardedLMHead(262144, 1536, 30.0, ctx=ctx, fused=True)
        for _ in range(args.warmup):
            fmerged = fhead(w_shard, x0)
        torch.cuda.synchronize()
        fsame = bool(torch.equal(fmerged.cand_idx, step.sel.cand_idx) and torch.equal(fmerged.argmax, step.sel.argmax))
        barrier(world)
        a.record()
        for _ in range(reps):
            fhead(w_shard, x0)
        b.record()
        torch.cuda.synchronize()
        fs_ms = max_over_ranks(a.elapsed_time(b) / reps, world, dev)
        fsame = max_over_ranks(0.0 if fsame else 1.0, world, dev) == 0.0
        barrier(world)
        fhead.close()
        sharded["fused_exchange"] = {"ms": round(fs_ms, 4), "GB/s": round(lm_bytes / (fs_ms / 1e3) / 1e9, 1),
                                     "launches_per_call": 1, "matches_unsharded": fsame}
        # where the fused head's time goes: the same shard's fused head
        # without any exchange (its GEMV + softcap + per-residue selection),
        # timed the same way; the rest is the candidate exchange (peer
        # stores, flag wait) and the merge
        barrier(world)
        a.record()
        for _ in range(reps):
            ctx.lmhead_select(w_shard, x0, head.rows, 1536, 30.0, row_offset=head.row0)
        b.record()
        torch.cuda.synchronize()
        shard_ms = max_over_ranks(a.elapsed_time(b) / reps, world, dev)
        barrier(world)
        shard_bytes = lm_bytes // world
        sharded["breakdown"] = {
            "shard_head_alone_ms": round(shard_ms, 4),
            "shard_head_alone_GB/s": round(shard_bytes / (shard_ms / 1e3) / 1e9, 1),
            "exchange_and_merge_ms": round(fs_ms - shard_ms, 4),
            "shard_bytes": shard_bytes,
            "what": "fused sharded head = this rank's shard head (GEMV + softcap + per-residue keys + last-CTA "
                    "merge) + peer stores of 2 KB to every rank + bounded flag wait + G-way merge"}

    # the step as a true dependency chain (layer l+1 reads layer l's output,
    # with the reference's norms between the GEMVs): one persistent launch for
    # the 35 layers + the LM head launch
    chained = None
    if args.batch == 1 and not args.no_chain:
        from q4k.decode import ChainedStep

        ch = ChainedStep(step)
        c_ms, c_graph = time_body(ch.run, reps)
        c_ms = max_over_ranks(c_ms, world, dev)
        ch_nohead = ChainedStep(step, with_head=False)
        cl_ms, cl_graph = time_body(ch_nohead.run, reps)
        cl_ms = max_over_ranks(cl_ms, world, dev)
        chained = {"ms": round(c_ms, 4), "tokens_per_s": round(world / (c_ms / 1e3), 1),
                   "GB/s": round(ch.weight_bytes() / (c_ms / 1e3) / 1e9, 1), "launches": ch.launches(),
                   "layers_only_ms": round(cl_ms, 4), "per_layer_us": round(cl_ms * 1e3 / ch.layers, 2),
                   "what": "35 layers chained (rms_norm -> q/k/v -> v norm + position-0 attention -> o -> "
                           "fused_norm_add -> rms_norm -> gate/up -> gelu_mul -> down -> fused_norm_add), "
                           "140 dependent stages in one cooperative launch, then final rms_norm + fused LM head"}
        del c_graph, cl_graph
        ch.close()
        ch_nohead.close()

    # end to end through the public API: pinned host inputs in, results out
    # the step's inputs (x_h | x_attn) and results (candidates | argmax) each
    # sit in one device buffer: one host->device and one device->host copy
    x_host = [torch.empty_like(step.inputs, device="cpu").pin_memory()]
    x_host[0].copy_(step.inputs)
    res = step.result_tensors()
    res_host = [torch.empty_like(t, device="cpu").pin_memory() for t in res]
    h2d = sum(t.numel() * t.element_size() for t in x_host)
    d2h = sum(t.numel() * t.element_size() for t in res_host)

    # one graph replay per token: input copy in, the step, result copy out
    io_graph = StepGraph(step, stream=s, host_io=(x_host[0], res_host[0]))

    def e2e_step():
        io_graph.replay()
        s.synchronize()

    for _ in range(args.warmup):
        e2e_step()
    barrier(world)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        e2e_step()
    e2e_s = max_over_ranks(time.perf_counter() - t0, world, dev)
    e2e_value = world * bytes_step * args.steps / e2e_s / 1e9

    pk = peaks()
    traffic = None
    if PROFILE_TRAFFIC.exists() and args.batch == 1:
        for line in PROFILE_TRAFFIC.read_text().splitlines():
            parts = line.split()
            if len(parts) == 2 and parts[0] == "stage0_engine":
                traffic = int(parts[1])
    roofline = {
        "kernel": "engine_kernel, plan stage 0 (210 GEMVs + fused LM head in one launch)",
        "bound": "hbm",
        "achieved": round(s0_gbs, 1),
        "peak": pk["hbm_gbs"],
        "peak_source": pk["source"],
        "unit": "GB/s",
        "frac": round(s0_gbs / pk["hbm_gbs"], 4),
        "traffic": traffic,
        "algorithmic_bytes_per_launch": s0_bytes,
        "avg_launch_us": round(s0_ms * 1e3, 2),
    }
    kernels = {"stage0_engine": {"ms": round(s0_ms, 4), "GB/s": round(s0_gbs, 1),
                                 "frac_of_peak": round(s0_gbs / pk["hbm_gbs"], 4)},
               "stage1_engine": {"ms": round(s1_ms, 4), "GB/s": round(s1_gbs, 1),
                                 "frac_of_peak": round(s1_gbs / pk["hbm_gbs"], 4)},
               "serial_step": {"ms": round(serial_ms, 4), "launches": step.serial_calls_per_step(),
                               "GB/s": round(bytes_step / (serial_ms / 1e3) / 1e9, 1),
                               "tokens_per_s": round(args.batch / (serial_ms / 1e3), 1)}}
    if lm_ms:
        kernels["lmhead_select"] = {"ms": round(lm_ms, 4), "GB/s": round(lm_bytes / (lm_ms / 1e3) / 1e9, 1),
                                    "frac_of_peak": round(lm_bytes / (lm_ms / 1e3) / 1e9 / pk["hbm_gbs"], 4)}
    if sweep4:
        kernels["sweep_batch4"] = sweep4
    if batched is not None:
        kernels["c4_batched"] = batched
    if real:
        real["lmhead_q6k"]["frac_of_peak"] = round(real["lmhead_q6k"]["GB/s"] / pk["hbm_gbs"], 4)
        kernels["e2b_real_q4km"] = real
    if chained:
        kernels["chained_step"] = chained
    if sharded:
        sharded["frac_of_peak"] = round(sharded["GB/s"] / (world * pk["hbm_gbs"]), 4)
        kernels["lmhead_sharded"] = sharded

    cpu = None
    if world == 1 and not args.no_cpu:
        mats = step.sample_matrices(layers=1)
        threads = os.cpu_count() or 1
        variants = cpu_baseline_variants(mats, args.cpu_seconds, bytes_step)
        head = variants[f"fused_{threads}core" + ("s" if threads > 1 else "")]
        nbytes = sum(w.nbytes + 4 * (M + N) for w, M, N in mats)
        cpu = {"value": head["GB/s"], "unit": UNIT, "cores": threads, "kind": "port",
               "sample": f"layer 0's 7 GEMVs ({nbytes / 1e6:.1f} MB of Q4_K+f32 I/O), repeated for "
                         f"{args.cpu_seconds / 4:.1f} s per variant; value = fused Q4_K decode + RNE f16 + "
                         f"WGSL-order f32 dot on all {threads} host threads",
               "tokens_per_s_equiv": head["tokens_per_s_equiv"],
               "variants": variants}

    line = {
        "metric": METRIC,
        "value": round(value, 1),
        "unit": UNIT,
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms_per_step, 4),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic (seeded Q4_K super-blocks + N(0,1) f32 activations)",
        "config": {
            "workload": f"c3 decode-step weight sweep, E2B-shaped, M={args.batch}",
            "layers": 35, "hidden": 1536, "q": 2048, "kv": 256, "ffn": 6144, "vocab": 262144,
            "batch": args.batch, "weight_bytes_per_step": step.weight_bytes(),
            "algorithmic_bytes_per_step": bytes_step,
            "l2": "inputs larger than L2 (923 MB of weights per step vs 126 MB L2)",
            "parallelism": f"replicas x{world}" if world > 1 else "single GPU",
            "step": f"plan: stage 0 = 210 GEMVs + fused LM head, stage 1 = 35 x gelu_mul->down; "
                    f"{step.plan().launches()} launches per step; CUDA graph replay",
        },
        "tokens_per_s": round(tokens_per_s, 1),
        "roofline": roofline,
        "kernels": kernels,
        "cpu_baseline": cpu,
        "e2e": {"value": round(e2e_value, 1), "unit": UNIT, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "tokens_per_s": round(world * args.batch * args.steps / e2e_s, 1)},
        "gpu_launches": launches * args.steps,
        "clocks": clk,
    }
    if rank == 0:
        print(json.dumps(line), flush=True)
    del graph, io_graph, s0_graph, serial_graph
    ctx.close()
    if world > 1:
        import torch.distributed as dist

        dist.destroy_process_group()


# ---- profiler cases ---------------------------------------------------------------------------

CASES = ("gemv", "lmhead", "sweep", "gemm", "q6head", "ple", "downs", "gemmplan", "chain")


def run_case(args) -> None:
    """Small, self-contained launches of one kernel for profiler captures
    (`--case`), a few hundred MB of device memory at most; the process exits
    after `--reps` runs and prints nothing that is a bench value.

      gemv    rotates over 35 distinct 6144x1536 Q4_K matrices (186 MB, more than
              the 126 MB L2, so each launch reads its weights from HBM), --batch rows
      lmhead  the fused 262144-row LM head (226 MB)
      sweep   the decode-step plan of q4k.decode with --layers layers (default 8:
              159 MB of layer weights plus a 16384-row LM head), --batch rows
      gemm    q4k_gemm on one 6144x1536 matrix with --batch activation rows
              (default 512; --f16x: q4k_gemm_f16x)
      q6head  the fused LM head on a 131072x1536 Q6_K matrix in the device layout
      ple     per-layer-embedding stage 1 for --batch tokens on a 262144 x 35
              super-block Q5_K table (1.6 GB, made on the device), a new random
              token each rep
      downs   the decode step's second plan stage alone (gelu_mul + the 35 down
              projections 1536x6144, 186 MB, 4 warps per tile)
      gemmplan  config 4's GEMM plan on --layers layers (default 8: 159 MB) at --batch
              activation rows (default 512), f16 activations (--exact: hi + lo)
      chain   the chained decode step over --layers layers (default 8), no LM head
    """
    import torch

    from q4k import Context, synth

    dev = torch.device("cuda", 0)
    ctx = Context(0)
    if args.case == "gemv":
        M, N = 6144, 1536
        ws = [torch.from_numpy(synth.q4k_matrix(M, N, synth.seed_for(3, 8 * i + 4))).to(dev) for i in range(35)]
        x = torch.from_numpy(synth.activations(args.batch, N, 1)).to(dev)
        y = torch.empty((args.batch, M), dtype=torch.float32, device=dev)
        for r in range(args.reps):
            ctx.gemv(ws[r % len(ws)], x, M, N, out=y)
    elif args.case == "gemm":
        M, N = 6144, 1536
        w = torch.from_numpy(synth.q4k_matrix(M, N, synth.seed_for(4, 1))).to(dev)
        T = args.batch if args.batch > 1 else 512
        x = torch.from_numpy(synth.activations(T, N, 2)).to(dev)
        y = torch.empty((T, M), dtype=torch.float32, device=dev)
        for _ in range(args.reps):
            ctx.gemm(w, x, M, N, out=y, f16x=args.f16x)
    elif args.case == "sweep":
        from q4k.decode import DecodeStep, E2BShape

        step = DecodeStep(ctx, E2BShape(layers=args.layers, vocab=16384), batch=args.batch)
        for _ in range(args.reps):
            step.run()
    elif args.case == "gemmplan":
        from q4k.decode import BatchedSweep, DecodeStep, E2BShape

        step = DecodeStep(ctx, E2BShape(layers=args.layers, vocab=256), batch=1)
        bs = BatchedSweep(step, args.batch if args.batch > 1 else 512, exact=args.exact)
        for _ in range(args.reps):
            bs.run()
        torch.cuda.synchronize()
        bs.close()
    elif args.case == "chain":
        from q4k.decode import ChainedStep, DecodeStep, E2BShape

        step = DecodeStep(ctx, E2BShape(layers=args.layers, vocab=256), batch=1)
        ch = ChainedStep(step, with_head=False)
        for _ in range(args.reps):
            ch.run()
        torch.cuda.synchronize()
        ch.close()
    elif args.case == "downs":
        from q4k.decode import DecodeStep, E2BShape

        step = DecodeStep(ctx, E2BShape(vocab=256), batch=1)
        step.run()  # gate/up outputs for the stage below
        p = step.plan(stages=(1,))
        for _ in range(args.reps):
            p.run()
    elif args.case == "ple":
        vocab, layers, T = 262144, 35, args.batch
        gen = torch.Generator(device=dev).manual_seed(7)
        table = torch.randint(0, 256, (vocab * layers, 176), dtype=torch.uint8, device=dev, generator=gen)
        table[:, 0:4] = torch.empty((vocab * layers, 2), dtype=torch.float16, device=dev).uniform_(
            0.0, 4e-3, generator=gen).view(torch.uint8)
        proj = torch.randn((T, layers * 256), device=dev, generator=gen)
        norm = torch.ones(256, dtype=torch.float16, device=dev).view(torch.int16)
        for _ in range(args.reps):
            tok = torch.randint(0, vocab, (T,), dtype=torch.int32, device=dev, generator=gen)
            ctx.ple_stage1(table, tok, vocab, layers, proj, norm)
    elif args.case == "q6head":
        V, N = 131072, 1536
        w = ctx.q6k_repack(torch.from_numpy(synth.q6k_matrix(V, N, synth.seed_for(5, 999)).reshape(-1)).to(dev),
                           V, N)
        x = torch.from_numpy(synth.activations(1, N, 1)).to(dev)
        for _ in range(args.reps):
            ctx.q6k_lmhead_select(w, x[0], V, N, 30.0)
    else:  # lmhead
        V, N = 262144, 1536
        w = torch.from_numpy(synth.q4k_matrix(V, N, synth.seed_for(3, 999))).to(dev)
        x = torch.from_numpy(synth.activations(1, N, 1)).to(dev)
        for _ in range(args.reps):
            ctx.lmhead_select(w, x[0], V, N, 30.0)
    torch.cuda.synchronize()
    ctx.check()
    ctx.close()
    print(f"case {args.case} done", flush=True)


# ---- reference arm --------------------------------------------------------------------------

def run_reference(args) -> None:
    world, rank, _ = dist_env()
    if rank != 0:
        return
    sys.path.insert(0, str(ROOT / "oracle"))
    from q4k.decode import DecodeStep  # noqa: F401  (shapes / seeds only; no GPU used)
    from q4k import synth
    from q4k.decode import E2BShape, layer_shapes, matrix_seed

    shape = E2BShape()
    mats = []
    for name, (M, N) in layer_shapes(shape).items():
        mats.append((synth.q4k_matrix(M, N, matrix_seed(0, name)), M, N))
    per_layer = sum(synth.q4k_bytes(M, N) + 4 * args.batch * (M + N) for M, N in layer_shapes(shape).values())
    bytes_step_full = shape.layers * per_layer + synth.q4k_bytes(shape.vocab, shape.hidden)
    threads = os.cpu_count() or 1
    for _ in range(args.warmup):
        cpu_sample_rate(mats, 0.0, threads)
    rates, total_el, total_bytes = [], 0.0, 0
    for _ in range(args.steps):
        gbs, el, nbytes, passes = cpu_sample_rate(mats, 0.0, threads)
        rates.append(gbs)
        total_el += el
        total_bytes += nbytes * passes
    value = total_bytes / total_el / 1e9
    line = {
        "metric": METRIC,
        "value": round(value, 3),
        "unit": UNIT,
        "impl": "reference",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(total_el / args.steps * 1e3, 3),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic (seeded Q4_K super-blocks + N(0,1) f32 activations)",
        "config": {"workload": f"c3 decode-step weight sweep, E2B-shaped, M={args.batch}", "batch": args.batch,
                   "sample_per_step": "layer 0's 7 GEMVs (19.9 MB Q4_K)",
                   "full_step_bytes": bytes_step_full},
        "cpu_baseline": {"value": round(value, 3), "unit": UNIT, "cores": threads, "kind": "port",
                         "sample": "layer 0's 7 GEMVs per step; CPU restatement of gguf.ts Q4_K decode + "
                                   "f32ToF16Array RNE + matmul_quant.wgsl order (the reference is TypeScript+WGSL: "
                                   "its WebGPU path is unavailable on this box)"},
        "e2e": {"value": round(value, 3), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "tokens_per_s": round(value * 1e9 / bytes_step_full, 4),
    }
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--batch", type=int, default=1, help="activation rows per step (config 3: 1 or 4)")
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--cpu-seconds", type=float, default=16.0, help="CPU baseline: total seconds over its 4 variants")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--no-real", action="store_true", help="skip the real-E2B-shape (Q4_K + Q6_K) sweep")
    ap.add_argument("--no-c4", action="store_true", help="skip the config-4 batched sweeps")
    ap.add_argument("--no-chain", action="store_true", help="skip the chained (layer-dependent) decode step")
    ap.add_argument("--case", choices=CASES, default=None,
                    help="run one kernel's small profiler case instead of the benchmark (see run_case)")
    ap.add_argument("--reps", type=int, default=40, help="--case: launches to run")
    ap.add_argument("--layers", type=int, default=8, help="--case sweep: layers of the plan")
    ap.add_argument("--f16x", action="store_true", help="--case gemm: activations rounded to f16 (q4k_gemm_f16x)")
    ap.add_argument("--exact", action="store_true", help="--case gemmplan: exact f16 hi + lo activations")
    args = ap.parse_args()
    if args.case is not None:
        run_case(args)
        return
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
