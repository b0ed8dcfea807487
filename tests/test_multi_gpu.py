"""Vocabulary-parallel LM head on 2+ GPUs (NCCL), through torchrun.

Skipped with fewer than two visible GPUs.  Each rank checks that the merged
candidates of the sharded head equal the unsharded head's (mgpu_sharded_worker.py).
"""
from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parents[1]


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_sharded_lmhead_over_nccl():
    n = min(torch.cuda.device_count(), 8)
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={n}", "--master-addr=127.0.0.1", "--master-port=29517",
           str(ROOT / "tests" / "mgpu_sharded_worker.py")]
    r = subprocess.run(cmd, capture_output=True, text=True, env=dict(os.environ))
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-4000:]
    assert sum(line.endswith(" ok") for line in r.stdout.splitlines()) == n, r.stdout
