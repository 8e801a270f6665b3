"""The fused dequant + all-gather (trc_cuda_dequant_many_to_peers) on two GPUs: two torchrun
ranks, plain peer stores over NVLink, bit-exact against the oracle on every rank. Skipped on a
box with one GPU."""
from __future__ import annotations

import subprocess
import sys
from pathlib import Path

import pytest
import torch

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parents[1]


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_dequant_all_gather_two_ranks():
    cmd = ["timeout", "-k", "30", "240", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node", "2", "--master-addr", "127.0.0.1", "--master-port", "29531",
           str(ROOT / "tests" / "peers_worker.py")]
    env = {**__import__("os").environ, "NCCL_NVLS_ENABLE": "0"}
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=300, env=env)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert r.stdout.count(": OK") == 2, r.stdout
