"""CPU: the reference arm of bench.py (train.cpp's own host dequant, timed on the host cores) keeps
the bench line's contract: one JSON line with the metric, config and units of our arm, its own
cpu_baseline and an e2e with no host<->device bytes; under torchrun only rank 0 runs and prints,
and every rank exits 0."""
from __future__ import annotations

import json
import os
import socket
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


def run(cmd: list[str], timeout: int = 300) -> subprocess.CompletedProcess:
    env = dict(os.environ)
    env.pop("RANK", None)
    return subprocess.run(cmd, cwd=ROOT, capture_output=True, text=True, timeout=timeout, env=env)


def json_lines(out: str) -> list[dict]:
    lines = []
    for ln in out.splitlines():
        ln = ln.strip()
        if ln.startswith("{"):
            lines.append(json.loads(ln))
    return lines


def check_line(d: dict, n_gpus: int, steps: int, warmup: int) -> None:
    for k in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
              "scaling", "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"):
        assert k in d, k
    assert d["impl"] == "reference"
    assert d["n_gpus"] == n_gpus and d["steps"] == steps and d["warmup"] == warmup
    assert d["unit"] == "GB/s" and d["higher_is_better"] is True and d["value"] > 0
    assert "workload" in d["config"]
    cb = d["cpu_baseline"]
    assert cb["kind"] in ("reference", "port") and cb["cores"] >= 1 and cb["value"] == d["value"] and cb["sample"]
    e2e = d["e2e"]
    assert e2e["value"] == d["value"] and e2e["unit"] == d["unit"]
    assert e2e["h2d_bytes_per_step"] == 0 and e2e["d2h_bytes_per_step"] == 0


def test_reference_arm_line():
    r = run([sys.executable, "bench.py", "--impl", "reference", "--steps", "2", "--warmup", "3"])
    assert r.returncode == 0, r.stderr[-2000:]
    lines = json_lines(r.stdout)
    assert len(lines) == 1
    check_line(lines[0], n_gpus=1, steps=2, warmup=3)


def free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_reference_arm_under_torchrun_prints_once():
    r = run([sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2",
             "--master-addr", "127.0.0.1", "--master-port", str(free_port()),
             "bench.py", "--impl", "reference", "--gpus", "2", "--steps", "1", "--warmup", "3"])
    assert r.returncode == 0, r.stderr[-2000:]
    lines = json_lines(r.stdout)
    assert len(lines) == 1  # rank 0 only
    check_line(lines[0], n_gpus=2, steps=1, warmup=3)


@pytest.mark.gpu
def test_our_arm_line():
    """Our arm on one GPU (headline only): the base contract's keys, the roofline and cpu_baseline
    objects, an e2e with the host bytes counted, the clock record, and one library launch per
    timed step."""
    r = run([sys.executable, "bench.py", "--no-secondary", "--steps", "3", "--warmup", "3"], timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = json_lines(r.stdout)
    assert len(lines) == 1
    d = lines[0]
    for k in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
              "scaling", "vs_baseline", "dtype", "data", "config", "roofline", "cpu_baseline", "e2e", "clocks",
              "gpu_launches"):
        assert k in d, k
    assert d["n_gpus"] == 1 and d["steps"] == 3 and d["warmup"] == 3 and d["value"] > 0
    rf = d["roofline"]
    assert rf["bound"] == "hbm" and rf["unit"] == "GB/s" and rf["peak"] > 0
    assert abs(rf["frac"] - rf["achieved"] / rf["peak"]) < 1e-3
    cb = d["cpu_baseline"]
    assert cb["value"] > 0 and cb["cores"] >= 1 and cb["kind"] in ("reference", "port")
    e2e = d["e2e"]
    assert e2e["value"] > 0 and e2e["h2d_bytes_per_step"] > 0 and e2e["d2h_bytes_per_step"] > 0
    assert e2e["value"] != d["value"]
    assert d["clocks"]["sm_max_mhz"]
    assert d["gpu_launches"] == d["steps"]  # one batched dequant launch per step
