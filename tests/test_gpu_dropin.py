"""GPU: the CUDA backend as a drop-in device behind train.cpp's unchanged API (tests/dropin/
test_dropin.cpp, linked against the reference library and libtrc_cuda_backend.so): conformance
mul_mat cases, training steps through the reference autograd (with and without the backend's
graph-level fusion), device-side GGUF warm start bit-identical to the reference loader, and the
allocation-failure path (a host-side fake; no GPU fault)."""
from __future__ import annotations

import os
import subprocess
from pathlib import Path

import pytest

import synth

pytestmark = pytest.mark.gpu

BIN = Path(__file__).resolve().parent / "dropin" / "_build" / "test_dropin"


@pytest.fixture(scope="module")
def gguf_path(tmp_path_factory):
    p = tmp_path_factory.mktemp("gguf") / "warm.gguf"
    tensors = []
    for i, (t, ne) in enumerate([(synth.TYPE_Q5_0, (1024, 96)), (synth.TYPE_Q4_0, (4096, 64)),
                                 (synth.TYPE_Q8_0, (512, 40)), (synth.TYPE_Q5_1, (4096, 33)),
                                 (synth.TYPE_Q4_1, (256, 7))]):
        n_blocks = ne[0] * ne[1] // 32
        tensors.append((f"w{i}", t, ne, synth.random_blocks(t, n_blocks, seed=500 + i)))
    synth.write_gguf(p, tensors)
    return p


def run(args, env_extra=None):
    if not BIN.exists():
        pytest.fail(f"{BIN} not built (make -C tests/dropin, needs the train.cpp headers)")
    env = dict(os.environ)
    env.update(env_extra or {})
    return subprocess.run([str(BIN), *args], capture_output=True, text=True, env=env, timeout=600)


def test_dropin_all_cases(gguf_path):
    r = run(["all", str(gguf_path)])
    print(r.stdout)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "PASS" in r.stdout


def test_dropin_without_graph_fusion(gguf_path):
    r = run(["all", str(gguf_path)], {"TRC_CUDA_NO_FUSION": "1"})
    assert r.returncode == 0, r.stdout + r.stderr


def test_allocation_failure_aborts_with_core_message():
    r = run(["alloc_fail"], {"TRC_CUDA_FAIL_ALLOC": "1"})
    assert r.returncode != 0
    assert "分配失败" in r.stderr, r.stderr


def test_dropin_bit_identical_with_simt_mul_mat(gguf_path):
    """With TRC_CUDA_MM_SIMT=1 every mul_mat sums in the reference's order, so whole training loops
    on the CUDA device (autograd backward, optimizer and grad-norm clip graphs included) end with
    parameters bit-identical to the reference CPU device."""
    r = run(["all", str(gguf_path)], {"TRC_CUDA_MM_SIMT": "1"})
    print(r.stdout)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "bit-identical (loss" in r.stdout
