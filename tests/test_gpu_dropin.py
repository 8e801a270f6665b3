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


@pytest.fixture(scope="module")
def model_gguf(tmp_path_factory):
    """A small model-like file: 14 tensors of every legacy type, sizes spread over two orders of
    magnitude (several larger than the loader's 1 MiB test staging), and one F32 tensor (which the
    reference loader handles)."""
    p = tmp_path_factory.mktemp("gguf") / "model.gguf"
    shapes = [(4096, 600), (1024, 96), (4096, 64), (512, 40), (4096, 33), (256, 7), (2048, 512), (4096, 128),
              (1024, 1024), (64, 64), (4096, 300), (128, 11), (2048, 256)]
    types = [synth.TYPE_Q5_1, synth.TYPE_Q4_0, synth.TYPE_Q8_0, synth.TYPE_Q5_0, synth.TYPE_Q4_1]
    tensors = []
    for i, ne in enumerate(shapes):
        t = types[i % len(types)]
        tensors.append((f"t{i}", t, ne, synth.random_blocks(t, ne[0] * ne[1] // 32, seed=700 + i)))
    f32 = synth.normal((48, 64), seed=799)
    tensors.append(("norm.weight", synth.TYPE_F32, (64, 48), f32))
    synth.write_gguf(p, tensors)
    return p, tensors


def test_sharded_model_load(model_gguf):
    """cuda_gguf_load_tensors over each rank's share (gguf_shard_tensors) at 1, 2 and 3 ranks:
    bit-identical to the reference loader, and the C++ plan equals sharding.lpt_shards over the same
    load bytes (packed or F32 bytes read + F32 bytes written)."""
    import re

    import sharding

    path, tensors = model_gguf
    r = run(["shard", str(path)])
    print(r.stdout)
    assert r.returncode == 0, r.stdout + r.stderr
    sizes = []
    for _, t, ne, data in tensors:
        n = ne[0] * ne[1]
        sizes.append(data.nbytes + 4 * n)
    for world in (1, 2, 3):
        want = sharding.lpt_shards(sizes, world)
        for rank in range(world):
            m = re.search(rf"^shard {world} {rank}:(.*)$", r.stdout, re.M)
            assert m, r.stdout
            got = [int(x) for x in m.group(1).split()]
            assert got == want[rank], (world, rank, got, want[rank])
