"""CPU: the backend's whole-model shard plan (gguf_shard_tensors, read from a GGUF header alone)
equals the Python LPT partition (train.cpp_b200/sharding.py) at 1..8 ranks, and the ranks' shares
partition the file. No GPU is needed: the plan only parses the file's header."""
from __future__ import annotations

import ctypes
from pathlib import Path

import pytest

import sharding
import synth

BACKEND = Path(__file__).resolve().parents[1] / "train.cpp_b200" / "lib" / "libtrc_cuda_backend.so"


@pytest.fixture(scope="module")
def backend():
    import oracle

    if not BACKEND.exists() or not oracle.ref_available():
        pytest.skip("backend library or oracle/_ref not built (both need the train.cpp sources)")
    # the backend takes train.cpp's core (GGUF reader, registry) from the host program: here the
    # reference compiled from its sources, loaded first with global symbol visibility
    ctypes.CDLL(str(oracle.REF_SO), mode=ctypes.RTLD_GLOBAL)
    L = ctypes.CDLL(str(BACKEND))
    L.trc_cuda_backend_gguf_shard_plan.restype = ctypes.c_int64
    L.trc_cuda_backend_gguf_shard_plan.argtypes = [ctypes.c_char_p, ctypes.c_int, ctypes.c_int,
                                                    ctypes.POINTER(ctypes.c_int64), ctypes.c_int64]
    return L


def test_plan_matches_python_lpt(backend, tmp_path):
    # a small model-like header (the blocks are tiny; only their sizes matter to the plan)
    shapes = [(64, 60), (32, 96), (128, 64), (64, 40), (256, 33), (32, 7), (64, 512), (128, 128), (32, 1024),
              (32, 32), (128, 300), (32, 11), (64, 256), (96, 96), (64, 2)]
    types = [synth.TYPE_Q5_1, synth.TYPE_Q4_0, synth.TYPE_Q8_0, synth.TYPE_Q5_0, synth.TYPE_Q4_1]
    tensors, sizes = [], []
    for i, ne in enumerate(shapes):
        t = types[i % len(types)]
        data = synth.random_blocks(t, ne[0] * ne[1] // 32, seed=i)
        tensors.append((f"t{i}", t, ne, data))
        sizes.append(data.nbytes + 4 * ne[0] * ne[1])
    f32 = synth.normal((8, 64), seed=99)
    tensors.append(("norm", synth.TYPE_F32, (64, 8), f32))
    sizes.append(f32.nbytes + 4 * f32.size)
    path = tmp_path / "m.gguf"
    synth.write_gguf(path, tensors)
    for world in range(1, 9):
        want = sharding.lpt_shards(sizes, world)
        seen = []
        for rank in range(world):
            buf = (ctypes.c_int64 * len(tensors))()
            n = backend.trc_cuda_backend_gguf_shard_plan(str(path).encode(), rank, world, buf, len(tensors))
            got = [buf[i] for i in range(n)]
            assert got == want[rank], (world, rank)
            seen += got
        assert sorted(seen) == list(range(len(tensors)))
    assert backend.trc_cuda_backend_gguf_shard_plan(str(path).encode(), 3, 3, None, 0) == -1
