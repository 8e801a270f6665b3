"""GPU: frozen quantized weights behind train.cpp's unchanged API (tests/dropin/test_dropin.cpp,
modes `packed` and `checkpoint`).

  * A weight allocated from the packed-weight buffer type (CUDA<i>_Q) is an F32 graph tensor whose
    F32 bytes never exist on the device: nn::Linear's forward and the gradient of its input through
    train.cpp's autograd run the dequant-in-prologue GEMM on its GGUF blocks. Results are bit for bit
    those of the same graph with W dequantized into an ordinary F32 tensor, within 1e-5 normwise of
    the CPU device, and the loaded weight takes its packed bytes of device memory, not its F32 bytes
    (the Linear workload's Q5_0 4096 x 14336 weight: 40 MB instead of 235 MB). The preflight reports
    any other op that would read a packed weight.
  * checkpoint_save / checkpoint_load of train.cpp over CUDA buffers: a model trained on the device,
    saved, and loaded onto a fresh CUDA model and a fresh CPU model gives bit-identical parameters
    and AdamW states on both."""
from __future__ import annotations

import pytest

import synth
from test_gpu_dropin import run

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def packed_gguf(tmp_path_factory):
    p = tmp_path_factory.mktemp("packed") / "weights.gguf"
    specs = [("linear_q5_0", synth.TYPE_Q5_0, (4096, 14336)),   # the Linear workload's weight
             ("small_q4_0", synth.TYPE_Q4_0, (1024, 96)), ("small_q4_1", synth.TYPE_Q4_1, (512, 300)),
             ("small_q5_1", synth.TYPE_Q5_1, (256, 72)), ("small_q8_0", synth.TYPE_Q8_0, (768, 260))]
    tensors = [(name, t, ne, synth.random_blocks(t, ne[0] * ne[1] // 32, seed=700 + i))
               for i, (name, t, ne) in enumerate(specs)]
    synth.write_gguf(p, tensors)
    return p


def test_packed_weights_linear_forward_and_dx(packed_gguf):
    r = run(["packed", str(packed_gguf), "2048"])
    print(r.stdout)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "bit-identical to the F32 device path" in r.stdout


def test_packed_weights_small_token_count(packed_gguf):
    """Fewer columns than a tile: the fused kernel's small-N plan, still bit for bit the F32 path."""
    r = run(["packed", str(packed_gguf), "40"])
    assert r.returncode == 0, r.stdout + r.stderr


def test_checkpoint_roundtrip_on_device(tmp_path):
    r = run(["checkpoint", str(tmp_path / "ckpt.gguf")])
    print(r.stdout)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "checkpoint round trip" in r.stdout
