"""GPU parity at the largest sizes: 64-bit indexing past 2^31 output elements in the dequant (one
tensor of 8.6 GB F32, single and batched entry points), and the GQA workload's full forward
(a 4.29 GB output, so TMA and epilogue offsets pass 2^32 bytes) and full broadcast-operand
gradient. Each output element depends only on its own block (dequant) or its own row and column
(mul_mat), so windows and planes of the full-size run are checked against the oracle run on those
windows and planes alone."""
from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
import synth
from conftest import normwise

pytestmark = pytest.mark.gpu

# 2^26 blocks of 32 weights is 2^31 weights; 4099 more make a ragged last run of blocks.
BIG_BLOCKS = (1 << 26) + 4099
WINDOW = 4096


@pytest.fixture(scope="module")
def tc():
    import trc_cuda

    trc_cuda.lib()
    assert torch.cuda.is_available()
    return trc_cuda


def bits_equal(got: np.ndarray, want: np.ndarray) -> bool:
    g, w = got.view(np.uint32), want.view(np.uint32)
    nan = np.isnan(want)
    return bool(np.array_equal(np.isnan(got), nan) and np.array_equal(g[~nan], w[~nan]))


def check_windows(qtype: int, blocks: torch.Tensor, out: torch.Tensor) -> None:
    """First blocks, the blocks around weight 2^31 and the last blocks, bit for bit."""
    bb = synth.BLOCK_BYTES[qtype]
    for b0 in (0, (1 << 26) - WINDOW // 2, BIG_BLOCKS - WINDOW):
        packed = blocks[b0 * bb:(b0 + WINDOW) * bb].cpu().numpy()
        want = oracle.dequant(qtype, packed, WINDOW)
        got = out[b0 * 32:(b0 + WINDOW) * 32].cpu().numpy()
        assert bits_equal(got, want), f"blocks {b0}..{b0 + WINDOW}"


def test_dequant_past_2_31_weights(tc):
    g = torch.Generator(device="cuda").manual_seed(31)
    t = synth.TYPE_Q4_0
    blocks = synth.random_blocks_torch(t, BIG_BLOCKS, g, "cuda")
    out = torch.full((BIG_BLOCKS * 32,), float("nan"), device="cuda")
    tc.gguf_tensor_to_f32(t, blocks, out=out)
    torch.cuda.synchronize()
    check_windows(t, blocks, out)
    assert tc.device_error() == 0


def test_batched_dequant_past_2_31_weights_and_bytes(tc):
    """Q8_0 at this size also puts the packed input past 2^31 bytes (2.28 GB); a small tensor in
    front makes the big job start at a nonzero run of the batch."""
    g = torch.Generator(device="cuda").manual_seed(32)
    small_t, big_t = synth.TYPE_Q5_1, synth.TYPE_Q8_0
    small = synth.random_blocks_torch(small_t, 1000, g, "cuda")
    big = synth.random_blocks_torch(big_t, BIG_BLOCKS, g, "cuda")
    out_small = torch.empty(1000 * 32, device="cuda")
    out_big = torch.full((BIG_BLOCKS * 32,), float("nan"), device="cuda")
    tc.dequantize_many([(small_t, small, out_small), (big_t, big, out_big)])
    torch.cuda.synchronize()
    assert bits_equal(out_small.cpu().numpy(), oracle.dequant(small_t, small.cpu().numpy(), 1000))
    check_windows(big_t, big, out_big)
    assert tc.device_error() == 0


@pytest.fixture(scope="module")
def gqa(tc):
    """The GQA workload at full size: A ggml [128, 2048, 8, 8], B [128, 2048, 32, 8]."""
    g = torch.Generator(device="cuda").manual_seed(5)
    A = torch.randn((8, 8, 2048, 128), generator=g, device="cuda")
    B = torch.randn((8, 32, 2048, 128), generator=g, device="cuda")
    return A, B


def test_gqa_full_forward_planes(tc, gqa):
    A, B = gqa
    D = tc.mul_mat(A, B)                              # ggml [2048, 2048, 32, 8]: 4.29 GB
    assert tuple(D.shape) == (8, 32, 2048, 2048)
    torch.cuda.synchronize()
    for i3, i2 in ((0, 0), (5, 17), (7, 31)):
        want = oracle.mul_mat(A[i3 % 8, i2 % 8].cpu().numpy(), B[i3, i2].cpu().numpy())[0, 0]
        assert normwise(D[i3, i2].cpu().numpy(), want) <= 1e-5, (i3, i2)
    del D
    assert tc.device_error() == 0


def test_gqa_full_broadcast_gradient_planes(tc, gqa):
    """dA = repeat_back(T(mul_mat(T(G), T(B)))) into A's layout: each of the 8 x 8 planes sums the
    products of 4 broadcast planes (i2 = g, g+8, g+16, g+24), K = 2048 each."""
    _, B = gqa
    g = torch.Generator(device="cuda").manual_seed(6)
    G = torch.randn((8, 32, 2048, 2048), generator=g, device="cuda") * 0.01
    dA = torch.zeros((8, 8, 2048, 128), device="cuda")
    tc.mul_mat_repeat_back(G.transpose(-1, -2), B.transpose(-1, -2), dA.transpose(-1, -2))
    torch.cuda.synchronize()
    for i3, ga in ((0, 0), (6, 3), (7, 7)):
        want = None
        for i2 in range(ga, 32, 8):                   # the reference's repeat_back order
            a_t = np.ascontiguousarray(G[i3, i2].cpu().numpy().T)
            b_t = np.ascontiguousarray(B[i3, i2].cpu().numpy().T)
            p = oracle.mul_mat(a_t, b_t)[0, 0]        # ggml [2048, 128] -> numpy (128, 2048)
            want = p if want is None else want + p
        got = dA[i3, ga].transpose(0, 1).cpu().numpy()
        assert normwise(np.ascontiguousarray(got), want) <= 1e-5, (i3, ga)
    del G
    assert tc.device_error() == 0
