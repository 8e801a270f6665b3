"""GPU parity of the fused dequant + mul_mat (weight decoded in the GEMM's producer stage, never
stored as F32): equal within tolerance to mul_mat on the device-dequantized weight and to the
oracle, for W and transpose(W) (forward and dX), all five formats."""
from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
import synth
from conftest import normwise

pytestmark = pytest.mark.gpu

TYPES = [synth.TYPE_Q4_0, synth.TYPE_Q4_1, synth.TYPE_Q5_0, synth.TYPE_Q5_1, synth.TYPE_Q8_0]
NAMES = {v: k for k, v in synth.TYPE_BY_NAME.items()}


@pytest.fixture(scope="module")
def tc():
    import trc_cuda

    trc_cuda.lib()
    return trc_cuda


def dev(x):
    return torch.from_numpy(np.ascontiguousarray(x)).cuda()


@pytest.mark.parametrize("one_cta", [False, True], ids=["pair", "one_cta"])
@pytest.mark.parametrize("transposed", [False, True], ids=["W", "WT"])
@pytest.mark.parametrize("qtype", TYPES, ids=lambda t: NAMES[t])
def test_fused_matches_dequant_then_mul_mat(tc, qtype, transposed, one_cta):
    w_ne0, w_ne1, n = 512, 400, 136  # W [k=512, m=400]; ragged M/N tiles
    blocks = synth.random_blocks(qtype, w_ne0 * w_ne1 // 32, seed=40 + qtype)
    Wf = oracle.dequant(qtype, blocks).reshape(w_ne1, w_ne0)  # numpy (ne1, ne0)
    K = w_ne1 if transposed else w_ne0
    x = np.random.default_rng(qtype).standard_normal((n, K)).astype(np.float32)
    want = oracle.mul_mat(np.swapaxes(Wf, -1, -2) if transposed else Wf, x)
    got = tc.mul_mat_q(qtype, dev(blocks), w_ne0, w_ne1, dev(x), transposed=transposed,
                       one_cta=one_cta, fused=True).cpu().numpy()
    assert got.shape == want.shape
    assert normwise(got, want) <= 1e-5
    Wd = tc.gguf_tensor_to_f32(qtype, dev(blocks)).reshape(w_ne1, w_ne0)
    two_step = tc.mul_mat(Wd.t() if transposed else Wd, dev(x), one_cta=one_cta).cpu().numpy()
    assert normwise(got, two_step) <= 2e-6
    assert tc.device_error() == 0


@pytest.mark.parametrize("one_cta", [False, True], ids=["pair", "one_cta"])
def test_fused_split_k_fills_the_last_wave(tc, one_cta):
    """The fused kernel split in K: 80 pair tiles on 74 pairs take a stream plan (the TMA-staged
    kernel); 160 single tiles on 148 SMs run as two parts each in the kernel whose split warps load
    the packed words from global memory, so their look-ahead crosses units of both parts."""
    qtype, w_ne0, w_ne1, n = synth.TYPE_Q4_1, 1024, 2560, 2048
    blocks = synth.random_blocks(qtype, w_ne0 * w_ne1 // 32, seed=81)
    Wf = oracle.dequant(qtype, blocks).reshape(w_ne1, w_ne0)
    x = np.random.default_rng(82).standard_normal((n, w_ne0)).astype(np.float32)
    want = oracle.mul_mat(Wf, x)
    out = torch.full((n, w_ne1), float("nan"), device="cuda")
    got = tc.mul_mat_q(qtype, dev(blocks), w_ne0, w_ne1, dev(x), out=out, one_cta=one_cta, fused=True).cpu().numpy()
    again = tc.mul_mat_q(qtype, dev(blocks), w_ne0, w_ne1, dev(x), one_cta=one_cta, fused=True).cpu().numpy()
    assert tc.device_error() == 0
    assert normwise(got, want.reshape(got.shape)) <= 1e-5
    assert np.array_equal(got.view(np.uint32), again.reshape(got.shape).view(np.uint32))  # deterministic


@pytest.mark.parametrize("w_ne0,w_ne1,n,launches", [
    (3840, 4096, 1280, 1),    # 75 pair tiles of 256 k-blocks: stream plan, at most two pieces a tile
    (2048, 8192, 1024, 2),    # 32 pair tiles of 512 k-blocks: stream plan, pieces 3-4 in the workspace
    (1024, 16384, 1024, 2),   # 16 pair tiles of 1024 k-blocks: four parts (two in the workspace)
], ids=["stream", "stream_workspace", "four_parts"])
def test_fused_transposed_split_k(tc, w_ne0, w_ne1, n, launches):
    """dX's kind of product, transpose(W) . dY (M = W's ne0, K = W's ne1), through the TMA-staged
    fused kernel under each split plan: the GEMM, plus the workspace add where pieces or parts go
    there. Deterministic, and within the bar (all of it against float64, 64 columns against the
    oracle)."""
    qtype = synth.TYPE_Q5_0
    blocks = synth.random_blocks(qtype, w_ne0 * w_ne1 // 32, seed=83 + w_ne1)
    Wf = oracle.dequant(qtype, blocks).reshape(w_ne1, w_ne0)
    dy = (np.random.default_rng(84).standard_normal((n, w_ne1)) * 1e-2).astype(np.float32)
    torch.cuda.synchronize()
    n0 = tc.launch_count()
    got = tc.mul_mat_q(qtype, dev(blocks), w_ne0, w_ne1, dev(dy), transposed=True, fused=True)
    assert tc.launch_count() - n0 == launches
    want64 = (dev(dy).double() @ dev(Wf).double()).cpu().numpy()
    got = got.cpu().numpy().reshape(n, w_ne0)
    again = tc.mul_mat_q(qtype, dev(blocks), w_ne0, w_ne1, dev(dy), transposed=True, fused=True).cpu().numpy()
    assert tc.device_error() == 0
    assert normwise(got, want64) <= 5e-6
    want = oracle.mul_mat(np.ascontiguousarray(Wf.T), dy[:64])[0, 0]
    assert normwise(got[:64], want) <= 1e-5
    assert np.array_equal(got.view(np.uint32), again.reshape(got.shape).view(np.uint32))


@pytest.mark.parametrize("transposed", [False, True], ids=["W", "WT"])
def test_two_step_equals_fused_kernel(tc, transposed):
    """The two implementations of mul_mat_q: W dequantized into scratch + the F32 kernel, and the
    fused kernel (the default here: CTA pairs, TMA-staged packed rows). W is bit-exact and both
    take the same tile and split-K plan, so the results agree bit for bit; both are within the bar
    of the reference."""
    qtype, w_ne0, w_ne1, n = synth.TYPE_Q4_1, 512, 1024, 1024
    blocks = synth.random_blocks(qtype, w_ne0 * w_ne1 // 32, seed=90)
    Wf = oracle.dequant(qtype, blocks).reshape(w_ne1, w_ne0)
    K = w_ne1 if transposed else w_ne0
    x = np.random.default_rng(91).standard_normal((n, K)).astype(np.float32)
    want = oracle.mul_mat(np.swapaxes(Wf, -1, -2) if transposed else Wf, x)
    torch.cuda.synchronize()
    n0 = tc.launch_count()
    two = tc.mul_mat_q(qtype, dev(blocks), w_ne0, w_ne1, dev(x), transposed=transposed, two_step=True)
    torch.cuda.synchronize()
    launched = tc.launch_count() - n0
    fused = tc.mul_mat_q(qtype, dev(blocks), w_ne0, w_ne1, dev(x), transposed=transposed)
    assert tc.device_error() == 0
    two, fused = two.cpu().numpy(), fused.cpu().numpy()
    assert launched >= 2  # the dequant, then the F32 GEMM (no B-tail pass)
    assert np.array_equal(two.view(np.uint32), fused.view(np.uint32))
    assert normwise(two, want.reshape(two.shape)) <= 1e-5


def test_two_step_accumulate_equals_fused_kernel(tc):
    """ACCUMULATE through both implementations (no split-K with ACCUMULATE, so the same plan):
    D += W^T dY on top of the same starting D, bit for bit, and within the bar of the reference."""
    qtype, w_ne0, w_ne1, n = synth.TYPE_Q8_0, 768, 512, 1024      # A = T(W): M 768, K 512
    blocks = synth.random_blocks(qtype, w_ne0 * w_ne1 // 32, seed=94)
    Wf = oracle.dequant(qtype, blocks).reshape(w_ne1, w_ne0)
    dy = (np.random.default_rng(95).standard_normal((n, w_ne1)) * 1e-2).astype(np.float32)
    d0 = np.random.default_rng(96).standard_normal((n, w_ne0)).astype(np.float32)
    outs = []
    for fused in (False, True):
        out = dev(d0)
        tc.mul_mat_q(qtype, dev(blocks), w_ne0, w_ne1, dev(dy), transposed=True, out=out, accumulate=True,
                     fused=fused, two_step=not fused)
        outs.append(out.cpu().numpy())
    assert tc.device_error() == 0
    assert np.array_equal(outs[0].view(np.uint32), outs[1].view(np.uint32))
    want = d0 + oracle.mul_mat(np.swapaxes(Wf, -1, -2), dy).reshape(d0.shape)
    assert normwise(outs[0], want) <= 1e-5


def test_simt_two_step_is_bit_exact_with_reference(tc):
    """mul_mat_q with simt=True: bit-exact dequant, then the SIMT kernel's reference summation, so
    the whole product is the reference's to the bit (also below 1024 columns)."""
    qtype, w_ne0, w_ne1, n = synth.TYPE_Q5_1, 256, 96, 40
    blocks = synth.random_blocks(qtype, w_ne0 * w_ne1 // 32, seed=92)
    Wf = oracle.dequant(qtype, blocks).reshape(w_ne1, w_ne0)
    x = np.random.default_rng(93).standard_normal((n, w_ne0)).astype(np.float32)
    want = oracle.mul_mat(Wf, x)
    got = tc.mul_mat_q(qtype, dev(blocks), w_ne0, w_ne1, dev(x), simt=True).cpu().numpy()
    assert np.array_equal(got.view(np.uint32), want.reshape(got.shape).view(np.uint32))
    assert tc.device_error() == 0


def test_fused_config_shape_slice(tc):
    """The fused Linear workload's weight (Q5_0, 4096 x 14336) against a token slice."""
    qtype, w_ne0, w_ne1 = synth.TYPE_Q5_0, 4096, 14336
    blocks = synth.random_blocks(qtype, w_ne0 * w_ne1 // 32, seed=3)
    Wf = oracle.dequant(qtype, blocks).reshape(w_ne1, w_ne0)
    x = np.random.default_rng(0).standard_normal((48, w_ne0)).astype(np.float32)
    got = tc.mul_mat_q(qtype, dev(blocks), w_ne0, w_ne1, dev(x), fused=True).cpu().numpy()
    assert normwise(got, oracle.mul_mat(Wf, x)) <= 1e-5
    dy = (np.random.default_rng(1).standard_normal((16, w_ne1)) * 1e-2).astype(np.float32)
    got_t = tc.mul_mat_q(qtype, dev(blocks), w_ne0, w_ne1, dev(dy), transposed=True, fused=True).cpu().numpy()
    assert normwise(got_t, oracle.mul_mat(np.swapaxes(Wf, -1, -2), dy)) <= 1e-5


def test_cfg1_cpu_runnable_config_in_full(tc):
    """BASELINE config 1 end to end: one Q4_0 weight ne=[4096,4096] (d ~ U[1e-3, 1e-2], uniform
    nibbles), dequantized on the device bit-exact, then mul_mat with X ne=[4096,512] ~ N(0,1) within
    1e-5 normwise of the reference summation (the oracle, threaded), both through the two-step path
    and through the fused dequant-in-prologue kernel."""
    qtype, ne0, ne1, n = synth.TYPE_Q4_0, 4096, 4096, 512
    blocks = synth.random_blocks(qtype, ne0 * ne1 // 32, seed=2024)
    Wf = oracle.dequant(qtype, blocks).reshape(ne1, ne0)
    got_w = tc.gguf_tensor_to_f32(qtype, dev(blocks)).cpu().numpy().reshape(ne1, ne0)
    assert np.array_equal(got_w.view(np.uint32), Wf.view(np.uint32))
    x = synth.normal((n, ne0), seed=2025)
    want = oracle.mul_mat(Wf, x)
    two_step = tc.mul_mat(dev(Wf), dev(x)).cpu().numpy()
    fused = tc.mul_mat_q(qtype, dev(blocks), ne0, ne1, dev(x), fused=True).cpu().numpy()
    assert normwise(two_step, want) <= 1e-5
    assert normwise(fused, want) <= 1e-5
    assert tc.device_error() == 0


@pytest.mark.parametrize("qtype", [synth.TYPE_Q4_0, synth.TYPE_Q4_1, synth.TYPE_Q5_0, synth.TYPE_Q5_1, synth.TYPE_Q8_0])
@pytest.mark.parametrize("transposed", [False, True], ids=["W", "WT"])
def test_fused_tma_staged_and_global_load_paths_agree(tc, qtype, transposed):
    """On CTA pairs the fused kernel stages each stage's packed bytes by TMA when the packed rows are
    16-byte aligned; otherwise its split warps load them from global memory. The same blocks at an
    aligned and at a 2-byte-offset address take the two paths: bit-identical results, ragged M/K
    (zero-filled rows and columns), within the bar of the reference."""
    w_ne0, w_ne1, n = 512, 300, 72                      # 16 blocks per row: aligned row pitch for every type
    bb = synth.BLOCK_BYTES[qtype]
    blocks = synth.random_blocks(qtype, w_ne0 * w_ne1 // 32, seed=120 + qtype)
    Wf = oracle.dequant(qtype, blocks).reshape(w_ne1, w_ne0)
    K = w_ne1 if transposed else w_ne0
    x = np.random.default_rng(121).standard_normal((n, K)).astype(np.float32)
    want = oracle.mul_mat(np.swapaxes(Wf, -1, -2) if transposed else Wf, x)
    aligned = dev(blocks)
    raw = torch.zeros(blocks.size + 16, dtype=torch.uint8, device="cuda")
    raw[2:2 + blocks.size] = aligned
    shifted = raw[2:2 + blocks.size]                    # 2 bytes off the 16-byte grid
    assert aligned.data_ptr() % 16 == 0 and shifted.data_ptr() % 16 == 2
    outs = [tc.mul_mat_q(qtype, wb, w_ne0, w_ne1, dev(x), transposed=transposed, fused=True).cpu().numpy()
            for wb in (aligned, shifted)]
    assert tc.device_error() == 0
    assert np.array_equal(outs[0].view(np.uint32), outs[1].view(np.uint32))
    assert normwise(outs[0], want.reshape(outs[0].shape)) <= 1e-5
    assert bb in (18, 20, 22, 24, 34)


@pytest.mark.parametrize("transposed", [False, True], ids=["W", "WT"])
def test_fused_batched_and_strided_b(tc, transposed):
    """b with ne[2] = 3, ne[3] = 2 planes (W broadcast over them, as nn::Linear on a [in, tokens,
    batch] input), and b as an MN-major (transposed) view: the fused kernel on CTA pairs with the
    TMA-staged packed bytes, within the bar of the reference on every plane."""
    qtype, w_ne0, w_ne1, n = synth.TYPE_Q8_0, 512, 384, 72
    blocks = synth.random_blocks(qtype, w_ne0 * w_ne1 // 32, seed=130)
    Wf = oracle.dequant(qtype, blocks).reshape(w_ne1, w_ne0)
    a = np.swapaxes(Wf, -1, -2) if transposed else Wf
    K = a.shape[-1]
    x = np.random.default_rng(131).standard_normal((2, 3, n, K)).astype(np.float32)
    want = oracle.mul_mat(a, x)
    got = tc.mul_mat_q(qtype, dev(blocks), w_ne0, w_ne1, dev(x), transposed=transposed).cpu().numpy()
    assert normwise(got, want) <= 1e-5
    xt = np.ascontiguousarray(np.swapaxes(x[0, 0], -1, -2))           # (K, n): b = transpose view, MN-major
    want_t = oracle.mul_mat(a, x[0, 0])
    got_t = tc.mul_mat_q(qtype, dev(blocks), w_ne0, w_ne1, dev(xt).t(), transposed=transposed).cpu().numpy()
    assert normwise(got_t.reshape(want_t.shape), want_t) <= 1e-5
    assert tc.device_error() == 0
