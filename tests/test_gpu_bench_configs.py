"""GPU parity on the exact GEMM configurations bench.py times, at their full sizes.

  * The Linear training step (Q5_0 weight ne=[4096,14336], 2048 tokens), through the same calls as
    the bench: mul_mat_q's default (the fused dequant-in-prologue kernel) and its two-step path (W
    dequantized into scratch, then the F32 kernel) for the forward and for dX = transpose(W) . dY
    (K = 14336, split-K in four parts), and dW for an F32 copy of W accumulated (ACCUMULATE) through
    the transposed view of its gradient buffer on top of a nonzero start.
  * The GQA batched broadcast step (A ne=[128,2048,8,p3], B ne=[128,2048,32,p3]) at p3 = 8 (one
    GPU) and p3 = 1 (one ne[3] plane per rank at 8 GPUs; another tile and split-K plan): forward,
    the plane-reducing dA and dB.

Two checks per product:
  * the whole output against a float64 product on the GPU, normwise <= 5e-6 (3xTF32 with fp32
    promotion measures ~2.3e-6 at every K; the reference's own fp32 summation is 2.4e-6 to 4.4e-6
    from exact);
  * a slice (64 token columns, or one (i2, i3) plane) against the oracle, which restates the
    reference's compute_mul_mat (src/backends/cpu/trc_cpu_ops.cpp:182-216) and its summation order
    bit for bit, normwise <= 1e-5; a narrower slice also against the reference compiled from its
    sources (oracle/_ref) where it is built. Each output element's reference sum depends only on
    its own row and column, so a slice of the full-size run equals the reference run on the slice.
The composed backward's products follow src/core/trc_autograd.cpp:487-503."""
from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
import synth
from conftest import normwise

pytestmark = pytest.mark.gpu

TOL_REF = 1e-5    # normwise against the reference summation
TOL_EXACT = 5e-6  # normwise against a float64 product
K, M, N = 4096, 14336, 2048


@pytest.fixture(scope="module")
def tc():
    import trc_cuda

    trc_cuda.lib()
    return trc_cuda


def err64(got: torch.Tensor, want64: torch.Tensor) -> float:
    return ((got.double() - want64).abs().max() / want64.abs().max()).item()


def cols(n: int, count: int, seed: int) -> np.ndarray:
    return np.sort(np.random.default_rng(seed).choice(n, count, replace=False))


@pytest.fixture(scope="module")
def linear(tc):
    g = torch.Generator(device="cuda").manual_seed(4)
    wq = torch.from_numpy(synth.random_blocks(synth.TYPE_Q5_0, K * M // 32, seed=21)).cuda()
    W = tc.gguf_tensor_to_f32(synth.TYPE_Q5_0, wq).view(M, K)          # ggml [4096, 14336]
    X = torch.randn((N, K), generator=g, device="cuda")                  # ggml [4096, 2048]
    dY = torch.randn((N, M), generator=g, device="cuda") * 1e-2          # ggml [14336, 2048]
    Wn = oracle.dequant(synth.TYPE_Q5_0, wq.cpu().numpy()).reshape(M, K)
    assert np.array_equal(W.cpu().numpy().view(np.uint32), Wn.view(np.uint32))
    return wq, W, X, dY, Wn


@pytest.mark.parametrize("two_step", [False, True], ids=["default_fused", "two_step"])
def test_linear_forward_full_size(tc, linear, two_step):
    wq, W, X, _, Wn = linear
    Y = torch.full((N, M), float("nan"), device="cuda")
    tc.mul_mat_q(synth.TYPE_Q5_0, wq, K, M, X, out=Y, two_step=two_step)
    torch.cuda.synchronize()
    assert tc.device_error() == 0
    assert err64(Y, X.double() @ W.double().t()) <= TOL_EXACT
    j = cols(N, 64, 1)
    want = oracle.mul_mat(Wn, X[j].cpu().numpy())[0, 0]                  # (64, M)
    assert normwise(Y[j].cpu().numpy(), want) <= TOL_REF
    if oracle.ref_available():
        got = Y[j[:8]].cpu().numpy()
        assert normwise(got, oracle.ref_mul_mat(Wn, False, X[j[:8]].cpu().numpy(), False)[0, 0]) <= TOL_REF


@pytest.mark.parametrize("two_step", [False, True], ids=["default_fused", "two_step"])
def test_linear_dx_full_size(tc, linear, two_step):
    """dX = mul_mat(transpose(W), dY): K = 14336, 4096 x 2048 outputs (128 pair tiles of 256 x 256),
    which the planner splits in four parts (two reduce into dX, two into a workspace added by one
    more kernel). A stream plan is not taken: the bands its tiles share (352 MB) exceed L2."""
    wq, W, _, dY, Wn = linear
    dX = torch.full((N, K), float("nan"), device="cuda")
    torch.cuda.synchronize()
    n0 = tc.launch_count()
    tc.mul_mat_q(synth.TYPE_Q5_0, wq, K, M, dY, transposed=True, out=dX, two_step=two_step)
    torch.cuda.synchronize()
    launched = tc.launch_count() - n0
    # two steps: dequant, GEMM, workspace add; fused: GEMM, workspace add
    assert launched == (3 if two_step else 2), launched
    assert tc.device_error() == 0
    assert err64(dX, dY.double() @ W.double()) <= TOL_EXACT
    j = cols(N, 64, 2)
    want = oracle.mul_mat(np.ascontiguousarray(Wn.T), dY[j].cpu().numpy())[0, 0]   # (64, K)
    assert normwise(dX[j].cpu().numpy(), want) <= TOL_REF


def test_linear_dw_accumulate_full_size(tc, linear):
    """dW for an F32 copy of W: the composed rule's T(mul_mat(T(dY), T(X))) + cont + acc into
    grad_acc, run as one GEMM that reduce-adds into the transposed view of the gradient buffer
    (K = 2048), on top of a nonzero gradient already there."""
    _, _, X, dY, _ = linear
    g = torch.Generator(device="cuda").manual_seed(5)
    base = torch.randn((M, K), generator=g, device="cuda") * 0.5
    dW = base.clone()
    tc.mul_mat(dY.t(), X.t(), out=dW.t(), accumulate=True)
    torch.cuda.synchronize()
    assert tc.device_error() == 0
    prod64 = dY.double().t() @ X.double()                                 # (M, K)
    assert err64(dW - base, prod64) <= TOL_EXACT
    assert err64(dW, base.double() + prod64) <= TOL_EXACT
    k = cols(K, 64, 3)
    want = oracle.mul_mat(np.ascontiguousarray(dY.cpu().numpy().T),
                          np.ascontiguousarray(X.cpu().numpy().T[k]))[0, 0]          # (64, M)
    got = (dW[:, k] - base[:, k]).t().cpu().numpy()
    assert normwise(got, want) <= TOL_REF
    # the reference adds its rounded product into grad_acc: base + product, one fp32 add
    want_acc = (base[:, k].t().cpu().numpy() + want).astype(np.float32)
    assert normwise(dW[:, k].t().cpu().numpy(), want_acc) <= TOL_REF


@pytest.mark.parametrize("p3", [8, 1])
def test_gqa_step_full_size(tc, p3):
    """The GQA step as the bench times it per rank: D = mul_mat(A, B) (A broadcast over ne[2] by 4),
    dA = repeat_back(T(mul_mat(T(G), T(B)))) in one plane-reducing GEMM written through T(dA), and
    dB = mul_mat(T(A), G)."""
    g = torch.Generator(device="cuda").manual_seed(60 + p3)
    A = torch.randn((p3, 8, 2048, 128), generator=g, device="cuda")
    B = torch.randn((p3, 32, 2048, 128), generator=g, device="cuda")
    G = torch.randn((p3, 32, 2048, 2048), generator=g, device="cuda")
    D = torch.full((p3, 32, 2048, 2048), float("nan"), device="cuda")
    dA = torch.full((p3, 8, 2048, 128), float("nan"), device="cuda")
    dB = torch.full((p3, 32, 2048, 128), float("nan"), device="cuda")
    tc.mul_mat(A, B, out=D)
    tc.mul_mat_repeat_back(G.transpose(-1, -2), B.transpose(-1, -2), dA.transpose(-1, -2))
    tc.mul_mat(A.transpose(-1, -2), G, out=dB)
    torch.cuda.synchronize()
    assert tc.device_error() == 0
    Ar = A.double().repeat(1, 4, 1, 1)                                     # plane i2 -> A plane i2 % 8
    # whole outputs against float64 (D in ne[3] chunks to bound the float64 temporaries)
    for i3 in range(p3):
        assert err64(D[i3], B[i3].double() @ Ar[i3].transpose(-1, -2)) <= TOL_EXACT, i3
    assert err64(dB, G.double() @ Ar) <= TOL_EXACT
    dA64 = (G.double().transpose(-1, -2) @ B.double()).view(p3, 4, 8, 2048, 128).sum(1)
    assert err64(dA, dA64) <= TOL_EXACT
    del Ar, dA64
    # one (i2, i3) plane of each product against the oracle
    i3, i2 = p3 - 1, 13
    a, b, gm = A[i3, i2 % 8].cpu().numpy(), B[i3, i2].cpu().numpy(), G[i3, i2].cpu().numpy()
    assert normwise(D[i3, i2].cpu().numpy(), oracle.mul_mat(a, b)[0, 0]) <= TOL_REF
    want_db = oracle.mul_mat(np.ascontiguousarray(a.T), gm)[0, 0]          # (2048, 128)
    assert normwise(dB[i3, i2].cpu().numpy(), want_db) <= TOL_REF
    ga = 5                                                                  # planes 5, 13, 21, 29
    want_da = None
    for p in range(ga, 32, 8):                                              # repeat_back's order
        prod = oracle.mul_mat(np.ascontiguousarray(G[i3, p].cpu().numpy().T),
                              np.ascontiguousarray(B[i3, p].cpu().numpy().T))[0, 0]   # (128, 2048)
        want_da = prod if want_da is None else want_da + prod
    assert normwise(np.ascontiguousarray(dA[i3, ga].t().cpu().numpy()), want_da) <= TOL_REF
    if oracle.ref_available():
        got = dB[i3, i2, :64].cpu().numpy()
        want = oracle.ref_mul_mat(np.ascontiguousarray(a.T), False, np.ascontiguousarray(gm[:64]), False)[0, 0]
        assert normwise(got, want) <= TOL_REF
