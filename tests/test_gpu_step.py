"""GPU parity of a whole training step of D = mul_mat(A, B) with loss = sum(mul(D, G)), executed
as the node list the reference autograd builds for it (trc_autograd.cpp:487-503):

    D = mul_mat(A, B); M = mul(D, G); L = sum(M)
    R = repeat(1.0 -> shape of M); dD = mul(R, G)
    dA' = mul_mat(T(dD), T(B)); [repeat_back when A broadcasts]; cont(T(dA')) -> acc into grad_acc(A)
    dB = mul_mat(T(A), dD) -> acc into grad_acc(B)

compared with the reference's own run of that graph (tests/golden/mul_mat_goldens.npz). With the
SIMT kernel the whole step is bit-identical to the reference; with the tensor-core kernel it is
within the normwise 1e-5 bar."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import normwise

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def tc():
    import trc_cuda

    trc_cuda.lib()
    return trc_cuda


def dev(x):
    return torch.from_numpy(np.ascontiguousarray(x)).cuda()


def run_step(tc, a_np, b_np, g_np, simt):
    A, B, G = dev(a_np), dev(b_np), dev(g_np)
    D = tc.mul_mat(A, B, simt=simt)
    M = tc.mul(D, G)
    L = tc.sum(M)
    one = torch.ones(1, device="cuda")
    R = tc.repeat(one, tc.ggml_ne(M))
    dD = tc.mul(R, G)
    ga = torch.zeros_like(A)
    gb = torch.zeros_like(B)
    dA_pre = tc.mul_mat(dD.transpose(-1, -2), B.transpose(-1, -2), simt=simt)  # [k? ] -> ne [ne1(B)...]
    dA_t = dA_pre.transpose(-1, -2)
    ane = tc.ggml_ne(A)
    if tc.ggml_ne(dA_t)[2:] != ane[2:]:
        dA = tc.repeat_back(dA_t, ane)
    else:
        dA = tc.cont(dA_t)
    tc.acc_(ga, dA, dA.stride(-2) * 4 if dA.dim() > 1 else dA.numel() * 4,
            (dA.stride(-3) if dA.dim() > 2 else dA.numel()) * 4,
            (dA.stride(-4) if dA.dim() > 3 else dA.numel()) * 4, 0)
    dB = tc.mul_mat(A.transpose(-1, -2), dD, simt=simt)
    tc.acc_(gb, dB.reshape(B.shape), B.stride(-2) * 4 if B.dim() > 1 else B.numel() * 4,
            (B.stride(-3) if B.dim() > 2 else B.numel()) * 4, (B.stride(-4) if B.dim() > 3 else B.numel()) * 4, 0)
    torch.cuda.synchronize()
    return D.cpu().numpy(), ga.cpu().numpy(), gb.cpu().numpy(), L.item()


@pytest.mark.parametrize("name", ["step_linear", "step_gqa", "step_ragged"])
def test_step_simt_bit_exact(tc, goldens, name):
    m = goldens["mul_mat"]
    d, da, db, _ = run_step(tc, m[name + "_a"], m[name + "_b"], m[name + "_g"], simt=True)
    for got, key in ((d, "_d"), (da, "_da"), (db, "_db")):
        want = m[name + key]
        assert np.array_equal(got.reshape(want.shape).view(np.uint32), want.view(np.uint32)), key


@pytest.mark.parametrize("name", ["step_linear", "step_gqa", "step_ragged"])
def test_step_tensor_core_within_tolerance(tc, goldens, name):
    m = goldens["mul_mat"]
    d, da, db, _ = run_step(tc, m[name + "_a"], m[name + "_b"], m[name + "_g"], simt=False)
    for got, key in ((d, "_d"), (da, "_da"), (db, "_db")):
        want = m[name + key]
        assert normwise(got.reshape(want.shape), want) <= 1e-5, key
    assert tc.device_error() == 0
