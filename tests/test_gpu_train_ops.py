"""GPU parity of the training-step ops (unaries, sum_rows / mean, AdamW, SGD, grad-norm clip)
against the oracle: bit for bit, on random data and edge values; sum_sqr_acc within one float ulp
(its double sum is taken in a parallel order)."""
from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle

pytestmark = pytest.mark.gpu

EDGE = np.array([0.0, -0.0, 1.0, -1.0, np.inf, -np.inf, np.nan, 1e-45, -1e-45, 1.17e-38, 3.4e38, -3.4e38,
                 1e-20, 65504.0, 0.5, 2.0], dtype=np.float32)


@pytest.fixture(scope="module")
def tc():
    import trc_cuda

    trc_cuda.lib()
    return trc_cuda


def dev(x):
    return torch.from_numpy(np.ascontiguousarray(x)).cuda()


def same(a, b):
    a, b = np.asarray(a, dtype=np.float32), np.asarray(b, dtype=np.float32)
    nan = np.isnan(b)
    return bool(np.array_equal(np.isnan(a), nan) and np.array_equal(a.view(np.uint32)[~nan], b.view(np.uint32)[~nan]))


def sample(n, seed, scale=1.0):
    x = (np.random.default_rng(seed).standard_normal(n) * scale).astype(np.float32)
    x[: EDGE.size] = EDGE
    return x


@pytest.mark.parametrize("op", range(7), ids=["sqr", "sqrt", "abs", "neg", "sgn", "step", "scale"])
@pytest.mark.parametrize("strided", [False, True])
def test_unary(tc, op, strided):
    x = sample(64 * 96, op).reshape(64, 96)
    src = dev(x).t() if strided else dev(x)  # a transposed view exercises the strided kernel
    want = oracle.unary(op, np.ascontiguousarray(x.T) if strided else x, 0.3125)
    got = tc.unary(op, src, param=0.3125).cpu().numpy().reshape(want.shape)
    assert same(got, want)


@pytest.mark.parametrize("take_mean", [False, True])
def test_sum_rows(tc, take_mean):
    x = sample(3 * 5 * 777, 7, 100.0).reshape(3, 5, 777)
    want = oracle.sum_rows(x, take_mean)
    got = tc.sum_rows(dev(x), mean=take_mean).cpu().numpy().reshape(want.shape)
    assert same(got, want)


@pytest.mark.parametrize("step", [1, 1000])
def test_adamw(tc, step):
    n = 1 << 20
    p, g = sample(n, 1), sample(n, 2, 0.1)
    m, v = sample(n, 3, 0.01), np.abs(sample(n, 4, 1e-3))
    lr, b1, b2 = 1e-3, 0.9, 0.999
    ps = [lr / (1 - b1 ** step), np.sqrt(1 - b2 ** step), 1 - lr * 0.01, b1, b2, 1e-8]
    P, G, M, V = dev(p), dev(g), dev(m), dev(v)
    tc.opt_step_adamw_(P, G, M, V, ps)
    wp, wm, wv = oracle.adamw(p, g, m, v, ps)
    assert same(P.cpu().numpy(), wp) and same(M.cpu().numpy(), wm) and same(V.cpu().numpy(), wv)


@pytest.mark.parametrize("ps", [[0.1, 0.0, 0.0, 0.0, 0.0, 1.0], [0.05, 0.9, 0.1, 1e-4, 0.0, 0.0],
                                [0.05, 0.9, 0.0, 1e-4, 1.0, 0.0], [0.05, 0.9, 0.0, 1e-4, 0.0, 1.0]],
                         ids=["plain", "dampening", "nesterov", "first"])
def test_sgd(tc, ps):
    n = 1 << 20
    p, g, mom = sample(n, 5), sample(n, 6, 0.1), sample(n, 7, 0.01)
    P, G, MOM = dev(p), dev(g), dev(mom)
    tc.opt_step_sgd_(P, G, MOM, ps)
    wp, wm = oracle.sgd(p, g, mom, ps)
    assert same(P.cpu().numpy(), wp) and same(MOM.cpu().numpy(), wm)


def test_grad_norm_clip(tc):
    x = sample(3_000_000, 8, 3.0)
    x[: EDGE.size] = 1.0
    acc = torch.tensor([2.5], device="cuda")
    tc.sum_sqr_acc_(acc, dev(x))
    want = oracle.sum_sqr_acc(2.5, x)
    got = acc.cpu().numpy()[0]
    assert abs(int(np.float32(got).view(np.uint32)) - int(np.float32(want).view(np.uint32))) <= 1
    norm = torch.tensor([float(want)], device="cuda")
    for max_norm in (1.0, 1e9):
        X = dev(x)
        tc.clip_scale_(X, norm, max_norm, 1e-6)
        assert same(X.cpu().numpy(), oracle.clip_scale(x, float(want), max_norm, 1e-6))
    assert tc.device_error() == 0
