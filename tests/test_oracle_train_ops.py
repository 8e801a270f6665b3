"""CPU: the oracle's restatements of the training-step ops (unaries, sum_rows / mean, AdamW, SGD,
grad-norm clip) against the reference's own CPU code (oracle/_ref), bit for bit, on random data and
on edge values (signed zeros, infinities, NaN, denormals, huge and tiny magnitudes)."""
from __future__ import annotations

import numpy as np
import pytest

import oracle

pytestmark = pytest.mark.skipif(not oracle.ref_available(), reason="oracle/_ref not built")

EDGE = np.array([0.0, -0.0, 1.0, -1.0, np.inf, -np.inf, np.nan, 1e-45, -1e-45, 1.17e-38, 3.4e38, -3.4e38,
                 1e-20, 65504.0, 0.5, 2.0], dtype=np.float32)


def bits(x):
    return np.asarray(x, dtype=np.float32).view(np.uint32)


def same(a, b):
    a, b = np.asarray(a, dtype=np.float32), np.asarray(b, dtype=np.float32)
    nan = np.isnan(b)
    return bool(np.array_equal(np.isnan(a), nan) and np.array_equal(bits(a)[~nan], bits(b)[~nan]))


def sample(n, seed, scale=1.0):
    rng = np.random.default_rng(seed)
    x = (rng.standard_normal(n) * scale).astype(np.float32)
    x[: EDGE.size] = EDGE
    return x


@pytest.mark.parametrize("op", range(7), ids=["sqr", "sqrt", "abs", "neg", "sgn", "step", "scale"])
def test_unary_matches_reference(op):
    x = sample(4096, op).reshape(2, 2, 32, 32)
    assert same(oracle.unary(op, x, 0.3125), oracle.ref_unary(op, x, 0.3125))


@pytest.mark.parametrize("take_mean", [False, True])
def test_sum_rows_matches_reference(take_mean):
    x = sample(3 * 5 * 777, 7, 100.0).reshape(3, 5, 777)
    assert same(oracle.sum_rows(x, take_mean), oracle.ref_sum_rows(x, take_mean))


def adamw_params(step):
    lr, beta1, beta2, eps, wd = 1e-3, 0.9, 0.999, 1e-8, 0.01
    bc1 = 1.0 - beta1 ** step
    bc2 = 1.0 - beta2 ** step
    return [lr / bc1, np.sqrt(bc2), 1.0 - lr * wd, beta1, beta2, eps]


@pytest.mark.parametrize("step", [1, 2, 1000])
def test_adamw_matches_reference(step):
    n = 5000
    p, g = sample(n, 1), sample(n, 2, 0.1)
    m, v = sample(n, 3, 0.01), np.abs(sample(n, 4, 1e-3))
    ps = adamw_params(step)
    for a, b in zip(oracle.adamw(p, g, m, v, ps), oracle.ref_adamw(p, g, m, v, ps)):
        assert same(a, b)


@pytest.mark.parametrize("ps", [
    [0.1, 0.0, 0.0, 0.0, 0.0, 1.0],        # plain SGD
    [0.05, 0.9, 0.0, 1e-4, 0.0, 1.0],      # momentum, first step
    [0.05, 0.9, 0.1, 1e-4, 0.0, 0.0],      # momentum with dampening
    [0.05, 0.9, 0.0, 1e-4, 1.0, 0.0],      # nesterov
], ids=["plain", "first", "dampening", "nesterov"])
def test_sgd_matches_reference(ps):
    n = 5000
    p, g, mom = sample(n, 5), sample(n, 6, 0.1), sample(n, 7, 0.01)
    for a, b in zip(oracle.sgd(p, g, mom, ps), oracle.ref_sgd(p, g, mom, ps)):
        assert same(a, b)


def test_grad_norm_clip_matches_reference():
    x = sample(100000, 8, 3.0)
    x[: EDGE.size] = 1.0  # a finite norm
    assert same(oracle.sum_sqr_acc(2.5, x), oracle.ref_sum_sqr_acc(2.5, x))
    norm = float(oracle.sum_sqr_acc(0.0, x))
    for max_norm in (1.0, 1e9):  # scaled down, and clamped to 1
        assert same(oracle.clip_scale(x, norm, max_norm, 1e-6), oracle.ref_clip_scale(x, norm, max_norm, 1e-6))
