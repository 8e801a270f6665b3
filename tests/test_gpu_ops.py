"""GPU parity: the graph ops of the composed backward, bit-exact against the oracle (same
per-element arithmetic and, for repeat_back, the same summation order as the reference)."""
from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def tc():
    import trc_cuda

    trc_cuda.lib()
    return trc_cuda


def dev(x):
    return torch.from_numpy(np.ascontiguousarray(x)).cuda()


def beq(a, b):
    return np.array_equal(np.ascontiguousarray(a).view(np.uint32), np.ascontiguousarray(b).view(np.uint32))


@pytest.mark.parametrize("shape", [(33, 70), (4, 3, 130, 66), (1, 1, 4096, 257)])
def test_cont_of_transpose(tc, shape):
    x = np.random.default_rng(0).standard_normal(shape).astype(np.float32)
    got = tc.cont(dev(x).transpose(-1, -2)).cpu().numpy()
    want = oracle.cont(np.swapaxes(x, -1, -2))
    assert beq(got.reshape(want.shape), want)


def test_cont_generic_permute(tc):
    x = np.random.default_rng(1).standard_normal((3, 4, 5, 6)).astype(np.float32)
    v = dev(x).permute(1, 0, 3, 2)
    assert beq(tc.cont(v).cpu().numpy(), oracle.cont(np.transpose(x, (1, 0, 3, 2))))


def test_cont_golden(tc, goldens):
    g = goldens["reference"]
    got = tc.cont(dev(g["transpose_cont_in0"]).transpose(-1, -2)).cpu().numpy()
    assert np.array_equal(got, g["transpose_cont_out"])


def test_acc_inplace_contiguous(tc):
    rng = np.random.default_rng(2)
    dst = rng.standard_normal((4096 + 7,)).astype(np.float32)
    b = rng.standard_normal((4096 + 7,)).astype(np.float32)
    want = oracle.acc_(dst.copy(), b, b.nbytes, b.nbytes, b.nbytes, 0)
    d = dev(dst)
    tc.acc_(d, dev(b), b.nbytes, b.nbytes, b.nbytes, 0)
    assert beq(d.cpu().numpy(), want)


def test_acc_inplace_strided_region(tc):
    rng = np.random.default_rng(3)
    dst = rng.standard_normal((5, 7, 9)).astype(np.float32)
    b = rng.standard_normal((2, 3, 4)).astype(np.float32)
    nb1, nb2, off = 9 * 4, 7 * 9 * 4, (1 * 63 + 2 * 9 + 3) * 4
    want = oracle.acc_(dst.copy(), b, nb1, nb2, nb2 * 5, off)
    d = dev(dst)
    tc.acc_(d, dev(b), nb1, nb2, nb2 * 5, off)
    assert beq(d.cpu().numpy(), want)


def test_acc_rejects_out_of_bounds_region(tc):
    d = torch.zeros(10, device="cuda")
    b = torch.ones(4, device="cuda")
    with pytest.raises(tc.TrcCudaError):
        tc.acc_(d, b, 16, 16, 16, 8 * 4)


@pytest.mark.parametrize("src_shape,dst_ne", [((8, 32, 48, 16), [16, 48, 8, 8]),  # GQA: sum 4 planes
                                              ((2, 6, 10, 12), [6, 5, 3, 1]),
                                              ((1, 1, 3, 4096), [4096, 1, 1, 1])])
def test_repeat_back(tc, src_shape, dst_ne):
    x = np.random.default_rng(4).standard_normal(src_shape).astype(np.float32)
    got = tc.repeat_back(dev(x), dst_ne).cpu().numpy()
    assert beq(got, oracle.repeat_back(x, dst_ne))


def test_repeat_back_of_transposed_view(tc):
    x = np.random.default_rng(5).standard_normal((8, 32, 16, 48)).astype(np.float32)  # [48,16,32,8]
    v = dev(x).transpose(-1, -2)  # ne [16, 48, 32, 8]
    got = tc.repeat_back(v, [16, 48, 8, 8]).cpu().numpy()
    assert beq(got, oracle.repeat_back(np.swapaxes(x, -1, -2), [16, 48, 8, 8]))


def test_repeat_and_golden(tc, goldens):
    g = goldens["reference"]
    x, want = g["repeat_in0"], g["repeat_out"]
    ne = list(want.shape)[::-1]
    assert np.array_equal(tc.repeat(dev(x), ne).cpu().numpy(), want)
    one = torch.ones(1, device="cuda")
    assert torch.equal(tc.repeat(one, [6, 5, 4, 3]), torch.ones((3, 4, 5, 6), device="cuda"))


@pytest.mark.parametrize("opname", ["add", "sub", "mul", "div"])
def test_binary_broadcast(tc, opname):
    rng = np.random.default_rng(6)
    a = rng.standard_normal((3, 4, 5, 6)).astype(np.float32)
    b = rng.standard_normal((1, 4, 1, 6)).astype(np.float32) + 2
    fn = getattr(tc, opname)
    npfn = {"add": np.add, "sub": np.subtract, "mul": np.multiply, "div": np.divide}[opname]
    assert beq(fn(dev(a), dev(b)).cpu().numpy(), npfn(a, b).astype(np.float32))
    c = rng.standard_normal((3, 4, 5, 6)).astype(np.float32) + 3
    assert beq(fn(dev(a), dev(c)).cpu().numpy(), npfn(a, c).astype(np.float32))


def test_sum_double_accumulation(tc):
    x = np.random.default_rng(7).standard_normal((3, 5, 7, 1001)).astype(np.float32)
    got = tc.sum(dev(x)).item()
    want = np.float32(np.sum(x.astype(np.float64)))
    assert abs(got - want) <= 1e-6 * max(1.0, abs(float(want)))
    v = dev(x).transpose(-1, -2)
    assert abs(tc.sum(v).item() - want) <= 1e-6 * max(1.0, abs(float(want)))


def test_fill(tc):
    t = torch.empty(12345, device="cuda")
    tc.fill_(t, 1.5)
    assert torch.all(t == 1.5)
