"""GPU parity: ggml mul_mat on the tcgen05 3xTF32 kernel (normwise <= 1e-5 against the reference)
and on the SIMT kernel (bit-exact against the reference), over the reference's conformance shapes,
its golden arrays, transposed views, modulo broadcasting, ragged tiles and config-size slices."""
from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
from conftest import normwise

pytestmark = pytest.mark.gpu

TOL = 1e-5  # normwise: max|gpu - cpu| / max|cpu| (north-star accuracy bar)


@pytest.fixture(scope="module")
def tc():
    import trc_cuda

    trc_cuda.lib()
    return trc_cuda


def dev(x):
    return torch.from_numpy(np.ascontiguousarray(x)).cuda()


def op(x, t):
    return x.transpose(-1, -2) if t else x


def npop(x, t):
    return np.swapaxes(x, -1, -2) if t else x


CONFORMANCE = {
    "basic": ((3, 5), False, (4, 5), False),
    "transposed_a": ((5, 3), True, (4, 5), False),
    "transposed_b": ((3, 5), False, (5, 4), True),
    "tile_boundary": ((70, 33), False, (66, 33), False),
    "batch": ((1, 1, 3, 5), False, (3, 2, 4, 5), False),
    "batch_bcast_div": ((1, 2, 3, 5), False, (1, 4, 4, 5), False),
    "batch_transposed": ((2, 2, 5, 3), True, (2, 2, 5, 4), True),
    "batch_tile_boundary": ((1, 1, 70, 33), False, (2, 2, 66, 33), False),
    "grid_z_65_planes": ((1, 1, 4, 8), False, (1, 65, 4, 8), False),
}


@pytest.mark.parametrize("simt", [False, True], ids=["auto", "simt"])
@pytest.mark.parametrize("case", list(CONFORMANCE))
def test_conformance_shapes(tc, case, simt):
    """The reference backend conformance cases (test_backend_conformance.cpp:455-553, 927-934)."""
    sa, ta, sb, tb = CONFORMANCE[case]
    rng = np.random.default_rng(1)
    a = rng.standard_normal(sa).astype(np.float32)
    b = rng.standard_normal(sb).astype(np.float32)
    want = oracle.mul_mat(npop(a, ta), npop(b, tb))
    got = tc.mul_mat(op(dev(a), ta), op(dev(b), tb), simt=simt).cpu().numpy()
    assert got.shape == want.shape
    if simt or tc.mul_mat_kernel(op(dev(a), ta), op(dev(b), tb), dev(want)) == tc.KERNEL_SIMT:
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
    else:
        assert normwise(got, want) <= TOL


@pytest.mark.parametrize("stem", ["mul_mat", "mul_mat_batch", "mul_mat_batch_bcast_div", "mul_mat_batch_tile"])
def test_reference_goldens(tc, goldens, stem):
    g = goldens["reference"]
    got = tc.mul_mat(dev(g[stem + "_in0"]), dev(g[stem + "_in1"])).cpu().numpy()
    want = g[stem + "_out"]
    assert np.all(np.abs(got - want) <= 1e-4 + 1e-3 * np.abs(want))


TC_CASES = ["fwd_basic", "fwd_ta", "fwd_tb", "fwd_tab", "fwd_odd", "fwd_bcast", "fwd_bcast_t"]


@pytest.mark.parametrize("name", TC_CASES)
def test_tensor_core_path_against_reference_fixture(tc, goldens, name):
    """Shapes with 16-byte-aligned strides run on the tcgen05 kernel: K-major and MN-major
    operands, ragged M/N/K tiles, broadcast planes."""
    m = goldens["mul_mat"]
    a, b = m[name + "_a"], m[name + "_b"]
    ta, tb = bool(m[name + "_ta"]), bool(m[name + "_tb"])
    want = m[name + "_d"]
    A, B = op(dev(a), ta), op(dev(b), tb)
    out = torch.empty(want.shape, dtype=torch.float32, device="cuda")
    kernel = tc.mul_mat_kernel(A, B, out)
    if name != "fwd_odd":
        assert kernel == tc.KERNEL_TCGEN05
    tc.mul_mat(A, B, out=out)
    assert normwise(out.cpu().numpy(), want) <= TOL
    assert tc.device_error() == 0


def test_accumulate_flag(tc):
    rng = np.random.default_rng(4)
    a = rng.standard_normal((96, 64)).astype(np.float32)
    b = rng.standard_normal((80, 64)).astype(np.float32)
    c = rng.standard_normal((80, 96)).astype(np.float32)
    want = oracle.mul_mat(a, b) + c
    out = dev(c)
    tc.mul_mat(dev(a), dev(b), out=out, accumulate=True)
    assert normwise(out.cpu().numpy(), want) <= TOL


def test_transposed_output_view(tc):
    """Output written through a transposed view (D contiguous along ne1): the kernel swaps operand
    roles so stores stay coalesced."""
    rng = np.random.default_rng(6)
    a = rng.standard_normal((300, 128)).astype(np.float32)
    b = rng.standard_normal((200, 128)).astype(np.float32)
    want = oracle.mul_mat(a, b)  # [m=300, n=200] -> numpy (200, 300)
    base = torch.empty((300, 200), dtype=torch.float32, device="cuda")
    out = base.t()  # ggml ne [300, 200] with nb0 = 800 B, nb1 = 4 B
    assert tc.mul_mat_kernel(dev(a), dev(b), out) == tc.KERNEL_TCGEN05
    tc.mul_mat(dev(a), dev(b), out=out)
    assert normwise(out.cpu().numpy(), want) <= TOL


@pytest.mark.parametrize("simt", [False, True], ids=["tcgen05", "simt"])
@pytest.mark.parametrize("k,m,n,b2,b3", [(128, 512, 512, 4, 2), (512, 2048, 2048, 4, 2)], ids=["default", "full"])
def test_stress_matmul_batch_known_answer(tc, simt, k, m, n, b2, b3):
    """The reference's batch-matmul stress case (tests/test_stress.cpp:415-480, both tiers): A has
    2 x 2 planes filled with 1, 2, 4, 8, B is 0.25 everywhere, so D[.., i2, i3] is exactly
    k * a[i2 % 2 + 2 (i3 % 2)] * 0.25. The reference checks 3 points per plane within 1e-3; every
    element is checked for equality here (the operands have no TF32 tails)."""
    av = torch.tensor([1.0, 2.0, 4.0, 8.0], device="cuda")
    A = av.view(2, 2, 1, 1).expand(2, 2, m, k).contiguous()   # torch (i3, i2, m, k): plane i2 + 2 i3
    B = torch.full((b3, b2, n, k), 0.25, device="cuda")
    D = tc.mul_mat(A, B, simt=simt)
    assert tuple(D.shape) == (b3, b2, n, m)
    i2 = torch.arange(b2, device="cuda").view(1, b2)
    i3 = torch.arange(b3, device="cuda").view(b3, 1)
    want = (k * av[(i2 % 2) + (i3 % 2) * 2] * 0.25).view(b3, b2, 1, 1).expand(b3, b2, n, m)
    assert torch.equal(D, want)
    assert tc.device_error() == 0


@pytest.mark.parametrize("k,m,n", [(4096, 4096, 64), (128, 2048, 96), (2048, 640, 72), (14336, 256, 16)])
def test_config_shaped_slices(tc, k, m, n):
    """Slices of the Linear / GQA / backward GEMMs at their true K, against the oracle."""
    rng = np.random.default_rng(k + m + n)
    a = rng.standard_normal((m, k)).astype(np.float32)
    b = rng.standard_normal((n, k)).astype(np.float32)
    want = oracle.mul_mat(a, b)
    got = tc.mul_mat(dev(a), dev(b)).cpu().numpy()
    assert normwise(got, want) <= TOL
    # the same product through transposed (MN-major) views of both operands
    at, bt = np.ascontiguousarray(a.T), np.ascontiguousarray(b.T)
    got_t = tc.mul_mat(dev(at).t(), dev(bt).t()).cpu().numpy()
    assert normwise(got_t, want) <= TOL


def test_full_size_linear_forward_vs_fp64(tc):
    """Y = W X at the fused Linear workload's full size (K=4096, M=14336, N=2048), normwise
    against a float64 product on the GPU (size-independent accuracy property). Measured: ~2.3e-6
    at every K from 256 to 14336 (the reference CPU's own error against exact is 2.4e-6 at
    K=4096 and 4.4e-6 at K=14336), so the bar here is 5e-6."""
    g = torch.Generator(device="cuda").manual_seed(0)
    W = torch.randn((14336, 4096), generator=g, device="cuda") * 0.005
    X = torch.randn((2048, 4096), generator=g, device="cuda")
    Y = tc.mul_mat(W, X)
    ref64 = (X.double() @ W.double().t())
    err = ((Y.double() - ref64).abs().max() / ref64.abs().max()).item()
    assert err <= 5e-6, err


@pytest.mark.parametrize("simt", [True, False], ids=["simt", "tcgen05"])
@pytest.mark.parametrize("transposed_out,accumulate", [(False, False), (True, False), (True, True)])
def test_mul_mat_repeat_back(tc, simt, transposed_out, accumulate):
    """d = repeat_back(mul_mat(a, b)) in one kernel: the broadcast-operand dA of the composed
    backward. SIMT is bit-exact with the reference's mul_mat + repeat_back; tcgen05 within 1e-5."""
    rng = np.random.default_rng(21)
    G = rng.standard_normal((2, 8, 40, 48)).astype(np.float32)      # ggml [48, 40, 8, 2]: dL/dD
    B = rng.standard_normal((2, 8, 40, 128)).astype(np.float32)     # ggml [128, 40, 8, 2]
    a_t, b_t = np.swapaxes(G, -1, -2), np.swapaxes(B, -1, -2)       # T(G) [40, 48, ..], T(B) [40, 128, ..]
    prod = oracle.mul_mat(a_t, b_t)                                  # [48, 128, 8, 2] -> numpy (2, 8, 128, 48)
    want = oracle.repeat_back(prod, [48, 128, 2, 2])                 # planes i2 % 2
    base = rng.standard_normal((2, 2, 48, 128)).astype(np.float32) if transposed_out else None
    if transposed_out:
        # write through the transposed view of a [128, 48, 2, 2] tensor (grad_acc of A)
        out_t = dev(base)
        out = out_t.transpose(-1, -2)
        if accumulate:
            want = want + np.swapaxes(base, -1, -2)
        else:
            out_t.zero_()
    else:
        out = torch.zeros((2, 2, 128, 48), device="cuda")
    tc.mul_mat_repeat_back(dev(G).transpose(-1, -2), dev(B).transpose(-1, -2), out, accumulate=accumulate, simt=simt)
    got = out.cpu().numpy()
    if simt and not accumulate:
        assert np.array_equal(np.ascontiguousarray(got).view(np.uint32), np.ascontiguousarray(want).view(np.uint32))
    else:
        assert normwise(np.ascontiguousarray(got), np.ascontiguousarray(want)) <= 1e-5
    assert tc.device_error() == 0


# ---- CTA pairs (tcgen05 cta_group::2) against one CTA per tile and the reference

PAIR_SHAPES = [
    # (K, M, N, a_transposed, b_transposed, planes): M > 128 takes the CTA-pair kernel by default
    (332, 300, 520, False, False, (1, 1)),    # ragged in every dimension, second CTA's rows partly out
    (256, 129, 257, False, False, (1, 1)),    # the pair's second CTA holds one row
    (300, 260, 72, True, True, (1, 1)),       # both operands MN-major (the dW layout)
    (520, 384, 300, True, False, (2, 3)),     # MN-major A, planes
    (4096, 512, 512, False, False, (1, 1)),   # several promotion chunks
]


@pytest.mark.parametrize("k,m,n,ta,tb,planes", PAIR_SHAPES)
def test_cta_pair_matches_single_cta_and_reference(tc, k, m, n, ta, tb, planes):
    rng = np.random.default_rng(k + m + n)
    p2, p3 = planes
    a = rng.standard_normal((p3, p2, m, k) if not ta else (p3, p2, k, m)).astype(np.float32)
    b = rng.standard_normal((p3, p2, n, k) if not tb else (p3, p2, k, n)).astype(np.float32)
    want = oracle.mul_mat(npop(a, ta), npop(b, tb))
    A, B = op(dev(a), ta), op(dev(b), tb)
    assert tc.mul_mat_kernel(A, B, tc.ggml_empty(tc.mul_mat_out_ne(A, B))) == tc.KERNEL_TCGEN05
    pair = tc.mul_mat(A, B).cpu().numpy()
    single = tc.mul_mat(A, B, one_cta=True).cpu().numpy()
    assert tc.device_error() == 0
    assert normwise(pair, want) <= TOL, normwise(pair, want)
    assert normwise(single, want) <= TOL, normwise(single, want)
    # same tiles' K order and promotion chunks: the two kernels agree to the last bits or close to it
    assert normwise(pair, single) <= 1e-6


@pytest.mark.parametrize("accumulate", [False, True])
def test_cta_pair_transposed_output_accumulate_and_plane_reduction(tc, accumulate):
    """dA of a broadcast product through a transposed output view with ACCUMULATE (the GQA
    backward shape, reduced), pair vs single CTA."""
    rng = np.random.default_rng(7)
    G = rng.standard_normal((2, 4, 300, 272)).astype(np.float32)      # ne [272, 300, 4, 2]
    Bm = rng.standard_normal((2, 4, 300, 136)).astype(np.float32)     # ne [136, 300, 4, 2]
    base = rng.standard_normal((2, 2, 272, 136)).astype(np.float32)   # dA, ne [136, 272, 2, 2]
    outs = []
    for one in (False, True):
        dA = dev(base.copy())
        # T(dA) (ne [272, 136, 2, 2]) (+)= repeat_back(mul_mat(T(G), T(B)))
        tc.mul_mat_repeat_back(dev(G).transpose(-1, -2), dev(Bm).transpose(-1, -2), dA.transpose(-1, -2),
                               accumulate=accumulate, one_cta=one)
        outs.append(dA.cpu().numpy())
    prod = oracle.mul_mat(np.swapaxes(G, -1, -2), np.swapaxes(Bm, -1, -2))   # numpy [2, 4, 136, 272]
    red = oracle.repeat_back(prod, [272, 136, 2, 2])                         # numpy [2, 2, 136, 272]
    want = np.swapaxes(red, -1, -2) + (base if accumulate else np.float32(0))
    for got in outs:
        assert normwise(got, want) <= TOL, normwise(got, want)
    assert normwise(outs[0], outs[1]) <= 1e-6
    assert tc.device_error() == 0


# ---- split-K (few tiles, long reductions): two CTAs per tile reduce-add into a zeroed D

# (1024, 1536, 1280): 30 pair tiles (60 single tiles) of 64 k-blocks, which stream runs would cut
# into five pieces: two parts, one wave
@pytest.mark.parametrize("k,m,n,one", [(8192, 128, 512, False), (4096, 256, 256, False), (4096, 256, 256, True),
                                       (1024, 1536, 1280, False), (1024, 1536, 1280, True)])
def test_split_k_few_tiles(tc, k, m, n, one):
    rng = np.random.default_rng(k + m + n)
    a = rng.standard_normal((m, k)).astype(np.float32)
    b = rng.standard_normal((n, k)).astype(np.float32)
    want = oracle.mul_mat(a, b)
    A, B = dev(a), dev(b)
    out = tc.ggml_empty(tc.mul_mat_out_ne(A, B))
    out.fill_(float("nan"))  # the kernel zeroes D itself before the split parts are added
    got = tc.mul_mat(A, B, out=out, one_cta=one).cpu().numpy()
    again = tc.mul_mat(A, B, one_cta=one).cpu().numpy()
    assert tc.device_error() == 0
    assert normwise(got, want) <= TOL, normwise(got, want)
    assert np.array_equal(got.view(np.uint32), again.view(np.uint32))  # deterministic


def _split_case(tc, k, m, n, one, seed, launches):
    """One split product: a (m, k) . b (n, k), D pre-filled with NaN (the plan zeroes what it
    reduces into), the launch count of the library's own kernels, the whole result against float64,
    64 columns against the oracle, and a second run bit-identical (the parts' order of arrival does
    not change the sum)."""
    rng = np.random.default_rng(seed)
    a = rng.standard_normal((m, k)).astype(np.float32)
    b = rng.standard_normal((n, k)).astype(np.float32)
    A, B = dev(a), dev(b)
    out = tc.ggml_empty(tc.mul_mat_out_ne(A, B))
    out.fill_(float("nan"))
    torch.cuda.synchronize()
    n0 = tc.launch_count()
    got = tc.mul_mat(A, B, out=out, one_cta=one)
    assert tc.launch_count() - n0 == launches
    want64 = (B.double() @ A.double().t()).cpu().numpy()
    got = got.cpu().numpy()
    again = tc.mul_mat(A, B, one_cta=one).cpu().numpy()
    assert tc.device_error() == 0
    assert normwise(got.reshape(want64.shape), want64) <= 5e-6
    want = oracle.mul_mat(a, b[:64])[0, 0]
    assert normwise(got.reshape(n, m)[:64], want) <= TOL
    assert np.array_equal(got.view(np.uint32), again.view(np.uint32))


@pytest.mark.parametrize("one", [False, True], ids=["pair", "one_cta"])
def test_split_k_four_parts(tc, one):
    """16 pair tiles (or 32 single tiles) of 1024 k-blocks: a stream plan would cut a tile into six
    pieces, so the planner takes four parts (one wave of quarter-length units). Parts 0 and 1 reduce
    into D, parts 2 and 3 into a workspace that one more kernel adds into D."""
    _split_case(tc, 16384, 1024, 1024, one, 75, launches=2)  # the GEMM and the workspace add


@pytest.mark.parametrize("one", [False, True], ids=["pair", "one_cta"])
def test_stream_k_last_wave(tc, one):
    """75 pair tiles on 74 pairs (or 150 tiles on 148 SMs) of 256 k-blocks: two waves unsplit; the
    stream plan deals the 75 x 16 k-chunks to the slots in equal runs of 16-17 chunks, so a tile is
    cut into at most two pieces, both reduce-added into the zeroed D (one launch)."""
    k, m, n = 4096, (3840 if not one else 1280), (1280 if not one else 3840)
    _split_case(tc, k, m, n, one, 76, launches=1)


@pytest.mark.parametrize("one", [False, True], ids=["pair", "one_cta"])
def test_stream_k_workspace(tc, one):
    """32 pair tiles on 74 pairs (or 64 tiles on 148 SMs) of 512 k-blocks (the GQA dA kind of
    shape): runs of 13-14 chunks cut a tile of 32 chunks into up to four pieces; the first two
    reduce into D, the third and fourth into the workspace added afterwards (two launches)."""
    m, n = (2048, 1024) if not one else (1024, 2048)
    _split_case(tc, 8192, m, n, one, 77, launches=2)


@pytest.mark.parametrize("one", [False, True], ids=["pair", "one_cta"])
def test_stream_k_after_whole_waves(tc, one):
    """448 pair tiles on 74 pairs of 64 k-blocks (the Linear forward's tile count; 896 single tiles
    on 148 SMs): five round-robin waves of whole tiles, stored, then the last 78 (or 156) tiles dealt
    in chunk runs of about four chunks."""
    _split_case(tc, 1024, 14336, 2048, one, 78, launches=1)


# Shapes around the last partial wave, where the planner takes stream plans: ragged M, N and K
# (edge tiles, a partial last k-chunk), broadcast planes, MN-major operands, both tile shapes, and
# a plan that cuts tiles into up to four pieces (pieces 3-4 in the workspace) or four parts.
# (M, N, K, one_cta, (a2, a3), (b2, b3), A MN-major, B MN-major)
SPLIT_SWEEP = [
    (2560, 1900, 1536, False, (1, 1), (1, 1), False, False),  # 80 pair tiles, ragged N
    (2300, 2300, 1024, False, (1, 1), (1, 1), True, False),   # 81 pair tiles, ragged M and N, MN-major A
    (1280, 3800, 2048, True, (1, 1), (1, 1), False, True),    # 150 single tiles, MN-major B
    (1000, 1024, 4096, True, (2, 1), (4, 2), False, False),   # 256 single tiles over 8 broadcast planes
    (512, 1536, 3072, False, (2, 2), (4, 2), False, False),   # 96 pair tiles over 8 planes
    (4096, 2600, 640, False, (1, 1), (1, 1), True, True),     # 176 pair tiles of 3 chunks, both MN-major
    (2400, 2048, 1000, False, (1, 1), (1, 1), False, False),  # K = 1000: a partial last k-block
    (1000, 2000, 8192, True, (1, 1), (1, 1), False, False),   # 64 single tiles cut into up to 4 pieces
    (300, 2048, 8192, True, (1, 1), (1, 1), False, False),    # 24 single tiles: four parts
]


@pytest.mark.parametrize("m,n,k,one,ap,bp,ta,tb", SPLIT_SWEEP)
def test_split_plans_sweep(tc, m, n, k, one, ap, bp, ta, tb):
    """Every plan the planner takes on these shapes gives the product within the float64 bar and
    the same bits on a second run. D starts as NaN: every element must be written."""
    g = torch.Generator(device="cuda").manual_seed(m + n + k)
    a2, a3 = ap
    b2, b3 = bp
    a_store = torch.randn((a3, a2, k, m) if ta else (a3, a2, m, k), generator=g, device="cuda")
    b_store = torch.randn((b3, b2, k, n) if tb else (b3, b2, n, k), generator=g, device="cuda")
    A, B = op(a_store, ta), op(b_store, tb)                                # logical (.., rows, K)
    out = torch.full((b3, b2, n, m), float("nan"), device="cuda")
    got = tc.mul_mat(A, B, out=out, one_cta=one).clone()
    again = tc.mul_mat(A, B, out=out, one_cta=one)
    assert tc.device_error() == 0
    Ar = A.double().repeat(b3 // a3, b2 // a2, 1, 1)
    want = B.double() @ Ar.transpose(-1, -2)                               # (b3, b2, n, m)
    assert ((got.double() - want).abs().max() / want.abs().max()).item() <= 5e-6
    assert torch.equal(got.view(torch.int32), again.view(torch.int32))


def test_split_k_plane_reduction_one_plane_group(tc):
    """The GQA dA product at one ne[3] plane per rank (the 8-GPU shape, reduced in size): M = 128
    after the orientation swap, few tiles, K = 2048 x 4 source planes."""
    rng = np.random.default_rng(11)
    G = rng.standard_normal((1, 8, 1024, 512)).astype(np.float32)     # ne [512, 1024, 8, 1]
    Bm = rng.standard_normal((1, 8, 1024, 128)).astype(np.float32)    # ne [128, 1024, 8, 1]
    dA = torch.full((1, 2, 512, 128), float("nan"), device="cuda")     # ne [128, 512, 2, 1]
    tc.mul_mat_repeat_back(dev(G).transpose(-1, -2), dev(Bm).transpose(-1, -2), dA.transpose(-1, -2))
    prod = oracle.mul_mat(np.swapaxes(G, -1, -2), np.swapaxes(Bm, -1, -2))   # numpy [1, 8, 128, 512]
    want = np.swapaxes(oracle.repeat_back(prod, [512, 128, 2, 1]), -1, -2)
    assert tc.device_error() == 0
    assert normwise(dA.cpu().numpy(), want) <= TOL


# ---- B's tails computed once before the launch vs inside every tile: the same values, bit for bit
# (the fused kernel takes the precomputed tails; for the F32 kernel the flag must change nothing)

@pytest.mark.parametrize("k,m,n,ta,tb,planes,one", [
    (332, 300, 520, False, False, (1, 1), False),
    (300, 260, 72, True, True, (1, 1), False),      # MN-major B through the 5-D map
    (520, 384, 300, True, False, (2, 3), False),    # planes
    (520, 384, 300, False, True, (2, 1), True),     # one CTA per tile
    (256, 512, 100, False, True, (1, 1), False),    # MN-major B of 100 rows: per-chunk loads, padded rows
])
def test_pretail_bit_identical(tc, k, m, n, ta, tb, planes, one):
    rng = np.random.default_rng(k * 7 + n)
    p2, p3 = planes
    a = rng.standard_normal((p3, p2, m, k) if not ta else (p3, p2, k, m)).astype(np.float32)
    b = rng.standard_normal((p3, p2, n, k) if not tb else (p3, p2, k, n)).astype(np.float32)
    A, B = op(dev(a), ta), op(dev(b), tb)
    got = tc.mul_mat(A, B, one_cta=one).cpu().numpy()
    base = tc.mul_mat(A, B, one_cta=one, no_pretail=True).cpu().numpy()
    assert tc.device_error() == 0
    assert np.array_equal(got.view(np.uint32), base.view(np.uint32))
    assert normwise(got, oracle.mul_mat(npop(a, ta), npop(b, tb))) <= TOL


@pytest.mark.parametrize("transposed,b_mn,one,n", [(False, False, False, 264), (True, False, False, 264),
                                                   (False, True, False, 96), (True, True, True, 100),
                                                   (False, False, True, 72)])
def test_pretail_bit_identical_fused(tc, transposed, b_mn, one, n):
    """The fused kernel with B's tails precomputed vs split in every tile: K-major and MN-major B
    (a transposed view; 100 rows takes the per-chunk loads and padded tail rows), pair and one CTA."""
    import synth

    w_ne0, w_ne1 = 1024, 520
    blocks = dev(synth.random_blocks(synth.TYPE_Q5_0, w_ne0 * w_ne1 // 32, seed=9))
    k = w_ne1 if transposed else w_ne0
    xn = np.random.default_rng(3).standard_normal((n, k)).astype(np.float32)
    x = dev(np.ascontiguousarray(xn.T)).t() if b_mn else dev(xn)  # same values, contiguous along n
    got = tc.mul_mat_q(synth.TYPE_Q5_0, blocks, w_ne0, w_ne1, x, transposed=transposed, one_cta=one,
                       fused=True).cpu().numpy()
    base = tc.mul_mat_q(synth.TYPE_Q5_0, blocks, w_ne0, w_ne1, x, transposed=transposed, one_cta=one, fused=True,
                        no_pretail=True).cpu().numpy()
    assert tc.device_error() == 0
    assert np.array_equal(got.view(np.uint32), base.view(np.uint32))
    Wf = oracle.dequant(synth.TYPE_Q5_0, blocks.cpu().numpy()).reshape(w_ne1, w_ne0)
    want = oracle.mul_mat(np.swapaxes(Wf, -1, -2) if transposed else Wf, xn)
    assert normwise(got, want) <= TOL
