"""CPU: pins the C restatement (oracle/trc_oracle.c) against the reference's own known answers,
its golden arrays, and the reference compiled from its sources (oracle/_ref), bit for bit."""
from __future__ import annotations

import numpy as np
import pytest

import oracle
import synth
from conftest import normwise

TYPES = [synth.TYPE_Q4_0, synth.TYPE_Q4_1, synth.TYPE_Q5_0, synth.TYPE_Q5_1, synth.TYPE_Q8_0]
NAMES = {v: k for k, v in synth.TYPE_BY_NAME.items()}


def test_fp16_decode_all_inputs_match_reference(ref):
    L = oracle.oracle_lib()
    got = np.array([L.oracle_fp16_to_fp32(h) for h in range(65536)], dtype=np.float32).view(np.uint32)
    want = np.array([ref.ref_fp16_to_fp32_bits(h) for h in range(65536)], dtype=np.uint32)
    assert np.array_equal(got, want)


def test_fp16_decode_matches_ieee():
    L = oracle.oracle_lib()
    h = np.arange(65536, dtype=np.uint16)
    got = np.array([L.oracle_fp16_to_fp32(int(x)) for x in h], dtype=np.float32)
    want = h.view(np.float16).astype(np.float32)
    finite = np.isfinite(want)
    assert np.array_equal(got[finite], want[finite])
    assert np.array_equal(np.isnan(got), np.isnan(want))


def test_fp16_encode_matches_reference(ref):
    L = oracle.oracle_lib()
    rng = np.random.default_rng(5)
    xs = np.concatenate([
        rng.uniform(-70000, 70000, 2000), rng.uniform(-1e-2, 1e-2, 2000), rng.uniform(-1e-6, 1e-6, 2000),
        np.float32([0.0, -0.0, 65504, 65519.99, 65520, 6.1e-5, 5.96e-8, 2.98e-8, 1e-3, 1e-2, np.inf, -np.inf]),
    ]).astype(np.float32)
    for x in xs:
        assert L.oracle_fp32_to_fp16(float(x)) == ref.ref_lib().ref_fp32_to_fp16(float(x)), x
    # and numpy's IEEE round-to-nearest-even (the generator's rounding)
    np_bits = xs.astype(np.float16).view(np.uint16)
    ours = np.array([L.oracle_fp32_to_fp16(float(x)) for x in xs], dtype=np.uint16)
    assert np.array_equal(ours, np_bits)


@pytest.mark.parametrize("qtype", TYPES, ids=lambda t: NAMES[t])
def test_dequant_known_answers(qtype, goldens):
    """The reference's tests/test_gguf.cpp:355-444 known answers (fixture checked against the
    reference when it was generated)."""
    g = goldens["dequant"]
    name = NAMES[qtype]
    got = oracle.dequant(qtype, g[f"kat_{name}_blocks"])
    assert np.array_equal(got, g[f"kat_{name}_out"])


@pytest.mark.parametrize("qtype", TYPES, ids=lambda t: NAMES[t])
def test_dequant_random_blocks_golden(qtype, goldens):
    g = goldens["dequant"]
    name = NAMES[qtype]
    got = oracle.dequant(qtype, g[f"rand_{name}_blocks"])
    assert np.array_equal(got.view(np.uint32), g[f"rand_{name}_out"].view(np.uint32))


@pytest.mark.parametrize("qtype", TYPES, ids=lambda t: NAMES[t])
def test_dequant_matches_reference_bitwise(qtype, ref):
    blocks = synth.random_blocks(qtype, 4099, seed=99 + qtype)
    # extreme scales too: subnormal, huge, negative, zero
    bb = synth.BLOCK_BYTES[qtype]
    v = blocks.reshape(-1, bb)
    for i, d in enumerate([0x0001, 0x03FF, 0x7BFF, 0x8001, 0xFBFF, 0x0000, 0x8000, 0x3C00]):
        v[i, 0:2] = np.frombuffer(np.uint16(d).tobytes(), dtype=np.uint8)
    got = oracle.dequant(qtype, blocks)
    want = ref.ref_dequant(qtype, blocks, 4099 * 32)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


def test_reference_rejects_ragged_quant_tensor(ref, tmp_path):
    """ne0 = 30 is not a whole number of Q4_0 blocks: the reference refuses the file
    (test_gguf.cpp:609-620); the device entry points refuse such sizes too."""
    p = tmp_path / "bad.gguf"
    synth.write_gguf(p, [("w", synth.TYPE_Q4_0, (30,), bytes(18))])
    assert not ref.ref_lib().ref_gguf_open(str(p).encode())


MM_CASES = {
    # name: (A base shape, transposed?, B base shape, transposed?)   numpy shapes = reversed ggml ne
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


def _op(x, t):
    return np.swapaxes(x, -1, -2) if t else x


@pytest.mark.parametrize("case", list(MM_CASES))
def test_mul_mat_oracle_matches_reference_bitwise(case, ref):
    sa, ta, sb, tb = MM_CASES[case]
    rng = np.random.default_rng(3)
    a = rng.standard_normal(sa).astype(np.float32)
    b = rng.standard_normal(sb).astype(np.float32)
    got = oracle.mul_mat(_op(a, ta), _op(b, tb), n_threads=3)
    want = ref.ref_mul_mat(a, ta, b, tb)
    assert got.shape == want.shape
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


@pytest.mark.parametrize("stem", ["mul_mat", "mul_mat_batch", "mul_mat_batch_bcast_div", "mul_mat_batch_tile"])
def test_mul_mat_oracle_reference_goldens(stem, goldens):
    """The reference's PyTorch goldens (cases.txt:26-29), with its tolerance atol 1e-4 + rtol 1e-3."""
    g = goldens["reference"]
    got = oracle.mul_mat(g[stem + "_in0"], g[stem + "_in1"])
    want = g[stem + "_out"]
    assert got.shape == want.shape
    assert np.all(np.abs(got - want) <= 1e-4 + 1e-3 * np.abs(want))


@pytest.mark.parametrize("stem", ["grad_mul_mat_batch", "grad_mul_mat_batch_div"])
def test_composed_backward_oracle_reference_goldens(stem, goldens):
    """grad_cases.txt: loss = sum(sqr(mul_mat(A, B))), so dL/dD = 2D; the composed backward
    (trc_autograd.cpp:487-503) is dA = repeat_back(T(mul_mat(T(G), T(B)))), dB = mul_mat(T(A), G)."""
    g = goldens["reference"]
    a, b = g[stem + "_in0"], g[stem + "_in1"]
    d = oracle.mul_mat(a, b)
    G = (d + d).astype(np.float32)
    ane = list(a.shape)[::-1] + [1] * (4 - a.ndim)
    da_full = np.swapaxes(oracle.mul_mat(np.swapaxes(G, -1, -2), np.swapaxes(b, -1, -2)), -1, -2)
    da = oracle.repeat_back(np.ascontiguousarray(da_full), ane).reshape(a.shape)
    db = oracle.mul_mat(np.swapaxes(a, -1, -2), G).reshape(b.shape)
    for got, key in ((da, "_grad0"), (db, "_grad1")):
        want = g[stem + key]
        assert np.all(np.abs(got - want) <= 1e-4 + 1e-3 * np.abs(want)), key


def test_repeat_and_transpose_cont_goldens(goldens):
    g = goldens["reference"]
    tc_in = g["transpose_cont_in0"]
    assert np.array_equal(oracle.cont(np.swapaxes(tc_in, -1, -2)), g["transpose_cont_out"])


@pytest.mark.parametrize("name", ["step_linear", "step_gqa", "step_ragged"])
def test_training_step_oracle_matches_reference(name, goldens):
    """Oracle composition of the composed backward vs the reference autograd run (fixture),
    bit-exact: loss = sum(mul(D, G)) injects dL/dD = G * 1.0."""
    m = goldens["mul_mat"]
    a, b, g = m[name + "_a"], m[name + "_b"], m[name + "_g"]
    d = oracle.mul_mat(a, b)
    ane = list(a.shape)[::-1] + [1] * (4 - a.ndim)
    da = np.swapaxes(oracle.mul_mat(np.swapaxes(g, -1, -2), np.swapaxes(b, -1, -2)), -1, -2)
    if a.ndim == 4 and a.shape != b.shape[:2] + a.shape[2:]:
        da = oracle.repeat_back(np.ascontiguousarray(da), ane)
    db = oracle.mul_mat(np.swapaxes(a, -1, -2), g)
    assert np.array_equal(d.reshape(m[name + "_d"].shape).view(np.uint32), m[name + "_d"].view(np.uint32))
    assert np.array_equal(np.ascontiguousarray(da).reshape(a.shape).view(np.uint32), m[name + "_da"].view(np.uint32))
    assert np.array_equal(db.reshape(b.shape).view(np.uint32), m[name + "_db"].view(np.uint32))


def test_acc_oracle_matches_reference_semantics():
    rng = np.random.default_rng(11)
    dst = rng.standard_normal((4, 6)).astype(np.float32)
    b = rng.standard_normal((2, 3)).astype(np.float32)
    want = dst.copy()
    want[1:3, 2:5] += b  # region: offset = (1 row * 6 + 2) * 4 bytes, nb1 = 24
    oracle.acc_(dst, b, 24, 0, 0, (6 + 2) * 4)
    assert np.array_equal(dst, want)


def test_normwise_metric():
    assert normwise(np.float32([1, 2]), np.float32([1, 2])) == 0.0
    assert abs(normwise(np.float32([1, 2.5]), np.float32([1, 2])) - 0.25) < 1e-12
