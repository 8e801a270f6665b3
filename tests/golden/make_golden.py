"""Regenerates tests/golden/*.npz. TEST INFRASTRUCTURE, run where the train.cpp source tree exists:

    python tests/golden/make_golden.py [TRAIN_CPP_SOURCE_DIR]

Three fixture files, all small:

  reference_goldens.npz  the reference's own PyTorch-generated golden arrays for this path, copied
                         verbatim from its tests/golden/ (cases.txt:26-29 mul_mat*, grad_cases.txt
                         grad_mul_mat_batch*, repeat, transpose_cont). Keys are the .npy stems.
  dequant_goldens.npz    packed blocks and the reference's gguf_tensor_to_f32 output for
                         (a) the five known-answer block patterns of the reference's
                         tests/test_gguf.cpp:355-444 and (b) 257 random blocks per format drawn like
                         the benchmark configurations (train.cpp_b200/synth.py, seed 1234).
  mul_mat_goldens.npz    inputs and the reference's outputs (oracle/_ref, CPU device + autograd)
                         for small mul_mat forward/backward cases with the shapes of the Linear and
                         GQA workloads, including transposed views and modulo broadcasting.
"""
from __future__ import annotations

import struct
import os
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent
sys.path.insert(0, str(ROOT / "train.cpp_b200"))
sys.path.insert(0, str(ROOT / "oracle"))

import synth  # noqa: E402
import oracle  # noqa: E402


def kat_blocks() -> dict[int, tuple[bytes, int]]:
    """The block patterns of the reference's dequant known-answer tests (test_gguf.cpp:355-444)."""
    nib = bytes(((j & 0x0F) | ((15 - j) << 4)) for j in range(16))      # low = j, high = 15 - j
    nib_r = bytes((((15 - j) & 0x0F) | (j << 4)) for j in range(16))    # low = 15 - j, high = j
    u16 = lambda x: struct.pack("<H", x)
    u32 = lambda x: struct.pack("<I", x)
    return {
        synth.TYPE_Q4_0: (u16(0x3800) + nib + u16(0x3400) + nib_r, 64),
        synth.TYPE_Q4_1: (u16(0x3400) + u16(0xBC00) + nib, 32),
        synth.TYPE_Q5_0: (u16(0x3C00) + u32(0) + nib + u16(0x3C00) + u32(0xFFFFFFFF) + nib, 64),
        synth.TYPE_Q5_1: (u16(0x3800) + u16(0x3000) + u32(0) + nib, 32),
        synth.TYPE_Q8_0: (u16(0x3000) + bytes((j - 16) & 0xFF for j in range(32)), 32),
    }


def kat_expected() -> dict[int, np.ndarray]:
    """Hand-computed expectations of the same tests (exact values)."""
    j = np.arange(16, dtype=np.float32)
    e = {}
    e[synth.TYPE_Q4_0] = np.concatenate([(j - 8) * 0.5, (7 - j) * 0.5, (7 - j) * 0.25, (j - 8) * 0.25])
    e[synth.TYPE_Q4_1] = np.concatenate([j * 0.25 - 1.0, (15 - j) * 0.25 - 1.0])
    e[synth.TYPE_Q5_0] = np.concatenate([j - 16, -1 - j, j, 15 - j])
    e[synth.TYPE_Q5_1] = np.concatenate([j * 0.5 + 0.125, (15 - j) * 0.5 + 0.125])
    e[synth.TYPE_Q8_0] = (np.arange(32, dtype=np.float32) - 16) * 0.125
    return {k: v.astype(np.float32) for k, v in e.items()}


def main(ref_dir: Path) -> None:
    # 1. the reference's own golden arrays for this path
    stems = ["mul_mat", "mul_mat_batch", "mul_mat_batch_bcast_div", "mul_mat_batch_tile",
             "grad_mul_mat_batch", "grad_mul_mat_batch_div", "repeat", "transpose_cont"]
    arrays = {}
    for f in sorted((ref_dir / "tests" / "golden").glob("*.npy")):
        if any(f.stem == s or f.stem.startswith(s + "_") for s in stems):
            if f.stem.startswith("mul_mat_batch_") and not any(f.stem.startswith(s + "_") for s in stems[1:4]):
                continue
            arrays[f.stem] = np.load(f)
    np.savez_compressed(HERE / "reference_goldens.npz", **arrays)

    # 2. dequant: KAT patterns + random blocks, with the reference's own outputs
    d = {}
    exp = kat_expected()
    for t, (raw, n) in kat_blocks().items():
        name = synth.TYPE_BY_NAME and [k for k, v in synth.TYPE_BY_NAME.items() if v == t][0]
        blocks = np.frombuffer(raw, dtype=np.uint8).copy()
        got = oracle.ref_dequant(t, blocks, n)
        assert np.array_equal(got, exp[t]), f"reference disagrees with its own KAT for {name}"
        d[f"kat_{name}_blocks"] = blocks
        d[f"kat_{name}_out"] = got
        rb = synth.random_blocks(t, 257, seed=1234 + t)
        d[f"rand_{name}_blocks"] = rb
        d[f"rand_{name}_out"] = oracle.ref_dequant(t, rb, 257 * 32)
    np.savez_compressed(HERE / "dequant_goldens.npz", **d)

    # 3. mul_mat forward/backward through the reference CPU device and autograd
    m = {}
    rng = np.random.Generator(np.random.PCG64(7))
    f32 = lambda *s: rng.standard_normal(s).astype(np.float32)
    # forward with views: (A base shape, A transposed?, B base shape, B transposed?)
    fwd = {
        "fwd_basic": ((3, 36), False, (5, 36), False),
        "fwd_ta": ((36, 68), True, (66, 36), False),
        "fwd_tb": ((70, 36), False, (36, 68), True),
        "fwd_tab": ((40, 132), True, (40, 260), True),
        "fwd_odd": ((70, 33), False, (66, 33), False),
        "fwd_bcast": ((2, 1, 70, 36), False, (2, 4, 66, 36), False),
        "fwd_bcast_t": ((2, 1, 36, 68), True, (2, 4, 36, 72), True),
    }
    for name, (sa, ta, sb, tb) in fwd.items():
        a, b = f32(*sa), f32(*sb)
        m[name + "_a"], m[name + "_b"] = a, b
        m[name + "_ta"], m[name + "_tb"] = np.int32(ta), np.int32(tb)
        m[name + "_d"] = oracle.ref_mul_mat(a, ta, b, tb)
    # training steps: loss = sum(mul(D, G)); A and B are PARAMs (shapes as numpy = reversed ne)
    steps = {
        "step_linear": ((96, 300), (40, 300)),           # W[k=300, m=96], X[k=300, n=40]: 2 promotion chunks
        "step_gqa": ((2, 2, 48, 16), (2, 8, 40, 16)),    # A[16,48,2,2] . B[16,40,8,2], bcast ne2 x4
        "step_ragged": ((70, 33), (66, 33)),
    }
    for name, (sa, sb) in steps.items():
        a, b = f32(*sa), f32(*sb)
        dshape = (sb[0], sb[1], sb[2], sa[-2]) if len(sb) == 4 else (sb[0], sa[0])
        g = (rng.standard_normal(dshape) * 1e-2).astype(np.float32)
        dd, da, db = oracle.ref_mul_mat_step(a, b, g)
        m.update({name + "_a": a, name + "_b": b, name + "_g": g, name + "_d": dd, name + "_da": da, name + "_db": db})
    np.savez_compressed(HERE / "mul_mat_goldens.npz", **m)
    for f in ("reference_goldens.npz", "dequant_goldens.npz", "mul_mat_goldens.npz"):
        print(f, (HERE / f).stat().st_size, "bytes")


if __name__ == "__main__":
    if len(sys.argv) > 1:
        src = Path(sys.argv[1])
    elif os.environ.get("TRC_REFERENCE_DIR"):
        src = Path(os.environ["TRC_REFERENCE_DIR"])
    else:
        sys.exit("usage: make_golden.py <train.cpp source dir>  (or set TRC_REFERENCE_DIR)")
    main(src)
