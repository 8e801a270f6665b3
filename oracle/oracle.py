"""TEST INFRASTRUCTURE: ctypes bindings of the parity oracle. Not product code.

Two CPU libraries, both used only by tests/, __graft_entry__.smoke() and bench.py's CPU baseline:

  * liboracle.so  -- trc_oracle.c, the C restatement of train.cpp's hot path (built on demand with
                     `make -C oracle`, plain gcc, so it can be rebuilt wherever the tests run);
  * libtrc_ref.so -- train.cpp's own CPU code compiled from its sources plus ref_shim.cpp
                     (`make -C oracle ref`; it needs the train.cpp source tree, so it is built where
                     that tree exists and travels as a prebuilt file).
"""
from __future__ import annotations

import ctypes
import os
import subprocess
import tempfile
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ORACLE_SO = HERE / "_build" / "liboracle.so"
REF_SO = HERE / "_ref" / "libtrc_ref.so"

_P, _I, _I64, _SZ = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_size_t
_NE = ctypes.c_int64 * 4
_NB = ctypes.c_size_t * 4

_oracle: ctypes.CDLL | None = None
_ref: ctypes.CDLL | None = None


def oracle_lib() -> ctypes.CDLL:
    global _oracle
    if _oracle is None:
        src = [HERE / "trc_oracle.c", HERE / "trc_oracle.h"]
        if not ORACLE_SO.exists() or any(s.stat().st_mtime > ORACLE_SO.stat().st_mtime for s in src):
            subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
        L = ctypes.CDLL(str(ORACLE_SO))
        L.oracle_fp16_to_fp32.restype = ctypes.c_float
        L.oracle_fp16_to_fp32.argtypes = [ctypes.c_uint16]
        L.oracle_fp32_to_fp16.restype = ctypes.c_uint16
        L.oracle_fp32_to_fp16.argtypes = [ctypes.c_float]
        L.oracle_block_bytes.restype = _SZ
        L.oracle_block_bytes.argtypes = [_I]
        L.oracle_dequant.restype = _I
        L.oracle_dequant.argtypes = [_I, _P, _I64, _P]
        L.oracle_mul_mat.restype = _I
        L.oracle_mul_mat.argtypes = [_P, _NE, _NB, _P, _NE, _NB, _P, _NE, _NB, _I]
        L.oracle_cont.restype = None
        L.oracle_cont.argtypes = [_P, _NE, _NB, _P]
        L.oracle_repeat_back.restype = None
        L.oracle_repeat_back.argtypes = [_P, _NE, _NB, _P, _NE]
        L.oracle_acc.restype = None
        L.oracle_acc.argtypes = [_P, _P, _NE, _NB, _SZ, _SZ, _SZ, _SZ]
        _F = ctypes.c_float
        L.oracle_unary.restype = None
        L.oracle_unary.argtypes = [_I, _P, _I64, _F, _P]
        L.oracle_sum_rows.restype = None
        L.oracle_sum_rows.argtypes = [_P, _I64, _I64, _I, _P]
        L.oracle_adamw.restype = None
        L.oracle_adamw.argtypes = [_P, _P, _P, _P, _I64, _P]
        L.oracle_sgd.restype = None
        L.oracle_sgd.argtypes = [_P, _P, _P, _I64, _P]
        L.oracle_sum_sqr_acc.restype = None
        L.oracle_sum_sqr_acc.argtypes = [_P, _P, _I64]
        L.oracle_clip_scale.restype = None
        L.oracle_clip_scale.argtypes = [_P, _I64, _F, _F, _F]
        _oracle = L
    return _oracle


def ref_available() -> bool:
    return REF_SO.exists()


def ref_lib() -> ctypes.CDLL:
    global _ref
    if _ref is None:
        if not REF_SO.exists():
            raise FileNotFoundError(f"{REF_SO} not built (make -C oracle ref, needs the train.cpp sources)")
        L = ctypes.CDLL(str(REF_SO))
        L.ref_fp16_to_fp32_bits.restype = ctypes.c_uint32
        L.ref_fp16_to_fp32_bits.argtypes = [ctypes.c_uint16]
        L.ref_fp32_to_fp16.restype = ctypes.c_uint16
        L.ref_fp32_to_fp16.argtypes = [ctypes.c_float]
        L.ref_gguf_open.restype = _P
        L.ref_gguf_open.argtypes = [ctypes.c_char_p]
        L.ref_gguf_close.restype = None
        L.ref_gguf_close.argtypes = [_P]
        L.ref_gguf_tensor_nelements.restype = _I64
        L.ref_gguf_tensor_nelements.argtypes = [_P, ctypes.c_char_p]
        L.ref_gguf_tensor_to_f32.restype = _I
        L.ref_gguf_tensor_to_f32.argtypes = [_P, ctypes.c_char_p, _P, _I64]
        L.ref_mul_mat.restype = _I
        L.ref_mul_mat.argtypes = [_P, _P, _I, _P, _P, _I, _P]
        L.ref_mul_mat_step.restype = _I
        L.ref_mul_mat_step.argtypes = [_P, _P, _P, _P, _P, _P, _P, _P]
        _F = ctypes.c_float
        L.ref_unary.restype = _I
        L.ref_unary.argtypes = [_I, _P, _P, _F, _P]
        L.ref_sum_rows.restype = _I
        L.ref_sum_rows.argtypes = [_P, _P, _I, _P]
        L.ref_opt_step_adamw.restype = _I
        L.ref_opt_step_adamw.argtypes = [_P, _P, _P, _P, _I64, _P]
        L.ref_opt_step_sgd.restype = _I
        L.ref_opt_step_sgd.argtypes = [_P, _P, _P, _I64, _P]
        L.ref_sum_sqr_acc.restype = _I
        L.ref_sum_sqr_acc.argtypes = [_P, _P, _I64]
        L.ref_clip_scale_inplace.restype = _I
        L.ref_clip_scale_inplace.argtypes = [_P, _I64, _F, _F, _F]
        _ref = L
    return _ref


# ------------------------------------------------------------------ helpers over numpy arrays

def _ne_nb(arr: np.ndarray) -> tuple:
    """ggml (ne, nb) of a float32 numpy array of up to 4 dims (last axis = ne0)."""
    ne = list(arr.shape)[::-1] + [1] * (4 - arr.ndim)
    nb = [s for s in arr.strides[::-1]] + [0] * (4 - arr.ndim)
    for d in range(arr.ndim, 4):
        nb[d] = nb[d - 1] * ne[d - 1] if d > 0 else 4
    return _NE(*ne), _NB(*nb)


def fp16_to_fp32(h: int) -> float:
    return oracle_lib().oracle_fp16_to_fp32(h)


def dequant(qtype: int, blocks: np.ndarray, n_blocks: int | None = None) -> np.ndarray:
    L = oracle_lib()
    bb = L.oracle_block_bytes(qtype)
    if n_blocks is None:
        n_blocks = blocks.nbytes // bb
    blocks = np.ascontiguousarray(blocks, dtype=np.uint8)
    out = np.empty(n_blocks * 32, dtype=np.float32)
    if L.oracle_dequant(qtype, blocks.ctypes.data, n_blocks, out.ctypes.data) != 0:
        raise ValueError(f"oracle_dequant rejected type {qtype}")
    return out


def mul_mat(a: np.ndarray, b: np.ndarray, n_threads: int | None = None) -> np.ndarray:
    """Oracle ggml mul_mat on numpy views (any strides; last axis = ne0). Bit-identical to the
    reference's compute_mul_mat."""
    ane, anb = _ne_nb(a)
    bne, bnb = _ne_nb(b)
    out = np.empty((bne[3], bne[2], bne[1], ane[1]), dtype=np.float32)
    dne, dnb = _ne_nb(out)
    if n_threads is None:
        n_threads = os.cpu_count() or 1
    # the C code reads through raw pointers: keep the base arrays alive via the views
    rc = oracle_lib().oracle_mul_mat(a.ctypes.data, ane, anb, b.ctypes.data, bne, bnb, out.ctypes.data, dne, dnb,
                                     n_threads)
    if rc != 0:
        raise ValueError("oracle_mul_mat: shape rule violated")
    return out


def cont(a: np.ndarray) -> np.ndarray:
    ne, nb = _ne_nb(a)
    out = np.empty(a.shape, dtype=np.float32)
    oracle_lib().oracle_cont(a.ctypes.data, ne, nb, out.ctypes.data)
    return out


def repeat_back(a: np.ndarray, dst_ne) -> np.ndarray:
    ne, nb = _ne_nb(a)
    dst_ne = list(dst_ne) + [1] * (4 - len(dst_ne))
    out = np.empty(dst_ne[::-1], dtype=np.float32)
    oracle_lib().oracle_repeat_back(a.ctypes.data, ne, nb, out.ctypes.data, _NE(*dst_ne))
    return out


def acc_(dst: np.ndarray, b: np.ndarray, nb1: int, nb2: int, nb3: int, offset: int) -> np.ndarray:
    ne, nb = _ne_nb(b)
    oracle_lib().oracle_acc(dst.ctypes.data, b.ctypes.data, ne, nb, nb1, nb2, nb3, offset)
    return dst


# ------------------------------------------------------------------ the compiled reference

def ref_fp16_to_fp32_bits(h: int) -> int:
    return ref_lib().ref_fp16_to_fp32_bits(h)


def ref_dequant_file(path: str, name: str) -> np.ndarray:
    """gguf_open + gguf_tensor_to_f32 of the reference on a GGUF file."""
    L = ref_lib()
    f = L.ref_gguf_open(str(path).encode())
    if not f:
        raise ValueError(f"reference rejected {path}")
    try:
        n = L.ref_gguf_tensor_nelements(f, name.encode())
        out = np.empty(n, dtype=np.float32)
        if L.ref_gguf_tensor_to_f32(f, name.encode(), out.ctypes.data, n) != 0:
            raise ValueError(f"reference gguf_tensor_to_f32 rejected {name}")
        return out
    finally:
        L.ref_gguf_close(f)


def ref_dequant(qtype: int, blocks: np.ndarray, ne0: int, ne1: int = 1) -> np.ndarray:
    """Reference host dequantization through a temporary GGUF file."""
    import sys
    sys.path.insert(0, str(HERE.parent / "train.cpp_b200"))
    import synth  # noqa: E402

    with tempfile.TemporaryDirectory() as td:
        p = Path(td) / "t.gguf"
        ne = (ne0,) if ne1 == 1 else (ne0, ne1)
        synth.write_gguf(p, [("w", qtype, ne, np.ascontiguousarray(blocks, dtype=np.uint8))])
        return ref_dequant_file(str(p), "w")


def ref_mul_mat(a_base: np.ndarray, a_trans: bool, b_base: np.ndarray, b_trans: bool) -> np.ndarray:
    """Reference mul_mat(op(A), op(B)) with A/B contiguous float32 arrays of up to 4 dims and op =
    identity or ggml transpose. Returns the contiguous result (numpy shape = reversed ne)."""
    a_base = np.ascontiguousarray(a_base, dtype=np.float32)
    b_base = np.ascontiguousarray(b_base, dtype=np.float32)
    ane = list(a_base.shape)[::-1] + [1] * (4 - a_base.ndim)
    bne = list(b_base.shape)[::-1] + [1] * (4 - b_base.ndim)
    opa = [ane[1], ane[0], ane[2], ane[3]] if a_trans else ane
    opb = [bne[1], bne[0], bne[2], bne[3]] if b_trans else bne
    out = np.empty((opb[3], opb[2], opb[1], opa[1]), dtype=np.float32)
    rc = ref_lib().ref_mul_mat(a_base.ctypes.data, _NE(*ane), int(a_trans), b_base.ctypes.data, _NE(*bne),
                               int(b_trans), out.ctypes.data)
    if rc != 0:
        raise RuntimeError("reference graph_compute failed")
    return out


def ref_mul_mat_step(a: np.ndarray, b: np.ndarray, g: np.ndarray):
    """Reference D = mul_mat(A, B), dA, dB through train.cpp's autograd with loss = sum(mul(D, G))."""
    a = np.ascontiguousarray(a, dtype=np.float32)
    b = np.ascontiguousarray(b, dtype=np.float32)
    g = np.ascontiguousarray(g, dtype=np.float32)
    ane = list(a.shape)[::-1] + [1] * (4 - a.ndim)
    bne = list(b.shape)[::-1] + [1] * (4 - b.ndim)
    d = np.empty((bne[3], bne[2], bne[1], ane[1]), dtype=np.float32)
    da = np.empty_like(a)
    db = np.empty_like(b)
    rc = ref_lib().ref_mul_mat_step(a.ctypes.data, _NE(*ane), b.ctypes.data, _NE(*bne), g.ctypes.data,
                                    d.ctypes.data, da.ctypes.data, db.ctypes.data)
    if rc != 0:
        raise RuntimeError("reference training step failed")
    return d, da, db


# ------------------------------------------------------------------ the rest of a training step

UNARY_SQR, UNARY_SQRT, UNARY_ABS, UNARY_NEG, UNARY_SGN, UNARY_STEP, UNARY_SCALE = range(7)


def _f32(x) -> np.ndarray:
    return np.ascontiguousarray(x, dtype=np.float32)


def _p6(params) -> np.ndarray:
    p = _f32(params)
    assert p.size == 6
    return p


def unary(op: int, x: np.ndarray, param: float = 0.0) -> np.ndarray:
    x = _f32(x)
    out = np.empty_like(x)
    oracle_lib().oracle_unary(op, x.ctypes.data, x.size, param, out.ctypes.data)
    return out


def sum_rows(x: np.ndarray, take_mean: bool = False) -> np.ndarray:
    """Row sums (or means) over the last axis; result keeps the other axes with a last axis of 1."""
    x = _f32(x)
    out = np.empty(x.shape[:-1] + (1,), dtype=np.float32)
    oracle_lib().oracle_sum_rows(x.ctypes.data, x.shape[-1], x.size // max(1, x.shape[-1]), int(take_mean),
                                 out.ctypes.data)
    return out


def adamw(p, g, m, v, params6):
    p, g, m, v = (_f32(a).copy() for a in (p, g, m, v))
    oracle_lib().oracle_adamw(p.ctypes.data, g.ctypes.data, m.ctypes.data, v.ctypes.data, p.size,
                              _p6(params6).ctypes.data)
    return p, m, v


def sgd(p, g, mom, params6):
    p, g, mom = (_f32(a).copy() for a in (p, g, mom))
    oracle_lib().oracle_sgd(p.ctypes.data, g.ctypes.data, mom.ctypes.data, p.size, _p6(params6).ctypes.data)
    return p, mom


def sum_sqr_acc(acc: float, x: np.ndarray) -> np.float32:
    a = np.array([acc], dtype=np.float32)
    x = _f32(x)
    oracle_lib().oracle_sum_sqr_acc(a.ctypes.data, x.ctypes.data, x.size)
    return a[0]


def clip_scale(x: np.ndarray, norm: float, max_norm: float, eps: float) -> np.ndarray:
    x = _f32(x).copy()
    oracle_lib().oracle_clip_scale(x.ctypes.data, x.size, norm, max_norm, eps)
    return x


def ref_unary(op: int, x: np.ndarray, param: float = 0.0) -> np.ndarray:
    x = _f32(x)
    out = np.empty_like(x)
    ne = list(x.shape)[::-1] + [1] * (4 - x.ndim)
    if ref_lib().ref_unary(op, x.ctypes.data, _NE(*ne), param, out.ctypes.data) != 0:
        raise RuntimeError("reference unary failed")
    return out


def ref_sum_rows(x: np.ndarray, take_mean: bool = False) -> np.ndarray:
    x = _f32(x)
    out = np.empty(x.shape[:-1] + (1,), dtype=np.float32)
    ne = list(x.shape)[::-1] + [1] * (4 - x.ndim)
    if ref_lib().ref_sum_rows(x.ctypes.data, _NE(*ne), int(take_mean), out.ctypes.data) != 0:
        raise RuntimeError("reference sum_rows failed")
    return out


def ref_adamw(p, g, m, v, params6):
    p, g, m, v = (_f32(a).copy() for a in (p, g, m, v))
    if ref_lib().ref_opt_step_adamw(p.ctypes.data, g.ctypes.data, m.ctypes.data, v.ctypes.data, p.size,
                                    _p6(params6).ctypes.data) != 0:
        raise RuntimeError("reference opt_step_adamw failed")
    return p, m, v


def ref_sgd(p, g, mom, params6):
    p, g, mom = (_f32(a).copy() for a in (p, g, mom))
    if ref_lib().ref_opt_step_sgd(p.ctypes.data, g.ctypes.data, mom.ctypes.data, p.size,
                                  _p6(params6).ctypes.data) != 0:
        raise RuntimeError("reference opt_step_sgd failed")
    return p, mom


def ref_sum_sqr_acc(acc: float, x: np.ndarray) -> np.float32:
    a = np.array([acc], dtype=np.float32)
    x = _f32(x)
    if ref_lib().ref_sum_sqr_acc(a.ctypes.data, x.ctypes.data, x.size) != 0:
        raise RuntimeError("reference sum_sqr_acc failed")
    return a[0]


def ref_clip_scale(x: np.ndarray, norm: float, max_norm: float, eps: float) -> np.ndarray:
    x = _f32(x).copy()
    if ref_lib().ref_clip_scale_inplace(x.ctypes.data, x.size, norm, max_norm, eps) != 0:
        raise RuntimeError("reference clip_scale_inplace failed")
    return x
