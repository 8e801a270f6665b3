"""CPU: the C-ABI library loads without a GPU, exports every entry point include/trc_cuda.h
declares, and its host-side argument checks reject what the reference's constructors reject
(these checks run before any CUDA call, so no device is needed)."""
from __future__ import annotations

import ctypes

import pytest

import trc_cuda


def test_library_exports_every_declared_symbol():
    L = trc_cuda.lib()
    declared = trc_cuda.exported_symbols()
    assert len(declared) >= 20
    missing = [n for n in declared if not hasattr(L, n)]
    assert not missing, missing
    assert L.trc_cuda_abi_version() == 1


def test_block_sizes_match_type_table():
    assert [trc_cuda.block_bytes(t) for t in (2, 3, 6, 7, 8)] == [18, 20, 22, 24, 34]
    assert trc_cuda.block_bytes(0) == 0 and trc_cuda.block_bytes(10) == 0  # F32, Q2_K


def test_status_strings():
    L = trc_cuda.lib()
    for s in (0, -1, -2, -3, -4, -5):
        assert L.trc_cuda_status_string(s)
    assert b"invalid" in L.trc_cuda_status_string(-1)


def _view(ne, nb, data=0x1000):
    v = trc_cuda.View()
    v.data = data
    for i in range(4):
        v.ne[i], v.nb[i] = ne[i], nb[i]
    return v


def test_mul_mat_shape_rules_rejected_on_host():
    L = trc_cuda.lib()
    a = _view([5, 3, 1, 1], [4, 20, 60, 60])
    b_bad_k = _view([6, 4, 1, 1], [4, 24, 96, 96])
    d = _view([3, 4, 1, 1], [4, 12, 48, 48])
    assert L.trc_cuda_mul_mat(ctypes.byref(a), ctypes.byref(b_bad_k), ctypes.byref(d), 0, None) == -1
    # b.ne2 % a.ne2 != 0 (the reference's mul_mat_batch2_abort case)
    a2 = _view([5, 3, 2, 1], [4, 20, 60, 120])
    b3 = _view([5, 4, 3, 1], [4, 20, 80, 240])
    d3 = _view([3, 4, 3, 1], [4, 12, 48, 144])
    assert L.trc_cuda_mul_mat(ctypes.byref(a2), ctypes.byref(b3), ctypes.byref(d3), 0, None) == -1
    # wrong output shape
    b = _view([5, 4, 1, 1], [4, 20, 80, 80])
    d_bad = _view([4, 3, 1, 1], [4, 16, 48, 48])
    assert L.trc_cuda_mul_mat(ctypes.byref(a), ctypes.byref(b), ctypes.byref(d_bad), 0, None) == -1


def test_dequant_argument_checks_on_host():
    L = trc_cuda.lib()
    assert L.trc_cuda_dequant(10, None, 1, None, None) == -2     # Q2_K: unsupported
    assert L.trc_cuda_dequant(2, None, -1, None, None) == -1     # negative size
    assert L.trc_cuda_dequant(2, None, 0, None, None) == 0       # empty tensor: nothing to do
    assert L.trc_cuda_dequant(2, ctypes.c_void_p(0x1001), 1, ctypes.c_void_p(0x2000), None) == -1  # odd address


def test_acc_bounds_rule_on_host():
    L = trc_cuda.lib()
    b = _view([4, 1, 1, 1], [4, 16, 16, 16])
    assert L.trc_cuda_acc(ctypes.c_void_p(0x1000), 16, ctypes.byref(b), 16, 16, 16, 4, None) == -1


def test_ggml_view_mapping_is_reversed_torch_layout():
    import torch

    t = torch.empty((2, 3, 5, 7))
    assert trc_cuda.ggml_ne(t) == [7, 5, 3, 2]
    with pytest.raises(trc_cuda.TrcCudaError):
        trc_cuda.view_of(t)  # host tensors are rejected: device memory only


def test_dequant_to_peers_argument_checks_on_host():
    """trc_cuda_dequant_many_to_peers rejects bad peer tables before any device call."""
    L = trc_cuda.lib()
    job = (trc_cuda.DequantJob * 1)()
    job[0].blocks = 0x10000
    job[0].out = 0x20000
    job[0].n_blocks = 4
    job[0].type = 2
    base = ctypes.c_void_p(0x20000)
    peers = (ctypes.c_void_p * 9)(*([0x40000] * 9))
    assert L.trc_cuda_dequant_many_to_peers(job, 1, base, peers, 9, None) == -1     # more than 8 peers
    assert L.trc_cuda_dequant_many_to_peers(job, 1, base, peers, -1, None) == -1    # negative count
    assert L.trc_cuda_dequant_many_to_peers(job, 1, None, peers, 1, None) == -1     # no local base
    assert L.trc_cuda_dequant_many_to_peers(job, 1, base, None, 1, None) == -1      # no peer table
    odd = (ctypes.c_void_p * 1)(0x40008)                                             # 8 bytes off the 16-byte grid
    assert L.trc_cuda_dequant_many_to_peers(job, 1, base, odd, 1, None) == -1
    null_peer = (ctypes.c_void_p * 1)(None)
    assert L.trc_cuda_dequant_many_to_peers(job, 1, base, null_peer, 1, None) == -1
    above = ctypes.c_void_p(0x20010)                                                 # output below the local base
    assert L.trc_cuda_dequant_many_to_peers(job, 1, above, peers, 1, None) == -1


def test_mul_mat_flag_values_match_header():
    import re
    from pathlib import Path

    hdr = (Path(__file__).resolve().parents[1] / "include" / "trc_cuda.h").read_text()
    flags = dict(re.findall(r"(TRC_CUDA_MM_\w+)\s*=\s*(\d+)u", hdr))
    assert int(flags["TRC_CUDA_MM_ACCUMULATE"]) == trc_cuda.MM_ACCUMULATE
    assert int(flags["TRC_CUDA_MM_SIMT"]) == trc_cuda.MM_SIMT
    assert int(flags["TRC_CUDA_MM_ONE_CTA"]) == trc_cuda.MM_ONE_CTA
    assert int(flags["TRC_CUDA_MM_FUSED"]) == trc_cuda.MM_FUSED
    assert int(flags["TRC_CUDA_MM_TWO_STEP"]) == trc_cuda.MM_TWO_STEP


def test_loader_wrappers_reject_bad_destinations_on_host():
    """The loaders write 32 floats per block at dst.data_ptr(): a host tensor, another dtype or a
    device tensor passed as the host source is refused before any library call."""
    import numpy as np
    import torch

    host = np.zeros(18 * 2, dtype=np.uint8)
    for load in (lambda d: trc_cuda.gguf_load_tensor(2, host, d, torch.empty(36, dtype=torch.uint8)),
                 lambda d: trc_cuda.gguf_load_tensor_static(2, host, d)):
        with pytest.raises(trc_cuda.TrcCudaError, match="float32"):
            load(torch.empty(64, dtype=torch.float16))
        with pytest.raises(trc_cuda.TrcCudaError, match="CUDA"):
            load(torch.empty(64, dtype=torch.float32))       # host memory, not device memory
    with pytest.raises(trc_cuda.TrcCudaError, match="contiguous"):
        trc_cuda.gguf_load_tensor_static(2, np.zeros((4, 18), dtype=np.uint8)[:, :9], torch.empty(64))
