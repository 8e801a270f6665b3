"""GPU: the allocation-free loader trc_cuda_load_quant_static, for callers that cannot call
cudaMalloc (their device memory belongs to another allocator or has a fixed budget). It must give
the oracle's F32 weights bit for bit (and so the same as trc_cuda_load_quant with a caller-provided
staging buffer) on two calls in a row through the same static staging array, without allocating
device memory, and it must refuse tensors larger than its fixed 64 MiB array. Collected last, so a
failure here leaves every other test already run; it passes alone in a fresh process as well as
after the other tests."""
from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

import synth

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def tc():
    import trc_cuda

    trc_cuda.lib()
    return trc_cuda


def _free_device_bytes(tc) -> int:
    free_b, total_b = ctypes.c_size_t(0), ctypes.c_size_t(0)
    tc.lib().trc_cuda_rt_mem_info.argtypes = [ctypes.POINTER(ctypes.c_size_t), ctypes.POINTER(ctypes.c_size_t)]
    assert tc.lib().trc_cuda_rt_mem_info(ctypes.byref(free_b), ctypes.byref(total_b)) == 0
    return free_b.value


def test_static_loader_matches_oracle_and_staged_loader_twice(tc):
    # the last case is above the 16 MB from which trc_cuda_load_quant splits its upload across a
    # second stream; the static loader always makes one copy on the caller's stream
    import oracle

    torch.cuda.synchronize()
    free_before_first = _free_device_bytes(tc)
    dummy = torch.empty(0, dtype=torch.float32, device="cuda")
    tc.gguf_load_tensor_static(synth.TYPE_Q4_0, np.zeros(0, dtype=np.uint8), dummy)  # zero-size warm-up
    torch.cuda.synchronize()
    # The 64 MiB array is reserved when the library's device code loads on this device. Earlier
    # library calls (other tests, or the module loading in the warm-up call above) have loaded it,
    # so the warm-up may at most account for that reserve (plus allocation granularity), never more.
    assert free_before_first - _free_device_bytes(tc) <= tc.STATIC_STAGING_BYTES + (2 << 20)
    cases = [(synth.TYPE_Q5_0, 4096 * 1024), (synth.TYPE_Q8_0, 4096 * 512 + 32 * 7),
             (synth.TYPE_Q8_0, 4096 * 5000)]
    for i, (qtype, n) in enumerate(cases):
        blocks = synth.random_blocks(qtype, n // 32, seed=900 + i)
        host = torch.from_numpy(blocks).pin_memory()
        staging = torch.empty(host.numel(), dtype=torch.uint8, device="cuda")
        want = torch.empty(n, dtype=torch.float32, device="cuda")
        tc.gguf_load_tensor(qtype, host, want, staging)
        outs = [torch.full((n,), float("nan"), dtype=torch.float32, device="cuda") for _ in range(2)]
        torch.cuda.synchronize()
        for out in outs:  # two calls in a row through the same static array
            free_before = _free_device_bytes(tc)
            tc.gguf_load_tensor_static(qtype, host, out)
            torch.cuda.synchronize()
            assert _free_device_bytes(tc) == free_before, "the allocation-free loader changed free device memory"
        w_oracle = oracle.dequant(qtype, blocks).view(np.uint32)
        assert np.array_equal(want.cpu().numpy().view(np.uint32), w_oracle)
        for out in outs:
            assert np.array_equal(out.cpu().numpy().view(np.uint32), w_oracle)
    assert tc.device_error() == 0


def test_static_loader_rejects_tensors_beyond_its_buffer(tc):
    qtype = synth.TYPE_Q8_0
    too_many = tc.STATIC_STAGING_BYTES // tc.block_bytes(qtype) + 1
    host = np.zeros(16, dtype=np.uint8)  # never read: the size check comes first
    out = torch.empty(32, dtype=torch.float32, device="cuda")
    rc = tc.lib().trc_cuda_load_quant_static(qtype, ctypes.c_void_p(host.ctypes.data), too_many, out.data_ptr(), None)
    assert rc == tc.ETOOBIG
    assert b"64 MiB" in tc.lib().trc_cuda_status_string(rc)
