"""GPU failure detection without a GPU fault: a kernel waits, with the library's bounded mbarrier
wait, on a barrier nothing arrives on. The wait runs out after a short limit, the device error word
reports it, the kernel returns by itself, and the context keeps working (a dequant afterwards is
bit-exact). The same bounded waits guard every pipeline barrier of the GEMM and dequant kernels."""
from __future__ import annotations

import time

import numpy as np
import pytest
import torch

import oracle
import synth

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def tc():
    import trc_cuda

    trc_cuda.lib()
    return trc_cuda


def test_bounded_wait_reports_and_context_survives(tc):
    assert tc.device_error() == 0  # reads and clears
    t0 = time.perf_counter()
    assert tc.selftest_wait_timeout(50_000_000)  # 50 ms: the wait gave up on its own
    dt = time.perf_counter() - t0
    assert 0.04 < dt < 5.0, dt
    assert tc.device_error(reset=False) == 8  # TRC_DEVERR_SELFTEST
    assert tc.device_error() == 8             # read and clear
    assert tc.device_error() == 0
    # the context is intact: a dequant right after is bit-exact
    blocks = synth.random_blocks(synth.TYPE_Q4_1, 4096, seed=77)
    got = tc.gguf_tensor_to_f32(synth.TYPE_Q4_1, torch.from_numpy(blocks).cuda()).cpu().numpy()
    assert np.array_equal(got.view(np.uint32), oracle.dequant(synth.TYPE_Q4_1, blocks).view(np.uint32))
    assert tc.device_error() == 0


@pytest.mark.parametrize("bulk", [False, True], ids=["st_global", "bulk_store"])
def test_stream_probe_writes_what_it_reads(tc, bulk):
    """The measurement-support streaming kernels: each warp's 512 input bytes land R times in order
    (word x incremented per copy), nothing past the R x input extent is touched; the bulk-store
    variant writes the same layout."""
    n16, ratio = 256 * 40, 5
    src = torch.arange(n16 * 4, dtype=torch.int32, device="cuda")
    out = torch.full((n16 * 4 * ratio + 64,), -7, dtype=torch.int32, device="cuda")
    tc.stream_probe(src.view(torch.float32), out.view(torch.float32), ratio, bulk=bulk)
    torch.cuda.synchronize()
    s = src.view(-1, 32, 4).cpu().numpy()        # [warp, lane, 4 words]
    o = out[: n16 * 4 * ratio].view(-1, ratio, 32, 4).cpu().numpy()
    for j in range(ratio):
        want = s.copy()
        want[:, :, 0] += j + 1
        assert np.array_equal(o[:, j], want)
    assert bool((out[n16 * 4 * ratio:] == -7).all())
