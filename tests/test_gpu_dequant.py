"""GPU parity: device dequantization (libtrc_cuda.so) vs the oracle and the reference's known
answers, bit for bit, on the KATs, random blocks at full config size, ragged tails, unaligned
buffers, batched jobs and the host-upload path."""
from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
import synth

pytestmark = pytest.mark.gpu

TYPES = [synth.TYPE_Q4_0, synth.TYPE_Q4_1, synth.TYPE_Q5_0, synth.TYPE_Q5_1, synth.TYPE_Q8_0]
NAMES = {v: k for k, v in synth.TYPE_BY_NAME.items()}


@pytest.fixture(scope="module")
def tc():
    import trc_cuda

    trc_cuda.lib()
    assert torch.cuda.is_available()
    return trc_cuda


def dev(x: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(x)).cuda()


def bits_equal(got: np.ndarray, want: np.ndarray) -> bool:
    g, w = got.view(np.uint32), want.view(np.uint32)
    nan = np.isnan(want)
    return bool(np.array_equal(np.isnan(got), nan) and np.array_equal(g[~nan], w[~nan]))


@pytest.mark.parametrize("qtype", TYPES, ids=lambda t: NAMES[t])
def test_known_answers(tc, goldens, qtype):
    g = goldens["dequant"]
    name = NAMES[qtype]
    out = tc.gguf_tensor_to_f32(qtype, dev(g[f"kat_{name}_blocks"])).cpu().numpy()
    assert np.array_equal(out, g[f"kat_{name}_out"])
    assert tc.device_error() == 0


@pytest.mark.parametrize("qtype", TYPES, ids=lambda t: NAMES[t])
def test_random_blocks_ragged_tail_golden(tc, goldens, qtype):
    """257 blocks: one full run plus a 1-block tail staged without the bulk copy."""
    g = goldens["dequant"]
    name = NAMES[qtype]
    out = tc.gguf_tensor_to_f32(qtype, dev(g[f"rand_{name}_blocks"])).cpu().numpy()
    assert bits_equal(out, g[f"rand_{name}_out"])


@pytest.mark.parametrize("qtype", TYPES, ids=lambda t: NAMES[t])
def test_full_config_tensor_bitwise(tc, qtype):
    """One 4096 x 11008 tensor per format (the dequant bandwidth workload)."""
    n_blocks = 4096 * 11008 // 32
    blocks = synth.random_blocks(qtype, n_blocks, seed=2024 + qtype)
    out = tc.gguf_tensor_to_f32(qtype, dev(blocks)).cpu().numpy()
    want = oracle.dequant(qtype, blocks)
    assert bits_equal(out, want)
    assert tc.device_error() == 0


@pytest.mark.parametrize("qtype", TYPES, ids=lambda t: NAMES[t])
def test_extreme_scales(tc, qtype):
    """Subnormal, maximal, zero, negative-zero, infinite and NaN fp16 scales."""
    blocks = synth.random_blocks(qtype, 300, seed=5)
    v = blocks.reshape(300, -1)
    specials = [0x0001, 0x03FF, 0x0400, 0x7BFF, 0x8001, 0xFBFF, 0x0000, 0x8000, 0x7C00, 0xFC00, 0x7E00, 0x7C01]
    for i, d in enumerate(specials):
        v[i, 0:2] = np.frombuffer(np.uint16(d).tobytes(), dtype=np.uint8)
        if qtype in (synth.TYPE_Q4_1, synth.TYPE_Q5_1):
            v[i + 20, 2:4] = np.frombuffer(np.uint16(d).tobytes(), dtype=np.uint8)  # the m field
    out = tc.gguf_tensor_to_f32(qtype, dev(blocks)).cpu().numpy()
    assert bits_equal(out, oracle.dequant(qtype, blocks))


@pytest.mark.parametrize("qtype", TYPES, ids=lambda t: NAMES[t])
def test_unaligned_buffers(tc, qtype):
    """Packed source 2 bytes past a 16-byte boundary and output 4 bytes past one: the kernel falls
    back to plain loads / scalar stores."""
    n = 1000
    blocks = synth.random_blocks(qtype, n, seed=77)
    raw = torch.zeros(blocks.size + 16, dtype=torch.uint8, device="cuda")
    raw[2:2 + blocks.size] = dev(blocks)
    out_raw = torch.zeros(n * 32 + 4, dtype=torch.float32, device="cuda")
    src = raw[2:2 + blocks.size]
    out = out_raw[1:1 + n * 32]
    tc.gguf_tensor_to_f32(qtype, src, out=out)
    assert bits_equal(out.cpu().numpy(), oracle.dequant(qtype, blocks))


def test_batch_alternating_output_alignment(tc):
    """Twenty jobs of 64 runs each (128 blocks per run) in one launch, outputs alternately 16-byte
    aligned (written by bulk copies from shared memory) and 4 bytes off (plain stores): every CTA
    handles several runs, so a plain-store run sits between bulk-copy runs that reuse the CTA's
    two output buffers."""
    jobs, want = [], []
    for j in range(20):
        t = TYPES[j % len(TYPES)]
        n = 64 * 128 - (j % 3) * 37                       # ragged last run in some jobs
        blocks = synth.random_blocks(t, n, seed=500 + j)
        base = torch.full((n * 32 + 4,), float("nan"), device="cuda")
        out = base[1:1 + n * 32] if j % 2 else base[: n * 32]
        jobs.append((t, dev(blocks), out))
        want.append(oracle.dequant(t, blocks))
    tc.dequantize_many(jobs)
    torch.cuda.synchronize()
    assert tc.device_error() == 0
    for (t, _, out), w in zip(jobs, want):
        assert bits_equal(out.cpu().numpy(), w), t


def test_batched_jobs_whole_model_slice(tc):
    """trc_cuda_dequant_many over a mixed set of tensors (the whole-model workload's formats and
    row shapes, at reduced row counts) in one launch."""
    shapes = [(synth.TYPE_Q5_1, 4096 * 64), (synth.TYPE_Q8_0, 4096 * 32), (synth.TYPE_Q4_0, 4096 * 96),
              (synth.TYPE_Q4_0, 11008 * 8), (synth.TYPE_Q8_0, 32 * 3), (synth.TYPE_Q5_1, 4096 * 64)]
    jobs, wants, outs = [], [], []
    for i, (t, n) in enumerate(shapes):
        b = synth.random_blocks(t, n // 32, seed=300 + i)
        o = torch.empty(n, dtype=torch.float32, device="cuda")
        jobs.append((t, dev(b), o))
        outs.append(o)
        wants.append(oracle.dequant(t, b))
    tc.dequantize_many(jobs)
    for o, w in zip(outs, wants):
        assert bits_equal(o.cpu().numpy(), w)


def test_prepared_batch_replays_and_spans_launches(tc):
    """DequantBatch: 300 jobs (more than one launch holds) built once and replayed; each replay
    rewrites every output bit-exactly, device-generated blocks included."""
    gen = torch.Generator(device="cuda").manual_seed(5)
    jobs, outs = [], []
    for i in range(300):
        t = TYPES[i % len(TYPES)]
        n_blocks = 4096 // 32 + (i % 7) * 3
        b = synth.random_blocks_torch(t, n_blocks, gen, "cuda")
        o = torch.empty(n_blocks * 32, dtype=torch.float32, device="cuda")
        jobs.append((t, b, o))
        outs.append(o)
    batch = tc.DequantBatch(jobs)
    assert len(batch) == 300
    launches = tc.launch_count()
    batch()
    assert tc.launch_count() - launches == 2
    for o in outs:
        o.fill_(float("nan"))
    batch()
    torch.cuda.synchronize()
    for (t, b, o) in jobs[::23]:
        assert bits_equal(o.cpu().numpy(), oracle.dequant(t, b.cpu().numpy()))
    assert tc.device_error() == 0


def test_load_from_pinned_host(tc):
    t = synth.TYPE_Q5_0
    n_blocks = 4096 * 64 // 32
    blocks = synth.random_blocks(t, n_blocks, seed=8)
    host = torch.from_numpy(blocks).pin_memory()
    staging = torch.empty(blocks.size, dtype=torch.uint8, device="cuda")
    dst = torch.empty(n_blocks * 32, dtype=torch.float32, device="cuda")
    tc.gguf_load_tensor(t, host, dst, staging)
    assert bits_equal(dst.cpu().numpy(), oracle.dequant(t, blocks))


def test_pipelined_upload_large_tensors_share_staging(tc):
    """Uploads of 16 MB or more cross PCIe in chunks on a second stream while the caller's stream
    dequantizes the chunks already landed. Two large tensors through ONE staging buffer, back to
    back: the second upload may not overwrite staging before the first dequant has read it."""
    jobs = [(synth.TYPE_Q8_0, 4096 * 11008 // 32, 31), (synth.TYPE_Q4_1, 4096 * 11008 // 32 + 77, 32)]
    host = [torch.from_numpy(synth.random_blocks(t, n, seed=sd)).pin_memory() for t, n, sd in jobs]
    staging = torch.empty(max(h.numel() for h in host), dtype=torch.uint8, device="cuda")
    outs = [torch.full((n * 32,), float("nan"), device="cuda") for _, n, _ in jobs]
    for _ in range(2):
        for (t, _, _), h, o in zip(jobs, host, outs):
            tc.gguf_load_tensor(t, h, o, staging)
    torch.cuda.synchronize()
    assert tc.device_error() == 0
    for (t, n, _), h, o in zip(jobs, host, outs):
        assert bits_equal(o.cpu().numpy(), oracle.dequant(t, h.numpy(), n))


def test_rejections(tc):
    blocks = dev(synth.random_blocks(synth.TYPE_Q4_0, 4, seed=1))
    with pytest.raises(tc.TrcCudaError):
        tc.gguf_tensor_to_f32(synth.TYPE_Q4_0, blocks, n_elems=30)  # ragged: not whole blocks
    with pytest.raises(tc.TrcCudaError):
        tc.gguf_tensor_to_f32(10, blocks)  # Q2_K: not a legacy format (the reference rejects it too)
    out = torch.empty(32, device="cuda")
    assert tc.lib().trc_cuda_dequant(10, blocks.data_ptr(), 1, out.data_ptr(), None) == -2
    assert tc.lib().trc_cuda_dequant(2, blocks.data_ptr(), -1, out.data_ptr(), None) == -1
    assert tc.lib().trc_cuda_dequant(2, blocks.data_ptr(), 0, out.data_ptr(), None) == 0


def test_loader_wrappers_reject_bad_device_destinations(tc):
    """A half/bf16 destination would be written past its end, a ragged or strided one partly:
    the loader wrappers refuse them (and a device tensor passed as the host source)."""
    host = torch.from_numpy(synth.random_blocks(synth.TYPE_Q4_0, 2, seed=3))
    staging = torch.empty(64, dtype=torch.uint8, device="cuda")
    bad = [torch.empty(64, dtype=torch.float16, device="cuda"), torch.empty(64, dtype=torch.bfloat16, device="cuda"),
           torch.empty(48, device="cuda"), torch.empty(128, device="cuda")[::2]]
    for dst in bad:
        with pytest.raises(tc.TrcCudaError):
            tc.gguf_load_tensor(synth.TYPE_Q4_0, host, dst, staging)
        with pytest.raises(tc.TrcCudaError):
            tc.gguf_load_tensor_static(synth.TYPE_Q4_0, host, dst)
    with pytest.raises(tc.TrcCudaError, match="host memory"):
        tc.gguf_load_tensor_static(synth.TYPE_Q4_0, host.cuda(), torch.empty(64, device="cuda"))
    with pytest.raises(tc.TrcCudaError):
        tc.gguf_tensor_to_f32(synth.TYPE_Q4_0, dev(host.numpy()), out=torch.empty(64, dtype=torch.float16, device="cuda"))
    assert tc.device_error() == 0


def test_peer_store_kernel_on_one_gpu(tc):
    """The dequant variant that writes every output also at the same offset of other buffers
    (trc_cuda_dequant_many_to_peers: the all-gather fused into the dequant, one peer per other
    GPU). Here the "peer" is a second buffer on the same GPU, so the kernel runs on one device:
    all five formats, a ragged tail, both copies bit-exact with the reference dequantizers."""
    import ctypes

    jobs, total = [], 0
    for i, qtype in enumerate(synth.BLOCK_BYTES):
        n_blocks = 3000 + 77 * i                                  # not a multiple of a run
        jobs.append((qtype, synth.random_blocks(qtype, n_blocks, seed=300 + i), total, n_blocks))
        total += n_blocks * 32
    local = torch.full((total,), float("nan"), device="cuda")
    mirror = torch.full((total,), float("nan"), device="cuda")
    packed = [dev(b) for _, b, _, _ in jobs]
    arr = (tc.DequantJob * len(jobs))()
    for k, ((qtype, _, off, n_blocks), p) in enumerate(zip(jobs, packed)):
        arr[k].blocks = p.data_ptr()
        arr[k].out = local.data_ptr() + 4 * off
        arr[k].n_blocks = n_blocks
        arr[k].type = qtype
    peers = (ctypes.c_void_p * 1)(mirror.data_ptr())
    st = tc.lib().trc_cuda_dequant_many_to_peers(arr, len(jobs), ctypes.c_void_p(local.data_ptr()), peers, 1, None)
    assert st == 0
    torch.cuda.synchronize()
    assert tc.device_error() == 0
    got_l, got_m = local.cpu().numpy(), mirror.cpu().numpy()
    for qtype, blocks, off, n_blocks in jobs:
        want = oracle.dequant(qtype, blocks, n_blocks)
        assert bits_equal(got_l[off:off + n_blocks * 32], want), qtype
        assert bits_equal(got_m[off:off + n_blocks * 32], want), qtype
