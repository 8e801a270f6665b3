"""One rank of the dequant all-gather parity check (run by tests/test_gpu_peers.py under
torchrun, one process per GPU): each rank dequantizes its own row range of two tensors straight
into every rank's buffer over NVLink (trc_cuda_dequant_many_to_peers), then checks the whole
buffer against the oracle, bit for bit."""
from __future__ import annotations

import os
import sys
from datetime import timedelta
from pathlib import Path

import numpy as np
import torch
import torch.distributed as dist

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT / "train.cpp_b200"))
sys.path.insert(0, str(ROOT / "oracle"))

import oracle  # noqa: E402
import sharding  # noqa: E402
import synth  # noqa: E402
import trc_cuda as tc  # noqa: E402

# (type, ne0, rows): a ragged row count so that the shards differ in size
TENSORS = [(synth.TYPE_Q5_1, 4096, 1001), (synth.TYPE_Q8_0, 1024, 77)]


def main() -> int:
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=timedelta(seconds=60), device_id=torch.device("cuda", local))
    total = sum(ne0 * rows for _, ne0, rows in TENSORS)
    buf = tc.PeerBuffer(total * 4)
    full = buf.tensor()
    full.fill_(float("nan"))
    torch.cuda.synchronize()
    dist.barrier()
    jobs, wants, off = [], [], 0
    for i, (t, ne0, rows) in enumerate(TENSORS):
        packed = synth.random_blocks(t, ne0 * rows // 32, seed=40 + i)  # identical on every rank
        wants.append(oracle.dequant(t, packed))
        rr = sharding.plane_range(rows, rank, world)
        bb = synth.BLOCK_BYTES[t]
        row_bytes = ne0 // 32 * bb
        mine = torch.from_numpy(packed[rr.start * row_bytes: rr.stop * row_bytes].copy()).cuda()
        jobs.append((t, mine, full[off + rr.start * ne0: off + rr.stop * ne0]))
        off += ne0 * rows
    tc.dequantize_to_peers(jobs, buf)
    torch.cuda.synchronize()
    dist.barrier()
    got = full.cpu().numpy()
    ok = np.array_equal(got.view(np.uint32), np.concatenate(wants).view(np.uint32))
    err = tc.device_error()
    dist.barrier()
    buf.close()
    dist.destroy_process_group()
    print(f"rank {rank}: {'OK' if ok and err == 0 else 'MISMATCH'} (device_error {err})", flush=True)
    return 0 if ok and err == 0 else 1


if __name__ == "__main__":
    sys.exit(main())
