"""CPU, world_size 2 over gloo: the multi-GPU host logic. Both ranks derive the same partition
with no exchange, the shards cover every unit exactly once, and the per-rank results of the
sharded work (computed here by the oracle in place of the device) reassemble into the
single-process result bit for bit."""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle
import sharding
import synth


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int, q) -> None:
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        # whole-model style: tensors of mixed formats, partitioned by algorithmic bytes
        tensors = [(synth.TYPE_Q5_1, 4096 * 8), (synth.TYPE_Q8_0, 4096 * 4), (synth.TYPE_Q4_0, 11008 * 2),
                   (synth.TYPE_Q4_0, 4096 * 6), (synth.TYPE_Q8_0, 4096 * 4), (synth.TYPE_Q4_0, 4096 * 2),
                   (synth.TYPE_Q5_1, 4096 * 8)]
        sizes = [n // 32 * (synth.BLOCK_BYTES[t] + 128) for t, n in tensors]
        plan = sharding.lpt_shards(sizes, world)
        plans = [None] * world
        dist.all_gather_object(plans, plan)
        mine = {}
        for i in plan[rank]:
            t, n = tensors[i]
            mine[i] = oracle.dequant(t, synth.random_blocks(t, n // 32, seed=i)).tobytes()
        gathered = [None] * world
        dist.all_gather_object(gathered, mine)
        # GQA-style batched mul_mat sharded by ne[3]
        rng = np.random.default_rng(0)
        A = rng.standard_normal((4, 2, 24, 16)).astype(np.float32)  # ne [16, 24, 2, 4]
        B = rng.standard_normal((4, 8, 20, 16)).astype(np.float32)  # ne [16, 20, 8, 4]
        pr = sharding.plane_range(4, rank, world)
        part = oracle.mul_mat(A[pr.start:pr.stop], B[pr.start:pr.stop], n_threads=1)
        parts = [None] * world
        dist.all_gather_object(parts, (pr.start, pr.stop, part))
        q.put((rank, plans, gathered, parts, tensors, sizes, A, B))
    finally:
        dist.destroy_process_group()


def test_two_rank_sharding_over_gloo():
    world = 2
    port = _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    rank, plans, gathered, parts, tensors, sizes, A, B = results[0]
    # identical plans without exchange; exact cover
    assert plans[0] == plans[1]
    covered = sorted(i for s in plans[0] for i in s)
    assert covered == list(range(len(tensors)))
    assert sharding.imbalance(sizes, plans[0]) < 1.5
    merged = {}
    for g in gathered:
        assert not (set(g) & set(merged))
        merged.update(g)
    for i, (t, n) in enumerate(tensors):
        want = oracle.dequant(t, synth.random_blocks(t, n // 32, seed=i)).tobytes()
        assert merged[i] == want
    full = oracle.mul_mat(A, B, n_threads=1)
    stitched = np.concatenate([p[2] for p in sorted(parts, key=lambda x: x[0])], axis=0)
    assert np.array_equal(stitched.view(np.uint32), full.view(np.uint32))


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_lpt_plan_of_whole_model(world):
    ts = synth.llama7b_tensors()
    sizes = [ne[0] * ne[1] // 32 * (synth.BLOCK_BYTES[t] + 128) for _, t, ne in ts]
    plan = sharding.lpt_shards(sizes, world)
    assert sorted(i for s in plan for i in s) == list(range(len(ts)))
    assert len(ts) == 226
    assert sharding.imbalance(sizes, plan) < 1.05
    assert sum(sizes) == 31_865_700_352  # 6,738,149,376 weights: 4.913 GB packed + 26.95 GB F32


def test_plane_ranges_cover():
    for world in (1, 2, 4, 8):
        rs = [sharding.plane_range(8, r, world) for r in range(world)]
        assert [i for r in rs for i in r] == list(range(8))
