"""Work partitioning of the hot path across GPUs (one process per GPU, no data-path collective).

* Whole-model dequantization shards by tensor: a byte-balanced greedy LPT over the tensors'
  algorithmic bytes (packed + F32), identical on every rank because it is a pure function of the
  tensor list.
* Batched mul_mat (and its composed backward) shards by ne[3]: rank r owns a contiguous range of
  i3 planes. Every plane of b (and its a-plane i3 % a3) lives on one rank, and repeat_back only
  reduces over ne[2], so the backward stays local.
"""
from __future__ import annotations

from typing import Sequence


def lpt_shards(sizes: Sequence[int], n_shards: int) -> list[list[int]]:
    """Greedy longest-processing-time partition of item indices by size; ties by index."""
    order = sorted(range(len(sizes)), key=lambda i: (-sizes[i], i))
    loads = [0] * n_shards
    shards: list[list[int]] = [[] for _ in range(n_shards)]
    for i in order:
        s = min(range(n_shards), key=lambda k: (loads[k], k))
        shards[s].append(i)
        loads[s] += sizes[i]
    for s in shards:
        s.sort()
    return shards


def plane_range(n3: int, rank: int, world: int) -> range:
    """Contiguous i3 planes owned by `rank` when ne[3] = n3 is split over `world` ranks."""
    lo = n3 * rank // world
    hi = n3 * (rank + 1) // world
    return range(lo, hi)


def imbalance(sizes: Sequence[int], shards: list[list[int]]) -> float:
    """max shard load / mean shard load (1.0 = perfect balance)."""
    loads = [sum(sizes[i] for i in s) for s in shards]
    mean = sum(loads) / max(1, len(loads))
    return max(loads) / mean if mean > 0 else 1.0
