"""Token-balanced sequence partition of a packed batch over the GPUs of one node.

Sequences are independent units of packed attention, so a batch shards with no collective
on the hot path: each rank gets whole sequences, builds its own ``cu_seqlens`` and runs the
kernels on them. The assignment is LPT (longest processing time first): sequences sorted
by cost, descending, each given to the least-loaded rank. Cost of a sequence of length L
over a layer pattern is ``alpha * L + beta * pairs(L)``: ``alpha`` weights the per-token
work (projections, loads) and ``beta`` the per-pair attention work.

The optional ``gather_pooled`` collects per-sequence pooled embeddings on every rank in the
original order (one NCCL ``all_gather`` per batch, off the hot path).
"""

from __future__ import annotations

import heapq
from dataclasses import dataclass
from typing import Sequence

import torch


def band_pairs(length: int, window: tuple[int, int] = (-1, -1), causal: bool = False) -> int:
    """Allowed query-key pairs of one head of one sequence (runtime/attention.py:157-170 band)."""
    left, right = window
    right = 0 if causal else right
    if left < 0 and right < 0:
        return length * length
    total = 0
    for i in range(length):
        lo = max(0, i - left) if left >= 0 else 0
        hi = min(length - 1, i + right) if right >= 0 else length - 1
        total += hi - lo + 1
    return total


def pattern_cost(length: int, layers: Sequence[tuple[tuple[int, int], bool]], alpha: float = 0.0,
                 beta: float = 1.0) -> float:
    return sum(alpha * length + beta * band_pairs(length, w, c) for w, c in layers)


@dataclass(frozen=True)
class Shard:
    rank: int
    indices: tuple[int, ...]   # original sequence indices, in the order they are packed on this rank
    lengths: tuple[int, ...]
    load: float

    @property
    def tokens(self) -> int:
        return sum(self.lengths)

    def cu_seqlens(self, device=None) -> torch.Tensor:
        cu = torch.zeros(len(self.lengths) + 1, dtype=torch.int32)
        if self.lengths:
            cu[1:] = torch.tensor(self.lengths, dtype=torch.int64).cumsum(0).to(torch.int32)
        return cu if device is None else cu.to(device)


def partition(lengths: Sequence[int], world: int, costs: Sequence[float] | None = None) -> list[Shard]:
    """LPT assignment of sequences to ``world`` ranks; deterministic (ties by index / rank)."""
    if world < 1:
        raise ValueError("world must be >= 1")
    lengths = [int(n) for n in lengths]
    costs = [float(n) for n in lengths] if costs is None else [float(c) for c in costs]
    if len(costs) != len(lengths):
        raise ValueError("costs and lengths differ in size")
    order = sorted(range(len(lengths)), key=lambda i: (-costs[i], i))
    heap = [(0.0, r) for r in range(world)]
    buckets: list[list[int]] = [[] for _ in range(world)]
    loads = [0.0] * world
    for i in order:
        load, r = heapq.heappop(heap)
        buckets[r].append(i)
        loads[r] = load + costs[i]
        heapq.heappush(heap, (loads[r], r))
    shards = []
    for r in range(world):
        idx = tuple(sorted(buckets[r]))  # keep original relative order inside a rank
        shards.append(Shard(r, idx, tuple(lengths[i] for i in idx), loads[r]))
    return shards


def gather_pooled(pooled: torch.Tensor, shard: Shard, shards: Sequence[Shard], group=None) -> torch.Tensor:
    """All-gather per-sequence rows ``[n_local, hidden]`` from every rank into the original
    order ``[n_total, hidden]``. Pads each rank's block to the largest rank count so a single
    ``all_gather_into_tensor`` (NCCL on GPUs, Gloo on CPU) moves it."""
    import torch.distributed as dist

    world = len(shards)
    width = max(len(s.indices) for s in shards)
    hidden = pooled.shape[1]
    block = pooled.new_zeros(width, hidden)
    block[: pooled.shape[0]] = pooled
    if dist.get_backend(group) == "gloo":
        parts = [torch.empty_like(block) for _ in range(world)]
        dist.all_gather(parts, block, group=group)
        stacked = torch.stack(parts)
    else:
        stacked = block.new_empty(world * width, hidden)
        dist.all_gather_into_tensor(stacked, block, group=group)
        stacked = stacked.view(world, width, hidden)
    n_total = sum(len(s.indices) for s in shards)
    out = pooled.new_empty(n_total, hidden)
    for s in shards:
        if s.indices:
            index = torch.tensor(s.indices, device=out.device)
            out.index_copy_(0, index, stacked[s.rank, : len(s.indices)])
    return out
