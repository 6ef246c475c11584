"""Data-parallel decode across the GPUs of one box: one process per GPU, sequences partitioned, no collective on the
data path (the reference runs one replica per GPU the same way: its model code refuses tensor parallelism,
plugins/vllm_lrkv/vllm_lrkv/models/qwen3_5_latent.py:101-102, and README.md:90 serves one replica per GPU).

Every decode sequence is independent: a rank holds the 16 layers' factors (a few MB per layer), the paged cache of its
own sequences, and runs the whole decode step on them. The only cross-rank traffic is host-side: a barrier that starts
a timed region on all ranks together and the maximum of the per-rank times.

* ``partition_lpt``: longest-processing-time split by context tokens with equal request counts per rank (at most one
  apart), so that every rank's step takes about the same time;
* ``partition_even``: contiguous split by count (the naive baseline, for comparison);
* ``HostGroup``: rank / world from the launcher's environment (torchrun's ``RANK``, ``WORLD_SIZE``, ``LOCAL_RANK``,
  ``MASTER_ADDR``/``MASTER_PORT``), a gloo process group with a short timeout, ``barrier`` and ``max``.
"""

from __future__ import annotations

import heapq
import os
from datetime import timedelta


def partition_lpt(lengths, world: int) -> list:
    """Indices of ``lengths`` per rank: requests longest first, each to the rank with the fewest context tokens among
    those still below their count quota (ceil or floor of len / world). Deterministic (ties go to the lower rank)."""
    n = len(lengths)
    if world < 1:
        raise ValueError("world must be >= 1")
    base, extra = divmod(n, world)
    quota = [base + (1 if r < extra else 0) for r in range(world)]
    order = sorted(range(n), key=lambda i: (-int(lengths[i]), i))
    heap = [(0, r) for r in range(world) if quota[r] > 0]
    heapq.heapify(heap)
    parts = [[] for _ in range(world)]
    for i in order:
        tokens, r = heapq.heappop(heap)
        parts[r].append(i)
        if len(parts[r]) < quota[r]:
            heapq.heappush(heap, (tokens + int(lengths[i]), r))
    return [sorted(p) for p in parts]


def partition_even(lengths, world: int) -> list:
    """Contiguous split by count: rank r gets requests [r * n / world, (r + 1) * n / world)."""
    n = len(lengths)
    return [list(range(r * n // world, (r + 1) * n // world)) for r in range(world)]


def imbalance(lengths, parts) -> float:
    """max over ranks of the rank's context tokens / the mean (1.0 = perfectly balanced)."""
    tot = [sum(int(lengths[i]) for i in p) for p in parts]
    mean = sum(tot) / max(1, len(tot))
    return max(tot) / mean if mean else 1.0


class HostGroup:
    """The ranks of one data-parallel run, from the launcher's environment. With a world of one nothing is
    initialised; otherwise a gloo group over ``MASTER_ADDR`` (default 127.0.0.1) whose calls fail after ``timeout_s``
    if a rank never joins, instead of waiting for good."""

    def __init__(self, timeout_s: float = 120.0):
        self.rank = int(os.environ.get("RANK", 0))
        self.world = int(os.environ.get("WORLD_SIZE", 1))
        self.local_rank = int(os.environ.get("LOCAL_RANK", 0))
        self.dist = None
        if self.world > 1:
            import torch.distributed as dist
            os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
            dist.init_process_group("gloo", rank=self.rank, world_size=self.world,
                                    timeout=timedelta(seconds=timeout_s))
            self.dist = dist

    def barrier(self) -> None:
        if self.dist is not None:
            self.dist.barrier()

    def max(self, x: float) -> float:
        if self.dist is None:
            return float(x)
        import torch
        t = torch.tensor([float(x)], dtype=torch.float64)
        self.dist.all_reduce(t, op=self.dist.ReduceOp.MAX)
        return float(t.item())

    def sum(self, x: float) -> float:
        if self.dist is None:
            return float(x)
        import torch
        t = torch.tensor([float(x)], dtype=torch.float64)
        self.dist.all_reduce(t, op=self.dist.ReduceOp.SUM)
        return float(t.item())

    def gather_float(self, x: float) -> list:
        """Every rank's ``x``, in rank order (a one-element list on a single rank)."""
        if self.dist is None:
            return [float(x)]
        import torch
        out = [torch.zeros(1, dtype=torch.float64) for _ in range(self.world)]
        self.dist.all_gather(out, torch.tensor([float(x)], dtype=torch.float64))
        return [float(t.item()) for t in out]

    def close(self) -> None:
        if self.dist is not None:
            self.dist.destroy_process_group()
            self.dist = None
