"""Replica data parallelism for batched independent-sequence decode.

One process per GPU.  The global set of sequences is partitioned into
contiguous per-rank shards; every rank holds a full copy of the weights and
its own sequences' KV caches.  Nothing is exchanged on the token path: the
only collectives are the host-side timing barrier and the max/sum reductions
of per-rank timings and counts, which run outside the decode loop.
"""
from __future__ import annotations

import os
from datetime import timedelta


def shard(total: int, rank: int, world: int) -> range:
    """Contiguous slice of [0, total) owned by `rank` (sizes differ by <= 1)."""
    if world <= 0 or not (0 <= rank < world):
        raise ValueError("bad rank/world")
    base, extra = divmod(total, world)
    start = rank * base + min(rank, extra)
    return range(start, start + base + (1 if rank < extra else 0))


def sequence_seed(global_index: int, base: int = 10_000) -> int:
    """Prompt seed of global sequence g: the same sequence gets the same prompt
    whichever rank (and however many ranks) decode it."""
    return base + int(global_index)


def env_rank():
    return (int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)),
            int(os.environ.get("LOCAL_RANK", 0)))


class Group:
    """Thin wrapper over torch.distributed for the bench's host-side sync."""

    def __init__(self, backend: str | None = None, timeout_s: int = 300):
        import torch
        import torch.distributed as dist

        self.dist = dist
        self.torch = torch
        self.rank, self.world, self.local_rank = env_rank()
        self.active = self.world > 1
        self.backend = backend or ("nccl" if torch.cuda.is_available() else "gloo")
        if self.active and not dist.is_initialized():
            kw = {"backend": self.backend, "timeout": timedelta(seconds=timeout_s)}
            if self.backend == "nccl":
                torch.cuda.set_device(self.local_rank)
                kw["device_id"] = torch.device("cuda", self.local_rank)
            dist.init_process_group(**kw)

    def _dev(self):
        if self.backend == "nccl":
            return self.torch.device("cuda", self.local_rank)
        return self.torch.device("cpu")

    def barrier(self):
        if self.active:
            self.dist.barrier()

    def reduce_max(self, x: float) -> float:
        if not self.active:
            return float(x)
        t = self.torch.tensor([float(x)], dtype=self.torch.float64, device=self._dev())
        self.dist.all_reduce(t, op=self.dist.ReduceOp.MAX)
        return float(t.item())

    def reduce_sum(self, x: float) -> float:
        if not self.active:
            return float(x)
        t = self.torch.tensor([float(x)], dtype=self.torch.float64, device=self._dev())
        self.dist.all_reduce(t, op=self.dist.ReduceOp.SUM)
        return float(t.item())

    def gather_ints(self, values):
        """All ranks' int lists, concatenated in rank order (equal lengths)."""
        if not self.active:
            return list(values)
        t = self.torch.tensor(list(values), dtype=self.torch.int64, device=self._dev())
        out = [self.torch.empty_like(t) for _ in range(self.world)]
        self.dist.all_gather(out, t)
        return [int(v) for o in out for v in o.tolist()]

    def close(self):
        if self.active and self.dist.is_initialized():
            self.dist.destroy_process_group()
