"""Data-parallel serving across the GPUs of one node: one model replica per GPU, independent requests sharded by
expected work, no collective on the hot path (the reference shards the same way: ``src/infer_omnidocbench.py:359-364``,
SGLang DP=8).  ``torch.distributed`` is used only around the timed region (barrier, max of the per-rank device times,
sum of committed tokens)."""
from __future__ import annotations

import heapq
import os
from datetime import timedelta
from typing import List, Sequence, Tuple

import torch
import torch.distributed as dist


def lpt_shards(work: Sequence[float], n: int) -> List[List[int]]:
    """Longest-processing-time-first partition of request indices into n shards (deterministic: ties by index)."""
    heap = [(0.0, r) for r in range(n)]
    shards: List[List[int]] = [[] for _ in range(n)]
    for i in sorted(range(len(work)), key=lambda i: (-work[i], i)):
        load, r = heapq.heappop(heap)
        shards[r].append(i)
        heapq.heappush(heap, (load + float(work[i]), r))
    return [sorted(s) for s in shards]


def dist_env() -> Tuple[int, int, int]:
    """(rank, world_size, local_rank) from the torchrun environment (1-process defaults)."""
    return int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)), int(os.environ.get("LOCAL_RANK", 0))


def init(backend: str, timeout_s: float = 120.0) -> None:
    rank, world, _ = dist_env()
    if world > 1 and not dist.is_initialized():
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        dist.init_process_group(backend=backend, rank=rank, world_size=world, timeout=timedelta(seconds=timeout_s))


def barrier(device=None) -> None:
    if dist.is_initialized():
        if device is not None and dist.get_backend() == "nccl":
            dist.barrier(device_ids=[device.index])
        else:
            dist.barrier()


def max_over_ranks(x: float, device=None) -> float:
    if not dist.is_initialized():
        return x
    t = torch.tensor([x], dtype=torch.float64, device=device if dist.get_backend() == "nccl" else "cpu")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def sum_over_ranks(x: float, device=None) -> float:
    if not dist.is_initialized():
        return x
    t = torch.tensor([x], dtype=torch.float64, device=device if dist.get_backend() == "nccl" else "cpu")
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return float(t.item())


def gather_objects(obj) -> list:
    """Every rank's `obj`, in rank order (outside the timed region only)."""
    if not dist.is_initialized():
        return [obj]
    out = [None] * dist.get_world_size()
    dist.all_gather_object(out, obj)
    return out


def finish() -> None:
    if dist.is_initialized():
        dist.destroy_process_group()


def balanced_shards(work: Sequence[float], n: int) -> List[List[int]]:
    """Equal-count shards (every replica runs the same batch size) with loads balanced by snake order over the
    requests sorted by expected work."""
    order = sorted(range(len(work)), key=lambda i: (-work[i], i))
    shards: List[List[int]] = [[] for _ in range(n)]
    for k, i in enumerate(order):
        r = k % (2 * n)
        shards[r if r < n else 2 * n - 1 - r].append(i)
    return [sorted(s) for s in shards]
