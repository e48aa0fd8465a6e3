"""Data-parallel plumbing with the reference's interface (distributed.py:1-72).

The reference runs one process per GPU: each rank decodes the prompts
``range(rank, N, size)`` (benchmark.py:175) and the pickled results are
gathered to rank 0 once at the end (benchmark.py:237-241).  Nothing in a
decoding step crosses GPUs, so this module is only the process plumbing;
the same function names and return conventions as the reference are kept
so its harness can import this module instead.  ``init`` takes the backend
as an argument (``"nccl"`` by default, ``"gloo"`` for CPU processes) and an
optional timeout; without ``RANK`` in the environment it warns and stays
single-process, like the reference.
"""
from __future__ import annotations

import os
import warnings
from datetime import timedelta
from typing import Any, Dict, Iterable, List, Optional

from torch import distributed as dist

__all__ = [
    "init",
    "is_initialized",
    "size",
    "rank",
    "local_size",
    "local_rank",
    "is_main",
    "barrier",
    "gather",
    "all_gather",
    "shard_indices",
    "gather_counters",
    "merge_counters",
]


def init(backend: str = "nccl", timeout: timedelta = timedelta(minutes=300)) -> None:
    """Join the process group from ``env://`` (distributed.py:18-22)."""
    if "RANK" not in os.environ:
        warnings.warn("Environment variable `RANK` is not set. Skipping distributed initialization.")
        return
    dist.init_process_group(backend=backend, init_method="env://", timeout=timeout)


def is_initialized() -> bool:
    return dist.is_initialized()


def size() -> int:
    return int(os.environ.get("WORLD_SIZE", 1))


def rank() -> int:
    return int(os.environ.get("RANK", 0))


def local_size() -> int:
    return int(os.environ.get("LOCAL_WORLD_SIZE", 1))


def local_rank() -> int:
    return int(os.environ.get("LOCAL_RANK", 0))


def is_main() -> bool:
    return rank() == 0


def barrier() -> None:
    if not is_initialized():
        return
    dist.barrier()


def gather(obj: Any, dst: int = 0) -> Optional[List[Any]]:
    """Rank-ordered list of every rank's ``obj`` on ``dst``, None elsewhere
    (distributed.py:55-64); ``[obj]`` when not initialised."""
    if not is_initialized():
        return [obj]
    if rank() == dst:
        objs: List[Any] = [None for _ in range(size())]
        dist.gather_object(obj, objs, dst=dst)
        return objs
    dist.gather_object(obj, dst=dst)
    return None


def all_gather(obj: Any) -> List[Any]:
    """Rank-ordered list of every rank's ``obj`` on every rank (distributed.py:67-72)."""
    if not is_initialized():
        return [obj]
    objs: List[Any] = [None for _ in range(size())]
    dist.all_gather_object(objs, obj)
    return objs


def shard_indices(n: int, rank_: Optional[int] = None, size_: Optional[int] = None) -> range:
    """The prompts this rank decodes: ``range(rank, n, size)`` (benchmark.py:175)."""
    r = rank() if rank_ is None else rank_
    s = size() if size_ is None else size_
    if s <= 0 or not 0 <= r < s:
        raise ValueError(f"rank {r} outside world of size {s}")
    return range(r, n, s)


def gather_counters(values, device=None):
    """Every rank's fixed-size counter vector, gathered in one collective.

    The reference gathers pickled response objects to rank 0
    (distributed.py:55-64, benchmark.py:237-241); the counters its analysis
    needs (tokens, rounds, accepted lengths, times) are fixed-size numbers,
    so here each rank contributes one float64 vector and a single
    ``all_gather_into_tensor`` (NCCL over NVLink for CUDA tensors, gloo on
    CPU) returns the [world, n] matrix on every rank.  Single-process: the
    [1, n] matrix of this rank."""
    import torch
    vec = torch.as_tensor(values, dtype=torch.float64)
    if device is not None:
        vec = vec.to(device)
    if not is_initialized():
        return vec.unsqueeze(0)
    out = torch.empty((dist.get_world_size() * vec.numel(),), dtype=torch.float64, device=vec.device)
    dist.all_gather_into_tensor(out, vec.contiguous())
    return out.view(dist.get_world_size(), vec.numel())


def merge_counters(per_rank: Iterable[Dict[str, float]]) -> Dict[str, float]:
    """Sum per-rank counters (tokens, steps, accepted lengths, times) after a
    ``gather``; the reference derives its acceptance and throughput figures
    from such totals over all responses."""
    total: Dict[str, float] = {}
    for counters in per_rank:
        for key, value in counters.items():
            total[key] = total.get(key, 0) + value
    return total
