"""Data-parallel replicas of the decode step: one process per GPU, streams bound to
replicas round-robin, no collective on the hot path.

Mirrors the reference's replica binding (RoundRobinBindingPolicy.bind,
sglang_omni/pipeline/replicas.py:304-318: the i-th request of a process goes to
replica i mod N).  Rows never mix inside the step, so a replica's frames depend
only on its own streams; the only cross-rank traffic is the benchmark's timing
reduction (max of the per-rank device times, sum of the frames).
"""

from __future__ import annotations

import itertools
import threading
from collections import defaultdict


class RoundRobinBinding:
    """Replica choice by arrival order: the i-th stream that a process (the talker
    stage, say) hands out goes to replica i mod N, whatever its request id.  One
    arrival counter per process name; safe to call from several threads."""

    def __init__(self) -> None:
        self._arrivals: defaultdict[str, itertools.count] = defaultdict(itertools.count)
        self._mu = threading.Lock()

    def bind(self, process_name: str, num_replicas: int, request_id: str | None = None) -> int:
        if num_replicas < 1:
            raise ValueError("num_replicas must be positive")
        with self._mu:
            arrival = next(self._arrivals[process_name])
        return arrival % num_replicas


def shard_streams(num_streams: int, world: int, rank: int) -> list[int]:
    """Stream ids bound to `rank` when num_streams arrive in order (round-robin)."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError("rank must lie in [0, world)")
    return list(range(rank, num_streams, world))


def aggregate_step_times(total_ms: float, e2e_ms: float, frames: float, dist=None, device=None):
    """(max over ranks of the device time, max of the end-to-end time, sum of frames).

    Every rank calls it with its own numbers (same collective order on all ranks)."""
    if dist is None or not dist.is_initialized() or dist.get_world_size() == 1:
        return float(total_ms), float(e2e_ms), float(frames)
    import torch

    t = torch.tensor([total_ms, e2e_ms], dtype=torch.float64, device=device)
    f = torch.tensor([frames], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    dist.all_reduce(f, op=dist.ReduceOp.SUM)
    return float(t[0]), float(t[1]), float(f[0])
