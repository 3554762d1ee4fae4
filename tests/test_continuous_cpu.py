"""Config 4's sharding on CPU: world size 2 over gloo, each rank running the C++
scheduler on its round-robin shard of the Poisson arrival trace (host only, codes
faked), then the benchmark's reduction (max of the times, sum of the frames).

- the shards are disjoint and cover the trace (RoundRobinBindingPolicy semantics,
  replicas.py:304-318 of the reference);
- every stream of a rank finishes with exactly its frames, no page is lost;
- the live rows per rank settle near the steady-state target the arrival rate was
  chosen for (Little's law), independent of the world size.
"""

from __future__ import annotations

import os
import socket
import sys
from pathlib import Path

import numpy as np
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parent.parent


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _serve_shard(trace, world: int, rank: int, max_batch: int = 96):
    """Run the scheduler over this rank's streams to the end; (frames, steps, mean live)."""
    from omni_b200.replicas import shard_streams
    from omni_b200.scheduler import OmniScheduler, SchedulerConfig

    mine = set(shard_streams(len(trace), world, rank))
    arrivals: dict[int, list] = {}
    for rid, step, L, F in trace:
        if rid in mine:
            arrivals.setdefault(step, []).append((rid, L, F))
    s = OmniScheduler(SchedulerConfig(num_pages=8192, page_size=16, max_batch=max_batch, max_context=8192 + 64,
                                      max_prefill_tokens=8192, page_seed=rank + 1))
    frames, live, step = {}, [], 0
    last = max(arrivals)
    while True:
        for rid, L, F in arrivals.get(step, []):
            s.add_request(rid, L, F)
        plan = s.get_next_batch_to_run(step)
        step += 1
        if plan.is_idle():
            st = s.stats()
            if step > last and st["waiting"] == 0 and st["running"] == 0:
                break
            continue
        rids = s.row_rids()[: plan.rows]
        for rid in rids:
            frames[rid] = frames.get(rid, 0) + 1
        live.append(plan.rows)
        s.process_batch_result(np.zeros(plan.rows, np.int64))
    s.check()
    assert s.stats()["free_pages"] == 8191
    want = {rid: F for rid, _, _, F in trace if rid in mine}
    assert frames == want
    return sum(frames.values()), step, float(np.mean(live[len(live) // 4: 3 * len(live) // 4]))


def _worker(rank: int, world: int, port: int, out_dir: str) -> None:
    for p in (str(ROOT), str(ROOT / "sglang-omni_b200")):
        if p not in sys.path:
            sys.path.insert(0, p)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from omni_b200.continuous import poisson_arrival_trace
        from omni_b200.replicas import aggregate_step_times

        trace = poisson_arrival_trace(256, world, 32, (8, 24))
        frames, steps, mean_live = _serve_shard(trace, world, rank)
        t, _, f = aggregate_step_times(float(steps), float(steps), float(frames), dist)
        np.save(os.path.join(out_dir, f"c4_{rank}.npy"), np.array([t, f, frames, mean_live]))
    finally:
        dist.destroy_process_group()


def test_trace_shards_cover_the_streams():
    from omni_b200.continuous import poisson_arrival_trace
    from omni_b200.replicas import shard_streams

    trace = poisson_arrival_trace(500, 4, 256, (64, 192))
    assert [t[0] for t in trace] == list(range(500))
    assert all(16 <= L <= 8192 and 64 <= F <= 192 for _, _, L, F in trace)
    steps = [t[1] for t in trace]
    assert steps == sorted(steps)
    shards = [set(shard_streams(500, 4, r)) for r in range(4)]
    assert set().union(*shards) == set(range(500)) and sum(map(len, shards)) == 500
    # 4 GPUs x 256 live / mean 128 frames = 8 arrivals per step
    assert 6.0 < 500 / (steps[-1] + 1) < 10.0


def test_two_ranks_serve_their_shards(tmp_path):
    world = 2
    port = _free_port()
    mp.start_processes(_worker, args=(world, port, str(tmp_path)), nprocs=world, join=True, start_method="spawn")
    res = [np.load(tmp_path / f"c4_{r}.npy") for r in range(world)]
    from omni_b200.continuous import poisson_arrival_trace

    trace = poisson_arrival_trace(256, world, 32, (8, 24))
    total = sum(F for _, _, _, F in trace)
    for t, f, frames, mean_live in res:
        assert f == total                     # the reduction sums the ranks' frames
        assert t == max(r[0] for r in res)    # and takes the slowest rank's time
        assert 16 < mean_live < 48            # about 32 live streams per rank
    assert sum(r[2] for r in res) == total


def test_one_rank_holds_the_same_steady_state():
    from omni_b200.continuous import poisson_arrival_trace

    trace = poisson_arrival_trace(256, 1, 32, (8, 24))
    frames, _, mean_live = _serve_shard(trace, 1, 0)
    assert frames == sum(F for _, _, _, F in trace)
    assert 16 < mean_live < 48
