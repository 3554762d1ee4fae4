"""The N > 1 path on CPU: data-parallel replicas over gloo, world size 2.

- round-robin stream binding covers every stream once (replicas.py:304-318 semantics);
- the benchmark's reduction: max of the per-rank device times, sum of frames;
- replicas are independent: two ranks each running the oracle's code predictor on
  their own shard produce exactly the codes of one process running all streams
  (rows never mix, predictor_layers.py:24-25).
"""

from __future__ import annotations

import os
import socket
import sys
from pathlib import Path

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parent.parent


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _predictor_codes(streams: list[int], seed: int = 0) -> np.ndarray:
    """Oracle code predictor for the given global stream ids (per-stream seeded inputs)."""
    from oracle.model import OracleTalker
    from omni_b200.config import PredictorConfig, TalkerConfig
    from omni_b200.predictor import init_predictor_weights
    from omni_b200.talker import init_talker_weights

    pc = PredictorConfig(num_hidden_layers=1, vocab_size=256, num_code_groups=4)
    cfg = TalkerConfig(num_hidden_layers=1, vocab_size=256, max_context=64, predictor=pc)
    o = OracleTalker(cfg, init_talker_weights(cfg, seed=seed, device="cpu"),
                     init_predictor_weights(pc, seed=seed + 1, device="cpu"))
    hid = torch.stack([torch.randn(cfg.hidden_size, generator=torch.Generator().manual_seed(1000 + s))
                       for s in streams]).bfloat16().float()
    c0 = torch.tensor([(37 * s) % cfg.vocab_size for s in streams])
    n = len(streams)
    sampling = dict(temperature=np.full(n, 0.9, np.float32), top_k=np.full(n, 50, np.int64),
                    top_p=np.full(n, 0.8, np.float32), seed=np.array([7 + s for s in streams], np.int64),
                    do_sample=np.ones(n, np.uint8), max_top_k=50, has_top_p=True)
    codes, _, _ = o.code_predictor(c0, hid, torch.tensor(streams), sampling)
    return codes


def _worker(rank: int, world: int, port: int, total: int, out_dir: str) -> None:
    for p in (str(ROOT), str(ROOT / "sglang-omni_b200")):
        if p not in sys.path:
            sys.path.insert(0, p)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from omni_b200.replicas import aggregate_step_times, shard_streams

        mine = shard_streams(total, world, rank)
        codes = _predictor_codes(mine)
        # per-rank device times and frames as bench.py reports them
        t, e, f = aggregate_step_times(10.0 + rank, 20.0 - rank, float(len(mine)), dist)
        np.save(os.path.join(out_dir, f"codes{rank}.npy"), codes)
        np.save(os.path.join(out_dir, f"agg{rank}.npy"), np.array([t, e, f]))
    finally:
        dist.destroy_process_group()


def test_round_robin_binding():
    from omni_b200.replicas import RoundRobinBinding, shard_streams

    b = RoundRobinBinding()
    assert [b.bind("talker", 3) for _ in range(7)] == [0, 1, 2, 0, 1, 2, 0]
    shards = [shard_streams(10, 3, r) for r in range(3)]
    assert sorted(sum(shards, [])) == list(range(10))
    with pytest.raises(ValueError):
        shard_streams(4, 2, 2)


def test_two_gloo_replicas_match_one_process(tmp_path):
    total, world = 6, 2
    port = _free_port()
    mp.start_processes(_worker, args=(world, port, total, str(tmp_path)), nprocs=world, start_method="spawn")
    from omni_b200.replicas import shard_streams

    single = _predictor_codes(list(range(total)))
    for r in range(world):
        got = np.load(tmp_path / f"codes{r}.npy")
        assert np.array_equal(got, single[shard_streams(total, world, r)])
        agg = np.load(tmp_path / f"agg{r}.npy")
        assert agg.tolist() == [11.0, 20.0, float(total)]  # max, max, sum over both ranks
