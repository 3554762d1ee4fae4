"""Continuous batching on the GPU: the C++ scheduler driving the B200 step.

- the row-move and admission kernels, bit-exact against torch / host restatements;
- a Poisson-like trace run to the end: every stream gets exactly its frames, the
  device page tables, seq_lens and request slots agree with the scheduler at every
  step, every page comes back;
- a stream's codes do not depend on the row it sits in or on the other streams
  (streams moved by compaction give the same codes as unmoved ones at the same
  decode bucket);
- CUDA-graph replay == eager; skipped (rolled-back) decode steps change nothing.
"""

from __future__ import annotations

import random

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = "cuda"


def build(*, max_batch=16, layers=2, num_pages=256, max_prefill=512, use_graphs=True, seed=0, eos=-1, moe=False,
          reserve_ratio=1.0, coalesce=0, emit=False):
    from omni_b200.config import MoEConfig, PredictorConfig, SamplingParams, TalkerConfig
    from omni_b200.continuous import ContinuousTalkerRunner
    from omni_b200.model_runner import TalkerDecodeRunner
    from omni_b200.scheduler import OmniScheduler, SchedulerConfig

    if moe:
        cfg = TalkerConfig(num_hidden_layers=layers, max_context=1024, moe=MoEConfig(),
                           predictor=PredictorConfig(vocab_size=1024, num_code_groups=32))
    else:
        cfg = TalkerConfig(num_hidden_layers=layers, max_context=1024)
    sc = SchedulerConfig(num_pages=num_pages, page_size=cfg.page_size, max_batch=max_batch, max_context=1024,
                         max_prefill_tokens=max_prefill, reserve_ratio=reserve_ratio, eos_token=eos,
                         page_seed=seed + 3, coalesce_requests=coalesce, emit_messages=emit,
                         codec_coalesce_frames=10 if emit else 0, codec_coalesce_early_frames=4 if emit else 0)
    runner = TalkerDecodeRunner(cfg, max_batch=max_batch + 1, num_pages=num_pages, seed=seed,
                                max_prefill_tokens=max_prefill)
    return ContinuousTalkerRunner(runner, OmniScheduler(sc), sampling=SamplingParams(), seed=seed,
                                  use_graphs=use_graphs)


def run_to_end(cr, arrivals, *, ready=None, check_state=False, max_steps=400):
    """arrivals: {step: [(rid, prompt_len, frames)]}; returns {rid: [frame codes]}."""
    frames: dict[int, list] = {}
    step = 0
    while step < max_steps:
        for rid, L, F in arrivals.get(step, []):
            cr.sched.add_request(rid, L, F)
        out = cr.step(now_us=step, ready=ready)
        step += 1
        if out is not None:
            for r, rid in enumerate(out.rids):
                frames.setdefault(rid, []).append(out.codes[r].copy())
            if check_state:
                device_matches_scheduler(cr)
        st = cr.sched.stats()
        if step > max(arrivals, default=0) and st["waiting"] == 0 and st["running"] == 0:
            break
    return frames


def device_matches_scheduler(cr):
    """seq_lens, request slots and req_to_token rows of the live rows agree with the
    scheduler's view (the scheduler state after the commit of the step)."""
    s, r = cr.sched, cr.runner
    rids = s.row_rids()
    live = [(row, rid) for row, rid in enumerate(rids) if rid >= 0]
    seq = r.seq_lens[: len(rids)].cpu().numpy()
    req = r.req_pool_indices[: len(rids)].cpu().numpy()
    r2t = r.r2t.req_to_token.cpu().numpy()
    P = r.cfg.page_size
    for row, rid in live:
        slot, L, pages = s.request_state(rid)
        assert seq[row] == L and req[row] == slot
        want = np.array([pages[t // P] * P + t % P for t in range(L)], dtype=np.int32)
        np.testing.assert_array_equal(r2t[slot, :L], want)


def test_move_rows_matches_torch():
    from omni_b200 import ops

    g = torch.Generator(device=DEV).manual_seed(1)
    ts = [torch.randint(0, 1 << 30, (40,), device=DEV, dtype=torch.long),
          torch.rand(40, 7, device=DEV, generator=g),                                   # 28-byte rows
          torch.randint(0, 255, (40, 3072), device=DEV, dtype=torch.uint8),             # mask rows
          torch.randint(0, 255, (40, 5), device=DEV, dtype=torch.uint8),                # unaligned rows
          torch.randn(40, 1024, device=DEV, generator=g).to(torch.bfloat16)]
    table = ops.RowTensors(ts)
    src = np.array([39, 30, 25, 33], dtype=np.int32)
    dst = np.array([0, 7, 3, 12], dtype=np.int32)
    want = [t.clone() for t in ts]
    for w in want:
        w[torch.from_numpy(dst).long()] = w[torch.from_numpy(src).long()]
    ops.move_rows(table, src, dst)
    torch.cuda.synchronize()
    for t, w in zip(ts, want):
        assert torch.equal(t, w)
    with pytest.raises(ValueError):
        ops.move_rows(table, np.array([1, 2], np.int32), np.array([2, 3], np.int32))


def test_admit_streams_matches_host():
    from omni_b200 import ops

    P, ctx = 16, 256
    r2t = torch.zeros(6, ctx, dtype=torch.int32, device=DEV)
    seq = torch.zeros(8, dtype=torch.long, device=DEV)
    req = torch.zeros(8, dtype=torch.long, device=DEV)
    lens = [5, 16, 33]
    pages = [[9], [4], [2, 7, 11]]
    indptr = np.cumsum([0] + [len(p) for p in pages]).astype(np.int32)
    flat = np.concatenate(pages).astype(np.int32)
    ops.admit_streams(rows=torch.tensor([3, 4, 5], dtype=torch.int32, device=DEV),
                      slots=torch.tensor([5, 0, 2], dtype=torch.int32, device=DEV),
                      prompt_lens=torch.tensor(lens, dtype=torch.long, device=DEV),
                      page_indptr=torch.from_numpy(indptr).to(DEV), pages=torch.from_numpy(flat).to(DEV),
                      req_to_token=r2t, page_size=P, seq_lens=seq, req_pool_indices=req)
    torch.cuda.synchronize()
    host = r2t.cpu().numpy()
    for slot, L, pg in zip((5, 0, 2), lens, pages):
        np.testing.assert_array_equal(host[slot, :L], [pg[t // P] * P + t % P for t in range(L)])
        assert (host[slot, L:] == 0).all()
    assert seq.tolist()[3:6] == lens and req.tolist()[3:6] == [5, 0, 2]


def poisson_trace(seed, streams, lam, max_prompt=120, frames=(2, 12)):
    rng = random.Random(seed)
    arrivals, rid, step = {}, 0, 0
    while rid < streams:
        k = min(streams - rid, np.random.default_rng(seed * 7919 + step).poisson(lam))
        for _ in range(k):
            arrivals.setdefault(step, []).append((rid, rng.randint(8, max_prompt), rng.randint(*frames)))
            rid += 1
        step += 1
    return arrivals


def test_continuous_trace_runs_every_stream_to_its_end():
    cr = build(max_batch=12, num_pages=96, max_prefill=400, emit=True)
    arrivals = poisson_trace(0, streams=30, lam=1.5)
    want = {rid: F for v in arrivals.values() for rid, _, F in v}
    frames = run_to_end(cr, arrivals, check_state=True)
    assert {rid: len(f) for rid, f in frames.items()} == want
    # the vocoder messages, through the shared-memory relay, carry every stream's
    # frames in order, the last one final
    import os
    import uuid

    from omni_b200.relay import CodecRelay

    name = f"/omni_relay_gpu_{os.getpid()}_{uuid.uuid4().hex[:6]}"
    tx, rx = CodecRelay(name, create=True), CodecRelay(name, create=False)
    msgs: dict[int, list] = {}
    backlog: list = []
    try:
        while True:
            backlog = cr.forward_messages(tx, backlog)
            while (m := rx.pop()) is not None:
                rid, first, codes, final = m
                msgs.setdefault(rid, []).append((first, codes, final))
            if not backlog:
                break
    finally:
        rx.close()
        tx.close()
    for rid, f in frames.items():
        got = msgs[rid]
        np.testing.assert_array_equal(np.concatenate([c for _, c, _ in got]), np.stack(f))
        assert [fin for _, _, fin in got] == [False] * (len(got) - 1) + [True]
    G = cr.runner.cfg.predictor.num_code_groups
    for f in frames.values():
        c = np.stack(f)
        assert c.shape[1] == G
        assert (c[:, 0] >= 0).all() and (c[:, 0] < cr.runner.cfg.vocab_size).all()
        assert (c[:, 1:] >= 0).all() and (c[:, 1:] < cr.runner.cfg.predictor.vocab_size).all()
    cr.sched.check()
    st = cr.sched.stats()
    assert st["free_pages"] == 95 and st["finished"] == 30
    assert cr.device_status() == 0
    assert cr.graph_steps > 0


def test_stream_codes_do_not_depend_on_their_row():
    """14 streams at the same decode bucket (16): in X stream 3 ends after two frames
    and stream 13 moves into its row; every other stream's codes equal those of run Y,
    where nobody moves."""
    lens = [20, 33, 8, 50, 17, 64, 12, 40, 29, 9, 61, 44, 23, 37]
    outs = []
    for short in (True, False):
        cr = build(max_batch=16, num_pages=128, max_prefill=600)
        arrivals = {0: [(i, L, 2 if (short and i == 3) else 6) for i, L in enumerate(lens)]}
        frames = run_to_end(cr, arrivals)
        outs.append(frames)
    x, y = outs
    assert len(x[3]) == 2 and len(y[3]) == 6
    for rid in range(len(lens)):
        n = len(x[rid])
        np.testing.assert_array_equal(np.stack(x[rid]), np.stack(y[rid])[:n], err_msg=f"stream {rid}")


def test_graph_replay_equals_eager_and_skips_change_nothing():
    arrivals = {0: [(i, 10 + 7 * i, 5 + (i % 4)) for i in range(10)]}
    ref = run_to_end(build(use_graphs=False), arrivals)
    got = run_to_end(build(use_graphs=True), arrivals)
    rng = random.Random(5)
    skipped = run_to_end(build(use_graphs=True), arrivals, ready=lambda plan: rng.random() > 0.3)
    for rid in ref:
        np.testing.assert_array_equal(np.stack(got[rid]), np.stack(ref[rid]))
        np.testing.assert_array_equal(np.stack(skipped[rid]), np.stack(ref[rid]))


def test_moe_continuous_mixed_steps():
    cr = build(max_batch=8, num_pages=64, max_prefill=256, moe=True)
    arrivals = poisson_trace(3, streams=10, lam=1.0, max_prompt=60, frames=(2, 6))
    want = {rid: F for v in arrivals.values() for rid, _, F in v}
    frames = run_to_end(cr, arrivals, check_state=True)
    assert {rid: len(f) for rid, f in frames.items()} == want
    cr.sched.check()
    assert cr.sched.stats()["free_pages"] == 63 and cr.device_status() == 0


def test_retraction_under_a_small_pool():
    """A pool too small for every stream's full context with no reserve: the scheduler
    retracts streams, their rows are compacted away, they come back as new prefills of
    their whole context and still produce exactly their frames; every page returns."""
    cr = build(max_batch=8, num_pages=24, max_prefill=256, reserve_ratio=0.0)
    arrivals = {0: [(i, 40 + 9 * i, 14) for i in range(6)]}
    want = {rid: F for v in arrivals.values() for rid, _, F in v}
    frames = run_to_end(cr, arrivals, check_state=True, max_steps=600)
    assert {rid: len(f) for rid, f in frames.items()} == want
    st = cr.sched.stats()
    assert st["retracted"] > 0
    assert st["free_pages"] == 23 and st["finished"] == 6
    assert cr.device_status() == 0
