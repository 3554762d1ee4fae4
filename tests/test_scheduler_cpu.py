"""The C++ continuous-batching scheduler (include/omni_sched.h) against the
pure-Python restatement in oracle/scheduler.py, and the reference's own
prefill-gate cases (tests/unit_test/scheduling/test_prefill_coalesce_gate.py of
the reference, restated with microsecond clocks).  Host code only: no GPU."""

from __future__ import annotations

import random

import numpy as np
import pytest

from omni_b200.scheduler import DECODE, IDLE, MIXED, OmniScheduler, SchedulerConfig
from oracle.scheduler import OracleScheduler, initial_free_stack


def make(**kw):
    base = dict(num_pages=64, page_size=4, max_batch=8, max_context=256, max_prefill_tokens=64)
    base.update(kw)
    return OmniScheduler(SchedulerConfig(**base)), OracleScheduler(**base)


def same_plan(p, o):
    assert p.mode == o.mode
    assert p.decode_rows == o.decode_rows
    assert list(zip(p.moves_src.tolist(), p.moves_dst.tolist())) == o.moves
    assert p.decode_pages.tolist() == o.decode_pages
    assert p.retracted.tolist() == o.retracted
    new = [(int(r), int(s), int(L), p.new_pages[p.new_page_indptr[i]: p.new_page_indptr[i + 1]].tolist())
           for i, (r, s, L) in enumerate(zip(p.new_rid, p.new_slot, p.new_prompt_len))]
    assert new == o.new


# ---------------------------------------------------------------------------
# allocator basics
# ---------------------------------------------------------------------------

def test_page_order_matches_restatement():
    for seed in (0, 1, 12345, 2**63 + 7):
        s, o = make(num_pages=40, page_seed=seed, max_prefill_tokens=200)
        s.add_request(1, 39 * 4 - 8, 1)
        o.add_request(1, 39 * 4 - 8, 1)
        p = s.get_next_batch_to_run(0)
        q = o.schedule(0)
        same_plan(p, q)
        got = p.new_pages.tolist()
        assert len(set(got)) == 37 and min(got) >= 1 and max(got) <= 39
        if seed == 0:
            assert got == list(range(1, 38))
    assert initial_free_stack(5, 0) == [4, 3, 2, 1]


def test_admission_decode_finish_cycle():
    s, _ = make()
    s.add_request(10, 5, 3)
    p = s.get_next_batch_to_run(0)
    assert p.mode == MIXED and p.decode_rows == 0 and p.new_rows == 1
    assert p.new_prompt_len.tolist() == [5] and p.new_pages.tolist() == [1, 2]
    assert s.process_batch_result([7]) == []
    slot, seq, pages = s.request_state(10)
    assert (seq, pages) == (5, [1, 2])
    p = s.get_next_batch_to_run(0)
    assert p.mode == DECODE and p.decode_rows == 1 and p.decode_pages.tolist() == []  # token 5 fits page 2
    s.process_batch_result([7])
    p = s.get_next_batch_to_run(0)
    assert p.mode == DECODE
    assert s.process_batch_result([7]) == [10]
    s.check()
    st = s.stats()
    assert st["running"] == 0 and st["free_pages"] == 63 and st["finished"] == 1 and st["frames"] == 3
    assert s.get_next_batch_to_run(0).mode == IDLE


def test_decode_opens_pages_in_row_order():
    s, _ = make(page_size=4)
    s.add_request(1, 4, 10)  # next token (index 4) opens a page
    s.add_request(2, 3, 10)
    s.add_request(3, 8, 10)
    p = s.get_next_batch_to_run(0)
    assert p.new_rows == 3
    s.process_batch_result([0, 0, 0])
    p = s.get_next_batch_to_run(0)
    assert p.mode == DECODE and p.decode_rows == 3
    # rows 0 and 2 open a page, in row order, off the top of the stack
    assert p.decode_pages.tolist() == [5, 6]
    s.check()


def test_compaction_moves_highest_rows_into_holes():
    s, _ = make(max_batch=8)
    for rid in range(6):
        s.add_request(rid, 3, 2 if rid in (1, 3) else 9)
    s.get_next_batch_to_run(0)
    s.process_batch_result([0] * 6)
    s.get_next_batch_to_run(0)
    assert sorted(s.process_batch_result([0] * 6)) == [1, 3]
    p = s.get_next_batch_to_run(0)
    # holes at rows 1 and 3; rows 5 and 4 fill them
    assert list(zip(p.moves_src.tolist(), p.moves_dst.tolist())) == [(5, 1), (4, 3)]
    assert s.row_rids() == [0, 5, 2, 4]
    s.check()


def test_eos_finishes_a_stream():
    s, _ = make(eos_token=99)
    s.add_request(1, 3, 50)
    s.add_request(2, 3, 50)
    s.get_next_batch_to_run(0)
    assert s.process_batch_result([99, 5]) == [1]
    p = s.get_next_batch_to_run(0)
    assert list(zip(p.moves_src.tolist(), p.moves_dst.tolist())) == [(1, 0)]
    assert s.row_rids() == [2]


def test_rollback_restores_the_free_stack_exactly():
    s, o = make(page_size=2)
    for rid in range(4):
        s.add_request(rid, 2 + rid, 20)
        o.add_request(rid, 2 + rid, 20)
    same_plan(s.get_next_batch_to_run(0), o.schedule(0))
    s.process_batch_result([0] * 4)
    o.commit([0] * 4)
    p = s.get_next_batch_to_run(0)
    q = o.schedule(0)
    same_plan(p, q)
    before = s.stats()["free_pages"]
    s.rollback_decode_prep_after_skip()
    o.rollback()
    assert s.stats()["free_pages"] == before + len(p.decode_pages)
    s.check()
    # the retried step opens the same pages
    same_plan(s.get_next_batch_to_run(0), o.schedule(0))
    s.process_batch_result([0] * 4)
    o.commit([0] * 4)
    s.check()


def test_rollback_only_for_decode_steps():
    s, _ = make()
    s.add_request(1, 3, 5)
    s.get_next_batch_to_run(0)
    with pytest.raises(ValueError):
        s.rollback_decode_prep_after_skip()
    s.process_batch_result([0])
    with pytest.raises(ValueError):
        s.process_batch_result([0])


def test_rejections_and_errors():
    s, _ = make(num_pages=8, page_size=4, max_context=40, max_prefill_tokens=16)
    s.add_request(1, 4, 4)
    with pytest.raises(ValueError):
        s.add_request(1, 4, 4)  # duplicate
    with pytest.raises(ValueError):
        s.add_request(2, 17, 1)  # over the prefill budget (no chunked prefill)
    with pytest.raises(ValueError):
        s.add_request(3, 16, 26)  # over max_context
    with pytest.raises(ValueError):
        s.add_request(4, 16, 20)  # 35 tokens: 9 pages > 7
    with pytest.raises(ValueError):
        s.add_request(5, 0, 3)
    with pytest.raises(ValueError):
        s.abort(42)
    with pytest.raises(ValueError):
        OmniScheduler(SchedulerConfig(num_pages=1))


def test_abort_waiting_and_running():
    s, o = make()
    for rid in range(3):
        s.add_request(rid, 3, 9)
        o.add_request(rid, 3, 9)
    same_plan(s.get_next_batch_to_run(0), o.schedule(0))
    s.process_batch_result([0] * 3)
    o.commit([0] * 3)
    s.add_request(7, 3, 9)
    o.add_request(7, 3, 9)
    s.abort(0)
    o.abort(0)
    s.abort(7)
    o.abort(7)
    same_plan(s.get_next_batch_to_run(0), o.schedule(0))
    s.check()


def test_retraction_when_the_pool_runs_dry():
    # 9 usable pages of 2 tokens; three streams that each want 4 pages
    s, o = make(num_pages=10, page_size=2, max_batch=4, max_context=64, reserve_ratio=0.0)
    for rid, L in ((1, 2), (2, 2), (3, 4)):
        s.add_request(rid, L, 6)
        o.add_request(rid, L, 6)
    saw_retract = False
    for step in range(40):
        p, q = s.get_next_batch_to_run(step), o.schedule(step)
        same_plan(p, q)
        s.check()
        saw_retract |= len(p.retracted) > 0
        if p.is_idle():
            break
        s.process_batch_result([0] * p.rows)
        o.commit([0] * p.rows)
    assert saw_retract
    st = s.stats()
    assert st["finished"] == 3 and st["free_pages"] == 9 and st["retracted"] >= 1


@pytest.mark.parametrize("seed", range(12))
def test_random_traces_match_the_restatement(seed):
    rng = random.Random(seed)
    kw = dict(num_pages=rng.choice([24, 48, 96]), page_size=rng.choice([1, 2, 4, 16]),
              max_batch=rng.choice([3, 8, 16]), max_context=512, max_prefill_tokens=rng.choice([24, 64, 200]),
              coalesce_requests=rng.choice([0, 3]), coalesce_when_idle=rng.random() < 0.5,
              coalesce_wait_us=rng.choice([0, 50]), prefill_decode_interval=rng.choice([0, 2]),
              reserve_ratio=rng.choice([0.0, 0.5, 1.0]), eos_token=rng.choice([-1, 3]),
              page_seed=rng.choice([0, rng.getrandbits(64)]))
    s, o = make(**kw)
    rid = 0
    now = 0
    for step in range(300):
        now += rng.randint(0, 40)
        for _ in range(rng.choice([0, 0, 1, 2])):
            L = rng.randint(1, min(kw["max_prefill_tokens"], 40))
            F = rng.randint(1, 30)
            try:
                o.add_request(rid, L, F)
                ok = True
            except ValueError:
                ok = False
            if ok:
                s.add_request(rid, L, F)
            else:
                with pytest.raises(ValueError):
                    s.add_request(rid, L, F)
            rid += 1
        if rng.random() < 0.05 and (o.waiting or o.rows):
            victim = rng.choice(list(o.streams))
            o.abort(victim)
            s.abort(victim)
        p, q = s.get_next_batch_to_run(now), o.schedule(now)
        same_plan(p, q)
        s.check()
        if p.is_idle():
            continue
        if p.mode == DECODE and rng.random() < 0.1:
            s.rollback_decode_prep_after_skip()
            o.rollback()
            s.check()
            continue
        codes = [rng.randint(0, 5) for _ in range(p.rows)]
        assert sorted(s.process_batch_result(codes)) == sorted(o.commit(codes))
        assert s.row_rids() == o.rows
    st = s.stats()
    assert st["waiting"] == len(o.waiting)


# ---------------------------------------------------------------------------
# the reference's prefill-gate cases (omni_scheduler.py:2096-2160)
# ---------------------------------------------------------------------------

def running_one(**kw):
    """A scheduler with one stream decoding (so the gate is not bypassed as idle)."""
    s, _ = make(max_batch=16, **kw)
    s.add_request(1000, 3, 100)
    # the first admission happens while idle: with coalesce_when_idle off it bypasses
    p = s.get_next_batch_to_run(0)
    assert p.new_rows == 1
    s.process_batch_result([0])
    return s


def admitted(s, now):
    p = s.get_next_batch_to_run(now)
    n = p.new_rows
    s.process_batch_result([0] * p.rows)
    return n


def test_gate_disabled_passes_through():
    s = running_one(coalesce_requests=0)
    s.add_request(1, 3, 5)
    assert admitted(s, 0) == 1


def test_gate_full_batch_passes_through_immediately():
    s = running_one(coalesce_requests=4, coalesce_wait_us=60_000)
    for r in range(4):
        s.add_request(r, 3, 5)
    assert admitted(s, 10) == 4


def test_gate_small_queue_held_until_oldest_expires():
    s = running_one(coalesce_requests=8, coalesce_wait_us=60_000)
    s.add_request(1, 3, 5)
    assert admitted(s, 100_000) == 0      # stamped at 100 ms
    s.add_request(2, 3, 5)
    assert admitted(s, 110_000) == 0      # the newcomer does not restart the window
    assert admitted(s, 130_000) == 0      # 30 ms of 60
    assert admitted(s, 160_000) == 2      # oldest past its deadline: both go


def test_gate_idle_loop_bypasses():
    s, _ = make(coalesce_requests=8, coalesce_wait_us=60_000)
    s.add_request(1, 3, 5)
    assert s.get_next_batch_to_run(0).new_rows == 1


def test_gate_idle_loop_can_coalesce_when_enabled():
    s, _ = make(coalesce_requests=8, coalesce_wait_us=10_000, coalesce_when_idle=True)
    s.add_request(1, 3, 5)
    assert s.get_next_batch_to_run(100_000).mode == IDLE
    assert s.get_next_batch_to_run(105_000).mode == IDLE
    assert s.get_next_batch_to_run(110_000).new_rows == 1


def test_gate_partial_admission_leftovers_release_immediately():
    # the expired wave is admitted only partly (prefill budget); the leftover keeps
    # its stamp and goes on the next pass
    s = running_one(coalesce_requests=8, coalesce_wait_us=60_000)
    s.add_request(1, 40, 5)
    s.add_request(2, 40, 5)
    assert admitted(s, 100_000) == 0
    assert admitted(s, 170_000) == 1   # 40 + 40 > 64 prefill tokens
    assert admitted(s, 170_001) == 1


def test_gate_newcomer_after_queue_drain_waits_its_own_window():
    s = running_one(coalesce_requests=8, coalesce_wait_us=60_000)
    s.add_request(1, 3, 5)
    assert admitted(s, 100_000) == 0
    s.abort(1)                         # abort just before the armer's deadline
    s.add_request(2, 3, 5)
    assert admitted(s, 159_000) == 0   # stamped at 159 ms
    assert admitted(s, 170_000) == 0   # past the armer's window, inside its own
    assert admitted(s, 219_000) == 1


def test_prefill_decode_interval_spaces_admissions():
    s = running_one(prefill_decode_interval=2)
    s.add_request(1, 3, 5)
    s.add_request(2, 3, 5)
    s.add_request(3, 3, 5)
    # the first admission of running_one set the interval: two decode-only steps first
    assert admitted(s, 0) == 0
    assert admitted(s, 0) == 0
    assert admitted(s, 0) == 3


def test_admission_keeps_the_reserve_free():
    s = running_one()  # one stream that will take 26 pages of the 63
    for r in range(3):
        s.add_request(r, 3, 50)  # 13 pages each over their life
    assert admitted(s, 0) == 2


def test_plan_arrays_are_numpy():
    s, _ = make()
    s.add_request(1, 3, 2)
    p = s.get_next_batch_to_run(0)
    assert isinstance(p.new_pages, np.ndarray) and p.new_pages.dtype == np.int32


# ---------------------------------------------------------------------------
# vocoder messages: the reference's codec-coalescing cases
# (tests/unit_test/qwen3_omni/test_talker_codec_coalesce.py), restated on the C++
# scheduler, plus random traces against the restatement
# ---------------------------------------------------------------------------

def emitter(n, frames, **kw):
    """n streams of `frames` frames each, all admitted in the first step."""
    cfg = dict(num_pages=256, page_size=4, max_batch=max(n, 2), max_context=512, max_prefill_tokens=64,
               emit_messages=True)
    cfg.update(kw)
    s = OmniScheduler(SchedulerConfig(**cfg))
    for r in range(n):
        s.add_request(r, 3, frames)
    return s


def step_frames(s, step):
    """One step; frame `step` of stream r is [r * 1000 + step, r + 100 + step]."""
    p = s.get_next_batch_to_run(0)
    rids = s.row_rids()[: p.rows]
    codes = np.array([[r * 1000 + step, r + 100 + step] for r in rids], np.int64)
    s.process_batch_result(codes)
    return {r: codes[i] for i, r in enumerate(rids)}


def test_messages_one_per_frame_when_coalescing_is_off():
    s = emitter(2, 5)
    for k in range(1, 6):
        step_frames(s, k)
    msgs = s.pop_messages(2)
    assert len(msgs) == 10 and all(m[2].shape == (1, 2) for m in msgs)
    assert [m[3] for m in msgs if m[0] == 0] == [False] * 4 + [True]


def test_messages_coalesce_after_threshold_with_newest_held():
    s = emitter(2, 100, codec_coalesce_frames=3)
    seen = [step_frames(s, k) for k in range(1, 4)]
    assert s.pop_messages(2) == []
    seen.append(step_frames(s, 4))
    msgs = s.pop_messages(2)
    assert len(msgs) == 2
    m0 = next(m for m in msgs if m[0] == 0)
    assert m0[1] == 1 and m0[2].shape == (3, 2)
    np.testing.assert_array_equal(m0[2], np.stack([f[0] for f in seen[:3]]))


@pytest.mark.parametrize("steps", [1, 2, 3, 4])
def test_finish_sends_the_last_frame_alone(steps):
    s = emitter(1, steps, codec_coalesce_frames=3)
    seen = [step_frames(s, k)[0] for k in range(1, steps + 1)]
    msgs = s.pop_messages(2)
    np.testing.assert_array_equal(msgs[-1][2], seen[-1][None])
    assert msgs[-1][3] and not any(m[3] for m in msgs[:-1])
    np.testing.assert_array_equal(np.concatenate([m[2] for m in msgs]), np.stack(seen))
    # coalesce 3: [1..3] flushed when frame 4 arrives, so 4 steps give [1-3], [4]
    assert len(msgs) == {1: 1, 2: 2, 3: 2, 4: 2}[steps]


def test_first_flush_uses_the_smaller_threshold():
    n, k, first = 2, 5, 2
    s = emitter(n, 100, codec_coalesce_frames=k, codec_coalesce_first_frames=first)
    for i in range(1, first + 2):
        step_frames(s, i)
    msgs = s.pop_messages(2)
    assert len(msgs) == n and all(m[2].shape[0] == first for m in msgs)
    for i in range(first + 2, first + 2 + k - 1):
        step_frames(s, i)
    assert s.pop_messages(2) == []
    step_frames(s, first + 1 + k)
    msgs = s.pop_messages(2)
    assert len(msgs) == n and all(m[2].shape[0] == k for m in msgs)


def test_early_frames_keep_the_vocoder_window_cadence():
    s = emitter(1, 200, codec_coalesce_frames=10, codec_coalesce_early_frames=12)
    ready_at, received = {}, 0
    for step in range(1, 42):
        step_frames(s, step)
        received += sum(m[2].shape[0] for m in s.pop_messages(2))
        for end in (2, 12, 22, 32):
            if received >= end:
                ready_at.setdefault(end, step)
    assert ready_at == {2: 2, 12: 12, 22: 23, 32: 33}


@pytest.mark.parametrize("early", [10, 12])
@pytest.mark.parametrize("steps", [9, 10, 11, 12, 13, 20, 21, 22, 23])
def test_early_frames_then_coalesced_tail_in_order(early, steps):
    s = emitter(1, steps, codec_coalesce_frames=10, codec_coalesce_early_frames=early)
    seen = [step_frames(s, k)[0] for k in range(1, steps + 1)]
    msgs = s.pop_messages(2)
    assert all(m[2].shape[0] == 1 for m in msgs[:early])
    np.testing.assert_array_equal(np.concatenate([m[2] for m in msgs]), np.stack(seen))
    assert [m[1] for m in msgs] == list(np.cumsum([1] + [m[2].shape[0] for m in msgs[:-1]]))


@pytest.mark.parametrize("seed", range(6))
def test_random_trace_messages_match_the_restatement(seed):
    rng = random.Random(100 + seed)
    kw = dict(num_pages=64, page_size=4, max_batch=6, max_context=256, max_prefill_tokens=48,
              reserve_ratio=rng.choice([0.0, 1.0]), eos_token=rng.choice([-1, 2]), emit_messages=True,
              codec_coalesce_frames=rng.choice([0, 1, 3, 5]), codec_coalesce_first_frames=rng.choice([0, 2]),
              codec_coalesce_early_frames=rng.choice([0, 2, 4]))
    s, o = make(**kw)
    rid = 0
    for step in range(200):
        if rng.random() < 0.4:
            L, F = rng.randint(1, 30), rng.randint(1, 25)
            o.add_request(rid, L, F)
            s.add_request(rid, L, F)
            rid += 1
        p, q = s.get_next_batch_to_run(step), o.schedule(step)
        same_plan(p, q)
        if p.is_idle():
            continue
        codes = [[rng.randint(0, 4), rng.randint(0, 99), rng.randint(0, 99)] for _ in range(p.rows)]
        assert sorted(s.process_batch_result(codes)) == sorted(o.commit(codes))
    got = [(r, f, c.tolist(), fin) for r, f, c, fin in s.pop_messages(3)]
    assert got == o.messages
    assert s.stats()["frames_emitted"] == sum(len(m[2]) for m in o.messages)
