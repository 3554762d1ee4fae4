"""Pure-Python restatement of the talker stage's continuous-batching policy —
TEST INFRASTRUCTURE ONLY (the C++ scheduler of the product is checked against it
decision by decision; nothing in the product package imports this module).

What it restates:
- the prefill-coalescing gate, sglang_omni/scheduling/omni_scheduler.py:2096-2160
  (`prefill_coalesce_waiting_requests`, `prefill_coalesce_holds`): off for
  coalesce_requests <= 1; bypassed by an idle decode loop unless
  coalesce_when_idle; open once coalesce_requests wait; else every waiting request
  without a stamp is stamped `now` and the gate holds while now - oldest stamp <
  the window.  Pinned to the reference's own gate tests
  (tests/unit_test/scheduling/test_prefill_coalesce_gate.py), restated in
  tests/test_scheduler_cpu.py;
- the event loop order, omni_scheduler.py:3616-3653 (schedule, run, process
  results);
- admission as upstream sglang's PrefillAdder does it (absent from the reference
  tree; restated at page granularity): first come first served while rows, the
  prefill token budget and free pages (minus reserve_ratio x the live streams'
  future pages) allow; admitted prompts share the forward with the decode rows;
- prepare_for_decode's page rule (a token at seq_len % page_size == 0 opens a
  page; pages come off a LIFO free stack in row order) and retract_decode's order
  (sort by (frames, -original prompt) descending, retract from the back);
- rollback_decode_prep_after_skip, sglang_omni/models/qwen3_omni/
  talker_scheduler.py:198-225 (opened pages back, seq_len - 1);
- the vocoder emission of sglang_omni/models/qwen3_omni/talker_model_runner.py:
  emit_code_chunks_and_feedback (:178-235), coalesce_threshold / flush_codec_rows
  (:268-298) and on_request_finished (:300-315).
Rows stay compact: the highest live rows fill the lowest holes.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field

IDLE, DECODE, MIXED = 0, 1, 2
_M64 = (1 << 64) - 1


def splitmix64_stream(seed: int):
    """Steele, Lea, Flood (2014) splitmix64 outputs for a 64-bit state."""
    s = seed & _M64
    while True:
        s = (s + 0x9E3779B97F4A7C15) & _M64
        z = s
        z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & _M64
        z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & _M64
        yield z ^ (z >> 31)


def initial_free_stack(num_pages: int, page_seed: int) -> list[int]:
    """Free stack (top = last element) handing out pages 1.. in order, or a
    Fisher-Yates permutation of them drawn from splitmix64."""
    order = list(range(1, num_pages))
    if page_seed:
        rng = splitmix64_stream(page_seed)
        for i in range(len(order), 1, -1):
            j = next(rng) % i
            order[i - 1], order[j] = order[j], order[i - 1]
    return order[::-1]


@dataclass
class _Stream:
    rid: int
    prompt_len: int
    orig_prompt_len: int
    max_frames: int
    frames_done: int = 0
    seq_len: int = 0
    stamp: int = -1
    slot: int = -1
    row: int = -1
    running: bool = False
    pages: list = field(default_factory=list)
    frames_seen: int = 0
    first_flush_done: bool = False
    pending: list = field(default_factory=list)   # [(frame index, codes)]


@dataclass
class OraclePlan:
    mode: int
    decode_rows: int
    moves: list            # [(src, dst)]
    decode_pages: list
    new: list              # [(rid, slot, prompt_len, pages)]
    retracted: list


class OracleScheduler:
    def __init__(self, *, num_pages, page_size, max_batch, max_context, max_prefill_tokens, coalesce_requests=0,
                 coalesce_when_idle=False, coalesce_wait_us=0, prefill_decode_interval=0, reserve_ratio=1.0,
                 eos_token=-1, page_seed=0, emit_messages=False, codec_coalesce_frames=0,
                 codec_coalesce_first_frames=0, codec_coalesce_early_frames=0):
        self.P = page_size
        self.num_pages = num_pages
        self.max_batch = max_batch
        self.max_context = max_context
        self.max_prefill_tokens = max_prefill_tokens
        self.coalesce_requests = coalesce_requests
        self.coalesce_when_idle = coalesce_when_idle
        self.coalesce_wait_us = coalesce_wait_us
        self.interval = prefill_decode_interval
        self.ratio = reserve_ratio
        self.eos = eos_token
        self.free = initial_free_stack(num_pages, page_seed)
        self.free_slots = list(range(max_batch - 1, -1, -1))
        self.waiting: list[int] = []
        self.streams: dict[int, _Stream] = {}
        self.rows: list[int] = []          # rid per row, -1 = hole
        self.interval_left = 0
        self.pending = None                # (mode, rows, opened rows, interval before)
        self.emit_messages = emit_messages
        self.coalesce = codec_coalesce_frames
        self.first = codec_coalesce_first_frames
        self.early = codec_coalesce_early_frames
        self.messages: list = []           # (rid, first frame, [codes...], final)

    # ------------------------------------------------------------------
    def add_request(self, rid, prompt_len, max_frames):
        final = prompt_len + max_frames - 1
        if (rid in self.streams or prompt_len <= 0 or max_frames <= 0 or prompt_len > self.max_prefill_tokens
                or final > self.max_context or -(-final // self.P) > self.num_pages - 1):
            raise ValueError("request rejected")
        self.streams[rid] = _Stream(rid, prompt_len, prompt_len, max_frames)
        self.waiting.append(rid)

    def abort(self, rid):
        s = self.streams.pop(rid)
        if s.running:
            self.rows[s.row] = -1
            self._release(s)
        else:
            self.waiting.remove(rid)

    def _release(self, s):
        self.free.extend(s.pages)
        s.pages = []
        if s.slot >= 0:
            self.free_slots.append(s.slot)
        s.slot, s.row, s.seq_len, s.running = -1, -1, 0, False

    def _compact(self):
        rows = self.rows
        while True:
            while rows and rows[-1] < 0:
                rows.pop()
            holes = [r for r, rid in enumerate(rows) if rid < 0]
            if not holes:
                return
            h = holes[0]
            rows[h] = rows.pop()
            self.streams[rows[h]].row = h

    def _gate_open(self, now, running):
        if self.coalesce_requests <= 1:
            return True
        if not self.coalesce_when_idle and running == 0:
            return True
        if len(self.waiting) >= self.coalesce_requests:
            return True
        for rid in self.waiting:
            s = self.streams[rid]
            if s.stamp < 0:
                s.stamp = now
        oldest = min([self.streams[r].stamp for r in self.waiting] + [now])
        return not (now - oldest < self.coalesce_wait_us)

    def _opening(self):
        return sum(1 for rid in self.rows if self.streams[rid].seq_len % self.P == 0)

    # ------------------------------------------------------------------
    def schedule(self, now):
        assert self.pending is None
        before = {rid: r for r, rid in enumerate(self.rows) if rid >= 0}
        self._compact()
        P = self.P
        B = len(self.rows)
        admit = []
        if self.waiting and self._gate_open(now, B) and B < self.max_batch and self.interval_left == 0:
            avail = len(self.free)
            used = 0
            future = 0.0
            for rid in self.rows:
                s = self.streams[rid]
                opens = int(s.seq_len % P == 0)
                used += opens
                future += float(-(-(s.seq_len + s.max_frames - s.frames_done) // P) - len(s.pages) - opens)
            if used <= avail:
                tokens = 0
                for rid in self.waiting:
                    if B + len(admit) >= self.max_batch:
                        break
                    s = self.streams[rid]
                    if tokens + s.prompt_len > self.max_prefill_tokens:
                        break
                    need = -(-s.prompt_len // P)
                    fut = float(-(-(s.prompt_len + s.max_frames - s.frames_done - 1) // P) - need)
                    keep = math.ceil(self.ratio * (future + fut))
                    if used + need + keep > avail:
                        break
                    admit.append(rid)
                    used += need
                    tokens += s.prompt_len
                    future += fut
        retracted = []
        if not admit and B > 0 and self._opening() > len(self.free):
            order = sorted(self.rows, key=lambda r: (self.streams[r].frames_done, -self.streams[r].orig_prompt_len),
                           reverse=True)
            while order and self._opening() > len(self.free):
                rid = order.pop()
                s = self.streams[rid]
                self.rows[s.row] = -1
                self._compact()
                s.prompt_len = s.seq_len
                self._release(s)
                retracted.append(rid)
            self.waiting[:0] = retracted
            B = len(self.rows)
        mode = IDLE if (B == 0 and not admit) else (DECODE if not admit else MIXED)
        moves = [(before[rid], r) for r, rid in enumerate(self.rows) if rid in before and before[rid] != r]
        decode_pages, opened = [], []
        for r, rid in enumerate(self.rows):
            s = self.streams[rid]
            if s.seq_len % P == 0:
                pg = self.free.pop()
                s.pages.append(pg)
                decode_pages.append(pg)
                opened.append(r)
            s.seq_len += 1
        new = []
        for rid in admit:
            s = self.streams[rid]
            self.waiting.remove(rid)
            s.running = True
            s.slot = self.free_slots.pop()
            s.row = len(self.rows)
            self.rows.append(rid)
            pages = [self.free.pop() for _ in range(-(-s.prompt_len // P))]
            s.pages.extend(pages)
            s.seq_len = s.prompt_len
            s.stamp = -1
            new.append((rid, s.slot, s.prompt_len, pages))
        interval_before = self.interval_left
        if mode == MIXED:
            self.interval_left = self.interval
        elif mode == DECODE and self.interval_left > 0:
            self.interval_left -= 1
        if mode != IDLE:
            self.pending = (mode, len(self.rows), opened, interval_before)
        return OraclePlan(mode, B, moves, decode_pages, new, retracted)

    def _flush(self, s, final=False):
        if s.pending:
            s.first_flush_done = True
            self.messages.append((s.rid, s.pending[0][0], [c for _, c in s.pending], final))
            s.pending = []

    def _emit(self, s, frame, done):
        idx = s.frames_done
        if self.coalesce <= 1:
            self.messages.append((s.rid, idx, [frame], done))
            return
        s.frames_seen += 1
        if s.frames_seen <= self.early:
            self.messages.append((s.rid, idx, [frame], done))
            return
        if self.early > 0:
            ready = len(s.pending) >= self.coalesce
        else:
            threshold = self.first if (self.first > 0 and not s.first_flush_done) else self.coalesce
            ready = len(s.pending) >= threshold
        if ready:
            self._flush(s)
        s.pending.append((idx, frame))
        if done:
            last = s.pending.pop()
            self._flush(s)
            s.pending.append(last)
            self._flush(s, final=True)

    def commit(self, codes):
        mode, n, _, _ = self.pending
        assert len(codes) == n
        finished = []
        for r in range(n):
            s = self.streams[self.rows[r]]
            s.frames_done += 1
            frame = list(codes[r]) if hasattr(codes[r], "__len__") else [codes[r]]
            done = s.frames_done >= s.max_frames or (self.eos >= 0 and frame[0] == self.eos)
            if self.emit_messages:
                self._emit(s, frame, done)
            if done:
                finished.append(s.rid)
                self.rows[r] = -1
                self._release(s)
                del self.streams[s.rid]
        self.pending = None
        return finished

    def rollback(self):
        mode, _, opened, interval_before = self.pending
        assert mode == DECODE
        for r in reversed(opened):
            s = self.streams[self.rows[r]]
            self.free.append(s.pages.pop())
        for rid in self.rows:
            self.streams[rid].seq_len -= 1
        self.interval_left = interval_before
        self.pending = None
