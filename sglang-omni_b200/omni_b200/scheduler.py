"""Host-side continuous batching of talker streams: the C++ scheduler of
libomni_b200.so (include/omni_sched.h) behind the calls of the reference's
OmniScheduler event loop.

The reference's talker stage runs ``event_loop_normal``
(sglang_omni/scheduling/omni_scheduler.py:3616-3653): queue the arrivals, call
``get_next_batch_to_run`` (:2000-2022, with the prefill-coalescing gate
:2096-2160 over the upstream sglang Scheduler), run the batch, then
``process_batch_result``.  A decode batch whose inputs are not ready is undone
by ``rollback_decode_prep_after_skip``
(sglang_omni/models/qwen3_omni/talker_scheduler.py:198-225).  The same calls
here return a :class:`StepPlan`: the row moves that keep the batch compact, the
decode rows with the pages they open, and the admitted streams (slot, prompt
length, prompt pages) that run in the same forward.  Everything is decided in
C++; this module only marshals arrays.
"""

from __future__ import annotations

import ctypes
import time
from dataclasses import dataclass

import numpy as np

from omni_b200 import _lib

IDLE, DECODE, MIXED = 0, 1, 2


class _Config(ctypes.Structure):
    _fields_ = [
        ("num_pages", ctypes.c_int64),
        ("page_size", ctypes.c_int32),
        ("max_batch", ctypes.c_int32),
        ("max_context", ctypes.c_int64),
        ("max_prefill_tokens", ctypes.c_int64),
        ("coalesce_requests", ctypes.c_int32),
        ("coalesce_when_idle", ctypes.c_int32),
        ("coalesce_wait_us", ctypes.c_int64),
        ("prefill_decode_interval", ctypes.c_int32),
        ("reserved0", ctypes.c_int32),
        ("reserve_ratio", ctypes.c_double),
        ("eos_token", ctypes.c_int64),
        ("page_seed", ctypes.c_uint64),
        ("emit_messages", ctypes.c_int32),
        ("codec_coalesce_frames", ctypes.c_int32),
        ("codec_coalesce_first_frames", ctypes.c_int32),
        ("codec_coalesce_early_frames", ctypes.c_int32),
    ]


class _Plan(ctypes.Structure):
    _fields_ = [
        ("mode", ctypes.c_int32),
        ("decode_rows", ctypes.c_int32),
        ("new_rows", ctypes.c_int32),
        ("num_moves", ctypes.c_int32),
        ("num_decode_pages", ctypes.c_int32),
        ("num_retracted", ctypes.c_int32),
        ("new_tokens", ctypes.c_int64),
        ("move_src", ctypes.c_void_p),
        ("move_dst", ctypes.c_void_p),
        ("decode_pages", ctypes.c_void_p),
        ("new_rid", ctypes.c_void_p),
        ("new_slot", ctypes.c_void_p),
        ("new_prompt_len", ctypes.c_void_p),
        ("new_page_indptr", ctypes.c_void_p),
        ("new_pages", ctypes.c_void_p),
        ("retracted_rid", ctypes.c_void_p),
    ]


@dataclass
class SchedulerConfig:
    """Knobs of the talker stage's batch policy (server args of the reference:
    max_running_requests, max_prefill_tokens, page_size, the prefill_coalesce_*
    fields and prefill_decode_interval of generation_batch_policy.py:153-180)."""

    num_pages: int
    page_size: int = 16
    max_batch: int = 256
    max_context: int = 8192 + 512
    max_prefill_tokens: int = 8192
    coalesce_requests: int = 0
    coalesce_when_idle: bool = False
    coalesce_wait_us: int = 0
    prefill_decode_interval: int = 0
    reserve_ratio: float = 1.0
    eos_token: int = -1
    page_seed: int = 0
    # vocoder messages (the talker runner's codec_coalesce_* arguments,
    # qwen3_omni/talker_model_runner.py:70-72)
    emit_messages: bool = False
    codec_coalesce_frames: int = 0
    codec_coalesce_first_frames: int = 0
    codec_coalesce_early_frames: int = 0

    def to_c(self) -> _Config:
        return _Config(self.num_pages, self.page_size, self.max_batch, self.max_context, self.max_prefill_tokens,
                       self.coalesce_requests, int(self.coalesce_when_idle), self.coalesce_wait_us,
                       self.prefill_decode_interval, 0, float(self.reserve_ratio), self.eos_token,
                       self.page_seed & 0xFFFFFFFFFFFFFFFF, int(self.emit_messages), self.codec_coalesce_frames,
                       self.codec_coalesce_first_frames, self.codec_coalesce_early_frames)


@dataclass
class StepPlan:
    """One step of the event loop (the batch get_next_batch_to_run hands back)."""

    mode: int
    decode_rows: int
    moves_src: np.ndarray      # i32: per-row state moves, applied before the step
    moves_dst: np.ndarray
    decode_pages: np.ndarray   # i32: pages the decode rows open, in row order
    new_rid: np.ndarray        # i64: admitted streams, rows decode_rows + i
    new_slot: np.ndarray       # i32: their req_to_token rows
    new_prompt_len: np.ndarray  # i64
    new_page_indptr: np.ndarray  # i32 [new + 1]
    new_pages: np.ndarray      # i32
    retracted: np.ndarray      # i64: streams sent back to the waiting queue
    new_tokens: int

    @property
    def new_rows(self) -> int:
        return int(self.new_rid.shape[0])

    @property
    def rows(self) -> int:
        """Rows whose layer-0 codes process_batch_result takes."""
        return self.decode_rows + self.new_rows

    def is_idle(self) -> bool:
        return self.mode == IDLE


class OmniScheduler:
    """The talker stage's continuous-batching scheduler (C++ core)."""

    def __init__(self, cfg: SchedulerConfig):
        self.cfg = cfg
        self._lib = _lib.load()
        self._c_cfg = cfg.to_c()
        h = self._lib.omni_sched_create(ctypes.byref(self._c_cfg))
        if not h:
            raise ValueError(f"omni_sched_create: {_lib.last_error()}")
        self._h = ctypes.c_void_p(h)
        B = cfg.max_batch
        self._bufs = {
            "move_src": np.zeros(B, np.int32), "move_dst": np.zeros(B, np.int32),
            "decode_pages": np.zeros(B, np.int32), "new_rid": np.zeros(B, np.int64),
            "new_slot": np.zeros(B, np.int32), "new_prompt_len": np.zeros(B, np.int64),
            "new_page_indptr": np.zeros(B + 1, np.int32), "new_pages": np.zeros(max(cfg.num_pages, 1), np.int32),
            "retracted_rid": np.zeros(B, np.int64),
        }
        self._plan = _Plan()
        for k, a in self._bufs.items():
            setattr(self._plan, k, a.ctypes.data)
        self._finished = np.zeros(B, np.int64)
        self._msg_buf: np.ndarray | None = None
        self._t0 = time.perf_counter()

    def close(self) -> None:
        if self._h:
            self._lib.omni_sched_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def _call(self, name: str, *args) -> None:
        _lib.check(getattr(self._lib, name)(self._h, *args), name)

    # ------------------------------------------------------------------
    def add_request(self, rid: int, prompt_len: int, max_frames: int) -> None:
        self._call("omni_sched_add_request", int(rid), int(prompt_len), int(max_frames))

    def abort(self, rid: int) -> None:
        self._call("omni_sched_abort", int(rid))

    def now_us(self) -> int:
        return int((time.perf_counter() - self._t0) * 1e6)

    def get_next_batch_to_run(self, now_us: int | None = None) -> StepPlan:
        self._call("omni_sched_schedule", int(self.now_us() if now_us is None else now_us), ctypes.byref(self._plan))
        p, b = self._plan, self._bufs
        n = p.new_rows
        return StepPlan(
            mode=p.mode, decode_rows=p.decode_rows,
            moves_src=b["move_src"][: p.num_moves].copy(), moves_dst=b["move_dst"][: p.num_moves].copy(),
            decode_pages=b["decode_pages"][: p.num_decode_pages].copy(),
            new_rid=b["new_rid"][:n].copy(), new_slot=b["new_slot"][:n].copy(),
            new_prompt_len=b["new_prompt_len"][:n].copy(), new_page_indptr=b["new_page_indptr"][: n + 1].copy(),
            new_pages=b["new_pages"][: int(b["new_page_indptr"][n]) if n else 0].copy(),
            retracted=b["retracted_rid"][: p.num_retracted].copy(), new_tokens=int(p.new_tokens))

    def process_batch_result(self, codes) -> list[int]:
        """Close the step with its rows' codes: [rows] layer-0 codes or [rows, G] whole
        frames (column 0 = layer 0; frames feed the vocoder messages); returns the
        finished rids."""
        c = np.asarray(codes, dtype=np.int64)
        if c.ndim == 1:
            c = c.reshape(-1, 1)
        c = np.ascontiguousarray(c)
        nf = ctypes.c_int64(0)
        self._call("omni_sched_commit", c.ctypes.data, c.shape[0], c.shape[1], self._finished.ctypes.data,
                   ctypes.byref(nf))
        return self._finished[: nf.value].tolist()

    def pop_messages(self, groups: int) -> list[tuple[int, int, np.ndarray, bool]]:
        """Drain the vocoder message queue: (rid, first frame, codes [frames, groups], final)."""
        out = []
        rid, first, frames, final = ctypes.c_int64(0), ctypes.c_int64(0), ctypes.c_int32(0), ctypes.c_int32(0)
        buf = self._msg_buf
        if buf is None or buf.shape[0] < 64 * groups:
            buf = self._msg_buf = np.zeros(64 * groups, np.int64)
        while True:
            rc = self._lib.omni_sched_pop_message(self._h, ctypes.byref(rid), ctypes.byref(first),
                                                  ctypes.byref(frames), ctypes.byref(final), buf.ctypes.data,
                                                  buf.shape[0])
            if rc == _lib.OMNI_ERR_CAPACITY:
                buf = self._msg_buf = np.zeros(buf.shape[0] * 4, np.int64)
                continue
            _lib.check(rc, "omni_sched_pop_message")
            if frames.value == 0:
                return out
            n = frames.value
            out.append((rid.value, first.value, buf[: n * groups].reshape(n, groups).copy(), bool(final.value)))

    def rollback_decode_prep_after_skip(self) -> None:
        self._call("omni_sched_rollback")

    # ------------------------------------------------------------------
    def stats(self) -> dict:
        out = np.zeros(10, np.int64)
        self._call("omni_sched_stats", out.ctypes.data, 10)
        keys = ("waiting", "running", "free_pages", "free_slots", "steps", "frames", "finished", "retracted",
                "messages", "frames_emitted")
        return dict(zip(keys, (int(v) for v in out)))

    def row_rids(self) -> list[int]:
        out = np.zeros(self.cfg.max_batch, np.int64)
        n = ctypes.c_int64(0)
        self._call("omni_sched_row_rids", out.ctypes.data, out.shape[0], ctypes.byref(n))
        return out[: n.value].tolist()

    def request_state(self, rid: int) -> tuple[int, int, list[int]]:
        """(slot, seq_len, pages) of a live stream."""
        slot, seq, n = ctypes.c_int32(0), ctypes.c_int64(0), ctypes.c_int64(0)
        self._call("omni_sched_request_state", int(rid), ctypes.byref(slot), ctypes.byref(seq), None, 0,
                   ctypes.byref(n))
        pages = np.zeros(max(n.value, 1), np.int32)
        self._call("omni_sched_request_state", int(rid), None, None, pages.ctypes.data, pages.shape[0],
                   ctypes.byref(n))
        return slot.value, seq.value, pages[: n.value].tolist()

    def check(self) -> None:
        """Raise if the allocator or the rows are inconsistent."""
        self._call("omni_sched_check")
