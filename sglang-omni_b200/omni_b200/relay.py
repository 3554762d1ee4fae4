"""The codec-frame relay between the talker stage and the vocoder stage: one
single-producer / single-consumer ring of messages in POSIX shared memory (the C
ring of libomni_b200.so, include/omni_relay.h).

It carries what the talker hands the vocoder (emit_code_chunks_and_feedback,
sglang_omni/models/qwen3_omni/talker_model_runner.py:178-235): a stream's code
chunk [frames, groups] with its first frame index and whether it is the stream's
last.  The reference moves such chunks through its generic stage relays
(sglang_omni/relay/shm.py: one shared-memory block per tensor and a control
message per transfer); code chunks are a few KB and already on the host after the
step's one device-to-host copy, so one persistent ring carries them instead.
"""

from __future__ import annotations

import ctypes

import numpy as np

from omni_b200 import _lib


class CodecRelay:
    """One side of a relay: create=True on the talker (producer), False on the vocoder."""

    def __init__(self, name: str, *, create: bool, capacity_bytes: int = 1 << 22):
        self._lib = _lib.load()
        self.name = name
        self.create = create
        h = self._lib.omni_relay_open(name.encode(), int(capacity_bytes), int(create))
        if not h:
            raise ValueError(f"omni_relay_open: {_lib.last_error()}")
        self._h = ctypes.c_void_p(h)
        self._buf = np.zeros(1 << 12, np.int64)

    def close(self, unlink: bool | None = None) -> None:
        if self._h:
            self._lib.omni_relay_close(self._h, int(self.create if unlink is None else unlink))
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def push(self, rid: int, first_frame: int, codes: np.ndarray, final: bool) -> bool:
        """Append one message; False when the ring is full (retry after the consumer drains)."""
        c = np.ascontiguousarray(codes, dtype=np.int64)
        if c.ndim == 1:
            c = c.reshape(1, -1)
        rc = self._lib.omni_relay_push(self._h, int(rid), int(first_frame), c.shape[0], c.shape[1], int(final),
                                       c.ctypes.data)
        if rc == _lib.OMNI_ERR_CAPACITY:
            return False
        _lib.check(rc, "omni_relay_push")
        return True

    def pop(self) -> tuple[int, int, np.ndarray, bool] | None:
        """The oldest message (rid, first frame, codes [frames, groups], final), or None."""
        rid, first = ctypes.c_int64(0), ctypes.c_int64(0)
        frames, groups, final = ctypes.c_int32(0), ctypes.c_int32(0), ctypes.c_int32(0)
        while True:
            rc = self._lib.omni_relay_pop(self._h, ctypes.byref(rid), ctypes.byref(first), ctypes.byref(frames),
                                          ctypes.byref(groups), ctypes.byref(final), self._buf.ctypes.data,
                                          self._buf.shape[0])
            if rc == _lib.OMNI_ERR_CAPACITY:
                self._buf = np.zeros(self._buf.shape[0] * 4, np.int64)
                continue
            _lib.check(rc, "omni_relay_pop")
            if frames.value == 0:
                return None
            n, g = frames.value, groups.value
            return rid.value, first.value, self._buf[: n * g].reshape(n, g).copy(), bool(final.value)

    def stats(self) -> dict:
        out = np.zeros(4, np.int64)
        _lib.check(self._lib.omni_relay_stats(self._h, out.ctypes.data, 4), "omni_relay_stats")
        return dict(zip(("pushed", "popped", "bytes_in_ring", "capacity"), (int(v) for v in out)))
