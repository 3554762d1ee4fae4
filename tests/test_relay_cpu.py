"""The codec-frame relay (include/omni_relay.h): ordered, lossless delivery of
variable-size code chunks between two processes through the shared-memory ring,
including wrap-around at the end of the ring and a full ring (push refuses,
nothing is lost).  Host code only."""

from __future__ import annotations

import os
import sys
import time
import uuid
from pathlib import Path

import numpy as np
import pytest
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parent.parent


def _name() -> str:
    return f"/omni_relay_test_{os.getpid()}_{uuid.uuid4().hex[:8]}"


def _message(i: int, groups: int = 32):
    rng = np.random.default_rng(i)
    frames = int(rng.integers(1, 12))
    return i, i * 3 + 1, rng.integers(0, 2048, (frames, groups)).astype(np.int64), bool(i % 7 == 0)


def test_roundtrip_order_and_wraparound():
    from omni_b200.relay import CodecRelay

    name = _name()
    tx = CodecRelay(name, create=True, capacity_bytes=8192)
    rx = CodecRelay(name, create=False)
    try:
        assert rx.pop() is None
        got = []
        for i in range(200):  # each message ~0.3-3 KB: many laps of the 8 KB ring
            m = _message(i)
            while not tx.push(*m):
                got.append(rx.pop())
            if i % 3 == 0:
                got.append(rx.pop())
        while (x := rx.pop()) is not None:
            got.append(x)
        got = [g for g in got if g is not None]
        assert len(got) == 200
        for i, (rid, first, codes, final) in enumerate(got):
            want = _message(i)
            assert (rid, first, final) == (want[0], want[1], want[3])
            np.testing.assert_array_equal(codes, want[2])
        st = tx.stats()
        assert st["pushed"] == st["popped"] == 200 and st["bytes_in_ring"] == 0
    finally:
        rx.close()
        tx.close()


def test_full_ring_refuses_without_loss():
    from omni_b200.relay import CodecRelay

    name = _name()
    tx = CodecRelay(name, create=True, capacity_bytes=4096)
    rx = CodecRelay(name, create=False)
    try:
        codes = np.arange(10 * 8, dtype=np.int64).reshape(10, 8)  # 680-byte records
        n = 0
        while tx.push(n, 0, codes, False):
            n += 1
        assert 4 <= n <= 6
        assert not tx.push(99, 0, codes, False)
        for k in range(n):
            rid, _, c, _ = rx.pop()
            assert rid == k
            np.testing.assert_array_equal(c, codes)
        assert rx.pop() is None and tx.push(n, 0, codes, True)
        with pytest.raises(ValueError):
            tx.push(1, 0, np.zeros((40, 8), np.int64), False)  # more than half the ring
    finally:
        rx.close()
        tx.close()


def test_open_errors():
    from omni_b200.relay import CodecRelay

    with pytest.raises(ValueError):
        CodecRelay(_name(), create=False)            # no such relay
    with pytest.raises(ValueError):
        CodecRelay(_name(), create=True, capacity_bytes=5000)  # not a power of two
    with pytest.raises(ValueError):
        CodecRelay("no_slash", create=True)


def _consumer(name: str, count: int, out: str) -> None:
    for p in (str(ROOT), str(ROOT / "sglang-omni_b200")):
        if p not in sys.path:
            sys.path.insert(0, p)
    from omni_b200.relay import CodecRelay

    rx = CodecRelay(name, create=False)
    got, deadline = [], time.time() + 60
    while len(got) < count and time.time() < deadline:
        m = rx.pop()
        if m is None:
            time.sleep(0.0005)
            continue
        got.append(m)
    np.save(out, np.array([len(got)] + [int(c.sum()) + r * 7 + f * 3 + int(fin) for r, f, c, fin in got]))
    rx.close(unlink=False)


def test_two_processes(tmp_path):
    from omni_b200.relay import CodecRelay

    name = _name()
    count = 3000
    tx = CodecRelay(name, create=True, capacity_bytes=1 << 14)
    try:
        ctx = mp.get_context("spawn")
        proc = ctx.Process(target=_consumer, args=(name, count, str(tmp_path / "rx.npy")))
        proc.start()
        deadline = time.time() + 60
        for i in range(count):
            m = _message(i)
            while not tx.push(*m):
                assert time.time() < deadline, "consumer stalled"
                time.sleep(0.0002)
        proc.join(timeout=90)
        assert proc.exitcode == 0
        res = np.load(tmp_path / "rx.npy")
        assert res[0] == count
        want = [int(c.sum()) + r * 7 + f * 3 + int(fin) for r, f, c, fin in (_message(i) for i in range(count))]
        assert res[1:].tolist() == want
    finally:
        tx.close()
