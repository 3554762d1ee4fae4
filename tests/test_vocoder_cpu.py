"""CPU checks of the vocoder-step oracle (streaming properties of the codec-state
exchanges, the SnakeBeta rounding points against eager bf16 ops, the float64 conv)."""

from __future__ import annotations

import pytest
import torch

from oracle import vocoder as ov


def eager_snake(x: torch.Tensor, alpha: torch.Tensor, beta: torch.Tensor, eps: float = 1e-9) -> torch.Tensor:
    """transformers' Qwen3-Omni SnakeBeta on channels-last rows, in the rows' dtype."""
    a = torch.exp(alpha)
    b = torch.exp(beta)
    return x + (1.0 / (b + eps)) * torch.pow(torch.sin(x * a), 2)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("with_residual", [False, True])
def test_snake_oracle_rounds_as_the_eager_ops(dtype, with_residual):
    g = torch.Generator().manual_seed(0)
    C = 96
    alpha = (torch.randn(C, generator=g) * 0.5).to(dtype)
    beta = (torch.randn(C, generator=g) * 0.5).to(dtype)
    conv = torch.randn(2, 17, C, generator=g).to(dtype)
    bias = torch.randn(C, generator=g).to(dtype)
    res = torch.randn(2, 17, C, generator=g).to(dtype) if with_residual else None
    out, total = ov.snake_beta(conv, bias, torch.exp(alpha), 1.0 / (torch.exp(beta) + 1e-9), res)
    expected_total = conv + bias + res if with_residual else conv + bias
    assert torch.equal(total, expected_total)
    assert torch.equal(out, eager_snake(expected_total, alpha, beta))


def test_single_output_conv_oracle_clamps_and_keeps_nan():
    g = torch.Generator().manual_seed(1)
    C, taps, L = 8, 7, 50
    padded = torch.randn(2, L + taps - 1, C, generator=g)
    padded[0, 10, 3] = float("nan")
    w = torch.randn(1, C, taps, generator=g)
    b = torch.randn(1, generator=g)
    y = ov.single_output_conv(padded, w, b, L)
    assert y.shape == (2, 1, L)
    assert torch.isnan(y[0, 0, 4:11]).all() and not torch.isnan(y[1]).any()
    finite = y[~torch.isnan(y)]
    assert finite.abs().max() <= 1 and (finite.abs() == 1).any()


@pytest.mark.parametrize("history", [2, 6, 54])
@pytest.mark.parametrize("chunks", [(10, 10, 7), (1, 2, 1, 3, 40), (32, 1, 32)])
def test_history_exchange_builds_the_causal_window(history, chunks):
    g = torch.Generator().manual_seed(history + len(chunks))
    slots, C, tail = 5, 3, 2
    total = sum(chunks)
    streams = torch.randn(slots, total, C, generator=g)
    pool = torch.randn(slots, history, C, generator=g)  # stale until the first (cold) call
    slot_index = torch.tensor([3, 0, 4])
    start = 0
    for i, n in enumerate(chunks):
        padded = torch.full((3, history + n + tail, C), 7.0)
        padded[:, history:history + n] = streams[slot_index, start:start + n]
        ov.history_exchange(padded, pool, slot_index, n, is_cold=i == 0)
        for r, s in enumerate(slot_index.tolist()):
            window = torch.zeros(history + n, C)
            lo = start - history
            src = streams[s, max(lo, 0):start + n]
            window[history + n - src.shape[0]:] = src
            assert torch.equal(padded[r, :history + n], window)
            assert not padded[r, history + n:].any()
        start += n


@pytest.mark.parametrize("overlap,emitted", [(3, 5), (4, 4)])
def test_overlap_exchange_is_the_whole_stream_overlap_add(overlap, emitted):
    g = torch.Generator().manual_seed(overlap)
    rows, C, chunks = 2, 4, 4
    pool = torch.zeros(rows, overlap, C)
    slot = torch.tensor([1, 0])
    pool_full = torch.zeros(2, overlap, C)
    pieces = [torch.randn(rows, emitted + overlap, C, generator=g) for _ in range(chunks)]
    # whole stream: chunk k lands at k * emitted, overlap-added
    whole = torch.zeros(rows, chunks * emitted + overlap, C)
    for k, pc in enumerate(pieces):
        whole[:, k * emitted:k * emitted + emitted + overlap] += pc
    got = []
    for k, pc in enumerate(pieces):
        out = pc.clone()
        ov.overlap_exchange(out, pool_full, slot, emitted, is_cold=k == 0)
        got.append(out[:, :emitted])
    assert torch.allclose(torch.cat(got, 1), whole[:, :chunks * emitted], atol=1e-6)
    del pool
