"""CPU restatement of the streaming vocoder step's kernels — TEST INFRASTRUCTURE ONLY.

PyTorch-CPU arithmetic, following:

- snake_beta: fused_bias_snake_beta (sglang_omni/kernels/bias_snake_beta.py:56-97):
  SnakeBeta(conv + bias [+ residual]), every intermediate rounded to the activations'
  dtype where the eager adds and SnakeBeta (transformers' Qwen3-Omni SnakeBeta: x +
  1 / (exp(beta) + eps) * sin(x * exp(alpha))^2) round: conv + bias, + residual, the
  phase, its sine, the square, the scaled square, the final add;
- single_output_conv: clamped_single_output_conv (single_output_conv.py:68-102), in
  float64 (the reference's own test compares against a float64 conv, test_single_output_
  conv.py:20-44), clamped to [-1, 1] with NaN kept, rounded once;
- history_exchange / overlap_exchange (codec_state.py:153-210), as index_select /
  index_copy restatements of the slot pools (the reference's tests state them so,
  tests/unit_test/kernels/test_codec_state.py:17-48).

Nothing in the product package imports this module.
"""

from __future__ import annotations

import torch


def snake_beta(conv_output: torch.Tensor, bias: torch.Tensor, alpha_scale: torch.Tensor,
               inverse_beta: torch.Tensor, residual: torch.Tensor | None = None):
    """(out, sum) for [B, L, C] activations in bf16 / fp16 (fp32 / fp64 also, unrounded)."""
    dt = conv_output.dtype
    wide = torch.float64 if dt == torch.float64 else torch.float32

    def r(x: torch.Tensor) -> torch.Tensor:
        return x.to(dt).to(wide)

    total = r(conv_output.to(wide) + bias.to(wide))
    if residual is not None:
        total = r(total + residual.to(wide))
    phase = r(total * alpha_scale.to(wide))
    sine = r(torch.sin(phase))
    sq = r(sine * sine)
    scaled = r(inverse_beta.to(wide) * sq)
    return (total + scaled).to(dt), total.to(dt)


def single_output_conv(padded: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor, length: int) -> torch.Tensor:
    """[B, 1, length] from channels-last padded [B, length + taps - 1, C], weight [1, C, taps]."""
    x = padded.double().transpose(1, 2)
    y = torch.nn.functional.conv1d(x, weight.double(), bias.double())[:, :, :length]
    nan = torch.isnan(y)
    y = y.clamp(min=-1, max=1)
    y[nan] = float("nan")
    return y.to(padded.dtype)


def history_exchange(padded: torch.Tensor, history_pool: torch.Tensor, slot_index: torch.Tensor,
                     new_samples: int, is_cold: bool) -> None:
    """In place: the slot histories in front of the new samples (zeros when cold), zeros
    after them; each slot keeps the last `history` samples of history ++ new."""
    h = int(history_pool.shape[1])
    idx = slot_index.long()
    if is_cold:
        padded[:, :h].zero_()
    else:
        padded[:, :h].copy_(history_pool.index_select(0, idx))
    padded[:, h + new_samples:].zero_()
    history_pool.index_copy_(0, idx, padded[:, new_samples:new_samples + h].clone())


def overlap_exchange(output: torch.Tensor, overlap_pool: torch.Tensor, slot_index: torch.Tensor,
                     emitted_samples: int, is_cold: bool) -> None:
    """In place: the slot overlaps added into the first samples (not when cold); each slot
    keeps the samples past the emitted ones."""
    o = int(overlap_pool.shape[1])
    idx = slot_index.long()
    if not is_cold:
        wide = torch.float64 if output.dtype == torch.float64 else torch.float32
        output[:, :o] = (output[:, :o].to(wide) + overlap_pool.index_select(0, idx).to(wide)).to(output.dtype)
    overlap_pool.index_copy_(0, idx, output[:, emitted_samples:emitted_samples + o].clone())
