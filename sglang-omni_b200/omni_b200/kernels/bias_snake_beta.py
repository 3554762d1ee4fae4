"""SnakeBeta of a conv's output plus its bias (and a residual), fused, on the B200 library.

Drop-in for sglang_omni/kernels/bias_snake_beta.py: the same SnakeBetaCoefficients and
fused_bias_snake_beta(conv_output, bias, coefficients, out, *, residual=None,
sum_out=None), rounded where the eager adds and SnakeBeta round in the activations'
dtype (bias_snake_beta.py:56-97).
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Protocol

import torch

from omni_b200 import _lib

_DTYPES = {torch.bfloat16: 0, torch.float16: 1, torch.float32: 2}


class SnakeBetaParameters(Protocol):
    alpha: torch.Tensor
    beta: torch.Tensor
    no_div_by_zero: float


@dataclass(frozen=True, kw_only=True)
class SnakeBetaCoefficients:
    """exp(alpha) and 1 / (exp(beta) + epsilon) per channel, computed by the ops the
    activation's forward runs (bias_snake_beta.py:28-43)."""

    alpha_scale: torch.Tensor
    inverse_beta: torch.Tensor

    @classmethod
    @torch.no_grad()
    def from_activation(cls, activation: SnakeBetaParameters) -> "SnakeBetaCoefficients":
        return cls(
            alpha_scale=torch.exp(activation.alpha),
            inverse_beta=1.0 / (torch.exp(activation.beta) + activation.no_div_by_zero),
        )


def fused_bias_snake_beta(
    conv_output: torch.Tensor,
    bias: torch.Tensor,
    coefficients: SnakeBetaCoefficients,
    out: torch.Tensor,
    *,
    residual: torch.Tensor | None = None,
    sum_out: torch.Tensor | None = None,
) -> None:
    """SnakeBeta(conv_output + bias, + residual if given) into out, the sum into sum_out if
    given.  [B, L, C] bf16 or fp16; rows of conv_output and out may sit in longer buffers,
    residual and sum_out are contiguous."""
    batch, length, channels = conv_output.shape
    if conv_output.stride()[1:] != (channels, 1) or out.stride()[1:] != (channels, 1):
        raise ValueError("each row of conv_output and out is one contiguous span")
    if any(t is not None and not t.is_contiguous() for t in (residual, sum_out)):
        raise ValueError("residual and sum_out are contiguous")
    params = [coefficients.alpha_scale.contiguous(), coefficients.inverse_beta.contiguous(), bias.contiguous()]
    _lib.call(
        "omni_bias_snake_beta",
        conv_output.data_ptr(),
        conv_output.stride(0),
        params[2].data_ptr(),
        _lib.ptr(residual),
        _lib.ptr(sum_out),
        out.data_ptr(),
        out.stride(0),
        params[0].data_ptr(),
        params[1].data_ptr(),
        batch,
        length,
        channels,
        _DTYPES[out.dtype],
        _lib.stream_of(out.device),
    )
