"""The windows of a causal conv's channels-last input as its GEMM operand, on the B200
library (omni_conv_window_gather): out[r * length + t, j * C + c] = padded[r, t + j *
dilation, c].  The code2wav runs each ungrouped causal conv as this gather and one
cuBLAS GEMM."""

from __future__ import annotations

import torch

from omni_b200 import _lib


def conv_window_gather(padded: torch.Tensor, length: int, taps: int, dilation: int) -> torch.Tensor:
    rows, samples, channels = padded.shape
    if padded.stride(2) != 1 or padded.stride(1) != channels:
        raise ValueError("padded samples are contiguous channel vectors")
    out = padded.new_empty(rows * length, taps * channels)
    _lib.call("omni_conv_window_gather", padded.data_ptr(), padded.stride(0), samples, rows, length, taps,
              dilation, channels, padded.element_size(), out.data_ptr(), _lib.stream_of(padded.device))
    return out
