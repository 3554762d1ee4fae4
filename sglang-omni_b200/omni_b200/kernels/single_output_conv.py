"""Clamped single-output-channel conv on the B200 library.

Drop-in for clamped_single_output_conv (sglang_omni/kernels/single_output_conv.py:
68-102): a stride-one, undilated conv from channels-last (B, length + taps - 1, C)
activations to one output channel, bias added, clamped to [-1, 1], accumulated in fp32
and rounded once.
"""

from __future__ import annotations

import torch

from omni_b200 import _lib

_DTYPES = {torch.bfloat16: 0, torch.float16: 1, torch.float32: 2}


def clamped_single_output_conv(padded: torch.Tensor, conv: torch.nn.Conv1d, length: int) -> torch.Tensor:
    batch, padded_length, channels = padded.shape
    taps = conv.kernel_size[0]
    if not (conv.out_channels == 1 and conv.stride == (1,) and conv.dilation == (1,) and conv.groups == 1):
        raise ValueError("a stride-one, undilated, ungrouped conv to one output channel")
    if padded_length != length + taps - 1:
        raise ValueError("the input carries the left context")
    if padded.stride(2) != 1 or padded.stride(1) != channels:
        raise ValueError("contiguous rows")
    output = padded.new_empty(batch, 1, length)
    _lib.call(
        "omni_clamped_single_output_conv",
        padded.data_ptr(),
        padded.stride(0),
        conv.weight.data_ptr(),
        conv.weight.stride(1),
        conv.weight.stride(2),
        conv.bias.data_ptr(),
        output.data_ptr(),
        batch,
        length,
        channels,
        taps,
        _DTYPES[padded.dtype],
        _lib.stream_of(padded.device),
    )
    return output
