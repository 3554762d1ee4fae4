"""In-place exchanges of per-slot codec state on the B200 library.

Drop-ins for history_exchange and overlap_exchange (sglang_omni/kernels/codec_state.py:
153-210): a causal conv's history in front of its new samples, and a transposed conv's
overlap added into its output.
"""

from __future__ import annotations

import torch

from omni_b200 import _lib

_DTYPES = {torch.bfloat16: 0, torch.float16: 1, torch.float32: 2}


def history_exchange(padded: torch.Tensor, history_pool: torch.Tensor, slot_index: torch.Tensor,
                     new_samples: int, is_cold: bool) -> None:
    """Fill a causal conv's (rows, history + new + tail, channels) input around the new
    samples: the slot's history in front (zeros for a cold slot), zeros after; then keep
    the last `history` samples of history and new samples as the slot's history."""
    rows, padded_samples, channels = padded.shape
    history = int(history_pool.shape[1])
    tail = padded_samples - history - new_samples
    if tail < 0:
        raise ValueError("padded must hold the history and the new samples")
    slots = slot_index if slot_index.dtype == torch.int64 else slot_index.to(torch.int64)
    _lib.call(
        "omni_history_exchange",
        padded.data_ptr(), *padded.stride(),
        history_pool.data_ptr(), *history_pool.stride(),
        slots.data_ptr(),
        rows, history, new_samples, tail, channels, int(bool(is_cold)), padded.element_size(),
        _lib.stream_of(padded.device),
    )


def overlap_exchange(output: torch.Tensor, overlap_pool: torch.Tensor, slot_index: torch.Tensor,
                     emitted_samples: int, is_cold: bool) -> None:
    """Add each slot's overlap into the front of a transposed conv's (rows, emitted +
    overlap, channels) output (not for a cold slot) and keep the samples past the emitted
    ones as the slot's overlap.  Needs emitted_samples >= the overlap."""
    rows, _, channels = output.shape
    overlap = int(overlap_pool.shape[1])
    slots = slot_index if slot_index.dtype == torch.int64 else slot_index.to(torch.int64)
    _lib.call(
        "omni_overlap_exchange",
        output.data_ptr(), *output.stride(),
        overlap_pool.data_ptr(), *overlap_pool.stride(),
        slots.data_ptr(),
        rows, overlap, emitted_samples, channels, int(bool(is_cold)), _DTYPES[output.dtype],
        _lib.stream_of(output.device),
    )
