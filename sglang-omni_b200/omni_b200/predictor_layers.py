"""The code predictor's fused layer ops on sm_100a.

Drop-in for sglang_omni/utils/predictor_layers.py: ``codebook_step``
(:963-993), ``add_rmsnorm_rounded`` (:603-622) and the decoder-layer stack
``FusedPredictorLayers`` (:996-1107), backed by libomni_b200.so.
"""

from __future__ import annotations

import torch

from omni_b200 import _lib

HIDDEN_SIZE = 1024


def codebook_step(
    logits: torch.Tensor,
    embedding_weight: torch.Tensor,
    codes: torch.Tensor,
    summed: torch.Tensor,
) -> torch.Tensor:
    """codes = argmax(logits) as torch.argmax picks it (first NaN, else first
    maximum); summed += embedding[codes] in place; returns the next pass's input
    rows (rows, 1, hidden).  logits is (rows, vocab) bf16, codes a (rows,) int64
    view (any row stride), summed (rows, hidden) bf16 with contiguous rows."""
    rows, vocab = logits.shape
    hidden = embedding_weight.shape[1]
    if summed.stride(1) != 1 or summed.stride(0) != hidden or logits.stride(1) != 1:
        raise ValueError("codebook_step needs contiguous logits and summed rows")
    codebook_input = torch.empty((rows, 1, hidden), device=summed.device, dtype=summed.dtype)
    _lib.call(
        "omni_codebook_step",
        logits.data_ptr(),
        rows,
        vocab,
        logits.stride(0),
        embedding_weight.data_ptr(),
        hidden,
        codes.data_ptr(),
        codes.stride(0),
        codebook_input.data_ptr(),
        summed.data_ptr(),
        _lib.stream_of(logits.device),
    )
    return codebook_input


__all__ = ["HIDDEN_SIZE", "codebook_step"]
