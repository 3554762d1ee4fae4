"""Fused codec-embedding gather for the code predictor, on sm_100a.

Drop-in for sglang_omni/models/qwen3_tts/predictor_kernels.py:87-229: same
signature, same False-without-writes contract for calls outside the kernel's
reach, backed by omni_gather_embedding_add.
"""

from __future__ import annotations

import torch

from omni_b200 import _lib


def contiguous_storage_ranges_overlap(first: torch.Tensor, second: torch.Tensor) -> bool:
    a0 = first.data_ptr()
    a1 = a0 + first.numel() * first.element_size()
    b0 = second.data_ptr()
    b1 = b0 + second.numel() * second.element_size()
    return a0 < b1 and b0 < a1


def gather_codec_embedding_and_add(
    token_ids: torch.Tensor,
    embedding_weight: torch.Tensor,
    gathered: torch.Tensor,
    accumulated: torch.Tensor,
    projected_weight: torch.Tensor | None = None,
    projected: torch.Tensor | None = None,
) -> bool:
    """gathered = embedding_weight[token_ids]; accumulated += gathered (bf16);
    with projected_weight also projected = projected_weight[token_ids].
    Returns False without writes when the caller must use its own path."""
    tensors = (token_ids, embedding_weight, gathered, accumulated)
    if not all(t.is_cuda for t in tensors):
        return False
    if token_ids.ndim != 1 or embedding_weight.ndim != 2 or gathered.ndim != 2 or accumulated.ndim != 2:
        return False
    batch = token_ids.shape[0]
    hidden = embedding_weight.shape[1]
    if batch == 0 or hidden == 0:
        return False
    if gathered.shape != (batch, hidden) or accumulated.shape != (batch, hidden):
        return False
    if token_ids.dtype not in (torch.int32, torch.int64):
        return False
    if any(t.dtype != torch.bfloat16 for t in (embedding_weight, gathered, accumulated)):
        return False
    if not (token_ids.device == embedding_weight.device == gathered.device == accumulated.device):
        return False
    if not all(t.is_contiguous() for t in tensors):
        return False
    if (
        contiguous_storage_ranges_overlap(gathered, accumulated)
        or contiguous_storage_ranges_overlap(gathered, embedding_weight)
        or contiguous_storage_ranges_overlap(accumulated, embedding_weight)
    ):
        return False
    assert (projected_weight is None) == (projected is None), "projected_weight and projected are passed together"
    psize = 0
    if projected_weight is not None:
        if not (
            projected_weight.ndim == 2
            and projected.ndim == 2
            and projected_weight.shape[0] == embedding_weight.shape[0]
            and projected_weight.shape[1] <= hidden
            and projected.shape == (batch, projected_weight.shape[1])
            and projected_weight.dtype == torch.bfloat16
            and projected.dtype == torch.bfloat16
            and projected_weight.device == projected.device == token_ids.device
            and projected_weight.is_contiguous()
            and projected.is_contiguous()
            and not contiguous_storage_ranges_overlap(projected, gathered)
            and not contiguous_storage_ranges_overlap(projected, accumulated)
            and not contiguous_storage_ranges_overlap(projected, projected_weight)
        ):
            return False
        psize = projected_weight.shape[1]
    if hidden % 8 != 0 or psize % 8 != 0:
        return False
    with torch.cuda.device(token_ids.device):
        rc = _lib.load().omni_gather_embedding_add(
            token_ids.data_ptr(),
            1 if token_ids.dtype == torch.int32 else 0,
            batch,
            embedding_weight.data_ptr(),
            hidden,
            gathered.data_ptr(),
            accumulated.data_ptr(),
            _lib.ptr(projected_weight),
            psize,
            _lib.ptr(projected),
            _lib.stream_of(token_ids.device),
        )
    if rc == _lib.OMNI_ERR_UNSUPPORTED:
        return False
    _lib.check(rc, "omni_gather_embedding_add")
    return True


__all__ = ["contiguous_storage_ranges_overlap", "gather_codec_embedding_and_add"]
