"""Seeded sampling of the code predictor's residual codebooks, on sm_100a.

Drop-in for sglang_omni/models/qwen3_tts/sampling_kernels.py: the same public
functions with the same arguments, return values and None-for-unsupported
contract (sampling_kernels.py:836-866), backed by omni_sample_topk_topp /
omni_sample_sorted_seeded of libomni_b200.so.

Semantics (identical to the reference's fused kernel and its torch fallback,
sglang_model.py:1987-2034):

- scores = f32(bf16 logits) / max(temperature, 1e-5);
- top-k candidates ordered by (score desc, index asc) for widths > 32; for
  widths <= 32 gathered in torch.topk's order and sorted by its unstable
  32-entry bitonic network (sampling_kernels.py:123-312, 462-516);
- softmax over ranks < top_k, top-p drops ranks with cdf - p >= top_p
  (rank 0 kept), log-probabilities;
- Gumbel-max with u = murmur3(seed lo, seed hi, position, rank) / (2^32 - 1)
  in float64 and sglang's endpoint clamp (sampling_kernels.py:67-78).

The kernel never reads device values on the host, so the call is CUDA-graph
capturable.
"""

from __future__ import annotations

import torch

from omni_b200 import _lib

FUSED_SAMPLER_VOCAB_SIZE = 2048
FUSED_RAW_LOGIT_TOP_KS = frozenset((4, 8, 16, 32, 50, 64, 128, 256, 512, 1024))
MAX_FUSED_VOCAB = 4096


def next_power_of_2(value: int) -> int:
    return 1 << (int(value) - 1).bit_length()


def fused_raw_logit_block_k(max_top_k: int) -> int | None:
    """The power-of-two selection width of a graph signature (sampling_kernels.py:792-804)."""
    if max_top_k not in FUSED_RAW_LOGIT_TOP_KS:
        return None
    if max_top_k <= 32:
        return 32
    return next_power_of_2(max_top_k)


def _rows_ok(batch: int, device: torch.device, tensors, dtypes) -> bool:
    for t, dt in zip(tensors, dtypes):
        if (
            t.device != device
            or t.ndim != 1
            or t.shape[0] != batch
            or not t.is_contiguous()
            or t.dtype is not dt
        ):
            return False
    return True


def sample_from_logits_with_seed_top_k_top_p(
    logits: torch.Tensor,
    temperatures: torch.Tensor,
    top_ks: torch.Tensor,
    top_ps: torch.Tensor,
    seeds: torch.Tensor,
    positions: torch.Tensor,
    *,
    max_top_k: int,
    has_top_p: bool,
) -> torch.Tensor | None:
    """Seeded temperature/top-k/top-p draw from raw bf16 logits [rows, vocab].

    Returns int64 token ids [rows], or None when the call is outside the fused
    contract (the caller keeps its own path), as the reference does.
    """
    block_k = fused_raw_logit_block_k(int(max_top_k))
    if (
        block_k is None
        or not logits.is_cuda
        or logits.ndim != 2
        or logits.dtype is not torch.bfloat16
        or not logits.is_contiguous()
        or logits.shape[1] % 8 != 0
        or logits.shape[1] > MAX_FUSED_VOCAB
        or logits.shape[1] < block_k
    ):
        return None
    batch = int(logits.shape[0])
    if batch == 0:
        return torch.empty((0,), device=logits.device, dtype=torch.long)
    if not _rows_ok(
        batch,
        logits.device,
        (temperatures, top_ks, top_ps, seeds, positions),
        (torch.float32, torch.long, torch.float32, torch.long, torch.long),
    ):
        return None
    out = torch.empty((batch,), device=logits.device, dtype=torch.long)
    with torch.cuda.device(logits.device):
        _lib.call(
            "omni_sample_topk_topp",
            logits.data_ptr(),
            batch,
            logits.shape[1],
            logits.stride(0),
            temperatures.data_ptr(),
            top_ks.data_ptr(),
            top_ps.data_ptr(),
            seeds.data_ptr(),
            positions.data_ptr(),
            int(max_top_k),
            1 if has_top_p else 0,
            out.data_ptr(),
            _lib.stream_of(logits.device),
        )
    return out


def sample_from_sorted_logprobs_with_seed_small_k(
    logprobs: torch.Tensor,
    sorted_idx: torch.Tensor,
    seeds: torch.Tensor,
    positions: torch.Tensor,
) -> torch.Tensor | None:
    """Seeded Gumbel-max over pre-sorted fp32 log-probabilities [rows, cols <= 1024]
    (sampling_kernels.py:721-790)."""
    if not (logprobs.is_cuda and sorted_idx.is_cuda and seeds.is_cuda and positions.is_cuda):
        return None
    if logprobs.ndim != 2 or sorted_idx.shape != logprobs.shape:
        return None
    if seeds.ndim != 1 or positions.ndim != 1:
        return None
    batch, cols = logprobs.shape
    if batch == 0:
        return torch.empty((0,), device=logprobs.device, dtype=torch.long)
    if seeds.shape[0] != batch or positions.shape[0] != batch:
        return None
    if cols <= 0 or cols > 1024:
        return None
    lp = logprobs.to(torch.float32).contiguous()
    idx = sorted_idx.to(torch.long).contiguous()
    sd = seeds.to(torch.long).contiguous()
    pos = positions.to(torch.long).contiguous()
    out = torch.empty((batch,), device=logprobs.device, dtype=torch.long)
    with torch.cuda.device(logprobs.device):
        _lib.call(
            "omni_sample_sorted_seeded",
            lp.data_ptr(),
            idx.data_ptr(),
            batch,
            cols,
            sd.data_ptr(),
            pos.data_ptr(),
            out.data_ptr(),
            _lib.stream_of(logprobs.device),
        )
    return out


def predictor_sample_step(
    logits: torch.Tensor,
    *,
    temperatures: torch.Tensor,
    top_ks: torch.Tensor,
    top_ps: torch.Tensor,
    seeds: torch.Tensor,
    positions: torch.Tensor,
    pos_mul: int,
    pos_add: int,
    do_sample: torch.Tensor | None,
    argmax_all: bool,
    max_top_k: int,
    has_top_p: bool,
    codes: torch.Tensor,
    table: torch.Tensor | None,
    gathered: torch.Tensor | None,
    summed: torch.Tensor | None,
    gathered_ss: torch.Tensor | None = None,
) -> None:
    """One fused residual-codebook step of the code predictor: sample (or argmax)
    the code from lm_head logits, write codes[:, 0], gather its embedding row into
    gathered and add it to summed (sglang_model.py:1819-1878).  Raises on an
    unsupported contract: the predictor loop has no other path."""
    rows = int(logits.shape[0])
    _lib.call(
        "omni_predictor_sample_step",
        logits.data_ptr(),
        rows,
        logits.shape[1],
        logits.stride(0),
        _lib.ptr(temperatures),
        _lib.ptr(top_ks),
        _lib.ptr(top_ps),
        _lib.ptr(seeds),
        _lib.ptr(positions),
        int(pos_mul),
        int(pos_add),
        _lib.ptr(do_sample),
        1 if argmax_all else 0,
        int(max_top_k) if not argmax_all else 32,
        1 if has_top_p else 0,
        codes.data_ptr(),
        codes.stride(0),
        _lib.ptr(table),
        0 if table is None else table.shape[1],
        _lib.ptr(gathered),
        _lib.ptr(summed),
        _lib.ptr(gathered_ss),
        _lib.stream_of(logits.device),
    )


def layer0_sample(
    logits: torch.Tensor,
    *,
    penalties: torch.Tensor,
    repetition_mask: torch.Tensor | None,
    suppress_mask: torch.Tensor | None,
    temperatures: torch.Tensor,
    top_ks: torch.Tensor,
    top_ps: torch.Tensor,
    min_ps: torch.Tensor | None,
    seeds: torch.Tensor,
    positions: torch.Tensor,
    max_top_k: int,
    out: torch.Tensor | None = None,
    rep_mask_update: torch.Tensor | None = None,
) -> torch.Tensor:
    """Layer-0 codec token draw from fp32 logits [rows, vocab]: repetition penalty,
    suppression, temperature, top-k/top-p/min-p and the seeded Gumbel draw
    (talker.py:1376-1412)."""
    rows, vocab = logits.shape
    if out is None:
        out = torch.empty((rows,), device=logits.device, dtype=torch.long)

    def u8(m):
        return None if m is None else m.view(torch.uint8)

    _lib.call(
        "omni_layer0_sample",
        logits.data_ptr(),
        rows,
        vocab,
        logits.stride(0),
        penalties.data_ptr(),
        _lib.ptr(u8(repetition_mask)),
        _lib.ptr(u8(suppress_mask)),
        temperatures.data_ptr(),
        top_ks.data_ptr(),
        top_ps.data_ptr(),
        _lib.ptr(min_ps),
        seeds.data_ptr(),
        positions.data_ptr(),
        int(max_top_k),
        out.data_ptr(),
        _lib.ptr(u8(rep_mask_update)),
        _lib.stream_of(logits.device),
    )
    return out


__all__ = [
    "FUSED_RAW_LOGIT_TOP_KS",
    "FUSED_SAMPLER_VOCAB_SIZE",
    "fused_raw_logit_block_k",
    "layer0_sample",
    "next_power_of_2",
    "predictor_sample_step",
    "sample_from_logits_with_seed_top_k_top_p",
    "sample_from_sorted_logprobs_with_seed_small_k",
]
