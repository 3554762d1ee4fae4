"""The code predictor's fused layer ops on sm_100a.

Drop-in for sglang_omni/utils/predictor_layers.py: ``codebook_step``
(:963-993), ``add_rmsnorm_rounded`` (:603-622), ``PredictorLayerShape``
(:626-635) and the decoder-layer stack ``FusedPredictorLayers`` (:996-1107),
with the same arguments and in-place contracts, backed by libomni_b200.so.

FusedPredictorLayers runs each layer as four tcgen05 GEMMs with fused
epilogues plus the cached attention (omni_b200.predictor's chain): the input
RMSNorm and the post-attention RMSNorm are folded into the columns of the qkv
and gate_up weights (their row scale is applied in the GEMM epilogue from the
sums of squares the previous residual epilogue wrote), the qkv epilogue does the
q/k RMSNorm, the neox rotary embedding and the K/V store at the row's cache slot,
and the o_proj / down epilogues add the residual.  The folded weights are built
once per layer weight and cached.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch

from omni_b200 import _lib, ops

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


def add_rmsnorm_rounded(x: torch.Tensor, residual: torch.Tensor, weight: torch.Tensor,
                        eps: float) -> tuple[torch.Tensor, torch.Tensor]:
    """In place: residual becomes bf16(x + residual), x becomes RMSNorm(residual) * weight;
    returns (x, residual) (predictor_layers.py:603-622).  Rows of HIDDEN_SIZE bf16, one
    warp a row: each lane squares and adds its eight values in column order without
    fused multiply-adds, the lanes combine by an xor butterfly 1, 2, 4, 8, 16, and the
    output is value * rstd * weight rounded once, as the reference's kernel does."""
    if (x.dtype is not torch.bfloat16 or residual.dtype is not torch.bfloat16 or weight.dtype is not torch.bfloat16
            or x.shape != residual.shape or x.ndim != 2 or x.shape[1] != HIDDEN_SIZE or x.stride(1) != 1
            or residual.stride(1) != 1 or not weight.is_contiguous() or weight.numel() != HIDDEN_SIZE):
        raise ValueError("add_rmsnorm_rounded needs bf16 [rows, 1024] rows and a bf16 [1024] weight")
    ops.rmsnorm(x, weight, eps, addend=residual, residual_out=residual, out=x)
    return x, residual


@dataclass(frozen=True)
class PredictorLayerShape:
    """The predictor layer's dimensions (predictor_layers.py:626-635); split_qkv and
    split_hidden (the reference's K split of its residual launches) are accepted for
    interface parity: the split here is planned by the GEMM itself."""

    hidden_size: int
    head_dim: int
    num_q_heads: int
    num_kv_heads: int
    intermediate_size: int
    split_qkv: int = 0
    split_hidden: int = 0


def _eps(module) -> float:
    for name in ("variance_epsilon", "eps"):
        v = getattr(module, name, None)
        if v is not None:
            return float(v)
    return 1e-6


class FusedPredictorLayers:
    """The predictor's decoder layers with q, the attention output, the residual stream
    and the MLP activation in buffers of max_rows rows (predictor_layers.py:996-1025)."""

    def __init__(self, shape: PredictorLayerShape, max_rows: int, device: torch.device,
                 dtype: torch.dtype = torch.bfloat16) -> None:
        if dtype is not torch.bfloat16:
            raise ValueError("the fused predictor layers run in bf16")
        if shape.hidden_size % 128 or shape.num_q_heads % shape.num_kv_heads:
            raise ValueError("hidden_size must be a multiple of 128 and Hq a multiple of Hkv")
        self.shape = shape
        self.max_rows = max_rows
        self.device = torch.device(device)
        bf = dict(device=self.device, dtype=dtype)
        H, D = shape.hidden_size, shape.head_dim
        self.q = torch.zeros(max_rows, shape.num_q_heads * D, **bf)
        self.attention_output = torch.zeros_like(self.q)
        self.residual = torch.zeros(max_rows, H, **bf)
        self.stream = torch.zeros(max_rows, H, **bf)  # the layer input, copied with its sums of squares
        self.activated = torch.zeros(max_rows, shape.intermediate_size, **bf)
        self.normed = torch.zeros(max_rows, H, **bf)
        f32 = dict(device=self.device, dtype=torch.float32)
        self.ss = torch.zeros(H // 128, max_rows, **f32)
        self.ss_in = torch.zeros(max_rows, **f32)
        self._folded: dict[tuple[int, int], torch.Tensor] = {}
        self._rope: dict[int, torch.Tensor] = {}

    def covers(self, rows: int) -> bool:
        return rows <= self.max_rows

    def _fold(self, weight: torch.Tensor, gain: torch.Tensor) -> torch.Tensor:
        key = (weight.data_ptr(), gain.data_ptr())
        w = self._folded.get(key)
        if w is None:
            w = ops.fold_norm(weight, gain)
            self._folded[key] = w
        return w

    def _cos_sin(self, attention, end: int) -> torch.Tensor:
        cache = getattr(getattr(attention, "rotary_emb", None), "cos_sin_cache", None)
        if cache is None:
            raise ValueError("the attention module carries no rotary_emb.cos_sin_cache")
        if cache.shape[0] < end:
            raise ValueError("rotary table shorter than the cache slots")
        if cache.dtype is torch.float32 and cache.is_contiguous():
            return cache
        key = cache.data_ptr()
        cs = self._rope.get(key)
        if cs is None:
            cs = cache.float().contiguous()
            self._rope[key] = cs
        return cs

    def forward(self, *, layers, final_norm, token_embeds: torch.Tensor, batch_size: int, cache_len: int,
                positions: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor) -> torch.Tensor:
        """token_embeds (batch, tokens, hidden) at slots cache_len onward; the caches are
        (layer, row, slot, kv head, head dim), the slot being the position (positions
        is row-major (batch, tokens) = cache_len + token, as in the reference).  Writes
        every layer's K/V at those slots and returns the final norm of the residual
        stream as (batch, tokens, hidden)."""
        shape = self.shape
        num_tokens, hidden = token_embeds.shape[1:]
        rows = batch_size * num_tokens
        if rows > self.max_rows:
            raise RuntimeError("FusedPredictorLayers buffers are too small for this batch")
        if hidden != shape.hidden_size:
            raise ValueError("token_embeds hidden size differs from the layer shape")
        L, _, slots, hkv, D = k_cache.shape
        if (v_cache.shape != k_cache.shape or hkv != shape.num_kv_heads or D != shape.head_dim
                or not k_cache.is_contiguous() or not v_cache.is_contiguous()):
            raise ValueError("caches must be contiguous (layer, row, slot, kv head, head dim)")
        end = cache_len + num_tokens
        if end > slots or len(layers) > L:
            raise ValueError("tokens past the cache slots or more layers than cache layers")
        del positions  # implied by the slots: position = slot = cache_len + token
        H, hq = shape.hidden_size, shape.num_q_heads
        parts = H // 128
        x = token_embeds.reshape(rows, hidden)
        stream, q, attn, act = self.stream[:rows], self.q[:rows], self.attention_output[:rows], self.activated[:rows]
        h = self.residual[:rows]
        ss_in = self.ss_in[:rows]
        # the layer input and its sums of squares (the folded input norm reads them)
        ops.add_sumsq(x, None, stream, ss_in)
        resid, ss, ss_parts = stream, ss_in, 1
        scale = 1.0 / math.sqrt(D)
        for li, layer in enumerate(layers):
            attention = layer.self_attn
            kc = k_cache[li].view(-1, hkv, D)
            vc = v_cache[li].view(-1, hkv, D)
            eps_in = _eps(layer.input_layernorm)
            ops.linear_fused(resid, self._fold(attention.qkv_proj.weight, layer.input_layernorm.weight), q,
                             epilogue=ops.EPI_QKV_ROPE, ss_in=ss, ss_in_parts=ss_parts, norm_eps=eps_in,
                             qkv=dict(num_q_heads=hq, num_kv_heads=hkv, head_dim=D,
                                      q_norm=attention.q_norm.weight, k_norm=attention.k_norm.weight,
                                      eps=_eps(attention.q_norm), cos_sin=self._cos_sin(attention, end),
                                      tokens_per_req=num_tokens, slot_stride=slots, slot_base=cache_len,
                                      k_cache=kc, v_cache=vc))
            ops.predictor_attention(q, kc, vc, num_q_heads=hq, num_kv_heads=hkv, head_dim=D,
                                    tokens_per_req=num_tokens, slot_stride=slots, slot_base=cache_len,
                                    sm_scale=scale, out=attn)
            ops.linear_fused(attn, attention.o_proj.weight, h, epilogue=ops.EPI_RESIDUAL, residual=resid,
                             ss_out=self.ss)
            resid, ss, ss_parts = h, self.ss, parts
            ops.linear_fused(h, self._fold(layer.mlp.gate_up_proj.weight, layer.post_attention_layernorm.weight),
                             act, epilogue=ops.EPI_SWIGLU, ss_in=self.ss, ss_in_parts=parts,
                             norm_eps=_eps(layer.post_attention_layernorm))
            ops.linear_fused(act, layer.mlp.down_proj.weight, h, epilogue=ops.EPI_RESIDUAL, residual=h,
                             ss_out=self.ss)
        normed = self.normed[:rows]
        ops.rmsnorm(resid, final_norm.weight, _eps(final_norm), out=normed)
        return normed.reshape(batch_size, num_tokens, hidden)


__all__ = ["HIDDEN_SIZE", "PredictorLayerShape", "FusedPredictorLayers", "add_rmsnorm_rounded", "codebook_step"]
