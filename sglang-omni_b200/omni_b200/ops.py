"""Tensor-level wrappers of the C-ABI kernels used by the talker and predictor.

Each function launches on the current torch stream and raises on a contract
violation (there is no alternative path).  Workspaces are owned by the caller
and must be zero-filled once before first use.
"""

from __future__ import annotations

import torch

from omni_b200 import _lib

EPI_STORE = 0
EPI_RESIDUAL = 1
EPI_SWIGLU = 2
EPI_F32 = 3


def linear_workspace_bytes(rows: int, k: int, n: int, epilogue: int = EPI_STORE, splits: int = 0) -> int:
    return int(_lib.load().omni_linear_workspace_bytes(rows, k, n, epilogue, splits))


def linear(
    x: torch.Tensor,
    w: torch.Tensor,
    *,
    epilogue: int = EPI_STORE,
    residual: torch.Tensor | None = None,
    out: torch.Tensor | None = None,
    workspace: torch.Tensor | None = None,
    splits: int = 0,
) -> torch.Tensor:
    """out = epilogue(x @ w.T) on the tcgen05 tensor cores; x [rows, K] bf16, w [N, K] bf16."""
    rows, k = x.shape
    n = w.shape[0]
    if out is None:
        if epilogue == EPI_SWIGLU:
            out = torch.empty((rows, n // 2), device=x.device, dtype=torch.bfloat16)
        elif epilogue == EPI_F32:
            out = torch.empty((rows, n), device=x.device, dtype=torch.float32)
        else:
            out = torch.empty((rows, n), device=x.device, dtype=torch.bfloat16)
    need = linear_workspace_bytes(rows, k, n, epilogue, splits)
    if need and (workspace is None or workspace.numel() * workspace.element_size() < need):
        workspace = torch.zeros(need, dtype=torch.uint8, device=x.device)
    _lib.call(
        "omni_linear",
        x.data_ptr(),
        rows,
        k,
        x.stride(0),
        w.data_ptr(),
        n,
        epilogue,
        _lib.ptr(residual),
        0 if residual is None else residual.stride(0),
        out.data_ptr(),
        out.stride(0),
        _lib.ptr(workspace),
        0 if workspace is None else workspace.numel() * workspace.element_size(),
        splits,
        _lib.stream_of(x.device),
    )
    return out


def rmsnorm(
    x: torch.Tensor,
    weight: torch.Tensor,
    eps: float,
    *,
    addend: torch.Tensor | None = None,
    residual_out: torch.Tensor | None = None,
    out: torch.Tensor | None = None,
) -> torch.Tensor:
    """out = RMSNorm(x [+ addend]) * weight; the bf16 sum goes to residual_out."""
    rows, hidden = x.shape
    if out is None:
        out = torch.empty_like(x)
    _lib.call(
        "omni_rmsnorm",
        x.data_ptr(),
        x.stride(0),
        _lib.ptr(addend),
        0 if addend is None else addend.stride(0),
        _lib.ptr(residual_out),
        0 if residual_out is None else residual_out.stride(0),
        weight.data_ptr(),
        float(eps),
        out.data_ptr(),
        out.stride(0),
        rows,
        hidden,
        _lib.stream_of(x.device),
    )
    return out


def qknorm_rope_store(
    qkv: torch.Tensor,
    *,
    num_q_heads: int,
    num_kv_heads: int,
    head_dim: int,
    q_norm: torch.Tensor,
    k_norm: torch.Tensor,
    eps: float,
    cos_sin: torch.Tensor,
    q_out: torch.Tensor,
    k_cache: torch.Tensor,
    v_cache: torch.Tensor,
    positions: torch.Tensor | None = None,
    cache_loc: torch.Tensor | None = None,
    tokens_per_req: int = 1,
    slot_stride: int = 1,
    slot_base: int = 0,
) -> None:
    _lib.call(
        "omni_qknorm_rope_store",
        qkv.data_ptr(),
        qkv.stride(0),
        qkv.shape[0],
        num_q_heads,
        num_kv_heads,
        head_dim,
        q_norm.data_ptr(),
        k_norm.data_ptr(),
        float(eps),
        cos_sin.data_ptr(),
        cos_sin.shape[0],
        _lib.ptr(positions),
        _lib.ptr(cache_loc),
        tokens_per_req,
        slot_stride,
        slot_base,
        q_out.data_ptr(),
        q_out.stride(0),
        k_cache.data_ptr(),
        v_cache.data_ptr(),
        _lib.stream_of(qkv.device),
    )


def paged_attention_workspace_bytes(rows: int, num_kv_heads: int, work_capacity: int) -> int:
    return int(_lib.load().omni_paged_attention_workspace_bytes(rows, num_kv_heads, work_capacity))


def paged_decode_attention(
    q: torch.Tensor,
    k_cache: torch.Tensor,
    v_cache: torch.Tensor,
    *,
    page_indptr: torch.Tensor,
    page_indices: torch.Tensor,
    seq_lens: torch.Tensor,
    work_indptr: torch.Tensor,
    num_q_heads: int,
    num_kv_heads: int,
    head_dim: int,
    page_size: int,
    pages_per_chunk: int,
    work_capacity: int,
    sm_scale: float,
    out: torch.Tensor,
    workspace: torch.Tensor,
    grid_ctas: int = 0,
) -> torch.Tensor:
    rows = seq_lens.shape[0]
    _lib.call(
        "omni_paged_decode_attention",
        q.data_ptr(),
        q.stride(0),
        k_cache.data_ptr(),
        v_cache.data_ptr(),
        page_indptr.data_ptr(),
        page_indices.data_ptr(),
        seq_lens.data_ptr(),
        work_indptr.data_ptr(),
        rows,
        num_q_heads,
        num_kv_heads,
        head_dim,
        page_size,
        pages_per_chunk,
        work_capacity,
        float(sm_scale),
        out.data_ptr(),
        out.stride(0),
        workspace.data_ptr(),
        workspace.numel() * workspace.element_size(),
        grid_ctas,
        _lib.stream_of(q.device),
    )
    return out


def predictor_attention(
    q: torch.Tensor,
    k_cache: torch.Tensor,
    v_cache: torch.Tensor,
    *,
    num_q_heads: int,
    num_kv_heads: int,
    head_dim: int,
    tokens_per_req: int,
    slot_stride: int,
    slot_base: int,
    sm_scale: float,
    out: torch.Tensor,
) -> torch.Tensor:
    _lib.call(
        "omni_predictor_attention",
        q.data_ptr(),
        q.stride(0),
        k_cache.data_ptr(),
        v_cache.data_ptr(),
        q.shape[0],
        num_q_heads,
        num_kv_heads,
        head_dim,
        tokens_per_req,
        slot_stride,
        slot_base,
        float(sm_scale),
        out.data_ptr(),
        out.stride(0),
        _lib.stream_of(q.device),
    )
    return out


def decode_prepare(
    *,
    seq_lens: torch.Tensor,
    req_pool_indices: torch.Tensor,
    req_to_token: torch.Tensor,
    page_size: int,
    free_pages: torch.Tensor,
    free_head: torch.Tensor,
    out_cache_loc: torch.Tensor,
    positions: torch.Tensor,
    page_indptr: torch.Tensor,
    page_indices: torch.Tensor,
    kv_indptr: torch.Tensor | None = None,
    kv_indices: torch.Tensor | None = None,
    work_indptr: torch.Tensor | None = None,
    pages_per_chunk: int = 8,
    status: torch.Tensor | None = None,
) -> None:
    _lib.call(
        "omni_decode_prepare",
        seq_lens.shape[0],
        seq_lens.data_ptr(),
        req_pool_indices.data_ptr(),
        req_to_token.data_ptr(),
        req_to_token.shape[1],
        page_size,
        free_pages.data_ptr(),
        free_pages.shape[0],
        free_head.data_ptr(),
        out_cache_loc.data_ptr(),
        positions.data_ptr(),
        _lib.ptr(kv_indptr),
        _lib.ptr(kv_indices),
        page_indptr.data_ptr(),
        page_indices.data_ptr(),
        _lib.ptr(work_indptr),
        pages_per_chunk,
        _lib.ptr(status),
        _lib.stream_of(seq_lens.device),
    )


def decode_rollback(
    *,
    seq_lens: torch.Tensor,
    req_pool_indices: torch.Tensor,
    req_to_token: torch.Tensor,
    page_size: int,
    out_cache_loc: torch.Tensor,
    free_head: torch.Tensor,
    freed_slots: torch.Tensor | None = None,
    num_freed: torch.Tensor | None = None,
) -> None:
    _lib.call(
        "omni_decode_rollback",
        seq_lens.shape[0],
        seq_lens.data_ptr(),
        req_pool_indices.data_ptr(),
        req_to_token.data_ptr(),
        req_to_token.shape[1],
        page_size,
        out_cache_loc.data_ptr(),
        free_head.data_ptr(),
        _lib.ptr(freed_slots),
        _lib.ptr(num_freed),
        _lib.stream_of(seq_lens.device),
    )


def rope_cos_sin_cache(max_position: int, head_dim: int, theta: float, device) -> torch.Tensor:
    """fp32 [max_position, head_dim]: cos of the half-dim frequencies, then sin
    (sglang RotaryEmbedding._compute_cos_sin_cache: inv_freq = theta^(-2i/d))."""
    inv_freq = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.float32) / head_dim))
    t = torch.arange(max_position, dtype=torch.float32)
    freqs = torch.outer(t, inv_freq)
    return torch.cat([freqs.cos(), freqs.sin()], dim=-1).contiguous().to(device)
