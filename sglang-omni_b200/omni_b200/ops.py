"""Tensor-level wrappers of the C-ABI kernels used by the talker and predictor.

Each function launches on the current torch stream and raises on a contract
violation (there is no alternative path).  Workspaces are owned by the caller
and must be zero-filled once before first use.
"""

from __future__ import annotations

import ctypes

import torch

from omni_b200 import _lib

EPI_STORE = 0
EPI_RESIDUAL = 1
EPI_SWIGLU = 2
EPI_F32 = 3
EPI_QKV_ROPE = 4
EPI_ROUTER = 5


class OmniLinearArgs(ctypes.Structure):
    """Mirror of OmniLinearArgs in include/omni_b200.h (same field order and types)."""

    _fields_ = [
        ("x", ctypes.c_void_p), ("rows", ctypes.c_int64), ("k", ctypes.c_int64), ("x_stride", ctypes.c_int64),
        ("w", ctypes.c_void_p), ("n", ctypes.c_int64), ("epilogue", ctypes.c_int32), ("splits", ctypes.c_int32),
        ("ss_in", ctypes.c_void_p), ("ss_in_parts", ctypes.c_int32), ("ss_in_stride", ctypes.c_int64),
        ("norm_dim", ctypes.c_int32), ("norm_eps", ctypes.c_float), ("residual", ctypes.c_void_p),
        ("residual_stride", ctypes.c_int64), ("y", ctypes.c_void_p), ("y_stride", ctypes.c_int64),
        ("ss_out", ctypes.c_void_p), ("ss_out_stride", ctypes.c_int64), ("num_q_heads", ctypes.c_int32),
        ("num_kv_heads", ctypes.c_int32), ("head_dim", ctypes.c_int32), ("q_norm", ctypes.c_void_p),
        ("k_norm", ctypes.c_void_p), ("qk_eps", ctypes.c_float), ("cos_sin", ctypes.c_void_p),
        ("max_position", ctypes.c_int64), ("positions", ctypes.c_void_p), ("cache_loc", ctypes.c_void_p),
        ("tokens_per_req", ctypes.c_int32), ("slot_stride", ctypes.c_int32), ("slot_base", ctypes.c_int32),
        ("k_cache", ctypes.c_void_p), ("v_cache", ctypes.c_void_p),
        ("topk_ids", ctypes.c_void_p), ("topk_weights", ctypes.c_void_p), ("top_k", ctypes.c_int32),
        ("l2_prefetch", ctypes.c_void_p), ("l2_prefetch_bytes", ctypes.c_int64),
    ]


def linear_fused(
    x: torch.Tensor,
    w: torch.Tensor,
    out: torch.Tensor,
    *,
    epilogue: int,
    ss_in: torch.Tensor | None = None,
    ss_in_parts: int = 0,
    norm_eps: float = 1e-6,
    residual: torch.Tensor | None = None,
    ss_out: torch.Tensor | None = None,
    qkv: dict | None = None,
    router: dict | None = None,
    splits: int = 0,
    l2_prefetch: torch.Tensor | None = None,
) -> torch.Tensor:
    """out = epilogue(rstd * (x @ w.T)) with the RMSNorm folded into w (gain already
    multiplied into its columns) and rstd from ss_in [parts, rows_cap] sums of squares.
    ss_out [parts, rows_cap] receives the output's per-tile sums of squares.
    qkv: head geometry, norms, rotary table and caches for EPI_QKV_ROPE.
    router: {"topk_ids": i32 [rows, k], "topk_weights": f32 [rows, k]} for EPI_ROUTER
    (out receives the bf16 router logits).
    l2_prefetch: a tensor (the next projection's weight) that this launch's CTAs
    prefetch into L2 at their start."""
    a = OmniLinearArgs()
    a.x = x.data_ptr()
    a.rows, a.k = x.shape
    a.x_stride = x.stride(0)
    a.w = w.data_ptr()
    a.n = w.shape[0]
    a.epilogue = epilogue
    a.splits = splits
    if ss_in is not None:
        a.ss_in = ss_in.data_ptr()
        a.ss_in_parts = ss_in_parts
        a.ss_in_stride = ss_in.stride(0) if ss_in.ndim == 2 else ss_in.shape[0]
        a.norm_dim = x.shape[1]
        a.norm_eps = norm_eps
    if residual is not None:
        a.residual = residual.data_ptr()
        a.residual_stride = residual.stride(0)
    a.y = out.data_ptr()
    a.y_stride = out.stride(0)
    if ss_out is not None:
        a.ss_out = ss_out.data_ptr()
        a.ss_out_stride = ss_out.stride(0)
    if qkv is not None:
        a.num_q_heads = qkv["num_q_heads"]
        a.num_kv_heads = qkv["num_kv_heads"]
        a.head_dim = qkv["head_dim"]
        a.q_norm = qkv["q_norm"].data_ptr()
        a.k_norm = qkv["k_norm"].data_ptr()
        a.qk_eps = qkv.get("eps", 1e-6)
        a.cos_sin = qkv["cos_sin"].data_ptr()
        a.max_position = qkv["cos_sin"].shape[0]
        if qkv.get("positions") is not None:
            a.positions = qkv["positions"].data_ptr()
            a.cache_loc = qkv["cache_loc"].data_ptr()
        else:
            a.tokens_per_req = qkv["tokens_per_req"]
            a.slot_stride = qkv["slot_stride"]
            a.slot_base = qkv["slot_base"]
        a.k_cache = qkv["k_cache"].data_ptr()
        a.v_cache = qkv["v_cache"].data_ptr()
    if router is not None:
        a.topk_ids = router["topk_ids"].data_ptr()
        a.topk_weights = router["topk_weights"].data_ptr()
        a.top_k = router["topk_ids"].shape[1]
    if l2_prefetch is not None:
        a.l2_prefetch = l2_prefetch.data_ptr()
        a.l2_prefetch_bytes = l2_prefetch.numel() * l2_prefetch.element_size()
    _lib.call("omni_linear_fused", ctypes.addressof(a), _lib.stream_of(x.device))
    return out


def add_sumsq(a: torch.Tensor, b: torch.Tensor | None, out: torch.Tensor, ss_out: torch.Tensor) -> torch.Tensor:
    """out = bf16(a + b) (or a copy of a); ss_out[r] = sum of squares of out[r]."""
    _lib.call("omni_add_sumsq", a.data_ptr(), a.stride(0), _lib.ptr(b), 0 if b is None else b.stride(0),
              out.data_ptr(), out.stride(0), ss_out.data_ptr(), a.shape[0], a.shape[1], _lib.stream_of(a.device))
    return out


def fold_norm(weight: torch.Tensor, gain: torch.Tensor) -> torch.Tensor:
    """W * diag(gain) rounded to bf16: the weight of a GEMM whose input RMSNorm is folded."""
    return (weight.float() * gain.float()[None, :]).to(torch.bfloat16).contiguous()


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


class RowTensors:
    """Descriptor table of per-row state tensors (row = first dimension) for
    move_rows; built once, the tensors stay at fixed addresses."""

    def __init__(self, tensors: list[torch.Tensor]):
        import ctypes

        if len(tensors) > 24:
            raise ValueError("move_rows takes at most 24 tensors")
        for t in tensors:
            if t.dim() < 1 or not t.is_contiguous():
                raise ValueError("per-row state tensors must be contiguous with rows first")
        self.tensors = list(tensors)
        n = len(tensors)
        self.bases = (ctypes.c_void_p * n)(*[t.data_ptr() for t in tensors])
        self.row_bytes = (ctypes.c_int64 * n)(*[t[0].numel() * t.element_size() for t in tensors])
        self.strides = (ctypes.c_int64 * n)(*[t.stride(0) * t.element_size() for t in tensors])
        self.device = tensors[0].device


def move_rows(table: RowTensors, src, dst) -> None:
    """Row dst[m] of every tensor of the table becomes a copy of row src[m]
    (batch compaction); src and dst are host int32 arrays of disjoint rows."""
    import numpy as np

    src = np.ascontiguousarray(src, dtype=np.int32)
    dst = np.ascontiguousarray(dst, dtype=np.int32)
    if src.shape != dst.shape:
        raise ValueError("src and dst differ in length")
    if src.size == 0:
        return
    rows = min(t.shape[0] for t in table.tensors)
    if int(max(src.max(), dst.max())) >= rows or int(min(src.min(), dst.min())) < 0:
        raise ValueError("row index outside the per-row tensors")
    if set(src.tolist()) & set(dst.tolist()):
        raise ValueError("move sources and destinations overlap")
    _lib.call("omni_move_rows", table.bases, table.row_bytes, table.strides, len(table.tensors), src.ctypes.data,
              dst.ctypes.data, src.shape[0], _lib.stream_of(table.device))


def admit_streams(*, rows: torch.Tensor, slots: torch.Tensor, prompt_lens: torch.Tensor, page_indptr: torch.Tensor,
                  pages: torch.Tensor, req_to_token: torch.Tensor, page_size: int, seq_lens: torch.Tensor,
                  req_pool_indices: torch.Tensor, status: torch.Tensor | None = None) -> None:
    """req_to_token rows of newly admitted streams from their page lists, and their
    batch rows' seq_len and request slot (see include/omni_b200.h)."""
    n = rows.shape[0]
    _lib.call("omni_admit_streams", n, rows.data_ptr(), slots.data_ptr(), prompt_lens.data_ptr(),
              page_indptr.data_ptr(), pages.data_ptr(), req_to_token.data_ptr(), req_to_token.shape[1], page_size,
              seq_lens.data_ptr(), req_pool_indices.data_ptr(), _lib.ptr(status), _lib.stream_of(rows.device))


def rope_cos_sin_cache(max_position: int, head_dim: int, theta: float, device) -> torch.Tensor:
    """fp32 [max_position, head_dim]: cos of the half-dim frequencies, then sin
    (sglang RotaryEmbedding._compute_cos_sin_cache: inv_freq = theta^(-2i/d))."""
    inv_freq = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.float32) / head_dim))
    t = torch.arange(max_position, dtype=torch.float32)
    freqs = torch.outer(t, inv_freq)
    return torch.cat([freqs.cos(), freqs.sin()], dim=-1).contiguous().to(device)


# ---------------------------------------------------------------------------
# MoE block (block-FP8 experts)
# ---------------------------------------------------------------------------
def moe_rmsnorm_quant(h: torch.Tensor, ss: torch.Tensor, ss_parts: int, gain: torch.Tensor, eps: float,
                      x: torch.Tensor, xq: torch.Tensor, xs: torch.Tensor) -> None:
    """x = RMSNorm(h) (bf16) with rstd from ss [parts, rows_cap]; xq/xs its per-row
    128-group e4m3 codes (uint8) and f32 scales."""
    rows, hidden = h.shape
    _lib.call("omni_moe_rmsnorm_quant", h.data_ptr(), h.stride(0), ss.data_ptr(), ss_parts, ss.stride(0),
              gain.data_ptr(), eps, rows, hidden, x.data_ptr(), x.stride(0), xq.data_ptr(), xs.data_ptr(),
              _lib.stream_of(h.device))


def moe_chunk_capacity(tokens: int, top_k: int, experts: int) -> int:
    return int(_lib.load().omni_moe_chunk_capacity(tokens, top_k, experts))


def moe_align_gather(topk_ids: torch.Tensor, experts: int, xq: torch.Tensor, xs: torch.Tensor,
                     permuted_q: torch.Tensor, permuted_s: torch.Tensor, slot_of: torch.Tensor,
                     expert_offsets: torch.Tensor, chunks: torch.Tensor, n_chunks: torch.Tensor) -> None:
    tokens, top_k = topk_ids.shape
    _lib.call("omni_moe_align_gather", topk_ids.data_ptr(), tokens, top_k, experts, xq.data_ptr(), xs.data_ptr(),
              xq.shape[1], permuted_q.data_ptr(), permuted_s.data_ptr(), slot_of.data_ptr(),
              expert_offsets.data_ptr(), chunks.data_ptr(), chunks.shape[0], n_chunks.data_ptr(),
              _lib.stream_of(topk_ids.device))


def moe_gate_up_fp8(permuted_q: torch.Tensor, permuted_s: torch.Tensor, w13: torch.Tensor, w13_scale: torch.Tensor,
                    chunks: torch.Tensor, n_chunks: torch.Tensor, act_q: torch.Tensor, act_s: torch.Tensor) -> None:
    experts, two_i, hidden = w13.shape
    _lib.call("omni_moe_gate_up_fp8", permuted_q.data_ptr(), permuted_s.data_ptr(), permuted_q.shape[0], hidden,
              w13.data_ptr(), w13_scale.data_ptr(), experts, two_i // 2, chunks.data_ptr(), n_chunks.data_ptr(),
              act_q.data_ptr(), act_s.data_ptr(), _lib.stream_of(w13.device))


def moe_down_fp8(act_q: torch.Tensor, act_s: torch.Tensor, w2: torch.Tensor, w2_scale: torch.Tensor,
                 chunks: torch.Tensor, n_chunks: torch.Tensor, y: torch.Tensor) -> None:
    experts, hidden, inter = w2.shape
    _lib.call("omni_moe_down_fp8", act_q.data_ptr(), act_s.data_ptr(), act_q.shape[0], inter, w2.data_ptr(),
              w2_scale.data_ptr(), experts, hidden, chunks.data_ptr(), n_chunks.data_ptr(), y.data_ptr(),
              y.stride(0), _lib.stream_of(w2.device))


def moe_combine(y: torch.Tensor, slot_of: torch.Tensor, topk_weights: torch.Tensor, x: torch.Tensor,
                shared_gate_weight: torch.Tensor, shared_out: torch.Tensor, h: torch.Tensor,
                ss_out: torch.Tensor | None) -> None:
    rows, hidden = h.shape
    _lib.call("omni_moe_combine", y.data_ptr(), y.stride(0), slot_of.data_ptr(), topk_weights.data_ptr(),
              slot_of.shape[1], x.data_ptr(), x.stride(0), shared_gate_weight.data_ptr(), shared_out.data_ptr(),
              shared_out.stride(0), h.data_ptr(), h.stride(0), _lib.ptr(ss_out),
              0 if ss_out is None else ss_out.stride(0), rows, hidden, _lib.stream_of(h.device))


def moe_align_gather_strided(topk_ids: torch.Tensor, tokens: int, top_k: int, experts: int, xq: torch.Tensor,
                             xq_stride: int, xs: torch.Tensor, xs_stride: int, hidden: int,
                             permuted_q: torch.Tensor, permuted_s: torch.Tensor, slot_of: torch.Tensor,
                             expert_offsets: torch.Tensor, chunks: torch.Tensor, n_chunks: torch.Tensor,
                             ids_stride: int) -> None:
    """moe_align_gather over strided rows (ids_stride int32s, xq_stride bytes, xs_stride floats);
    expert id -1 = no local expert for that entry."""
    _lib.call("omni_moe_align_gather_strided", topk_ids.data_ptr(), ids_stride, tokens, top_k, experts,
              xq.data_ptr(), xq_stride, xs.data_ptr(), xs_stride, hidden, permuted_q.data_ptr(),
              permuted_s.data_ptr(), slot_of.data_ptr(), expert_offsets.data_ptr(), chunks.data_ptr(),
              chunks.shape[0], n_chunks.data_ptr(), _lib.stream_of(permuted_q.device))


def moe_partial_sum(y: torch.Tensor, slot_of: torch.Tensor, weights: torch.Tensor, weights_stride: int,
                    out: torch.Tensor) -> None:
    rows, top_k = slot_of.shape
    _lib.call("omni_moe_partial_sum", y.data_ptr(), y.stride(0), slot_of.data_ptr(), weights.data_ptr(),
              weights_stride, top_k, rows, out.shape[1], out.data_ptr(), out.stride(0), _lib.stream_of(y.device))


def moe_combine_parts(parts: torch.Tensor, part_index: torch.Tensor, x: torch.Tensor,
                      shared_gate_weight: torch.Tensor, shared_out: torch.Tensor, h: torch.Tensor,
                      ss_out: torch.Tensor | None) -> None:
    rows, hidden = h.shape
    _lib.call("omni_moe_combine_parts", parts.data_ptr(), parts.stride(0), part_index.data_ptr(),
              part_index.shape[1], x.data_ptr(), x.stride(0), shared_gate_weight.data_ptr(), shared_out.data_ptr(),
              shared_out.stride(0), h.data_ptr(), h.stride(0), _lib.ptr(ss_out),
              0 if ss_out is None else ss_out.stride(0), rows, hidden, _lib.stream_of(h.device))


PREFILL_Q_TILE = 128


def extend_prepare(*, prefix_lens, extend_lens, req_pool_indices, req_to_token, page_size, seq_lens, qo_indptr,
                   out_cache_loc, positions, page_indptr, page_indices, tile_indptr=None, status=None) -> None:
    """Packing of an extend batch whose slots are reserved in req_to_token (see include/omni_b200.h)."""
    rows = prefix_lens.shape[0]
    _lib.call("omni_extend_prepare", rows, prefix_lens.data_ptr(), extend_lens.data_ptr(),
              req_pool_indices.data_ptr(), req_to_token.data_ptr(), req_to_token.shape[1], page_size,
              seq_lens.data_ptr(), qo_indptr.data_ptr(), out_cache_loc.data_ptr(), positions.data_ptr(),
              page_indptr.data_ptr(), page_indices.data_ptr(), _lib.ptr(tile_indptr), PREFILL_Q_TILE,
              _lib.ptr(status), _lib.stream_of(prefix_lens.device))


def prefill_attention(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, *, qo_indptr, seq_lens,
                      page_indptr, page_indices, tile_indptr, max_tiles: int, num_q_heads: int, num_kv_heads: int,
                      head_dim: int, page_size: int, sm_scale: float, out: torch.Tensor) -> torch.Tensor:
    """Causal extend attention over the paged pool; q/out rows are the extend rows (cu_seqlens qo_indptr)."""
    _lib.call("omni_prefill_attention", q.data_ptr(), q.stride(0), q.shape[0], k_cache.data_ptr(),
              v_cache.data_ptr(), k_cache.shape[0], qo_indptr.data_ptr(), seq_lens.data_ptr(),
              page_indptr.data_ptr(), page_indices.data_ptr(),
              tile_indptr.data_ptr(), qo_indptr.shape[0] - 1, max_tiles, num_q_heads, num_kv_heads, head_dim,
              page_size, sm_scale, out.data_ptr(), out.stride(0), _lib.stream_of(q.device))
    return out


def conv1d_gemm(padded: torch.Tensor, weight_mat: torch.Tensor, *, taps: int, dilation: int, length: int,
                out: torch.Tensor, bias: torch.Tensor | None = None, alpha_scale: torch.Tensor | None = None,
                inverse_beta: torch.Tensor | None = None, residual: torch.Tensor | None = None,
                sum_out: torch.Tensor | None = None) -> torch.Tensor:
    """Implicit-GEMM causal conv (omni_conv1d_gemm): padded [rows, positions, C_in] bf16 contiguous,
    weight_mat [C_out, taps * C_in], out [rows, length, C_out] (row stride may exceed
    length * C_out, as a padded buffer's body).  With alpha_scale: SnakeBeta(conv + bias
    [+ residual]) fused, the sum to sum_out."""
    rows, positions, cin = padded.shape
    cout = weight_mat.shape[0]
    if not padded.is_contiguous() or not weight_mat.is_contiguous() or weight_mat.shape[1] != taps * cin:
        raise ValueError("conv1d_gemm needs a contiguous padded input and a [C_out, taps * C_in] weight")
    if out.shape[-1] != cout or out.stride(-1) != 1 or (out.ndim == 3 and out.stride(1) != cout):
        raise ValueError("conv1d_gemm output rows are [length, C_out] channels last")
    _lib.call("omni_conv1d_gemm", padded.data_ptr(), rows, positions, cin, weight_mat.data_ptr(), cout, taps,
              dilation, length, out.data_ptr(), out.stride(0), _lib.ptr(bias), _lib.ptr(residual),
              _lib.ptr(sum_out), _lib.ptr(alpha_scale), _lib.ptr(inverse_beta), _lib.stream_of(padded.device))
    return out

