"""CPU restatement of the expert-parallel dispatch packing — TEST INFRASTRUCTURE ONLY.

Torch-on-CPU statement of what omni_moe_ep_pack (sglang-omni_b200/csrc/moe.cu) builds:
the destination ranks of every token (rank d holds experts [d e, (d + 1) e)), each
token's row in its destination blocks (token order), the packed rows (e4m3 codes,
group scales, the k ids local to the rank or -1, the k routing weights) and the
index of the partial each token gets back.  Used by the gloo plumbing test and as
the bit-exact reference of the kernel.
"""

from __future__ import annotations

import torch


def dispatch_plan(topk_ids: torch.Tensor, world: int, experts_per_rank: int, cap: int):
    """For tokens' global expert ids [T, k]: has[t, d] (token t goes to rank d), pos[t, d]
    (its row in block d), flat[t, d] (row in the send buffer; world*cap = discarded) and
    local_ids[t, d, k] (expert id on rank d, or -1)."""
    T = topk_ids.shape[0]
    dev = topk_ids.device
    ranks = torch.arange(world, device=dev)
    dest = torch.div(topk_ids.long(), experts_per_rank, rounding_mode="floor")  # [T, k]
    onehot = dest.unsqueeze(-1) == ranks  # [T, k, W]
    has = onehot.any(1)  # [T, W]
    pos = torch.cumsum(has.to(torch.int32), 0) - 1  # [T, W]
    flat = torch.where(has, ranks * cap + pos, torch.full_like(pos, world * cap))
    local = topk_ids.long().unsqueeze(1) - (ranks * experts_per_rank).view(1, world, 1)  # [T, W, k]
    local_ids = torch.where(onehot.permute(0, 2, 1), local, torch.full_like(local, -1)).to(torch.int32)
    del T
    return has, pos, flat, local_ids


def pack_rows(send: torch.Tensor, hidden: int, top_k: int, xq: torch.Tensor, xs: torch.Tensor,
              local_ids: torch.Tensor, weights: torch.Tensor, flat: torch.Tensor) -> None:
    """Writes the dispatched rows into send [world*cap + 1, row_bytes] (uint8; the last row
    takes the writes of tokens that skip a rank); rows no token lands in carry expert ids -1."""
    T, W = flat.shape
    G = hidden // 128
    idx = flat.reshape(-1)
    q = send[:, :hidden]
    s = send[:, hidden: hidden + 4 * G].view(torch.float32)
    ids = send[:, hidden + 4 * G: hidden + 4 * G + 4 * top_k].view(torch.int32)
    w = send[:, hidden + 4 * G + 4 * top_k: hidden + 4 * G + 8 * top_k].view(torch.float32)
    ids.fill_(-1)
    q.index_copy_(0, idx, xq.unsqueeze(1).expand(T, W, hidden).reshape(T * W, hidden))
    s.index_copy_(0, idx, xs.unsqueeze(1).expand(T, W, G).reshape(T * W, G))
    ids.index_copy_(0, idx, local_ids.reshape(T * W, top_k))
    w.index_copy_(0, idx, weights.unsqueeze(1).expand(T, W, top_k).reshape(T * W, top_k))


def part_index(has: torch.Tensor, pos: torch.Tensor, cap: int) -> torch.Tensor:
    """Row of the returned partial of token t from rank d (or -1), [T, W] int32."""
    W = has.shape[1]
    ranks = torch.arange(W, device=has.device)
    return torch.where(has, ranks * cap + pos, torch.full_like(pos, -1)).to(torch.int32).contiguous()
