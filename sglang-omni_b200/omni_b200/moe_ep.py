"""Expert-parallel variant of the talker's MoE block across the GPUs of one node.

Each of the W ranks holds E / W experts (rank d: experts [d E/W, (d+1) E/W)) and
routes its own tokens with the replicated router.  Per layer:

  dispatch  every token goes once to each rank that holds at least one of its
            top-k experts: its e4m3 row, group scales, the k expert ids local to
            that rank (-1 for the others) and the k routing weights travel as one
            packed row; each rank sends a fixed block of `cap` rows to every peer
            (unused rows carry no expert), one NCCL all-to-all over NVLink
  compute   the received rows go through the same align/gather and grouped FP8
            GEMMs as the single-GPU block, over the local experts only, and each
            received row's partial routed sum (its local experts, k order) is
            formed in bf16
  combine   the partial rows return by a second all-to-all; each token sums its
            partials in rank order, then adds the gated shared expert (computed
            locally, on a side stream that runs while the two all-to-alls and the
            local experts run) and the residual, as the single-GPU combine does

The send buffer, with each row's place in its destination block and the index of
the partial each token gets back, is built by one kernel (omni_moe_ep_pack).
Fixed-size blocks of `cap` rows keep every collective's split sizes constant, so no
host synchronisation sits inside the layer and the layer stays inside the step's
CUDA graph: NCCL's all-to-all takes its split sizes on the host, so blocks sized
from a device-side count exchange would cost a device-to-host copy and a stream
synchronisation per MoE layer (20 a step).  A rank receives cap rows from every peer
whatever the routing; with top-8 routing over 128 experts a token reaches most
ranks of an 8-GPU node, so the blocks are mostly full at the config-4 batch.  The routed sum is rounded once per rank
(the partial rows are bf16), so results agree with the single-GPU block within
the bf16 tolerance, not bit for bit.
"""

from __future__ import annotations

import torch

from omni_b200 import _lib, ops
from omni_b200.config import MoEConfig
from omni_b200.moe import MoEBlock


def packed_row_bytes(hidden: int, top_k: int) -> int:
    """Bytes of one dispatched row: e4m3 codes, group scales, k local ids, k weights (16-aligned)."""
    b = hidden + 4 * (hidden // 128) + 8 * top_k
    return (b + 15) // 16 * 16


def ep_pack(send: torch.Tensor, hidden: int, top_k: int, topk_ids: torch.Tensor, topk_weights: torch.Tensor,
            xq: torch.Tensor, xs: torch.Tensor, world: int, experts_per_rank: int, cap: int,
            part_index: torch.Tensor) -> None:
    """The dispatch send buffer in one launch (omni_moe_ep_pack): each token's packed row
    in the block of every rank that holds one of its experts (rows in token order),
    unused rows with expert ids -1, and part_index [T, world] (the row of each returned
    partial, -1 for none)."""
    T = topk_ids.shape[0]
    _lib.call("omni_moe_ep_pack", topk_ids.data_ptr(), topk_weights.data_ptr(), T, top_k, xq.data_ptr(),
              xq.stride(0), xs.data_ptr(), xs.stride(0), hidden, world, experts_per_rank, cap, send.data_ptr(),
              send.stride(0), part_index.data_ptr(), _lib.stream_of(send.device))


class ExpertParallelMoE:
    """One rank's share of the expert-parallel MoE block (buffers shared by the layers)."""

    def __init__(self, cfg: MoEConfig, hidden: int, *, max_tokens: int, group=None, device=None):
        import torch.distributed as dist

        self.dist = dist
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if cfg.num_experts % self.world:
            raise ValueError("experts must divide evenly over the ranks")
        self.cfg = cfg
        self.hidden = hidden
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        self.cap = max_tokens
        self.e_local = cfg.num_experts // self.world
        k = cfg.num_experts_per_tok
        W, dev = self.world, self.device
        self.row_bytes = packed_row_bytes(hidden, k)
        # tokens of this rank: norm, codes, routing, shared expert (single-GPU block buffers)
        self.local = MoEBlock(cfg, hidden, max_batch=max_tokens, device=dev)
        self.side = torch.cuda.Stream(dev)  # the shared expert, overlapped with the all-to-alls
        self.send = torch.zeros(W * self.cap, self.row_bytes, dtype=torch.uint8, device=dev)
        self.part_index = torch.zeros(self.cap, W, dtype=torch.int32, device=dev)
        self.recv = torch.zeros(W * self.cap, self.row_bytes, dtype=torch.uint8, device=dev)
        n_recv = W * self.cap
        pairs_cap = n_recv * k + 64
        self.permuted_q = torch.zeros(pairs_cap, hidden, dtype=torch.uint8, device=dev)
        self.permuted_s = torch.zeros(pairs_cap, hidden // 128, dtype=torch.float32, device=dev)
        self.slot_of = torch.zeros(n_recv, k, dtype=torch.int32, device=dev)
        self.expert_offsets = torch.zeros(self.e_local + 1, dtype=torch.int32, device=dev)
        self.chunks = torch.zeros(ops.moe_chunk_capacity(n_recv, k, self.e_local), 4, dtype=torch.int32, device=dev)
        self.n_chunks = torch.zeros(1, dtype=torch.int32, device=dev)
        self.act_q = torch.zeros(pairs_cap, cfg.moe_intermediate_size, dtype=torch.uint8, device=dev)
        self.act_s = torch.zeros(pairs_cap, cfg.moe_intermediate_size // 128, dtype=torch.float32, device=dev)
        self.y = torch.zeros(pairs_cap, hidden, dtype=torch.bfloat16, device=dev)
        self.ret_send = torch.zeros(n_recv, hidden, dtype=torch.bfloat16, device=dev)
        self.ret_recv = torch.zeros(n_recv, hidden, dtype=torch.bfloat16, device=dev)

    def local_weights(self, w: dict) -> dict:
        """This rank's slice of a full layer's MoE weights (experts r E/W .. (r+1) E/W)."""
        e0, e1 = self.rank * self.e_local, (self.rank + 1) * self.e_local
        out = dict(w)
        for key in ("w13", "w13_scale", "w2", "w2_scale"):
            out[key] = w[key][e0:e1].contiguous()
        return out

    def forward(self, h: torch.Tensor, ss: torch.Tensor, ss_parts: int, gain: torch.Tensor, eps: float,
                w_local: dict) -> None:
        """h [T, H] += MoE(RMSNorm(h)) in place for this rank's T tokens (T <= max_tokens);
        w_local = local_weights(full layer weights).  Every rank calls it (collectives)."""
        cfg, H, k = self.cfg, self.hidden, self.cfg.num_experts_per_tok
        W, cap, G = self.world, self.cap, H // 128
        T = h.shape[0]
        m = self.local
        x, xq, xs = m.x[:T], m.xq[:T], m.xs[:T]
        ids, tw = m.topk_ids[:T], m.topk_weights[:T]
        ops.moe_rmsnorm_quant(h, ss, ss_parts, gain, eps, x, xq, xs)
        ops.linear_fused(x, w_local["gate"], m.router_logits[:T], epilogue=ops.EPI_ROUTER,
                         router={"topk_ids": ids, "topk_weights": tw})
        # the gated shared expert runs on a side stream while the routed tokens go out,
        # through the local experts and back: the two all-to-alls overlap it
        main = torch.cuda.current_stream(h.device)
        self.side.wait_stream(main)
        with torch.cuda.stream(self.side):
            ops.linear_fused(x, w_local["shared_gate_up"], m.shared_act[:T], epilogue=ops.EPI_SWIGLU)
            ops.linear_fused(m.shared_act[:T], w_local["shared_down"], m.shared_out[:T], epilogue=ops.EPI_STORE)
        pidx = self.part_index[:T]
        ep_pack(self.send, H, k, ids, tw, xq, xs, W, self.e_local, cap, pidx)
        self.dist.all_to_all_single(self.recv, self.send, group=self.group)
        rb = self.row_bytes
        ids_view = self.recv[:, H + 4 * G:].view(torch.int32)
        xs_view = self.recv[:, H:].view(torch.float32)
        w_view = self.recv[:, H + 4 * G + 4 * k:].view(torch.float32)
        n = W * cap
        ops.moe_align_gather_strided(ids_view, n, k, self.e_local, self.recv, rb, xs_view, rb // 4, H,
                                     self.permuted_q, self.permuted_s, self.slot_of, self.expert_offsets,
                                     self.chunks, self.n_chunks, ids_stride=rb // 4)
        ops.moe_gate_up_fp8(self.permuted_q, self.permuted_s, w_local["w13"], w_local["w13_scale"], self.chunks,
                            self.n_chunks, self.act_q, self.act_s)
        ops.moe_down_fp8(self.act_q, self.act_s, w_local["w2"], w_local["w2_scale"], self.chunks, self.n_chunks,
                         self.y)
        ops.moe_partial_sum(self.y, self.slot_of, w_view, rb // 4, self.ret_send)
        self.dist.all_to_all_single(self.ret_recv, self.ret_send, group=self.group)
        main.wait_stream(self.side)
        ops.moe_combine_parts(self.ret_recv, pidx, x, w_local["shared_expert_gate"], m.shared_out[:T], h, ss)
