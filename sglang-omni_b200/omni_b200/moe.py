"""The talker's sparse MoE block with block-FP8 experts on sm_100a.

Mirrors Qwen3OmniMoeTalkerSparseMoeBlock.forward
(sglang_omni/models/qwen3_omni/components/talker.py:325-351) over
Qwen3OmniMoeThinkerTextSparseMoeBlock (thinker_model.py:405-470): the
post-attention RMSNorm output x feeds the router gate (bf16 logits, softmax,
top-k, renormalised: TopK with renormalize=norm_topk_prob), the routed
FusedMoE experts (e4m3 weights with per-128x128 block scales, activations
quantised per token per 128-group: quantization.py:124-167) and the shared
expert gated by sigmoid(shared_expert_gate(x)); the block output is added to
the residual stream.

Per layer: rmsnorm_quant, router GEMM (fused top-k), align/gather, gate/up and
down grouped FP8 GEMMs, the shared expert's two bf16 GEMMs, and the combine
(routed sum + gated shared + residual add + sums of squares for the next norm).
"""

from __future__ import annotations

import torch

from omni_b200 import ops
from omni_b200.config import MoEConfig

FP8_MAX = 448.0


def quantize_block_fp8(w: torch.Tensor, block: int = 128) -> tuple[torch.Tensor, torch.Tensor]:
    """Block quantisation of expert weights [E, R, C] (R, C multiples of block):
    scale = max(amax(block), 1e-10) / 448, q = e4m3(w / scale).  Returns the codes as
    uint8 [E, R, C] and the scales f32 [E, R / block, C / block]."""
    e, r, c = w.shape
    wb = w.float().reshape(e, r // block, block, c // block, block)
    amax = wb.abs().amax(dim=(2, 4)).clamp_min(1e-10)
    scale = amax / FP8_MAX
    q = (wb / scale[:, :, None, :, None]).clamp(-FP8_MAX, FP8_MAX).to(torch.float8_e4m3fn)
    return q.reshape(e, r, c).view(torch.uint8).contiguous(), scale.contiguous()


def dequantize_block_fp8(q: torch.Tensor, scale: torch.Tensor, block: int = 128) -> torch.Tensor:
    e, r, c = q.shape
    v = q.view(torch.float8_e4m3fn).float().reshape(e, r // block, block, c // block, block)
    return (v * scale[:, :, None, :, None]).reshape(e, r, c)


def init_moe_weights(cfg: MoEConfig, hidden: int, *, generator: torch.Generator, device) -> dict:
    """Seeded random MoE layer: router gate and shared expert bf16 N(0, 0.02^2); expert
    weights N(0, 0.02^2) quantised to e4m3 with per-128x128 block scales."""
    E, I, Is = cfg.num_experts, cfg.moe_intermediate_size, cfg.shared_expert_intermediate_size

    def lin(*shape):
        return (torch.randn(*shape, generator=generator, device=device) * 0.02).to(torch.bfloat16)

    w13 = torch.randn(E, 2 * I, hidden, generator=generator, device=device) * 0.02
    w2 = torch.randn(E, hidden, I, generator=generator, device=device) * 0.02
    w13_q, w13_s = quantize_block_fp8(w13, cfg.fp8_block)
    w2_q, w2_s = quantize_block_fp8(w2, cfg.fp8_block)
    return {
        "gate": lin(E, hidden),
        "w13": w13_q, "w13_scale": w13_s, "w2": w2_q, "w2_scale": w2_s,
        "shared_gate_up": lin(2 * Is, hidden), "shared_down": lin(hidden, Is),
        "shared_expert_gate": lin(1, hidden),
    }


MAX_ALIGN_TOKENS = 4096  # omni_moe_align_gather's token limit


class MoEBlock:
    """Fixed-address buffers for one talker's MoE layers (shared across layers)."""

    def __init__(self, cfg: MoEConfig, hidden: int, *, max_batch: int, device):
        if cfg.fp8_block != 128:
            raise ValueError("the block-FP8 kernels use 128 x 128 weight blocks")
        self.cfg = cfg
        self.hidden = hidden
        self.device = torch.device(device)
        B, H, E, k = max_batch, hidden, cfg.num_experts, cfg.num_experts_per_tok
        I, Is = cfg.moe_intermediate_size, cfg.shared_expert_intermediate_size
        dev = self.device
        bf = dict(device=dev, dtype=torch.bfloat16)
        self.max_batch = B
        # the align/gather kernel takes at most MAX_ALIGN_TOKENS tokens: larger batches
        # (the prompt rows of a mixed step) run through the block in chunks of rows
        B = min(B, MAX_ALIGN_TOKENS)
        self.chunk_rows = B
        self.rows_cap = B * k + 64  # the last 64-row activation box stays inside the buffer
        self.x = torch.zeros(B, H, **bf)
        self.xq = torch.zeros(B, H, dtype=torch.uint8, device=dev)
        self.xs = torch.zeros(B, H // 128, dtype=torch.float32, device=dev)
        self.router_logits = torch.zeros(B, E, **bf)
        self.topk_ids = torch.zeros(B, k, dtype=torch.int32, device=dev)
        self.topk_weights = torch.zeros(B, k, dtype=torch.float32, device=dev)
        self.permuted_q = torch.zeros(self.rows_cap, H, dtype=torch.uint8, device=dev)
        self.permuted_s = torch.zeros(self.rows_cap, H // 128, dtype=torch.float32, device=dev)
        self.slot_of = torch.zeros(B, k, dtype=torch.int32, device=dev)
        self.expert_offsets = torch.zeros(E + 1, dtype=torch.int32, device=dev)
        self.chunks = torch.zeros(ops.moe_chunk_capacity(B, k, E), 4, dtype=torch.int32, device=dev)
        self.n_chunks = torch.zeros(1, dtype=torch.int32, device=dev)
        self.act_q = torch.zeros(self.rows_cap, I, dtype=torch.uint8, device=dev)
        self.act_s = torch.zeros(self.rows_cap, I // 128, dtype=torch.float32, device=dev)
        self.y = torch.zeros(self.rows_cap, H, **bf)
        self.shared_act = torch.zeros(B, Is, **bf)
        self.shared_out = torch.zeros(B, H, **bf)

    def forward(self, h: torch.Tensor, ss: torch.Tensor, ss_parts: int, gain: torch.Tensor, eps: float,
                w: dict) -> None:
        """h [B, H] += MoE(RMSNorm(h)) in place; ss [H/128, B_cap] receives the new rows'
        per-128-feature sums of squares.  ss holds h's sums of squares on entry.  Rows are
        independent: more than chunk_rows rows go through in chunks."""
        B = h.shape[0]
        if B > self.max_batch:
            raise RuntimeError("MoE block: more rows than its capacity")
        for c in range(0, B, self.chunk_rows):
            n = min(self.chunk_rows, B - c)
            self._forward_rows(h[c:c + n], ss[:, c:c + n], ss_parts, gain, eps, w)

    def _forward_rows(self, h: torch.Tensor, ss: torch.Tensor, ss_parts: int, gain: torch.Tensor, eps: float,
                      w: dict) -> None:
        B = h.shape[0]
        x, xq, xs = self.x[:B], self.xq[:B], self.xs[:B]
        ids, tw = self.topk_ids[:B], self.topk_weights[:B]
        ops.moe_rmsnorm_quant(h, ss, ss_parts, gain, eps, x, xq, xs)
        ops.linear_fused(x, w["gate"], self.router_logits[:B], epilogue=ops.EPI_ROUTER,
                         router={"topk_ids": ids, "topk_weights": tw})
        ops.moe_align_gather(ids, self.cfg.num_experts, xq, xs, self.permuted_q, self.permuted_s, self.slot_of[:B],
                             self.expert_offsets, self.chunks, self.n_chunks)
        ops.moe_gate_up_fp8(self.permuted_q, self.permuted_s, w["w13"], w["w13_scale"], self.chunks, self.n_chunks,
                            self.act_q, self.act_s)
        ops.moe_down_fp8(self.act_q, self.act_s, w["w2"], w["w2_scale"], self.chunks, self.n_chunks, self.y)
        ops.linear_fused(x, w["shared_gate_up"], self.shared_act[:B], epilogue=ops.EPI_SWIGLU)
        ops.linear_fused(self.shared_act[:B], w["shared_down"], self.shared_out[:B], epilogue=ops.EPI_STORE)
        ops.moe_combine(self.y, self.slot_of[:B], tw, x, w["shared_expert_gate"], self.shared_out[:B], h, ss)
