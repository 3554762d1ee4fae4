"""The dense Qwen3 talker decode forward on sm_100a.

Mirrors Qwen3TTSTalker.forward / Qwen3OmniTalker.forward at decode
(sglang_omni/models/qwen3_tts/sglang_model.py:1273-1302;
sglang_omni/models/qwen3_omni/components/talker.py:1259-1340): the decode
input row (feedback embedding + text embedding) through L decoder layers
(RMSNorm -> QKV -> q/k RMSNorm -> neox RoPE + paged KV store -> paged GQA decode
attention -> o_proj + residual -> RMSNorm -> SwiGLU MLP + residual), the final
RMSNorm and the codec head in fp32, then the layer-0 codec token draw
(sample_decode_tokens, talker.py:1376-1412).

Per layer the forward is 5 launches, all but the attention tcgen05 GEMMs with
fused epilogues: qkv (folded input RMSNorm + q/k RMSNorm + RoPE + KV store),
paged attention, o_proj (+residual, row sums of squares), gate_up (folded
post-attention RMSNorm + SwiGLU), down (+residual, row sums of squares).  With
cfg.moe the MLP is the sparse MoE block (omni_b200.moe.MoEBlock,
Qwen3OmniMoeTalkerSparseMoeBlock, talker.py:325-351).
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch

from omni_b200 import ops
from omni_b200.config import TalkerConfig
from omni_b200.kv_cache import PagedKVPool
from omni_b200.moe import MoEBlock, init_moe_weights
from omni_b200.sampling_kernels import layer0_sample


def init_talker_weights(cfg: TalkerConfig, *, seed: int, device, dtype=torch.bfloat16) -> dict:
    """Seeded random weights: linears and embeddings N(0, 0.02^2), norm gains 1 + N(0, 0.05^2)."""
    g = torch.Generator(device=device).manual_seed(seed)
    H, D = cfg.hidden_size, cfg.head_dim
    hq, hkv, I, V = cfg.num_attention_heads, cfg.num_key_value_heads, cfg.intermediate_size, cfg.vocab_size

    def lin(*shape):
        return (torch.randn(*shape, generator=g, device=device) * 0.02).to(dtype)

    def gain(n):
        return (1.0 + 0.05 * torch.randn(n, generator=g, device=device)).to(dtype)

    layers = []
    for _ in range(cfg.num_hidden_layers):
        layer = {
            "input_layernorm": gain(H),
            "qkv_proj": lin((hq + 2 * hkv) * D, H),
            "q_norm": gain(D),
            "k_norm": gain(D),
            "o_proj": lin(H, hq * D),
            "post_attention_layernorm": gain(H),
        }
        if cfg.moe is None:
            layer["gate_up_proj"] = lin(2 * I, H)
            layer["down_proj"] = lin(H, I)
        else:
            layer["moe"] = init_moe_weights(cfg.moe, H, generator=g, device=device)
        layers.append(layer)
    return {"layers": layers, "norm": gain(H), "codec_head": lin(V, H), "codec_embedding": lin(V, H)}


@dataclass
class ExtendForwardBatch:
    """Device tensors of the extend part of a mixed batch (ForwardBatch.init_new, extend mode)."""

    streams: int
    tokens: int                  # total extend rows
    qo_indptr: torch.Tensor      # i32 [streams + 1] (cu_seqlens)
    seq_lens: torch.Tensor       # i64 [streams] prefix + extend
    page_indptr: torch.Tensor    # i32 [streams + 1]
    page_indices: torch.Tensor   # i32
    tile_indptr: torch.Tensor    # i32 [streams + 1] query tiles of the prefill attention
    max_tiles: int


@dataclass
class DecodeForwardBatch:
    """Device tensors of one packed decode batch (ForwardBatch.init_new at decode)."""

    batch_size: int
    positions: torch.Tensor       # i64 [B]
    seq_lens: torch.Tensor        # i64 [B] (after this step's token)
    out_cache_loc: torch.Tensor   # i64 [B]
    req_pool_indices: torch.Tensor
    page_indptr: torch.Tensor     # i32 [B + 1]
    page_indices: torch.Tensor    # i32
    work_indptr: torch.Tensor     # i32 [B + 1]
    work_capacity: int
    pages_per_chunk: int


class DenseTalker:
    def __init__(self, cfg: TalkerConfig, weights: dict, *, max_batch: int, device, kv_pool: PagedKVPool,
                 expert_parallel: bool = False, max_rows: int = 0):
        self.cfg = cfg
        self.w = weights
        self.device = torch.device(device)
        self.max_batch = max_batch
        self.kv = kv_pool
        H, D = cfg.hidden_size, cfg.head_dim
        hq, hkv, I, V = cfg.num_attention_heads, cfg.num_key_value_heads, cfg.intermediate_size, cfg.vocab_size
        bf = dict(device=self.device, dtype=torch.bfloat16)
        B = max_batch
        # rows of one forward: the decode rows plus, in a mixed step, the extend rows
        R = max(max_rows, B)
        self.max_rows = R
        self.cos_sin = ops.rope_cos_sin_cache(cfg.max_context, D, cfg.rope_theta, self.device)
        self.h = torch.zeros(R, H, **bf)
        self.q = torch.zeros(R, hq * D, **bf)
        self.attn = torch.zeros(R, hq * D, **bf)
        self.act = torch.zeros(R, I, **bf)
        self.hidden = torch.zeros(B, H, **bf)
        # the rows that produce logits in a mixed step (decode rows + last extend row of each stream)
        self.h_sel = torch.zeros(B, H, **bf)
        self.logits = torch.zeros(B, V, dtype=torch.float32, device=self.device)
        self.sampled_token_ids = torch.zeros(B, dtype=torch.long, device=self.device)
        self.attn_workspace: torch.Tensor | None = None
        self.scale = 1.0 / math.sqrt(D)
        # layer-0 sampling state (talker.py:836-1010 buffers)
        f32 = dict(device=self.device, dtype=torch.float32)
        self.repetition_penalties = torch.ones(B, **f32)
        self.repetition_mask = torch.zeros(B, V, dtype=torch.uint8, device=self.device)
        self.suppress_mask = torch.zeros(B, V, dtype=torch.uint8, device=self.device)
        self.sampling_temperatures = torch.ones(B, **f32)
        self.sampling_top_ks = torch.full((B,), 50, dtype=torch.long, device=self.device)
        self.sampling_top_ps = torch.ones(B, **f32)
        self.sampling_min_ps = torch.zeros(B, **f32)
        self.sampling_seeds = torch.zeros(B, dtype=torch.long, device=self.device)
        self.max_top_k = 50
        # folded RMSNorms: each norm's gain is multiplied into the columns of the GEMM it feeds;
        # ss holds the per-row sums of squares of the residual stream (one part per 128 features)
        self.folded = [{"qkv": ops.fold_norm(lw["qkv_proj"], lw["input_layernorm"]),
                        "gate_up": (ops.fold_norm(lw["gate_up_proj"], lw["post_attention_layernorm"])
                                    if "gate_up_proj" in lw else None)}
                       for lw in self.w["layers"]]
        self.moe = None
        self.moe_local_w = None
        if cfg.moe is not None and expert_parallel:
            # experts sharded over the ranks of the default process group (moe_ep)
            from omni_b200.moe_ep import ExpertParallelMoE

            self.moe = ExpertParallelMoE(cfg.moe, H, max_tokens=B, device=self.device)
            self.moe_local_w = [self.moe.local_weights(lw["moe"]) for lw in self.w["layers"]]
        elif cfg.moe is not None:
            # sized for a mixed step's rows (decode rows + prompt tokens)
            self.moe = MoEBlock(cfg.moe, H, max_batch=R, device=self.device)
        self.codec_head_folded = ops.fold_norm(self.w["codec_head"], self.w["norm"])
        self.ss = torch.zeros(H // 128, R, dtype=torch.float32, device=self.device)
        self.ss_sel = torch.zeros(H // 128, B, dtype=torch.float32, device=self.device)
        self.qkv_raw = None  # raw qkv rows of a prompt-sized mixed step (allocated at the first one)

    def ensure_attention_workspace(self, work_capacity: int) -> None:
        need = ops.paged_attention_workspace_bytes(self.max_batch, self.cfg.num_key_value_heads, work_capacity)
        if self.attn_workspace is None or self.attn_workspace.numel() < need:
            self.attn_workspace = torch.zeros(need, dtype=torch.uint8, device=self.device)

    def forward(self, feedback: torch.Tensor, text: torch.Tensor | None, fb: DecodeForwardBatch) -> torch.Tensor:
        """Decode forward of B rows whose input is feedback (+ text); leaves the residual
        stream in self.h (its sums of squares in self.ss, for the final norm applied by the
        predictor's opening pass), fills self.logits (fp32) and returns them [B, V].

        Per layer 4 projections + attention: the qkv GEMM carries the input RMSNorm (folded),
        q/k RMSNorm, RoPE and the KV store; o_proj and down add the residual and emit the
        sums of squares the next folded norm needs."""
        cfg = self.cfg
        B = fb.batch_size
        H, D = cfg.hidden_size, cfg.head_dim
        hq, hkv = cfg.num_attention_heads, cfg.num_key_value_heads
        eps = cfg.rms_norm_eps
        h, q, attn, act = self.h[:B], self.q[:B], self.attn[:B], self.act[:B]
        ss = self.ss
        parts = H // 128
        self.ensure_attention_workspace(fb.work_capacity)
        ops.add_sumsq(feedback, text, h, ss[0])
        ss_parts = 1
        for li, lw in enumerate(self.w["layers"]):
            kc, vc = self.kv.k_buffer[li], self.kv.v_buffer[li]
            ops.linear_fused(h, self.folded[li]["qkv"], q, epilogue=ops.EPI_QKV_ROPE, ss_in=ss, ss_in_parts=ss_parts,
                             norm_eps=eps, qkv=dict(num_q_heads=hq, num_kv_heads=hkv, head_dim=D, q_norm=lw["q_norm"],
                                                    k_norm=lw["k_norm"], eps=eps, cos_sin=self.cos_sin,
                                                    positions=fb.positions, cache_loc=fb.out_cache_loc,
                                                    k_cache=kc, v_cache=vc))
            ops.paged_decode_attention(q, kc, vc, page_indptr=fb.page_indptr, page_indices=fb.page_indices,
                                       seq_lens=fb.seq_lens, work_indptr=fb.work_indptr, num_q_heads=hq,
                                       num_kv_heads=hkv, head_dim=D, page_size=cfg.page_size,
                                       pages_per_chunk=fb.pages_per_chunk, work_capacity=fb.work_capacity,
                                       sm_scale=self.scale, out=attn, workspace=self.attn_workspace)
            ops.linear_fused(attn, lw["o_proj"], h, epilogue=ops.EPI_RESIDUAL, residual=h, ss_out=ss)
            if "moe" in lw:
                mw = self.moe_local_w[li] if self.moe_local_w is not None else lw["moe"]
                self.moe.forward(h, ss, parts, lw["post_attention_layernorm"], eps, mw)
            else:
                ops.linear_fused(h, self.folded[li]["gate_up"], act, epilogue=ops.EPI_SWIGLU, ss_in=ss,
                                 ss_in_parts=parts, norm_eps=eps)
                ops.linear_fused(act, lw["down_proj"], h, epilogue=ops.EPI_RESIDUAL, residual=h, ss_out=ss)
            ss_parts = parts
        logits = self.logits[:B]
        ops.linear_fused(h, self.codec_head_folded, logits, epilogue=ops.EPI_F32, ss_in=ss, ss_in_parts=parts,
                         norm_eps=eps)
        return logits

    def forward_mixed(self, feedback: torch.Tensor, text: torch.Tensor | None, fb: DecodeForwardBatch,
                      prompt_embeds: torch.Tensor, ext: "ExtendForwardBatch", positions: torch.Tensor,
                      cache_loc: torch.Tensor, select: torch.Tensor) -> torch.Tensor:
        """One fused forward of a mixed batch: fb.batch_size decode rows (input feedback +
        text) followed by ext.tokens extend rows (input prompt_embeds, compose_prefill_embeds
        talker_model_runner.py:347-425), through every layer together; decode rows attend over
        their paged context, extend rows causally over their stream's pages (the extend forward
        writes their KV into the pool, talker.py:438-491 in extend mode).  positions /
        cache_loc cover all rows.  Logits of the rows in `select` (manual_extend_logits,
        talker.py:1344-1360: decode rows and each stream's last extend row) are returned."""
        cfg = self.cfg
        Bd, Te = fb.batch_size, ext.tokens
        R = Bd + Te
        H, D = cfg.hidden_size, cfg.head_dim
        hq, hkv = cfg.num_attention_heads, cfg.num_key_value_heads
        eps = cfg.rms_norm_eps
        h, q, attn, act = self.h[:R], self.q[:R], self.attn[:R], self.act[:R]
        ss = self.ss
        parts = H // 128
        if R > self.max_rows:
            raise RuntimeError("mixed batch exceeds the talker's row capacity")
        if self.moe is not None and self.moe_local_w is not None:
            raise NotImplementedError("mixed prefill + decode with expert-parallel MoE")
        self.ensure_attention_workspace(fb.work_capacity)
        if Bd > 0:
            ops.add_sumsq(feedback, text, h[:Bd], ss[0, :Bd])
        ops.add_sumsq(prompt_embeds, None, h[Bd:R], ss[0, Bd:R])
        ss_parts = 1
        # prompt-sized batches: the qkv projection as a plain GEMM (the tile-loop kernel)
        # into a raw buffer, then the q/k head norms, rotary and K/V store as their own
        # pass; the same values, rounded at the same points, as the fused qkv epilogue,
        # whose per-row work measured slower at these sizes
        split_qkv = R > 256
        if split_qkv and (self.qkv_raw is None or self.qkv_raw.shape[0] < R):
            self.qkv_raw = torch.empty(self.max_rows, (hq + 2 * hkv) * D, device=self.device, dtype=torch.bfloat16)
        for li, lw in enumerate(self.w["layers"]):
            kc, vc = self.kv.k_buffer[li], self.kv.v_buffer[li]
            if split_qkv:
                raw = self.qkv_raw[:R]
                ops.linear_fused(h, self.folded[li]["qkv"], raw, epilogue=ops.EPI_STORE, ss_in=ss,
                                 ss_in_parts=ss_parts, norm_eps=eps)
                ops.qknorm_rope_store(raw, num_q_heads=hq, num_kv_heads=hkv, head_dim=D, q_norm=lw["q_norm"],
                                      k_norm=lw["k_norm"], eps=eps, cos_sin=self.cos_sin, q_out=q, k_cache=kc,
                                      v_cache=vc, positions=positions[:R], cache_loc=cache_loc[:R])
            else:
                ops.linear_fused(h, self.folded[li]["qkv"], q, epilogue=ops.EPI_QKV_ROPE, ss_in=ss,
                                 ss_in_parts=ss_parts, norm_eps=eps,
                                 qkv=dict(num_q_heads=hq, num_kv_heads=hkv, head_dim=D, q_norm=lw["q_norm"],
                                          k_norm=lw["k_norm"], eps=eps, cos_sin=self.cos_sin,
                                          positions=positions[:R], cache_loc=cache_loc[:R], k_cache=kc, v_cache=vc))
            if Bd > 0:
                ops.paged_decode_attention(q[:Bd], kc, vc, page_indptr=fb.page_indptr, page_indices=fb.page_indices,
                                           seq_lens=fb.seq_lens, work_indptr=fb.work_indptr, num_q_heads=hq,
                                           num_kv_heads=hkv, head_dim=D, page_size=cfg.page_size,
                                           pages_per_chunk=fb.pages_per_chunk, work_capacity=fb.work_capacity,
                                           sm_scale=self.scale, out=attn[:Bd], workspace=self.attn_workspace)
            ops.prefill_attention(q[Bd:R], kc, vc, qo_indptr=ext.qo_indptr, seq_lens=ext.seq_lens,
                                  page_indptr=ext.page_indptr, page_indices=ext.page_indices,
                                  tile_indptr=ext.tile_indptr, max_tiles=ext.max_tiles, num_q_heads=hq,
                                  num_kv_heads=hkv, head_dim=D, page_size=cfg.page_size, sm_scale=self.scale,
                                  out=attn[Bd:R])
            ops.linear_fused(attn, lw["o_proj"], h, epilogue=ops.EPI_RESIDUAL, residual=h, ss_out=ss)
            if "moe" in lw:
                self.moe.forward(h, ss, parts, lw["post_attention_layernorm"], eps, lw["moe"])
            else:
                ops.linear_fused(h, self.folded[li]["gate_up"], act, epilogue=ops.EPI_SWIGLU, ss_in=ss,
                                 ss_in_parts=parts, norm_eps=eps)
                ops.linear_fused(act, lw["down_proj"], h, epilogue=ops.EPI_RESIDUAL, residual=h, ss_out=ss)
            ss_parts = parts
        n = select.shape[0]
        torch.index_select(h, 0, select, out=self.h_sel[:n])
        torch.index_select(ss[:, :R], 1, select, out=self.ss_sel[:, :n])
        logits = self.logits[:n]
        ops.linear_fused(self.h_sel[:n], self.codec_head_folded, logits, epilogue=ops.EPI_F32, ss_in=self.ss_sel,
                         ss_in_parts=parts, norm_eps=eps)
        return logits

    def sample_decode_tokens(self, logits: torch.Tensor, fb: DecodeForwardBatch) -> torch.Tensor:
        """Repetition penalty, suppression and the seeded layer-0 draw
        (sample_decode_tokens, talker.py:1376-1412); marks the drawn token in the
        repetition mask for the next step."""
        B = fb.batch_size
        out = self.sampled_token_ids[:B]
        layer0_sample(
            logits,
            penalties=self.repetition_penalties[:B],
            repetition_mask=self.repetition_mask[:B],
            suppress_mask=self.suppress_mask[:B],
            temperatures=self.sampling_temperatures[:B],
            top_ks=self.sampling_top_ks[:B],
            top_ps=self.sampling_top_ps[:B],
            min_ps=self.sampling_min_ps[:B],
            seeds=self.sampling_seeds[:B],
            positions=fb.positions,
            max_top_k=self.max_top_k,
            out=out,
            rep_mask_update=self.repetition_mask[:B],
        )
        return out
