"""The code predictor ("subtalker") of the Qwen3 talkers on sm_100a.

Mirrors Qwen3TTSCodePredictor / Qwen3TTSTalker.code_predictor_forward
(sglang_omni/models/qwen3_tts/sglang_model.py:447-490, 1317-1346, 1743-1879)
and the Qwen3-Omni greedy variant (talker.py:1633-1732): per frame, one
two-token pass [talker hidden, embedding of the layer-0 code] at cache slots
0 and 1, then for each residual codebook j: lm_head[j] -> sample (or argmax)
code j+1 -> gather its embedding (summed += it) -> a one-token pass at slot
j + 2.  Every launch goes to libomni_b200.so; all buffers are allocated once
for max_batch rows so the loop can be captured in a CUDA graph.
"""

from __future__ import annotations

import math

import torch

from omni_b200 import ops
from omni_b200.config import PredictorConfig
from omni_b200.sampling_kernels import fused_raw_logit_block_k, predictor_sample_step


def init_predictor_weights(cfg: PredictorConfig, *, seed: int, device, dtype=torch.bfloat16) -> dict:
    """Seeded random weights: linears N(0, 0.02^2), norm gains 1 + N(0, 0.05^2)."""
    g = torch.Generator(device=device).manual_seed(seed)
    H, D = cfg.hidden_size, cfg.head_dim
    hq, hkv, I, V = cfg.num_attention_heads, cfg.num_key_value_heads, cfg.intermediate_size, cfg.vocab_size

    def lin(*shape):
        return (torch.randn(*shape, generator=g, device=device) * 0.02).to(dtype)

    def gain(n):
        return (1.0 + 0.05 * torch.randn(n, generator=g, device=device)).to(dtype)

    layers = []
    for _ in range(cfg.num_hidden_layers):
        layers.append({
            "input_layernorm": gain(H),
            "qkv_proj": lin((hq + 2 * hkv) * D, H),
            "q_norm": gain(D),
            "k_norm": gain(D),
            "o_proj": lin(H, hq * D),
            "post_attention_layernorm": gain(H),
            "gate_up_proj": lin(2 * I, H),
            "down_proj": lin(H, I),
        })
    G = cfg.num_code_groups
    return {
        "layers": layers,
        "norm": gain(H),
        "lm_head": lin(G - 1, V, H),
        "codec_embedding": lin(G - 1, V, H),
    }


class CodePredictor:
    """Predictor stack + residual-codebook loop with persistent buffers."""

    def __init__(self, cfg: PredictorConfig, weights: dict, *, max_batch: int, device, layer0_embedding: torch.Tensor):
        self.cfg = cfg
        self.w = weights
        self.device = torch.device(device)
        self.max_batch = max_batch
        self.layer0_embedding = layer0_embedding  # the talker's codec embedding [V0, H]
        H, D = cfg.hidden_size, cfg.head_dim
        hq, hkv, I = cfg.num_attention_heads, cfg.num_key_value_heads, cfg.intermediate_size
        G, S = cfg.num_code_groups, cfg.cache_len
        R = 2 * max_batch
        bf = dict(device=self.device, dtype=torch.bfloat16)
        self.cos_sin = ops.rope_cos_sin_cache(S, D, cfg.rope_theta, self.device)
        L = cfg.num_hidden_layers
        self.k_cache = torch.zeros(L, max_batch * S, hkv, D, **bf)
        self.v_cache = torch.zeros(L, max_batch * S, hkv, D, **bf)
        self.pair = torch.zeros(R, H, **bf)
        self.h = torch.zeros(R, H, **bf)
        self.normed = torch.zeros(R, H, **bf)
        self.qkv = torch.zeros(R, (hq + 2 * hkv) * D, **bf)
        self.q = torch.zeros(R, hq * D, **bf)
        self.attn = torch.zeros(R, hq * D, **bf)
        self.act = torch.zeros(R, I, **bf)
        self.out = torch.zeros(R, H, **bf)
        self.next_in = torch.zeros(max_batch, H, **bf)
        # lm_head logits of codebook j; codebook 0 is computed on all 2B rows of the
        # opening pair pass and read at the odd (layer-0 token) rows
        self.logits = torch.zeros(G - 1, R, cfg.vocab_size, **bf)
        f32 = dict(device=self.device, dtype=torch.float32)
        self.ss = torch.zeros(H // 128, R, **f32)     # residual stream sums of squares per 128-feature tile
        self.pair_ss = torch.zeros(R, **f32)           # opening pair rows
        self.next_ss = torch.zeros(max_batch, **f32)   # gathered embedding rows
        self.folded = [{"qkv": ops.fold_norm(lw["qkv_proj"], lw["input_layernorm"]),
                        "gate_up": ops.fold_norm(lw["gate_up_proj"], lw["post_attention_layernorm"])}
                       for lw in weights["layers"]]
        self.lm_head_folded = torch.stack([ops.fold_norm(weights["lm_head"][j], weights["norm"])
                                           for j in range(G - 1)])
        self.output_codes = torch.zeros(max_batch, G, dtype=torch.long, device=self.device)
        self.zero_positions = torch.zeros(max_batch, dtype=torch.long, device=self.device)
        self.output_embeds = torch.zeros(max_batch, H, **bf)
        # per-row residual sampling state (sub_*_tensor of sglang_model.py:1115-1140)
        self.sub_temperature_tensor = torch.full((max_batch,), 0.9, dtype=torch.float32, device=self.device)
        self.sub_top_k_tensor = torch.full((max_batch,), 50, dtype=torch.long, device=self.device)
        self.sub_top_p_tensor = torch.ones(max_batch, dtype=torch.float32, device=self.device)
        self.sub_sampling_seed_tensor = torch.zeros(max_batch, dtype=torch.long, device=self.device)
        self.sub_do_sample_tensor = torch.ones(max_batch, dtype=torch.uint8, device=self.device)
        self.sub_sampled_max_top_k = 50
        self.sub_sampled_has_top_p = True
        self.sub_has_sampled_rows = True
        self.sub_has_argmax_rows = False
        ws = 0
        for rows in (max_batch, R):
            for k, n, e in ((H, (hq + 2 * hkv) * D, 0), (hq * D, H, 1), (H, 2 * I, 2), (I, H, 1),
                            (H, cfg.vocab_size, 0)):
                ws = max(ws, ops.linear_workspace_bytes(rows, k, n, e))
        self.workspace = torch.zeros(max(ws, 256), dtype=torch.uint8, device=self.device)
        self.scale = 1.0 / math.sqrt(D)
        # each projection prefetches into L2 the weight of the projection two launches
        # later in the chain (qkv -> gate_up, o -> down, gate_up -> next qkv / lm_head, ...)
        self.prefetch_l2 = True

    # ------------------------------------------------------------------
    def set_sampling(self, *, temperature, top_k, top_p, seeds, do_sample, batch: int, row0: int = 0) -> None:
        """Stage per-row residual sampling parameters of rows row0 .. row0 + batch
        (the subtalker rows of prepare_decode_buffers, sglang_model.py:1162-1270): a
        greedy row is staged as temperature 1, top-p 1, top-k 1, a sampled row's
        temperature is clamped to at least 1e-5, and the batch signature (ladder width,
        top-p flag) comes from the sampled rows.  With row0 > 0 the batch-wide flags
        widen to cover both parts."""
        from omni_b200.staging import predictor_signature

        rows = slice(row0, row0 + batch)
        ds = [bool(v) for v in torch.as_tensor(do_sample).reshape(-1).tolist()]
        t_in = [float(v) for v in torch.as_tensor(temperature, dtype=torch.float64).reshape(-1).tolist()]
        k_in = [int(v) for v in torch.as_tensor(top_k).reshape(-1).tolist()]
        p_in = [float(v) for v in torch.as_tensor(top_p, dtype=torch.float64).reshape(-1).tolist()]
        temps = [max(t, 1e-5) if d else 1.0 for t, d in zip(t_in, ds)]
        ks = [k if d else 1 for k, d in zip(k_in, ds)]
        ps = [p if d else 1.0 for p, d in zip(p_in, ds)]
        self.sub_temperature_tensor[rows].copy_(torch.tensor(temps, dtype=torch.float32), non_blocking=True)
        self.sub_top_k_tensor[rows].copy_(torch.tensor(ks, dtype=torch.long), non_blocking=True)
        self.sub_top_p_tensor[rows].copy_(torch.tensor(ps, dtype=torch.float32), non_blocking=True)
        self.sub_sampling_seed_tensor[rows].copy_(torch.as_tensor(seeds, dtype=torch.long), non_blocking=True)
        self.sub_do_sample_tensor[rows].copy_(torch.tensor(ds, dtype=torch.uint8), non_blocking=True)
        prev = (self.sub_has_sampled_rows, self.sub_has_argmax_rows, self.sub_sampled_max_top_k,
                self.sub_sampled_has_top_p) if row0 > 0 else None
        sampled = [i for i, d in enumerate(ds) if d]
        sig = predictor_signature([ks[i] for i in sampled], [ps[i] for i in sampled], self.cfg.vocab_size)
        if sig["has_unbounded_top_k"]:
            raise ValueError("unbounded subtalker top_k is outside the fused sampler's contract")
        self.sub_has_sampled_rows = bool(sampled)
        self.sub_has_argmax_rows = len(sampled) != len(ds)
        self.sub_sampled_max_top_k = sig["max_top_k"] if sampled else 4
        self.sub_sampled_has_top_p = sig["has_top_p"]
        if prev is not None:
            self.sub_has_sampled_rows = self.sub_has_sampled_rows or prev[0]
            self.sub_has_argmax_rows = self.sub_has_argmax_rows or prev[1]
            self.sub_sampled_max_top_k = max(self.sub_sampled_max_top_k, prev[2])
            self.sub_sampled_has_top_p = self.sub_sampled_has_top_p or prev[3]
        assert fused_raw_logit_block_k(self.sub_sampled_max_top_k) is not None

    # ------------------------------------------------------------------
    def _chain(self, after: list) -> list:
        ws = []
        for li, lw in enumerate(self.w["layers"]):
            ws += [self.folded[li]["qkv"], lw["o_proj"], self.folded[li]["gate_up"], lw["down_proj"]]
        return ws + list(after)

    def forward_tokens(self, x: torch.Tensor, x_ss: torch.Tensor, *, batch: int, tokens: int,
                       cache_len: int, after: list | None = None) -> torch.Tensor:
        """The predictor stack on rows (request, token) at slots cache_len.. with input
        sums of squares x_ss (one part); leaves the residual stream in self.h and its sums
        of squares in self.ss, the input of the folded final norm of the lm_head
        (predictor_forward_tokens, sglang_model.py:2036-2098).  after: the weights the
        stream's next projections use (for the L2 prefetch of the last layers)."""
        cfg = self.cfg
        rows = batch * tokens
        H, D = cfg.hidden_size, cfg.head_dim
        hq, hkv = cfg.num_attention_heads, cfg.num_key_value_heads
        eps = cfg.rms_norm_eps
        h, q, attn, act = self.h[:rows], self.q[:rows], self.attn[:rows], self.act[:rows]
        parts = H // 128
        chain = self._chain(after or []) if self.prefetch_l2 else []

        def pf(i):
            return chain[i + 2] if i + 2 < len(chain) else None

        resid, ss_in, ss_parts = x, x_ss, 1
        for li, lw in enumerate(self.w["layers"]):
            ops.linear_fused(resid, self.folded[li]["qkv"], q, epilogue=ops.EPI_QKV_ROPE, ss_in=ss_in,
                             ss_in_parts=ss_parts, norm_eps=eps, l2_prefetch=pf(4 * li),
                             qkv=dict(num_q_heads=hq, num_kv_heads=hkv, head_dim=D, q_norm=lw["q_norm"],
                                      k_norm=lw["k_norm"], eps=eps, cos_sin=self.cos_sin, tokens_per_req=tokens,
                                      slot_stride=cfg.cache_len, slot_base=cache_len, k_cache=self.k_cache[li],
                                      v_cache=self.v_cache[li]))
            ops.predictor_attention(q, self.k_cache[li], self.v_cache[li], num_q_heads=hq, num_kv_heads=hkv,
                                    head_dim=D, tokens_per_req=tokens, slot_stride=cfg.cache_len,
                                    slot_base=cache_len, sm_scale=self.scale, out=attn)
            ops.linear_fused(attn, lw["o_proj"], h, epilogue=ops.EPI_RESIDUAL, residual=resid, ss_out=self.ss,
                             l2_prefetch=pf(4 * li + 1))
            resid, ss_in, ss_parts = h, self.ss, parts
            ops.linear_fused(h, self.folded[li]["gate_up"], act, epilogue=ops.EPI_SWIGLU, ss_in=self.ss,
                             ss_in_parts=parts, norm_eps=eps, l2_prefetch=pf(4 * li + 2))
            ops.linear_fused(act, lw["down_proj"], h, epilogue=ops.EPI_RESIDUAL, residual=h, ss_out=self.ss,
                             l2_prefetch=pf(4 * li + 3))
        return h

    def codebook_logits(self, j: int, batch: int) -> torch.Tensor:
        """The lm_head logits of residual codebook j + 1 for the batch's rows."""
        return self.logits[0, 1: 2 * batch: 2] if j == 0 else self.logits[j, :batch]

    def code_predictor_forward(
        self,
        layer0_codes: torch.Tensor,
        talker_hidden: torch.Tensor,
        semantic_positions: torch.Tensor | None = None,
        *,
        final_norm: torch.Tensor | None = None,
        final_ss: torch.Tensor | None = None,
        final_eps: float = 1e-6,
        hidden_out: torch.Tensor | None = None,
    ) -> tuple[torch.Tensor, torch.Tensor]:
        """(layer0_codes [B, 1] i64, talker_hidden [B, 1, H] bf16, semantic_positions [B] or
        None) -> (codes [B, G, 1] i64, summed [B, 1, H] bf16), the reference's
        code_predictor_forward (sglang_model.py:1317-1346): talker_hidden is the talker's
        normalized final hidden state.
        Fast path of the fused decode step: with final_norm (gain) and final_ss (row sums
        of squares [parts, rows] of the talker's last residual), talker_hidden is that
        residual and the talker's final RMSNorm is applied on the way in; the normalized
        rows then also go to hidden_out when given."""
        if (final_norm is None) != (final_ss is None):
            raise ValueError("final_norm and final_ss are given together")
        cfg = self.cfg
        if layer0_codes.ndim == 2:
            layer0_codes = layer0_codes[:, 0]
        if talker_hidden.ndim == 3:
            talker_hidden = talker_hidden[:, 0]
        B = layer0_codes.shape[0]
        if B > self.max_batch:
            raise RuntimeError("code predictor buffers are too small for this batch")
        H, G = cfg.hidden_size, cfg.num_code_groups
        if semantic_positions is None:
            # (the reference then samples unseeded; here every row draws at position 0)
            semantic_positions = self.zero_positions[:B]
        elif semantic_positions.ndim == 2:
            semantic_positions = semantic_positions.reshape(-1)
        codes = self.output_codes[:B]
        summed = self.output_embeds[:B]
        pair = self.pair[: 2 * B]
        from omni_b200 import _lib

        if talker_hidden.dtype is not torch.bfloat16 or talker_hidden.shape[-1] != H or talker_hidden.stride(-1) != 1:
            raise ValueError("talker_hidden must be bf16 [B, 1, H] with unit feature stride")
        if layer0_codes.dtype is not torch.long or not layer0_codes.is_contiguous():
            layer0_codes = layer0_codes.to(torch.long).contiguous()
        _lib.call("omni_predictor_pair_inputs", layer0_codes.data_ptr(), talker_hidden.data_ptr(),
                  talker_hidden.stride(0), _lib.ptr(final_norm), _lib.ptr(final_ss),
                  final_ss.shape[0] if final_ss is not None else 0, final_ss.stride(0) if final_ss is not None else 0,
                  float(final_eps), _lib.ptr(hidden_out), self.layer0_embedding.data_ptr(), B, H,
                  pair.data_ptr(), summed.data_ptr(), self.pair_ss.data_ptr(), codes.data_ptr(), codes.stride(0),
                  _lib.stream_of(self.device))
        w0 = self.w["layers"][0]
        nxt = [self.folded[0]["qkv"], w0["o_proj"]]
        h = self.forward_tokens(pair, self.pair_ss, batch=B, tokens=2, cache_len=0,
                                after=[self.lm_head_folded[0]] + nxt)
        argmax_all = not self.sub_has_sampled_rows
        parts = H // 128
        eps = cfg.rms_norm_eps
        for j in range(G - 1):
            rows = 2 * B if j == 0 else B
            ops.linear_fused(h[:rows], self.lm_head_folded[j], self.logits[j, :rows], epilogue=ops.EPI_STORE,
                             ss_in=self.ss, ss_in_parts=parts, norm_eps=eps,
                             l2_prefetch=nxt[1] if self.prefetch_l2 and j < G - 2 else None)
            predictor_sample_step(
                self.codebook_logits(j, B),
                temperatures=self.sub_temperature_tensor[:B],
                top_ks=self.sub_top_k_tensor[:B],
                top_ps=self.sub_top_p_tensor[:B],
                seeds=self.sub_sampling_seed_tensor[:B],
                positions=semantic_positions,
                pos_mul=G - 1,
                pos_add=j + 1,
                do_sample=self.sub_do_sample_tensor[:B] if self.sub_has_argmax_rows else None,
                argmax_all=argmax_all,
                max_top_k=self.sub_sampled_max_top_k,
                has_top_p=self.sub_sampled_has_top_p,
                codes=codes[:, j + 1],
                table=self.w["codec_embedding"][j],
                gathered=self.next_in[:B],
                summed=summed,
                gathered_ss=self.next_ss[:B],
            )
            if j < G - 2:
                h = self.forward_tokens(self.next_in[:B], self.next_ss[:B], batch=B, tokens=1, cache_len=2 + j,
                                        after=[self.lm_head_folded[j + 1]] + (nxt if j + 1 < G - 2 else []))
        return codes.unsqueeze(-1), summed.unsqueeze(1)
