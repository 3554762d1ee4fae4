"""CPU restatement of the talker decode step — TEST INFRASTRUCTURE ONLY.

fp32 PyTorch-CPU arithmetic on the bf16 weights, rounding to bf16 where the
reference's plain path keeps bf16 tensors (outputs of every projection, norm,
rotary and attention; the residual stream), following:

- talker layer: Qwen3OmniMoeThinkerTextAttention + dense MLP
  (sglang_omni/models/qwen3_omni/components/thinker_model.py:152-402,
  talker.py:216-247), decode forward talker.py:438-491;
- MoE layer (moe_block): router gate + TopK(renormalize) + block-FP8 FusedMoE +
  sigmoid-gated shared expert (talker.py:325-351, thinker_model.py:405-470,
  quantization.py:124-167), with the routing and the e4m3 quantisation done by
  omni_oracle.c (orc_moe_route, orc_quant_fp8_group) and the expert GEMMs in
  fp32 on the dequantised operands;
- paged GQA decode attention over req_to_token slots (RadixAttention decode,
  thinker_model.py:373-379), softmax in fp32;
- layer-0 draw: omni_oracle.c orc_layer0_sample (talker.py:1376-1412);
- code predictor: code_predictor_forward_incremental
  (sglang_model.py:1743-1879), predictor_forward_tokens (:2036-2098),
  predictor_cached_self_attention (:2168-2233), seeded residual sampler
  omni_oracle.c orc_sample_topk_topp.

Also the CPU baseline that bench.py times on the host cores.
"""

from __future__ import annotations

import math

import numpy as np
import torch

from oracle import sampler as orc

BF16 = torch.bfloat16


def rb(x: torch.Tensor) -> torch.Tensor:
    """Round an fp32 tensor to bf16 and back (a bf16 storage point)."""
    return x.to(BF16).float()


def rmsnorm(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps) * w


def rope_cache(max_pos: int, d: int, theta: float) -> torch.Tensor:
    inv = 1.0 / (theta ** (torch.arange(0, d, 2, dtype=torch.float32) / d))
    f = torch.outer(torch.arange(max_pos, dtype=torch.float32), inv)
    return torch.cat([f.cos(), f.sin()], -1)


def rope_neox(x: torch.Tensor, cs: torch.Tensor) -> torch.Tensor:
    """x [..., heads, d]; cs [..., d] broadcast over heads."""
    d = x.shape[-1]
    cos, sin = cs[..., None, : d // 2], cs[..., None, d // 2:]
    a, b = x[..., : d // 2], x[..., d // 2:]
    return torch.cat([a * cos - b * sin, b * cos + a * sin], -1)


def to_f32(weights) -> dict | list | torch.Tensor:
    """fp32 CPU copies; e4m3 codes (uint8) and their scales are copied unchanged."""
    if isinstance(weights, dict):
        return {k: to_f32(v) for k, v in weights.items()}
    if isinstance(weights, list):
        return [to_f32(v) for v in weights]
    if weights.dtype == torch.uint8:
        return weights.detach().cpu()
    return weights.detach().float().cpu()


def dequant_rows(q: np.ndarray, scales: np.ndarray, group: int = 128) -> torch.Tensor:
    """e4m3 codes [rows, cols] with per-row group scales [rows, cols / group] -> fp32."""
    v = orc.e4m3_to_f32(q)
    return torch.from_numpy(v * np.repeat(scales, group, axis=1))


def dequant_expert(q: torch.Tensor, scale: torch.Tensor, block: int = 128) -> torch.Tensor:
    """One expert's e4m3 weight [R, C] with its 128x128 block scales [R/128, C/128] -> fp32."""
    v = torch.from_numpy(orc.e4m3_to_f32(q.numpy()))
    s = scale.repeat_interleave(block, 0).repeat_interleave(block, 1)
    return v * s


def moe_block(x: torch.Tensor, w: dict, top_k: int):
    """MoE block output (bf16-rounded fp32 [B, H]) for the normed rows x, plus the
    router logits (bf16-rounded), top-k ids and weights."""
    B, H = x.shape
    logits = rb(x @ w["gate"].t())
    ids, tw = orc.moe_route(logits.numpy(), top_k)
    xq, xs = orc.quant_fp8_group(x.numpy())
    xd = dequant_rows(xq, xs)
    I = w["w13"].shape[1] // 2
    y = torch.zeros(B, top_k, H)
    for e in np.unique(ids):
        tok, slot = np.nonzero(ids == e)
        w13 = dequant_expert(w["w13"][e], w["w13_scale"][e])
        w2 = dequant_expert(w["w2"][e], w["w2_scale"][e])
        gu = xd[tok] @ w13.t()
        a = rb(torch.nn.functional.silu(rb(gu[:, :I])) * rb(gu[:, I:]))
        aq, as_ = orc.quant_fp8_group(a.numpy())
        y[tok, slot] = rb(dequant_rows(aq, as_) @ w2.t())
    routed = torch.zeros(B, H)
    twt = torch.from_numpy(tw)
    for kk in range(top_k):
        routed = routed + twt[:, kk: kk + 1] * y[:, kk]
    routed = rb(routed)
    sg = rb(x @ w["shared_expert_gate"].t())
    gus = x @ w["shared_gate_up"].t()
    Is = gus.shape[1] // 2
    sa = rb(torch.nn.functional.silu(rb(gus[:, :Is])) * rb(gus[:, Is:]))
    so = rb(sa @ w["shared_down"].t())
    shared = rb(so * torch.sigmoid(sg))
    return rb(routed + shared), logits, ids, tw


def bits(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


class OracleTalker:
    """fp32 CPU decode step of the dense talker + code predictor."""

    def __init__(self, cfg, talker_w: dict, predictor_w: dict):
        self.cfg = cfg
        self.w = to_f32(talker_w)
        self.pw = to_f32(predictor_w)
        self.cs = rope_cache(cfg.max_context, cfg.head_dim, cfg.rope_theta)
        pc = cfg.predictor
        self.pcs = rope_cache(pc.cache_len, pc.head_dim, pc.rope_theta)

    # ------------------------------------------------------------------
    def talker_forward(self, feedback, text, positions, out_cache_loc, seq_lens, req_to_token, k_pool, v_pool):
        """One decode forward; k_pool/v_pool: fp32 [L, slots, hkv, d] updated in place.
        Returns (logits fp32 [B, V], hidden bf16-rounded [B, H])."""
        B = feedback.shape[0]
        x = rb(feedback.float() + (text.float() if text is not None else 0.0))
        ctx = [req_to_token[b, : int(seq_lens[b])].long() for b in range(B)]
        x = self.forward_rows(x, positions, out_cache_loc, ctx, k_pool, v_pool)
        hidden = rb(rmsnorm(x, self.w["norm"], self.cfg.rms_norm_eps))
        return hidden @ self.w["codec_head"].t(), hidden

    def mixed_forward(self, feedback, text, positions, out_cache_loc, seq_lens, req_to_token, prompt_embeds,
                      ext_positions, ext_cache_loc, ext_ctx, select, k_pool, v_pool):
        """A mixed batch: decode rows (as talker_forward) followed by extend rows (prompt
        embeddings, positions, slots, and for each row the slots it attends, causal within its
        stream) through the layers together; logits/hidden of the rows in `select`."""
        B = feedback.shape[0]
        xd = rb(feedback.float() + (text.float() if text is not None else 0.0))
        x = torch.cat([xd, prompt_embeds.float()], 0)
        ctx = [req_to_token[b, : int(seq_lens[b])].long() for b in range(B)] + list(ext_ctx)
        pos = torch.cat([torch.as_tensor(positions), torch.as_tensor(ext_positions)])
        loc = torch.cat([torch.as_tensor(out_cache_loc), torch.as_tensor(ext_cache_loc)])
        x = self.forward_rows(x, pos, loc, ctx, k_pool, v_pool)
        hidden = rb(rmsnorm(x[select], self.w["norm"], self.cfg.rms_norm_eps))
        return hidden @ self.w["codec_head"].t(), hidden

    def forward_rows(self, x, positions, cache_locs, ctx_slots, k_pool, v_pool):
        """The decoder layers over rows x [R, H] (bf16-rounded fp32): row r sits at position
        positions[r], writes its K/V at slot cache_locs[r] and attends the slots ctx_slots[r]
        (its own slot included).  Returns the residual stream after the last layer."""
        cfg = self.cfg
        D = cfg.head_dim
        hq, hkv = cfg.num_attention_heads, cfg.num_key_value_heads
        eps = cfg.rms_norm_eps
        R = x.shape[0]
        cs = self.cs[torch.as_tensor(positions).long()]
        loc = torch.as_tensor(cache_locs).long()
        scale = 1.0 / math.sqrt(D)
        for li, lw in enumerate(self.w["layers"]):
            n = rb(rmsnorm(x, lw["input_layernorm"], eps))
            qkv = rb(n @ lw["qkv_proj"].t())
            q = qkv[:, : hq * D].view(R, hq, D)
            k = qkv[:, hq * D: (hq + hkv) * D].view(R, hkv, D)
            v = qkv[:, (hq + hkv) * D:].view(R, hkv, D)
            q = rb(rmsnorm(q, lw["q_norm"], eps))
            k = rb(rmsnorm(k, lw["k_norm"], eps))
            q = rb(rope_neox(q, cs))
            k = rb(rope_neox(k, cs))
            k_pool[li, loc] = k
            v_pool[li, loc] = v
            att = torch.empty(R, hq, D)
            for r in range(R):
                slots = ctx_slots[r]
                kk = k_pool[li, slots]  # [L, hkv, D]
                vv = v_pool[li, slots]
                qb = q[r].view(hkv, hq // hkv, D)
                sc = torch.einsum("hgd,lhd->hgl", qb, kk) * scale
                p = torch.softmax(sc, -1)
                att[r] = torch.einsum("hgl,lhd->hgd", p, vv).reshape(hq, D)
            att = rb(att.reshape(R, hq * D))
            x = rb(x + att @ lw["o_proj"].t())
            n = rb(rmsnorm(x, lw["post_attention_layernorm"], eps))
            if "moe" in lw:
                out, _, _, _ = moe_block(n, lw["moe"], cfg.moe.num_experts_per_tok)
                x = rb(x + out)
                continue
            gu = n @ lw["gate_up_proj"].t()
            I = gu.shape[1] // 2
            a = rb(torch.nn.functional.silu(rb(gu[:, :I])) * rb(gu[:, I:]))
            x = rb(x + a @ lw["down_proj"].t())
        return x

    # ------------------------------------------------------------------
    def predictor_tokens(self, x, k_cache, v_cache, *, batch, tokens, cache_len):
        """x [batch*tokens, H] rows (request, token) at slots cache_len..; caches fp32
        [L, batch, S, hkv, d] updated in place; returns final-normed rows."""
        pc = self.cfg.predictor
        D, hq, hkv, eps = pc.head_dim, pc.num_attention_heads, pc.num_key_value_heads, pc.rms_norm_eps
        rows = batch * tokens
        pos = cache_len + torch.arange(tokens).repeat(batch)
        cs = self.pcs[pos]
        scale = 1.0 / math.sqrt(D)
        h = x
        for li, lw in enumerate(self.pw["layers"]):
            n = rb(rmsnorm(h, lw["input_layernorm"], eps))
            qkv = rb(n @ lw["qkv_proj"].t())
            q = qkv[:, : hq * D].view(rows, hq, D)
            k = qkv[:, hq * D: (hq + hkv) * D].view(rows, hkv, D)
            v = qkv[:, (hq + hkv) * D:].view(rows, hkv, D)
            q = rb(rope_neox(rb(rmsnorm(q, lw["q_norm"], eps)), cs))
            k = rb(rope_neox(rb(rmsnorm(k, lw["k_norm"], eps)), cs))
            k_cache[li, :, cache_len: cache_len + tokens] = k.view(batch, tokens, hkv, D)
            v_cache[li, :, cache_len: cache_len + tokens] = v.view(batch, tokens, hkv, D)
            end = cache_len + tokens
            kk = k_cache[li, :, :end].transpose(1, 2).repeat_interleave(hq // hkv, 1)  # [b, hq, end, D]
            vv = v_cache[li, :, :end].transpose(1, 2).repeat_interleave(hq // hkv, 1)
            qq = q.view(batch, tokens, hq, D).transpose(1, 2)
            s = qq @ kk.transpose(-1, -2) * scale
            mask = torch.arange(end)[None, :] > (cache_len + torch.arange(tokens))[:, None]
            s = s.masked_fill(mask, float("-inf"))
            att = rb((torch.softmax(s, -1) @ vv).transpose(1, 2).reshape(rows, hq * D))
            h = rb(h + att @ lw["o_proj"].t())
            n = rb(rmsnorm(h, lw["post_attention_layernorm"], eps))
            gu = n @ lw["gate_up_proj"].t()
            I = gu.shape[1] // 2
            a = rb(torch.nn.functional.silu(rb(gu[:, :I])) * rb(gu[:, I:]))
            h = rb(h + a @ lw["down_proj"].t())
        return rb(rmsnorm(h, self.pw["norm"], eps))

    def code_predictor(self, c0, talker_hidden, semantic_positions, sampling, *, forced_codes=None):
        """Returns (codes [B, G] i64, summed bf16 bits [B, H], lm_head logits [G-1, B, V] fp32).
        With forced_codes [B, G], the loop feeds those codes instead of its own draws
        (teacher forcing), so every pass sees the same inputs as the device run."""
        pc = self.cfg.predictor
        G, H = pc.num_code_groups, pc.hidden_size
        B = c0.shape[0]
        S, hkv, D = pc.cache_len, pc.num_key_value_heads, pc.head_dim
        kc = torch.zeros(pc.num_hidden_layers, B, S, hkv, D)
        vc = torch.zeros_like(kc)
        table0 = self.w["codec_embedding"]
        e0 = table0[c0]
        summed = bits(e0.to(BF16))
        codes = np.zeros((B, G), np.int64)
        codes[:, 0] = c0.numpy()
        pair = torch.stack([talker_hidden.float(), e0], 1).reshape(2 * B, H)
        out = self.predictor_tokens(pair, kc, vc, batch=B, tokens=2, cache_len=0)
        last = out.view(B, 2, H)[:, 1]
        all_logits = torch.zeros(G - 1, B, pc.vocab_size)
        for j in range(G - 1):
            logits = rb(last @ self.pw["lm_head"][j].t())
            all_logits[j] = logits
            pos = semantic_positions.numpy() * (G - 1) + (j + 1)
            drawn = orc.sample_topk_topp(bits(logits.to(BF16)), sampling["temperature"], sampling["top_k"],
                                         sampling["top_p"], sampling["seed"], pos,
                                         max_top_k=sampling["max_top_k"], has_top_p=sampling["has_top_p"])
            am = np.argmax(logits.numpy(), axis=1)  # first NaN, else first maximum (torch.argmax)
            drawn = np.where(np.asarray(sampling["do_sample"], bool), drawn, am)
            code = drawn if forced_codes is None else forced_codes[:, j + 1]
            codes[:, j + 1] = code
            table = bits(self.pw["codec_embedding"][j].to(BF16))
            gathered, summed = orc.gather_add(code, table, summed)
            if j < G - 2:
                nxt = orc.bf16_bits_to_f32(gathered)
                last = self.predictor_tokens(torch.from_numpy(nxt), kc, vc, batch=B, tokens=1, cache_len=2 + j)
        return codes, summed, all_logits

    def layer0(self, logits, state):
        return orc.layer0_sample(logits.numpy(), state["penalties"], state["rep_mask"], state["suppress_mask"],
                                 state["temperature"], state["top_k"], state["top_p"], state["min_p"], state["seed"],
                                 state["positions"], max_top_k=state["max_top_k"])
