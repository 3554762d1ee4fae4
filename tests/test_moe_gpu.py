"""GPU parity of the MoE block (block-FP8 experts) against the CPU oracle.

- e4m3 quantisation of the normed rows and of the expert activations, the
  router's top-k ids and weights, the expert-sorted order and work list:
  bit-exact against omni_oracle.c given the device's own inputs to each step;
- grouped FP8 GEMMs: against an fp32 GEMM of the dequantised operands
  (cosine >= 0.9999, max-abs <= 1e-2 x scale for the bf16 outputs; the
  re-quantised activation codes may sit one e4m3 step apart where the fp32
  value lies within rounding of a code boundary);
- the whole block: against oracle.model.moe_block, within the bf16 tolerance
  of the north-star contract (cosine >= 0.999, max-abs <= 2e-2 x scale).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import sampler as orc
from oracle.model import dequant_expert, dequant_rows, moe_block, rb, to_f32

pytestmark = pytest.mark.gpu

DEV = "cuda"


def close(got, ref, rel=1e-2, cos_min=0.9999):
    g = got.float().flatten().cpu()
    r = ref.float().flatten().cpu()
    assert torch.isfinite(g).all()
    cos = torch.nn.functional.cosine_similarity(g, r, dim=0).item()
    err = (g - r).abs().max().item()
    scale = r.abs().max().item()
    assert cos >= cos_min and err <= rel * scale + 1e-6, f"cos={cos:.6f} err={err:.4g} scale={scale:.4g}"


def make_block(tokens=48, seed=0, hidden=1024):
    from omni_b200.config import MoEConfig
    from omni_b200.moe import MoEBlock, init_moe_weights

    cfg = MoEConfig()
    g = torch.Generator(device=DEV).manual_seed(seed)
    w = init_moe_weights(cfg, hidden, generator=g, device=DEV)
    blk = MoEBlock(cfg, hidden, max_batch=tokens, device=DEV)
    h = torch.randn(tokens, hidden, generator=g, device=DEV).to(torch.bfloat16)
    gain = (1.0 + 0.05 * torch.randn(hidden, generator=g, device=DEV)).to(torch.bfloat16)
    ss = h.float().view(tokens, hidden // 128, 128).pow(2).sum(-1).t().contiguous()
    return cfg, w, blk, h, gain, ss


@pytest.mark.parametrize("tokens", [1, 48, 256])
def test_rmsnorm_quant(tokens):
    from omni_b200 import ops

    cfg, w, blk, h, gain, ss = make_block(tokens)
    x, xq, xs = blk.x[:tokens], blk.xq[:tokens], blk.xs[:tokens]
    ops.moe_rmsnorm_quant(h, ss, 8, gain, 1e-6, x, xq, xs)
    torch.cuda.synchronize()
    ref = h.float() * torch.rsqrt(h.float().pow(2).mean(-1, keepdim=True) + 1e-6) * gain.float()
    close(x, ref)
    q, s = orc.quant_fp8_group(x.float().cpu().numpy())
    assert np.array_equal(xq.cpu().numpy(), q)
    assert np.array_equal(xs.cpu().numpy().view(np.uint32), s.view(np.uint32))


@pytest.mark.parametrize("tokens", [1, 48, 256])
def test_router_topk_bit_exact(tokens):
    from omni_b200 import ops

    cfg, w, blk, h, gain, ss = make_block(tokens, seed=1)
    x = blk.x[:tokens]
    x.copy_(h)
    ids, tw = blk.topk_ids[:tokens], blk.topk_weights[:tokens]
    logits = blk.router_logits[:tokens]
    ops.linear_fused(x, w["gate"], logits, epilogue=ops.EPI_ROUTER, router={"topk_ids": ids, "topk_weights": tw})
    torch.cuda.synchronize()
    close(logits, x.float() @ w["gate"].float().t())
    want_ids, want_w = orc.moe_route(logits.float().cpu().numpy(), cfg.num_experts_per_tok)
    assert np.array_equal(ids.cpu().numpy(), want_ids)
    assert np.array_equal(tw.cpu().numpy().view(np.uint32), want_w.view(np.uint32))


def test_router_ties_take_the_lower_expert():
    """Equal logits give equal probabilities: the lower expert index wins each tie."""
    from omni_b200 import ops

    tokens, H = 4, 1024
    x = torch.zeros(tokens, H, device=DEV, dtype=torch.bfloat16)
    x[:, 0] = 1.0
    gate = torch.zeros(128, H, device=DEV, dtype=torch.bfloat16)
    gate[:, 0] = torch.tensor([0.5 if e % 3 == 0 else 0.25 for e in range(128)], dtype=torch.bfloat16)
    ids = torch.zeros(tokens, 8, dtype=torch.int32, device=DEV)
    tw = torch.zeros(tokens, 8, dtype=torch.float32, device=DEV)
    logits = torch.zeros(tokens, 128, device=DEV, dtype=torch.bfloat16)
    ops.linear_fused(x, gate, logits, epilogue=ops.EPI_ROUTER, router={"topk_ids": ids, "topk_weights": tw})
    torch.cuda.synchronize()
    assert ids[0].tolist() == [0, 3, 6, 9, 12, 15, 18, 21]
    want_ids, want_w = orc.moe_route(logits.float().cpu().numpy(), 8)
    assert np.array_equal(ids.cpu().numpy(), want_ids)
    assert np.allclose(tw.cpu().numpy(), 1.0 / 8)


@pytest.mark.parametrize("tokens,skew", [(1, False), (48, False), (256, False), (256, True)])
def test_align_gather_bit_exact(tokens, skew):
    from omni_b200 import ops

    cfg, w, blk, h, gain, ss = make_block(tokens, seed=2)
    rng = np.random.default_rng(tokens)
    E, k = cfg.num_experts, cfg.num_experts_per_tok
    if skew:  # every token picks experts 0..7: each of them holds 256 rows (8 chunks of 32)
        ids_np = np.tile(np.arange(k, dtype=np.int32), (tokens, 1))
    else:
        ids_np = np.stack([rng.permutation(E)[:k] for _ in range(tokens)]).astype(np.int32)
    ids = torch.from_numpy(ids_np).to(DEV)
    xq = torch.randint(0, 255, (tokens, 1024), dtype=torch.uint8, device=DEV)
    xs = torch.rand(tokens, 8, device=DEV)
    ops.moe_align_gather(ids, E, xq, xs, blk.permuted_q, blk.permuted_s, blk.slot_of[:tokens], blk.expert_offsets,
                         blk.chunks, blk.n_chunks)
    torch.cuda.synchronize()
    offsets, pairs = orc.moe_permute(ids_np, E)
    assert blk.expert_offsets.cpu().numpy().tolist() == offsets.tolist()
    slot_of = blk.slot_of[:tokens].cpu().numpy().reshape(-1)
    want = np.empty(tokens * k, np.int64)
    want[pairs] = np.arange(tokens * k)
    assert slot_of.tolist() == want.tolist()
    pq = blk.permuted_q.cpu().numpy()
    for i in range(tokens * k):
        assert np.array_equal(pq[slot_of[i]], xq[i // k].cpu().numpy())
    n = int(blk.n_chunks.item())
    ch = blk.chunks[:n].cpu().numpy()
    cnt = np.diff(offsets)
    want_ch = [(e, offsets[e] + c * 32, min(32, cnt[e] - c * 32)) for e in range(E) for c in range((cnt[e] + 31) // 32)]
    assert [tuple(r[:3]) for r in ch] == want_ch


@pytest.mark.parametrize("tokens", [1, 48, 256])
def test_grouped_fp8_gemms(tokens):
    from omni_b200 import ops

    cfg, w, blk, h, gain, ss = make_block(tokens, seed=3)
    x, xq, xs = blk.x[:tokens], blk.xq[:tokens], blk.xs[:tokens]
    ops.moe_rmsnorm_quant(h, ss, 8, gain, 1e-6, x, xq, xs)
    ids, tw = blk.topk_ids[:tokens], blk.topk_weights[:tokens]
    ops.linear_fused(x, w["gate"], blk.router_logits[:tokens], epilogue=ops.EPI_ROUTER,
                     router={"topk_ids": ids, "topk_weights": tw})
    ops.moe_align_gather(ids, cfg.num_experts, xq, xs, blk.permuted_q, blk.permuted_s, blk.slot_of[:tokens],
                         blk.expert_offsets, blk.chunks, blk.n_chunks)
    ops.moe_gate_up_fp8(blk.permuted_q, blk.permuted_s, w["w13"], w["w13_scale"], blk.chunks, blk.n_chunks,
                        blk.act_q, blk.act_s)
    ops.moe_down_fp8(blk.act_q, blk.act_s, w["w2"], w["w2_scale"], blk.chunks, blk.n_chunks, blk.y)
    torch.cuda.synchronize()
    A = tokens * cfg.num_experts_per_tok
    off = blk.expert_offsets.cpu().numpy()
    pq, ps = blk.permuted_q[:A].cpu().numpy(), blk.permuted_s[:A].cpu().numpy()
    aq, as_ = blk.act_q[:A].cpu().numpy(), blk.act_s[:A].cpu().numpy()
    y = blk.y[:A].float().cpu()
    I = cfg.moe_intermediate_size
    wc = to_f32({k: w[k] for k in ("w13", "w13_scale", "w2", "w2_scale")})
    xd = dequant_rows(pq, ps)
    ad_dev = dequant_rows(aq, as_)
    act_ref = torch.zeros(A, I)
    y_ref = torch.zeros(A, 1024)
    for e in range(cfg.num_experts):
        r0, r1 = int(off[e]), int(off[e + 1])
        if r1 == r0:
            continue
        gu = xd[r0:r1] @ dequant_expert(wc["w13"][e], wc["w13_scale"][e]).t()
        act_ref[r0:r1] = rb(torch.nn.functional.silu(rb(gu[:, :I])) * rb(gu[:, I:]))
        y_ref[r0:r1] = ad_dev[r0:r1] @ dequant_expert(wc["w2"][e], wc["w2_scale"][e]).t()
    # activation codes: the oracle's quantisation of the fp32 reference activation
    q_ref, s_ref = orc.quant_fp8_group(act_ref.numpy())
    close(ad_dev, dequant_rows(q_ref, s_ref), rel=0.07, cos_min=0.999)
    assert (aq == q_ref).mean() >= 0.97
    close(torch.from_numpy(as_), torch.from_numpy(s_ref), rel=1e-2, cos_min=0.9999)
    # down projection of the device's own activation codes: fp32 GEMM tolerance
    close(y, y_ref)


@pytest.mark.parametrize("tokens", [1, 48, 256])
def test_moe_block_matches_oracle(tokens):
    cfg, w, blk, h, gain, ss = make_block(tokens, seed=4)
    h0 = h.clone()
    blk.forward(h, ss, 8, gain, 1e-6, w)
    torch.cuda.synchronize()
    n = rb(h0.float().cpu() * torch.rsqrt(h0.float().cpu().pow(2).mean(-1, keepdim=True) + 1e-6)
           * gain.float().cpu())
    out, _, ids, _ = moe_block(n, to_f32(w), cfg.num_experts_per_tok)
    ref = rb(h0.float().cpu() + out)
    close(h, ref, rel=2e-2, cos_min=0.999)
    # the block's own increment, which carries the routed and shared experts
    close(h.float() - h0.float(), out, rel=5e-2, cos_min=0.995)
    # the sums of squares of the new residual stream, per 128-feature part
    want_ss = h.float().view(tokens, 8, 128).pow(2).sum(-1).t()
    close(ss[:, :tokens], want_ss, rel=1e-5, cos_min=0.99999)


def test_moe_block_is_deterministic():
    cfg, w, blk, h, gain, ss = make_block(64, seed=5)
    outs = []
    for _ in range(2):
        hh, s2 = h.clone(), ss.clone()
        blk.forward(hh, s2, 8, gain, 1e-6, w)
        outs.append(hh)
    torch.cuda.synchronize()
    assert torch.equal(outs[0], outs[1])
