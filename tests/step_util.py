"""Shared check of one decode step against the CPU oracle (used by the step and config tests).

- packing (positions, slots, page table, free-page head): bit-exact;
- talker logits and final hidden: cosine >= 0.999, max-abs <= 2e-2 x scale (the
  north-star bf16 contract), the new K/V at their slots at cosine >= 0.999;
- the layer-0 draw and every residual draw: bit-exact against the oracle sampler
  applied to the device's own logits (with the staged penalty / suppress masks);
- predictor lm_head logits under teacher forcing: the same tolerance plus one bf16
  ulp of output rounding; the summed codec embeddings: bit-exact.
"""

from __future__ import annotations

import numpy as np
import torch

from oracle import sampler as orc
from oracle.model import OracleTalker, bits

DEV = "cuda"


def cos_err(a: torch.Tensor, b: torch.Tensor):
    a, b = a.float().flatten().cpu(), b.float().flatten().cpu()
    cos = torch.nn.functional.cosine_similarity(a, b, dim=0).item()
    return cos, (a - b).abs().max().item(), b.abs().max().item()


def err_quantile(a: torch.Tensor, b: torch.Tensor, q: float = 0.999) -> float:
    d = (a.float().flatten().cpu() - b.float().flatten().cpu()).abs()
    return torch.quantile(d, q).item() if d.numel() <= 16_000_000 else d.max().item()


def bf16_ulp(scale: float) -> float:
    """The spacing of bf16 values at magnitude `scale` (>= 1)."""
    return 2.0 ** (np.floor(np.log2(max(scale, 1.0))) - 7)


def check_step_against_oracle(r, *, use_graph: bool = False, tol: float = 2e-2, depth_ulps: int = 0) -> dict:
    """Runs one step of runner r (eager, or its captured graph) and checks it against the
    oracle; returns the measured agreement figures.

    Hidden states and logits: cosine >= 0.999 and max-abs <= tol x scale, plus
    depth_ulps bf16 steps at the scale for deep stacks (the GPU and the oracle round to
    bf16 at the same storage points but accumulate in different orders, so a residual
    value can land one bf16 step apart and the difference carries through the following
    layers); with depth_ulps > 0 the 99.9th percentile of the error must still be within
    tol x scale."""
    cfg = r.cfg
    B = r.batch_size
    # snapshot the pre-step state for the oracle
    seq0 = r.seq_lens[:B].cpu().numpy()
    r2t0 = r.r2t.req_to_token[:B].cpu().numpy()
    free = r.allocator.free_pages.cpu().numpy()
    head0 = int(r.allocator.free_head.item())
    kpool = r.kv.k_buffer.float().cpu()
    vpool = r.kv.v_buffer.float().cpu()
    feedback = r.predictor.output_embeds[:B].clone().cpu()
    text = r.text_embeds[:B].clone().cpu()
    t = r.talker
    l0_state = dict(penalties=t.repetition_penalties[:B].cpu().numpy(), rep_mask=t.repetition_mask[:B].cpu().numpy(),
                    suppress_mask=t.suppress_mask[:B].cpu().numpy(), temperature=t.sampling_temperatures[:B].cpu().numpy(),
                    top_k=t.sampling_top_ks[:B].cpu().numpy(), top_p=t.sampling_top_ps[:B].cpu().numpy(),
                    min_p=t.sampling_min_ps[:B].cpu().numpy(), seed=t.sampling_seeds[:B].cpu().numpy(),
                    max_top_k=t.max_top_k)
    p = r.predictor
    sub = dict(temperature=p.sub_temperature_tensor[:B].cpu().numpy(), top_k=p.sub_top_k_tensor[:B].cpu().numpy(),
               top_p=p.sub_top_p_tensor[:B].cpu().numpy(), seed=p.sub_sampling_seed_tensor[:B].cpu().numpy(),
               do_sample=p.sub_do_sample_tensor[:B].cpu().numpy(), max_top_k=p.sub_sampled_max_top_k,
               has_top_p=p.sub_sampled_has_top_p)

    r.step(use_graph=use_graph)
    torch.cuda.synchronize()

    # ---- packing: bit-exact ----
    sl, r2t1, loc, pos, _, _, pgp, pgi, head1 = orc.decode_prepare(seq0, np.arange(B), r2t0, cfg.page_size, free,
                                                                   free_head=head0)
    assert r.seq_lens[:B].cpu().numpy().tolist() == sl.tolist()
    assert r.out_cache_loc[:B].cpu().numpy().tolist() == loc.tolist()
    assert r.positions[:B].cpu().numpy().tolist() == pos.tolist()
    assert r.page_indptr[: B + 1].cpu().numpy().tolist() == pgp.tolist()
    assert r.page_indices[: pgp[-1]].cpu().numpy().tolist() == pgi.tolist()
    assert np.array_equal(r.r2t.req_to_token[:B].cpu().numpy(), r2t1)
    assert int(r.allocator.free_head.item()) == head1

    # ---- talker: bf16 tolerance ----
    o = OracleTalker(cfg, r.w, r.predictor.w)
    logits_o, hidden_o = o.talker_forward(feedback, text, torch.from_numpy(pos), torch.from_numpy(loc),
                                          torch.from_numpy(sl), torch.from_numpy(r2t1), kpool, vpool)
    figures = {}
    cos, err, scale = cos_err(t.hidden[:B], hidden_o)
    q999 = err_quantile(t.hidden[:B], hidden_o)
    figures["hidden"] = (cos, err, scale, q999)
    assert cos >= 0.999 and err <= tol * max(scale, 1.0) + depth_ulps * bf16_ulp(scale), (cos, err, scale, q999)
    assert q999 <= tol * max(scale, 1.0), (cos, err, scale, q999)
    cos, err, scale = cos_err(t.logits[:B], logits_o)
    q999 = err_quantile(t.logits[:B], logits_o)
    figures["logits"] = (cos, err, scale, q999)
    assert cos >= 0.999 and err <= tol * max(scale, 1.0) + depth_ulps * bf16_ulp(scale), (cos, err, scale, q999)
    assert q999 <= tol * max(scale, 1.0), (cos, err, scale, q999)
    # K/V written at the new slots
    kdev = r.kv.k_buffer[:, torch.from_numpy(loc).to(DEV)].float().cpu()
    cos, err, scale = cos_err(kdev, kpool[:, torch.from_numpy(loc)])
    assert cos >= 0.999, cos

    # ---- layer-0 draw: bit-exact given the device logits ----
    l0_state["positions"] = pos
    c0 = t.sampled_token_ids[:B].cpu()
    assert o.layer0(t.logits[:B].cpu(), l0_state).tolist() == c0.tolist()
    # the drawn token is marked in the repetition mask
    assert t.repetition_mask[torch.arange(B, device=DEV), c0.to(DEV)].all()

    # ---- predictor: teacher-forced logits within tolerance, draws bit-exact ----
    codes = p.output_codes[:B].cpu().numpy()
    assert codes[:, 0].tolist() == c0.tolist()
    codes_o, summed_o, logits_po = o.code_predictor(c0, t.hidden[:B].cpu(), torch.from_numpy(pos), sub,
                                                    forced_codes=codes)
    G = cfg.predictor.num_code_groups
    for j in range(G - 1):
        lg = p.codebook_logits(j, B)
        cos, err, scale = cos_err(lg, logits_po[j])
        figures[f"predictor_logits_{j}"] = (cos, err, scale)
        # these logits are stored in bf16: on top of the 2e-2 tolerance, one rounding
        # of the output may land on the neighbouring bf16 value (one ulp at the scale)
        ulp = 2.0 ** (np.floor(np.log2(max(scale, 1.0))) - 7)
        assert cos >= 0.999 and err <= tol * max(scale, 1.0) + ulp, (j, cos, err, scale)
        drawn = orc.sample_topk_topp(bits(lg), sub["temperature"], sub["top_k"], sub["top_p"], sub["seed"],
                                     pos * (G - 1) + (j + 1), max_top_k=sub["max_top_k"], has_top_p=sub["has_top_p"])
        am = np.argmax(lg.float().cpu().numpy(), axis=1)
        want = np.where(sub["do_sample"].astype(bool), drawn, am)
        assert codes[:, j + 1].tolist() == want.tolist(), j
    assert np.array_equal(bits(p.output_embeds[:B]), summed_o)
    return figures
