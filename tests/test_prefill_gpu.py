"""Extend (prefill) path of the mixed batch on the GPU.

- extend packing (slots, positions, cu_seqlens, page lists, q tiles): bit-exact
  against the oracle;
- causal extend attention over the paged pool (pages randomly permuted, streams
  with and without a prefix, lengths around the 128-query tile, the 128-key tile and
  16-token page edges) against a torch fp32 reference: cosine >= 0.999, max-abs <= 2e-2
  x scale; both kernels (two query heads of a KV head a CTA when the group size is
  even, one head otherwise).
"""

from __future__ import annotations

import math

import numpy as np
import pytest
import torch

from oracle import sampler as orc

pytestmark = pytest.mark.gpu
DEV = "cuda"
P = 16


def _reserve(streams, max_ctx, seed):
    """Scheduler-side reservation: every stream's prefix + extend tokens on permuted pages."""
    rng = np.random.default_rng(seed)
    need = [math.ceil((pre + ext) / P) for pre, ext in streams]
    num_pages = sum(need) + 8
    perm = rng.permutation(num_pages).astype(np.int32)
    r2t = np.zeros((len(streams) + 2, max_ctx), np.int32)
    req = rng.permutation(len(streams) + 2)[: len(streams)].astype(np.int64)
    off = 0
    for i, (pre, ext) in enumerate(streams):
        L = pre + ext
        pages = perm[off: off + need[i]]
        off += need[i]
        slots = (pages[:, None] * P + np.arange(P)[None, :]).reshape(-1)[:L]
        r2t[req[i], :L] = slots
    return r2t, req, num_pages


def _pack(streams, r2t, req):
    pre = torch.tensor([s[0] for s in streams], dtype=torch.long, device=DEV)
    ext = torch.tensor([s[1] for s in streams], dtype=torch.long, device=DEV)
    rows = len(streams)
    total = int(ext.sum())
    out = dict(seq_lens=torch.zeros(rows, dtype=torch.long, device=DEV),
               qo_indptr=torch.zeros(rows + 1, dtype=torch.int32, device=DEV),
               out_cache_loc=torch.zeros(total, dtype=torch.long, device=DEV),
               positions=torch.zeros(total, dtype=torch.long, device=DEV),
               page_indptr=torch.zeros(rows + 1, dtype=torch.int32, device=DEV),
               page_indices=torch.zeros(sum(math.ceil(sum(s) / P) for s in streams) + 1, dtype=torch.int32,
                                        device=DEV),
               tile_indptr=torch.zeros(rows + 1, dtype=torch.int32, device=DEV))
    from omni_b200 import ops

    ops.extend_prepare(prefix_lens=pre, extend_lens=ext, req_pool_indices=torch.from_numpy(req).to(DEV),
                       req_to_token=torch.from_numpy(r2t).to(DEV), page_size=P, **out)
    return out


STREAMS = [(0, 1), (0, 63), (0, 64), (0, 65), (0, 127), (0, 128), (0, 129), (0, 200), (37, 50), (5, 1),
           (16, 16), (100, 300), (250, 7)]


def test_extend_prepare_matches_oracle():
    r2t, req, _ = _reserve(STREAMS, 512, 0)
    got = _pack(STREAMS, r2t, req)
    torch.cuda.synchronize()
    sl, qo, loc, pos, pgp, pgi, tp = orc.extend_prepare([s[0] for s in STREAMS], [s[1] for s in STREAMS], req, r2t, P)
    assert got["seq_lens"].cpu().numpy().tolist() == sl.tolist()
    assert got["qo_indptr"].cpu().numpy().tolist() == qo.tolist()
    assert got["out_cache_loc"].cpu().numpy().tolist() == loc.tolist()
    assert got["positions"].cpu().numpy().tolist() == pos.tolist()
    assert got["page_indptr"].cpu().numpy().tolist() == pgp.tolist()
    assert got["page_indices"].cpu().numpy()[: len(pgi)].tolist() == pgi.tolist()
    assert got["tile_indptr"].cpu().numpy().tolist() == tp.tolist()


# config 2's prompt lengths reach 4096: the key-tile ring wraps many times
LONG_STREAMS = [(0, 4096), (0, 2048), (0, 3001), (300, 2500), (0, 64), (4000, 96)]


@pytest.mark.parametrize("hq,hkv,streams,spike", [(16, 2, STREAMS, False), (8, 4, STREAMS, False),
                                                   (12, 4, STREAMS, False), (8, 8, STREAMS, False),
                                                   (16, 2, LONG_STREAMS, False), (16, 2, LONG_STREAMS, True),
                                                   (12, 4, LONG_STREAMS, True)],
                         ids=["gqa8-pairs", "gqa2-pairs", "gqa3-single", "mha-single", "long-prompts",
                              "rescale-split-pairs", "rescale-split-single"])
def test_prefill_attention_matches_fp32(hq, hkv, streams, spike):
    """spike: the key at position 300 of every stream gets +40 in dimension 0 and every
    query row +-4 there (random sign), so the rows with + see their running max jump by
    about 20 (log2 units, past the 2^8 rescale threshold) at that key while the rows
    beside them in the same warp do not: the rescale runs for part of a warp."""
    from omni_b200 import ops

    STREAMS_ = streams
    D = 128
    r2t, req, num_pages = _reserve(STREAMS_, 8192, 1)
    pk = _pack(STREAMS_, r2t, req)
    g = torch.Generator(device=DEV).manual_seed(3)
    kc = torch.randn(num_pages * P, hkv, D, generator=g, device=DEV).to(torch.bfloat16)
    vc = torch.randn(num_pages * P, hkv, D, generator=g, device=DEV).to(torch.bfloat16)
    total = sum(s[1] for s in STREAMS_)
    q = torch.randn(total, hq * D, generator=g, device=DEV).to(torch.bfloat16)
    if spike:
        sign = torch.randint(0, 2, (total, hq), generator=g, device=DEV).to(torch.bfloat16) * 2 - 1
        q.view(total, hq, D)[:, :, 0] = 4 * sign
        for i, (pre, ext) in enumerate(STREAMS_):
            if pre + ext > 300:
                kc[int(r2t[req[i], 300]), :, 0] = 40.0
    out = torch.full((total, hq * D), float("nan"), device=DEV, dtype=torch.bfloat16)
    max_tiles = sum(math.ceil(s[1] / ops.PREFILL_Q_TILE) for s in STREAMS_)
    scale = 1 / math.sqrt(D)
    ops.prefill_attention(q, kc, vc, qo_indptr=pk["qo_indptr"], seq_lens=pk["seq_lens"],
                          page_indptr=pk["page_indptr"], page_indices=pk["page_indices"],
                          tile_indptr=pk["tile_indptr"], max_tiles=max_tiles + 3, num_q_heads=hq, num_kv_heads=hkv,
                          head_dim=D, page_size=P, sm_scale=scale, out=out)
    torch.cuda.synchronize()
    ref = torch.zeros(total, hq, D)
    qf = q.float().cpu().view(total, hq, D)
    kf, vf = kc.float().cpu(), vc.float().cpu()
    q0 = 0
    for i, (pre, ext) in enumerate(STREAMS_):
        L = pre + ext
        slots = torch.from_numpy(r2t[req[i], :L].astype(np.int64))
        mask = torch.arange(L)[None, :] > (pre + torch.arange(ext))[:, None]
        for h in range(hq):  # one head at a time keeps the [ext, L] scores small
            k = kf[slots, h // (hq // hkv)]  # [L, D]
            v = vf[slots, h // (hq // hkv)]
            s_ = (qf[q0: q0 + ext, h] @ k.t()) * scale
            s_ = s_.masked_fill(mask, float("-inf"))
            ref[q0: q0 + ext, h] = torch.softmax(s_, -1) @ v
        q0 += ext
    got = out.float().cpu().view(total, hq, D)
    assert torch.isfinite(got).all()
    cos = torch.nn.functional.cosine_similarity(got.flatten(), ref.flatten(), dim=0).item()
    err = (got - ref).abs().max().item()
    scale_ = ref.abs().max().item()
    assert cos >= 0.999 and err <= 2e-2 * scale_, (cos, err, scale_)
