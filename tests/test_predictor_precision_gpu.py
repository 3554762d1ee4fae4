"""The fused predictor layers track fp32 like the plain bf16 path does: the reference's
precision rule (test_predictor_kernels.py:312-340) restated.

Over a predictor sequence (the opening two-token pass, then one-token passes at slots
2, 3, 4, 5) the GPU path's relative distance to an fp32 computation of the same layers
stays within 1.25 x the plain path's distance + 1e-4 at every pass, in the final-normed
output and in the K cache.  The plain path is the oracle's restatement of the
reference's eager bf16 path (fp32 arithmetic, bf16 at each storage point); the fp32
computation is the same code with those rounding points removed.  The GPU path folds the
norms into the GEMMs, sums in its own order and rounds at the same storage points: the
rule says that none of that may cost precision.
"""

from __future__ import annotations

import dataclasses

import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _rel(a: torch.Tensor, ref: torch.Tensor) -> float:
    return ((a.float() - ref).norm() / ref.norm()).item()


@pytest.mark.parametrize("batch", [1, 3, 12, 64])
def test_fused_predictor_tracks_fp32_like_the_plain_path(batch):
    import oracle.model as om
    from omni_b200.config import CONFIG0_PREDICTOR, TalkerConfig
    from omni_b200.predictor import CodePredictor, init_predictor_weights

    dev = torch.device(DEV)
    pc = dataclasses.replace(CONFIG0_PREDICTOR, num_hidden_layers=3)
    cfg = TalkerConfig(num_hidden_layers=1, predictor=pc)
    H, S, L = pc.hidden_size, pc.cache_len, pc.num_hidden_layers
    hkv, D = pc.num_key_value_heads, pc.head_dim
    w = init_predictor_weights(pc, seed=3 + batch, device=dev)
    emb0 = torch.zeros(16, H, dtype=torch.bfloat16, device=dev)
    gpu = CodePredictor(pc, w, max_batch=batch, device=dev, layer0_embedding=emb0)
    oracle = om.OracleTalker(cfg, {"layers": []}, w)
    g = torch.Generator(device=dev).manual_seed(4 + batch)
    steps = [torch.randn(batch * 2, H, generator=g, device=dev).to(torch.bfloat16)]
    steps += [torch.randn(batch, H, generator=g, device=dev).to(torch.bfloat16) for _ in range(4)]

    plain_k = torch.zeros(L, batch, S, hkv, D)
    plain_v = torch.zeros_like(plain_k)
    ref_k = torch.zeros_like(plain_k)
    ref_v = torch.zeros_like(plain_k)
    norm = w["norm"].float().cpu()
    cache_len = 0
    rb = om.rb
    for x in steps:
        tokens = x.shape[0] // batch
        h = gpu.forward_tokens(x, x.float().pow(2).sum(-1).contiguous(), batch=batch, tokens=tokens,
                               cache_len=cache_len)
        torch.cuda.synchronize()
        fused = rb(om.rmsnorm(h.float().cpu(), norm, pc.rms_norm_eps))
        xc = x.float().cpu()
        plain = oracle.predictor_tokens(xc, plain_k, plain_v, batch=batch, tokens=tokens, cache_len=cache_len)
        try:
            om.rb = lambda t: t  # the same layers in fp32: no bf16 storage points
            expected = oracle.predictor_tokens(xc, ref_k, ref_v, batch=batch, tokens=tokens, cache_len=cache_len)
        finally:
            om.rb = rb
        e_plain, e_fused = _rel(plain, expected), _rel(fused, expected)
        assert e_fused <= 1.25 * e_plain + 1e-4, (cache_len, e_plain, e_fused)
        cache_len += tokens
    gk = gpu.k_cache.float().cpu().view(L, batch, S, hkv, D)[:, :, :cache_len]
    assert _rel(gk, ref_k[:, :, :cache_len]) <= 1.25 * _rel(plain_k[:, :, :cache_len], ref_k[:, :, :cache_len])
