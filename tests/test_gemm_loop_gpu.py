"""The persistent tile-loop GEMM (prefill-sized batches, one CTA per SM, two TMEM
accumulators) against the split-K kernel at one split.

Both sum each output's whole K in TMEM in the same k order and apply the same fused
epilogue code, so the loop's epilogues must match bit for bit: store and residual with
the row sums of squares (folded RMSNorm on the way in) and SwiGLU; the store case is also
held to an fp32 reference.  The qkv, fp32 and router epilogues stay on the split-K
kernel at these sizes; their cases check that the auto-planned and the one-split calls
agree.  Row counts leave a partial last row tile; the auto-planned call (splits=0) takes
the loop once the batch has at least one (row tile, feature tile) pair per SM, with
256-row tiles when those are enough for every SM and 128-row tiles otherwise (the edge
cases cover both).
"""

from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _gen(seed):
    return torch.Generator(device=DEV).manual_seed(seed)


def _both(fn):
    a = fn(0)
    b = fn(1)
    torch.cuda.synchronize()
    return a, b


@pytest.mark.parametrize("rows,k,n", [(2500, 1024, 1024), (4133, 3072, 1024), (1000, 2048, 3072)])
def test_loop_store_and_residual_match_split_k(rows, k, n):
    from omni_b200 import ops

    g = _gen(rows + k)
    x = torch.randn(rows, k, generator=g, device=DEV).to(torch.bfloat16)
    w = (torch.randn(n, k, generator=g, device=DEV) * 0.02).to(torch.bfloat16)
    res = torch.randn(rows, n, generator=g, device=DEV).to(torch.bfloat16)
    ss_in = x.float().view(rows, k // 128, 128).pow(2).sum(-1).t().contiguous()

    def store(splits):
        y = torch.empty(rows, n, device=DEV, dtype=torch.bfloat16)
        ops.linear_fused(x, w, y, epilogue=ops.EPI_STORE, ss_in=ss_in, ss_in_parts=k // 128, splits=splits)
        return y

    def resid(splits):
        y = torch.empty(rows, n, device=DEV, dtype=torch.bfloat16)
        ss = torch.full((n // 128, rows), -1.0, device=DEV)
        ops.linear_fused(x, w, y, epilogue=ops.EPI_RESIDUAL, residual=res, ss_out=ss, splits=splits)
        return y, ss

    a, b = _both(store)
    assert torch.equal(a, b)
    rstd = torch.rsqrt(ss_in.sum(0) / k + 1e-6)
    ref = (x.float() @ w.float().t()) * rstd[:, None]
    cos = torch.nn.functional.cosine_similarity(a.float().flatten(), ref.flatten(), dim=0).item()
    assert cos >= 0.9999 and (a.float() - ref).abs().max().item() <= 2e-2 * ref.abs().max().item()
    (ya, sa), (yb, sb) = _both(resid)
    assert torch.equal(ya, yb) and torch.equal(sa, sb)
    torch.testing.assert_close(sa.sum(0), ya.float().pow(2).sum(1), rtol=1e-4, atol=1e-2)


def test_loop_swiglu_matches_split_k():
    from omni_b200 import ops

    rows, k, inter = 3001, 1024, 3072
    g = _gen(5)
    x = torch.randn(rows, k, generator=g, device=DEV).to(torch.bfloat16)
    w = (torch.randn(2 * inter, k, generator=g, device=DEV) * 0.02).to(torch.bfloat16)
    ss_in = x.float().view(rows, 8, 128).pow(2).sum(-1).t().contiguous()

    def run(splits):
        y = torch.empty(rows, inter, device=DEV, dtype=torch.bfloat16)
        ops.linear_fused(x, w, y, epilogue=ops.EPI_SWIGLU, ss_in=ss_in, ss_in_parts=8, splits=splits)
        return y

    a, b = _both(run)
    assert torch.equal(a, b)


def test_loop_qkv_rope_store_matches_split_k():
    from omni_b200 import ops

    rows, k, hq, hkv, D = 2777, 1024, 16, 2, 128
    n = (hq + 2 * hkv) * D
    g = _gen(9)
    x = torch.randn(rows, k, generator=g, device=DEV).to(torch.bfloat16)
    w = (torch.randn(n, k, generator=g, device=DEV) * 0.02).to(torch.bfloat16)
    qn = (1 + 0.1 * torch.randn(D, generator=g, device=DEV)).to(torch.bfloat16)
    kn = (1 + 0.1 * torch.randn(D, generator=g, device=DEV)).to(torch.bfloat16)
    cos_sin = ops.rope_cos_sin_cache(8192, D, 1e6, torch.device(DEV))
    positions = torch.randint(0, 8192, (rows,), generator=g, device=DEV)
    slots = torch.randperm(rows + 100, generator=g, device=DEV)[:rows]
    ss_in = x.float().view(rows, 8, 128).pow(2).sum(-1).t().contiguous()

    def run(splits):
        q = torch.empty(rows, hq * D, device=DEV, dtype=torch.bfloat16)
        kc = torch.zeros(rows + 100, hkv, D, device=DEV, dtype=torch.bfloat16)
        vc = torch.zeros(rows + 100, hkv, D, device=DEV, dtype=torch.bfloat16)
        ops.linear_fused(x, w, q, epilogue=ops.EPI_QKV_ROPE, ss_in=ss_in, ss_in_parts=8, splits=splits,
                         qkv=dict(num_q_heads=hq, num_kv_heads=hkv, head_dim=D, q_norm=qn, k_norm=kn, eps=1e-6,
                                  cos_sin=cos_sin, positions=positions, cache_loc=slots, k_cache=kc, v_cache=vc))
        return q, kc, vc

    (qa, ka, va), (qb, kb, vb) = _both(run)
    assert torch.equal(qa, qb) and torch.equal(ka, kb) and torch.equal(va, vb)


def test_loop_f32_and_router_match_split_k():
    from omni_b200 import ops

    g = _gen(11)
    rows, k = 19000, 1024
    x = torch.randn(rows, k, generator=g, device=DEV).to(torch.bfloat16)
    w = (torch.randn(128, k, generator=g, device=DEV) * 0.05).to(torch.bfloat16)

    def f32(splits):
        y = torch.empty(rows, 128, device=DEV, dtype=torch.float32)
        ops.linear_fused(x, w, y, epilogue=ops.EPI_F32, splits=splits)
        return y

    def router(splits):
        y = torch.empty(rows, 128, device=DEV, dtype=torch.bfloat16)
        ids = torch.full((rows, 8), -1, device=DEV, dtype=torch.int32)
        tw = torch.zeros(rows, 8, device=DEV, dtype=torch.float32)
        ops.linear_fused(x, w, y, epilogue=ops.EPI_ROUTER, splits=splits,
                         router={"topk_ids": ids, "topk_weights": tw})
        return y, ids, tw

    a, b = _both(f32)
    assert torch.equal(a, b)
    (ya, ia, wa), (yb, ib, wb) = _both(router)
    assert torch.equal(ya, yb) and torch.equal(ia, ib) and torch.equal(wa, wb)
    from omni_b200 import device_status

    assert device_status() == 0


def test_qkv_as_store_then_qknorm_pass_equals_fused_epilogue():
    """The mixed step's prompt-sized path (plain GEMM into raw qkv rows, then the q/k head
    norms, rotary and K/V store as their own pass) writes the same bits as the fused qkv
    epilogue: both round the projection to bf16, sum the head's squares in the same order
    and round the normed and rotated values at the same points."""
    from omni_b200 import ops

    rows, k, hq, hkv, D = 1500, 1024, 16, 2, 128
    n = (hq + 2 * hkv) * D
    g = _gen(21)
    x = torch.randn(rows, k, generator=g, device=DEV).to(torch.bfloat16)
    w = (torch.randn(n, k, generator=g, device=DEV) * 0.02).to(torch.bfloat16)
    qn = (1 + 0.1 * torch.randn(D, generator=g, device=DEV)).to(torch.bfloat16)
    kn = (1 + 0.1 * torch.randn(D, generator=g, device=DEV)).to(torch.bfloat16)
    cos_sin = ops.rope_cos_sin_cache(8192, D, 1e6, torch.device(DEV))
    positions = torch.randint(0, 8192, (rows,), generator=g, device=DEV)
    slots = torch.randperm(rows + 64, generator=g, device=DEV)[:rows]
    ss_in = x.float().view(rows, 8, 128).pow(2).sum(-1).t().contiguous()

    def caches():
        return (torch.zeros(rows + 64, hkv, D, device=DEV, dtype=torch.bfloat16),
                torch.zeros(rows + 64, hkv, D, device=DEV, dtype=torch.bfloat16))

    q1 = torch.empty(rows, hq * D, device=DEV, dtype=torch.bfloat16)
    k1, v1 = caches()
    ops.linear_fused(x, w, q1, epilogue=ops.EPI_QKV_ROPE, ss_in=ss_in, ss_in_parts=8,
                     qkv=dict(num_q_heads=hq, num_kv_heads=hkv, head_dim=D, q_norm=qn, k_norm=kn, eps=1e-6,
                              cos_sin=cos_sin, positions=positions, cache_loc=slots, k_cache=k1, v_cache=v1))
    raw = torch.empty(rows, n, device=DEV, dtype=torch.bfloat16)
    ops.linear_fused(x, w, raw, epilogue=ops.EPI_STORE, ss_in=ss_in, ss_in_parts=8)
    q2 = torch.empty(rows, hq * D, device=DEV, dtype=torch.bfloat16)
    k2, v2 = caches()
    ops.qknorm_rope_store(raw, num_q_heads=hq, num_kv_heads=hkv, head_dim=D, q_norm=qn, k_norm=kn, eps=1e-6,
                          cos_sin=cos_sin, q_out=q2, k_cache=k2, v_cache=v2, positions=positions, cache_loc=slots)
    torch.cuda.synchronize()
    assert torch.equal(q1, q2) and torch.equal(k1, k2) and torch.equal(v1, v2)


@pytest.mark.parametrize("rows,k,n,epi", [
    (2369, 64, 1024, "store"),       # 128-row tiles: one k-step; the last row tile holds one row
    (18945, 128, 128, "residual"),   # 128-row tiles: one feature tile, 149 row tiles
    (9473, 256, 256, "swiglu"),      # 128-row tiles: two SwiGLU output tiles of 64
    (2433, 1024, 1024, "residual"),  # 128-row tiles: 152 tiles, barely more than one per SM
    (4609, 64, 1024, "store"),       # 256-row tiles: 152 tiles, the last holding one row
    (5000, 3072, 1024, "residual"),  # 256-row tiles: a partial last tile of 136 rows
])
def test_loop_edges_match_split_k(rows, k, n, epi):
    from omni_b200 import ops

    g = _gen(rows + k + n)
    x = torch.randn(rows, k, generator=g, device=DEV).to(torch.bfloat16)
    w = (torch.randn(n, k, generator=g, device=DEV) * 0.05).to(torch.bfloat16)
    res = torch.randn(rows, n, generator=g, device=DEV).to(torch.bfloat16)
    code = {"store": ops.EPI_STORE, "residual": ops.EPI_RESIDUAL, "swiglu": ops.EPI_SWIGLU}[epi]
    width = n // 2 if epi == "swiglu" else n

    def run(splits):
        y = torch.full((rows, width), float("nan"), device=DEV, dtype=torch.bfloat16)
        ss = torch.full((max(n // 128, 1), rows), -1.0, device=DEV) if epi == "residual" else None
        ops.linear_fused(x, w, y, epilogue=code, residual=res if epi == "residual" else None, ss_out=ss,
                         splits=splits)
        return y, ss

    (ya, sa), (yb, sb) = _both(run)
    assert torch.isfinite(ya.float()).all()
    assert torch.equal(ya, yb)
    if sa is not None:
        assert torch.equal(sa, sb)
