"""GPU numerics of the talker-layer kernels against plain PyTorch fp32 references,
and bit-exact parity of the packing kernels against the CPU oracle.

Tolerances (bf16 outputs): cosine >= 0.9999 and max-abs <= 1e-2 x max|ref| for
projections, norms and attention; integer outputs exactly equal.
"""

from __future__ import annotations

import math

import numpy as np
import pytest
import torch

from oracle import sampler as orc

pytestmark = pytest.mark.gpu

DEV = "cuda"


def close(got: torch.Tensor, ref: torch.Tensor, rel: float = 1e-2, cos_min: float = 0.9999):
    g = got.float().flatten()
    r = ref.float().flatten()
    assert torch.isfinite(g).all()
    cos = torch.nn.functional.cosine_similarity(g, r, dim=0).item()
    err = (g - r).abs().max().item()
    scale = r.abs().max().item()
    assert cos >= cos_min and err <= rel * scale + 1e-6, f"cos={cos:.6f} err={err:.4g} scale={scale:.4g}"


# ---------------------------------------------------------------------------
# tcgen05 GEMM
# ---------------------------------------------------------------------------
GEMM_CASES = [
    (64, 1024, 2560, 0),
    (64, 2048, 1024, 1),
    (64, 1024, 6144, 2),
    (64, 3072, 1024, 1),
    (64, 1024, 3072, 3),
    (128, 1024, 2048, 0),
    (1, 1024, 1024, 0),
    (17, 1024, 128, 1),
    (256, 1024, 1024, 2),
    (300, 1024, 1024, 0),
    (600, 256, 384, 3),
]


@pytest.mark.parametrize("rows,k,n,epi", GEMM_CASES)
@pytest.mark.parametrize("splits", [0, 1, 3, 16])
def test_linear_matches_fp32(rows, k, n, epi, splits):
    from omni_b200 import ops

    g = torch.Generator(device=DEV).manual_seed(rows * 7 + k + n + epi)
    x = torch.randn(rows, k, device=DEV, generator=g).to(torch.bfloat16)
    w = (torch.randn(n, k, device=DEV, generator=g) * 0.02).to(torch.bfloat16)
    res = torch.randn(rows, n, device=DEV, generator=g).to(torch.bfloat16) if epi == 1 else None
    out = ops.linear(x, w, epilogue=epi, residual=res, splits=splits)
    ref = x.float() @ w.float().t()
    if epi == 1:
        ref = ref + res.float()
    if epi == 2:
        gate, up = ref[:, : n // 2].bfloat16().float(), ref[:, n // 2:].bfloat16().float()
        ref = torch.nn.functional.silu(gate) * up
    torch.cuda.synchronize()
    close(out, ref)


def test_linear_residual_in_place_and_repeatable():
    from omni_b200 import ops

    rows, k, n = 64, 2048, 1024
    x = torch.randn(rows, k, device=DEV).to(torch.bfloat16)
    w = (torch.randn(n, k, device=DEV) * 0.02).to(torch.bfloat16)
    res = torch.randn(rows, n, device=DEV).to(torch.bfloat16)
    ref = x.float() @ w.float().t() + res.float()
    ws = torch.zeros(ops.linear_workspace_bytes(rows, k, n, 1), dtype=torch.uint8, device=DEV)
    y = res.clone()
    ops.linear(x, w, epilogue=1, residual=y, out=y, workspace=ws)
    close(y, ref)
    # split-K counters are restored: a second launch on the same workspace gives identical bits
    y2 = res.clone()
    ops.linear(x, w, epilogue=1, residual=y2, out=y2, workspace=ws)
    assert torch.equal(y, y2)


# ---------------------------------------------------------------------------
# norms and rotary
# ---------------------------------------------------------------------------
def ref_rmsnorm(x, w, eps):
    x = x.float()
    return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps) * w.float()


@pytest.mark.parametrize("rows", [1, 7, 64, 130])
def test_rmsnorm_and_add_rmsnorm(rows):
    from omni_b200 import ops

    h = 1024
    x = torch.randn(rows, h, device=DEV).to(torch.bfloat16)
    r = torch.randn(rows, h, device=DEV).to(torch.bfloat16)
    w = (1 + 0.1 * torch.randn(h, device=DEV)).to(torch.bfloat16)
    close(ops.rmsnorm(x, w, 1e-6), ref_rmsnorm(x, w, 1e-6))
    res_out = torch.empty_like(r)
    out = ops.rmsnorm(x, w, 1e-6, addend=r, residual_out=res_out)
    s = (x.float() + r.float()).bfloat16()
    assert torch.equal(res_out, s)
    close(out, ref_rmsnorm(s, w, 1e-6))


def ref_qknorm_rope(qkv, hq, hkv, d, qn, kn, eps, cos_sin, pos):
    rows = qkv.shape[0]
    q = qkv[:, : hq * d].float().view(rows, hq, d)
    k = qkv[:, hq * d: (hq + hkv) * d].float().view(rows, hkv, d)
    v = qkv[:, (hq + hkv) * d:].view(rows, hkv, d)

    def norm(t, w):
        return (t * torch.rsqrt(t.pow(2).mean(-1, keepdim=True) + eps) * w.float()).bfloat16().float()

    q, k = norm(q, qn), norm(k, kn)
    cs = cos_sin[pos]
    cos, sin = cs[:, None, : d // 2], cs[:, None, d // 2:]

    def rot(t):
        a, b = t[..., : d // 2], t[..., d // 2:]
        return torch.cat([a * cos - b * sin, b * cos + a * sin], -1)

    return rot(q), rot(k), v


@pytest.mark.parametrize("hq,hkv,d", [(16, 2, 128), (16, 8, 64)])
def test_qknorm_rope_store_paged(hq, hkv, d):
    from omni_b200 import ops

    rows, slots = 37, 512
    qkv = torch.randn(rows, (hq + 2 * hkv) * d, device=DEV).to(torch.bfloat16)
    qn = (1 + 0.1 * torch.randn(d, device=DEV)).to(torch.bfloat16)
    kn = (1 + 0.1 * torch.randn(d, device=DEV)).to(torch.bfloat16)
    cos_sin = ops.rope_cos_sin_cache(8192, d, 1e6, DEV)
    pos = torch.randint(0, 8192, (rows,), device=DEV)
    loc = torch.randperm(slots, device=DEV)[:rows]
    q_out = torch.empty(rows, hq * d, device=DEV, dtype=torch.bfloat16)
    kc = torch.zeros(slots, hkv, d, device=DEV, dtype=torch.bfloat16)
    vc = torch.zeros_like(kc)
    ops.qknorm_rope_store(qkv, num_q_heads=hq, num_kv_heads=hkv, head_dim=d, q_norm=qn, k_norm=kn, eps=1e-6,
                          cos_sin=cos_sin, q_out=q_out, k_cache=kc, v_cache=vc, positions=pos, cache_loc=loc)
    rq, rk, rv = ref_qknorm_rope(qkv, hq, hkv, d, qn, kn, 1e-6, cos_sin, pos)
    close(q_out.view(rows, hq, d), rq)
    close(kc[loc], rk)
    assert torch.equal(vc[loc], rv)
    untouched = torch.ones(slots, dtype=torch.bool, device=DEV)
    untouched[loc] = False
    assert (kc[untouched] == 0).all()


def test_qknorm_rope_store_predictor_slots():
    from omni_b200 import ops

    hq, hkv, d, G1, B = 16, 8, 64, 17, 5
    qkv = torch.randn(2 * B, (hq + 2 * hkv) * d, device=DEV).to(torch.bfloat16)
    qn = torch.ones(d, device=DEV, dtype=torch.bfloat16)
    kn = torch.ones(d, device=DEV, dtype=torch.bfloat16)
    cos_sin = ops.rope_cos_sin_cache(G1, d, 1e6, DEV)
    q_out = torch.empty(2 * B, hq * d, device=DEV, dtype=torch.bfloat16)
    kc = torch.zeros(B * G1, hkv, d, device=DEV, dtype=torch.bfloat16)
    vc = torch.zeros_like(kc)
    ops.qknorm_rope_store(qkv, num_q_heads=hq, num_kv_heads=hkv, head_dim=d, q_norm=qn, k_norm=kn, eps=1e-6,
                          cos_sin=cos_sin, q_out=q_out, k_cache=kc, v_cache=vc, tokens_per_req=2, slot_stride=G1,
                          slot_base=0)
    pos = torch.arange(2, device=DEV).repeat(B)
    slots = torch.arange(B, device=DEV).repeat_interleave(2) * G1 + pos
    rq, rk, rv = ref_qknorm_rope(qkv, hq, hkv, d, qn, kn, 1e-6, cos_sin, pos)
    close(kc[slots], rk)
    assert torch.equal(vc[slots], rv)


# ---------------------------------------------------------------------------
# attention
# ---------------------------------------------------------------------------
def build_paged(seq_lens, hkv, d, page, gen):
    npages = [(L + page - 1) // page for L in seq_lens]
    total = sum(npages)
    pool_pages = int(total * 1.25) + 4
    perm = torch.randperm(pool_pages, generator=gen)[:total]
    page_ids, off = [], 0
    for n in npages:
        page_ids.append(perm[off: off + n])
        off += n
    kc = torch.randn(pool_pages * page, hkv, d, generator=gen).to(torch.bfloat16)
    vc = torch.randn(pool_pages * page, hkv, d, generator=gen).to(torch.bfloat16)
    return page_ids, kc, vc


@pytest.mark.parametrize("lens", [[1, 15, 16, 17, 100, 1000, 8192, 33], [556] * 64, [16] * 3])
@pytest.mark.parametrize("ppc", [1, 8])
def test_paged_decode_attention(lens, ppc):
    from omni_b200 import ops

    gen = torch.Generator().manual_seed(len(lens) + ppc)
    hq, hkv, d, page = 16, 2, 128, 16
    page_ids, kc, vc = build_paged(lens, hkv, d, page, gen)
    rows = len(lens)
    q = torch.randn(rows, hq, d, generator=gen).to(torch.bfloat16)
    page_indptr = torch.tensor(np.concatenate([[0], np.cumsum([len(p) for p in page_ids])]), dtype=torch.int32)
    page_indices = torch.cat(page_ids).to(torch.int32)
    nwork = [(len(p) + ppc - 1) // ppc for p in page_ids]
    work_indptr = torch.tensor(np.concatenate([[0], np.cumsum(nwork)]), dtype=torch.int32)
    cap = int(work_indptr[-1])
    ws = torch.zeros(ops.paged_attention_workspace_bytes(rows, hkv, cap), dtype=torch.uint8, device=DEV)
    out = torch.empty(rows, hq, d, device=DEV, dtype=torch.bfloat16)
    scale = 1 / math.sqrt(d)
    seq = torch.tensor(lens, dtype=torch.int64)
    for rep in range(2):  # second launch reuses the restored merge counters
        ops.paged_decode_attention(q.to(DEV), kc.to(DEV), vc.to(DEV), page_indptr=page_indptr.to(DEV),
                                   page_indices=page_indices.to(DEV), seq_lens=seq.to(DEV),
                                   work_indptr=work_indptr.to(DEV), num_q_heads=hq, num_kv_heads=hkv, head_dim=d,
                                   page_size=page, pages_per_chunk=ppc, work_capacity=cap, sm_scale=scale, out=out,
                                   workspace=ws)
        torch.cuda.synchronize()
        for b, L in enumerate(lens):
            slots = (page_ids[b][:, None] * page + torch.arange(page)[None, :]).reshape(-1)[:L]
            k = kc[slots].float()  # [L, hkv, d]
            v = vc[slots].float()
            qb = q[b].float().view(hkv, hq // hkv, d)
            s = torch.einsum("hgd,lhd->hgl", qb, k) * scale
            p = torch.softmax(s, -1)
            ref = torch.einsum("hgl,lhd->hgd", p, v).reshape(hq, d)
            close(out[b].cpu(), ref, rel=2e-2, cos_min=0.999)


@pytest.mark.parametrize("hq,hkv,d", [(16, 8, 64), (8, 8, 128), (16, 4, 128)])
@pytest.mark.parametrize("tokens,base", [(2, 0), (1, 5), (1, 15)])
def test_predictor_attention(tokens, base, hq, hkv, d):
    from omni_b200 import ops

    G1, B = 17, 6
    rows = B * tokens
    q = torch.randn(rows, hq * d, device=DEV).to(torch.bfloat16)
    kc = torch.randn(B * G1, hkv, d, device=DEV).to(torch.bfloat16)
    vc = torch.randn(B * G1, hkv, d, device=DEV).to(torch.bfloat16)
    out = torch.empty(rows, hq * d, device=DEV, dtype=torch.bfloat16)
    ops.predictor_attention(q, kc, vc, num_q_heads=hq, num_kv_heads=hkv, head_dim=d, tokens_per_req=tokens,
                            slot_stride=G1, slot_base=base, sm_scale=1 / math.sqrt(d), out=out)
    qr = q.float().view(B, tokens, hq, d).transpose(1, 2)
    k = kc.float().view(B, G1, hkv, d)[:, : base + tokens].transpose(1, 2).repeat_interleave(hq // hkv, 1)
    v = vc.float().view(B, G1, hkv, d)[:, : base + tokens].transpose(1, 2).repeat_interleave(hq // hkv, 1)
    s = qr @ k.transpose(-1, -2) / math.sqrt(d)
    mask = torch.arange(base + tokens, device=DEV)[None, :] > (base + torch.arange(tokens, device=DEV))[:, None]
    s = s.masked_fill(mask, float("-inf"))
    ref = (torch.softmax(s, -1) @ v).transpose(1, 2).reshape(rows, hq * d)
    close(out, ref, rel=2e-2, cos_min=0.999)


# ---------------------------------------------------------------------------
# packing (bit-exact against the oracle)
# ---------------------------------------------------------------------------
@pytest.mark.parametrize("rows,page", [(64, 16), (5, 4), (1100, 16)])
def test_decode_prepare_matches_oracle(rows, page):
    from omni_b200 import ops

    rng = np.random.default_rng(rows)
    max_ctx = 256
    lens = rng.integers(1, max_ctx - 1, rows)
    lens[: min(rows, 4)] = [page, 2 * page - 1, 1, page + 1][: min(rows, 4)]
    num_pages = int(sum((lens + page) // page)) + 64
    perm = rng.permutation(num_pages).astype(np.int32)
    r2t = np.zeros((rows + 3, max_ctx), np.int32)
    head = 0
    req = rng.permutation(rows + 3)[:rows].astype(np.int64)
    for i, L in enumerate(lens):
        for t in range(L):
            if t % page == 0:
                pg = perm[head]
                head += 1
            r2t[req[i], t] = pg * page + t % page
    want = orc.decode_prepare(lens, req, r2t, page, perm, free_head=head)
    t = lambda a, dt=None: torch.tensor(a, device=DEV, dtype=dt)  # noqa: E731
    seq = t(lens, torch.int64)
    r2t_d = t(r2t)
    total = int(lens.sum()) + rows
    out_loc = torch.empty(rows, dtype=torch.int64, device=DEV)
    pos = torch.empty(rows, dtype=torch.int64, device=DEV)
    page_indptr = torch.empty(rows + 1, dtype=torch.int32, device=DEV)
    page_indices = torch.empty(total, dtype=torch.int32, device=DEV)
    kv_indptr = torch.empty(rows + 1, dtype=torch.int32, device=DEV)
    kv_indices = torch.empty(total, dtype=torch.int32, device=DEV)
    work_indptr = torch.empty(rows + 1, dtype=torch.int32, device=DEV)
    free_head = t([head], torch.int64)
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    ops.decode_prepare(seq_lens=seq, req_pool_indices=t(req, torch.int64), req_to_token=r2t_d, page_size=page,
                       free_pages=t(perm), free_head=free_head, out_cache_loc=out_loc, positions=pos,
                       page_indptr=page_indptr, page_indices=page_indices, kv_indptr=kv_indptr,
                       kv_indices=kv_indices, work_indptr=work_indptr, pages_per_chunk=8, status=status)
    sl, r2t2, loc, p, kvp, kvi, pgp, pgi, head2 = want
    assert status.item() == 0
    assert seq.cpu().numpy().tolist() == sl.tolist()
    assert np.array_equal(r2t_d.cpu().numpy(), r2t2)
    assert out_loc.cpu().numpy().tolist() == loc.tolist()
    assert pos.cpu().numpy().tolist() == p.tolist()
    assert kv_indptr.cpu().numpy().tolist() == kvp.tolist()
    assert kv_indices[: kvp[-1]].cpu().numpy().tolist() == kvi.tolist()
    assert page_indptr.cpu().numpy().tolist() == pgp.tolist()
    assert page_indices[: pgp[-1]].cpu().numpy().tolist() == pgi.tolist()
    npg = np.diff(pgp)
    assert work_indptr.cpu().numpy().tolist() == np.concatenate([[0], np.cumsum((npg + 7) // 8)]).tolist()
    assert free_head.item() == head2
    # rollback restores the state and frees exactly the opened pages
    freed = torch.empty(rows, dtype=torch.int64, device=DEV)
    nfreed = torch.zeros(1, dtype=torch.int64, device=DEV)
    ops.decode_rollback(seq_lens=seq, req_pool_indices=t(req, torch.int64), req_to_token=r2t_d, page_size=page,
                        out_cache_loc=out_loc, free_head=free_head, freed_slots=freed, num_freed=nfreed)
    sl_o, _, freed_o = orc.decode_rollback(sl, req, r2t2, page, loc)
    assert seq.cpu().numpy().tolist() == sl_o.tolist() == lens.tolist()
    assert freed[: nfreed.item()].cpu().numpy().tolist() == freed_o.tolist()
    assert free_head.item() == head


def test_rollback_known_answer(golden):
    """talker test_talker.py:1118-1134: page 4, seq_lens [5, 7], out_cache_loc [16, 22] frees [16]."""
    from omni_b200 import ops

    g = golden["rollback"]
    seq = torch.tensor(g["seq_lens"], device=DEV)
    r2t = torch.ones(2, 8, dtype=torch.int32, device=DEV)
    free_head = torch.tensor([10], device=DEV)
    freed = torch.empty(2, dtype=torch.int64, device=DEV)
    n = torch.zeros(1, dtype=torch.int64, device=DEV)
    ops.decode_rollback(seq_lens=seq, req_pool_indices=torch.tensor([0, 1], device=DEV), req_to_token=r2t,
                        page_size=4, out_cache_loc=torch.tensor(g["out_cache_loc"], device=DEV),
                        free_head=free_head, freed_slots=freed, num_freed=n)
    assert freed[: n.item()].tolist() == g["freed"][0]
    assert seq.tolist() == g["seq_lens_after"]
    assert r2t.tolist() == g["req_to_token_after"]
    assert free_head.item() == 9


# ---------------------------------------------------------------------------
# fused projections (folded RMSNorm, qkv epilogue, row sums of squares)
# ---------------------------------------------------------------------------
@pytest.mark.parametrize("rows", [1, 64, 128])
def test_linear_fused_folded_norm_and_sumsq(rows):
    from omni_b200 import ops

    H, N = 1024, 3072
    g = torch.Generator(device=DEV).manual_seed(rows)
    x = (torch.randn(rows, H, device=DEV, generator=g) * 3).to(torch.bfloat16)
    res = torch.randn(rows, H, device=DEV, generator=g).to(torch.bfloat16)
    gain = (1 + 0.1 * torch.randn(H, device=DEV, generator=g)).to(torch.bfloat16)
    w = (torch.randn(N, H, device=DEV, generator=g) * 0.02).to(torch.bfloat16)
    wo = (torch.randn(H, N, device=DEV, generator=g) * 0.02).to(torch.bfloat16)
    # input row + its sum of squares
    s = torch.empty_like(x)
    ss1 = torch.empty(rows, device=DEV)
    ops.add_sumsq(x, res, s, ss1)
    ref_s = (x.float() + res.float()).bfloat16()
    assert torch.equal(s, ref_s)
    torch.testing.assert_close(ss1, ref_s.float().pow(2).sum(1), rtol=1e-5, atol=1e-3)
    # folded RMSNorm -> projection
    y = torch.empty(rows, N, device=DEV, dtype=torch.bfloat16)
    ops.linear_fused(s, ops.fold_norm(w, gain), y, epilogue=ops.EPI_STORE, ss_in=ss1, ss_in_parts=1, norm_eps=1e-6)
    ref = ref_rmsnorm(ref_s, gain, 1e-6).bfloat16().float() @ w.float().t()
    close(y, ref, rel=2e-2, cos_min=0.9995)
    # residual epilogue emits per-tile sums of squares of its bf16 output
    a = torch.randn(rows, N, device=DEV, generator=g).to(torch.bfloat16)
    out = s.clone()
    ss8 = torch.zeros(H // 128, rows, device=DEV)
    ops.linear_fused(a, wo, out, epilogue=ops.EPI_RESIDUAL, residual=out, ss_out=ss8)
    close(out, a.float() @ wo.float().t() + s.float())
    torch.testing.assert_close(ss8.sum(0), out.float().pow(2).sum(1), rtol=1e-4, atol=1e-2)
    torch.testing.assert_close(ss8[3], out[:, 384:512].float().pow(2).sum(1), rtol=1e-4, atol=1e-2)
    # SwiGLU with the folded norm and 8-part sums of squares
    wgu = (torch.randn(2 * N, H, device=DEV, generator=g) * 0.02).to(torch.bfloat16)
    act = torch.empty(rows, N, device=DEV, dtype=torch.bfloat16)
    ops.linear_fused(out, ops.fold_norm(wgu, gain), act, epilogue=ops.EPI_SWIGLU, ss_in=ss8, ss_in_parts=8,
                     norm_eps=1e-6)
    gu = ref_rmsnorm(out, gain, 1e-6).bfloat16().float() @ wgu.float().t()
    ref_act = torch.nn.functional.silu(gu[:, :N].bfloat16().float()) * gu[:, N:].bfloat16().float()
    close(act, ref_act, rel=2e-2, cos_min=0.9995)
    # an L2 prefetch of another weight (odd size) leaves the results unchanged
    act2 = torch.empty_like(act)
    ops.linear_fused(out, ops.fold_norm(wgu, gain), act2, epilogue=ops.EPI_SWIGLU, ss_in=ss8, ss_in_parts=8,
                     norm_eps=1e-6, l2_prefetch=wo.view(-1)[: wo.numel() - 24])
    torch.cuda.synchronize()
    assert torch.equal(act2, act)


@pytest.mark.parametrize("hq,hkv,d,implicit", [(16, 2, 128, False), (16, 8, 64, True)])
def test_linear_fused_qkv_rope_store(hq, hkv, d, implicit):
    from omni_b200 import ops

    rows, H = 12, 1024
    g = torch.Generator(device=DEV).manual_seed(d)
    x = (torch.randn(rows, H, device=DEV, generator=g) * 2).to(torch.bfloat16)
    ss = x.float().pow(2).sum(1).contiguous()
    gain = (1 + 0.1 * torch.randn(H, device=DEV, generator=g)).to(torch.bfloat16)
    w = (torch.randn((hq + 2 * hkv) * d, H, device=DEV, generator=g) * 0.02).to(torch.bfloat16)
    qn = (1 + 0.1 * torch.randn(d, device=DEV, generator=g)).to(torch.bfloat16)
    kn = (1 + 0.1 * torch.randn(d, device=DEV, generator=g)).to(torch.bfloat16)
    if implicit:
        G1, T, base = 17, 2, 0
        cos_sin = ops.rope_cos_sin_cache(G1, d, 1e6, DEV)
        pos = torch.arange(T, device=DEV).repeat(rows // T) + base
        loc = torch.arange(rows // T, device=DEV).repeat_interleave(T) * G1 + pos
        slots = (rows // T) * G1
        geo = dict(tokens_per_req=T, slot_stride=G1, slot_base=base)
    else:
        cos_sin = ops.rope_cos_sin_cache(4096, d, 1e6, DEV)
        pos = torch.randint(0, 4096, (rows,), device=DEV)
        slots = 256
        loc = torch.randperm(slots, device=DEV)[:rows]
        geo = dict(positions=pos, cache_loc=loc)
    kc = torch.zeros(slots, hkv, d, device=DEV, dtype=torch.bfloat16)
    vc = torch.zeros_like(kc)
    q = torch.empty(rows, hq * d, device=DEV, dtype=torch.bfloat16)
    ops.linear_fused(x, ops.fold_norm(w, gain), q, epilogue=ops.EPI_QKV_ROPE, ss_in=ss, ss_in_parts=1, norm_eps=1e-6,
                     qkv=dict(num_q_heads=hq, num_kv_heads=hkv, head_dim=d, q_norm=qn, k_norm=kn, eps=1e-6,
                              cos_sin=cos_sin, k_cache=kc, v_cache=vc, **geo))
    qkv_ref = (ref_rmsnorm(x, gain, 1e-6).bfloat16().float() @ w.float().t()).bfloat16()
    rq, rk, rv = ref_qknorm_rope(qkv_ref, hq, hkv, d, qn, kn, 1e-6, cos_sin, pos)
    close(q.view(rows, hq, d), rq, rel=3e-2, cos_min=0.999)
    close(kc[loc], rk, rel=3e-2, cos_min=0.999)
    close(vc[loc], rv, rel=3e-2, cos_min=0.999)
