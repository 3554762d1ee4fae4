"""The reference-shaped Python boundary, called with the reference's own arguments.

- TalkerModel.forward(input_ids, positions, forward_batch, input_embeds=...) in decode
  (Qwen3-TTS and Qwen3-Omni flavors) and in a mixed extend batch against the CPU
  oracle: logits / hidden within the bf16 contract;
- TalkerModel.code_predictor_forward(layer0_codes, talker_hidden, semantic_positions)
  with exactly those three arguments and an already normalized hidden state: every
  draw bit-exact given the device logits, the teacher-forced logits within tolerance,
  the summed embeddings bit-exact;
- add_rmsnorm_rounded(x, residual, weight, eps) in place: the residual bit-exact, x
  within one bf16 step of an fp32 restatement of the reference kernel's arithmetic;
- FusedPredictorLayers.forward(*, layers, final_norm, token_embeds, batch_size,
  cache_len, positions, k_cache, v_cache) over reference-shaped layer modules against
  the oracle's predictor stack, the caches at the written slots included;
- torch.ops.omni_b200.* equal, bit for bit, to the Python drop-ins they wrap.
"""

from __future__ import annotations

import math
from types import SimpleNamespace

import numpy as np
import pytest
import torch

from oracle import sampler as orc
from oracle.model import OracleTalker, bits
from step_util import cos_err

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _runner(flavor, layers=2, lens=(16, 1, 33, 100, 200, 15, 64, 17), seed=0, prompts=()):
    from omni_b200.config import TalkerConfig
    from omni_b200.model_runner import TalkerDecodeRunner

    cfg = TalkerConfig(num_hidden_layers=layers, max_context=1024)
    pages = sum((L + 16) // 16 for L in lens) + sum((L + 15) // 16 for L in prompts) + 32
    r = TalkerDecodeRunner(cfg, max_batch=len(lens) + len(prompts), num_pages=pages, seed=seed, flavor=flavor,
                           max_prefill_tokens=sum(prompts))
    r.admit(list(lens), seed=seed + 5)
    return r


def _sub_state(p, B):
    return dict(temperature=p.sub_temperature_tensor[:B].cpu().numpy(), top_k=p.sub_top_k_tensor[:B].cpu().numpy(),
                top_p=p.sub_top_p_tensor[:B].cpu().numpy(), seed=p.sub_sampling_seed_tensor[:B].cpu().numpy(),
                do_sample=p.sub_do_sample_tensor[:B].cpu().numpy(), max_top_k=p.sub_sampled_max_top_k,
                has_top_p=p.sub_sampled_has_top_p)


def _check_predictor(r, o, c0, hidden, pos, B):
    """The predictor outputs in r against the oracle under teacher forcing."""
    p = r.predictor
    G = r.cfg.predictor.num_code_groups
    sub = _sub_state(p, B)
    codes = p.output_codes[:B].cpu().numpy()
    assert codes[:, 0].tolist() == c0.tolist()
    codes_o, summed_o, logits_po = o.code_predictor(torch.as_tensor(c0), hidden.cpu(), torch.as_tensor(pos), sub,
                                                    forced_codes=codes)
    for j in range(G - 1):
        lg = p.codebook_logits(j, B)
        cos, err, scale = cos_err(lg, logits_po[j])
        ulp = 2.0 ** (np.floor(np.log2(max(scale, 1.0))) - 7)
        assert cos >= 0.999 and err <= 2e-2 * max(scale, 1.0) + ulp, (j, cos, err, scale)
        drawn = orc.sample_topk_topp(bits(lg), sub["temperature"], sub["top_k"], sub["top_p"], sub["seed"],
                                     np.asarray(pos) * (G - 1) + (j + 1), max_top_k=sub["max_top_k"],
                                     has_top_p=sub["has_top_p"])
        am = np.argmax(lg.float().cpu().numpy(), axis=1)
        assert codes[:, j + 1].tolist() == np.where(sub["do_sample"].astype(bool), drawn, am).tolist(), j
    assert np.array_equal(bits(p.output_embeds[:B]), summed_o)


@pytest.mark.parametrize("flavor", ["tts", "omni"])
def test_talker_forward_and_code_predictor_forward_with_reference_arguments(flavor):
    from omni_b200.talker_model import TalkerModel

    r = _runner(flavor)
    model = TalkerModel(r)
    B, cfg = r.batch_size, r.cfg
    g = torch.Generator(device=DEV).manual_seed(3)
    rows = torch.randn(B, cfg.hidden_size, generator=g, device=DEV).to(torch.bfloat16)
    seq0 = r.seq_lens[:B].cpu().numpy()
    r2t0 = r.r2t.req_to_token[:B].cpu().numpy()
    free, head0 = r.allocator.free_pages.cpu().numpy(), int(r.allocator.free_head.item())
    kpool, vpool = r.kv.k_buffer.float().cpu(), r.kv.v_buffer.float().cpu()
    fb = r.build_forward_batch()
    out = model.forward(None, fb.positions, fb, input_embeds=rows)
    torch.cuda.synchronize()
    sl, r2t1, loc, pos, *_ = orc.decode_prepare(seq0, np.arange(B), r2t0, cfg.page_size, free, free_head=head0)
    o = OracleTalker(cfg, r.w, r.predictor.w)
    logits_o, hidden_o = o.talker_forward(rows.cpu(), None, torch.from_numpy(pos), torch.from_numpy(loc),
                                          torch.from_numpy(sl), torch.from_numpy(r2t1), kpool, vpool)
    assert out.next_token_logits.dtype == torch.float32 and out.next_token_logits.shape == (B, cfg.vocab_size)
    for got, want in ((out.next_token_logits, logits_o), (out.hidden_states, hidden_o)):
        cos, err, scale = cos_err(got, want)
        assert cos >= 0.999 and err <= 2e-2 * max(scale, 1.0), (cos, err, scale)
    hidden = out.hidden_states.clone()
    if flavor == "omni":
        # the Omni talker's decode forward draws layer 0 and runs the predictor itself
        c0 = model.sampled_token_ids[:B].cpu().numpy()
        _check_predictor(r, o, c0, hidden, pos, B)
        return
    c0 = model.sample_decode_tokens(out.next_token_logits, fb)
    codes, summed = model.code_predictor_forward(c0.unsqueeze(1), hidden.unsqueeze(1), fb.positions)
    torch.cuda.synchronize()
    assert codes.shape == (B, cfg.predictor.num_code_groups, 1) and summed.shape == (B, 1, cfg.hidden_size)
    _check_predictor(r, o, c0.cpu().numpy(), hidden, pos, B)


def test_talker_forward_mixed_extend_batch():
    from omni_b200.talker_model import ForwardMode, TalkerModel

    lens, prompts = (16, 33, 100), (20, 70)
    r = _runner("tts", lens=lens, prompts=prompts, seed=6)
    g = torch.Generator(device=DEV).manual_seed(8)
    r.admit_prefill(list(prompts), seed=9)
    model = TalkerModel(r)
    B, cfg = r.batch_size, r.cfg
    dec_rows = torch.randn(B, cfg.hidden_size, generator=g, device=DEV).to(torch.bfloat16)
    rows = torch.cat([dec_rows, r.prompt_embeds])
    seq0 = r.seq_lens[:B].cpu().numpy()
    r2t0 = r.r2t.req_to_token.cpu().numpy()
    free, head0 = r.allocator.free_pages.cpu().numpy(), int(r.allocator.free_head.item())
    kpool, vpool = r.kv.k_buffer.float().cpu(), r.kv.v_buffer.float().cpu()
    fb = r.build_forward_batch()
    assert fb.forward_mode is ForwardMode.MIXED and fb.forward_mode.is_extend()
    out = model.forward(None, fb.positions, fb, input_embeds=rows)
    torch.cuda.synchronize()
    sl, r2t1, loc, pos, *_ = orc.decode_prepare(seq0, np.arange(B), r2t0[:B], cfg.page_size, free, free_head=head0)
    ext_pos, ext_loc, ext_ctx = [], [], []
    for i, L in enumerate(prompts):
        slots = torch.from_numpy(r2t0[B + i, :L].astype(np.int64))
        ext_pos += list(range(L))
        ext_loc += slots.tolist()
        ext_ctx += [slots[: j + 1] for j in range(L)]
    o = OracleTalker(cfg, r.w, r.predictor.w)
    select = list(range(B)) + [B + int(x) for x in np.cumsum(prompts) - 1]
    logits_o, hidden_o = o.mixed_forward(dec_rows.cpu(), None, torch.from_numpy(pos), torch.from_numpy(loc),
                                         torch.from_numpy(sl), torch.from_numpy(r2t1), r.prompt_embeds.cpu(),
                                         ext_pos, ext_loc, ext_ctx, torch.tensor(select), kpool, vpool)
    for got, want in ((out.next_token_logits, logits_o), (out.hidden_states, hidden_o)):
        cos, err, scale = cos_err(got, want)
        assert cos >= 0.999 and err <= 2e-2 * max(scale, 1.0), (cos, err, scale)


def _restated_add_rmsnorm(x, r, w, eps):
    """fp32 restatement of the reference kernel (predictor_layers.py:104-142): lanes of 8
    consecutive columns, squares added in column order without fusion, xor butterfly."""
    s = (x.float() + r.float()).to(torch.bfloat16)
    v = s.float().view(x.shape[0], -1, 32, 8)  # [rows, blocks, lane, j]
    acc = torch.zeros(x.shape[0], 32)
    for b in range(v.shape[1]):
        for j in range(8):
            acc = acc + v[:, b, :, j] * v[:, b, :, j]
    for off in (1, 2, 4, 8, 16):
        acc = acc + acc[:, torch.arange(32) ^ off]
    rstd = torch.rsqrt(acc[:, 0] / x.shape[1] + eps)
    return (s.float() * rstd[:, None] * w.float()[None, :]).to(torch.bfloat16), s


def test_add_rmsnorm_rounded_in_place():
    from omni_b200 import torch_ops
    from omni_b200.predictor_layers import add_rmsnorm_rounded

    g = torch.Generator(device=DEV).manual_seed(1)
    for rows in (1, 64, 300):
        x = torch.randn(rows, 1024, generator=g, device=DEV).to(torch.bfloat16)
        res = torch.randn(rows, 1024, generator=g, device=DEV).to(torch.bfloat16)
        w = (1 + 0.1 * torch.randn(1024, generator=g, device=DEV)).to(torch.bfloat16)
        want_x, want_r = _restated_add_rmsnorm(x.cpu(), res.cpu(), w.cpu(), 1e-6)
        x2, r2 = x.clone(), res.clone()
        out_x, out_r = add_rmsnorm_rounded(x, res, w, 1e-6)
        assert out_x.data_ptr() == x.data_ptr() and out_r.data_ptr() == res.data_ptr()
        torch.cuda.synchronize()
        assert torch.equal(res.cpu(), want_r)
        diff = (x.cpu().float() - want_x.float()).abs()
        ulp = want_x.float().abs().clamp(min=1e-30).log2().floor().sub(7).exp2()
        assert bool((diff <= ulp).all()), diff.max().item()
        torch_ops.load()
        torch.ops.omni_b200.add_rmsnorm_rounded(x2, r2, w, 1e-6)
        assert torch.equal(x2, x) and torch.equal(r2, res)


def _layer_modules(pw, cos_sin):
    layers = []
    for lw in pw["layers"]:
        attn = SimpleNamespace(qkv_proj=SimpleNamespace(weight=lw["qkv_proj"]),
                               q_norm=SimpleNamespace(weight=lw["q_norm"], variance_epsilon=1e-6),
                               k_norm=SimpleNamespace(weight=lw["k_norm"], variance_epsilon=1e-6),
                               o_proj=SimpleNamespace(weight=lw["o_proj"]),
                               rotary_emb=SimpleNamespace(cos_sin_cache=cos_sin))
        layers.append(SimpleNamespace(
            input_layernorm=SimpleNamespace(weight=lw["input_layernorm"], variance_epsilon=1e-6),
            self_attn=attn,
            post_attention_layernorm=SimpleNamespace(weight=lw["post_attention_layernorm"], variance_epsilon=1e-6),
            mlp=SimpleNamespace(gate_up_proj=SimpleNamespace(weight=lw["gate_up_proj"]),
                                down_proj=SimpleNamespace(weight=lw["down_proj"]))))
    return layers


def test_fused_predictor_layers_forward_matches_oracle():
    from omni_b200 import ops
    from omni_b200.config import PredictorConfig, TalkerConfig
    from omni_b200.predictor import init_predictor_weights
    from omni_b200.predictor_layers import FusedPredictorLayers, PredictorLayerShape
    from omni_b200.talker import init_talker_weights

    pc = PredictorConfig()
    cfg = TalkerConfig(num_hidden_layers=1, predictor=pc)
    pw = init_predictor_weights(pc, seed=2, device=DEV)
    tw = init_talker_weights(cfg, seed=2, device=DEV)
    o = OracleTalker(cfg, tw, pw)
    shape = PredictorLayerShape(hidden_size=pc.hidden_size, head_dim=pc.head_dim, num_q_heads=pc.num_attention_heads,
                                num_kv_heads=pc.num_key_value_heads, intermediate_size=pc.intermediate_size)
    batch, S = 24, pc.cache_len
    fused = FusedPredictorLayers(shape, max_rows=2 * batch, device=torch.device(DEV))
    layers = _layer_modules(pw, ops.rope_cos_sin_cache(S, pc.head_dim, pc.rope_theta, DEV))
    final_norm = SimpleNamespace(weight=pw["norm"], variance_epsilon=1e-6)
    kc = torch.zeros(pc.num_hidden_layers, batch, S, pc.num_key_value_heads, pc.head_dim, dtype=torch.bfloat16,
                     device=DEV)
    vc = torch.zeros_like(kc)
    kco, vco = kc.float().cpu(), vc.float().cpu()
    g = torch.Generator(device=DEV).manual_seed(4)
    for cache_len, tokens in ((0, 2), (2, 1), (3, 1)):
        x = (torch.randn(batch, tokens, pc.hidden_size, generator=g, device=DEV) * 0.05).to(torch.bfloat16)
        positions = (cache_len + torch.arange(tokens, device=DEV)).repeat(batch)
        got = fused.forward(layers=layers, final_norm=final_norm, token_embeds=x, batch_size=batch,
                            cache_len=cache_len, positions=positions, k_cache=kc, v_cache=vc)
        torch.cuda.synchronize()
        want = o.predictor_tokens(x.float().cpu().reshape(-1, pc.hidden_size), kco, vco, batch=batch, tokens=tokens,
                                  cache_len=cache_len)
        cos, err, scale = cos_err(got.reshape(-1, pc.hidden_size), want)
        assert got.shape == (batch, tokens, pc.hidden_size)
        assert cos >= 0.999 and err <= 2e-2 * max(scale, 1.0), (cache_len, cos, err, scale)
        end = cache_len + tokens
        cos, _, _ = cos_err(kc[:, :, cache_len:end], kco[:, :, cache_len:end])
        assert cos >= 0.999, cos


def test_torch_ops_equal_the_python_drop_ins():
    from omni_b200 import ops, torch_ops
    from omni_b200.predictor_kernels import gather_codec_embedding_and_add
    from omni_b200.predictor_layers import codebook_step
    from omni_b200.sampling_kernels import sample_from_logits_with_seed_top_k_top_p

    torch_ops.load()
    tops = torch.ops.omni_b200
    g = torch.Generator(device=DEV).manual_seed(11)
    rows, vocab, H = 37, 2048, 1024
    logits = torch.randn(rows, vocab, generator=g, device=DEV).mul(3).to(torch.bfloat16)
    temps = torch.full((rows,), 0.9, device=DEV)
    top_ks = torch.randint(1, 51, (rows,), generator=g, device=DEV)
    top_ps = torch.full((rows,), 0.8, device=DEV)
    seeds = torch.randint(0, 2**31 - 1, (rows,), generator=g, device=DEV)
    pos = torch.randint(0, 10_000, (rows,), generator=g, device=DEV)
    a = sample_from_logits_with_seed_top_k_top_p(logits, temps, top_ks, top_ps, seeds, pos, max_top_k=50,
                                                 has_top_p=True)
    b = tops.sample_topk_topp(logits, temps, top_ks, top_ps, seeds, pos, 50, True)
    assert torch.equal(a, b)
    table = (torch.randn(vocab, H, generator=g, device=DEV) * 0.02).to(torch.bfloat16)
    summed0 = torch.randn(rows, H, generator=g, device=DEV).to(torch.bfloat16)
    c1, s1 = torch.zeros(rows, dtype=torch.long, device=DEV), summed0.clone()
    c2, s2 = torch.zeros(rows, dtype=torch.long, device=DEV), summed0.clone()
    n1 = codebook_step(logits, table, c1, s1)
    n2 = tops.codebook_step(logits, table, c2, s2)
    assert torch.equal(c1, c2) and torch.equal(s1, s2) and torch.equal(n1, n2)
    g1, a1 = torch.empty(rows, H, dtype=torch.bfloat16, device=DEV), summed0.clone()
    g2, a2 = torch.empty(rows, H, dtype=torch.bfloat16, device=DEV), summed0.clone()
    assert gather_codec_embedding_and_add(c1, table, g1, a1)
    assert tops.gather_codec_embedding_and_add(c1, table, g2, a2)
    assert torch.equal(g1, g2) and torch.equal(a1, a2)
    x = torch.randn(64, 1024, generator=g, device=DEV).to(torch.bfloat16)
    w = (torch.randn(512, 1024, generator=g, device=DEV) * 0.02).to(torch.bfloat16)
    y1 = ops.linear(x, w)
    y2 = torch.empty_like(y1)
    tops.linear(x, w, y2, ops.EPI_STORE)
    assert torch.equal(y1, y2)
    # paged attention: the op against the ops wrapper on one shared case
    lens = [1, 17, 300, 2000]
    npg = [math.ceil(L / 16) for L in lens]
    perm = torch.randperm(sum(npg) + 4, generator=torch.Generator().manual_seed(0))[: sum(npg)].to(torch.int32)
    kc = torch.randn((sum(npg) + 4) * 16, 2, 128, generator=g, device=DEV).to(torch.bfloat16)
    vc = torch.randn_like(kc)
    q = torch.randn(len(lens), 16, 128, generator=g, device=DEV).to(torch.bfloat16)
    indptr = torch.tensor(np.concatenate([[0], np.cumsum(npg)]), dtype=torch.int32, device=DEV)
    seq = torch.tensor(lens, dtype=torch.long, device=DEV)
    cap = 2 * 148 + len(lens)
    ws = torch.zeros(ops.paged_attention_workspace_bytes(len(lens), 2, cap), dtype=torch.uint8, device=DEV)
    o1 = torch.empty_like(q)
    o2 = torch.empty_like(q)
    ops.paged_decode_attention(q.view(len(lens), -1), kc, vc, page_indptr=indptr, page_indices=perm.to(DEV),
                               seq_lens=seq, work_indptr=indptr, num_q_heads=16, num_kv_heads=2, head_dim=128,
                               page_size=16, pages_per_chunk=1, work_capacity=cap, sm_scale=1 / math.sqrt(128),
                               out=o1.view(len(lens), -1), workspace=ws)
    tops.paged_decode_attention(q, kc, vc, indptr, perm.to(DEV), seq, 1 / math.sqrt(128), o2, ws, cap)
    torch.cuda.synchronize()
    assert torch.equal(o1, o2)
