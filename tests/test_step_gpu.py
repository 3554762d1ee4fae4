"""One full decode step (packing -> talker -> layer-0 draw -> code predictor) on
the GPU against the CPU oracle.

- packing (positions, slots, page table): bit-exact;
- talker logits and final hidden: cosine >= 0.999, max-abs <= 2e-2 x scale
  (bf16 tolerance of the north-star contract);
- every drawn token (layer 0 and 15 residual codebooks): bit-exact against the
  oracle sampler applied to the device's own logits;
- predictor lm_head logits with the device's codes fed back (teacher forcing):
  bf16 tolerance plus one bf16 ulp of output rounding (they are stored in bf16);
  summed codec embeddings: bit-exact;
- CUDA-graph replay == eager, bit for bit; rows never mix (batch invariance).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import sampler as orc
from oracle.model import OracleTalker
from step_util import check_step_against_oracle, cos_err

pytestmark = pytest.mark.gpu

DEV = "cuda"


def make_runner(layers=2, lens=(16, 1, 33, 100, 200, 15, 64, 17), seed=0, max_batch=8, sampling=None, moe=False):
    from omni_b200.config import MoEConfig, PredictorConfig, SamplingParams, TalkerConfig
    from omni_b200.model_runner import TalkerDecodeRunner

    if moe:  # the config-3 geometry: 128 experts top-8, 31 residual codebooks of 1024
        cfg = TalkerConfig(num_hidden_layers=layers, max_context=1024, moe=MoEConfig(),
                           predictor=PredictorConfig(vocab_size=1024, num_code_groups=32))
    else:
        cfg = TalkerConfig(num_hidden_layers=layers, max_context=1024)
    pages = sum((L + 16) // 16 for L in lens) + 32
    r = TalkerDecodeRunner(cfg, max_batch=max_batch, num_pages=pages, seed=seed)
    r.admit(list(lens), sampling=sampling or SamplingParams(), seed=seed + 5)
    g = torch.Generator(device=DEV).manual_seed(seed + 11)
    r.text_embeds.normal_(generator=g)
    r.predictor.output_embeds.normal_(generator=g)
    return r


@pytest.mark.parametrize("dosample,moe", [(True, False), (False, False), (True, True)])
def test_decode_step_matches_oracle(dosample, moe):
    from omni_b200.config import SamplingParams

    r = make_runner(sampling=SamplingParams(subtalker_dosample=dosample), moe=moe)
    check_step_against_oracle(r, use_graph=False)


@pytest.mark.parametrize("moe", [False, True])
def test_graph_replay_is_bit_identical_to_eager(moe):
    a = make_runner(seed=1, moe=moe)
    b = make_runner(seed=1, moe=moe)
    b.capture(warmup=1)
    a.step(use_graph=False)  # the same number of steps as b's warm-up
    for _ in range(3):
        a.step(use_graph=False)
        b.step(use_graph=True)
        torch.cuda.synchronize()
        assert torch.equal(a.predictor.output_codes, b.predictor.output_codes)
        assert torch.equal(a.talker.logits, b.talker.logits)
        assert torch.equal(a.predictor.output_embeds, b.predictor.output_embeds)
        assert torch.equal(a.seq_lens, b.seq_lens)


@pytest.mark.parametrize("moe", [False, True])
def test_rows_never_mix(moe):
    """A row's frame does not depend on the other rows of the batch (with MoE: nor on
    which rows share its experts)."""
    lens = (16, 1, 33, 100, 200, 15, 64, 17)
    full = make_runner(lens=lens, seed=2, moe=moe)
    full.step(use_graph=False)
    part = make_runner(lens=lens[:4], seed=2, moe=moe)
    # same per-row inputs: copy the full runner's initial feedback/text rows of the first 4 streams
    ref = make_runner(lens=lens, seed=2, moe=moe)
    part.text_embeds[:4].copy_(ref.text_embeds[:4])
    part.predictor.output_embeds[:4].copy_(ref.predictor.output_embeds[:4])
    part.talker.sampling_seeds[:4].copy_(ref.talker.sampling_seeds[:4])
    part.predictor.sub_sampling_seed_tensor[:4].copy_(ref.predictor.sub_sampling_seed_tensor[:4])
    # KV pool contents of the first 4 streams' slots
    n4 = sum((L + 15) // 16 for L in lens[:4])
    slots_full = ref.r2t.req_to_token[:4]
    slots_part = part.r2t.req_to_token[:4]
    for i, L in enumerate(lens[:4]):
        part.kv.k_buffer[:, slots_part[i, :L].long()] = ref.kv.k_buffer[:, slots_full[i, :L].long()]
        part.kv.v_buffer[:, slots_part[i, :L].long()] = ref.kv.v_buffer[:, slots_full[i, :L].long()]
    del n4
    part.step(use_graph=False)
    torch.cuda.synchronize()
    assert torch.equal(part.predictor.output_codes[:4], full.predictor.output_codes[:4])
    assert torch.equal(part.talker.logits[:4], full.talker.logits[:4])


def test_public_decode_api_round_trip():
    r = make_runner(seed=4)
    r.capture(warmup=1)
    B = r.batch_size
    text = torch.randn(B, r.cfg.hidden_size).to(torch.bfloat16).pin_memory()
    codes = r.decode(text)
    assert codes.shape == (B, r.cfg.predictor.num_code_groups)
    assert (codes[:, 0] < r.cfg.vocab_size).all() and (codes[:, 1:] < r.cfg.predictor.vocab_size).all()
    assert torch.equal(codes, r.predictor.output_codes[:B].cpu())
    from omni_b200 import device_status

    assert device_status() == 0


@pytest.mark.parametrize("prompts", [(20, 70), (150, 260)], ids=["fused-qkv", "prompt-sized"])
def test_mixed_prefill_decode_step_matches_oracle(prompts):
    """Config 2's fused forward at small size: 3 decode streams + 2 new streams (prompts of
    20 and 70 rows; or 150 and 260, over 256 rows, where the projections take the tile loop
    and the qkv projection its separate norm / rotary / store pass) in one forward; logits /
    hidden of the decode rows and of each new stream's last prompt row within the bf16
    tolerance, the prompts' KV in the pool, the layer-0 draws bit-exact given the device
    logits."""
    from omni_b200.config import SamplingParams, TalkerConfig
    from omni_b200.model_runner import TalkerDecodeRunner

    lens = (16, 33, 100)
    cfg = TalkerConfig(num_hidden_layers=2, max_context=1024)
    pages = sum((L + 16) // 16 for L in lens) + sum((L + 15) // 16 for L in prompts) + 32
    r = TalkerDecodeRunner(cfg, max_batch=5, num_pages=pages, seed=6, max_prefill_tokens=sum(prompts))
    r.admit(list(lens), sampling=SamplingParams(), seed=7)
    g = torch.Generator(device=DEV).manual_seed(8)
    r.text_embeds.normal_(generator=g)
    r.predictor.output_embeds.normal_(generator=g)
    r.admit_prefill(list(prompts), seed=9)
    B = r.batch_size
    seq0 = r.seq_lens[:B].cpu().numpy()
    r2t0 = r.r2t.req_to_token.cpu().numpy()
    free = r.allocator.free_pages.cpu().numpy()
    head0 = int(r.allocator.free_head.item())
    kpool = r.kv.k_buffer.float().cpu()
    vpool = r.kv.v_buffer.float().cpu()
    feedback = r.predictor.output_embeds[:B].clone().cpu()
    text = r.text_embeds[:B].clone().cpu()
    prompt = r.prompt_embeds.clone().cpu()
    t = r.talker
    n = B + len(prompts)
    l0_state = dict(penalties=t.repetition_penalties[:n].cpu().numpy(), rep_mask=t.repetition_mask[:n].cpu().numpy(),
                    suppress_mask=t.suppress_mask[:n].cpu().numpy(), temperature=t.sampling_temperatures[:n].cpu().numpy(),
                    top_k=t.sampling_top_ks[:n].cpu().numpy(), top_p=t.sampling_top_ps[:n].cpu().numpy(),
                    min_p=t.sampling_min_ps[:n].cpu().numpy(), seed=t.sampling_seeds[:n].cpu().numpy(),
                    max_top_k=t.max_top_k)
    r.step(use_graph=False)
    torch.cuda.synchronize()
    assert int(r.status.item()) == 0
    sl, r2t1, loc, pos, _, _, pgp, pgi, head1 = orc.decode_prepare(seq0, np.arange(B), r2t0[:B], cfg.page_size, free,
                                                                   free_head=head0)
    # extend rows: positions 0..L-1 at the reserved slots; token j attends its stream's first j+1 slots
    ext_pos, ext_loc, ext_ctx = [], [], []
    for i, L in enumerate(prompts):
        slots = torch.from_numpy(r2t0[B + i, :L].astype(np.int64))
        ext_pos += list(range(L))
        ext_loc += slots.tolist()
        ext_ctx += [slots[: j + 1] for j in range(L)]
    assert r.row_positions[B: B + sum(prompts)].cpu().tolist() == ext_pos
    assert r.row_cache_loc[B: B + sum(prompts)].cpu().tolist() == ext_loc
    assert r.row_cache_loc[:B].cpu().numpy().tolist() == loc.tolist()
    o = OracleTalker(cfg, r.w, r.predictor.w)
    select = list(range(B)) + [B + int(x) for x in np.cumsum(prompts) - 1]
    logits_o, hidden_o = o.mixed_forward(feedback, text, torch.from_numpy(pos), torch.from_numpy(loc),
                                         torch.from_numpy(sl), torch.from_numpy(r2t1), prompt, ext_pos, ext_loc,
                                         ext_ctx, torch.tensor(select), kpool, vpool)
    cos, err, scale = cos_err(t.logits[:n], logits_o)
    assert cos >= 0.999 and err <= 2e-2 * max(scale, 1.0), (cos, err, scale)
    cos, err, scale = cos_err(t.hidden[:n], hidden_o)
    assert cos >= 0.999 and err <= 2e-2 * max(scale, 1.0), (cos, err, scale)
    kdev = r.kv.k_buffer[:, torch.tensor(ext_loc, device=DEV)].float().cpu()
    cos, err, scale = cos_err(kdev, kpool[:, torch.tensor(ext_loc)])
    assert cos >= 0.999, cos
    l0_state["positions"] = np.array(pos.tolist() + [L - 1 for L in prompts])
    c0 = t.sampled_token_ids[:n].cpu()
    assert o.layer0(t.logits[:n].cpu(), l0_state).tolist() == c0.tolist()
    assert r.predictor.output_codes[:n, 0].cpu().tolist() == c0.tolist()


def test_staged_requests_drive_the_layer0_draw():
    """prepare_decode_buffers through the runner: requests with prior output ids,
    repetition penalties, suppress lists and cold-start clones (Qwen3-TTS flavor:
    control range but EOS, leading silence) are staged into the device tensors exactly
    as omni_b200.staging stages them; the step's layer-0 draw is bit-exact against the
    oracle under those masks and never lands on a suppressed id; a clone's silence ids
    are released after leading_silence_mask_frames frames."""
    from omni_b200.config import SamplingParams, TalkerConfig
    from omni_b200.model_runner import TalkerDecodeRunner
    from omni_b200.staging import TTS, CodecControl, TalkerRequest

    lens = (16, 1, 33, 100, 200, 15, 64, 17)
    cfg = TalkerConfig(num_hidden_layers=2, max_context=1024)
    rng = np.random.default_rng(5)
    silence = tuple(int(x) for x in rng.choice(2048, 24, replace=False))
    ctl = CodecControl(codec_eos_token_id=2150, leading_silence_mask_frames=2, silence_codec_ids=silence)
    pages = sum((L + 16) // 16 for L in lens) + 32
    r = TalkerDecodeRunner(cfg, max_batch=8, num_pages=pages, seed=3, flavor=TTS, codec_control=ctl)
    reqs = []
    for i in range(8):
        sp = SamplingParams(repetition_penalty=[1.05, 1.0, 1.5, 2.0][i % 4], temperature=[0.9, 0.7][i % 2],
                            top_k=[50, 20, 64, 4][i % 4], top_p=[0.8, 1.0, 0.95][i % 3],
                            subtalker_dosample=i != 3)
        clone = i in (0, 2, 6)  # cold-start clones have emitted nothing yet
        prior = [] if clone else [int(x) for x in rng.integers(0, 2048, int(rng.integers(0, 40)))]
        reqs.append(TalkerRequest(rid=f"s{i}", seed=None if i == 5 else 100 + i, sampling=sp, output_ids=prior,
                                  suppress_tokens=[int(x) for x in rng.integers(0, 3072, 5)] if i % 2 else None,
                                  mask_leading_silence=clone))
    r.admit(list(lens), requests=reqs, seed=4)
    g = torch.Generator(device=DEV).manual_seed(9)
    r.text_embeds.normal_(generator=g)
    r.predictor.output_embeds.normal_(generator=g)
    st = r.stage_requests(reqs)
    t, p = r.talker, r.predictor
    B = 8
    assert np.array_equal(t.repetition_mask[:B].cpu().numpy(), st.repetition_mask)
    assert np.array_equal(t.suppress_mask[:B].cpu().numpy(), st.suppress_mask)
    assert t.sampling_seeds[:B].cpu().tolist() == st.seeds.tolist()
    assert t.sampling_top_ks[:B].cpu().tolist() == st.top_ks.tolist()
    assert p.sub_sampling_seed_tensor[:B].cpu().tolist() == st.sub_seeds.tolist()
    assert p.sub_top_k_tensor[:B].cpu().tolist() == st.sub_top_ks.tolist()
    assert p.sub_do_sample_tensor[:B].cpu().tolist() == st.sub_do_sample.tolist()
    masked = [set(np.nonzero(st.suppress_mask[i])[0].tolist()) for i in range(B)]
    assert r.silence_rows.tolist() == [i in (0, 2, 6) for i in range(B)]
    assert all(set(silence) <= masked[i] for i in (0, 2, 6))
    check_step_against_oracle(r, use_graph=False)  # bit-exact draw under the staged masks
    c0 = t.sampled_token_ids[:B].cpu().tolist()
    assert all(c not in masked[i] for i, c in enumerate(c0))
    # the public decode API keeps the frame count (step() is the device-only path);
    # the clones' silence ids stay masked for their first 2 frames, then are released
    r.capture(warmup=1)
    text = torch.randn(B, cfg.hidden_size).to(torch.bfloat16).pin_memory()
    codes = r.decode(text)
    assert all(int(codes[i, 0]) not in masked[i] for i in range(B))
    assert r.silence_rows.tolist() == [i in (0, 2, 6) for i in range(B)]
    codes = r.decode(text)
    assert all(int(codes[i, 0]) not in masked[i] for i in range(B))
    assert not r.silence_rows.any()
    assert np.array_equal(t.suppress_mask[:B].cpu().numpy(), r.base_suppress[:B])


@pytest.mark.parametrize("batch", [1, 3, 16])
def test_pair_pass_matches_two_one_token_passes(batch):
    """The predictor's opening two-token pass (rows (request, token), slots 0 and 1, causal)
    against two one-token passes (slot 0, then slot 1 over the cached slot 0): the
    residual stream of both tokens and the K/V of both slots within the bf16 GEMM rounding
    tolerance the reference uses for the same check (atol 2^-6, rtol 2^-7;
    test_predictor_cuda_graph.py:637-672)."""
    import dataclasses

    from omni_b200.config import CONFIG0_PREDICTOR
    from omni_b200.predictor import CodePredictor, init_predictor_weights

    dev = torch.device(DEV)
    cfg = dataclasses.replace(CONFIG0_PREDICTOR, num_hidden_layers=2)
    H, S = cfg.hidden_size, cfg.cache_len
    w = init_predictor_weights(cfg, seed=batch, device=dev)
    emb0 = torch.zeros(16, H, dtype=torch.bfloat16, device=dev)
    pair = CodePredictor(cfg, w, max_batch=batch, device=dev, layer0_embedding=emb0)
    serial = CodePredictor(cfg, w, max_batch=batch, device=dev, layer0_embedding=emb0)
    g = torch.Generator(device=dev).manual_seed(batch)
    embeds = torch.randn(batch, 2, H, generator=g, device=dev).to(torch.bfloat16)

    def sumsq(x):
        return x.float().pow(2).sum(-1).contiguous()

    x2 = embeds.reshape(2 * batch, H).contiguous()
    h_pair = pair.forward_tokens(x2, sumsq(x2), batch=batch, tokens=2, cache_len=0).clone()
    x0 = embeds[:, 0].contiguous()
    h0 = serial.forward_tokens(x0, sumsq(x0), batch=batch, tokens=1, cache_len=0).clone()
    x1 = embeds[:, 1].contiguous()
    h1 = serial.forward_tokens(x1, sumsq(x1), batch=batch, tokens=1, cache_len=1).clone()
    torch.cuda.synchronize()
    tol = dict(atol=2 ** -6, rtol=2 ** -7)
    torch.testing.assert_close(h_pair.view(batch, 2, H)[:, 0].float(), h0.float(), **tol)
    torch.testing.assert_close(h_pair.view(batch, 2, H)[:, 1].float(), h1.float(), **tol)
    slots = (torch.arange(batch, device=dev)[:, None] * S + torch.arange(2, device=dev)[None, :]).reshape(-1)
    for cache_p, cache_s in ((pair.k_cache, serial.k_cache), (pair.v_cache, serial.v_cache)):
        torch.testing.assert_close(cache_p[:, slots].float(), cache_s[:, slots].float(), **tol)
