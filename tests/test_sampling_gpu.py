"""GPU parity of the sampling kernels against the CPU oracle (bit-exact tokens).

Cases follow the reference's sampler tests
(tests/unit_test/qwen3_tts/test_sampling_kernels.py): widths on the ladder,
top-p on/off, ties and signed zeros, hash endpoints, argmax known answers.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import decode_bf16_b64
from oracle import sampler as orc

pytestmark = pytest.mark.gpu

LADDER = (4, 8, 16, 32, 50, 64, 128, 256, 512, 1024)


def _bits_to_bf16_tensor(bits: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(bits.astype(np.uint16).view(np.int16)).view(torch.bfloat16).cuda()


def _bf16_bits(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().view(torch.int16).numpy().view(np.uint16)


def _row_params(rng, rows, max_top_k, *, top_p_mode="mixed"):
    temps = rng.choice([0.5, 0.9, 1.0, 1.3, 0.0], size=rows).astype(np.float32)
    top_ks = rng.integers(1, max_top_k + 1, size=rows).astype(np.int64)
    top_ks[0] = max_top_k
    if top_p_mode == "mixed":
        top_ps = rng.choice([0.0, 0.3, 0.8, 0.95, 1.0], size=rows).astype(np.float32)
    else:
        top_ps = np.ones(rows, np.float32)
    seeds = rng.integers(0, 2**31 - 1, size=rows).astype(np.int64)
    positions = rng.integers(0, 1 << 20, size=rows).astype(np.int64)
    return temps, top_ks, top_ps, seeds, positions


def _logits(rng, rows, vocab, kind):
    if kind == "normal":
        x = rng.standard_normal((rows, vocab)).astype(np.float32) * 3
    elif kind == "ties":  # few distinct values: many threshold ties
        x = np.round(rng.standard_normal((rows, vocab)) * 2).astype(np.float32) / 2
    elif kind == "zeros":  # signed zeros, -inf and large ties
        x = rng.choice(np.array([0.0, -0.0, 1.0, -1.0, -np.inf, 2.0], np.float32), size=(rows, vocab))
        x[:, 0] = 2.0
    else:
        raise ValueError(kind)
    return orc.f32_to_bf16_bits(x)


def _run_gpu(bits, temps, top_ks, top_ps, seeds, positions, max_top_k, has_top_p):
    from omni_b200.sampling_kernels import sample_from_logits_with_seed_top_k_top_p

    out = sample_from_logits_with_seed_top_k_top_p(
        _bits_to_bf16_tensor(bits),
        torch.from_numpy(temps).cuda(),
        torch.from_numpy(top_ks).cuda(),
        torch.from_numpy(top_ps).cuda(),
        torch.from_numpy(seeds).cuda(),
        torch.from_numpy(positions).cuda(),
        max_top_k=max_top_k,
        has_top_p=has_top_p,
    )
    assert out is not None
    return out.cpu().numpy()


@pytest.mark.parametrize("max_top_k", LADDER)
@pytest.mark.parametrize("kind", ["normal", "ties", "zeros"])
def test_sampler_matches_oracle_across_ladder(max_top_k, kind):
    rng = np.random.default_rng(max_top_k * 7 + len(kind))
    for rows, vocab in [(37, 2048), (8, 1024), (5, 4096)]:
        if LADDER.index(max_top_k) >= 0 and max(32, max_top_k) > vocab:
            continue
        bits = _logits(rng, rows, vocab, kind)
        params = _row_params(rng, rows, max_top_k)
        for has_top_p in (False, True):
            got = _run_gpu(bits, *params, max_top_k, has_top_p)
            want = orc.sample_topk_topp(bits, *params, max_top_k=max_top_k, has_top_p=has_top_p)
            assert np.array_equal(got, want), (rows, vocab, kind, has_top_p, np.nonzero(got != want))


@pytest.mark.parametrize("rows", [1, 64, 256])
def test_sampler_config0_shapes(rows):
    rng = np.random.default_rng(rows)
    bits = _logits(rng, rows, 2048, "normal")
    params = _row_params(rng, rows, 50)
    got = _run_gpu(bits, *params, 50, True)
    want = orc.sample_topk_topp(bits, *params, max_top_k=50, has_top_p=True)
    assert np.array_equal(got, want)


def test_sampler_matches_reference_golden(golden):
    for case in golden["residual_sampler"]:
        bits = decode_bf16_b64(case)
        params = [np.array(case[k], dt) for k, dt in (("temperatures", np.float32), ("top_ks", np.int64),
                                                      ("top_ps", np.float32), ("seeds", np.int64),
                                                      ("positions", np.int64))]
        got = _run_gpu(bits, *params, case["max_top_k"], case["has_top_p"])
        assert got.tolist() == case["tokens"], case["id"]


@pytest.mark.parametrize("name", ["config0", "config3"])
def test_sampler_reproduces_the_reference_at_scale(name, sampler_scale_golden):
    """12 000 rows of untied random bf16 logits at the config-0 / config-3 sampling
    parameters (tests/golden/scale_inputs.py): every token equals the one the
    reference's own torch sampler drew (tests/golden/make_golden.py)."""
    import sys

    from conftest import GOLDEN

    sys.path.insert(0, str(GOLDEN))
    from scale_inputs import scale_case

    bits, temps, top_ks, top_ps, seeds, positions, max_top_k = scale_case(name)
    got = _run_gpu(bits, temps, top_ks, top_ps, seeds, positions, max_top_k, True)
    want = sampler_scale_golden[name]
    mism = np.nonzero(got != want)[0]
    assert mism.size == 0, f"{mism.size} of {want.size} rows differ (first {mism[:10].tolist()})"


def test_fused_sampler_at_uint32_max_hash():
    # test_sampling_kernels.py:151-186
    logits = np.full((1, 2048), -200.0, np.float32)
    logits[0, :49] = -np.arange(49, dtype=np.float32)
    logits[0, 49] = -100.0
    bits = orc.f32_to_bf16_bits(logits)
    params = (np.ones(1, np.float32), np.array([50]), np.ones(1, np.float32), np.array([0x572AB199]), np.zeros(1, np.int64))
    got = _run_gpu(bits, *params, 50, False)
    want = orc.sample_topk_topp(bits, *params, max_top_k=50, has_top_p=False)
    assert got.tolist() == want.tolist()


def test_sorted_sampler_golden_and_random(golden):
    from omni_b200.sampling_kernels import sample_from_sorted_logprobs_with_seed_small_k

    for case in golden["sorted_sampler"]:
        lp = torch.tensor(case["logprobs"], dtype=torch.float32).cuda()
        idx = torch.tensor(case["sorted_idx"]).cuda()
        out = sample_from_sorted_logprobs_with_seed_small_k(lp, idx, torch.tensor([case["seed"]]).cuda(),
                                                            torch.tensor([case["position"]]).cuda())
        assert int(out[0]) == case["token"]
    rng = np.random.default_rng(3)
    for rows, cols in [(1, 1), (3, 2), (7, 30), (16, 64), (5, 1024)]:
        p = rng.random((rows, cols)).astype(np.float32)
        lp = np.log(p / p.sum(1, keepdims=True)).astype(np.float32)
        idx = rng.integers(0, 8192, (rows, cols))
        seeds = np.arange(17, 17 + rows)
        pos = np.arange(3, 3 + rows)
        out = sample_from_sorted_logprobs_with_seed_small_k(torch.from_numpy(lp).cuda(), torch.from_numpy(idx).cuda(),
                                                            torch.from_numpy(seeds).cuda(), torch.from_numpy(pos).cuda())
        assert np.array_equal(out.cpu().numpy(), orc.sample_sorted(lp, idx, seeds, pos))


def test_codebook_step_known_answer():
    from omni_b200.predictor_layers import codebook_step

    rng = np.random.default_rng(7)
    vocab, hidden, rows = 2048, 1024, 8
    logits = rng.standard_normal((rows, vocab)).astype(np.float32)
    logits[0, 9] = logits[0, 1700] = logits[0].max() + 1
    logits[1, 30] = logits[1, 4] = np.nan
    logits[2] = -np.inf
    logits[3, 11] = logits[3, 2047] = np.inf
    lbits = orc.f32_to_bf16_bits(logits)
    table = orc.f32_to_bf16_bits(rng.standard_normal((vocab, hidden)).astype(np.float32))
    summed = orc.f32_to_bf16_bits(rng.standard_normal((rows, hidden)).astype(np.float32))
    codes = torch.full((rows, 16), -1, dtype=torch.long, device="cuda")
    s = _bits_to_bf16_tensor(summed)
    inp = codebook_step(_bits_to_bf16_tensor(lbits), _bits_to_bf16_tensor(table), codes[:, 5], s)
    want_codes, want_g, want_s = orc.codebook_step(lbits, table, summed)
    assert want_codes[:4].tolist() == [9, 4, 0, 11]
    assert codes[:, 5].cpu().tolist() == want_codes.tolist()
    assert (codes[:, :5] == -1).all() and (codes[:, 6:] == -1).all()
    assert np.array_equal(_bf16_bits(inp[:, 0]), want_g)
    assert np.array_equal(_bf16_bits(s), want_s)


@pytest.mark.parametrize("argmax_rows", [False, True])
def test_predictor_sample_step_fused_gather(argmax_rows):
    from omni_b200.sampling_kernels import predictor_sample_step

    rng = np.random.default_rng(11)
    rows, vocab, hidden, G = 64, 2048, 1024, 16
    bits = _logits(rng, rows, vocab, "normal")
    temps, top_ks, top_ps, seeds, _ = _row_params(rng, rows, 50)
    sem = rng.integers(0, 500, rows).astype(np.int64)
    j = 6
    positions = sem * (G - 1) + (j + 1)
    do_sample = np.ones(rows, np.uint8)
    if argmax_rows:
        do_sample[::3] = 0
    table = orc.f32_to_bf16_bits(rng.standard_normal((vocab, hidden)).astype(np.float32) * 0.02)
    summed = orc.f32_to_bf16_bits(rng.standard_normal((rows, hidden)).astype(np.float32))
    codes = torch.zeros((rows, G), dtype=torch.long, device="cuda")
    gathered = torch.empty((rows, hidden), dtype=torch.bfloat16, device="cuda")
    s = _bits_to_bf16_tensor(summed)
    cuda = lambda a: torch.from_numpy(a).cuda()  # noqa: E731
    predictor_sample_step(
        _bits_to_bf16_tensor(bits), temperatures=cuda(temps), top_ks=cuda(top_ks), top_ps=cuda(top_ps),
        seeds=cuda(seeds), positions=cuda(sem), pos_mul=G - 1, pos_add=j + 1, do_sample=cuda(do_sample),
        argmax_all=False, max_top_k=50, has_top_p=True, codes=codes[:, j + 1], table=_bits_to_bf16_tensor(table),
        gathered=gathered, summed=s)
    want = orc.sample_topk_topp(bits, temps, top_ks, top_ps, seeds, positions, max_top_k=50, has_top_p=True)
    am, _, _ = orc.codebook_step(bits, table)
    want = np.where(do_sample.astype(bool), want, am)
    assert codes[:, j + 1].cpu().numpy().tolist() == want.tolist()
    wg, ws = orc.gather_add(want, table, summed)
    assert np.array_equal(_bf16_bits(gathered), wg)
    assert np.array_equal(_bf16_bits(s), ws)


def test_gather_codec_embedding_and_add_contract():
    from omni_b200.predictor_kernels import gather_codec_embedding_and_add

    rng = np.random.default_rng(5)
    rows, vocab, hidden, psize = 9, 2048, 1024, 512
    table = torch.randn(vocab, hidden, device="cuda").to(torch.bfloat16)
    ptable = torch.randn(vocab, psize, device="cuda").to(torch.bfloat16)
    tokens = torch.from_numpy(rng.integers(0, vocab, rows)).cuda()
    gathered = torch.empty(rows, hidden, device="cuda", dtype=torch.bfloat16)
    acc = torch.randn(rows, hidden, device="cuda").to(torch.bfloat16)
    projected = torch.empty(rows, psize, device="cuda", dtype=torch.bfloat16)
    acc0 = acc.clone()
    assert gather_codec_embedding_and_add(tokens, table, gathered, acc, ptable, projected)
    torch.cuda.synchronize()
    assert torch.equal(gathered, table[tokens])
    assert torch.equal(acc, (acc0.float() + table[tokens].float()).to(torch.bfloat16))
    assert torch.equal(projected, ptable[tokens])
    # int32 ids
    acc1 = acc0.clone()
    assert gather_codec_embedding_and_add(tokens.int(), table, gathered, acc1)
    assert torch.equal(acc1, (acc0.float() + table[tokens].float()).to(torch.bfloat16))
    # overlap and dtype violations: False and no writes
    before = acc.clone()
    assert not gather_codec_embedding_and_add(tokens, table, acc, acc)
    assert not gather_codec_embedding_and_add(tokens, table.float(), gathered, acc)
    assert not gather_codec_embedding_and_add(tokens.cpu(), table, gathered, acc)
    assert torch.equal(acc, before)


def test_sampler_returns_none_outside_contract():
    from omni_b200.sampling_kernels import sample_from_logits_with_seed_top_k_top_p

    rows = 3
    args = [torch.ones(rows, device="cuda"), torch.full((rows,), 8, device="cuda", dtype=torch.long),
            torch.ones(rows, device="cuda"), torch.zeros(rows, device="cuda", dtype=torch.long),
            torch.zeros(rows, device="cuda", dtype=torch.long)]
    lg = torch.randn(rows, 2048, device="cuda").to(torch.bfloat16)
    assert sample_from_logits_with_seed_top_k_top_p(lg, *args, max_top_k=7, has_top_p=False) is None
    assert sample_from_logits_with_seed_top_k_top_p(lg.float(), *args, max_top_k=8, has_top_p=False) is None
    assert sample_from_logits_with_seed_top_k_top_p(lg[:, :2047], *args, max_top_k=8, has_top_p=False) is None
    assert sample_from_logits_with_seed_top_k_top_p(lg.cpu(), *[a.cpu() for a in args], max_top_k=8,
                                                    has_top_p=False) is None
    empty = sample_from_logits_with_seed_top_k_top_p(lg[:0], *[a[:0] for a in args], max_top_k=8, has_top_p=False)
    assert empty is not None and empty.shape == (0,)


@pytest.mark.parametrize("max_top_k", [1, 8, 50, 256])
def test_layer0_sampler_matches_oracle(max_top_k):
    from omni_b200.sampling_kernels import layer0_sample

    rng = np.random.default_rng(max_top_k)
    rows, vocab = 64, 3072
    logits = (rng.standard_normal((rows, vocab)) * 4).astype(np.float32)
    logits[:, ::97] = np.round(logits[:, ::97])  # some ties
    pen = rng.choice([1.0, 1.05, 1.3], rows).astype(np.float32)
    rep = (rng.random((rows, vocab)) < 0.02).astype(np.uint8)
    sup = np.zeros((rows, vocab), np.uint8)
    sup[:, vocab - 1024:] = 1
    sup[:, vocab - 1024 + 5] = 0  # an allowed control token (EOS)
    temps = rng.choice([0.7, 0.9, 1.0], rows).astype(np.float32)
    top_ks = rng.integers(1, max_top_k + 1, rows).astype(np.int64)
    top_ps = rng.choice([0.8, 1.0, 0.5], rows).astype(np.float32)
    min_ps = rng.choice([0.0, 0.05], rows).astype(np.float32)
    seeds = rng.integers(0, 2**31 - 1, rows).astype(np.int64)
    pos = rng.integers(0, 8192, rows).astype(np.int64)
    cuda = lambda a: torch.from_numpy(a).cuda()  # noqa: E731
    got = layer0_sample(cuda(logits), penalties=cuda(pen), repetition_mask=cuda(rep).bool(),
                        suppress_mask=cuda(sup).bool(), temperatures=cuda(temps), top_ks=cuda(top_ks),
                        top_ps=cuda(top_ps), min_ps=cuda(min_ps), seeds=cuda(seeds), positions=cuda(pos),
                        max_top_k=max_top_k)
    want = orc.layer0_sample(logits, pen, rep, sup, temps, top_ks, top_ps, min_ps, seeds, pos, max_top_k=max_top_k)
    assert np.array_equal(got.cpu().numpy(), want)
    assert not np.any(np.isin(want, np.arange(vocab - 1024, vocab)[np.arange(1024) != 5]))


def test_no_device_timeouts_recorded():
    from omni_b200 import device_status

    assert device_status() == 0
