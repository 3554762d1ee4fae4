"""The CPU oracle pinned against the reference's golden vectors and known answers.

Fixtures come from tests/golden/make_golden.py, which executes the reference's
own functions; known answers are the reference's unit-test constants.
"""

from __future__ import annotations

import numpy as np
import pytest

from conftest import decode_bf16_b64
from oracle import sampler as orc


def test_hash_matches_reference_murmur(golden):
    for case in golden["hashes"]:
        got = [orc.murmur_hash(case["seed"], case["position"], c) for c in range(64)]
        assert got == case["hash"], case["seed"]


def test_hash_endpoints_known_answers():
    # sglang_omni tests/unit_test/qwen3_tts/test_sampling_kernels.py:73-148
    assert orc.murmur_hash(0, 1_707_985_137, 0) == 0xFFFFFFFF
    assert orc.murmur_hash(0x804B40E3, 0, 49) == 0
    assert orc.murmur_hash(0x572AB199, 0, 49) == 0xFFFFFFFF


def test_gumbel_endpoint_clamps():
    # hash 0 -> log u clamped to -DBL_MAX; hash 2^32-1 -> log u clamped to -2^-32
    assert orc.gumbel(0) == pytest.approx(-np.log(np.finfo(np.float64).max), rel=1e-15)
    assert orc.gumbel(0xFFFFFFFF) == pytest.approx(-np.log(2.0**-32), rel=1e-15)


def test_sorted_sampler_golden(golden):
    for case in golden["sorted_sampler"]:
        tok = orc.sample_sorted(np.array(case["logprobs"], np.float32), np.array(case["sorted_idx"]),
                                [case["seed"]], [case["position"]])
        assert int(tok[0]) == case["token"]
    # known answer: logprobs [-100, 0] at the uint32-max hash -> rank 1 -> token 9
    assert orc.sample_sorted(np.array([[-100.0, 0.0]], np.float32), np.array([[7, 9]]), [0],
                             [1_707_985_137])[0] == 9


def test_residual_sampler_matches_reference_torch_path(golden):
    total = mism = 0
    for case in golden["residual_sampler"]:
        logits = decode_bf16_b64(case)
        got = orc.sample_topk_topp(logits, case["temperatures"], case["top_ks"], case["top_ps"], case["seeds"],
                                   case["positions"], max_top_k=case["max_top_k"], has_top_p=case["has_top_p"])
        total += len(got)
        mism += int((got != np.array(case["tokens"])).sum())
    # The reference's CPU softmax/log differ from the oracle's by an ulp at most;
    # on these tie-free cases every drawn token agrees.
    assert mism == 0, f"{mism}/{total} tokens differ"


def test_argmax_known_answer():
    # test_predictor_kernels.py:622-646: ties -> first, NaN -> first NaN, all -inf -> 0
    rng = np.random.default_rng(7)
    vocab, hidden = 2048, 16
    logits = rng.standard_normal((4, vocab)).astype(np.float32)
    logits[0, 9] = logits[0, 1700] = logits[0].max() + 1
    logits[1, 30] = logits[1, 4] = np.nan
    logits[2] = -np.inf
    logits[3, 11] = logits[3, 2047] = np.inf
    table = orc.f32_to_bf16_bits(rng.standard_normal((vocab, hidden)).astype(np.float32))
    summed = orc.f32_to_bf16_bits(rng.standard_normal((4, hidden)).astype(np.float32))
    codes, gathered, new_summed = orc.codebook_step(orc.f32_to_bf16_bits(logits), table, summed)
    assert codes.tolist() == [9, 4, 0, 11]
    assert np.array_equal(gathered, table[codes])
    want = orc.f32_to_bf16_bits(orc.bf16_bits_to_f32(summed) + orc.bf16_bits_to_f32(table[codes]))
    assert np.array_equal(new_summed, want)


def test_layer0_penalty_known_answer(golden):
    g = golden["layer0_penalty"]
    logits = np.array(g["logits"], np.float32)
    rows, vocab = logits.shape
    # pad to the sampler's vocab granularity with -inf columns (never drawn)
    pad = np.full((rows, 32 - vocab), -np.inf, np.float32)
    lg = np.concatenate([logits, pad], 1)
    rep = np.concatenate([np.array(g["rep_mask"], np.uint8), np.zeros((rows, 32 - vocab), np.uint8)], 1)
    sup = np.concatenate([np.array(g["suppress_mask"], np.uint8), np.zeros((rows, 32 - vocab), np.uint8)], 1)
    toks, processed = orc.layer0_sample(lg, g["penalties"], rep, sup, [1.0, 1.0], [1, 1], [1.0, 1.0], None,
                                        [0, 0], [0, 0], max_top_k=1, return_processed=True)
    want = np.array([[np.inf if v is None else v for v in r] for r in g["processed"]], np.float64)
    want[np.isinf(want)] = -np.inf
    np.testing.assert_allclose(processed[:, :vocab].astype(np.float64), want, rtol=0, atol=1e-6)
    # top_k = 1 is greedy: the reference's argmax answer
    assert toks.tolist() == g["argmax_tokens"]


def test_rollback_known_answer(golden):
    g = golden["rollback"]
    r2t = np.ones((2, 8), np.int32)
    sl, r2t_after, freed = orc.decode_rollback(g["seq_lens"], g["req_pool_indices"], r2t, g["page_size"],
                                               g["out_cache_loc"])
    assert freed.tolist() == g["freed"][0]
    assert sl.tolist() == g["seq_lens_after"]
    assert r2t_after.tolist() == g["req_to_token_after"]


def test_exp_log_error_bounds():
    rng = np.random.default_rng(0)
    xs = np.concatenate([rng.uniform(-100, 88, 4000), rng.uniform(-1, 1, 4000)]).astype(np.float32)
    for x in xs:
        ref = np.exp(np.float64(x))
        assert abs(orc.expf(x) - ref) <= 1.0 * np.spacing(np.float32(ref)) + 1e-45
    ys = np.exp(rng.uniform(-80, 80, 4000)).astype(np.float32)
    for y in ys:
        ref = np.log(np.float64(y))
        assert abs(orc.logf(y) - ref) <= 2.0 * abs(np.spacing(np.float32(ref)))
    zs = rng.uniform(0, 1, 4000)
    for z in zs:
        ref = np.log(z)
        assert abs(orc.log64(z) - ref) <= 2.0 * abs(np.spacing(ref))
    assert orc.logf(0.0) == -np.inf and orc.log64(0.0) == -np.inf and orc.expf(-200.0) == 0.0


def test_decode_prepare_pages():
    # two streams, page 4: row 0 at len 4 opens a page, row 1 at len 6 does not
    r2t = np.zeros((2, 16), np.int32)
    r2t[0, :4] = [8, 9, 10, 11]
    r2t[1, :6] = [20, 21, 22, 23, 4, 5]
    out = orc.decode_prepare([4, 6], [0, 1], r2t, 4, free_pages=np.array([7, 3], np.int32))
    sl, r2t2, loc, pos, kv_indptr, kv_indices, page_indptr, page_indices, head = out
    assert sl.tolist() == [5, 7]
    assert loc.tolist() == [28, 6]
    assert pos.tolist() == [4, 6]
    assert kv_indptr.tolist() == [0, 5, 12]
    assert kv_indices.tolist() == [8, 9, 10, 11, 28, 20, 21, 22, 23, 4, 5, 6]
    assert page_indices.tolist() == [2, 7, 5, 1]
    assert head == 1
    # the pages opened by this step are exactly what the rollback frees
    _, _, freed = orc.decode_rollback(sl, [0, 1], r2t2, 4, loc)
    assert freed.tolist() == [28]


def test_moe_route_renormalised_topk():
    rng = np.random.default_rng(1)
    lg = rng.standard_normal((16, 128)).astype(np.float32)
    ids, w = orc.moe_route(lg, 8)
    p = np.exp(lg - lg.max(1, keepdims=True))
    p /= p.sum(1, keepdims=True)
    want = np.argsort(-p, axis=1, kind="stable")[:, :8]
    assert np.array_equal(ids, want)
    np.testing.assert_allclose(w.sum(1), 1.0, rtol=1e-6)
    offsets, pairs = orc.moe_permute(ids, 128)
    assert offsets[-1] == 16 * 8
    flat = ids.reshape(-1)
    assert np.all(np.diff(flat[pairs]) >= 0)


def test_e4m3_codes_match_torch_float8():
    """The oracle's e4m3 encoder/decoder against torch.float8_e4m3fn, the dtype the
    reference's block-FP8 path quantises into (clamped to +-448 first)."""
    import torch

    rng = np.random.default_rng(7)
    mags = np.float32(10.0) ** rng.uniform(-4, 3, 4000).astype(np.float32)
    vals = np.concatenate([rng.standard_normal(4000).astype(np.float32) * mags,
                           np.array([0.0, -0.0, 448, -448, 449, 464, 465, 1e9, 2**-9, 2**-10, 3 * 2**-11, 2**-6,
                                     0.0009765625, 240, 248, 256, 272], np.float32)])
    want = torch.from_numpy(vals).clamp(-448, 448).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    assert np.array_equal(orc.e4m3_from_f32(vals), want)
    dec = orc.e4m3_to_f32(np.arange(256))
    tdec = torch.arange(256, dtype=torch.uint8).view(torch.float8_e4m3fn).float().numpy()
    assert np.array_equal(np.nan_to_num(dec, nan=-1.0), np.nan_to_num(tdec, nan=-1.0))


def test_group_quant_matches_torch_restatement():
    """per_token_group_quant_fp8: scale = max(amax, 1e-10) / 448, q = e4m3(clamp(x / scale))."""
    import torch

    rng = np.random.default_rng(8)
    x = rng.standard_normal((5, 384)).astype(np.float32)
    x[2, 128:256] = 0.0  # an all-zero group takes the 1e-10 floor
    q, s = orc.quant_fp8_group(x, 128)
    xt = torch.from_numpy(x).view(5, 3, 128)
    amax = xt.abs().amax(-1, keepdim=True).clamp_min(1e-10)
    ts = amax / 448.0
    tq = (xt / ts).clamp(-448, 448).to(torch.float8_e4m3fn).view(torch.uint8).view(5, 384).numpy()
    assert np.array_equal(q, tq)
    assert np.array_equal(s, ts.view(5, 3).numpy())
