"""Request staging (prepare_decode_buffers) and seeds against the reference, executed.

The fixtures come from tests/golden/make_golden.py (main_staging), which runs the
reference's own functions on fake request sets: blake2b seed derivation and the
Qwen3-TTS seed split, Qwen3OmniTalker.prepare_decode_buffers, the Qwen3-TTS codec
suppression (control range but EOS, leading silence) and Qwen3TTSTalker's subtalker
staging.  omni_b200.staging must reproduce every staged value and mask exactly.

The large residual-sampler golden (12 000 rows per case of untied random bf16
logits at the config-0 / config-3 sampling parameters, tokens from the reference's
torch sampler) is checked here against the CPU oracle, which the GPU sampler
equals bit for bit (tests/test_sampling_gpu.py checks the device on the same rows).
"""

from __future__ import annotations

import sys

import numpy as np
import pytest

from conftest import GOLDEN
from omni_b200 import staging
from omni_b200.config import SamplingParams
from omni_b200.seed import derive_sampling_seed, resolve_row_seed
from oracle import sampler as orc

sys.path.insert(0, str(GOLDEN))
from scale_inputs import SCALE_CASES, scale_case  # noqa: E402


def test_seed_derivation_matches_reference(staging_golden):
    for c in staging_golden["derive"]:
        assert derive_sampling_seed(c["namespace"], c["seed"], c["label"]) == c["value"], c
    for c in staging_golden["resolve_row_seed"]:
        assert resolve_row_seed(c["seed"]) == c["value"], c
    for c in staging_golden["unseeded_rows"]:
        assert staging.unseeded_row_seed(c["rid"], c["row"]) == c["value"], c


def test_qwen3_tts_request_seeds_match_reference(staging_golden):
    for c in staging_golden["tts_seeds"]:
        assert list(staging.qwen3_tts_sampling_seeds(c["seed"])) == c["semantic_subtalker"], c
    with pytest.raises(ValueError):
        staging.normalize_qwen3_tts_seed(1.5)
    with pytest.raises(ValueError):
        staging.normalize_qwen3_tts_seed(True)


def _omni_requests(g):
    out = []
    for d in g["requests"]:
        sp = SamplingParams(temperature=d["temperature"], top_k=d["top_k"], top_p=d["top_p"], min_p=d["min_p"],
                            repetition_penalty=d["penalty"])
        out.append(staging.TalkerRequest(rid=d["rid"], seed=d["seed"], sampling=sp, output_ids=d["output_ids"],
                                         suppress_tokens=d["suppress"], codec_suppress_tokens=d["codec_suppress"]))
    return out


def test_omni_prepare_decode_buffers_matches_reference(staging_golden):
    g = staging_golden["omni_prepare_decode_buffers"]
    st = staging.stage_decode_buffers(_omni_requests(g), flavor=staging.OMNI, vocab=g["vocab"], predictor_vocab=2048)
    assert st.repetition_mask.tolist() == g["repetition_mask"]
    assert st.suppress_mask.tolist() == g["suppress_mask"]
    assert st.seeds.tolist() == g["seeds"]
    assert st.top_ks.tolist() == g["top_ks"]
    for mine, key in ((st.repetition_penalties, "repetition_penalties"), (st.temperatures, "temperatures"),
                      (st.top_ps, "top_ps"), (st.min_ps, "min_ps")):
        assert mine.astype(np.float32).tolist() == np.asarray(g[key], np.float32).tolist(), key


def test_tts_codec_suppression_matches_reference(staging_golden):
    g = staging_golden["tts_codec_suppress"]
    ctl = staging.CodecControl(codec_eos_token_id=g["codec_eos_token_id"],
                               leading_silence_mask_frames=g["leading_silence_mask_frames"],
                               silence_codec_ids=tuple(g["silence_codec_ids"]))
    reqs = [staging.TalkerRequest(rid=f"t{i}", seed=i, output_ids=[0] * r["frames"],
                                  mask_leading_silence=r["mask_leading_silence"])
            for i, r in enumerate(g["rows"])]
    st = staging.stage_decode_buffers(reqs, flavor=staging.TTS, vocab=g["vocab"], predictor_vocab=2048, control=ctl)
    for i, want in enumerate(g["masked"]):
        assert np.nonzero(st.suppress_mask[i])[0].tolist() == want, i
        # the base row (after the leading frames) is the control range but EOS alone
        assert np.nonzero(st.base_suppress_mask[i])[0].tolist() == g["masked"][0]
    assert st.silence_rows.tolist() == [len(m) != len(g["masked"][0]) for m in g["masked"]]


def test_tts_subtalker_staging_matches_reference(staging_golden):
    g = staging_golden["tts_prepare_decode_buffers"]
    reqs = []
    for i, d in enumerate(g["requests"]):
        sp = SamplingParams(subtalker_dosample=d["dosample"], subtalker_temperature=d["temperature"],
                            subtalker_top_p=d["top_p"], subtalker_top_k=d["top_k"])
        reqs.append(staging.TalkerRequest(rid=f"s{i}", seed=d["seed"], sampling=sp))
    st = staging.stage_decode_buffers(reqs, flavor=staging.TTS, vocab=3072, predictor_vocab=g["predictor_vocab"])
    assert st.seeds.tolist() == g["semantic_seeds"]
    assert st.sub_seeds.tolist() == g["seeds"]
    assert st.sub_top_ks.tolist() == g["top_ks"]
    assert st.sub_do_sample.astype(bool).tolist() == g["do_sample"]
    assert st.sub_temperatures.tolist() == np.asarray(g["temperatures"], np.float32).tolist()
    assert st.sub_top_ps.tolist() == np.asarray(g["top_ps"], np.float32).tolist()
    sig = st.signature
    assert sig["max_top_k"] == g["max_top_k"] and sig["has_top_p"] == g["has_top_p"]
    assert sig["has_sampled_rows"] == g["has_sampled_rows"] and sig["has_argmax_rows"] == g["has_argmax_rows"]
    assert sig["has_unbounded_top_k"] == g["has_unbounded_top_k"]


@pytest.mark.parametrize("name", [c[0] for c in SCALE_CASES])
def test_oracle_sampler_reproduces_the_reference_at_scale(name, sampler_scale_golden):
    """Every one of the 12 000 rows: the oracle (hence the GPU sampler, which equals it
    bit for bit) draws the reference torch sampler's token."""
    bits, temps, top_ks, top_ps, seeds, positions, max_top_k = scale_case(name)
    got = orc.sample_topk_topp(bits, temps, top_ks, top_ps, seeds, positions, max_top_k=max_top_k, has_top_p=True)
    want = sampler_scale_golden[name]
    mism = np.nonzero(got != want)[0]
    assert mism.size == 0, f"{mism.size} of {want.size} rows differ (first {mism[:10].tolist()})"
