"""Incremental code2wav decode on the B200 (omni_b200/code2wav.py with the library's
SnakeBeta, history / overlap exchange and clamped single-output-conv kernels), bf16.

bf16 through the forty-odd layers of the network moves the waveform by about 0.6 % (relative
L2) against a float64 forward on random weights, so the checks are: against the
float64 whole-sequence transformers forward within 5 %; decodes in different splits
within 5 % of each other; and the library kernels against the oracle's on the same
torch ops within 5 %.  The exact equivalence of any split runs in float64 on the CPU
(tests/test_code2wav_cpu.py)."""

from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu
pytest.importorskip("transformers")

from code2wav_util import decode_in_chunks, oracle_kernels, small_code2wav  # noqa: E402

DEV = "cuda"
TOL = 0.05


def _rel(a, b):
    return float((a.float() - b.float()).norm() / b.float().norm())


@pytest.fixture(scope="module")
def setup():
    codes = torch.randint(0, 32, (3, 4, 37), generator=torch.Generator().manual_seed(1))
    with torch.no_grad():
        ref = small_code2wav(gain=0.5).double()(codes).float()
    model = small_code2wav(gain=0.5).to(device=DEV, dtype=torch.bfloat16)
    return codes.to(DEV), ref, model


def _decode(model, codes, splits, kernels=None):
    from omni_b200.code2wav import Qwen3OmniIncrementalCodec

    codec = Qwen3OmniIncrementalCodec(model, kernels=kernels)
    pool = codec.make_pool(num_slots=6, ring_frames=codec.layout.retained + max(splits))
    return decode_in_chunks(codec, pool, codes, torch.tensor([4, 0, 2], device=DEV), splits).cpu()


@pytest.mark.parametrize("splits", [[37], [5, 1, 12, 19], [10, 10, 10, 7]])
def test_slot_decode_matches_the_whole_forward(setup, splits):
    codes, ref, model = setup
    wav = _decode(model, codes, splits)
    assert wav.shape == ref.shape and torch.isfinite(wav).all()
    assert _rel(wav, ref) < TOL


def test_splits_agree(setup):
    codes, _, model = setup
    assert _rel(_decode(model, codes, [5, 1, 12, 19]), _decode(model, codes, [37])) < TOL


def test_library_kernels_match_the_oracle_kernels(setup):
    codes, _, model = setup
    splits = [8, 29]
    assert _rel(_decode(model, codes, splits), _decode(model, codes, splits, oracle_kernels())) < TOL
