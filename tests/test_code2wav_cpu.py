"""Incremental code2wav decode (omni_b200/code2wav.py) on the CPU, in float64, with the
oracle's kernels: a stream's frames decoded in any split give the waveform of the
whole-sequence transformers forward (the property Qwen3OmniIncrementalCodec states,
sglang_omni/models/qwen3_omni/components/code2wav.py:378-381)."""

from __future__ import annotations

import pytest
import torch

pytest.importorskip("transformers")

from code2wav_util import decode_in_chunks, oracle_kernels, small_code2wav  # noqa: E402
from omni_b200.code2wav import Qwen3OmniIncrementalCodec  # noqa: E402


@pytest.fixture(scope="module")
def model():
    # float64 end to end: the decode in chunks must agree with the whole forward up to
    # summation order
    return small_code2wav().double()


def _codes(model, rows, frames, seed=1):
    g = torch.Generator().manual_seed(seed)
    q = model.config.num_quantizers
    return torch.randint(0, model.config.codebook_size, (rows, q, frames), generator=g)


@pytest.mark.parametrize("splits", [[37], [1, 36], [5, 1, 12, 19], [3] * 12 + [1], [9, 9, 9, 10], [1] * 37])
def test_any_split_gives_the_whole_sequence_waveform(model, splits):
    codes = _codes(model, 3, sum(splits))
    with torch.no_grad():
        whole = model(codes)
    codec = Qwen3OmniIncrementalCodec(model, kernels=oracle_kernels())
    pool = codec.make_pool(num_slots=6, ring_frames=codec.layout.retained + max(splits))
    wav = decode_in_chunks(codec, pool, codes, torch.tensor([4, 0, 2]), splits)
    assert wav.shape == whole.shape
    assert (whole.abs() < 1).float().mean() > 0.5, "waveform mostly clamped: the check would be weak"
    torch.testing.assert_close(wav, whole, atol=1e-10, rtol=0)


def test_streams_in_other_slots_do_not_disturb_a_stream(model):
    codes = _codes(model, 2, 24, seed=3)
    with torch.no_grad():
        whole = model(codes)
    codec = Qwen3OmniIncrementalCodec(model, kernels=oracle_kernels())
    pool = codec.make_pool(num_slots=4, ring_frames=codec.layout.retained + 8)
    other = _codes(model, 2, 16, seed=4)
    a, b = torch.tensor([1, 3]), torch.tensor([0, 2])
    parts = [codec.decode_slots(codes[..., :8], pool, a, first_decode=True)]
    codec.decode_slots(other[..., :8], pool, b, first_decode=True)
    parts.append(codec.decode_slots(codes[..., 8:16], pool, a, first_decode=False))
    codec.decode_slots(other[..., 8:16], pool, b, first_decode=False)
    parts.append(codec.decode_slots(codes[..., 16:], pool, a, first_decode=False))
    torch.testing.assert_close(torch.cat(parts, -1), whole, atol=1e-10, rtol=0)


def test_state_layout_matches_the_network(model):
    codec = Qwen3OmniIncrementalCodec(model, kernels=oracle_kernels())
    lay = codec.layout
    hist = {k: n for k, _, n in lay.histories}
    assert hist["decoder.0"] == 6 and hist["decoder.final"] == 6
    assert hist["decoder.1.residual.2.conv1"] == 6 * 9 and hist["decoder.1.residual.0.conv2"] == 0
    ovl = {k: n for k, _, n in lay.overlaps}
    assert ovl["upsample.0.transconv"] == 0 and ovl["decoder.1.transconv"] == 8 and ovl["decoder.4.transconv"] == 3
    assert lay.retained == model.config.sliding_window - 1
    assert codec.samples_per_frame() == 1920


def test_the_ring_must_hold_the_window(model):
    codec = Qwen3OmniIncrementalCodec(model, kernels=oracle_kernels())
    pool = codec.make_pool(num_slots=1, ring_frames=codec.layout.retained + 4)
    codes = _codes(model, 1, 9)
    codec.decode_slots(codes[..., :4], pool, torch.tensor([0]), first_decode=True)
    with pytest.raises(ValueError):
        codec.decode_slots(codes[..., 4:], pool, torch.tensor([0]), first_decode=False)
