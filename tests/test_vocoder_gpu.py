"""GPU parity of the vocoder-step kernels (through the C ABI) with the eager ops and the
oracle, mirroring the reference's kernel tests (tests/unit_test/kernels/)."""

from __future__ import annotations

import pytest
import torch

from oracle import vocoder as ov

pytestmark = pytest.mark.gpu
DEV = "cuda"


def eager_snake(x, alpha, beta, eps=1e-9):
    a = torch.exp(alpha)
    b = torch.exp(beta)
    return x + (1.0 / (b + eps)) * torch.pow(torch.sin(x * a), 2)


class _Snake:
    def __init__(self, channels, dtype):
        self.alpha = (torch.randn(channels, device=DEV) * 0.5).to(dtype)
        self.beta = (torch.randn(channels, device=DEV) * 0.5).to(dtype)
        self.no_div_by_zero = 1e-9


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("channels", [96, 1536])
@pytest.mark.parametrize("with_residual,with_sum", [(False, False), (False, True), (True, False), (True, True)])
def test_bias_snake_matches_the_eager_adds_and_snake(dtype, channels, with_residual, with_sum):
    from omni_b200.kernels.bias_snake_beta import SnakeBetaCoefficients, fused_bias_snake_beta

    torch.manual_seed(0)
    act = _Snake(channels, dtype)
    conv_buffer = torch.randn(3, 41, channels, device=DEV, dtype=dtype)
    conv_output = conv_buffer[:, 2:39]
    bias = torch.randn(channels, device=DEV, dtype=dtype)
    residual = torch.randn(3, 37, channels, device=DEV, dtype=dtype)
    padded_input = torch.zeros(3, 46, channels, device=DEV, dtype=dtype)
    sum_out = torch.zeros(3, 37, channels, device=DEV, dtype=dtype)
    fused_bias_snake_beta(conv_output, bias, SnakeBetaCoefficients.from_activation(act), padded_input[:, 6:43],
                          residual=residual if with_residual else None, sum_out=sum_out if with_sum else None)
    torch.cuda.synchronize()
    expected_sum = conv_output + bias + residual if with_residual else conv_output + bias
    expected = eager_snake(expected_sum, act.alpha, act.beta)
    assert torch.equal(padded_input[:, 6:43], expected)
    assert not padded_input[:, :6].any() and not padded_input[:, 43:].any()
    assert torch.equal(sum_out, expected_sum) if with_sum else not sum_out.any()
    # the CPU oracle (torch.sin on the host) agrees to within one unit of the last place
    ref, _ = ov.snake_beta(conv_output.cpu(), bias.cpu(), torch.exp(act.alpha).cpu(),
                           (1.0 / (torch.exp(act.beta) + 1e-9)).cpu(), residual.cpu() if with_residual else None)
    got = padded_input[:, 6:43].cpu()
    diff = (got.float() - ref.float()).abs()
    ulp = ref.float().abs().clamp(min=1e-3) * (2.0 ** -7 if dtype == torch.bfloat16 else 2.0 ** -10)
    assert (diff <= ulp).all()


def _conv(channels, dtype, taps=7):
    conv = torch.nn.Conv1d(channels, 1, taps).to(device=DEV, dtype=dtype)
    return conv


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("channels", [8, 96])
def test_single_output_conv_is_the_clamped_conv_rounded_once(dtype, channels):
    from omni_b200.kernels.single_output_conv import clamped_single_output_conv

    torch.manual_seed(0)
    conv = _conv(channels, dtype)
    padded = torch.randn(3, 300 + 6, channels, device=DEV, dtype=dtype)
    with torch.inference_mode():
        actual = clamped_single_output_conv(padded, conv, 300)
    expected = ov.single_output_conv(padded.cpu(), conv.weight.detach().cpu(), conv.bias.detach().cpu(), 300)
    assert actual.shape == (3, 1, 300) and actual.is_contiguous()
    assert (expected.abs() == 1).any() and (expected.abs() < 1).any()
    torch.testing.assert_close(actual.cpu(), expected)


def test_single_output_conv_gives_a_position_the_same_bits_in_any_split():
    from omni_b200.kernels.single_output_conv import clamped_single_output_conv

    torch.manual_seed(0)
    conv = _conv(96, torch.bfloat16)
    padded = torch.randn(3, 1000 + 6, 96, device=DEV, dtype=torch.bfloat16)
    with torch.inference_mode():
        whole = clamped_single_output_conv(padded, conv, 1000)
        parts = torch.cat([clamped_single_output_conv(padded[:, :417 + 6], conv, 417),
                           clamped_single_output_conv(padded[:, 417:], conv, 583)], dim=-1)
        row = clamped_single_output_conv(padded[1:2], conv, 1000)
    assert torch.equal(parts, whole)
    assert torch.equal(row, whole[1:2])


@pytest.mark.parametrize("history", [2, 6, 54])
@pytest.mark.parametrize("chunks", [(10, 10, 7), (1, 2, 1, 3, 40), (32, 1, 32)])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_history_exchange_matches_the_oracle(history, chunks, dtype):
    from omni_b200.kernels.codec_state import history_exchange

    g = torch.Generator().manual_seed(history + len(chunks))
    slots, C, tail = 5, 70, 3  # two channel blocks
    total = sum(chunks)
    streams = torch.randn(slots, total, C, generator=g).to(dtype)
    pool_dev = torch.randn(slots, history, C, generator=g).to(dtype).to(DEV)
    pool_ref = pool_dev.cpu().clone()
    slot_index = torch.tensor([3, 0, 4])
    start = 0
    for i, n in enumerate(chunks):
        padded = torch.full((3, history + n + tail, C), 7.0).to(dtype)
        padded[:, history:history + n] = streams[slot_index, start:start + n]
        dev = padded.to(DEV)
        history_exchange(dev, pool_dev, slot_index.to(DEV), n, is_cold=i == 0)
        ov.history_exchange(padded, pool_ref, slot_index, n, is_cold=i == 0)
        torch.cuda.synchronize()
        assert torch.equal(dev.cpu(), padded)
        assert torch.equal(pool_dev.cpu(), pool_ref)
        start += n


@pytest.mark.parametrize("overlap,emitted", [(3, 5), (4, 4), (12, 40)])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
def test_overlap_exchange_matches_the_oracle(overlap, emitted, dtype):
    from omni_b200.kernels.codec_state import overlap_exchange

    g = torch.Generator().manual_seed(overlap)
    rows, C = 3, 130
    pool_dev = torch.randn(4, overlap, C, generator=g).to(dtype).to(DEV)
    pool_ref = pool_dev.cpu().clone()
    slot = torch.tensor([2, 0, 3])
    for k in range(3):
        out = torch.randn(rows, emitted + overlap, C, generator=g).to(dtype)
        dev = out.to(DEV)
        overlap_exchange(dev, pool_dev, slot.to(DEV), emitted, is_cold=k == 0)
        ov.overlap_exchange(out, pool_ref, slot, emitted, is_cold=k == 0)
        torch.cuda.synchronize()
        assert torch.equal(dev.cpu(), out)
        assert torch.equal(pool_dev.cpu(), pool_ref)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("channels,taps,dilation", [(96, 7, 1), (384, 7, 3), (768, 7, 9), (8, 7, 9), (192, 1, 1)])
def test_conv_window_gather_is_the_strided_window_copy(dtype, channels, taps, dilation):
    from omni_b200.kernels.conv_window import conv_window_gather

    torch.manual_seed(0)
    rows, length = 5, 37
    history = (taps - 1) * dilation
    padded = torch.randn(rows, history + length, channels, device=DEV).to(dtype)
    got = conv_window_gather(padded, length, taps, dilation)
    want = padded.as_strided((rows, length, taps, channels), (padded.stride(0), channels, dilation * channels, 1))
    assert torch.equal(got, want.reshape(rows * length, taps * channels))


def test_conv_window_gather_rejects_a_short_input():
    from omni_b200.kernels.conv_window import conv_window_gather

    padded = torch.zeros(2, 10, 96, device=DEV, dtype=torch.bfloat16)
    with pytest.raises(ValueError):
        conv_window_gather(padded, 8, 7, 1)
