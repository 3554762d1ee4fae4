"""Shared pieces of the code2wav tests: a small random-weight transformers
Qwen3OmniMoeCode2Wav (the reference's code2wav network, code2wav.py:326-376 subclasses
it) and the oracle kernels behind the incremental decoder's kernel interface."""

from __future__ import annotations

from types import SimpleNamespace

import torch

from oracle import vocoder as ov


# decoder_dim 128: the last decoder block has 8 channels, the fewest the library's
# SnakeBeta kernel takes (16-byte vectors of bf16)
def small_code2wav(seed: int = 0, *, hidden=64, heads=4, kv_heads=2, layers=2, window=8, quantizers=4,
                   codebook=32, decoder_dim=128, rates=(8, 5, 4, 3), gain=1.0):
    from transformers.models.qwen3_omni_moe.configuration_qwen3_omni_moe import Qwen3OmniMoeCode2WavConfig
    from transformers.models.qwen3_omni_moe.modeling_qwen3_omni_moe import Qwen3OmniMoeCode2Wav

    cfg = Qwen3OmniMoeCode2WavConfig(
        codebook_size=codebook, hidden_size=hidden, num_attention_heads=heads, num_key_value_heads=kv_heads,
        num_hidden_layers=layers, intermediate_size=2 * hidden, sliding_window=window, num_quantizers=quantizers,
        decoder_dim=decoder_dim, upsample_rates=list(rates), upsampling_ratios=[2, 2])
    cfg._attn_implementation = "sdpa"
    torch.manual_seed(seed)
    model = Qwen3OmniMoeCode2Wav(cfg).eval()
    g = torch.Generator().manual_seed(seed)
    with torch.no_grad():
        for name, p in model.named_parameters():
            if name.endswith(("alpha", "beta")):
                p.copy_(0.3 * torch.randn(p.shape, generator=g))
            elif name.endswith("scale") or name.endswith("gamma"):
                p.copy_(0.5 + 0.5 * torch.rand(p.shape, generator=g))
            elif p.dim() == 1:
                p.copy_(0.1 * torch.randn(p.shape, generator=g) + (1.0 if "norm" in name else 0.0))
            else:
                fan_in = p[0].numel() if "code_embedding" not in name else 1
                p.copy_(gain * torch.randn(p.shape, generator=g) / max(fan_in, 1) ** 0.5)
        # the residual stacks grow the activations: scale the last conv so that the
        # waveform of a probe sequence sits mostly inside the clamp
        final = model.decoder[-1].conv
        seen = []
        hook = final.register_forward_hook(lambda m, i, o: seen.append(o))
        model(torch.randint(0, codebook, (1, quantizers, 24), generator=g))
        hook.remove()
        final.bias.zero_()
        final.weight.mul_(0.3 / float(seen[0].std()))
    return model


def oracle_kernels() -> SimpleNamespace:
    def coefficients(act):
        return SimpleNamespace(alpha_scale=torch.exp(act.alpha),
                               inverse_beta=1.0 / (torch.exp(act.beta) + act.no_div_by_zero))

    def snake(conv_output, bias, coeff, out, *, residual=None, sum_out=None):
        o, s = ov.snake_beta(conv_output, bias, coeff.alpha_scale, coeff.inverse_beta, residual)
        if sum_out is not None:
            sum_out.copy_(s)
        out.copy_(o)

    def single(padded, conv, length):
        return ov.single_output_conv(padded, conv.weight, conv.bias, length)

    def windows(padded, length, taps, dilation):
        rows, samples, ch = padded.shape
        view = padded.as_strided((rows, length, taps, ch), (padded.stride(0), ch, dilation * ch, 1),
                                 padded.storage_offset())
        return view.reshape(rows * length, taps * ch)

    return SimpleNamespace(coefficients=coefficients, snake=snake, history_exchange=ov.history_exchange,
                           overlap_exchange=ov.overlap_exchange, single_output_conv=single, conv_windows=windows)


def decode_in_chunks(codec, pool, codes: torch.Tensor, slots: torch.Tensor, splits) -> torch.Tensor:
    """The streams' waveform from decodes of `splits` frames each, concatenated."""
    out, t = [], 0
    for i, n in enumerate(splits):
        out.append(codec.decode_slots(codes[..., t:t + n], pool, slots, first_decode=i == 0))
        t += n
    assert t == codes.shape[-1]
    return torch.cat(out, dim=-1)
