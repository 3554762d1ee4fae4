"""The implicit-GEMM causal conv (omni_conv1d_gemm, tcgen05) on the GPU.

- against an fp32 torch conv1d of the same bf16 operands over the code2wav's conv
  shapes (7-tap dilated convs at 1, 3 and 9; 1x1 convs; the transposed convs' GEMMs;
  C_in a multiple of 64 or of 32 only), lengths off the 128-position tile, the output
  written into a longer (padded) buffer: cosine >= 0.9999, max-abs <= 1e-2 x scale;
- the fused SnakeBeta epilogue bit-equal to the plain conv followed by
  omni_bias_snake_beta (with and without the residual and the stored sum): both round
  the conv to bf16 first and then follow the same rounding points.
"""

from __future__ import annotations

import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu
DEV = "cuda"

SHAPES = [
    # rows, length, C_in, C_out, taps, dilation
    (3, 200, 64, 96, 7, 1),
    (2, 130, 96, 96, 7, 9),
    (4, 40, 1024, 1536, 7, 1),
    (2, 320, 768, 768, 7, 3),
    (2, 77, 192, 192, 1, 1),
    (1, 500, 384, 384, 7, 9),
    (2, 20, 1536, 768 * 16, 1, 1),
    (5, 1, 96, 96, 7, 3),
]


def _case(rows, length, cin, cout, taps, dil, seed):
    g = torch.Generator(device=DEV).manual_seed(seed)
    hist = (taps - 1) * dil
    padded = torch.randn(rows, hist + length, cin, generator=g, device=DEV).to(torch.bfloat16)
    w = (torch.randn(cout, cin, taps, generator=g, device=DEV) / (cin * taps) ** 0.5).to(torch.bfloat16)
    w_mat = w.permute(0, 2, 1).reshape(cout, taps * cin).contiguous()
    return padded, w, w_mat, g


@pytest.mark.parametrize("shape", SHAPES, ids=[f"{s[2]}x{s[3]}k{s[4]}d{s[5]}" for s in SHAPES])
def test_conv_gemm_matches_fp32_conv(shape):
    from omni_b200 import ops

    rows, length, cin, cout, taps, dil = shape
    padded, w, w_mat, _ = _case(*shape, seed=sum(shape))
    # the output is the body of a longer buffer (a next conv's padded input with history 5)
    buf = torch.full((rows, 5 + length, cout), float("nan"), dtype=torch.bfloat16, device=DEV)
    out = buf[:, 5:]
    ops.conv1d_gemm(padded, w_mat, taps=taps, dilation=dil, length=length, out=out)
    torch.cuda.synchronize()
    ref = F.conv1d(padded.float().transpose(1, 2), w.float(), None, 1, 0, dil).transpose(1, 2)
    got = out.float()
    assert torch.isfinite(got).all()
    assert torch.isnan(buf[:, :5].float()).all(), "wrote outside the output rows"
    cos = F.cosine_similarity(got.flatten(), ref.flatten(), dim=0).item()
    err = (got - ref).abs().max().item()
    scale = ref.abs().max().item()
    assert cos >= 0.9999 and err <= 1e-2 * scale, (cos, err, scale)


@pytest.mark.parametrize("residual,sum_out", [(False, False), (True, True), (False, True)])
@pytest.mark.parametrize("shape", [(2, 300, 192, 192, 7, 3), (3, 50, 768, 384, 7, 1), (2, 129, 96, 96, 1, 1)])
def test_fused_snake_equals_conv_then_snake(shape, residual, sum_out):
    from omni_b200 import ops
    from omni_b200.kernels.bias_snake_beta import SnakeBetaCoefficients, fused_bias_snake_beta

    rows, length, cin, cout, taps, dil = shape
    padded, _, w_mat, g = _case(*shape, seed=7 + sum(shape))
    bias = (0.1 * torch.randn(cout, generator=g, device=DEV)).to(torch.bfloat16)
    coeff = SnakeBetaCoefficients(alpha_scale=(1 + 0.3 * torch.randn(cout, generator=g, device=DEV)).to(torch.bfloat16),
                                  inverse_beta=(1 + 0.3 * torch.rand(cout, generator=g, device=DEV)).to(torch.bfloat16))
    res = torch.randn(rows, length, cout, generator=g, device=DEV).to(torch.bfloat16) if residual else None
    y = torch.empty(rows, length, cout, dtype=torch.bfloat16, device=DEV)
    ops.conv1d_gemm(padded, w_mat, taps=taps, dilation=dil, length=length, out=y)
    want = torch.empty_like(y)
    want_sum = torch.empty_like(y) if sum_out else None
    fused_bias_snake_beta(y, bias, coeff, want, residual=res, sum_out=want_sum)
    got = torch.empty_like(y)
    got_sum = torch.empty_like(y) if sum_out else None
    ops.conv1d_gemm(padded, w_mat, taps=taps, dilation=dil, length=length, out=got, bias=bias,
                    alpha_scale=coeff.alpha_scale, inverse_beta=coeff.inverse_beta, residual=res, sum_out=got_sum)
    torch.cuda.synchronize()
    assert torch.equal(got, want)
    if sum_out:
        assert torch.equal(got_sum, want_sum)
    from omni_b200 import device_status

    assert device_status() == 0
