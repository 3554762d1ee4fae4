"""A bounded device wait that runs out ends the kernel with a status, not a hang.

Every spin in the library's kernels is an mbarrier wait with a poll limit: on
timeout the waiting warp records a status word, the CTA skips its remaining
work, frees its tensor memory and returns.  omni_gemm_wait_probe launches the
real tcgen05 GEMM kernel with a producer that issues no copies (nothing is in
flight) and a short poll limit, so that the MMA warp's wait for its first stages
and the producer's wait for a free stage both run out.  The test checks that the
launch returns, that omni_device_status reports the timeout, and that after a
status reset the same GEMM, run normally, is correct with a clean status word.
"""

from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("splits", [1, 4])
def test_gemm_wait_runs_out_and_the_next_call_succeeds(splits):
    from omni_b200 import _lib, ops

    lib = _lib.load()
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(3)
    rows, k, n = 64, 1024, 512
    x = torch.randn(rows, k, generator=g, device=dev).to(torch.bfloat16)
    w = (torch.randn(n, k, generator=g, device=dev) * 0.02).to(torch.bfloat16)
    y = torch.full((rows, n), 7.0, dtype=torch.bfloat16, device=dev)
    torch.cuda.synchronize()
    _lib.device_status(reset=True)
    rc = lib.omni_gemm_wait_probe(x.data_ptr(), rows, k, w.data_ptr(), n, y.data_ptr(), splits, 2000,
                                  torch.cuda.current_stream().cuda_stream)
    assert rc == 0, _lib.last_error()
    torch.cuda.synchronize()  # the kernel returned
    status = _lib.device_status(reset=True)
    assert status in (_lib.OMNI_DEV_TIMEOUT_TMA, _lib.OMNI_DEV_TIMEOUT_MMA), hex(status)
    assert bool((y == 7.0).all()), "an aborted GEMM must not store"
    assert _lib.device_status() == 0
    # the context is intact: the normal GEMM on the same operands is right
    out = torch.empty(rows, n, dtype=torch.bfloat16, device=dev)
    ops.linear(x, w, out=out, splits=splits)
    torch.cuda.synchronize()
    ref = x.float() @ w.float().t()
    cos = torch.nn.functional.cosine_similarity(out.float().flatten(), ref.flatten(), dim=0).item()
    assert cos >= 0.9999, cos
    assert _lib.device_status() == 0


def test_probe_rejects_a_zero_limit():
    from omni_b200 import _lib

    lib = _lib.load()
    assert lib.omni_gemm_wait_probe(None, 64, 1024, None, 512, None, 1, 0, None) == _lib.OMNI_ERR_INVALID
