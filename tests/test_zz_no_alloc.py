"""The allocation-free paged attention entry point against the workspace one.

omni_paged_decode_attention_noalloc exists for callers that may not allocate
device memory (a host that owns all device memory, a real-time audio thread
that must not block in cudaMalloc): it draws its scratch from an array built
into the library.  This test calls it twice in a row through the C ABI on two
different cases (other lengths, row count, range split and seed), so that the
second call runs over the first call's leftovers in the shared array, and
requires each output to equal, bit for bit, omni_paged_decode_attention's on
the same case with a caller-provided workspace (both run the same kernels on
the same inputs).  With two or more GPUs it repeats the check on device 1 after
device 0, since the array, its address and the kernel's shared-memory
attribute are per device.  It is collected last so that a run stopping at the
first failure has already run every other test; it also passes alone in a fresh
process.
"""

from __future__ import annotations

import math

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _paged_case(lens, ppc, seed, dev=DEV):
    gen = torch.Generator().manual_seed(seed)
    hq, hkv, d, page = 16, 2, 128, 16
    npages = [(L + page - 1) // page for L in lens]
    pool_pages = int(sum(npages) * 1.25) + 4
    perm = torch.randperm(pool_pages, generator=gen)[: sum(npages)].to(torch.int32)
    kc = torch.randn(pool_pages * page, hkv, d, generator=gen).to(torch.bfloat16).to(dev)
    vc = torch.randn(pool_pages * page, hkv, d, generator=gen).to(torch.bfloat16).to(dev)
    q = torch.randn(len(lens), hq, d, generator=gen).to(torch.bfloat16).to(dev)
    page_indptr = torch.tensor(np.concatenate([[0], np.cumsum(npages)]), dtype=torch.int32, device=dev)
    work = [(n + ppc - 1) // ppc for n in npages]
    work_indptr = torch.tensor(np.concatenate([[0], np.cumsum(work)]), dtype=torch.int32, device=dev)
    seq = torch.tensor(lens, dtype=torch.int64, device=dev)
    return dict(q=q, kc=kc, vc=vc, page_indptr=page_indptr, page_indices=perm.to(dev), seq=seq,
                work_indptr=work_indptr, cap=int(sum(work)), hq=hq, hkv=hkv, d=d, page=page)


def _run_pair(lib, c, ppc, ctas, dev):
    """(workspace-path output, no-alloc output) of one case on device dev."""
    from omni_b200 import _lib

    rows = c["seq"].shape[0]
    scale = 1.0 / math.sqrt(c["d"])
    with torch.cuda.device(dev):
        stream = torch.cuda.current_stream().cuda_stream
        common = (c["q"].data_ptr(), c["q"].stride(0), c["kc"].data_ptr(), c["vc"].data_ptr(),
                  c["page_indptr"].data_ptr(), c["page_indices"].data_ptr(), c["seq"].data_ptr(),
                  c["work_indptr"].data_ptr(), rows, c["hq"], c["hkv"], c["d"], c["page"], ppc, c["cap"], scale)
        ws_bytes = lib.omni_paged_attention_workspace_bytes(rows, c["hkv"], c["cap"])
        ws = torch.zeros(ws_bytes, dtype=torch.uint8, device=dev)
        ref = torch.empty(rows, c["hq"], c["d"], dtype=torch.bfloat16, device=dev)
        rc = lib.omni_paged_decode_attention(*common, ref.data_ptr(), ref.stride(0), ws.data_ptr(), ws_bytes, ctas,
                                             stream)
        assert rc == 0, _lib.last_error()
        out = torch.full_like(ref, float("nan"))
        rc = lib.omni_paged_decode_attention_noalloc(*common, out.data_ptr(), out.stride(0), ctas, stream)
        assert rc == 0, _lib.last_error()
        torch.cuda.synchronize(dev)
    return ref, out


CASES = [
    # (lengths, pages_per_chunk, grid_ctas, seed)
    ([1, 15, 16, 17, 100, 1000, 8192, 33, 556, 64], 1, 0, 1),
    ([4000, 2, 700, 16, 129, 3333, 48, 5000, 1, 250, 900, 77, 1500], 8, 37, 2),
]


def _check_device(dev):
    from omni_b200 import _lib

    lib = _lib.load()
    for lens, ppc, ctas, seed in CASES:
        c = _paged_case(lens, ppc, seed, dev)
        ref, out = _run_pair(lib, c, ppc, ctas, dev)
        assert torch.isfinite(ref.float()).all()
        assert torch.equal(out, ref), (lens, (out.float() - ref.float()).abs().max().item())


def test_noalloc_attention_matches_workspace_entry_point():
    """Two different cases in a row on device 0, each bit-equal to the workspace path."""
    _check_device("cuda:0")


def test_noalloc_attention_on_a_second_device():
    """The per-device array, address and kernel attribute: device 1 after device 0."""
    if torch.cuda.device_count() < 2:
        pytest.skip("one GPU visible")
    _check_device("cuda:0")
    _check_device("cuda:1")


def test_noalloc_attention_rejects_scratch_beyond_its_array():
    from omni_b200 import _lib

    lib = _lib.load()
    rc = lib.omni_paged_decode_attention_noalloc(None, 0, None, None, None, None, None, None, 64, 16, 2, 128, 16, 1,
                                                 1 << 20, 0.088, None, 0, 0, None)
    assert rc == _lib.OMNI_ERR_CAPACITY
    assert "8 MiB" in _lib.last_error()
    # a size whose byte count would overflow is refused as invalid, not wrapped
    rc = lib.omni_paged_decode_attention_noalloc(None, 0, None, None, None, None, None, None, 64, 16, 2, 128, 16, 1,
                                                 1 << 56, 0.088, None, 0, 0, None)
    assert rc == _lib.OMNI_ERR_INVALID
