"""The allocation-free paged attention entry point against the workspace one.

omni_paged_decode_attention_noalloc exists for callers that may not allocate
device memory (a host that owns all device memory, a real-time audio thread
that must not block in cudaMalloc): it draws its scratch from an array built
into the library.  This test calls it twice in a row through the C ABI — the
second call checks that the shared array's merge counters start at zero again —
and compares each output with omni_paged_decode_attention's, which uses a
caller-provided workspace, within the attention tolerance of the other tests.
It is collected last so that a run stopping at the first failure has already
run every other test; it also passes alone in a fresh process.
"""

from __future__ import annotations

import math

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _paged_case(lens, ppc, seed):
    gen = torch.Generator().manual_seed(seed)
    hq, hkv, d, page = 16, 2, 128, 16
    npages = [(L + page - 1) // page for L in lens]
    pool_pages = int(sum(npages) * 1.25) + 4
    perm = torch.randperm(pool_pages, generator=gen)[: sum(npages)].to(torch.int32)
    kc = torch.randn(pool_pages * page, hkv, d, generator=gen).to(torch.bfloat16).to(DEV)
    vc = torch.randn(pool_pages * page, hkv, d, generator=gen).to(torch.bfloat16).to(DEV)
    q = torch.randn(len(lens), hq, d, generator=gen).to(torch.bfloat16).to(DEV)
    page_indptr = torch.tensor(np.concatenate([[0], np.cumsum(npages)]), dtype=torch.int32, device=DEV)
    work = [(n + ppc - 1) // ppc for n in npages]
    work_indptr = torch.tensor(np.concatenate([[0], np.cumsum(work)]), dtype=torch.int32, device=DEV)
    seq = torch.tensor(lens, dtype=torch.int64, device=DEV)
    return dict(q=q, kc=kc, vc=vc, page_indptr=page_indptr, page_indices=perm.to(DEV), seq=seq,
                work_indptr=work_indptr, cap=int(sum(work)), hq=hq, hkv=hkv, d=d, page=page)


def _close(got, ref, rel=2e-2, cos_min=0.999):
    g, r = got.float().flatten(), ref.float().flatten()
    assert torch.isfinite(g).all()
    cos = torch.nn.functional.cosine_similarity(g, r, dim=0).item()
    err = (g - r).abs().max().item()
    assert cos >= cos_min and err <= rel * r.abs().max().item() + 1e-6, (cos, err)


@pytest.mark.parametrize("ppc", [1, 8])
def test_noalloc_attention_matches_workspace_entry_point(ppc):
    from omni_b200 import _lib

    lib = _lib.load()
    c = _paged_case([1, 15, 16, 17, 100, 1000, 8192, 33, 556, 64], ppc, seed=ppc)
    rows = c["seq"].shape[0]
    scale = 1.0 / math.sqrt(c["d"])
    stream = torch.cuda.current_stream().cuda_stream
    common = (c["q"].data_ptr(), c["q"].stride(0), c["kc"].data_ptr(), c["vc"].data_ptr(), c["page_indptr"].data_ptr(),
              c["page_indices"].data_ptr(), c["seq"].data_ptr(), c["work_indptr"].data_ptr(), rows, c["hq"], c["hkv"],
              c["d"], c["page"], ppc, c["cap"], scale)
    ws_bytes = lib.omni_paged_attention_workspace_bytes(rows, c["hkv"], c["cap"])
    ws = torch.zeros(ws_bytes, dtype=torch.uint8, device=DEV)
    ref = torch.empty(rows, c["hq"], c["d"], dtype=torch.bfloat16, device=DEV)
    rc = lib.omni_paged_decode_attention(*common, ref.data_ptr(), ref.stride(0), ws.data_ptr(), ws_bytes, 0, stream)
    assert rc == 0, _lib.last_error()
    for _ in range(2):
        out = torch.full_like(ref, float("nan"))
        rc = lib.omni_paged_decode_attention_noalloc(*common, out.data_ptr(), out.stride(0), 0, stream)
        assert rc == 0, _lib.last_error()
        torch.cuda.synchronize()
        _close(out, ref)


def test_noalloc_attention_rejects_scratch_beyond_its_array():
    from omni_b200 import _lib

    lib = _lib.load()
    rc = lib.omni_paged_decode_attention_noalloc(None, 0, None, None, None, None, None, None, 64, 16, 2, 128, 16, 1,
                                                 1 << 20, 0.088, None, 0, 0, None)
    assert rc == _lib.OMNI_ERR_CAPACITY
    assert "8 MiB" in _lib.last_error()
