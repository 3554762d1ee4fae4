"""The C-ABI library loads and exports every entry point include/omni_b200.h declares.

No compute call is made here (CPU-only test); only symbol presence and the
pure-host entry points.
"""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent


def declared_symbols() -> list[str]:
    text = "\n".join(p.read_text() for p in sorted((ROOT / "include").glob("*.h")))
    return sorted(set(re.findall(r"OMNI_API\s+[\w\s\*]+?\b(omni_\w+)\s*\(", text)))


def test_header_declares_entry_points():
    names = declared_symbols()
    assert "omni_sample_topk_topp" in names and "omni_version" in names


def test_library_exports_every_declared_symbol():
    from omni_b200 import _lib

    lib = _lib.load()
    for name in declared_symbols():
        assert hasattr(lib, name), f"{name} declared in include/ but not exported"
        assert name in _lib.SIGNATURES, f"{name} has no ctypes signature"


def test_version_and_error_string():
    from omni_b200 import _lib

    lib = _lib.load()
    assert b"sm_100a" in lib.omni_version()
    assert isinstance(lib.omni_last_error(), bytes)


def test_unsupported_contract_is_reported_without_launch():
    """An off-ladder width is rejected on the host before any device work."""
    from omni_b200 import _lib

    lib = _lib.load()
    rc = lib.omni_sample_topk_topp(None, 4, 2048, 2048, None, None, None, None, None, 7, 0, None, None)
    assert rc == _lib.OMNI_ERR_UNSUPPORTED
    assert "ladder" in _lib.last_error()
    assert lib.omni_sample_sorted_seeded(None, None, 1, 0, None, None, None, None) == _lib.OMNI_ERR_UNSUPPORTED
    assert ctypes.sizeof(ctypes.c_void_p) == 8


def test_torch_ops_are_registered_with_their_schemas():
    """The TORCH_LIBRARY layer loads and registers every op with the reference-shaped
    schema; the fake kernels let torch trace calls without a GPU."""
    import torch
    from torch._subclasses.fake_tensor import FakeTensorMode

    from omni_b200 import torch_ops

    torch_ops.load()
    schemas = {n: str(getattr(torch.ops.omni_b200, n).default._schema) for n in torch_ops.OPS}
    assert "int max_top_k, bool has_top_p) -> Tensor" in schemas["sample_topk_topp"]
    assert "Tensor(a!) x, Tensor(b!) residual, Tensor weight, float eps) -> ()" in schemas["add_rmsnorm_rounded"]
    assert "-> bool" in schemas["gather_codec_embedding_and_add"]
    with FakeTensorMode():
        logits = torch.empty(5, 2048, dtype=torch.bfloat16)
        f = torch.empty(5, dtype=torch.float32)
        i = torch.empty(5, dtype=torch.long)
        out = torch.ops.omni_b200.sample_topk_topp(logits, f, i, f, i, i, 50, True)
        assert out.shape == (5,) and out.dtype == torch.long
        summed = torch.empty(5, 1024, dtype=torch.bfloat16)
        nxt = torch.ops.omni_b200.codebook_step(logits, torch.empty(2048, 1024, dtype=torch.bfloat16), i, summed)
        assert nxt.shape == (5, 1, 1024)
