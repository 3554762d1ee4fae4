"""torch.ops.omni_b200.*: the dispatcher-registered drop-in kernels.

Loads libomni_torch_ops.so (sglang-omni_b200/torch_ext/omni_torch_ops.cpp, a
TORCH_LIBRARY over libomni_b200.so's C ABI) and registers a fake (meta) kernel for
each op so that torch.compile can trace calls without running them.  The ops:

- ``sample_topk_topp(logits, temperatures, top_ks, top_ps, seeds, positions, max_top_k, has_top_p) -> Tensor``
- ``gather_codec_embedding_and_add(token_ids, embedding_weight, gathered!, accumulated!) -> bool``
- ``codebook_step(logits, embedding_weight, codes!, summed!) -> Tensor``
- ``add_rmsnorm_rounded(x!, residual!, weight, eps) -> ()``
- ``paged_decode_attention(q, k_cache, v_cache, page_indptr, page_indices, seq_lens, sm_scale, out!, workspace!, work_capacity) -> ()``
- ``linear(x, w, out!, epilogue, residual=None) -> ()``

(``!`` = written in place.)  The library is built by sglang-omni_b200/build.py
(build_torch_ops); a missing library raises, there is no fallback.
"""

from __future__ import annotations

import torch

from omni_b200 import _lib

LIB_PATH = _lib.LIB_PATH.parent / "libomni_torch_ops.so"
_loaded = False


def load() -> None:
    """Load the operator library once (after libomni_b200.so, which it links)."""
    global _loaded
    if _loaded:
        return
    if not LIB_PATH.exists():
        raise RuntimeError(f"omni_b200 torch op library not found at {LIB_PATH}; build it with "
                           "`python sglang-omni_b200/build.py`")
    _lib.load()
    torch.ops.load_library(str(LIB_PATH))
    _register_fakes()
    _loaded = True


def _register_fakes() -> None:
    reg = torch.library.register_fake

    @reg("omni_b200::sample_topk_topp")
    def _(logits, temperatures, top_ks, top_ps, seeds, positions, max_top_k, has_top_p):
        return logits.new_empty((logits.shape[0],), dtype=torch.long)

    @reg("omni_b200::gather_codec_embedding_and_add")
    def _(token_ids, embedding_weight, gathered, accumulated):
        return True

    @reg("omni_b200::codebook_step")
    def _(logits, embedding_weight, codes, summed):
        return summed.new_empty((logits.shape[0], 1, embedding_weight.shape[1]))

    @reg("omni_b200::add_rmsnorm_rounded")
    def _(x, residual, weight, eps):
        return None

    @reg("omni_b200::paged_decode_attention")
    def _(q, k_cache, v_cache, page_indptr, page_indices, seq_lens, sm_scale, out, workspace, work_capacity):
        return None

    @reg("omni_b200::linear")
    def _(x, w, out, epilogue, residual=None):
        return None


OPS = ("sample_topk_topp", "gather_codec_embedding_and_add", "codebook_step", "add_rmsnorm_rounded",
       "paged_decode_attention", "linear")
