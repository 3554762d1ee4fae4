"""Paged KV pool, request-to-token table and page allocator, resident in HBM.

The layout follows sglang's MHATokenToKVPool / ReqToTokenPool that the
reference's talker writes through (thinker_model.py:314-345, base.py:577-623):
per layer K and V buffers of [slots, kv_heads, head_dim] with slot =
page * page_size + offset, and req_to_token[req, position] = slot.  The free
page list lives on the device (omni_decode_prepare pops it in row order); the
host mirrors only the count, so admission checks need no device read.
"""

from __future__ import annotations

import torch


class PagedKVPool:
    def __init__(self, *, num_layers: int, num_pages: int, page_size: int, num_kv_heads: int, head_dim: int,
                 device, dtype=torch.bfloat16):
        self.num_layers = num_layers
        self.num_pages = num_pages
        self.page_size = page_size
        slots = num_pages * page_size
        self.k_buffer = torch.zeros(num_layers, slots, num_kv_heads, head_dim, dtype=dtype, device=device)
        self.v_buffer = torch.zeros(num_layers, slots, num_kv_heads, head_dim, dtype=dtype, device=device)

    @property
    def bytes_per_token_per_layer(self) -> int:
        return 2 * self.k_buffer.shape[2] * self.k_buffer.shape[3] * self.k_buffer.element_size()


class ReqToTokenPool:
    def __init__(self, *, max_reqs: int, max_context: int, device):
        self.req_to_token = torch.zeros(max_reqs, max_context, dtype=torch.int32, device=device)


class PageAllocator:
    """A stack of free page ids on the device, consumed by omni_decode_prepare."""

    def __init__(self, free_pages: torch.Tensor, device):
        self.free_pages = free_pages.to(device=device, dtype=torch.int32).contiguous()
        self.free_head = torch.zeros(1, dtype=torch.int64, device=device)
        self.host_head = 0

    @property
    def available(self) -> int:
        return self.free_pages.shape[0] - self.host_head

    def reserve_host(self, seq_lens_host, page_size: int) -> int:
        """Pages the next decode step opens (rows whose new token starts a page);
        raises when the pool cannot hold them (capacity, as the reference's allocator)."""
        need = sum(1 for L in seq_lens_host if L % page_size == 0)
        if need > self.available:
            raise RuntimeError("KV pool exhausted: no free page for the next decode step")
        self.host_head += need
        return need

    def alloc_prefix(self, n: int) -> torch.Tensor:
        """Take n pages on the host side (prefill of synthetic contexts)."""
        if n > self.available:
            raise RuntimeError("KV pool exhausted")
        pages = self.free_pages[self.host_head: self.host_head + n]
        self.host_head += n
        self.free_head.fill_(self.host_head)
        return pages
