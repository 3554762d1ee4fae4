"""Host restatements of two pieces of csrc/prefill_attention.cu and csrc/common.cuh
that the GPU parity tests only see through their results.

* f2_to_bf2 (common.cuh): the softmax packs P to bf16 by Veltkamp splitting,
  g = v * (2^16 + 1), hi = g + (v - g), in float32 round-to-nearest arithmetic.
  Its claim is bit-identity with the round-to-nearest-even conversion of
  pack_bf2 for zero and every normal float32; checked here over whole binades
  (each 2^23 values), ties included, with numpy's float32 arithmetic, which
  rounds like the device's .rn forms.
* block_work (prefill_attention.cu): the CTA of linear grid index w serves query
  tile total - 1 - w // heads and head slot w % heads.  Every (tile, slot) is
  served exactly once, CTAs beyond total * heads do nothing, and the tiles start
  last to first.
"""

from __future__ import annotations

import numpy as np
import pytest


def veltkamp_bf16(u: np.ndarray) -> np.ndarray:
    x = u.view(np.float32)
    g = (x * np.float32(65537.0)).astype(np.float32)
    d = (x - g).astype(np.float32)
    return ((g + d).astype(np.float32)).view(np.uint32)


def rne_bf16(u: np.ndarray) -> np.ndarray:
    return (u + np.uint32(0x7FFF) + ((u >> 16) & np.uint32(1))) & np.uint32(0xFFFF0000)


@pytest.mark.parametrize("exponent", [-126, -125, -40, -9, -1, 0, 7, 8])
def test_veltkamp_pack_is_round_to_nearest_even(exponent):
    u = np.uint32((exponent + 127) << 23) + np.arange(1 << 23, dtype=np.uint32)
    got = veltkamp_bf16(u)
    assert np.all((got & np.uint32(0xFFFF)) == 0)
    np.testing.assert_array_equal(got, rne_bf16(u))


def test_veltkamp_pack_of_zero():
    z = np.zeros(1, np.uint32)
    np.testing.assert_array_equal(veltkamp_bf16(z), z)


def block_work(w: int, total: int, heads: int):
    if w >= total * heads:
        return None
    return total - 1 - w // heads, w % heads


@pytest.mark.parametrize("total,heads,max_tiles", [(0, 8, 4), (1, 1, 1), (37, 8, 40), (302, 8, 302), (5, 3, 9)])
def test_block_work_covers_each_tile_once(total, heads, max_tiles):
    seen = []
    for y in range(heads):
        for x in range(max_tiles):
            item = block_work(y * max_tiles + x, total, heads)
            if item is not None:
                seen.append(item)
    assert sorted(seen) == [(t, h) for t in range(total) for h in range(heads)]
    tiles = [t for t, _ in seen]
    assert tiles == sorted(tiles, reverse=True)
