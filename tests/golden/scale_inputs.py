"""Seeded inputs of the large residual-sampler golden (shared by its generator and its tests).

Each case draws `rows` rows of N(0, sigma^2) logits rounded to bf16 whose top_k + 1
largest values are distinct and above the rest of the row ("untied": a tie inside the
sampler's top-k window would make torch's CPU top-k order, the CUDA network's order
and the reference's Triton order legitimately differ); colliding values in the window
are pushed down to the next free bf16 value, keeping their order.
Seeds are uniform over the positive int32 range and positions follow the
predictor's layout pos = semantic_pos * (G - 1) + (j + 1).
"""

from __future__ import annotations

import numpy as np

# (name, rows, vocab, temperature, top_k, top_p, codebooks G, sigma, rng seed)
SCALE_CASES = [
    ("config0", 12000, 2048, 0.9, 50, 0.8, 16, 2.5, 2024),
    ("config3", 12000, 1024, 0.9, 50, 0.8, 32, 2.5, 2025),
]


def _bf16_keys(bits: np.ndarray) -> np.ndarray:
    """uint16 bf16 patterns -> int32 keys whose order is the values' order (no NaN here)."""
    b = bits.astype(np.int32)
    return np.where(b & 0x8000, -(b & 0x7FFF), b)


def _keys_bf16(keys: np.ndarray) -> np.ndarray:
    return np.where(keys < 0, (-keys) | 0x8000, keys).astype(np.uint16)


def untied_bf16_logits(rows: int, vocab: int, sigma: float, rng: np.random.Generator, top: int) -> np.ndarray:
    """uint16 bf16 bit patterns [rows, vocab] of N(0, sigma^2) logits whose `top` largest
    values are distinct and strictly above every other value of the row (the sampler's
    top-k window never sees a tie; values below it may repeat and never matter)."""
    x = (rng.standard_normal((rows, vocab)) * sigma).astype(np.float32)
    u = x.view(np.uint32)
    bits = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)  # round to nearest even
    keys = _bf16_keys(bits).astype(np.int64)
    order = np.argsort(-keys, axis=1, kind="stable")
    sk = np.take_along_axis(keys, order, axis=1)
    # descending and strictly decreasing over the first `top` places, the rest below them:
    # k'[i] = min_{j <= i}(k[j] + j) - i over the window, then clamp the tail
    idx = np.arange(top, dtype=np.int64)[None, :]
    head = np.minimum.accumulate(sk[:, :top] + idx, axis=1) - idx
    sk[:, :top] = head
    sk[:, top:] = np.minimum(sk[:, top:], head[:, -1:] - 1)
    out = np.empty_like(sk)
    np.put_along_axis(out, order, sk, axis=1)
    return _keys_bf16(out.astype(np.int32))


def scale_case(name: str):
    """(logits_bits [rows, vocab] uint16, temperatures, top_ks, top_ps, seeds, positions, max_top_k)."""
    case = next(c for c in SCALE_CASES if c[0] == name)
    _, rows, vocab, temp, top_k, top_p, G, sigma, seed = case
    rng = np.random.default_rng(seed)
    bits = untied_bf16_logits(rows, vocab, sigma, rng, top_k + 1)
    temps = np.full(rows, temp, dtype=np.float32)
    top_ks = np.full(rows, top_k, dtype=np.int64)
    top_ps = np.full(rows, top_p, dtype=np.float32)
    seeds = rng.integers(0, 2**31 - 1, rows, dtype=np.int64)
    sem = rng.integers(0, 4096, rows, dtype=np.int64)
    j = rng.integers(0, G - 1, rows, dtype=np.int64)
    positions = sem * (G - 1) + j + 1
    return bits, temps, top_ks, top_ps, seeds, positions, top_k
