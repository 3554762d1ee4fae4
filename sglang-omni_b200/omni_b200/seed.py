"""Per-row sampling seeds: the host logic of sglang_omni/sampling/seed.py:18-48.

A request seed is masked to a positive int32; derived child seeds hash
``namespace:seed[:label]`` with blake2b (8-byte digest, little endian).
"""

from __future__ import annotations

import hashlib
import os

SAMPLING_SEED_MASK = 0x7FFFFFFF


def new_random_sampling_seed() -> int:
    """A fresh random positive-int32 seed for rows the caller left unseeded."""
    return int.from_bytes(os.urandom(4), "little") & SAMPLING_SEED_MASK


def derive_sampling_seed(namespace: str, public_seed: object, label: str | None = None) -> int:
    """Stable positive-int32 child seed of public request state (seed.py:24-34)."""
    parts = [namespace, str(public_seed)]
    if label is not None:
        parts.append(label)
    digest = hashlib.blake2b(":".join(parts).encode("utf-8"), digest_size=8).digest()
    return int.from_bytes(digest, "little") & SAMPLING_SEED_MASK


def resolve_row_seed(public_seed: int | None) -> int:
    """The user's seed masked to a positive int32, else a fresh random seed (seed.py:37-44)."""
    if public_seed is None:
        return new_random_sampling_seed()
    return int(public_seed) & SAMPLING_SEED_MASK


__all__ = ["SAMPLING_SEED_MASK", "derive_sampling_seed", "new_random_sampling_seed", "resolve_row_seed"]
