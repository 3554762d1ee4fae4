"""Shared pytest setup: import paths, the ``gpu`` marker, golden fixtures."""

from __future__ import annotations

import base64
import json
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent
for p in (ROOT, ROOT / "sglang-omni_b200"):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))

GOLDEN = ROOT / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")


def pytest_collection_modifyitems(config, items):
    try:
        import torch

        has_gpu = torch.cuda.is_available()
    except Exception:  # pragma: no cover
        has_gpu = False
    if has_gpu:
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


@pytest.fixture(scope="session")
def golden():
    return json.loads((GOLDEN / "reference_golden.json").read_text())


@pytest.fixture(scope="session")
def staging_golden():
    return json.loads((GOLDEN / "staging_golden.json").read_text())


@pytest.fixture(scope="session")
def sampler_scale_golden():
    with np.load(GOLDEN / "sampler_scale_golden.npz") as z:
        return {k: z[k].astype(np.int64) for k in z.files}


def decode_bf16_b64(case) -> np.ndarray:
    raw = base64.b64decode(case["logits_bf16_b64"])
    return np.frombuffer(raw, dtype="<u2").reshape(case["shape"]).copy()
