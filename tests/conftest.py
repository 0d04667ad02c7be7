"""pytest configuration: the `gpu` marker and shared helpers."""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent
GOLDEN = Path(__file__).resolve().parent / "golden"
sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")


def pytest_collection_modifyitems(config, items):
    import torch

    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device in this process")
    for it in items:
        if "gpu" in it.keywords:
            it.add_marker(skip)


def golden(name: str) -> dict:
    with np.load(GOLDEN / f"{name}.npz") as z:
        return {k: z[k] for k in z.files}


def bf16_from_bits(b: np.ndarray) -> np.ndarray:
    return (b.astype(np.uint32) << 16).view(np.float32)


def ulp_diff_bf16(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    """|a - b| in bf16 ulps (both inputs exactly bf16-valued float32)."""
    ia = (a.astype(np.float32).view(np.int32) >> 16).astype(np.int64)
    ib = (b.astype(np.float32).view(np.int32) >> 16).astype(np.int64)
    # map sign-magnitude to a monotone integer line
    ia = np.where(ia < 0, -(ia & 0x7FFF), ia)
    ib = np.where(ib < 0, -(ib & 0x7FFF), ib)
    return np.abs(ia - ib)
