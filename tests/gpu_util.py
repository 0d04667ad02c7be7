"""Helpers shared by the GPU parity tests."""

from __future__ import annotations

import numpy as np
import torch

from fusion_b200 import ops

DEV = "cuda"


def to_np(t: torch.Tensor) -> np.ndarray:
    return t.detach().float().cpu().numpy()


def bf(a: np.ndarray) -> torch.Tensor:
    """float32 array of bf16 values -> bf16 cuda tensor (exact)."""
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).to(DEV).to(torch.bfloat16)


def finish() -> None:
    torch.cuda.synchronize()
    ops.check_status()


def assert_bf16_close(got: np.ndarray, ref: np.ndarray, max_ulp: int = 1, frac: float = 1e-3):
    from conftest import ulp_diff_bf16

    d = ulp_diff_bf16(got, ref)
    assert d.max() <= max_ulp, f"max ulp diff {d.max()}"
    assert (d > 0).mean() <= frac, f"{(d > 0).mean():.2e} of elements differ"


def rel_err(got, ref) -> float:
    """max-abs error / max|ref|  (glm52/common.py:186-190)."""
    got = np.asarray(got, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    return float(np.abs(got - ref).max() / max(np.abs(ref).max(), 1e-6))


def assert_sum_close(got: np.ndarray, ref: np.ndarray):
    """For bf16 results of fp32 sums whose summation order differs: one bf16 ulp of the
    result (2^-7 relative), plus a small absolute slack where the sum cancels to ~0."""
    got = np.asarray(got, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    tol = 2.0 ** -7 * np.abs(ref) + 1e-4 * np.abs(ref).max()
    bad = np.abs(got - ref) > tol
    assert not bad.any(), f"{bad.sum()} elements off, worst {np.abs(got - ref).max():.3g}"
