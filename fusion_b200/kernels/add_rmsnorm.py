"""Fusion #3 — residual add + RMSNorm (drop-in for glm52/kernels/add_rmsnorm.py:234-246).

    h1  = bf16(x + res)                                  (the new residual)
    out = bf16( bf16(h1 * rsqrt(mean(h1^2) + eps)) * w )  (glm52/reference.py:22-33)

One sm_100a kernel (`add_rmsnorm_kernel`), flags select fused / add-only / norm-only;
the fused and unfused chains are bitwise identical.
"""

from __future__ import annotations

from .. import ops

HIDDEN = 6144


def fused_add_rmsnorm(x, res, w, h1, out, cfg=None):
    """FUSED: 2 reads + 2 writes."""
    ops.add_rmsnorm(x, res, w, h1, out, eps=(cfg or {}).get("eps", 1e-5))


def add_only(x, res, h1, cfg=None):
    """h1 = x + res (2 reads + 1 write)."""
    ops.add_rmsnorm(x, res, None, h1, None, do_norm=False)


def norm_only(h1, w, out, cfg=None):
    """out = rmsnorm(h1) * w (1 read + 1 write)."""
    ops.add_rmsnorm(h1, None, w, None, out, eps=(cfg or {}).get("eps", 1e-5), do_add=False)
