"""Fusion #10 — expert merge + residual add (drop-in for glm52/kernels/merge_resadd.py:243-255).

    m   = bf16( sum_k w[t,k] * Y[t,k,:] )   (Y unweighted [T, topk, H], fp32 sum)
    out = bf16( m + res )                   (ROUND_MID: m rounded first, as the reference)

With ROUND_MID (default) fused and unfused are bitwise identical.
"""

from __future__ import annotations

from .. import ops

HIDDEN = 6144
TOPK = 8


def fused_merge_resadd(y, wt, res, out, cfg=None):
    ops.merge(y, wt, res, None, out, round_mid=bool((cfg or {}).get("ROUND_MID", 1)))


def merge_only(y, wt, m, cfg=None):
    ops.merge(y, wt, None, None, m, round_mid=True)


def resadd_only(m, res, out, cfg=None):
    ops.add(m, res, out)
