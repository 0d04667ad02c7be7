"""Router pieces (drop-in for glm52/kernels/norm_router.py:337-390).

`router_gemm(x2, wgt, logits, cfg)`: logits = x2.float() @ wgt.float(), where `wgt` is
the [H, E] layout of `wgt_from_gate` (bf16 as in the reference's Triton path, or fp32).
It runs on tcgen05 tensor cores: the weight is converted once per weight version to
K-major bf16 planes (1 plane for bf16, 3 exact planes for fp32), K is split across CTAs
and the fp32 partial planes are summed in a fixed order.

`topk_only(logits, topw, topi, cfg)`: sigmoid, top-k (descending), renormalise, x scale —
like the reference's Triton topk_only it takes no correction bias (norm_router.py:221-239);
`topk_biased` is the full reference.router selection (glm52/reference.py:62-79).

The fused norm+router variants are compositions of the unfused kernels (the reference
measured the fused forms harmful on every device, log/LOG-09-consolidated-results.md).
"""

from __future__ import annotations

import torch

from .. import ops
from . import _ws
from .add_rmsnorm import fused_add_rmsnorm, norm_only

NUM_EXPERTS = 256
TOP_K = 8


def wgt_from_gate(gate_w: torch.Tensor) -> torch.Tensor:
    """[E, H] (nn.Linear) -> [H, E], the reference's router weight layout."""
    return gate_w.t().contiguous()


def _planes(wgt: torch.Tensor) -> tuple[torch.Tensor, int]:
    if wgt.dtype == torch.float32:
        return _ws.converted(wgt, "planes3", lambda: ops.router_split_weight(
            wgt.t().contiguous())), 3
    return _ws.converted(wgt, "planes1", lambda: ops.router_transpose_weight(wgt)), 1


def _logits_partial(x2, wgt):
    wa, planes = _planes(wgt)
    T, H = x2.shape
    E = wa.shape[0]
    ns = ops.router_nsplit(T, H, E, planes)
    part = _ws.scratch("router_partial", ns * T * E, torch.float32, x2.device).view(ns, T, E)
    ops.router_logits(x2, wa, planes, part, ns)
    return part, ns


def router_gemm(x2, wgt, logits, cfg=None):
    part, ns = _logits_partial(x2, wgt)
    T, E = logits.shape
    k = TOP_K if E >= TOP_K else 1
    tw = _ws.scratch("router_tw", T * k, torch.float32, x2.device).view(T, k)
    ti = _ws.scratch("router_ti", T * k, torch.int32, x2.device).view(T, k)
    ops.router_topk(part, ns, None, logits, tw, ti)  # sums the planes into `logits`


def topk_only(logits, topw, topi, cfg=None):
    cfg = cfg or {}
    ops.router_topk(logits.unsqueeze(0), 1, None, None, topw, topi,
                    scale=cfg.get("scale", 2.5), renorm=bool(cfg.get("NORM_PROB", True)))


def topk_biased(logits, bias, topw, topi, cfg=None):
    cfg = cfg or {}
    ops.router_topk(logits.unsqueeze(0), 1, bias, None, topw, topi,
                    scale=cfg.get("scale", 2.5), renorm=bool(cfg.get("NORM_PROB", True)))


def router_topk(x2, wgt, bias, topw, topi, logits=None, cfg=None):
    """Router GEMM + selection with the correction bias (reference.router)."""
    cfg = cfg or {}
    part, ns = _logits_partial(x2, wgt)
    ops.router_topk(part, ns, bias, logits, topw, topi, scale=cfg.get("scale", 2.5),
                    renorm=bool(cfg.get("NORM_PROB", True)))


# ---- unfused pieces / compositions ----------------------------------------------------
def rmsnorm_only(x, w, x2, cfg=None):
    norm_only(x, w, x2, cfg)


def add_rmsnorm_only(x, res, w, h1, x2, cfg=None):
    fused_add_rmsnorm(x, res, w, h1, x2, cfg)


def fused_norm_router(x, w, x2, wgt, logits, cfg=None):
    norm_only(x, w, x2, cfg)
    router_gemm(x2, wgt, logits, cfg)


def fused_add_norm_router(x, res, w, h1, x2, wgt, logits, cfg=None):
    fused_add_rmsnorm(x, res, w, h1, x2, cfg)
    router_gemm(x2, wgt, logits, cfg)


def fused_norm_router_topk(x, w, x2, wgt, topw, topi, cfg=None):
    norm_only(x, w, x2, cfg)
    router_topk(x2, wgt, None, topw, topi, cfg=cfg)


def fused_add_norm_router_topk(x, res, w, h1, x2, wgt, topw, topi, cfg=None):
    fused_add_rmsnorm(x, res, w, h1, x2, cfg)
    router_topk(x2, wgt, None, topw, topi, cfg=cfg)
