"""Fusion #11 (half fused, F11b') — lazy pre-norm on the router and the w13 GEMM
(drop-in for glm52/kernels/lazy_prenorm.py).

For an affine RMSNorm, ((h * rstd) * w) @ B == (h @ (w[:, None] * B)) * rstd: the norm
weight is folded into B's K dimension once at load (`fold_weight_*`), the GEMM reads the
un-normalised h1 and the output rows are scaled by the row's rstd afterwards. As in the
reference's F11b', rstd comes from its own small kernel (`launch_rstd`), so the GEMM
mainloop is the plain one; with `rstd=None` and `fuse_norm=True` the launchers compute
it themselves. `sq_mode` (how the Triton kernel accumulates the sum of squares) has no
counterpart here; the mapping keys of `cfg` do not apply.

    launch_rstd(x, rstd, cfg, eps)                                 (lazy_prenorm.py:371)
    launch_router(a, b[K,N], c[M,N] fp32, cfg, fuse_norm, ...)     (lazy_prenorm.py:457)
    launch_moe_gateup(a, b[E,N,K], c[T*top_k,N], sorted_token_ids, expert_ids,
                      num_tokens_post_padded, num_valid_tokens, top_k, cfg, fuse_norm,
                      ...)                                         (lazy_prenorm.py:402)
"""

from __future__ import annotations

import torch

from .. import ops
from . import _ws


def fold_weight_rowmajor(b: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    """B is [K, N] (contraction dim first): row k scaled by w[k]."""
    out = torch.empty_like(b)
    ops.fold_weight(b.contiguous(), w, out, by_row=True)
    return out


def fold_weight_nk(bt: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    """B^T is [..., N, K] (nn.Linear / sglang w13 layout): column k scaled by w[k]."""
    out = torch.empty_like(bt)
    ops.fold_weight(bt.contiguous(), w, out, by_row=False)
    return out


def smem_bytes(cfg: dict) -> int:
    """The reference's Triton pipeline estimate (kept for signature compatibility)."""
    return cfg["num_stages"] * 2 * cfg["BLOCK_K"] * (cfg["BLOCK_M"] + cfg["BLOCK_N"])


def launch_rstd(x, rstd, cfg=None, eps: float = 1e-5):
    ops.row_rstd(x, rstd, eps)


def _rstd_for(a, rstd, eps):
    if rstd is not None:
        return rstd
    r = _ws.scratch("lazy_rstd", a.shape[0], torch.float32, a.device)
    ops.row_rstd(a, r, eps)
    return r


def launch_router(a, b, c, cfg=None, fuse_norm: bool = True, eps: float = 1e-5,
                  sq_mode: int = 0, rstd=None):
    """a: [M, K] bf16 (h1 when fuse_norm, else x2). b: [K, N] bf16 (w-folded when
    fuse_norm). c: [M, N] fp32 = (a @ b) * rstd (fuse_norm) or a @ b."""
    M, K = a.shape
    N = c.shape[1]
    wa = _ws.converted(b, "lazy_router_nk", lambda: ops.router_transpose_weight(b))
    ns = ops.router_nsplit(M, K, N, 1)
    part = _ws.scratch("lazy_router_part", ns * M * N, torch.float32, a.device).view(ns, M, N)
    ops.router_logits(a, wa, 1, part, ns)
    ops.scale_sum_planes(part, ns, _rstd_for(a, rstd, eps) if fuse_norm else None, c)


def launch_moe_gateup(a, b, c, sorted_token_ids, expert_ids, num_tokens_post_padded,
                      num_valid_tokens, top_k, cfg, fuse_norm: bool, eps: float = 1e-5,
                      sq_mode: int = 0, rstd=None):
    """a: [T, K] bf16. b: [E, N, K] bf16 (w-folded when fuse_norm). c: [T*top_k, N] bf16,
    row = flat (token, slot) id; c = bf16((a[t] @ b[e].T) * rstd[t]) when fuse_norm."""
    bm = int((cfg or {}).get("BLOCK_M", 16))
    if bm not in (16, 32, 64, 128, 256) or sorted_token_ids.numel() % bm:
        raise ValueError(f"BLOCK_M={bm}: must be 16..256 and divide the layout length")
    EM = sorted_token_ids.numel()
    K = a.shape[1]
    xs = _ws.scratch("lazy_gateup_rows", EM * K, torch.bfloat16, a.device).view(EM, K)
    ops.permute_rows(a, sorted_token_ids, num_tokens_post_padded, top_k, num_valid_tokens, xs, EM)
    scale = _rstd_for(a, rstd, eps) if fuse_norm else None
    g = ops.gemm_group(b, xs, c, expert_ids=expert_ids, ntp=num_tokens_post_padded,
                       max_blocks=EM // bm, row_map=sorted_token_ids,
                       row_limit=num_valid_tokens, row_scale=scale,
                       flags=ops.GEMM_SCALE_TOKEN if fuse_norm else 0,
                       live_ids=sorted_token_ids, live_limit=num_valid_tokens,
                       token_div=top_k)
    ops.grouped_gemm([g], b.shape[-2], K, ops.FUS_EPI_BF16, bm)
