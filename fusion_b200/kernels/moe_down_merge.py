"""Fusions #8 / #9 — grouped down (w2) GEMM + expert merge (+ residual)
(drop-in for glm52/kernels/moe_down_merge.py:427-577).

`launch_down` applies the routing weight in the epilogue (MUL_ROUTED_WEIGHT, as the
reference always does) and either scatters bf16 rows to c[flat] (fuse_merge=False) or
accumulates into the pre-seeded [T, H] output (fuse_merge=True). The reference does the
latter with fp32/bf16 atomics; here the grouped GEMM writes the weighted rows and one
merge kernel adds their top-k sum to the seed with a single rounding (deterministic, and
no atomics on bf16).
"""

from __future__ import annotations

import torch

from .. import ops
from . import _ws
from .layout import moe_align_capacity
from .moe_gateup import _block_m


def _down_rows(a, w2, y, topk_weights_flat, sti, eid, ntp, num_valid_tokens, bm):
    EM = sti.numel()
    K = a.shape[1]
    a_rows = _ws.scratch("down_rows", EM * K, torch.bfloat16, a.device).view(EM, K)
    ops.permute_rows(a, sti, ntp, 1, num_valid_tokens, a_rows, EM)
    g = ops.gemm_group(w2, a_rows, y, expert_ids=eid, ntp=ntp, max_blocks=EM // bm, row_map=sti,
                       row_limit=num_valid_tokens, row_scale=topk_weights_flat,
                       live_ids=sti, live_limit=num_valid_tokens)
    ops.grouped_gemm([g], w2.shape[-2], K, ops.FUS_EPI_BF16, bm)


def launch_down(a, w2, c, topk_weights_flat, sorted_token_ids, expert_ids,
                num_tokens_post_padded, num_valid_tokens, top_k, cfg, fuse_merge: bool):
    """a: [rows, I] bf16 (row = flat id). w2: [E, H, I]. c: [rows, H], or the pre-seeded
    [T, H] output when fuse_merge."""
    bm = _block_m(cfg, sorted_token_ids)
    if not fuse_merge:
        _down_rows(a, w2, c, topk_weights_flat, sorted_token_ids, expert_ids,
                   num_tokens_post_padded, num_valid_tokens, bm)
        return
    T, H = c.shape
    y = _ws.scratch("down_y", T * top_k * H, torch.bfloat16, a.device).view(T * top_k, H)
    _down_rows(a, w2, y, topk_weights_flat, sorted_token_ids, expert_ids,
               num_tokens_post_padded, num_valid_tokens, bm)
    ops.merge(y.view(T, top_k, H), None, c, None, c, round_mid=False)


def launch_down_token_major(a, w2, out, topk_weights, topk_ids, residual, top_k, cfg,
                            add_residual: bool):
    """Strategy (b) of the reference: out[t] = sum_k w_k * (a[t*top_k+k] @ w2[e_k]^T)
    (+ residual), with no [T, top_k, H] tensor visible to the caller."""
    T = topk_ids.shape[0]
    H = w2.shape[1]
    bm = 16
    sti, eid, ntp = moe_align_capacity(topk_ids, bm, w2.shape[0])
    y = _ws.scratch("down_tm_y", T * top_k * H, torch.bfloat16, a.device).view(T * top_k, H)
    _down_rows(a, w2, y, topk_weights.reshape(-1).contiguous(), sti, eid, ntp, T * top_k, bm)
    ops.merge(y.view(T, top_k, H), None, residual if add_residual else None, None, out,
              round_mid=False)


def launch_moe_sum(c3, out, residual, topk, cfg, add_residual: bool):
    """out = bf16(sum_k c3[t, k] (+ residual)), fp32 accumulation (sglang moe_sum_reduce)."""
    T, H = out.shape
    ops.merge(c3.reshape(T, topk, H), None, residual if add_residual else None, None, out,
              round_mid=False)


def launch_resadd(x, r, o, cfg=None):
    ops.add(x, r, o)


def launch_seed(o, r, cfg, from_residual: bool):
    ops.seed(o, r if from_residual else None)
