"""Fusion #6 — grouped up/gate (w13) GEMM, optional SwiGLU epilogue
(drop-in for glm52/kernels/moe_gateup.py:199-266).

`launch_gateup(a, w13, c, sorted_token_ids, expert_ids, num_tokens_post_padded,
num_valid_tokens, top_k, I, cfg, fused)` keeps the sglang dispatch semantics: A rows are
gathered with `flat // top_k`, output rows are the flat ids, pads are skipped. On B200 the
gather is one permutation kernel into a dense scratch operand (TMA needs dense rows), then
the tcgen05 grouped GEMM (`fusion_b200/csrc/gemm.cu`) with either the plain bf16 epilogue
([rows, 2I]) or the fused SwiGLU epilogue ([rows, I], silu on the fp32 accumulators, as
the reference's FUSE_ACT does). `cfg["BLOCK_M"]` must be the layout's block size.
"""

from __future__ import annotations

import torch

from .. import ops
from . import _ws


def _block_m(cfg, sorted_token_ids) -> int:
    bm = int((cfg or {}).get("BLOCK_M", 16))
    if bm not in (16, 32, 64, 128, 256):
        raise ValueError(f"BLOCK_M={bm}: the sm_100a kernel takes 16, 32, 64, 128 or 256")
    if sorted_token_ids.numel() % bm:
        raise ValueError("sorted_token_ids length is not a multiple of BLOCK_M")
    return bm


def launch_gateup(a, w13, c, sorted_token_ids, expert_ids, num_tokens_post_padded,
                  num_valid_tokens, top_k, I, cfg, fused: bool):
    """a: [T, H] bf16. w13: [E, 2I, H] bf16. c: [T*top_k, I if fused else 2I] bf16."""
    bm = _block_m(cfg, sorted_token_ids)
    EM = sorted_token_ids.numel()
    H = a.shape[1]
    xs = _ws.scratch("gateup_rows", EM * H, torch.bfloat16, a.device).view(EM, H)
    ops.permute_rows(a, sorted_token_ids, num_tokens_post_padded, top_k, num_valid_tokens, xs, EM)
    g = ops.gemm_group(w13, xs, c, expert_ids=expert_ids, ntp=num_tokens_post_padded,
                       max_blocks=EM // bm, row_map=sorted_token_ids,
                       row_limit=num_valid_tokens,
                       flags=ops.GEMM_SWIGLU_EXACT if fused else 0,
                       live_ids=sorted_token_ids, live_limit=num_valid_tokens)
    ops.grouped_gemm([g], w13.shape[-2], H, ops.FUS_EPI_SWIGLU if fused else ops.FUS_EPI_BF16, bm)


def launch_silu_and_mul(x, y, cfg=None):
    """[M, 2I] -> [M, I]: bf16(silu(gate) * up)."""
    ops.silu_and_mul(x, y)
