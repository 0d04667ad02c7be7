"""Dispatch layout on the device (drop-in for glm52/reference.py:85-128
moe_align_block_size, the sglang layout; see fusion_b200/csrc/align.cu)."""

from __future__ import annotations

import torch

from .. import ops


def moe_align_block_size(topk_ids: torch.Tensor, block_m: int, num_experts: int):
    """Returns (sorted_token_ids, expert_ids, num_tokens_post_padded) sized exactly like
    the reference's (one device->host read of the padded total, as the reference does)."""
    ids = topk_ids.contiguous().to(torch.int32)
    numel = ids.numel()
    cap = (numel + num_experts * (block_m - 1) + block_m - 1) // block_m * block_m
    s = torch.empty(cap, dtype=torch.int32, device=ids.device)
    e = torch.empty(cap // block_m, dtype=torch.int32, device=ids.device)
    n = torch.zeros(1, dtype=torch.int32, device=ids.device)
    ops.moe_align(ids, num_experts, block_m, s, e, n)
    total = int(n.item())
    return s[:total], e[: total // block_m], n


def moe_align_capacity(topk_ids: torch.Tensor, block_m: int, num_experts: int):
    """Same layout in worst-case-sized buffers, with no host synchronisation."""
    ids = topk_ids.contiguous().to(torch.int32)
    numel = ids.numel()
    cap = (numel + num_experts * (block_m - 1) + block_m - 1) // block_m * block_m
    s = torch.empty(cap, dtype=torch.int32, device=ids.device)
    e = torch.empty(cap // block_m, dtype=torch.int32, device=ids.device)
    n = torch.zeros(1, dtype=torch.int32, device=ids.device)
    ops.moe_align(ids, num_experts, block_m, s, e, n)
    return s, e, n
