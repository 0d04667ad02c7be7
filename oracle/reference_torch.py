"""The reference's MoE block as torch CPU ops — TEST INFRASTRUCTURE ONLY.

A restatement of glm52_h200/reference.py's framework path with the same torch
operations in the same order, so that it runs at the reference's own CPU speed (bf16
``linear`` through torch's CPU BLAS, the per-expert ``nonzero`` loop, ``index_add_``).
``bench.py`` times it as the reference arm and as the CPU baseline; the numpy
restatement in ``reference_np.py`` stays the parity oracle (its fp32 upcasts make it
several times slower than the reference on the same cores). ``oracle/time_reference.py``
checks this module bit-for-bit against the reference imported from a checkout.

Nothing here loads the CUDA library: inputs come from ``synth_np`` as numpy arrays.
"""

from __future__ import annotations

import torch

from .reference_np import RMS_NORM_EPS, ROUTED_SCALING_FACTOR, TOPK

F = torch.nn.functional


def rmsnorm(x: torch.Tensor, w: torch.Tensor, eps: float = RMS_NORM_EPS) -> torch.Tensor:
    """reference.py:57-62: fp32 statistics, bf16 normalised value, then the bf16 weight."""
    xf = x.float()
    var = xf.pow(2).mean(-1, keepdim=True)
    return (xf * torch.rsqrt(var + eps)).to(x.dtype) * w


def add_rmsnorm(x, residual, w, eps: float = RMS_NORM_EPS):
    """reference.py:65-70: (normed, h1) with h1 = bf16(x + residual)."""
    h = (x.float() + residual.float()).to(x.dtype)
    return rmsnorm(h, w, eps), h


def silu_and_mul(x: torch.Tensor) -> torch.Tensor:
    """reference.py:73-77: silu(gate) * up in fp32, result in the input dtype."""
    d = x.shape[-1] // 2
    g, u = x[..., :d].float(), x[..., d:].float()
    return (F.silu(g) * u).to(x.dtype)


def router(x, gate_w, bias, topk: int = TOPK, scale: float = ROUTED_SCALING_FACTOR):
    """reference.py:138-173 with n_group = 1: fp32 logits, sigmoid, bias only in the
    choice, top-k, renormalised weights times the scaling factor."""
    logits = F.linear(x.float(), gate_w.float())
    scores = logits.sigmoid()
    choice = scores + bias
    ids = choice.topk(topk, dim=-1).indices
    w = scores.gather(1, ids)
    w = w / w.sum(-1, keepdim=True).clamp_min(1e-20)
    return logits, (w * scale).float(), ids.int()


def moe_mlp(x, w13, w2, topk_weights, topk_ids, num_experts: int) -> torch.Tensor:
    """reference.py:228-259: per expert (all ``num_experts``, one ``nonzero`` each), bf16
    linear -> bf16 SwiGLU -> bf16 linear, weighted fp32 ``index_add_``, bf16 result.
    ``w13`` / ``w2`` are indexable by expert (a stacked tensor or a dict of the routed
    experts' weights)."""
    T, H = x.shape
    out = torch.zeros(T, H, dtype=torch.float32)
    for e in range(num_experts):
        sel = (topk_ids == e).nonzero(as_tuple=False)
        if sel.numel() == 0:
            continue
        rows, ks = sel[:, 0], sel[:, 1]
        h = F.linear(x[rows], w13[e])
        y = F.linear(silu_and_mul(h), w2[e]).float()
        out.index_add_(0, rows, y * topk_weights[rows, ks].unsqueeze(1))
    return out.to(x.dtype)


def shared_expert_mlp(x, w13_s, w2_s) -> torch.Tensor:
    """reference.py:294-311: fp32 linear, bf16 h, SwiGLU, fp32 linear; fp32 result."""
    h = F.linear(x.float(), w13_s.float())
    return F.linear(silu_and_mul(h.to(x.dtype)).float(), w2_s.float())


@torch.no_grad()
def moe_block(h, r, gamma, gate_w, bias, w13, w2, w13_s, w2_s, num_experts: int):
    """The block as glm52/bench/bench_layer.py:365-374 composes its check: out =
    bf16(moe_mlp(x2).float() + h1 + shared(x2)). Tensors are CPU torch tensors (bf16
    activations and weights, fp32 router weight and bias)."""
    x2, h1 = add_rmsnorm(h, r, gamma)
    _, tw, ti = router(x2, gate_w, bias)
    routed = moe_mlp(x2, w13, w2, tw, ti, num_experts).float()
    out = (routed + h1.float() + shared_expert_mlp(x2, w13_s, w2_s)).to(h.dtype)
    return {"out": out, "topk_weights": tw, "topk_ids": ti, "h1": h1, "x2": x2}
