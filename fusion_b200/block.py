"""The GLM-5.2 MoE block on one GPU: weights, workspace and the forward call.

``MoEBlock.forward`` is one call into ``fus_moe_block_forward`` (8 kernel launches, no
host synchronisation, see ``csrc/block.cu``). ``MoEBlock.capture`` records that call
in a CUDA graph for a fixed T, which removes the per-launch host cost at decode sizes.

Reference: the block as glm52/bench/bench_layer.py:365-374 composes it, chained like
build_chain (bench_layer.py:395-481) without o_proj.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass

import torch

from . import _lib as L
from . import ops


@dataclass
class BlockOutputs:
    out: torch.Tensor    # [T, H] bf16  = h1 + routed + shared
    h1: torch.Tensor     # [T, H] bf16  new residual
    topw: torch.Tensor   # [T, k] fp32
    topi: torch.Tensor   # [T, k] int32


class MoEBlock:
    """Holds device weights in the reference's layouts:
    gamma [H] bf16, gate_w [E,H] fp32 (or bf16), bias [E] fp32 | None,
    w13 [E,2I,H] bf16, w2 [E,H,I] bf16, shared w13s [2I,H] / w2s [H,I] bf16 | None.
    n_group / topk_group > 1 select noaux_tc grouped routing (DeepSeek-V3-style)."""

    def __init__(self, gamma, gate_w, bias, w13, w2, w13s=None, w2s=None, *, topk: int = 8,
                 eps: float = 1e-5, routed_scale: float = 2.5, renorm: bool = True,
                 n_group: int = 1, topk_group: int = 1):
        self.E, twoI, self.H = w13.shape
        self.I = twoI // 2
        self.topk = topk
        self.device = w13.device
        if gate_w.dtype == torch.float32:
            self.wa, self.nplanes = ops.router_split_weight(gate_w), 3
        else:
            self.wa, self.nplanes = gate_w.contiguous(), 1
        self._keep = [gamma, bias, w13, w2, w13s, w2s, self.wa]
        d = L.BlockDesc()
        d.H, d.I, d.E, d.topk = self.H, self.I, self.E, topk
        d.eps, d.routed_scale, d.renorm = eps, routed_scale, int(renorm)
        d.gamma = gamma.data_ptr()
        d.wa = self.wa.data_ptr()
        d.nplanes = self.nplanes
        d.bias = bias.data_ptr() if bias is not None else None
        d.w13, d.w2 = w13.data_ptr(), w2.data_ptr()
        d.w13s = w13s.data_ptr() if w13s is not None else None
        d.w2s = w2s.data_ptr() if w2s is not None else None
        d.n_group, d.topk_group = n_group, topk_group  # noaux_tc grouping (1: GLM-5.2)
        d.flags = 0
        self.desc = d
        self._ws: torch.Tensor | None = None
        self._graphs: dict[int, tuple] = {}

    # ------------------------------------------------------------------------------
    def block_n(self, T: int) -> int:
        return int(L.lib().fus_moe_block_pick_block_n(T, self.E, self.topk))

    def workspace_bytes(self, T: int, block_n: int = 0) -> int:
        return int(L.lib().fus_moe_block_workspace(ctypes.byref(self.desc), T, block_n))

    def _workspace(self, nbytes: int) -> torch.Tensor:
        # zero once: the block keeps its counters zero between calls
        if self._ws is None or self._ws.numel() < nbytes:
            self._ws = torch.zeros(nbytes, dtype=torch.uint8, device=self.device)
        return self._ws

    def alloc_outputs(self, T: int) -> BlockOutputs:
        dev = self.device
        return BlockOutputs(
            out=torch.empty(T, self.H, dtype=torch.bfloat16, device=dev),
            h1=torch.empty(T, self.H, dtype=torch.bfloat16, device=dev),
            topw=torch.empty(T, self.topk, dtype=torch.float32, device=dev),
            topi=torch.empty(T, self.topk, dtype=torch.int32, device=dev),
        )

    def forward(self, h: torch.Tensor, r: torch.Tensor, outs: BlockOutputs | None = None,
                block_n: int = 0, workspace: torch.Tensor | None = None) -> BlockOutputs:
        T = h.shape[0]
        assert h.is_contiguous() and r.is_contiguous() and h.shape == (T, self.H)
        if outs is None:
            outs = self.alloc_outputs(T)
        if T == 0:  # an empty batch: nothing to compute
            return outs
        nbytes = self.workspace_bytes(T, block_n)
        ws = workspace if workspace is not None else self._workspace(nbytes)
        L.call("fus_moe_block_forward", ctypes.byref(self.desc), h.data_ptr(), r.data_ptr(), T,
               block_n, outs.out.data_ptr(), outs.h1.data_ptr(), outs.topw.data_ptr(),
               outs.topi.data_ptr(), ws.data_ptr(), ws.numel(),
               torch.cuda.current_stream().cuda_stream, ops.status_tensor().data_ptr())
        return outs

    __call__ = forward

    # ------------------------------------------------------------------------------
    def capture(self, T: int, block_n: int = 0):
        """Record forward() for T tokens in a CUDA graph with static buffers.
        Returns (graph, h_in, r_in, outs): copy inputs into h_in / r_in, replay."""
        if T in self._graphs:
            return self._graphs[T]
        h = torch.zeros(T, self.H, dtype=torch.bfloat16, device=self.device)
        r = torch.zeros_like(h)
        outs = self.alloc_outputs(T)
        ws = torch.zeros(self.workspace_bytes(T, block_n), dtype=torch.uint8, device=self.device)
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            self.forward(h, r, outs, block_n, ws)  # warm-up (sets kernel attributes)
        torch.cuda.current_stream().wait_stream(s)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            self.forward(h, r, outs, block_n, ws)
        self._graphs[T] = (g, h, r, outs, ws)
        return self._graphs[T]
