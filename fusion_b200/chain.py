"""The MoE block as an explicit chain of launches (one Python callable per kernel).

Same kernels and the same order as ``fus_moe_block_forward``, but issued one by one
through the C ABI, so a caller can put CUDA events between them (per-kernel timing,
roofline of the dominant kernel) or swap one step for a variant. This is the
B200 counterpart of the reference's layer-chain driver
(glm52/bench/bench_layer.py:395-481 build_chain, without o_proj).
"""

from __future__ import annotations

from typing import Callable

import torch

from . import ops
from .block import BlockOutputs, MoEBlock


class BlockChain:
    def __init__(self, blk: MoEBlock, T: int, block_n: int = 0, persist: bool = True):
        self.blk, self.T = blk, T
        H, I, E, K = blk.H, blk.I, blk.E, blk.topk
        self.bn = block_n or blk.block_n(T)
        bn = self.bn
        dev = blk.device
        self.R = R = T * K
        cap = R + E * (bn - 1)
        self.cap = cap = (cap + bn - 1) // bn * bn
        self.max_blocks = min(min(R, E) + R // bn, cap // bn)
        self.nsplit = ops.router_nsplit(T, H, E, blk.nplanes)
        bf = torch.bfloat16
        self.small = T <= 16 and E <= 256 and E % 2 == 0 and T * K <= 256 and blk.nplanes in (1, 3)
        self.x2 = torch.empty(T, H, dtype=bf, device=dev)
        self.partial = torch.empty(self.nsplit, T, E, dtype=torch.float32, device=dev)
        self.sorted = torch.empty(cap, dtype=torch.int32, device=dev)
        self.eids = torch.empty(cap // bn, dtype=torch.int32, device=dev)
        self.ntp = torch.zeros(1, dtype=torch.int32, device=dev)
        nws = ops.moe_align_workspace(R, E)
        self.align_ws = torch.empty(max(nws, 16), dtype=torch.uint8, device=dev)
        self.xs = None if self.small else torch.empty(cap, H, dtype=bf, device=dev)
        self.act = torch.empty(cap, I, dtype=bf, device=dev)
        self.act_s = torch.empty(T, I, dtype=bf, device=dev)
        # decode: y in pair order (fused merge); prefill: rows in dispatch order (dense
        # tile stores) over the permuted rows (dead after w13), merged through pos_of
        self.y = torch.empty(R, H, dtype=bf, device=dev) if self.small else self.xs
        self.pos_of = torch.empty(R, dtype=torch.int32, device=dev)
        self.ys = torch.empty(T, H, dtype=torch.float32, device=dev)
        self.tiles = ops.gemm_tiles(H, ops.FUS_EPI_BF16, bn)
        self.counters = torch.zeros(T * self.tiles, dtype=torch.int32, device=dev)
        self.done = torch.zeros(4, dtype=torch.int32, device=dev)
        self.logits = torch.empty(T, E, dtype=torch.float32, device=dev)
        self.outs: BlockOutputs = blk.alloc_outputs(T)
        self.shared = blk.desc.w13s is not None
        self.np_flag = 0 if persist else ops.GEMM_NO_PERSIST

    def steps(self, h: torch.Tensor, r: torch.Tensor) -> list[tuple[str, Callable[[], None]]]:
        b, o = self.blk, self.outs
        H, I, E, K, T, bn = b.H, b.I, b.E, b.topk, self.T, self.bn
        keep = b._keep
        gamma, bias, w13, w2, w13s, w2s = keep[0], keep[1], keep[2], keep[3], keep[4], keep[5]

        ws = (ops.GEMM_W_STREAM if self.R / E <= bn else 0) | self.np_flag
        wss = ops.GEMM_W_STREAM if T <= bn else 0

        def w13_step():
            if self.small:  # rows gathered by dispatch position inside the GEMM
                gs = [ops.gemm_group(w13, self.x2, self.act, expert_ids=self.eids, ntp=self.ntp,
                                     max_blocks=self.max_blocks, row_limit=self.cap,
                                     flags=ops.GEMM_SWIGLU_EXACT | ws, live_ids=self.sorted,
                                     live_limit=self.R, gather_ids=self.sorted, gather_div=K)]
            else:
                gs = [ops.gemm_group(w13, self.xs, self.act, expert_ids=self.eids, ntp=self.ntp,
                                     max_blocks=self.max_blocks, row_limit=self.cap,
                                     flags=ops.GEMM_SWIGLU_EXACT | ws, live_ids=self.sorted,
                                     live_limit=self.R)]
            if self.shared:
                gs.append(ops.gemm_group(w13s, self.x2, self.act_s, max_blocks=-(-T // bn),
                                         row_limit=T, flags=ops.GEMM_SWIGLU_EXACT | wss))
            ops.grouped_gemm(gs, 2 * I, H, ops.FUS_EPI_SWIGLU, bn)

        def w2_groups(merge: bool):
            mf = ops.GEMM_MERGE if merge else 0
            if merge:
                g0 = ops.gemm_group(w2, self.act, self.y, expert_ids=self.eids, ntp=self.ntp,
                                    max_blocks=self.max_blocks, row_map=self.sorted,
                                    row_limit=self.R, flags=ws | mf, live_ids=self.sorted,
                                    live_limit=self.R, token_div=K)
            else:
                g0 = ops.gemm_group(w2, self.act, self.y, expert_ids=self.eids, ntp=self.ntp,
                                    max_blocks=self.max_blocks, row_limit=self.cap, flags=ws,
                                    live_ids=self.sorted, live_limit=self.R)
            gs = [g0]
            if self.shared:
                gs.append(ops.gemm_group(w2s, self.act_s, self.ys, max_blocks=-(-T // bn),
                                         row_limit=T, flags=ops.GEMM_OUT_F32 | mf | wss))
            return gs

        def w2_merge_step():  # decode: merge fused into the w2 epilogue
            ops.grouped_gemm_merge(w2_groups(True), H, I, bn, counters=self.counters,
                                   y3=self.y.view(T, K, H), w=o.topw, res=o.h1,
                                   extra=self.ys if self.shared else None, out=o.out,
                                   parts=K + (1 if self.shared else 0))

        def w2_step():
            ops.grouped_gemm(w2_groups(False), H, I, ops.FUS_EPI_BF16, bn)

        def merge_step():
            ops.merge_pos(self.y, self.pos_of, K, o.topw, o.h1,
                          self.ys if self.shared else None, o.out)

        if self.small:
            front = [("route_small", lambda: ops.route_small(
                h, r, gamma, b.wa, b.nplanes, bias, o.h1, self.x2, self.logits, o.topw, o.topi,
                bn, self.sorted, self.eids, self.ntp, self.done, self.counters))]
        else:
            front = [
                ("add_rmsnorm", lambda: ops.add_rmsnorm(h, r, gamma, o.h1, self.x2)),
                ("router_gemm", lambda: ops.router_logits(self.x2, b.wa, b.nplanes,
                                                          self.partial, self.nsplit)),
                ("router_topk", lambda: ops.router_topk(self.partial, self.nsplit, bias, None,
                                                        o.topw, o.topi)),
                ("moe_align", lambda: ops.moe_align(o.topi, E, bn, self.sorted, self.eids,
                                                    self.ntp, self.align_ws, self.pos_of,
                                                    ops.ALIGN_BALANCED)),
                ("permute", lambda: ops.permute_rows(self.x2, self.sorted, self.ntp, K, self.R,
                                                     self.xs, self.cap)),
            ]
        if self.small:
            return front + [("w13_swiglu", w13_step), ("w2_merge", w2_merge_step)]
        return front + [("w13_swiglu", w13_step), ("w2", w2_step), ("merge", merge_step)]

    def run(self, h, r) -> BlockOutputs:
        for _, fn in self.steps(h, r):
            fn()
        return self.outs
