"""Expert-parallel MoE block across GPUs of one node (one process per GPU).

Rank g of W owns routed experts [g*E/W, (g+1)*E/W) (w13 [E/W, 2I, H], w2 [E/W, H, I]);
the RMSNorm weight, the router and the shared expert are replicated. Every rank runs the
block on its own tokens (weak scaling):

  1. add+RMSNorm, router, top-k on the local tokens                     (local kernels)
  2. plan: destination rank and local expert of every (token, slot) pair (fus_ep_plan),
     pairs stably sorted by destination (fus_moe_align over the destinations)
  3. dispatch: one x2 row + its local expert id per pair, NCCL all_to_all (the per-rank
     counts are exchanged first, they set the split sizes)
  4. the owner runs its grouped w13+SwiGLU and w2 GEMMs on the rows it received
  5. combine: the expert rows travel back by the inverse all_to_all (same order) and are
     put back in slot order (fus_ep_unpack)
  6. shared expert on the local tokens, merge: out = bf16(sum_k w_k y_k + h1 + shared)

The exchange logic is written once (`ExpertParallelMoE`) over a backend that supplies
the local compute: `CudaEPBackend` (the sm_100a kernels) here; the CPU tests run the same
exchange over gloo with a numpy backend. The reference has no multi-GPU path
(log/LOG-00-plan-and-filter.md:41); SURVEY §8e gives the design.
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from . import ops


class ExpertParallelMoE:
    def __init__(self, backend, group=None):
        self.be = backend
        self.group = group
        self.W = dist.get_world_size(group) if dist.is_initialized() else 1

    def _a2a(self, out: torch.Tensor, inp: torch.Tensor, out_splits, in_splits):
        if self.W == 1:
            out.copy_(inp)
            return
        # bf16 rows travel as int32 pairs of their bit patterns (every backend moves int32;
        # rows have an even width, and splits count rows, so they are unchanged)
        o = out.view(torch.int32) if out.dtype == torch.bfloat16 else out
        i = inp.view(torch.int32) if inp.dtype == torch.bfloat16 else inp
        dist.all_to_all_single(o, i, list(out_splits), list(in_splits), group=self.group)

    def forward(self, h: torch.Tensor, r: torch.Tensor) -> dict:
        be = self.be
        h1, x2, topw, topi = be.route(h, r)
        T, K = topi.shape
        send_ids, leid, counts = be.plan(topi, self.W)  # counts: per-destination pair counts
        rows, leid_send = be.pack(x2, send_ids, leid, K)
        cnt = torch.tensor(counts, dtype=torch.int64, device=rows.device)
        recv_cnt = torch.empty_like(cnt)
        self._a2a(recv_cnt, cnt, [1] * self.W, [1] * self.W)
        in_counts = [int(v) for v in recv_cnt.tolist()]
        n_in = sum(in_counts)
        recv_rows = torch.empty(n_in, rows.shape[1], dtype=rows.dtype, device=rows.device)
        recv_leid = torch.empty(n_in, dtype=leid_send.dtype, device=rows.device)
        self._a2a(recv_rows, rows, in_counts, counts)
        self._a2a(recv_leid, leid_send, in_counts, counts)
        y_recv = be.local_experts(recv_rows, recv_leid)
        ret = torch.empty(T * K, rows.shape[1], dtype=y_recv.dtype, device=rows.device)
        self._a2a(ret, y_recv, counts, in_counts)
        y_flat = be.unpack(ret, send_ids, T * K)
        ys = be.shared(x2)
        out = be.merge(y_flat, topw, h1, ys)
        return {"out": out, "h1": h1, "topw": topw, "topi": topi, "rows_in": n_in}

    def forward_fixed(self, h: torch.Tensor, r: torch.Tensor) -> dict:
        """Small-batch step with fixed split sizes (no host synchronisation, capturable in
        a CUDA graph): every rank sends every peer a block of S = T*topk slots, unused
        slots carry local expert -1 (holes the owner skips)."""
        be = self.be
        h1, x2, topw, topi = be.route(h, r)
        T, K = topi.shape
        S = T * K
        shared = be.shared_begin(x2) if hasattr(be, "shared_begin") else None
        send_rows, send_leid, slots = be.dispatch_fixed(x2, topi, self.W, S)
        recv_rows = torch.empty_like(send_rows)
        recv_leid = torch.empty_like(send_leid)
        eq = [S] * self.W
        self._a2a(recv_rows, send_rows, eq, eq)
        self._a2a(recv_leid, send_leid, eq, eq)
        y_recv = be.local_experts_holes(recv_rows, recv_leid)
        y_ret = torch.empty_like(y_recv)
        self._a2a(y_ret, y_recv, eq, eq)
        y_flat = be.gather_rows(y_ret, slots, T * K)
        ys = be.shared_end(shared) if shared is not None else be.shared(x2)
        out = be.merge(y_flat, topw, h1, ys)
        return {"out": out, "h1": h1, "topw": topw, "topi": topi}

    __call__ = forward


class EPDecodeGraph:
    """`forward_fixed` for a fixed T recorded in a CUDA graph (NCCL all_to_all included);
    copy inputs into `h` / `r`, call `replay()`, read `out`."""

    def __init__(self, ep: ExpertParallelMoE, T: int, H: int, device):
        self.ep = ep
        self.h = torch.zeros(T, H, dtype=torch.bfloat16, device=device)
        self.r = torch.zeros_like(self.h)
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            for _ in range(2):
                ep.forward_fixed(self.h, self.r)
        torch.cuda.current_stream().wait_stream(s)
        torch.cuda.synchronize()
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self.res = ep.forward_fixed(self.h, self.r)
        self.out = self.res["out"]

    def replay(self):
        self.graph.replay()
        return self.out


class CudaEPBackend:
    """Local compute of one rank on its GPU with the library's kernels."""

    def __init__(self, gamma, gate_w, bias, w13_local, w2_local, w13s, w2s, *, E: int,
                 rank: int, topk: int = 8, eps: float = 1e-5, routed_scale: float = 2.5):
        self.gamma, self.bias, self.w13, self.w2 = gamma, bias, w13_local, w2_local
        self.w13s, self.w2s = w13s, w2s
        self.E, self.E_loc, self.topk = E, w13_local.shape[0], topk
        self.rank, self.eps, self.scale = rank, eps, routed_scale
        self.H, self.I = w13_local.shape[2], w13_local.shape[1] // 2
        if gate_w.dtype == torch.float32:
            self.wa, self.nplanes = ops.router_split_weight(gate_w), 3
        else:
            self.wa, self.nplanes = gate_w.contiguous(), 1
        self.dev = w13_local.device

    def shared_begin(self, x2):
        """Start the shared expert on a side stream (it overlaps the exchange and the
        routed experts); `shared_end` joins it."""
        side = torch.cuda.Stream(device=self.dev)
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            ys = self.shared(x2)
        return side, ys

    def shared_end(self, handle):
        side, ys = handle
        torch.cuda.current_stream().wait_stream(side)
        if ys is not None:
            ys.record_stream(torch.cuda.current_stream())
        return ys

    def route(self, h, r):
        T, H = h.shape
        bf = torch.bfloat16
        if T <= 16 and self.E <= 256:
            # decode: norm + router + top-k in one launch (its dispatch layout over all E
            # experts is not needed here and goes to scratch)
            h1 = torch.empty(T, H, dtype=bf, device=self.dev)
            x2 = torch.empty(T, H, dtype=bf, device=self.dev)
            logits = torch.empty(T, self.E, dtype=torch.float32, device=self.dev)
            topw = torch.empty(T, self.topk, dtype=torch.float32, device=self.dev)
            topi = torch.empty(T, self.topk, dtype=torch.int32, device=self.dev)
            cap = T * self.topk + self.E * 15
            cap = (cap + 15) // 16 * 16
            if not hasattr(self, "_route_done"):
                self._route_done = torch.zeros(4, dtype=torch.int32, device=self.dev)
            sorted_ids = torch.empty(cap, dtype=torch.int32, device=self.dev)
            eids = torch.empty(cap // 16, dtype=torch.int32, device=self.dev)
            ntp = torch.empty(1, dtype=torch.int32, device=self.dev)
            ops.route_small(h, r, self.gamma, self.wa, self.nplanes, self.bias, h1, x2, logits,
                            topw, topi, 16, sorted_ids, eids, ntp, self._route_done,
                            eps=self.eps, scale=self.scale)
            return h1, x2, topw, topi
        h1, x2 = torch.empty(T, H, dtype=bf, device=self.dev), torch.empty(T, H, dtype=bf,
                                                                          device=self.dev)
        ops.add_rmsnorm(h, r, self.gamma, h1, x2, eps=self.eps)
        ns = ops.router_nsplit(T, H, self.E, self.nplanes)
        part = torch.empty(ns, T, self.E, dtype=torch.float32, device=self.dev)
        ops.router_logits(x2, self.wa, self.nplanes, part, ns)
        topw = torch.empty(T, self.topk, dtype=torch.float32, device=self.dev)
        topi = torch.empty(T, self.topk, dtype=torch.int32, device=self.dev)
        ops.router_topk(part, ns, self.bias, None, topw, topi, scale=self.scale)
        return h1, x2, topw, topi

    def plan(self, topi, W: int):
        R = topi.numel()
        dest = torch.empty(R, dtype=torch.int32, device=self.dev)
        leid = torch.empty(R, dtype=torch.int32, device=self.dev)
        counts = torch.empty(W, dtype=torch.int32, device=self.dev)
        ops.ep_plan(topi, self.E_loc, W, dest, leid, counts)
        send_ids = torch.empty(R, dtype=torch.int32, device=self.dev)
        eids = torch.empty(R, dtype=torch.int32, device=self.dev)
        ntp = torch.zeros(1, dtype=torch.int32, device=self.dev)
        ops.moe_align(dest, W, 1, send_ids, eids, ntp)  # stable sort by destination
        return send_ids, leid, [int(v) for v in counts.tolist()]

    def pack(self, x2, send_ids, leid, topk: int):
        n = send_ids.numel()
        rows = torch.empty(n, x2.shape[1], dtype=x2.dtype, device=self.dev)
        leid_out = torch.empty(n, dtype=torch.int32, device=self.dev)
        ops.ep_pack(x2, send_ids, n, topk, leid, rows, leid_out)
        return rows, leid_out

    def local_experts(self, rows, leid):
        n, H = rows.shape
        I, E = self.I, self.E_loc
        y = torch.empty(n, H, dtype=torch.bfloat16, device=self.dev)
        if n == 0:
            return y
        per = n / E
        bn = 16 if per <= 12 else 32 if per <= 24 else 64 if per <= 48 else 128 if per <= 128 else 256
        cap = (n + E * (bn - 1) + bn - 1) // bn * bn
        sorted_ids = torch.empty(cap, dtype=torch.int32, device=self.dev)
        eids = torch.empty(cap // bn, dtype=torch.int32, device=self.dev)
        ntp = torch.zeros(1, dtype=torch.int32, device=self.dev)
        ops.moe_align(leid.view(n, 1), E, bn, sorted_ids, eids, ntp)
        xs = torch.empty(cap, H, dtype=torch.bfloat16, device=self.dev)
        ops.permute_rows(rows, sorted_ids, ntp, 1, n, xs, cap)
        act = torch.empty(cap, I, dtype=torch.bfloat16, device=self.dev)
        maxb = min(min(n, E) + n // bn, cap // bn)
        ws = ops.GEMM_W_STREAM if per <= bn else 0
        g = ops.gemm_group(self.w13, xs, act, expert_ids=eids, ntp=ntp, max_blocks=maxb,
                           row_limit=cap, flags=ops.GEMM_SWIGLU_EXACT | ws,
                           live_ids=sorted_ids, live_limit=n)
        ops.grouped_gemm([g], 2 * I, H, ops.FUS_EPI_SWIGLU, bn)
        g2 = ops.gemm_group(self.w2, act, y, expert_ids=eids, ntp=ntp, max_blocks=maxb,
                            row_map=sorted_ids, row_limit=n, flags=ws, live_ids=sorted_ids,
                            live_limit=n)
        ops.grouped_gemm([g2], H, I, ops.FUS_EPI_BF16, bn)
        return y

    def dispatch_fixed(self, x2, topi, W: int, S: int):
        rows = torch.empty(W * S, x2.shape[1], dtype=x2.dtype, device=self.dev)
        leid = torch.empty(W * S, dtype=torch.int32, device=self.dev)
        slots = torch.empty(topi.numel(), dtype=torch.int32, device=self.dev)
        ops.ep_dispatch_small(x2, topi, self.E_loc, W, S, rows, leid, slots)
        return rows, leid, slots

    def local_experts_holes(self, rows, leid):
        """Expert rows for a slot buffer with holes (local expert -1): the token rows are
        gathered by dispatch position inside the w13 GEMM (no permutation pass)."""
        n, H = rows.shape
        I, E, bn = self.I, self.E_loc, 16
        y = torch.empty(n, H, dtype=torch.bfloat16, device=self.dev)
        cap = (n + E * (bn - 1) + bn - 1) // bn * bn
        sorted_ids = torch.empty(cap, dtype=torch.int32, device=self.dev)
        eids = torch.empty(cap // bn, dtype=torch.int32, device=self.dev)
        ntp = torch.zeros(1, dtype=torch.int32, device=self.dev)
        ops.moe_align(leid.view(n, 1), E, bn, sorted_ids, eids, ntp)
        act = torch.empty(cap, I, dtype=torch.bfloat16, device=self.dev)
        maxb = min(min(n, E) + n // bn, cap // bn)
        ws = ops.GEMM_W_STREAM
        g = ops.gemm_group(self.w13, rows, act, expert_ids=eids, ntp=ntp, max_blocks=maxb,
                           row_limit=cap, flags=ops.GEMM_SWIGLU_EXACT | ws,
                           live_ids=sorted_ids, live_limit=n, gather_ids=sorted_ids,
                           gather_div=1)
        ops.grouped_gemm([g], 2 * I, H, ops.FUS_EPI_SWIGLU, bn)
        g2 = ops.gemm_group(self.w2, act, y, expert_ids=eids, ntp=ntp, max_blocks=maxb,
                            row_map=sorted_ids, row_limit=n, flags=ws, live_ids=sorted_ids,
                            live_limit=n)
        ops.grouped_gemm([g2], H, I, ops.FUS_EPI_BF16, bn)
        return y

    def gather_rows(self, y_ret, slots, R: int):
        y = torch.empty(R, y_ret.shape[1], dtype=y_ret.dtype, device=self.dev)
        n = torch.full((1,), R, dtype=torch.int32, device=self.dev)
        ops.permute_rows(y_ret, slots, n, 1, y_ret.shape[0], y, R)
        return y

    def unpack(self, ret, send_ids, R: int):
        y = torch.empty(R, ret.shape[1], dtype=ret.dtype, device=self.dev)
        ops.ep_unpack(ret, send_ids, R, y)
        return y

    def shared(self, x2):
        if self.w13s is None:
            return None
        T, H = x2.shape
        I = self.I
        bn = 16 if T <= 16 else 32 if T <= 32 else 64 if T <= 64 else 128 if T <= 128 else 256
        act = torch.empty(T, I, dtype=torch.bfloat16, device=self.dev)
        ys = torch.empty(T, H, dtype=torch.float32, device=self.dev)
        nb = -(-T // bn)
        ws = ops.GEMM_W_STREAM if T <= bn else 0
        ops.grouped_gemm([ops.gemm_group(self.w13s, x2, act, max_blocks=nb, row_limit=T,
                                         flags=ops.GEMM_SWIGLU_EXACT | ws)],
                         2 * I, H, ops.FUS_EPI_SWIGLU, bn)
        ops.grouped_gemm([ops.gemm_group(self.w2s, act, ys, max_blocks=nb, row_limit=T,
                                         flags=ops.GEMM_OUT_F32 | ws)],
                         H, I, ops.FUS_EPI_BF16, bn)
        return ys

    def merge(self, y_flat, topw, h1, ys):
        T, K = topw.shape
        out = torch.empty_like(h1)
        ops.merge(y_flat.view(T, K, -1), topw, h1, ys, out, round_mid=False)
        return out


def shard_weights(base_seed: int, rank: int, world: int, dims, device) -> dict:
    """This rank's slice of the seeded block weights (bit-identical to the slice of the
    single-GPU weights) plus the replicated ones."""
    from . import synth

    E_loc = dims.E // world
    n13 = 2 * dims.I * dims.H
    n2 = dims.H * dims.I
    return {
        "gamma": synth.make("gamma", (dims.H,), base_seed, device),
        "gate_w": synth.make("gate_w", (dims.E, dims.H), base_seed, device),
        "bias": synth.make("bias", (dims.E,), base_seed, device),
        "w13": synth.make("w13", (E_loc, 2 * dims.I, dims.H), base_seed, device,
                          offset=rank * E_loc * n13),
        "w2": synth.make("w2", (E_loc, dims.H, dims.I), base_seed, device,
                         offset=rank * E_loc * n2),
        "w13s": synth.make("w13s", (2 * dims.I, dims.H), base_seed, device),
        "w2s": synth.make("w2s", (dims.H, dims.I), base_seed, device),
    }
