"""Expert-parallel MoE block across GPUs of one node (one process per GPU).

Rank g of W owns routed experts [g*E/W, (g+1)*E/W) (w13 [E/W, 2I, H], w2 [E/W, H, I]);
the RMSNorm weight, the router and the shared expert are replicated. Every rank runs the
block on its own tokens (weak scaling):

  1. add+RMSNorm, router, top-k on the local tokens                     (local kernels)
  2. plan: destination rank and local expert of every (token, slot) pair (fus_ep_plan),
     pairs stably sorted by destination (fus_moe_align over the destinations)
  3. dispatch: one x2 row per (token, owning rank) with its slots' local expert ids
     (deduplicated, the default) or one per (token, slot) pair, NCCL all_to_all (the
     per-rank counts are exchanged first, they set the split sizes)
  4. the owner runs its grouped w13+SwiGLU and w2 GEMMs on the rows it received
  5. combine: the expert rows travel back by the inverse all_to_all (same order) and are
     put back in slot order (fus_ep_unpack)
  6. shared expert on the local tokens, merge: out = bf16(sum_k w_k y_k + h1 + shared)

The exchange logic is written once (`ExpertParallelMoE`) over a backend that supplies
the local compute: `CudaEPBackend` (the sm_100a kernels) here; the CPU tests run the same
exchange over gloo with a numpy backend. Small batches (decode) exchange fixed slot
blocks: over NCCL all_to_all (`forward_fixed`), or with `P2PExchange` by direct stores
into the peers' exchange buffers over NVLink and flag waits (`forward_p2p`, no
collective launch at all). The reference has no multi-GPU path
(log/LOG-00-plan-and-filter.md:41).
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

    def forward(self, h: torch.Tensor, r: torch.Tensor, dispatch: str = "dedup",
                combine: str = "pairs") -> dict:
        """Variable-size step (prefill). dispatch="dedup" (default): `forward_dedup`, a
        token's row travels once per owning rank (5.25 rows per token at 8 ranks under
        uniform routing, against 8); bit-identical to dispatch="pairs" (`forward_pairs`,
        one x2 row per (token, slot) pair each way) with the default combine."""
        if dispatch == "pairs":
            return self.forward_pairs(h, r)
        if dispatch != "dedup":
            raise ValueError(f"dispatch={dispatch!r}: 'pairs' or 'dedup'")
        return self.forward_dedup(h, r, combine)

    def forward_dedup(self, h: torch.Tensor, r: torch.Tensor, combine: str = "pairs") -> dict:
        """Variable-size step (prefill) with deduplicated dispatch: a token's x2 row travels
        once to each rank that owns at least one of its experts, with its K slots' local
        experts (-1 for slots owned elsewhere).

        combine="pairs" (default): the owner returns one expert row per pair, written by its
          w2 GEMM straight into the order the source expects; the source merges them with
          the same arithmetic as one GPU.
        combine="partial": the owner returns one row per (token, rank), the bf16-rounded
          partial sum_k w_k y_k over its experts (fewer bytes; the extra rounding of the
          partial can move the output by an ulp)."""
        if combine not in ("pairs", "partial"):
            raise ValueError(f"combine={combine!r}: 'pairs' or 'partial'")
        be = self.be
        h1, x2, topw, topi = be.route(h, r)
        T, K = topi.shape
        W = self.W
        ys = None
        if hasattr(be, "plan_finish"):
            # the counts travel to the host while the GPU runs the shared expert (queued
            # behind the copy on the same stream), so the host's wait and the launches
            # that follow it overlap GPU work
            plan = be.plan_dedup(topi, W, with_pair_pos=combine == "pairs", defer=True)
            ys = be.shared(x2)
            be.plan_finish(plan)
        else:
            plan = be.plan_dedup(topi, W, with_pair_pos=combine == "pairs")
        counts = plan["counts"]  # [rows, pairs] per destination
        rows_out = [c[0] for c in counts]
        pairs_out = [c[1] for c in counts]
        n_send = sum(rows_out)
        rows, leid, meta = be.pack_dedup(x2, n_send, topi, topw, W, plan, combine)
        cnt = torch.tensor(counts, dtype=torch.int64, device=rows.device)
        recv_cnt = torch.empty_like(cnt)
        self._a2a(recv_cnt, cnt, [1] * W, [1] * W)
        rc = recv_cnt.tolist()
        rows_in = [int(c[0]) for c in rc]
        pairs_in = [int(c[1]) for c in rc]
        n_in = sum(rows_in)
        H = rows.shape[1]
        recv_rows = torch.empty(n_in, H, dtype=rows.dtype, device=rows.device)
        recv_leid = torch.empty(n_in, K, dtype=leid.dtype, device=rows.device)
        self._a2a(recv_rows, rows, rows_in, rows_out)
        self._a2a(recv_leid, leid, rows_in, rows_out)
        if combine == "pairs":
            recv_ret = torch.empty(n_in, K, dtype=meta.dtype, device=rows.device)
            self._a2a(recv_ret, meta, rows_in, rows_out)
            y = be.local_experts_return(recv_rows, recv_leid, recv_ret, rows_in, pairs_in)
            ret = torch.empty(sum(pairs_out), H, dtype=y.dtype, device=rows.device)
            self._a2a(ret, y, pairs_out, pairs_in)
            if ys is None:
                ys = be.shared(x2)
            out = be.merge_pairs(ret, plan["pair_pos"], topw, h1, ys)
        else:
            wts, pos = meta
            recv_w = torch.empty(n_in, K, dtype=wts.dtype, device=rows.device)
            self._a2a(recv_w, wts, rows_in, rows_out)
            part = be.local_experts_dedup(recv_rows, recv_leid, recv_w, sum(pairs_in))
            # returned partials, plus one zero row that the positions of a token's other
            # slots on the same rank point at
            ret = torch.empty(n_send + 1, H, dtype=part.dtype, device=rows.device)
            ret[n_send].zero_()
            self._a2a(ret[:n_send], part, rows_out, rows_in)
            if ys is None:
                ys = be.shared(x2)
            out = be.merge_dedup(ret, pos, h1, ys)
        return {"out": out, "h1": h1, "topw": topw, "topi": topi, "rows_in": n_in,
                "pairs_in": sum(pairs_in)}

    def forward_pairs(self, h: torch.Tensor, r: torch.Tensor) -> dict:
        """Variable-size step shipping one row per (token, slot) pair (no deduplication);
        the returned expert rows are merged at the source exactly as on one GPU."""
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
        return {"out": out, "h1": h1, "topw": topw, "topi": topi, "rows_in": n_in,
                "pairs_in": n_in}

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


    def forward_p2p(self, h: torch.Tensor, r: torch.Tensor, x: "P2PExchange") -> dict:
        """`forward_fixed` with the three all_to_alls replaced by peer stores into the
        exchange buffers and flag waits (x.S >= T*topk slots per source)."""
        be = self.be
        h1, x2, topw, topi = be.route(h, r)
        T, K = topi.shape
        shared = be.shared_begin(x2)
        slots = torch.empty(T * K, dtype=torch.int32, device=x2.device)
        ops.ep_p2p_dispatch(x2, topi, be.E_loc, x.W, x.S, x.rank, x.peer_rows, x.peer_leid,
                            x.peer_dflags, x.epoch, slots)
        ops.ep_p2p_wait(x.dflags, x.epoch, x.W)
        y_recv = be.local_experts_holes(x.recv_rows, x.recv_leid)
        ops.ep_p2p_combine(y_recv, x.recv_leid, x.W, x.S, x.rank, x.peer_ret, x.peer_cflags,
                           x.epoch)
        ops.ep_p2p_wait(x.cflags, x.epoch, x.W)
        ys = be.shared_end(shared)
        out = torch.empty_like(h1)
        ops.merge_pos(x.ret_rows, slots, K, topw, h1, ys, out)
        return {"out": out, "h1": h1, "topw": topw, "topi": topi}


class P2PExchange:
    """This rank's exchange buffer, exported through CUDA IPC, and the addresses of every
    rank's (W ranks of one node, S slots per source, H features). Layout per rank:
    recv_rows [W*S, H] bf16, recv_leid [W*S] int32, ret_rows [W*S, H] bf16, dflags [W],
    cflags [W] int32; plus a local step counter (epoch). Collective: every rank of the
    group constructs it together."""

    def __init__(self, S: int, H: int, device, group=None):
        self.group = group
        self.W = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.S, self.H = S, H
        W, n = self.W, self.W * S
        offs, o = {}, 0
        for name, nbytes in (("recv_rows", n * H * 2), ("recv_leid", n * 4),
                             ("ret_rows", n * H * 2), ("dflags", W * 4), ("cflags", W * 4)):
            offs[name] = o
            o = (o + nbytes + 255) // 256 * 256
        self.buf = torch.zeros(o, dtype=torch.uint8, device=device)
        self.epoch = torch.zeros(1, dtype=torch.int32, device=device)
        b = self.buf
        self.recv_rows = b[offs["recv_rows"]:offs["recv_rows"] + n * H * 2].view(torch.bfloat16).view(n, H)
        self.recv_leid = b[offs["recv_leid"]:offs["recv_leid"] + n * 4].view(torch.int32)
        self.ret_rows = b[offs["ret_rows"]:offs["ret_rows"] + n * H * 2].view(torch.bfloat16).view(n, H)
        self.dflags = b[offs["dflags"]:offs["dflags"] + W * 4].view(torch.int32)
        self.cflags = b[offs["cflags"]:offs["cflags"] + W * 4].view(torch.int32)
        torch.cuda.synchronize(device)
        handle, off = ops.ipc_handle(self.buf)
        if self.W > 1:
            allh = [None] * self.W
            dist.all_gather_object(allh, (handle, off), group=group)
        else:
            allh = [(handle, off)]
        self._opened = []
        bases = []
        for w, (h, o_) in enumerate(allh):
            if w == self.rank:
                bases.append(self.buf.data_ptr())
            else:
                p = ops.ipc_open(h, o_)
                self._opened.append((p, o_))
                bases.append(p)

        def table(name):
            return torch.tensor([bb + offs[name] for bb in bases], dtype=torch.int64,
                                device=device)

        self.peer_rows, self.peer_leid = table("recv_rows"), table("recv_leid")
        self.peer_ret, self.peer_dflags, self.peer_cflags = (table("ret_rows"), table("dflags"),
                                                             table("cflags"))
        if self.W > 1:
            dist.barrier(group=group)  # every buffer zeroed and mapped before any store

    def close(self):
        """Unmap the peers' buffers (collective; no step may be in flight)."""
        torch.cuda.synchronize()
        if self.W > 1:
            dist.barrier(group=self.group)
        for p, o in self._opened:
            ops.ipc_close(p, o)
        self._opened = []


class EPDecodeStep:
    """The decode step of one rank as ONE library call (fus_ep_p2p_decode_forward: seven
    launches chained with programmatic dependent launch over the NVLink exchange) for a
    fixed T; `capture()` records it in a CUDA graph. Collective: every rank builds it."""

    def __init__(self, be: "CudaEPBackend", T: int, group=None):
        import ctypes

        from . import _lib as L

        self.be, self.T = be, T
        self.x = P2PExchange(T * be.topk, be.H, be.dev, group)
        d = L.BlockDesc()
        d.H, d.I, d.E, d.topk = be.H, be.I, be.E, be.topk
        d.eps, d.routed_scale, d.renorm = be.eps, be.scale, 1
        d.gamma, d.wa, d.nplanes = be.gamma.data_ptr(), be.wa.data_ptr(), be.nplanes
        d.bias = be.bias.data_ptr() if be.bias is not None else None
        d.w13, d.w2 = be.w13.data_ptr(), be.w2.data_ptr()
        d.w13s = be.w13s.data_ptr() if be.w13s is not None else None
        d.w2s = be.w2s.data_ptr() if be.w2s is not None else None
        self._blk = d
        x = self.x
        p = L.EPP2PDesc()
        p.blk = ctypes.pointer(d)
        p.E_loc, p.W, p.rank, p.S = be.E_loc, x.W, x.rank, x.S
        p.peer_rows, p.peer_leid, p.peer_dflags = (x.peer_rows.data_ptr(), x.peer_leid.data_ptr(),
                                                   x.peer_dflags.data_ptr())
        p.peer_ret, p.peer_cflags = x.peer_ret.data_ptr(), x.peer_cflags.data_ptr()
        p.recv_rows, p.recv_leid, p.ret_rows = (x.recv_rows.data_ptr(), x.recv_leid.data_ptr(),
                                                x.ret_rows.data_ptr())
        p.dflags, p.cflags, p.epoch = x.dflags.data_ptr(), x.cflags.data_ptr(), x.epoch.data_ptr()
        self.desc = p
        nbytes = int(L.lib().fus_ep_p2p_decode_workspace(ctypes.byref(p), T))
        if nbytes == 0:
            raise ValueError("ep_p2p_decode: bad sizes")
        self.ws = torch.zeros(nbytes, dtype=torch.uint8, device=be.dev)
        bf = torch.bfloat16
        # h and r as the two halves of one buffer: a caller fills both with one copy
        self.hr = torch.zeros(2, T, be.H, dtype=bf, device=be.dev)
        self.h, self.r = self.hr[0], self.hr[1]
        self.out = torch.empty_like(self.h)
        self.h1 = torch.empty_like(self.h)
        self.topw = torch.empty(T, be.topk, dtype=torch.float32, device=be.dev)
        self.topi = torch.empty(T, be.topk, dtype=torch.int32, device=be.dev)
        self.graph = None

    def forward(self) -> torch.Tensor:
        """One step on the inputs in `h` / `r`; returns `out` (also fills h1/topw/topi)."""
        import ctypes

        from . import _lib as L

        L.call("fus_ep_p2p_decode_forward", ctypes.byref(self.desc), self.h.data_ptr(),
               self.r.data_ptr(), self.T, self.out.data_ptr(), self.h1.data_ptr(),
               self.topw.data_ptr(), self.topi.data_ptr(), self.ws.data_ptr(),
               self.ws.numel(), torch.cuda.current_stream().cuda_stream,
               ops.status_tensor().data_ptr())
        return self.out

    def capture(self):
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            for _ in range(2):
                self.forward()
        torch.cuda.current_stream().wait_stream(s)
        torch.cuda.synchronize()
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self.forward()
        return self

    def replay(self) -> torch.Tensor:
        self.graph.replay()
        return self.out

    def close(self):
        """Collective: drop the recorded step (it holds the peers' buffer addresses), then
        unmap the peers' exchange buffers."""
        torch.cuda.synchronize()
        self.graph = None
        self.x.close()


class EPDecodeGraph:
    """The fixed-slot decode step for a fixed T recorded in a CUDA graph; copy inputs into
    `h` / `r`, call `replay()`, read `out`. exchange="p2p": NVLink peer stores
    (`forward_p2p`), "nccl": all_to_all (`forward_fixed`)."""

    def __init__(self, ep: ExpertParallelMoE, T: int, H: int, device, exchange: str = "p2p"):
        self.ep = ep
        # h and r as the two halves of one buffer: a caller fills both with one copy
        self.hr = torch.zeros(2, T, H, dtype=torch.bfloat16, device=device)
        self.h, self.r = self.hr[0], self.hr[1]
        self.x = None
        if exchange == "p2p":
            self.x = P2PExchange(T * ep.be.topk, H, device, ep.group)
            step = lambda: ep.forward_p2p(self.h, self.r, self.x)  # noqa: E731
        else:
            step = lambda: ep.forward_fixed(self.h, self.r)  # noqa: E731
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            for _ in range(2):
                step()
        torch.cuda.current_stream().wait_stream(s)
        torch.cuda.synchronize()
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self.res = step()
        self.out = self.res["out"]

    def replay(self):
        self.graph.replay()
        return self.out

    def close(self):
        """Collective when the exchange is NVLink: drop the graph, unmap the peers."""
        torch.cuda.synchronize()
        self.graph = None
        if self.x is not None:
            self.x.close()


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

    def plan_dedup(self, topi, W: int, with_pair_pos: bool = True, defer: bool = False) -> dict:
        """Send plan of the deduplicated dispatch. defer=True leaves the per-destination
        counts on their way to the host (`plan_finish` reads them), so the caller can
        queue more GPU work behind the copy before it waits."""
        T, K = topi.shape
        keys = torch.empty(T * W, dtype=torch.int32, device=self.dev)
        counts = torch.empty(2 * W, dtype=torch.int32, device=self.dev)
        ops.ep_plan_dedup(topi, self.E_loc, W, keys, counts)
        send_ids = torch.empty(T * W, dtype=torch.int32, device=self.dev)
        eids = torch.empty(T * W, dtype=torch.int32, device=self.dev)
        ntp = torch.zeros(1, dtype=torch.int32, device=self.dev)
        ops.moe_align(keys, W, 1, send_ids, eids, ntp)  # stable sort by destination
        plan = {"send_ids": send_ids, "counts_dev": counts}
        if with_pair_pos:
            # each pair's position among the pairs stably sorted by destination = the row
            # of its expert output in what the owners return
            R = T * K
            dest = torch.empty(R, dtype=torch.int32, device=self.dev)
            leid = torch.empty(R, dtype=torch.int32, device=self.dev)
            pc = torch.empty(W, dtype=torch.int32, device=self.dev)
            ops.ep_plan(topi, self.E_loc, W, dest, leid, pc)
            srt = torch.empty(R, dtype=torch.int32, device=self.dev)
            e2 = torch.empty(R, dtype=torch.int32, device=self.dev)
            n2 = torch.zeros(1, dtype=torch.int32, device=self.dev)
            plan["pair_pos"] = torch.empty(T, K, dtype=torch.int32, device=self.dev)
            ops.moe_align(dest, W, 1, srt, e2, n2, pos_of=plan["pair_pos"])
        plan["W"] = W
        if defer:
            host = torch.empty(2 * W, dtype=torch.int32, pin_memory=True)
            host.copy_(counts, non_blocking=True)
            ev = torch.cuda.Event()
            ev.record()
            plan["_host"] = (host, ev)
            return plan
        return self.plan_finish(plan, counts)

    def plan_finish(self, plan: dict, counts=None) -> dict:
        """The host side of the plan: per destination [rows, pairs]."""
        W = plan["W"]
        if counts is None:
            host, ev = plan.pop("_host")
            ev.synchronize()
            c = host.tolist()
        else:
            c = counts.tolist()
        plan["counts"] = [[c[d], c[W + d]] for d in range(W)]
        return plan

    def pack_dedup(self, x2, n: int, topi, topw, W: int, plan: dict, combine: str):
        T, K = topi.shape
        rows = torch.empty(n, x2.shape[1], dtype=x2.dtype, device=self.dev)
        leid = torch.empty(n, K, dtype=torch.int32, device=self.dev)
        if combine == "pairs":
            ret = torch.empty(n, K, dtype=torch.int32, device=self.dev)
            ops.ep_pack_dedup(x2, plan["send_ids"], n, W, topi, topw, self.E_loc, rows, leid,
                              pair_pos=plan["pair_pos"], counts=plan["counts_dev"], ret_out=ret)
            return rows, leid, ret
        wts = torch.empty(n, K, dtype=torch.float32, device=self.dev)
        pos = torch.empty(T, K, dtype=torch.int32, device=self.dev)
        ops.ep_pack_dedup(x2, plan["send_ids"], n, W, topi, topw, self.E_loc, rows, leid,
                          w_out=wts, pos=pos, zero_row=n)
        return rows, leid, (wts, pos)

    def _dedup_layout(self, rows, leid, pairs: int):
        """Dispatch layout over the received rows' live slots, the permuted token rows and
        the w13 + SwiGLU GEMM; returns what the w2 launch needs."""
        n, H = rows.shape
        K = leid.shape[1]
        I, E = self.I, self.E_loc
        R = n * K
        per = pairs / E
        bn = 16 if per <= 12 else 32 if per <= 24 else 64 if per <= 48 else 128 if per <= 128 else 256
        cap = (R + E * (bn - 1) + bn - 1) // bn * bn
        sorted_ids = torch.empty(cap, dtype=torch.int32, device=self.dev)
        eids = torch.empty(cap // bn, dtype=torch.int32, device=self.dev)
        ntp = torch.zeros(1, dtype=torch.int32, device=self.dev)
        ops.moe_align(leid, E, bn, sorted_ids, eids, ntp)
        xs = torch.empty(cap, H, dtype=torch.bfloat16, device=self.dev)
        ops.permute_rows(rows, sorted_ids, ntp, K, R, xs, cap)
        act = torch.empty(cap, I, dtype=torch.bfloat16, device=self.dev)
        maxb = min(min(pairs, E) + pairs // bn, cap // bn)
        ws = ops.GEMM_W_STREAM if per <= bn else 0
        g = ops.gemm_group(self.w13, xs, act, expert_ids=eids, ntp=ntp, max_blocks=maxb,
                           row_limit=cap, flags=ops.GEMM_SWIGLU_EXACT | ws,
                           live_ids=sorted_ids, live_limit=R)
        ops.grouped_gemm([g], 2 * I, H, ops.FUS_EPI_SWIGLU, bn)
        return dict(bn=bn, sorted_ids=sorted_ids, eids=eids, ntp=ntp, act=act, maxb=maxb,
                    ws=ws, R=R)

    def local_experts_return(self, rows, leid, ret_idx, rows_in, pairs_in):
        """Expert rows of every received pair, in the order the sources expect them back:
        source s's pairs at [sum(pairs_in[:s]), ...), each at its ret_idx."""
        n, H = rows.shape
        P = sum(pairs_in)
        y = torch.empty(P, H, dtype=torch.bfloat16, device=self.dev)
        if n == 0 or P == 0:
            return y
        L = self._dedup_layout(rows, leid, P)
        def prefix(v):
            out = [0]
            for c in v:
                out.append(out[-1] + c)
            return torch.tensor(out, dtype=torch.int32, device=self.dev)
        rowmap = torch.empty_like(L["sorted_ids"])
        ops.ep_return_rowmap(L["sorted_ids"], ret_idx, leid.shape[1], prefix(rows_in),
                             prefix(pairs_in), rowmap, ntp=L["ntp"])
        g2 = ops.gemm_group(self.w2, L["act"], y, expert_ids=L["eids"], ntp=L["ntp"],
                            max_blocks=L["maxb"], row_map=rowmap, row_limit=P, flags=L["ws"],
                            live_ids=L["sorted_ids"], live_limit=L["R"])
        ops.grouped_gemm([g2], H, self.I, ops.FUS_EPI_BF16, L["bn"])
        return y

    def merge_pairs(self, ret, pair_pos, topw, h1, ys):
        out = torch.empty_like(h1)
        ops.merge_pos(ret, pair_pos, topw.shape[1], topw, h1, ys, out)
        return out

    def local_experts_dedup(self, rows, leid, wts, pairs: int):
        """Partial rows sum_k w_k y_k over this rank's experts of each received row (slots
        with local expert -1 belong to other ranks)."""
        n, H = rows.shape
        out = torch.empty(n, H, dtype=torch.bfloat16, device=self.dev)
        if n == 0 or pairs == 0:
            return out
        L = self._dedup_layout(rows, leid, pairs)
        y = torch.empty(L["R"], H, dtype=torch.bfloat16, device=self.dev)  # slot order
        g2 = ops.gemm_group(self.w2, L["act"], y, expert_ids=L["eids"], ntp=L["ntp"],
                            max_blocks=L["maxb"], row_map=L["sorted_ids"], row_limit=L["R"],
                            flags=L["ws"], live_ids=L["sorted_ids"], live_limit=L["R"])
        ops.grouped_gemm([g2], H, self.I, ops.FUS_EPI_BF16, L["bn"])
        ops.ep_partial_sum(y, leid, wts, out)
        return out

    def merge_dedup(self, ret, pos, h1, ys):
        out = torch.empty_like(h1)
        ops.merge_pos(ret, pos, pos.shape[1], None, h1, ys, out)
        return out

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
