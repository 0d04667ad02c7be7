"""CPU backend for fusion_b200.ep.ExpertParallelMoE built on the numpy oracle (test-only):
lets the expert-parallel exchange run on gloo CPU ranks."""

from __future__ import annotations

import numpy as np
import torch

from oracle import reference_np as O


def _bf(a: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).to(torch.bfloat16)


class NumpyEPBackend:
    def __init__(self, w: dict, E: int, world: int, rank: int, topk: int):
        self.w = {k: (v.float().numpy() if v is not None else None) for k, v in w.items()}
        self.E, self.E_loc, self.topk = E, E // world, topk
        self.rank = rank

    def route(self, h, r):
        x2, h1 = O.add_rmsnorm(h.float().numpy(), r.float().numpy(), self.w["gamma"])
        _, tw, ti = O.router(x2, self.w["gate_w"], self.w["bias"], topk=self.topk)
        return _bf(h1), _bf(x2), torch.from_numpy(tw), torch.from_numpy(ti)

    def plan(self, topi, W: int):
        t = topi.reshape(-1).numpy()
        dest = t // self.E_loc
        send = np.argsort(dest, kind="stable").astype(np.int32)
        counts = np.bincount(dest, minlength=W).tolist()
        return torch.from_numpy(send), torch.from_numpy((t % self.E_loc).astype(np.int32)), counts

    def pack(self, x2, send_ids, leid, topk: int):
        s = send_ids.long()
        return x2[s // topk].contiguous(), leid[s].contiguous()

    def local_experts(self, rows, leid):
        x = rows.float().numpy()
        y = np.zeros((x.shape[0], x.shape[1]), dtype=np.float32)
        lid = leid.numpy()
        for i in range(x.shape[0]):
            w13 = self.w["w13"][lid[i]]
            w2 = self.w["w2"][lid[i]]
            hh = O.bf16(x[i:i + 1] @ w13.T)
            y[i] = O.bf16(O.silu_and_mul(hh) @ w2.T)[0]
        return _bf(y)

    def dispatch_fixed(self, x2, topi, W: int, S: int):
        t = topi.reshape(-1).numpy()
        K = topi.shape[1]
        dest = t // self.E_loc
        rows = torch.zeros(W * S, x2.shape[1], dtype=x2.dtype)
        leid = torch.full((W * S,), -1, dtype=torch.int32)
        slots = torch.zeros(t.size, dtype=torch.int32)
        used = [0] * W
        for i, d in enumerate(dest):
            slot = d * S + used[d]
            used[d] += 1
            rows[slot] = x2[i // K]
            leid[slot] = int(t[i] % self.E_loc)
            slots[i] = slot
        return rows, leid, slots

    def local_experts_holes(self, rows, leid):
        keep = torch.nonzero(leid >= 0).flatten()
        y = torch.zeros(rows.shape[0], rows.shape[1], dtype=torch.bfloat16)
        if keep.numel():
            y[keep] = self.local_experts(rows[keep], leid[keep])
        return y

    def gather_rows(self, y_ret, slots, R: int):
        return y_ret[slots.long()].contiguous()

    def unpack(self, ret, send_ids, R: int):
        y = torch.empty(R, ret.shape[1], dtype=ret.dtype)
        y[send_ids.long()] = ret
        return y

    def shared(self, x2):
        return torch.from_numpy(O.shared_expert_mlp(x2.float().numpy(), self.w["w13s"],
                                                    self.w["w2s"]))

    def merge(self, y_flat, topw, h1, ys):
        T, K = topw.shape
        y = y_flat.float().numpy().reshape(T, K, y_flat.shape[1])
        acc = (y * topw.numpy()[..., None]).sum(1) + h1.float().numpy() + ys.numpy()
        return _bf(acc)
