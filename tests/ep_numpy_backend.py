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

    def plan_dedup(self, topi, W: int, with_pair_pos: bool = True) -> dict:
        ti = topi.numpy()
        T, K = ti.shape
        dest = ti // self.E_loc
        keys = np.full((T, W), -1, dtype=np.int64)
        for t in range(T):
            for d in set(dest[t].tolist()):
                keys[t, d] = d
        flat = keys.reshape(-1)
        send = np.nonzero(flat >= 0)[0]
        send = send[np.argsort(flat[send], kind="stable")].astype(np.int32)
        counts = [[int((keys[:, d] == d).sum()), int((dest == d).sum())] for d in range(W)]
        plan = {"send_ids": torch.from_numpy(send), "counts": counts}
        if with_pair_pos:
            order = np.argsort(dest.reshape(-1), kind="stable")
            pp = np.empty(T * K, dtype=np.int32)
            pp[order] = np.arange(T * K, dtype=np.int32)
            plan["pair_pos"] = torch.from_numpy(pp.reshape(T, K))
        return plan

    def pack_dedup(self, x2, n: int, topi, topw, W: int, plan: dict, combine: str):
        ti, tw = topi.numpy(), topw.numpy()
        T, K = ti.shape
        leid = np.full((n, K), -1, dtype=np.int32)
        ret = np.full((n, K), -1, dtype=np.int32)
        wts = np.zeros((n, K), dtype=np.float32)
        pos = np.full((T, K), n, dtype=np.int32)
        ids = plan["send_ids"].numpy()
        base = np.concatenate([[0], np.cumsum([c[1] for c in plan["counts"]])])
        for p, i in enumerate(ids):
            t, d = divmod(int(i), W)
            first = True
            for k in range(K):
                if ti[t, k] // self.E_loc == d:
                    leid[p, k] = ti[t, k] % self.E_loc
                    wts[p, k] = tw[t, k]
                    if combine == "pairs":
                        ret[p, k] = int(plan["pair_pos"][t, k]) - base[d]
                    if first:
                        pos[t, k] = p
                        first = False
        rows = x2[torch.from_numpy(ids.astype(np.int64) // W)].contiguous()
        if combine == "pairs":
            return rows, torch.from_numpy(leid), torch.from_numpy(ret)
        return rows, torch.from_numpy(leid), (torch.from_numpy(wts), torch.from_numpy(pos))

    def local_experts_return(self, rows, leid, ret_idx, rows_in, pairs_in):
        n, K = leid.shape
        y = torch.zeros(sum(pairs_in), rows.shape[1], dtype=torch.bfloat16)
        rp = np.concatenate([[0], np.cumsum(rows_in)])
        pp = np.concatenate([[0], np.cumsum(pairs_in)])
        lid, ri = leid.numpy(), ret_idx.numpy()
        for i in range(n):
            s = int(np.searchsorted(rp, i, side="right") - 1)
            for j in range(K):
                if lid[i, j] >= 0:
                    y[pp[s] + ri[i, j]] = self.local_experts(rows[i:i + 1], leid[i, j:j + 1])[0]
        return y

    def merge_pairs(self, ret, pair_pos, topw, h1, ys):
        T, K = topw.shape
        y = ret.float().numpy()[pair_pos.numpy().astype(np.int64)]
        acc = (y * topw.numpy()[..., None]).sum(1) + h1.float().numpy() + ys.numpy()
        return _bf(acc)

    def local_experts_dedup(self, rows, leid, wts, pairs: int):
        n, K = leid.shape
        lid, w = leid.numpy(), wts.numpy()
        out = np.zeros((n, rows.shape[1]), dtype=np.float32)
        for i in range(n):
            for j in range(K):
                if lid[i, j] < 0:
                    continue
                y = self.local_experts(rows[i:i + 1], leid[i, j:j + 1]).float().numpy()[0]
                out[i] += w[i, j] * y
        return _bf(out)

    def merge_dedup(self, ret, pos, h1, ys):
        r = ret.float().numpy()
        acc = r[pos.numpy().astype(np.int64)].sum(1) + h1.float().numpy() + ys.numpy()
        return _bf(acc)

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
