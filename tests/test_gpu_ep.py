"""GPU tests of expert parallelism: the plan/pack/unpack kernels (per pair and
deduplicated) against their definitions, the EP path on one rank against the single-GPU
block, and (with two GPUs visible) two NCCL ranks against the single-GPU block on the
same tokens."""

from __future__ import annotations

import datetime
import os
import socket
import sys
from pathlib import Path

import numpy as np
import pytest
import torch

from fusion_b200 import ops, synth
from fusion_b200.block import MoEBlock
from fusion_b200.ep import (CudaEPBackend, EPDecodeGraph, EPDecodeStep, ExpertParallelMoE,
                            P2PExchange, shard_weights)
from oracle import reference_np as O
from gpu_util import DEV, finish

pytestmark = pytest.mark.gpu
HERE = Path(__file__).resolve().parent
D = synth.Dims()


def test_ep_plan_pack_unpack_kernels():
    T, K, E, W, H = 300, 8, 256, 4, 6144
    rng = np.random.default_rng(1)
    ids = np.stack([rng.choice(E, K, replace=False) for _ in range(T)]).astype(np.int32)
    topi = torch.from_numpy(ids).to(DEV)
    E_loc = E // W
    dest = torch.empty(T * K, dtype=torch.int32, device=DEV)
    leid = torch.empty_like(dest)
    counts = torch.empty(W, dtype=torch.int32, device=DEV)
    ops.ep_plan(topi, E_loc, W, dest, leid, counts)
    send = torch.empty(T * K, dtype=torch.int32, device=DEV)
    eids = torch.empty_like(send)
    ntp = torch.zeros(1, dtype=torch.int32, device=DEV)
    ops.moe_align(dest, W, 1, send, eids, ntp)
    x = torch.randn(T, H, device=DEV).to(torch.bfloat16)
    rows = torch.empty(T * K, H, dtype=torch.bfloat16, device=DEV)
    lo = torch.empty(T * K, dtype=torch.int32, device=DEV)
    ops.ep_pack(x, send, T * K, K, leid, rows, lo)
    y = torch.empty_like(rows)
    ops.ep_unpack(rows, send, T * K, y)
    finish()
    flat = ids.reshape(-1)
    assert np.array_equal(dest.cpu().numpy(), flat // E_loc)
    assert np.array_equal(leid.cpu().numpy(), flat % E_loc)
    assert np.array_equal(counts.cpu().numpy(), np.bincount(flat // E_loc, minlength=W))
    ref_send = np.argsort(flat // E_loc, kind="stable")
    assert np.array_equal(send.cpu().numpy(), ref_send)
    assert torch.equal(rows, x[torch.from_numpy(ref_send // K).to(DEV)])
    assert np.array_equal(lo.cpu().numpy(), (flat % E_loc)[ref_send])
    assert torch.equal(y, x.repeat_interleave(K, 0))  # unpack inverts pack


def test_ep_dedup_plan_pack_partial_kernels():
    """Deduplicated dispatch: keys / counts / send order / packed rows and slot metadata /
    merge positions bit-exact against their definitions; the owner's partial sum within
    bf16 rounding of the fp32 sum."""
    T, K, E, W, H = 300, 8, 256, 4, 6144
    rng = np.random.default_rng(2)
    ids = np.stack([rng.choice(E, K, replace=False) for _ in range(T)]).astype(np.int32)
    topi = torch.from_numpy(ids).to(DEV)
    topw = torch.rand(T, K, device=DEV)
    E_loc = E // W
    keys = torch.empty(T * W, dtype=torch.int32, device=DEV)
    counts = torch.empty(2 * W, dtype=torch.int32, device=DEV)
    ops.ep_plan_dedup(topi, E_loc, W, keys, counts)
    send = torch.empty(T * W, dtype=torch.int32, device=DEV)
    eids = torch.empty_like(send)
    ntp = torch.zeros(1, dtype=torch.int32, device=DEV)
    ops.moe_align(keys, W, 1, send, eids, ntp)
    finish()
    dest = ids // E_loc
    on = np.zeros((T, W), bool)
    for t in range(T):
        on[t, dest[t]] = True
    ref_keys = np.where(on, np.arange(W)[None, :], -1).reshape(-1)
    assert np.array_equal(keys.cpu().numpy(), ref_keys)
    n = int(on.sum())
    assert np.array_equal(counts.cpu().numpy(),
                          np.concatenate([on.sum(0), np.bincount(dest.reshape(-1), minlength=W)]))
    ref_send = np.nonzero(ref_keys >= 0)[0]
    ref_send = ref_send[np.argsort(ref_keys[ref_send], kind="stable")]
    assert int(ntp.item()) == n
    assert np.array_equal(send[:n].cpu().numpy(), ref_send)
    # each pair's position among the pairs stably sorted by destination
    pdest = torch.empty(T * K, dtype=torch.int32, device=DEV)
    pleid, pc = torch.empty_like(pdest), torch.empty(W, dtype=torch.int32, device=DEV)
    ops.ep_plan(topi, E_loc, W, pdest, pleid, pc)
    srt, e2 = torch.empty_like(pdest), torch.empty_like(pdest)
    pair_pos = torch.empty(T, K, dtype=torch.int32, device=DEV)
    ops.moe_align(pdest, W, 1, srt, e2, torch.zeros(1, dtype=torch.int32, device=DEV),
                  pos_of=pair_pos)
    x = torch.randn(T, H, device=DEV).to(torch.bfloat16)
    rows = torch.empty(n, H, dtype=torch.bfloat16, device=DEV)
    leid = torch.empty(n, K, dtype=torch.int32, device=DEV)
    ret = torch.empty(n, K, dtype=torch.int32, device=DEV)
    ops.ep_pack_dedup(x, send, n, W, topi, topw, E_loc, rows, leid, pair_pos=pair_pos,
                      counts=counts, ret_out=ret)
    rows2, leid2 = torch.empty_like(rows), torch.empty_like(leid)
    wts = torch.empty(n, K, dtype=torch.float32, device=DEV)
    pos = torch.empty(T, K, dtype=torch.int32, device=DEV)
    ops.ep_pack_dedup(x, send, n, W, topi, topw, E_loc, rows2, leid2, w_out=wts, pos=pos,
                      zero_row=n)
    finish()
    tw = topw.cpu().numpy()
    order = np.argsort(dest.reshape(-1), kind="stable")
    ref_pp = np.empty(T * K, np.int64)
    ref_pp[order] = np.arange(T * K)
    ref_pp = ref_pp.reshape(T, K)
    assert np.array_equal(pair_pos.cpu().numpy(), ref_pp)
    base = np.concatenate([[0], np.cumsum(np.bincount(dest.reshape(-1), minlength=W))])
    ref_leid = np.full((n, K), -1, np.int32)
    ref_ret = np.full((n, K), -1, np.int32)
    ref_w = np.zeros((n, K), np.float32)
    ref_pos = np.full((T, K), n, np.int32)
    for p, i in enumerate(ref_send):
        t, d = divmod(int(i), W)
        mine = np.nonzero(dest[t] == d)[0]
        ref_leid[p, mine] = ids[t, mine] % E_loc
        ref_ret[p, mine] = ref_pp[t, mine] - base[d]
        ref_w[p, mine] = tw[t, mine]
        ref_pos[t, mine[0]] = p
    assert torch.equal(rows, x[torch.from_numpy(ref_send // W).to(DEV)])
    assert torch.equal(rows2, rows) and torch.equal(leid2, leid)
    assert np.array_equal(leid.cpu().numpy(), ref_leid)
    assert np.array_equal(ret.cpu().numpy(), ref_ret)
    assert np.array_equal(wts.cpu().numpy(), ref_w)
    assert np.array_equal(pos.cpu().numpy(), ref_pos)
    # owner: rows arriving from 3 sources (this batch split 40 / 0 / rest rows), the
    # row map sends slot f of row i to pair_prefix[s] + ret[f]; pads stay past the rows
    rows_in = [40, 0, n - 40]
    pairs_in = [int((ref_leid[:40] >= 0).sum()), 0, int((ref_leid[40:] >= 0).sum())]
    rp = torch.tensor([0, 40, 40, n], dtype=torch.int32, device=DEV)
    pp = torch.tensor([0, pairs_in[0], pairs_in[0], sum(pairs_in)], dtype=torch.int32,
                      device=DEV)
    # each source's return indices: a permutation of its own pairs
    ret_src = np.full((n, K), -1, np.int32)
    for lo, hi in ((0, 40), (40, n)):
        live = ref_leid[lo:hi] >= 0
        blk = ret_src[lo:hi]
        blk[live] = rng.permutation(int(live.sum()))
    flat_live = np.nonzero(ref_leid.reshape(-1) >= 0)[0]
    sorted_ids = np.concatenate([flat_live, np.full(5, n * K)]).astype(np.int32)
    rowmap = torch.empty(sorted_ids.size, dtype=torch.int32, device=DEV)
    ops.ep_return_rowmap(torch.from_numpy(sorted_ids).to(DEV),
                         torch.from_numpy(ret_src).to(DEV), K, rp, pp, rowmap)
    finish()
    ref_map = []
    for f in sorted_ids:
        if f >= n * K:
            ref_map.append(int(f))
            continue
        i = f // K
        src = 0 if i < 40 else 2
        ref_map.append(int([0, pairs_in[0], pairs_in[0]][src] + ret_src.reshape(-1)[f]))
    assert np.array_equal(rowmap.cpu().numpy(), np.array(ref_map))
    assert ops.read_status() == 0
    # a layout buffer longer than its padded total: the tail is never written by
    # moe_align (junk here, negative and in-range values) and must not be read
    junk = np.concatenate([sorted_ids, np.array([-7, 3, 1 << 30, 0], np.int32)])
    ntp = torch.tensor([sorted_ids.size], dtype=torch.int32, device=DEV)
    rowmap2 = torch.empty(junk.size, dtype=torch.int32, device=DEV)
    ops.ep_return_rowmap(torch.from_numpy(junk).to(DEV), torch.from_numpy(ret_src).to(DEV), K,
                         rp, pp, rowmap2, ntp=ntp)
    finish()
    assert np.array_equal(rowmap2.cpu().numpy(), np.array(ref_map + [n * K] * 4))
    # owner: partial = bf16(sum over its slots of w * y); hole rows hold NaN and must be
    # skipped, not multiplied by a zero weight
    y = torch.randn(n * K, H, device=DEV).to(torch.bfloat16)
    y[torch.from_numpy(np.nonzero(ref_leid.reshape(-1) < 0)[0]).to(DEV)] = float("nan")
    part = torch.empty(n, H, dtype=torch.bfloat16, device=DEV)
    ops.ep_partial_sum(y, leid, wts, part)
    finish()
    yf = torch.nan_to_num(y.float().view(n, K, H), nan=0.0)
    ref = (yf * torch.from_numpy(ref_w).to(DEV)[..., None]).sum(1)
    got = part.float()
    assert torch.isfinite(got).all()
    assert float((got - ref).abs().max()) <= float(ref.abs().max()) * 2 ** -7


def test_align_skips_holes():
    rng = np.random.default_rng(5)
    ids = rng.integers(-1, 64, size=(300, 1)).astype(np.int32)  # -1: holes
    t = torch.from_numpy(ids).to(DEV)
    bm, E = 16, 64
    cap = (300 + E * (bm - 1) + bm - 1) // bm * bm
    s_ = torch.empty(cap, dtype=torch.int32, device=DEV)
    e_ = torch.empty(cap // bm, dtype=torch.int32, device=DEV)
    n_ = torch.zeros(1, dtype=torch.int32, device=DEV)
    ops.moe_align(t, E, bm, s_, e_, n_)
    finish()  # no BAD_EXPERT raised for holes
    keep = np.nonzero(ids.reshape(-1) >= 0)[0]
    rs, re_, rn = O.moe_align_block_size(ids.reshape(-1)[keep], bm, E)
    rs = np.where(rs < keep.size, keep[np.minimum(rs, keep.size - 1)], 300)  # back to flat ids
    n = int(n_.item())
    assert n == int(rn[0])
    assert np.array_equal(s_[:n].cpu().numpy(), rs)
    assert np.array_equal(e_[: n // bm].cpu().numpy(), re_)


def _parity(out, ref):
    o, r = out.float().cpu().numpy(), ref.float().cpu().numpy()
    rms = float(np.sqrt((r.astype(np.float64) ** 2).mean()))
    assert float(np.abs(o - r).max()) <= 1e-2 * rms


@pytest.mark.parametrize("T,fixed", [(1, False), (64, False), (1, True), (16, True)])
def test_ep_single_rank_matches_block(T, fixed):
    w = synth.make_block_weights(404, D, DEV)
    blk = MoEBlock(w["gamma"], w["gate_w"], w["bias"], w["w13"], w["w2"], w["w13s"], w["w2s"])
    be = CudaEPBackend(w["gamma"], w["gate_w"], w["bias"], w["w13"], w["w2"], w["w13s"],
                       w["w2s"], E=D.E, rank=0)
    h, r = synth.make_inputs(31 + T, T, D, DEV)
    ref = blk(h, r)
    ep = ExpertParallelMoE(be)
    res = ep.forward_fixed(h, r) if fixed else ep.forward_pairs(h, r)
    finish()
    assert torch.equal(res["topi"], ref.topi)
    assert torch.equal(res["h1"].view(torch.int16), ref.h1.view(torch.int16))
    _parity(res["out"], ref.out)
    if not fixed:
        # deduplicated dispatch (one row per token here) returning one expert row per
        # pair merges exactly like the per-pair exchange
        res_dd = ep.forward_dedup(h, r)
        finish()
        assert torch.equal(res_dd["out"].view(torch.int16), res["out"].view(torch.int16))
        assert res_dd["rows_in"] == T and res_dd["pairs_in"] == T * D.topk
        # partial-sum combine: the owner's bf16 partial adds a rounding before the final
        # sum, so an element may move by up to an ulp of itself
        res_part = ep.forward_dedup(h, r, combine="partial")
        finish()
        o, rr = res_part["out"].float(), ref.out.float()
        rms = float(rr.pow(2).mean().sqrt())
        assert bool(((o - rr).abs() <= 1e-2 * rms + rr.abs() * 2 ** -7).all())
    if fixed:
        # the NVLink exchange (here its loopback on one rank) gives the same bits
        x = P2PExchange(T * D.topk, D.H, DEV)
        for _ in range(2):  # the second step reuses the buffers with the next epoch
            res_p = ep.forward_p2p(h, r, x)
            finish()
            assert torch.equal(res_p["out"].view(torch.int16), res["out"].view(torch.int16))
        x.close()
        for exchange in ("nccl", "p2p"):
            g = EPDecodeGraph(ep, T, D.H, DEV, exchange=exchange)
            g.h.copy_(h)
            g.r.copy_(r)
            for _ in range(2):
                out = g.replay()
                finish()
                assert torch.equal(out.view(torch.int16), res["out"].view(torch.int16))
            g.close()
        # the whole step as one library call (PDL-chained launches), eager and graphed
        st = EPDecodeStep(be, T)
        st.h.copy_(h)
        st.r.copy_(r)
        for _ in range(2):
            out = st.forward()
            finish()
            assert torch.equal(out.view(torch.int16), res["out"].view(torch.int16))
        st.capture()
        for _ in range(2):
            out = st.replay()
            finish()
            assert torch.equal(out.view(torch.int16), res["out"].view(torch.int16))
        assert torch.equal(st.topi, res["topi"])
        st.close()


def test_p2p_wait_times_out_with_status():
    """A flag that nothing raises: the bounded wait gives up and reports FUS_ERR_TIMEOUT;
    the context stays usable."""
    flags = torch.zeros(2, dtype=torch.int32, device=DEV)
    epoch = torch.ones(1, dtype=torch.int32, device=DEV)
    ops.read_status()
    ops.ep_p2p_wait(flags, epoch, 2, timeout_ns=20_000_000)  # 20 ms
    assert ops.read_status() & ops.ERR_TIMEOUT
    flags.fill_(1)
    ops.ep_p2p_wait(flags, epoch, 2, timeout_ns=20_000_000)
    assert ops.read_status() == 0
    finish()


def _two_rank_worker(rank, port, q):
    sys.path.insert(0, str(HERE.parent))
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    # a collective that waits longer than this ends the rank with an error instead of
    # holding the test
    dist.init_process_group("nccl", rank=rank, world_size=2,
                            device_id=torch.device("cuda", rank),
                            timeout=datetime.timedelta(seconds=120))

    def stage(name):  # progress on stderr: a stuck rank shows where it stopped
        print(f"[two-rank test, rank {rank}] {name}", file=sys.stderr, flush=True)

    try:
        stage("init done")
        w = shard_weights(404, rank, 2, D, "cuda")
        be = CudaEPBackend(w["gamma"], w["gate_w"], w["bias"], w["w13"], w["w2"], w["w13s"],
                           w["w2s"], E=D.E, rank=rank)
        ep = ExpertParallelMoE(be)
        h, r = synth.make_inputs(70 + rank, 24, D, "cuda")
        out = ep(h, r, dispatch="pairs")["out"]
        stage("prefill step (all_to_all) done")
        out_dd = ep(h, r, dispatch="dedup")["out"]
        torch.cuda.synchronize()
        ops.check_status()
        stage("prefill step (deduplicated dispatch) done")
        h2, r2 = synth.make_inputs(90 + rank, 2, D, "cuda")
        g = EPDecodeGraph(ep, 2, D.H, "cuda", exchange="nccl")  # all_to_all in a CUDA graph
        g.h.copy_(h2)
        g.r.copy_(r2)
        out2 = g.replay()
        stage("decode graph (all_to_all) done")
        gp = EPDecodeGraph(ep, 2, D.H, "cuda", exchange="p2p")  # NVLink peer stores
        gp.h.copy_(h2)
        gp.r.copy_(r2)
        for _ in range(3):
            out3 = gp.replay()
        stage("decode graph (NVLink) done")
        st = EPDecodeStep(be, 2).capture()  # one library call per step, graphed
        st.h.copy_(h2)
        st.r.copy_(r2)
        for _ in range(3):
            out4 = st.replay()
        stage("decode step (one call) done")
        torch.cuda.synchronize()
        ops.check_status()
        same = bool(torch.equal(out2.view(torch.int16), out3.view(torch.int16)) and
                    torch.equal(out2.view(torch.int16), out4.view(torch.int16)) and
                    torch.equal(out.view(torch.int16), out_dd.view(torch.int16)))
        q.put((rank, (out.float().cpu().numpy(), out2.float().cpu().numpy(), same)))
        stage("results sent")
        del g  # the graph holds NCCL work: release it before the communicator
        torch.cuda.synchronize()
        gp.close()
        st.close()
        dist.barrier()
    except BaseException as e:  # noqa: BLE001 - report, so the parent does not wait out its timeout
        import traceback

        q.put((rank, f"rank {rank} failed: {e!r}\n{traceback.format_exc()}"))
        raise
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_ep_two_nccl_ranks_match_block():
    import torch.multiprocessing as mp

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    ps = [ctx.Process(target=_two_rank_worker, args=(r, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    # drain before joining: a child cannot exit while its result is still in the pipe
    try:
        outs = {}
        while len(outs) < 2:
            rank, res = q.get(timeout=240)
            # a rank that fails posts its traceback at once (its peer may be stuck in a
            # collective until the process-group timeout)
            assert not isinstance(res, str), res
            outs[rank] = res
        for p in ps:
            p.join(timeout=60)
    finally:
        for p in ps:  # results are in (or never came): do not let a child hold the test
            if p.is_alive():
                p.terminate()
                p.join(timeout=10)
    w = synth.make_block_weights(404, D, DEV)
    blk = MoEBlock(w["gamma"], w["gate_w"], w["bias"], w["w13"], w["w2"], w["w13s"], w["w2s"])
    for rank in range(2):
        assert outs[rank][2], ("NVLink exchange differs from the all_to_all exchange, or "
                               "the deduplicated dispatch from the per-pair one")
        for (seed, T), got in zip(((70, 24), (90, 2)), outs[rank][:2]):
            h, r = synth.make_inputs(seed + rank, T, D, DEV)
            ref = blk(h, r)
            finish()
            _parity(torch.from_numpy(got), ref.out)
