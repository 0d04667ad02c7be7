"""GPU tests of expert parallelism: the plan/pack/unpack kernels against their
definitions, the EP path on one rank against the single-GPU block, and (with two GPUs
visible) two NCCL ranks against the single-GPU block on the same tokens."""

from __future__ import annotations

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
    res = ep.forward_fixed(h, r) if fixed else ep(h, r)
    finish()
    assert torch.equal(res["topi"], ref.topi)
    assert torch.equal(res["h1"].view(torch.int16), ref.h1.view(torch.int16))
    _parity(res["out"], ref.out)
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
    dist.init_process_group("nccl", rank=rank, world_size=2,
                            device_id=torch.device("cuda", rank))
    try:
        w = shard_weights(404, rank, 2, D, "cuda")
        be = CudaEPBackend(w["gamma"], w["gate_w"], w["bias"], w["w13"], w["w2"], w["w13s"],
                           w["w2s"], E=D.E, rank=rank)
        ep = ExpertParallelMoE(be)
        h, r = synth.make_inputs(70 + rank, 24, D, "cuda")
        out = ep(h, r)["out"]
        h2, r2 = synth.make_inputs(90 + rank, 2, D, "cuda")
        g = EPDecodeGraph(ep, 2, D.H, "cuda", exchange="nccl")  # all_to_all in a CUDA graph
        g.h.copy_(h2)
        g.r.copy_(r2)
        out2 = g.replay()
        gp = EPDecodeGraph(ep, 2, D.H, "cuda", exchange="p2p")  # NVLink peer stores
        gp.h.copy_(h2)
        gp.r.copy_(r2)
        for _ in range(3):
            out3 = gp.replay()
        st = EPDecodeStep(be, 2).capture()  # one library call per step, graphed
        st.h.copy_(h2)
        st.r.copy_(r2)
        for _ in range(3):
            out4 = st.replay()
        torch.cuda.synchronize()
        ops.check_status()
        same = bool(torch.equal(out2.view(torch.int16), out3.view(torch.int16)) and
                    torch.equal(out2.view(torch.int16), out4.view(torch.int16)))
        q.put((rank, (out.float().cpu().numpy(), out2.float().cpu().numpy(), same)))
        del g  # the graph holds NCCL work: release it before the communicator
        torch.cuda.synchronize()
        gp.close()
        st.close()
        dist.barrier()
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
    outs = dict(q.get(timeout=240) for _ in range(2))
    for p in ps:
        p.join(timeout=60)
        if p.is_alive():  # results are in; do not let a slow teardown hold the test
            p.terminate()
            p.join(timeout=10)
    w = synth.make_block_weights(404, D, DEV)
    blk = MoEBlock(w["gamma"], w["gate_w"], w["bias"], w["w13"], w["w2"], w["w13s"], w["w2s"])
    for rank in range(2):
        assert outs[rank][2], "NVLink exchange differs from the all_to_all exchange"
        for (seed, T), got in zip(((70, 24), (90, 2)), outs[rank][:2]):
            h, r = synth.make_inputs(seed + rank, T, D, DEV)
            ref = blk(h, r)
            finish()
            _parity(torch.from_numpy(got), ref.out)
