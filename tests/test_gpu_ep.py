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
from fusion_b200.ep import CudaEPBackend, ExpertParallelMoE, shard_weights
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


def _parity(out, ref):
    o, r = out.float().cpu().numpy(), ref.float().cpu().numpy()
    rms = float(np.sqrt((r.astype(np.float64) ** 2).mean()))
    assert float(np.abs(o - r).max()) <= 1e-2 * rms


@pytest.mark.parametrize("T", [1, 64])
def test_ep_single_rank_matches_block(T):
    w = synth.make_block_weights(404, D, DEV)
    blk = MoEBlock(w["gamma"], w["gate_w"], w["bias"], w["w13"], w["w2"], w["w13s"], w["w2s"])
    be = CudaEPBackend(w["gamma"], w["gate_w"], w["bias"], w["w13"], w["w2"], w["w13s"],
                       w["w2s"], E=D.E, rank=0)
    h, r = synth.make_inputs(31 + T, T, D, DEV)
    ref = blk(h, r)
    res = ExpertParallelMoE(be)(h, r)
    finish()
    assert torch.equal(res["topi"], ref.topi)
    assert torch.equal(res["h1"].view(torch.int16), ref.h1.view(torch.int16))
    _parity(res["out"], ref.out)


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
        h, r = synth.make_inputs(70 + rank, 24, D, "cuda")
        out = ExpertParallelMoE(be)(h, r)["out"]
        torch.cuda.synchronize()
        q.put((rank, out.float().cpu().numpy()))
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
        assert p.exitcode == 0
    w = synth.make_block_weights(404, D, DEV)
    blk = MoEBlock(w["gamma"], w["gate_w"], w["bias"], w["w13"], w["w2"], w["w13s"], w["w2s"])
    for rank in range(2):
        h, r = synth.make_inputs(70 + rank, 24, D, DEV)
        ref = blk(h, r)
        finish()
        _parity(torch.from_numpy(outs[rank]), ref.out)
