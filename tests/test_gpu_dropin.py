"""GPU tests of the drop-in surface (fusion_b200.kernels.*, the layer-chain driver):
same names and arguments as glm52/kernels/*.py, checked against the oracle / torch fp32
and for the reference's fused == unfused identities."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from fusion_b200 import synth
from fusion_b200.bench import bench_layer as BL
from fusion_b200.kernels import add_rmsnorm as KN
from fusion_b200.kernels import layout as KL
from fusion_b200.kernels import merge_resadd as KM
from fusion_b200.kernels import moe_down_merge as KD
from fusion_b200.kernels import moe_gateup as KG
from fusion_b200.kernels import norm_router as KR
from gpu_util import DEV, finish, rel_err, to_np
from oracle import reference_np as O

pytestmark = pytest.mark.gpu
H, I, E, K = 6144, 2048, 256, 8


@pytest.fixture(scope="module")
def moe():
    T = 40
    d = synth.Dims(E=16)  # 16 experts keep the weights small; ids drawn from 16
    w13 = synth.make("w13", (16, 2 * I, H), 3, DEV)
    w2 = synth.make("w2", (16, H, I), 3, DEV)
    x = synth.make("h", (T, H), 3, DEV)
    rng = np.random.default_rng(0)
    ids = torch.from_numpy(np.stack([rng.choice(16, K, replace=False) for _ in range(T)])
                           .astype(np.int32)).to(DEV)
    tw = torch.rand(T, K, device=DEV)
    return dict(T=T, w13=w13, w2=w2, x=x, ids=ids, tw=tw)


def test_gateup_fused_vs_unfused(moe):
    T, x, w13, ids = moe["T"], moe["x"], moe["w13"], moe["ids"]
    sti, eid, ntp = KL.moe_align_block_size(ids, 16, 16)
    inter = torch.empty(T * K, 2 * I, dtype=torch.bfloat16, device=DEV)
    act = torch.empty(T * K, I, dtype=torch.bfloat16, device=DEV)
    act_f = torch.empty_like(act)
    KG.launch_gateup(x, w13, inter, sti, eid, ntp, T * K, K, I, {"BLOCK_M": 16}, False)
    KG.launch_silu_and_mul(inter, act, {})
    KG.launch_gateup(x, w13, act_f, sti, eid, ntp, T * K, K, I, {"BLOCK_M": 16}, True)
    finish()
    # torch fp32 reference of the unfused rows
    flat = torch.arange(T * K, device=DEV)
    e = ids.reshape(-1).long()
    ref = torch.stack([x[f // K].float() @ w13[e[f]].float().t() for f in flat.tolist()])
    assert rel_err(inter.float().cpu().numpy(), ref.cpu().numpy()) < 1e-2
    r_act = torch.nn.functional.silu(ref[:, :I]) * ref[:, I:]
    assert rel_err(act.float().cpu().numpy(), r_act.cpu().numpy()) < 1e-2
    assert rel_err(act_f.float().cpu().numpy(), r_act.cpu().numpy()) < 1e-2


@pytest.mark.parametrize("bm", [16, 64])
def test_down_variants_agree(moe, bm):
    T, w2, ids, tw = moe["T"], moe["w2"], moe["ids"], moe["tw"]
    a = (torch.randn(T * K, I, device=DEV)).to(torch.bfloat16)
    sti, eid, ntp = KL.moe_align_block_size(ids, bm, 16)
    tw_flat = tw.flatten().contiguous()
    y3 = torch.zeros(T * K, H, dtype=torch.bfloat16, device=DEV)
    KD.launch_down(a, w2, y3, tw_flat, sti, eid, ntp, T * K, K, {"BLOCK_M": bm}, False)
    res = synth.make("r", (T, H), 4, DEV)
    out_sum = torch.empty(T, H, dtype=torch.bfloat16, device=DEV)
    KD.launch_moe_sum(y3.view(T, K, H), out_sum, res, K, {}, True)
    out_at = torch.empty_like(out_sum)
    KD.launch_seed(out_at, res, {}, True)
    KD.launch_down(a, w2, out_at, tw_flat, sti, eid, ntp, T * K, K, {"BLOCK_M": bm}, True)
    out_tm = torch.empty_like(out_sum)
    KD.launch_down_token_major(a, w2, out_tm, tw, ids, res, K, {}, True)
    finish()
    e = ids.reshape(-1).long()
    ref_rows = torch.stack([(a[f].float() @ w2[e[f]].float().t()) * tw_flat[f]
                            for f in range(T * K)])
    assert rel_err(y3.float().cpu().numpy(), ref_rows.cpu().numpy()) < 1e-2
    ref = ref_rows.view(T, K, H).sum(1) + res.float()
    for o in (out_sum, out_at, out_tm):
        assert rel_err(o.float().cpu().numpy(), ref.cpu().numpy()) < 1e-2
    assert torch.equal(out_sum.view(torch.int16), out_at.view(torch.int16))


def test_norm_and_merge_identities():
    T = 33
    x = synth.make("h", (T, H), 5, DEV)
    r = synth.make("r", (T, H), 5, DEV)
    g = synth.make("gamma", (H,), 5, DEV)
    h1a, x2a, h1b, x2b = (torch.empty_like(x) for _ in range(4))
    KN.fused_add_rmsnorm(x, r, g, h1a, x2a, {})
    KN.add_only(x, r, h1b, {})
    KN.norm_only(h1b, g, x2b, {})
    y = synth.make("h", (T, K, H), 6, DEV)
    wt = torch.rand(T, K, device=DEV)
    fused, m, unf = (torch.empty(T, H, dtype=torch.bfloat16, device=DEV) for _ in range(3))
    KM.fused_merge_resadd(y, wt, r, fused, {})
    KM.merge_only(y, wt, m, {})
    KM.resadd_only(m, r, unf, {})
    finish()
    assert torch.equal(x2a.view(torch.int16), x2b.view(torch.int16))
    assert torch.equal(fused.view(torch.int16), unf.view(torch.int16))  # ROUND_MID identity


def test_router_dropin_matches_oracle():
    T = 20
    x2 = synth.make("h", (T, H), 8, DEV)
    gw = synth.make("gate_w", (E, H), 8, DEV)
    logits = torch.empty(T, E, device=DEV)
    KR.router_gemm(x2, KR.wgt_from_gate(gw), logits, {})  # fp32 [H, E] weight: 3 planes
    tw = torch.empty(T, K, device=DEV)
    ti = torch.empty(T, K, dtype=torch.int32, device=DEV)
    KR.topk_only(logits, tw, ti, {})
    finish()
    ol = O.router_logits(to_np(x2), to_np(gw))
    np.testing.assert_allclose(to_np(logits), ol, atol=5e-5, rtol=0)
    ow, oi = O.router_select(ol, None)
    same = np.all(ti.cpu().numpy() == oi, axis=1)
    assert same.mean() > 0.9
    np.testing.assert_allclose(to_np(tw)[same], ow[same], rtol=2e-5, atol=2e-6)


def test_layer_chain_driver_all_configs_correct():
    w = synth.make_block_weights(0, synth.Dims(), DEV)
    for regime in ("decode_bs1", "decode_bs32"):
        res = BL.run_regime(regime, rep=3, weights=w, verbose=False)
        bad = {k: v["rel_err_vs_fp32_ref"] for k, v in res["rows"].items() if not v["correct"]}
        assert not bad, bad
        assert res["best"] is not None
