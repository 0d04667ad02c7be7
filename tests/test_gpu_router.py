"""GPU parity: router logits (3-plane fp32 on tcgen05) and sigmoid noaux_tc top-k
against the reference's golden vectors and the oracle. Ids are compared bit-exactly
on every row whose top-9 choice scores are separated by more than 1e-5."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import bf16_from_bits, golden
from fusion_b200 import ops, synth
from gpu_util import DEV, bf, finish, to_np
from oracle import reference_np as O

pytestmark = pytest.mark.gpu
GAP = 1e-5


def gpu_router(x2, gw, bias, topk=8, planes=3):
    T, H = x2.shape
    E = gw.shape[0]
    wa = ops.router_split_weight(gw) if planes == 3 else ops.router_transpose_weight(gw.t().contiguous())
    ns = ops.router_nsplit(T, H, E, planes)
    part = torch.empty(ns, T, E, dtype=torch.float32, device=DEV)
    ops.router_logits(x2, wa, planes, part, ns)
    logits = torch.empty(T, E, dtype=torch.float32, device=DEV)
    tw = torch.empty(T, topk, dtype=torch.float32, device=DEV)
    ti = torch.empty(T, topk, dtype=torch.int32, device=DEV)
    ops.router_topk(part, ns, bias, logits, tw, ti)
    finish()
    return to_np(logits), to_np(tw), ti.cpu().numpy()


def separated_rows(logits, bias, k=8):
    s = O.sigmoid(logits)
    c = s + (bias if bias is not None else 0)
    top = -np.sort(-c, axis=1)[:, : k + 1]
    return np.all(np.diff(-top, axis=1) > GAP, axis=1)


def check_ids(ti, ref_ids, logits_ref, bias):
    ok = separated_rows(logits_ref, bias)
    assert ok.mean() > 0.5
    assert np.array_equal(ti[ok], ref_ids[ok])
    # ambiguous rows still pick the same set of experts up to the tie
    for t in np.nonzero(~ok)[0]:
        assert len(set(ti[t]) ^ set(ref_ids[t])) <= 2


def test_router_golden():
    g = golden("router")
    seed = int(g["seed"])
    x2 = bf(bf16_from_bits(g["x2"]))
    gw = synth.make("gate_w", (256, 6144), seed, DEV)
    bias = synth.make("bias", (256,), seed, DEV)
    lg, tw, ti = gpu_router(x2, gw, bias)
    np.testing.assert_allclose(lg, g["logits"], rtol=0, atol=5e-5)
    check_ids(ti, g["topk_ids"], g["logits"], to_np(bias))
    same = np.all(ti == g["topk_ids"], axis=1)
    np.testing.assert_allclose(tw[same], g["topk_weights"][same], rtol=2e-5, atol=2e-6)
    lg0, tw0, ti0 = gpu_router(x2, gw, None)
    check_ids(ti0, g["topk_ids_nobias"], g["logits_nobias"], None)


def test_router_grouped_golden():
    """noaux_tc group masking (n_group=8, topk_group=4) on the reference's own logits:
    ids bit-exact against its golden ids, weights to fp32 rounding; and against the
    oracle on fresh logits at several T (ties between groups / experts are rare but the
    oracle breaks them by lower index exactly like the kernel)."""
    g = golden("router")
    T = int(g["T"])
    bias = synth.make("bias", (256,), int(g["seed"]), DEV)
    part = torch.from_numpy(g["logits"]).to(DEV).view(1, T, 256).contiguous()
    tw = torch.empty(T, 8, dtype=torch.float32, device=DEV)
    ti = torch.empty(T, 8, dtype=torch.int32, device=DEV)
    ops.router_topk(part, 1, bias, None, tw, ti, n_group=8, topk_group=4)
    finish()
    assert np.array_equal(np.sort(ti.cpu().numpy(), 1), np.sort(g["topk_ids_grouped"], 1))
    assert np.array_equal(ti.cpu().numpy(), g["topk_ids_grouped"])
    np.testing.assert_allclose(tw.cpu().numpy(), g["topk_weights_grouped"], rtol=2e-6, atol=1e-7)
    for Tn, (ng, tg) in ((1, (8, 4)), (77, (8, 4)), (300, (4, 2)), (64, (32, 3))):
        lg = synth.make("r", (Tn, 256), 5 + Tn, "cpu").float().numpy() * 3.0
        pt = torch.from_numpy(lg).to(DEV).view(1, Tn, 256).contiguous()
        tw = torch.empty(Tn, 8, dtype=torch.float32, device=DEV)
        ti = torch.empty(Tn, 8, dtype=torch.int32, device=DEV)
        ops.router_topk(pt, 1, bias, None, tw, ti, n_group=ng, topk_group=tg)
        finish()
        ow, oi = O.router_select(lg, to_np(bias), n_group=ng, topk_group=tg)
        assert np.array_equal(ti.cpu().numpy(), oi), (Tn, ng, tg)
        np.testing.assert_allclose(tw.cpu().numpy(), ow, rtol=2e-6, atol=1e-7)


@pytest.mark.parametrize("T", [1, 33, 256, 2048, 8192])
def test_router_vs_oracle(T):
    x2 = synth.make("h", (T, 6144), 21 + T, DEV)
    gw = synth.make("gate_w", (256, 6144), 21, DEV)
    bias = synth.make("bias", (256,), 21, DEV)
    lg, tw, ti = gpu_router(x2, gw, bias)
    olg = O.router_logits(to_np(x2), to_np(gw))
    # two fp32 dot products of length H summed in different orders: each is within
    # H*u*sum|x w| of the exact value (u = 2^-24); the bar is 32*u*sum|x w| (about 1.5e-4
    # here), plus 5e-5 for logits whose terms cancel
    mag = np.abs(to_np(x2)) @ np.abs(to_np(gw)).T
    err = np.abs(lg - olg)
    assert np.all(err <= 5e-5 + 32 * 2.0**-24 * mag), float((err - 32 * 2.0**-24 * mag).max())
    ow, oi = O.router_select(olg, to_np(bias))
    check_ids(ti, oi, olg, to_np(bias))
    same = np.all(ti == oi, axis=1)
    np.testing.assert_allclose(tw[same], ow[same], rtol=2e-5, atol=2e-6)


def test_router_bf16_weight_plane():
    """norm_router.router_gemm's bf16 [H, E] weight (one plane)."""
    T = 40
    x2 = synth.make("h", (T, 6144), 31, DEV)
    wgt = synth.make("w13", (6144, 256), 31, DEV)  # bf16 [H, E]
    lg, tw, ti = gpu_router(x2, wgt.t().contiguous(), None, planes=1)
    ref = to_np(x2) @ to_np(wgt)
    np.testing.assert_allclose(lg, ref, rtol=0, atol=5e-5)
