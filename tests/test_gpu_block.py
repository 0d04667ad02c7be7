"""GPU parity of the whole MoE block (one C-ABI call) against the reference.

Two references, both on identical seeded inputs:
  * the reference's fp32 path (moe_mlp_exact_fp32 + h1 + exact shared expert): the
    north-star bar, max-abs error <= 2e-2 * rms(out);
  * the reference's framework chain (bf16 at every kernel boundary): its own layer
    check, max-abs / max|ref| <= 5e-2 (glm52/bench/bench_layer.py:573).
T=2: the reference's own outputs (golden vectors). T=1 and T=32: the CPU oracle.
T=256 and T=2048: a torch fp32 GPU restatement of the exact path on the block's own
routing (ids are checked separately against the oracle router)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import bf16_from_bits, golden
from fusion_b200 import ops, synth
from fusion_b200.block import MoEBlock
from gpu_util import DEV, finish, to_np
from oracle import reference_np as O

pytestmark = pytest.mark.gpu
D = synth.Dims()


@pytest.fixture(scope="module")
def weights_404():
    w = synth.make_block_weights(404, D, DEV)
    yield w
    del w
    torch.cuda.empty_cache()


def make_block(w):
    return MoEBlock(w["gamma"], w["gate_w"], w["bias"], w["w13"], w["w2"], w.get("w13s"),
                    w.get("w2s"))


def parity(out: np.ndarray, exact: np.ndarray, bar: float = 2e-2) -> float:
    """North-star bar against the fp32 path."""
    rms = float(np.sqrt((exact.astype(np.float64) ** 2).mean()))
    err = float(np.abs(out.astype(np.float64) - exact).max())
    assert err <= bar * rms, f"max-abs {err:.4g} > {bar} * rms {rms:.4g}"
    return err / rms


def framework_check(out: np.ndarray, fw: np.ndarray):
    """The reference's own layer check against its framework chain."""
    err = float(np.abs(out.astype(np.float64) - fw).max() / np.abs(fw).max())
    assert err <= 5e-2, err


def test_block_t2_golden(weights_404):
    g = golden("block_full_t2")
    blk = make_block(weights_404)
    h, r = synth.make_inputs(404, 2, D, DEV)
    o = blk(h, r)
    finish()
    assert np.array_equal(to_np(o.h1), bf16_from_bits(g["h1"]))
    assert np.array_equal(o.topi.cpu().numpy(), g["topk_ids"])
    np.testing.assert_allclose(to_np(o.topw), g["topk_weights"], rtol=2e-5, atol=2e-6)
    parity(to_np(o.out), g["out_exact"])
    framework_check(to_np(o.out), bf16_from_bits(g["out"]))


def oracle_block(w, h, r):
    cpu = {k: to_np(v) for k, v in w.items() if k in ("gamma", "gate_w", "bias", "w13s", "w2s")}
    cache = {}

    def get(name):
        def f(e):
            if (name, e) not in cache:
                cache[(name, e)] = to_np(w[name][e])
            return cache[(name, e)]
        return f

    res = O.moe_block(to_np(h), to_np(r), cpu["gamma"], cpu["gate_w"], cpu["bias"], get("w13"),
                      get("w2"), cpu.get("w13s"), cpu.get("w2s"), D.E)
    res["exact"] = O.moe_block_exact_fp32(res["x2"], res["h1"], res["topk_weights"],
                                          res["topk_ids"], get("w13"), get("w2"),
                                          cpu.get("w13s"), cpu.get("w2s"), D.E)
    return res


@pytest.mark.parametrize("T", [1, 32])
def test_block_vs_oracle(weights_404, T):
    blk = make_block(weights_404)
    h, r = synth.make_inputs(405 + T, T, D, DEV)
    o = blk(h, r)
    finish()
    ref = oracle_block(weights_404, h, r)
    assert np.array_equal(to_np(o.h1), ref["h1"])
    assert np.array_equal(o.topi.cpu().numpy(), ref["topk_ids"])
    parity(to_np(o.out), ref["exact"])
    framework_check(to_np(o.out), ref["out"])


def torch_block_exact(w, x2, h1, topw, topi):
    """fp32 GPU restatement of the oracle's exact path (moe_block_exact_fp32)."""
    T, H = x2.shape
    I = w["w2"].shape[2]
    out = torch.zeros(T, H, device=DEV)
    xf = x2.float()
    for e in torch.unique(topi).tolist():
        rows, ks = torch.nonzero(topi == e, as_tuple=True)
        hh = xf[rows] @ w["w13"][e].float().t()
        a = torch.nn.functional.silu(hh[:, :I]) * hh[:, I:]
        out.index_add_(0, rows, (a @ w["w2"][e].float().t()) * topw[rows, ks][:, None])
    hs = xf @ w["w13s"].float().t()
    s = (torch.nn.functional.silu(hs[:, :I]) * hs[:, I:]) @ w["w2s"].float().t()
    return out + h1.float() + s


@pytest.mark.parametrize("T,zipf", [(256, False), (2048, False), (2048, True), (8192, False),
                                    (8192, True)])
def test_block_large_vs_torch_fp32(weights_404, T, zipf):
    if zipf:  # BASELINE config 4 routing skew: a few experts get hundreds of tokens
        weights_404 = dict(weights_404, bias=synth.zipf_bias(DEV))
    blk = make_block(weights_404)
    h, r = synth.make_inputs(500 + T, T, D, DEV)
    o = blk(h, r)
    finish()
    x2, h1 = O.add_rmsnorm(to_np(h), to_np(r), to_np(weights_404["gamma"]))
    assert np.array_equal(to_np(o.h1), h1)
    # ids against the oracle router on rows whose top-9 gaps exceed 1e-5
    lg = O.router_logits(x2, to_np(weights_404["gate_w"]))
    ow, oi = O.router_select(lg, to_np(weights_404["bias"]))
    s = O.sigmoid(lg) + to_np(weights_404["bias"])
    top = -np.sort(-s, axis=1)[:, :9]
    sep = np.all(np.diff(-top, axis=1) > 1e-5, axis=1)
    assert np.array_equal(o.topi.cpu().numpy()[sep], oi[sep])
    ref = torch_block_exact(weights_404, torch.from_numpy(x2).to(DEV).to(torch.bfloat16),
                            o.h1, o.topw, o.topi)
    parity(to_np(o.out), to_np(ref))


def test_block_graph_replay_matches_eager(weights_404):
    blk = make_block(weights_404)
    T = 8
    h, r = synth.make_inputs(77, T, D, DEV)
    eager = blk(h, r)
    g, hin, rin, outs, _ = blk.capture(T)
    hin.copy_(h)
    rin.copy_(r)
    g.replay()
    finish()
    assert torch.equal(outs.out.view(torch.int16), eager.out.view(torch.int16))
    assert torch.equal(outs.topi, eager.topi)


@pytest.mark.parametrize("T", [3, 16])
def test_fused_merge_matches_merge_kernel_and_rearms(weights_404, T):
    """The w2 epilogue's last-arriver merge equals the standalone merge kernel bit for
    bit (same summation order) and leaves its counters at zero."""
    from fusion_b200.chain import BlockChain

    blk = make_block(weights_404)
    ch = BlockChain(blk, T)
    h, r = synth.make_inputs(900 + T, T, D, DEV)
    for _ in range(2):  # second call exercises the re-armed counters
        ch.run(h, r)
    finish()
    ref = torch.empty_like(ch.outs.out)
    ops.merge(ch.y.view(T, D.topk, D.H), ch.outs.topw, ch.outs.h1, ch.ys, ref, round_mid=False)
    finish()
    assert torch.equal(ch.outs.out.view(torch.int16), ref.view(torch.int16))
    assert int(ch.counters.abs().sum().item()) == 0
    eager = blk(h, r)
    finish()
    assert torch.equal(eager.out.view(torch.int16), ref.view(torch.int16))


@pytest.mark.parametrize("T", [1, 5, 16])
def test_route_small_equals_separate_kernels(weights_404, T):
    """The one-launch decode front end reproduces add_rmsnorm + router + top-k + layout."""
    w = weights_404
    blk = make_block(w)
    h, r = synth.make_inputs(1200 + T, T, D, DEV)
    bn, E, K = 16, D.E, D.topk
    cap = (T * K + E * (bn - 1) + bn - 1) // bn * bn
    h1a, x2a = torch.empty_like(h), torch.empty_like(h)
    ops.add_rmsnorm(h, r, w["gamma"], h1a, x2a)
    ns = ops.router_nsplit(T, D.H, E, blk.nplanes)
    part = torch.empty(ns, T, E, device=DEV)
    ops.router_logits(x2a, blk.wa, blk.nplanes, part, ns)
    twa = torch.empty(T, K, device=DEV)
    tia = torch.empty(T, K, dtype=torch.int32, device=DEV)
    lga = torch.empty(T, E, device=DEV)
    ops.router_topk(part, ns, w["bias"], lga, twa, tia)
    sa = torch.full((cap,), -1, dtype=torch.int32, device=DEV)
    ea = torch.full((cap // bn,), -1, dtype=torch.int32, device=DEV)
    na = torch.zeros(1, dtype=torch.int32, device=DEV)
    ops.moe_align(tia, E, bn, sa, ea, na)
    h1b, x2b = torch.empty_like(h), torch.empty_like(h)
    twb, tib, lgb = torch.empty_like(twa), torch.empty_like(tia), torch.empty_like(lga)
    sb, eb = torch.full_like(sa, -1), torch.full_like(ea, -1)
    nb = torch.zeros(1, dtype=torch.int32, device=DEV)
    done = torch.zeros(4, dtype=torch.int32, device=DEV)
    junk = torch.full((64,), 7, dtype=torch.int32, device=DEV)
    for _ in range(2):  # the ticket re-arms
        ops.route_small(h, r, w["gamma"], blk.wa, blk.nplanes, w["bias"], h1b, x2b, lgb, twb,
                        tib, bn, sb, eb, nb, done, junk)
    finish()
    assert torch.equal(h1a.view(torch.int16), h1b.view(torch.int16))
    assert torch.equal(x2a.view(torch.int16), x2b.view(torch.int16))
    assert torch.equal(tia, tib)
    np.testing.assert_allclose(twb.cpu().numpy(), twa.cpu().numpy(), rtol=1e-6, atol=1e-7)
    n = int(na.item())
    assert int(nb.item()) == n and torch.equal(sa[:n], sb[:n])
    assert torch.equal(ea[: n // bn], eb[: n // bn])
    assert int(done.sum().item()) == 0 and int(junk.abs().sum().item()) == 0


def test_workspace_reused_across_sizes(weights_404):
    """One workspace serves calls of different T (decode and prefill paths alternating)."""
    blk = make_block(weights_404)
    for seed, T in ((70, 24), (90, 2), (71, 300), (91, 2), (92, 1)):
        h, r = synth.make_inputs(seed, T, D, DEV)
        o = blk(h, r)
        finish()
        fresh = make_block(weights_404)(h, r)
        finish()
        assert torch.equal(o.out.view(torch.int16), fresh.out.view(torch.int16))


def test_empty_batch_is_a_no_op(weights_404):
    """T = 0 through the block and the drop-in entry points: no error, nothing written
    (the reference's torch functions accept empty batches)."""
    from fusion_b200 import ops
    from fusion_b200.kernels import add_rmsnorm as KN
    from fusion_b200.kernels import merge_resadd as KM
    from fusion_b200.kernels import norm_router as KR

    blk = make_block(weights_404)
    h = torch.empty(0, D.H, dtype=torch.bfloat16, device=DEV)
    o = blk(h, torch.empty_like(h))
    assert o.out.shape == (0, D.H) and o.topi.shape == (0, D.topk)
    KN.fused_add_rmsnorm(h, h, weights_404["gamma"], torch.empty_like(h), torch.empty_like(h), {})
    lg = torch.empty(0, D.E, dtype=torch.float32, device=DEV)
    KR.router_gemm(h, KR.wgt_from_gate(weights_404["gate_w"].to(torch.bfloat16)), lg, {})
    KR.topk_only(lg, torch.empty(0, D.topk, device=DEV),
                 torch.empty(0, D.topk, dtype=torch.int32, device=DEV), {})
    y = torch.empty(0, D.topk, D.H, dtype=torch.bfloat16, device=DEV)
    KM.fused_merge_resadd(y, torch.empty(0, D.topk, device=DEV), h, torch.empty_like(h), {})
    ids = torch.empty(0, D.topk, dtype=torch.int32, device=DEV)
    cap = D.E * 15 + 16
    s = torch.full((cap,), -7, dtype=torch.int32, device=DEV)
    e = torch.full((cap // 16,), -7, dtype=torch.int32, device=DEV)
    n = torch.full((1,), -7, dtype=torch.int32, device=DEV)
    ops.moe_align(ids, D.E, 16, s, e, n)
    a = torch.empty(0, 32768, dtype=torch.bfloat16, device=DEV)
    ops.oproj_resadd(a, torch.zeros(D.H, 32768, dtype=torch.bfloat16, device=DEV), h,
                     torch.empty_like(h))
    finish()
    assert int(n.item()) == 0


@pytest.mark.parametrize("T", [1, 9, 64])
def test_grouped_routing_block(weights_404, T):
    """noaux_tc group masking (n_group 8, topk_group 4) through the whole block: the fused
    decode front end (T <= 16) and the separate router kernels give the oracle's grouped
    ids wherever the choice scores are separated, and the block output stays within the
    exact-fp32 bar computed from those ids."""
    w = weights_404
    blk = MoEBlock(w["gamma"], w["gate_w"], w["bias"], w["w13"], w["w2"], w["w13s"], w["w2s"],
                   n_group=8, topk_group=4)
    h, r = synth.make_inputs(123 + T, T, D, DEV)
    o = blk(h, r)
    finish()
    x2, h1 = O.add_rmsnorm(to_np(h), to_np(r), to_np(w["gamma"]))
    lg = O.router_logits(x2, w["gate_w"].cpu().numpy())
    ow, oi = O.router_select(lg, w["bias"].cpu().numpy(), n_group=8, topk_group=4)
    ti = o.topi.cpu().numpy()
    # the masked choice scores: rows whose top-9 are separated by > 1e-5 must match exactly
    ch = O.sigmoid(lg) + w["bias"].cpu().numpy()
    g = ch.reshape(T, 8, D.E // 8)
    keep = O.topk_desc(np.sort(g, -1)[..., -2:].sum(-1), 4)
    mask = np.zeros((T, 8), dtype=np.float32)
    np.put_along_axis(mask, keep, 1.0, axis=1)
    ch = (g * mask[..., None]).reshape(T, D.E)
    top9 = -np.sort(-ch, axis=1)[:, :9]
    clear = np.all(np.diff(-top9, axis=1) > 1e-5, axis=1)
    assert np.array_equal(ti[clear], oi[clear])
    same = np.all(ti == oi, axis=1)
    np.testing.assert_allclose(o.topw.cpu().numpy()[same], ow[same], rtol=2e-5, atol=2e-6)
