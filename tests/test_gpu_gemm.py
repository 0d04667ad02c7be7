"""GPU parity of the tcgen05 grouped GEMM against a torch fp32 reference (floating
point: bf16 outputs within rel-err 1e-2 of max|ref|, fp32 outputs within 1e-5)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from fusion_b200 import ops
from gpu_util import DEV, finish, rel_err
from oracle import reference_np as O

pytestmark = pytest.mark.gpu


def layout(T, K, E, bn, seed):
    rng = np.random.default_rng(seed)
    ids = np.stack([rng.choice(E, K, replace=False) for _ in range(T)]).astype(np.int32)
    s, e, n = O.moe_align_block_size(ids, bn, E)
    cap = s.size
    return (ids, torch.from_numpy(s).to(DEV), torch.from_numpy(e).to(DEV),
            torch.from_numpy(n).to(DEV), cap)


def ref_rows(x_sorted, w, eids, bn, fn):
    """fp32 per block: fn(x_rows_fp32, w[e] fp32)."""
    outs = []
    for b in range(eids.numel()):
        e = int(eids[b])
        outs.append(fn(x_sorted[b * bn:(b + 1) * bn].float(), w[e].float()))
    return torch.cat(outs)


@pytest.mark.parametrize("bn", [16, 32, 64, 128, 256])
def test_swiglu_and_down_small(bn):
    T, K, E, H, I = 150, 4, 6, 512, 128
    ids, s, eids, ntp, cap = layout(T, K, E, bn, bn)
    R = T * K
    x = (torch.randn(T, H, device=DEV) * 0.5).to(torch.bfloat16)
    w13 = (torch.randn(E, 2 * I, H, device=DEV) * 0.05).to(torch.bfloat16)
    w2 = (torch.randn(E, H, I, device=DEV) * 0.05).to(torch.bfloat16)
    xs = torch.empty(cap, H, dtype=torch.bfloat16, device=DEV)
    ops.permute_rows(x, s, ntp, K, R, xs)
    act = torch.full((cap, I), float("nan"), dtype=torch.bfloat16, device=DEV)
    g = ops.gemm_group(w13, xs, act, expert_ids=eids, ntp=ntp, max_blocks=cap // bn,
                       row_limit=cap)
    ops.grouped_gemm([g], 2 * I, H, ops.FUS_EPI_SWIGLU, bn)
    finish()

    def swiglu(xr, w):
        h = xr @ w.t()
        return torch.nn.functional.silu(h[:, :I]) * h[:, I:]

    ref = ref_rows(xs, w13, eids.cpu(), bn, swiglu)
    live = torch.from_numpy(s.cpu().numpy() < R)  # dispatch pads are neither read nor written
    assert rel_err(act.float().cpu()[live].numpy(), ref.cpu()[live].numpy()) < 1e-2

    # down projection with routed-weight scale, scattered to flat rows
    scale = torch.rand(R, device=DEV)
    y = torch.full((R, H), float("nan"), dtype=torch.bfloat16, device=DEV)
    g2 = ops.gemm_group(w2, act, y, expert_ids=eids, ntp=ntp, max_blocks=cap // bn, row_map=s,
                        row_limit=R, row_scale=scale, live_ids=s, live_limit=R)
    ops.grouped_gemm([g2], H, I, ops.FUS_EPI_BF16, bn)
    finish()
    yref = torch.empty(R, H, device=DEV)
    down = ref_rows(act, w2, eids.cpu(), bn, lambda a, w: a @ w.t())  # pad rows: garbage, unused
    sc = s.cpu().numpy()
    valid = torch.from_numpy(np.nonzero(sc < R)[0]).to(DEV)
    yref[s[valid].long()] = down[valid] * scale[s[valid].long()][:, None]
    assert not torch.isnan(y.float()).any()
    assert rel_err(y.float().cpu().numpy(), yref.cpu().numpy()) < 1e-2


def test_two_groups_real_dims():
    """Routed (sorted, 8 experts) + dense shared group in one launch at GLM dims;
    K = 6144 runs 96 k-steps through the ring (many phase flips)."""
    T, K, E, H, I, bn = 3, 8, 16, 6144, 2048, 16
    ids, s, eids, ntp, cap = layout(T, K, E, bn, 5)
    R = T * K
    x = (torch.randn(T, H, device=DEV)).to(torch.bfloat16)
    w13 = (torch.randn(E, 2 * I, H, device=DEV) * 0.02).to(torch.bfloat16)
    w13s = (torch.randn(2 * I, H, device=DEV) * 0.02).to(torch.bfloat16)
    xs = torch.empty(cap, H, dtype=torch.bfloat16, device=DEV)
    ops.permute_rows(x, s, ntp, K, R, xs)
    act = torch.empty(cap, I, dtype=torch.bfloat16, device=DEV)
    act_s = torch.empty(T, I, dtype=torch.bfloat16, device=DEV)
    maxb = min(R, E) + R // bn
    g0 = ops.gemm_group(w13, xs, act, expert_ids=eids, ntp=ntp, max_blocks=maxb, row_limit=cap)
    g1 = ops.gemm_group(w13s, x, act_s, max_blocks=1, row_limit=T)
    ops.grouped_gemm([g0, g1], 2 * I, H, ops.FUS_EPI_SWIGLU, bn)
    finish()

    def swiglu(xr, w):
        h = xr @ w.t()
        return torch.nn.functional.silu(h[:, :I]) * h[:, I:]

    ref = ref_rows(xs, w13, eids.cpu(), bn, swiglu)
    live = torch.from_numpy(s.cpu().numpy() < R)
    assert rel_err(act.float().cpu()[live].numpy(), ref.cpu()[live].numpy()) < 1e-2
    refs = swiglu(x.float(), w13s.float())
    assert rel_err(act_s.float().cpu().numpy(), refs.cpu().numpy()) < 1e-2


@pytest.mark.parametrize("T,ksplit", [(5, 1), (5, 6), (130, 3)])
def test_f32_planes_splitk(T, ksplit):
    E, H = 256, 1024
    x = torch.randn(T, H, device=DEV).to(torch.bfloat16)
    w = torch.randn(E, H, device=DEV) * 0.02
    wa = ops.router_split_weight(w)
    ks = 3 * H // 64
    kps = -(-ks // ksplit)
    ksplit = -(-ks // kps)
    part = torch.zeros(ksplit, T, E, device=DEV)
    bn = 16 if T <= 16 else 256
    g = ops.gemm_group(wa, x, part, max_blocks=-(-T // bn), row_limit=T)
    ops.grouped_gemm([g], E, H, ops.FUS_EPI_F32, bn, a_kplanes=3, ksplit=ksplit,
                     split_stride=T * E)
    finish()
    got = part.sum(0)
    ref = x.double() @ w.double().t()
    assert (got.double() - ref).abs().max().item() < 1e-4


@pytest.mark.parametrize("bn", [16, 128])
def test_gathered_rows_equal_permuted_rows(bn):
    """B rows gathered by the GEMM itself (TMA gather4 by dispatch position) give the same
    bits as the same GEMM over rows permuted beforehand."""
    T, K, E, H, I = 70, 8, 8, 1024, 256
    ids, s, eids, ntp, cap = layout(T, K, E, bn, 11 + bn)
    R = T * K
    x = (torch.randn(T, H, device=DEV)).to(torch.bfloat16)
    w13 = (torch.randn(E, 2 * I, H, device=DEV) * 0.05).to(torch.bfloat16)
    xs = torch.zeros(cap, H, dtype=torch.bfloat16, device=DEV)
    ops.permute_rows(x, s, ntp, K, R, xs)
    a1 = torch.zeros(cap, I, dtype=torch.bfloat16, device=DEV)
    a2 = torch.zeros(cap, I, dtype=torch.bfloat16, device=DEV)
    g1 = ops.gemm_group(w13, xs, a1, expert_ids=eids, ntp=ntp, max_blocks=cap // bn,
                        row_limit=cap, live_ids=s, live_limit=R)
    g2 = ops.gemm_group(w13, x, a2, expert_ids=eids, ntp=ntp, max_blocks=cap // bn,
                        row_limit=cap, live_ids=s, live_limit=R, gather_ids=s, gather_div=K)
    ops.grouped_gemm([g1], 2 * I, H, ops.FUS_EPI_SWIGLU, bn)
    ops.grouped_gemm([g2], 2 * I, H, ops.FUS_EPI_SWIGLU, bn)
    finish()
    live = torch.from_numpy(s.cpu().numpy() < R).to(DEV)
    assert torch.equal(a1[live].view(torch.int16), a2[live].view(torch.int16))


@pytest.mark.parametrize("bn", [64, 128, 256])
@pytest.mark.parametrize("epi", ["swiglu", "swiglu_gather", "bf16", "bf16_dense"])
def test_persistent_equals_one_tile_per_cta(bn, epi):
    """The persistent prefill kernel (one CTA per SM looping over tiles) gives the same
    bits as one tile per CTA, routed + dense groups: permuted or gathered token rows,
    scattered rows with row map / scale, dense rows in dispatch order (TMA tile stores),
    fp32 output."""
    T, K, E, H, I = 512, 8, 16, 2048, 1024
    ids, s, eids, ntp, cap = layout(T, K, E, bn, 3 + bn)
    R = T * K
    maxb = min(R, E) + R // bn
    if epi.startswith("swiglu"):
        gather = epi == "swiglu_gather"
        x = (torch.randn(T, H, device=DEV)).to(torch.bfloat16)
        w = (torch.randn(E, 2 * I, H, device=DEV) * 0.03).to(torch.bfloat16)
        ws = (torch.randn(2 * I, H, device=DEV) * 0.03).to(torch.bfloat16)
        xs = torch.empty(cap, H, dtype=torch.bfloat16, device=DEV)
        ops.permute_rows(x, s, ntp, K, R, xs)
        outs = []
        for flag in (0, ops.GEMM_NO_PERSIST):
            a = torch.zeros(cap, I, dtype=torch.bfloat16, device=DEV)
            a_s = torch.zeros(T, I, dtype=torch.bfloat16, device=DEV)
            gs = [ops.gemm_group(w, x if gather else xs, a, expert_ids=eids, ntp=ntp,
                                 max_blocks=maxb, row_limit=cap, live_ids=s, live_limit=R,
                                 flags=flag | ops.GEMM_SWIGLU_EXACT,
                                 gather_ids=s if gather else None, gather_div=K),
                  ops.gemm_group(ws, x, a_s, max_blocks=-(-T // bn), row_limit=T,
                                 flags=ops.GEMM_SWIGLU_EXACT)]
            ops.grouped_gemm(gs, 2 * I, H, ops.FUS_EPI_SWIGLU, bn)
            outs.append((a, a_s))
        finish()
        live = torch.from_numpy(s.cpu().numpy() < R).to(DEV)
        assert torch.equal(outs[0][0][live].view(torch.int16), outs[1][0][live].view(torch.int16))
        assert torch.equal(outs[0][1].view(torch.int16), outs[1][1].view(torch.int16))
    else:
        a = (torch.randn(cap, I, device=DEV)).to(torch.bfloat16)
        a_s = (torch.randn(T, I, device=DEV)).to(torch.bfloat16)
        w = (torch.randn(E, H, I, device=DEV) * 0.03).to(torch.bfloat16)
        ws = (torch.randn(H, I, device=DEV) * 0.03).to(torch.bfloat16)
        scale = torch.rand(R, device=DEV)
        outs = []
        dense = epi == "bf16_dense"
        for flag in (0, ops.GEMM_NO_PERSIST):
            y = torch.zeros(cap if dense else R, H, dtype=torch.bfloat16, device=DEV)
            ys = torch.zeros(T, H, dtype=torch.float32, device=DEV)
            if dense:  # rows stay in dispatch order
                g0 = ops.gemm_group(w, a, y, expert_ids=eids, ntp=ntp, max_blocks=maxb,
                                    row_limit=cap, live_ids=s, live_limit=R, flags=flag)
            else:
                g0 = ops.gemm_group(w, a, y, expert_ids=eids, ntp=ntp, max_blocks=maxb,
                                    row_map=s, row_limit=R, row_scale=scale, live_ids=s,
                                    live_limit=R, flags=flag)
            gs = [g0,
                  ops.gemm_group(ws, a_s, ys, max_blocks=-(-T // bn), row_limit=T,
                                 flags=ops.GEMM_OUT_F32)]
            ops.grouped_gemm(gs, H, I, ops.FUS_EPI_BF16, bn)
            outs.append((y, ys))
        finish()
        assert torch.equal(outs[0][1], outs[1][1])
        ref = ref_rows(a, w, eids.cpu(), bn, lambda aa, ww: aa @ ww.t())
        sc = s.cpu().numpy()
        valid = torch.from_numpy(np.nonzero(sc < R)[0]).to(DEV)
        if dense:  # pad rows of the dense output are unspecified: compare live rows
            y0, y1 = outs[0][0][valid], outs[1][0][valid]
            assert torch.equal(y0.view(torch.int16), y1.view(torch.int16))
            assert rel_err(y0.float().cpu().numpy(), ref[valid].cpu().numpy()) < 1e-2
        else:
            assert torch.equal(outs[0][0].view(torch.int16), outs[1][0].view(torch.int16))
            yref = torch.zeros(R, H, device=DEV)
            yref[s[valid].long()] = ref[valid] * scale[s[valid].long()][:, None]
            assert rel_err(outs[0][0].float().cpu().numpy(), yref.cpu().numpy()) < 1e-2


@pytest.mark.parametrize("layout", ["reference", "balanced"])
@pytest.mark.parametrize("epi", ["swiglu", "bf16"])
def test_pair_tiles_ragged_experts(epi, layout):
    """SM-pair tiles (2-CTA clusters, M = 256, each SM staging half of the token block)
    give the same bits as the single-CTA persistent kernel and as one tile per CTA, on
    expert blocks holding 1 .. 256 live tokens (token boxes of 16 / 64 / 128 rows per
    CTA), with a dense second group (fp32 output on the down projection); and match an
    fp32 reference. Experts with two blocks (300, 257 and 511 tokens) and three (513), in
    the reference layout (full block + remainder) and the balanced one; on the down
    projection both the 512-row pair tiles (default) and the 256-row ones."""
    counts = [1, 17, 100, 130, 256, 300, 513, 40, 257, 511]
    E, bn = len(counts), 256
    ids = np.concatenate([np.full(c, e, np.int32) for e, c in enumerate(counts)])
    ids = np.random.default_rng(5).permutation(ids)[:, None]
    T = ids.shape[0]
    if layout == "reference":
        s_np, e_np, n_np = O.moe_align_block_size(ids, bn, E)
        s, eids, ntp = (torch.from_numpy(v).to(DEV) for v in (s_np, e_np, n_np))
    else:
        cap0 = (T + E * (bn - 1) + bn - 1) // bn * bn
        # entries past the padded total are not written: pads and expert 0 there
        s = torch.full((cap0,), T, dtype=torch.int32, device=DEV)
        eids = torch.zeros(cap0 // bn, dtype=torch.int32, device=DEV)
        ntp = torch.zeros(1, dtype=torch.int32, device=DEV)
        ops.moe_align(torch.from_numpy(ids).to(DEV), E, bn, s, eids, ntp,
                      flags=ops.ALIGN_BALANCED)
        s_np = s.cpu().numpy()
    cap, R = s_np.size, T
    maxb = cap // bn
    if epi == "swiglu":
        H, I = 1024, 4096  # w13: 2I = 8192 weight rows, 16 pair tiles per block
        x = torch.randn(T, H, device=DEV).to(torch.bfloat16)
        w = (torch.randn(E, 2 * I, H, device=DEV) * 0.03).to(torch.bfloat16)
        ws = (torch.randn(2 * I, H, device=DEV) * 0.03).to(torch.bfloat16)
        xs = torch.empty(cap, H, dtype=torch.bfloat16, device=DEV)
        ops.permute_rows(x, s, ntp, 1, R, xs)
        w_rows, K, n_out, epi_id, xin, xsh = 2 * I, H, I, ops.FUS_EPI_SWIGLU, xs, x
        fl = ops.GEMM_SWIGLU_EXACT
    else:
        H, I = 6144, 1024  # w2: 6144 weight rows, 24 pair tiles per block
        a = torch.randn(cap, I, device=DEV).to(torch.bfloat16)
        a_s = torch.randn(T, I, device=DEV).to(torch.bfloat16)
        w = (torch.randn(E, H, I, device=DEV) * 0.03).to(torch.bfloat16)
        ws = (torch.randn(H, I, device=DEV) * 0.03).to(torch.bfloat16)
        w_rows, K, n_out, epi_id, xin, xsh = H, I, H, ops.FUS_EPI_BF16, a, a_s
        fl = 0
    outs = []
    for flag in (0, ops.GEMM_PAIR_NARROW, ops.GEMM_NO_PAIR, ops.GEMM_NO_PERSIST):
        o = torch.zeros(cap, n_out, dtype=torch.bfloat16, device=DEV)
        # the shared group writes fp32 on the down projection (as the prefill block does)
        o_s = torch.zeros(T, n_out, dtype=torch.bfloat16 if epi == "swiglu" else torch.float32,
                          device=DEV)
        fls = fl if epi == "swiglu" else ops.GEMM_OUT_F32
        gs = [ops.gemm_group(w, xin, o, expert_ids=eids, ntp=ntp, max_blocks=maxb,
                             row_limit=cap, live_ids=s, live_limit=R, flags=flag | fl),
              ops.gemm_group(ws, xsh, o_s, max_blocks=-(-T // bn), row_limit=T, flags=fls)]
        ops.grouped_gemm(gs, w_rows, K, epi_id, bn)
        outs.append((o, o_s))
    finish()
    live = torch.from_numpy(s_np < R).to(DEV)
    for o, o_s in outs[1:]:
        assert torch.equal(outs[0][0][live].view(torch.int16), o[live].view(torch.int16))
        assert torch.equal(outs[0][1], o_s) if o_s.dtype == torch.float32 else \
            torch.equal(outs[0][1].view(torch.int16), o_s.view(torch.int16))
    if epi == "swiglu":
        def fn(xx, ww):
            h = xx @ ww.t()
            return torch.nn.functional.silu(h[:, :I]) * h[:, I:]
    else:
        def fn(xx, ww):
            return xx @ ww.t()
    ref = ref_rows(xin, w, eids.cpu(), bn, fn)
    assert rel_err(outs[0][0][live].float().cpu().numpy(), ref[live].cpu().numpy()) < 1e-2
    ref_s = fn(xsh.float(), ws.float())
    assert rel_err(outs[0][1].float().cpu().numpy(), ref_s.cpu().numpy()) < 1e-2
