"""GPU parity of the half-fused lazy pre-norm (glm52/kernels/lazy_prenorm.py, F11b'):
rstd kernel, load-time weight folding, the router (fp32 logits scaled by rstd after the
GEMM) against the oracle's restatement and the reference's exact fp32 logits
(golden lazy_prenorm.npz), and the grouped w13 GEMM with the per-token rstd epilogue."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import golden
from fusion_b200 import ops, synth
from fusion_b200.kernels import lazy_prenorm as KL
from gpu_util import DEV, finish, to_np
from oracle import reference_np as O

pytestmark = pytest.mark.gpu
D = synth.Dims()


def test_rstd_and_fold():
    h = synth.make("h", (37, D.H), 3, DEV)
    w = synth.make("gamma", (D.H,), 3, DEV)
    r = torch.empty(37, dtype=torch.float32, device=DEV)
    KL.launch_rstd(h, r, None)
    gw = synth.make("gate_w", (D.E, D.H), 3, DEV).to(torch.bfloat16)
    f_nk = KL.fold_weight_nk(gw, w)
    f_kn = KL.fold_weight_rowmajor(gw.t().contiguous(), w)
    finish()
    np.testing.assert_allclose(to_np(r), O.row_rstd(to_np(h)), rtol=2e-6, atol=0)
    assert np.array_equal(to_np(f_nk), O.fold_weight_nk(to_np(gw), to_np(w)))
    assert np.array_equal(to_np(f_kn), O.fold_weight_rowmajor(to_np(gw).T.copy(), to_np(w)))


def test_lazy_router_golden_and_oracle():
    g = golden("lazy_prenorm")
    seed, T = int(g["seed"]), int(g["T"])
    h = synth.make("h", (T, D.H), seed, DEV)
    w = synth.make("gamma", (D.H,), seed, DEV)
    gw32 = synth.make("gate_w", (D.E, D.H), seed, DEV)
    gw = gw32.to(torch.bfloat16)  # the F11 router GEMM takes a bf16 weight
    b = KL.fold_weight_rowmajor(gw.t().contiguous(), w)  # [K, N], load time
    for rstd in (None, torch.empty(T, dtype=torch.float32, device=DEV)):
        if rstd is not None:
            KL.launch_rstd(h, rstd, None)
        c = torch.empty(T, D.E, dtype=torch.float32, device=DEV)
        KL.launch_router(h, b, c, None, True, rstd=rstd)
        finish()
        got = to_np(c)
        ref = O.lazy_router_logits(to_np(h), to_np(b))
        np.testing.assert_allclose(got, ref, rtol=0, atol=1e-4)
        # the reference's exact fp32 logits (fp32 weight): bf16 weight + folding stay
        # within the block's bar
        ex = g["logits_exact"]
        rms = float(np.sqrt((ex.astype(np.float64) ** 2).mean()))
        assert float(np.abs(got - ex).max()) <= 2e-2 * rms
    # fuse_norm off: the plain router GEMM on x2
    x2 = synth.make("r", (T, D.H), seed, DEV)
    c = torch.empty(T, D.E, dtype=torch.float32, device=DEV)
    KL.launch_router(x2, gw.t().contiguous(), c, None, False)
    finish()
    np.testing.assert_allclose(to_np(c), O.router_logits(to_np(x2), to_np(gw)), rtol=0,
                               atol=1e-4)


@pytest.mark.parametrize("T,bm", [(5, 16), (300, 64)])
def test_lazy_moe_gateup(T, bm):
    """c[flat] = bf16((h[t] @ folded_w13[e].T) * rstd[t]) for every routed pair."""
    E, K, I = 16, D.H, 256
    rng = np.random.default_rng(T)
    ids = np.stack([rng.choice(E, 4, replace=False) for _ in range(T)]).astype(np.int32)
    s, e, n = O.moe_align_block_size(ids, bm, E)
    s_t, e_t, n_t = (torch.from_numpy(x).to(DEV) for x in (s, e, n))
    h = synth.make("h", (T, K), 9 + T, DEV)
    w = synth.make("gamma", (K,), 9, DEV)
    w13 = synth.make("w13", (E, 2 * I, K), 9, DEV)
    b = KL.fold_weight_nk(w13, w)
    c = torch.zeros(T * 4, 2 * I, dtype=torch.bfloat16, device=DEV)
    KL.launch_moe_gateup(h, b, c, s_t, e_t, n_t, T * 4, 4, {"BLOCK_M": bm}, True)
    finish()
    hb, bb = to_np(h), to_np(b)
    rs = O.row_rstd(hb)
    flat = ids.reshape(-1)
    ref = np.stack([O.bf16((hb[i // 4] @ bb[flat[i]].T) * rs[i // 4]) for i in range(T * 4)])
    got = to_np(c)
    err = np.abs(got - ref)
    # one rounding of an fp32 sum whose order differs from numpy's: one bf16 ulp, plus
    # fp32 ordering noise where a K = 6144 dot product cancels to near zero
    ulp = np.exp2(np.floor(np.log2(np.maximum(np.abs(ref), 1e-30))) - 7)
    rms = float(np.sqrt((ref.astype(np.float64) ** 2).mean()))
    bound = ulp + 1e-3 * rms
    assert np.all(err <= bound), (float((err / bound).max()), int((err > bound).sum()))
    assert float((err > 0).mean()) < 0.05
