"""GPU parity: ResAdd+RMSNorm, SwiGLU, merge, residual add, seed — against the oracle."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import bf16_from_bits, golden
from fusion_b200 import ops, synth
from gpu_util import DEV, assert_bf16_close, assert_sum_close, bf, finish, to_np
from oracle import reference_np as O

pytestmark = pytest.mark.gpu


def test_add_rmsnorm_golden():
    g = golden("addnorm")
    h, r, gam = (bf(bf16_from_bits(g[k])) for k in ("h", "r", "gamma"))
    T, N = h.shape
    h1 = torch.empty_like(h)
    x2 = torch.empty_like(h)
    ops.add_rmsnorm(h, r, gam, h1, x2)
    finish()
    assert np.array_equal(to_np(h1), bf16_from_bits(g["h1"]))
    assert_bf16_close(to_np(x2), bf16_from_bits(g["x2"]))


@pytest.mark.parametrize("T", [1, 7, 256, 8192])
def test_add_rmsnorm_fused_vs_unfused_vs_oracle(T):
    N = 6144
    h = synth.make("h", (T, N), 11, DEV)
    r = synth.make("r", (T, N), 11, DEV)
    gam = synth.make("gamma", (N,), 11, DEV)
    h1, x2 = torch.empty_like(h), torch.empty_like(h)
    ops.add_rmsnorm(h, r, gam, h1, x2)
    h1b, x2b = torch.empty_like(h), torch.empty_like(h)
    ops.add_rmsnorm(h, r, None, h1b, None, do_norm=False)   # add_only
    ops.add_rmsnorm(h1b, None, gam, None, x2b, do_add=False)  # norm_only
    finish()
    assert torch.equal(h1.view(torch.int16), h1b.view(torch.int16))
    assert torch.equal(x2.view(torch.int16), x2b.view(torch.int16))  # fused == unfused bitwise
    ox2, oh1 = O.add_rmsnorm(to_np(h), to_np(r), to_np(gam))
    assert np.array_equal(to_np(h1), oh1)
    assert_bf16_close(to_np(x2), ox2)


def test_add_rmsnorm_small_hidden():
    T, N = 3, 256
    h = synth.make("h", (T, N), 12, DEV)
    r = synth.make("r", (T, N), 12, DEV)
    gam = synth.make("gamma", (N,), 12, DEV)
    h1, x2 = torch.empty_like(h), torch.empty_like(h)
    ops.add_rmsnorm(h, r, gam, h1, x2)
    finish()
    ox2, oh1 = O.add_rmsnorm(to_np(h), to_np(r), to_np(gam))
    assert np.array_equal(to_np(h1), oh1)
    assert_bf16_close(to_np(x2), ox2)


def test_silu_and_mul_golden_and_oracle():
    g = golden("mlp_small")
    x = bf(bf16_from_bits(g["inter"]))
    y = torch.empty(x.shape[0], x.shape[1] // 2, dtype=torch.bfloat16, device=DEV)
    ops.silu_and_mul(x, y)
    finish()
    assert_bf16_close(to_np(y), bf16_from_bits(g["act"]), frac=2e-2)
    xb = synth.make("h", (300, 4096), 13, DEV)
    yb = torch.empty(300, 2048, dtype=torch.bfloat16, device=DEV)
    ops.silu_and_mul(xb, yb)
    finish()
    assert_bf16_close(to_np(yb), O.silu_and_mul(to_np(xb)), frac=2e-2)


def test_merge_golden():
    g = golden("mlp_small")
    y = bf(bf16_from_bits(g["y"]))
    tw = torch.from_numpy(g["tw"]).to(DEV)
    out = torch.empty(y.shape[0], y.shape[2], dtype=torch.bfloat16, device=DEV)
    ops.merge(y, tw, None, None, out)  # merge_only
    finish()
    assert_sum_close(to_np(out), bf16_from_bits(g["merged"]))


@pytest.mark.parametrize("T", [1, 33, 2048])
def test_merge_resadd_shared(T):
    H, K = 6144, 8
    y = synth.make("h", (T, K, H), 14, DEV)
    res = synth.make("r", (T, H), 14, DEV)
    ext = synth.make("h", (T, H), 15, DEV)
    w = torch.rand(T, K, device=DEV)
    out = torch.empty(T, H, dtype=torch.bfloat16, device=DEV)
    ops.merge(y, w, res, ext, out, round_mid=True)
    # unfused chain: merge_only then resadd twice must agree bitwise on the mid rounding
    m = torch.empty_like(out)
    ops.merge(y, w, None, None, m)
    finish()
    mo = O.expert_merge(to_np(y), to_np(w))
    assert_sum_close(to_np(m), mo)
    ref = O.bf16(to_np(m) + to_np(res) + to_np(ext))
    assert_sum_close(to_np(out), ref)
    # unweighted sum (moe_sum) with residual
    o2 = torch.empty_like(out)
    ops.merge(y, None, res, None, o2, round_mid=False)
    finish()
    ref2 = O.bf16(to_np(y).sum(1) + to_np(res))
    assert_sum_close(to_np(o2), ref2)


def test_add_and_seed():
    a = synth.make("h", (37, 6144), 16, DEV)
    b = synth.make("r", (37, 6144), 16, DEV)
    o = torch.empty_like(a)
    ops.add(a, b, o)
    s = torch.full_like(a, 3.0)
    ops.seed(s)
    s2 = torch.empty_like(a)
    ops.seed(s2, a)
    finish()
    assert np.array_equal(to_np(o), O.bf16(to_np(a) + to_np(b)))
    assert torch.count_nonzero(s) == 0
    assert torch.equal(s2, a)


@pytest.mark.parametrize("T", [3, 600])
def test_merge_pos_equals_merge_over_pair_order(T):
    """Merging rows stored in dispatch order through pos_of gives the bits of merging
    the same rows in pair order (same summation order)."""
    K, H = 8, 6144
    g = torch.Generator(device="cpu").manual_seed(T)
    R = T * K
    rows = R + 37  # dispatch order with room for pads
    perm = torch.randperm(rows, generator=g)[:R].to(torch.int32)  # pos_of
    y_disp = torch.randn(rows, H, generator=g).to(torch.bfloat16)
    y_pair = y_disp[perm.long()]
    w = torch.rand(T, K, generator=g)
    h1 = torch.randn(T, H, generator=g).to(torch.bfloat16)
    ys = torch.randn(T, H, generator=g)
    y_disp, y_pair, perm, w, h1, ys = (a.to(DEV) for a in (y_disp, y_pair, perm, w, h1, ys))
    o1 = torch.empty(T, H, dtype=torch.bfloat16, device=DEV)
    o2 = torch.empty_like(o1)
    ops.merge(y_pair.view(T, K, H), w, h1, ys, o1, round_mid=False)
    ops.merge_pos(y_disp, perm, K, w, h1, ys, o2)
    finish()
    assert torch.equal(o1.view(torch.int16), o2.view(torch.int16))
