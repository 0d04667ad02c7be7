"""GPU parity of o_proj + ResAdd1 (glm52/kernels/oproj_resadd.py) against the oracle
(oracle.reference_np.oproj_resadd, the fp32 formula of glm52/bench/bench_layer.py:355):
decode (K = 32768, split-K planes) and prefill (K = 16384, residual in the GEMM
epilogue), fused and unfused numerics, and the drop-in chains."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from fusion_b200 import ops, synth
from fusion_b200.kernels import oproj_resadd as KO
from gpu_util import DEV, finish, to_np
from oracle import reference_np as O

pytestmark = pytest.mark.gpu
H = 6144


def inputs(T, K, seed):
    a = synth.make("h", (T, K), seed, DEV)
    w_kn = (synth.make("w2", (K, H), seed, DEV).float() * 0.5).to(torch.bfloat16)
    r = synth.make("r", (T, H), seed, DEV)
    return a, w_kn, r


def ulp(x):
    return np.exp2(np.floor(np.log2(np.maximum(np.abs(x), 1e-30))) - 7)


def check(out, ref, c_ref=None):
    """fused (one rounding): the block bar, max-abs <= 2e-2 * rms(ref). Unfused (c rounded
    to bf16 before the add, c_ref = the oracle's c): the fp32 sums of GEMM and numpy
    differ in order, so c can land one bf16 ulp apart (a few where the dot product
    cancels to near zero); the bar is one ulp of |c| plus one ulp of the output per
    element, plus 1e-3 * rms(ref) for those cancellations."""
    o, rf = to_np(out), ref
    err = np.abs(o - rf)
    if c_ref is None:
        rms = float(np.sqrt((rf.astype(np.float64) ** 2).mean()))
        assert float(err.max()) <= 2e-2 * rms, float(err.max()) / rms
    else:
        rms = float(np.sqrt((rf.astype(np.float64) ** 2).mean()))
        bound = ulp(c_ref) + ulp(rf) + 1e-3 * rms
        bad = err > bound
        assert not bad.any(), (float((err / bound).max()), int(bad.sum()), float(err.max()),
                               np.argwhere(bad)[:3].tolist(), o[bad][:3].tolist(),
                               rf[bad][:3].tolist(), c_ref[bad][:3].tolist())
    assert float((err > 0).mean()) < 0.05


@pytest.mark.parametrize("T,K", [(1, 32768), (4, 32768), (48, 32768), (300, 16384)])
@pytest.mark.parametrize("fused", [True, False])
def test_oproj_resadd_vs_oracle(T, K, fused):
    a, w_kn, r = inputs(T, K, 7 + T)
    w_nk = w_kn.t().contiguous()
    out = torch.empty(T, H, dtype=torch.bfloat16, device=DEV)
    ops.oproj_resadd(a, w_nk, r, out, fuse=fused)
    finish()
    ref = O.oproj_resadd(to_np(a), to_np(w_kn), to_np(r), fused=fused)
    check(out, ref, None if fused else O.oproj_resadd(to_np(a), to_np(w_kn), None, fused=False))


@pytest.mark.parametrize("T,K", [(2, 32768), (512, 16384)])
def test_dropin_chains(T, K):
    """The drop-in chains (fused, unfused, unfused split-K with acc32) against the oracle;
    the reference's [K, N] weight is used as given."""
    a, w_kn, r = inputs(T, K, 11 + T)
    ref_f = O.oproj_resadd(to_np(a), to_np(w_kn), to_np(r), fused=True)
    ref_u = O.oproj_resadd(to_np(a), to_np(w_kn), to_np(r), fused=False)
    out = torch.empty(T, H, dtype=torch.bfloat16, device=DEV)
    cmat = torch.empty_like(out)
    acc32 = torch.zeros(T, H, dtype=torch.float32, device=DEV)
    for f in KO.make_fused_chain(a, w_kn, r, out, acc32, {}):
        f()
    finish()
    check(out, ref_f)
    for f in KO.make_unfused_chain(a, w_kn, r, out, cmat, acc32, {}, {}):
        f()
    finish()
    check(out, ref_u, O.oproj_resadd(to_np(a), to_np(w_kn), None, fused=False))
    for f in KO.make_unfused_chain(a, w_kn, r, out, cmat, acc32, {"SPLIT_K": 4}, {}):
        f()  # split-K keeps c in fp32: one rounding, the fused numerics
    finish()
    check(out, ref_f)
