"""Generate the golden vectors that pin the CPU oracle to the reference.

Runs the REFERENCE's own torch functions (glm52_h200/reference.py, imported from a
checkout of HansonZhang-cuhksz/fusion) on seeded inputs from fusion_b200's
bit-reproducible generator and stores inputs (when small) and outputs as .npz.
Needs a checkout of the reference (its directory in ``FUSION_REFERENCE``) and the
built library (for the host-side generator); the committed .npz files are what the
tests read, so the reference is not needed at test time.

    FUSION_REFERENCE=<checkout of HansonZhang-cuhksz/fusion> python tests/golden/make_golden.py
"""

from __future__ import annotations

import os
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent
sys.path.insert(0, str(ROOT))
if "FUSION_REFERENCE" not in os.environ:
    raise SystemExit("set FUSION_REFERENCE to a checkout of HansonZhang-cuhksz/fusion")
sys.path.insert(0, os.environ["FUSION_REFERENCE"])

import glm52_h200.reference as R  # noqa: E402  (the reference under test)

from fusion_b200 import synth  # noqa: E402

torch.manual_seed(0)
BF = torch.bfloat16


def bits(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def f32(t: torch.Tensor) -> np.ndarray:
    return t.float().contiguous().numpy()


def gen_addnorm():
    T, N = 5, 6144
    h = synth.make("h", (T, N), 101)
    r = synth.make("r", (T, N), 101)
    g = synth.make("gamma", (N,), 101)
    x2, h1 = R.add_rmsnorm(h, r, g)
    np.savez_compressed(HERE / "addnorm.npz", h=bits(h), r=bits(r), gamma=bits(g), h1=bits(h1),
                        x2=bits(x2))


def gen_router():
    T, H, E = 16, 6144, 256
    x2 = synth.make("h", (T, H), 202)  # a bf16 N(0,1) activation
    gw = synth.make("gate_w", (E, H), 202)
    bias = synth.make("bias", (E,), 202)
    lg, w, ids = R.router(x2, gw, bias)
    lg0, w0, ids0 = R.router(x2, gw, None)
    _, wg, idsg = R.router(x2, gw, bias, n_group=8, topk_group=4)
    np.savez_compressed(HERE / "router.npz", seed=202, T=T, x2=bits(x2), logits=f32(lg),
                        topk_weights=f32(w), topk_ids=ids.numpy(), logits_nobias=f32(lg0),
                        topk_weights_nobias=f32(w0), topk_ids_nobias=ids0.numpy(),
                        topk_weights_grouped=f32(wg), topk_ids_grouped=idsg.numpy())


def gen_align():
    E = 256
    g = torch.Generator().manual_seed(7)
    cases = {
        "t1_bm16": (torch.randint(0, E, (1, 8), generator=g), 16),
        "t7_bm16": (torch.randint(0, E, (7, 8), generator=g), 16),
        "t64_bm16": (torch.randint(0, E, (64, 8), generator=g), 16),
        "t300_bm64": (torch.randint(0, E, (300, 8), generator=g), 64),
        "t1024_bm128": (torch.randint(0, E, (1024, 8), generator=g), 128),
        # skew: half of the pairs go to 3 experts; every other expert may be empty
        "skew_t512_bm32": (torch.where(torch.rand(512, 8, generator=g) < 0.5,
                                       torch.randint(0, 3, (512, 8), generator=g),
                                       torch.randint(0, E, (512, 8), generator=g)), 32),
        "one_expert_t50_bm16": (torch.full((50, 8), 3), 16),
        "t1200_bm16": (torch.randint(0, E, (1200, 8), generator=g), 16),
    }
    out = {}
    for name, (ids, bm) in cases.items():
        ids = ids.int()
        s, e, n = R.moe_align_block_size(ids, bm, E)
        out[f"{name}_ids"] = ids.numpy()
        out[f"{name}_bm"] = np.array(bm)
        out[f"{name}_sorted"] = s.numpy()
        out[f"{name}_eids"] = e.numpy()
        out[f"{name}_ntp"] = n.numpy()
    np.savez_compressed(HERE / "align.npz", **out)


def gen_mlp_small():
    """Reduced dims (H=256, I=128, E=16, topk=4) so inputs fit in a fixture."""
    T, H, I, E, K = 12, 256, 128, 16, 4
    x = synth.make("h", (T, H), 303)
    w13 = synth.make("w13", (E, 2 * I, H), 303)
    w2 = synth.make("w2", (E, H, I), 303)
    w13s = synth.make("w13s", (1, 2 * I, H), 303)
    w2s = synth.make("w2s", (1, H, I), 303)
    gw = synth.make("gate_w", (E, H), 303)
    _, tw, ti = R.router(x, gw, None, topk=K)
    routed = R.moe_mlp(x, w13, w2, tw, ti)
    exact = R.moe_mlp_exact_fp32(x, w13, w2, tw, ti)
    shared = R.shared_expert_mlp(x, w13s, w2s)
    y = synth.make("r", (T, K, H), 303)
    merged = R.expert_merge(y, tw)
    inter = synth.make("h", (T, 2 * I), 304)
    act = R.silu_and_mul(inter)
    # the weights are regenerated from seed 303 by the tests (too large to store)
    np.savez_compressed(HERE / "mlp_small.npz", seed=303, x=bits(x), tw=f32(tw), ti=ti.numpy(),
                        routed=bits(routed), exact=f32(exact), shared=f32(shared), y=bits(y),
                        merged=bits(merged), inter=bits(inter), act=bits(act))


def gen_block_full():
    """Full GLM-5.2 dims at T=2; the 16 routed experts are regenerated from seeds."""
    T, seed = 2, 404
    d = synth.Dims()
    h = synth.make("h", (T, d.H), seed)
    r = synth.make("r", (T, d.H), seed)
    gamma = synth.make("gamma", (d.H,), seed)
    gw = synth.make("gate_w", (d.E, d.H), seed)
    bias = synth.make("bias", (d.E,), seed)
    x2, h1 = R.add_rmsnorm(h, r, gamma)
    _, tw, ti = R.router(x2, gw, bias)
    used = sorted(set(ti.flatten().tolist()))
    w13 = torch.zeros(d.E, 2 * d.I, d.H, dtype=BF)
    w2 = torch.zeros(d.E, d.H, d.I, dtype=BF)
    for e in used:
        w13[e] = synth.expert_weight("w13", e, d, seed)
        w2[e] = synth.expert_weight("w2", e, d, seed)
    w13s = synth.make("w13s", (2 * d.I, d.H), seed)
    w2s = synth.make("w2s", (d.H, d.I), seed)
    routed = R.moe_mlp(x2, w13, w2, tw, ti)
    out = (routed.float() + h1.float() + R.shared_expert_mlp(x2, w13s, w2s)).to(BF)
    # the exact fp32 path: moe_mlp_exact_fp32 + h1 + shared expert with the exact SwiGLU
    hs = torch.nn.functional.linear(x2.float(), w13s.float())
    s_exact = torch.nn.functional.linear(R.silu_and_mul_exact_fp32(hs), w2s.float())
    exact = R.moe_mlp_exact_fp32(x2, w13, w2, tw, ti) + h1.float() + s_exact
    np.savez_compressed(HERE / "block_full_t2.npz", seed=seed, T=T, h1=bits(h1), x2=bits(x2),
                        topk_weights=f32(tw), topk_ids=ti.numpy(), routed=bits(routed),
                        out=bits(out), out_exact=f32(exact))


def gen_lazy_prenorm():
    """The reference's exact lazy-pre-norm router logits (reference.py:123,
    router_logits_exact_fp32) at GLM dims; h, w, gate_w regenerated from the seed."""
    T, seed = 8, 505
    d = synth.Dims()
    h = synth.make("h", (T, d.H), seed)
    w = synth.make("gamma", (d.H,), seed)
    gw = synth.make("gate_w", (d.E, d.H), seed)
    lg = R.router_logits_exact_fp32(h, w, gw)
    np.savez_compressed(HERE / "lazy_prenorm.npz", seed=seed, T=T, logits_exact=f32(lg))


if __name__ == "__main__":
    gen_lazy_prenorm()
    gen_addnorm()
    gen_router()
    gen_align()
    gen_mlp_small()
    gen_block_full()
    for p in sorted(HERE.glob("*.npz")):
        print(p.name, p.stat().st_size)
