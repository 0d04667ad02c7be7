"""Pin the CPU oracle (oracle/reference_np.py) to the reference's own outputs.

The golden vectors were produced by running glm52_h200/reference.py itself on seeded
inputs (tests/golden/make_golden.py). Integer outputs must match bit for bit; bf16
outputs may differ by the reference's own summation-order noise (<= 1 bf16 ulp on a
handful of elements)."""

from __future__ import annotations

import numpy as np
import torch

from conftest import bf16_from_bits, golden, ulp_diff_bf16
from fusion_b200 import synth
from oracle import reference_np as O


def test_add_rmsnorm_matches_reference():
    g = golden("addnorm")
    h, r, gam = (bf16_from_bits(g[k]) for k in ("h", "r", "gamma"))
    x2, h1 = O.add_rmsnorm(h, r, gam)
    assert np.array_equal(h1, bf16_from_bits(g["h1"]))  # bit-exact residual
    d = ulp_diff_bf16(x2, bf16_from_bits(g["x2"]))
    assert d.max() <= 1 and (d > 0).mean() < 1e-3


def test_router_matches_reference():
    g = golden("router")
    seed, T = int(g["seed"]), int(g["T"])
    x2 = bf16_from_bits(g["x2"])
    gw = synth.make("gate_w", (256, 6144), seed).numpy()
    bias = synth.make("bias", (256,), seed).numpy()
    lg, w, ids = O.router(x2, gw, bias)
    np.testing.assert_allclose(lg, g["logits"], rtol=1e-5, atol=2e-5)
    assert np.array_equal(ids, g["topk_ids"])
    np.testing.assert_allclose(w, g["topk_weights"], rtol=2e-6, atol=1e-6)
    _, w0, ids0 = O.router(x2, gw, None)
    assert np.array_equal(ids0, g["topk_ids_nobias"])
    np.testing.assert_allclose(w0, g["topk_weights_nobias"], rtol=2e-6, atol=1e-6)
    _, wg, idsg = O.router(x2, gw, bias, n_group=8, topk_group=4)
    assert np.array_equal(idsg, g["topk_ids_grouped"])
    np.testing.assert_allclose(wg, g["topk_weights_grouped"], rtol=2e-6, atol=1e-6)


def test_moe_align_matches_reference_bit_exact():
    g = golden("align")
    names = sorted({k.rsplit("_", 1)[0] for k in g if k.endswith("_ids")})
    assert len(names) >= 8
    for n in names:
        s, e, ntp = O.moe_align_block_size(g[f"{n}_ids"], int(g[f"{n}_bm"]), 256)
        assert np.array_equal(s, g[f"{n}_sorted"]), n
        assert np.array_equal(e, g[f"{n}_eids"]), n
        assert np.array_equal(ntp, g[f"{n}_ntp"]), n


def _small_weights(seed):
    E, H, I = 16, 256, 128
    w13 = synth.make("w13", (E, 2 * I, H), seed).float().numpy()
    w2 = synth.make("w2", (E, H, I), seed).float().numpy()
    w13s = synth.make("w13s", (1, 2 * I, H), seed).float().numpy()[0]
    w2s = synth.make("w2s", (1, H, I), seed).float().numpy()[0]
    return w13, w2, w13s, w2s


def test_moe_mlp_shared_merge_match_reference():
    g = golden("mlp_small")
    w13, w2, w13s, w2s = _small_weights(int(g["seed"]))
    x = bf16_from_bits(g["x"])
    tw, ti = g["tw"], g["ti"]
    routed = O.moe_mlp(x, lambda e: w13[e], lambda e: w2[e], tw, ti, 16)
    ref = bf16_from_bits(g["routed"])
    assert ulp_diff_bf16(routed, ref).max() <= 2
    exact = O.moe_mlp_exact_fp32(x, lambda e: w13[e], lambda e: w2[e], tw, ti, 16)
    np.testing.assert_allclose(exact, g["exact"], rtol=1e-4, atol=1e-5)
    shared = O.shared_expert_mlp(x, w13s, w2s)
    np.testing.assert_allclose(shared, g["shared"], rtol=1e-3, atol=1e-4)
    merged = O.expert_merge(bf16_from_bits(g["y"]), tw)
    assert ulp_diff_bf16(merged, bf16_from_bits(g["merged"])).max() <= 1
    act = O.silu_and_mul(bf16_from_bits(g["inter"]))
    assert ulp_diff_bf16(act, bf16_from_bits(g["act"])).max() <= 1


def test_full_block_t2_matches_reference():
    g = golden("block_full_t2")
    seed, T = int(g["seed"]), int(g["T"])
    d = synth.Dims()
    h = synth.make("h", (T, d.H), seed).float().numpy()
    r = synth.make("r", (T, d.H), seed).float().numpy()
    gamma = synth.make("gamma", (d.H,), seed).float().numpy()
    gw = synth.make("gate_w", (d.E, d.H), seed).numpy()
    bias = synth.make("bias", (d.E,), seed).numpy()
    cache = {}

    def get(name):
        def f(e):
            if (name, e) not in cache:
                cache[(name, e)] = synth.expert_weight(name, e, d, seed).float().numpy()
            return cache[(name, e)]
        return f

    w13s = synth.make("w13s", (2 * d.I, d.H), seed).float().numpy()
    w2s = synth.make("w2s", (d.H, d.I), seed).float().numpy()
    res = O.moe_block(h, r, gamma, gw, bias, get("w13"), get("w2"), w13s, w2s, d.E)
    assert np.array_equal(res["h1"], bf16_from_bits(g["h1"]))
    assert np.array_equal(res["topk_ids"], g["topk_ids"])
    np.testing.assert_allclose(res["topk_weights"], g["topk_weights"], rtol=2e-6, atol=1e-6)
    out, ref = res["out"], bf16_from_bits(g["out"])
    rms = float(np.sqrt((ref.astype(np.float64) ** 2).mean()))
    assert np.abs(out - ref).max() <= 2e-2 * rms
    # ulps explode near zero (a cancelling sum); count mismatches instead
    assert (ulp_diff_bf16(out, ref) > 1).mean() < 2e-3
    exact = O.moe_block_exact_fp32(res["x2"], res["h1"], res["topk_weights"], res["topk_ids"],
                                   get("w13"), get("w2"), w13s, w2s, d.E)
    np.testing.assert_allclose(exact, g["out_exact"], rtol=1e-4, atol=1e-4)


def test_lazy_prenorm_exact_logits_match_reference():
    """router_logits_exact_fp32 (reference.py:123) on the reference's own output; the
    half-fused form (folded bf16 weight, rstd after the GEMM) stays within 2e-2 * rms."""
    g = golden("lazy_prenorm")
    seed, T = int(g["seed"]), int(g["T"])
    d = synth.Dims()
    h = synth.make("h", (T, d.H), seed).float().numpy()
    w = synth.make("gamma", (d.H,), seed).float().numpy()
    gw = synth.make("gate_w", (d.E, d.H), seed).float().numpy()
    ex = O.router_logits_exact_fp32(h, w, gw)
    np.testing.assert_allclose(ex, g["logits_exact"], rtol=0, atol=2e-5)
    lz = O.lazy_router_logits(h, O.fold_weight_rowmajor(gw.T.copy(), w))
    rms = float(np.sqrt((ex.astype(np.float64) ** 2).mean()))
    assert float(np.abs(lz - ex).max()) <= 2e-2 * rms


def test_numpy_generator_matches_library_bits():
    """oracle/synth_np.py (the CPU arms' input generator, which loads no CUDA library)
    gives the bits of the library's host generator for every stream, including a slice
    taken from an element offset (one expert of the stacked weights)."""
    from oracle import synth_np as S

    for name, shape, off in (("h", (3, 6144), 0), ("r", (2, 512), 0), ("gamma", (6144,), 0),
                             ("gate_w", (256, 64), 0), ("bias", (256,), 0),
                             ("w13", (64, 96), 5 * 64 * 96), ("w2", (96, 32), 77),
                             ("w13s", (16, 40), 0), ("w2s", (40, 8), 0)):
        a = S.make(name, shape, 7, offset=off)
        b = synth.make(name, shape, 7, offset=off).float().numpy()
        assert np.array_equal(a.view(np.uint32), b.view(np.uint32)), name


def test_torch_restatement_block_t2_matches_reference():
    """oracle/reference_torch.py (the CPU path bench.py times as the reference arm) gives
    the reference's own block outputs on the golden case: h1, top-k ids and the bf16
    output bit for bit, the routing weights to fp32 rounding."""
    import torch

    from oracle import reference_torch as RT
    from oracle import synth_np as S

    g = golden("block_full_t2")
    seed, T = int(g["seed"]), int(g["T"])
    H, I, E = 6144, 2048, 256
    bf = torch.bfloat16
    h = torch.from_numpy(S.make("h", (T, H), seed)).to(bf)
    r = torch.from_numpy(S.make("r", (T, H), seed)).to(bf)
    gamma = torch.from_numpy(S.make("gamma", (H,), seed)).to(bf)
    gw = torch.from_numpy(S.make("gate_w", (E, H), seed))
    bias = torch.from_numpy(S.make("bias", (E,), seed))
    used = sorted(set(g["topk_ids"].flatten().tolist()))
    w13 = {e: torch.from_numpy(S.expert_weight("w13", e, H, I, seed)).to(bf) for e in used}
    w2 = {e: torch.from_numpy(S.expert_weight("w2", e, H, I, seed)).to(bf) for e in used}
    w13s = torch.from_numpy(S.make("w13s", (2 * I, H), seed)).to(bf)
    w2s = torch.from_numpy(S.make("w2s", (H, I), seed)).to(bf)
    res = RT.moe_block(h, r, gamma, gw, bias, w13, w2, w13s, w2s, E)
    assert np.array_equal(res["h1"].view(torch.int16).numpy().view(np.uint16), g["h1"])
    assert np.array_equal(res["topk_ids"].numpy(), g["topk_ids"])
    np.testing.assert_allclose(res["topk_weights"].numpy(), g["topk_weights"], rtol=2e-6,
                               atol=1e-6)
    out = res["out"].view(torch.int16).numpy().view(np.uint16)
    assert (out != g["out"]).mean() < 2e-3
    ref = bf16_from_bits(g["out"])
    rms = float(np.sqrt((ref.astype(np.float64) ** 2).mean()))
    assert np.abs(res["out"].float().numpy() - ref).max() <= 2e-2 * rms
